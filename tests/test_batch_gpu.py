"""Continuous-batching verify step (SpecBatch) on the GPU vs the oracle, request by request.

One step packs several requests of different cached lengths and block sizes (more than 32 rows
in total, so the projections run in several launches) into one verify forward over a
position-major KV pool. Each request's logits rows must match the oracle's single-request
forward of the same block at the same length (bars as in test_forward_gpu.py); the cache rows
the step wrote must match the oracle's; lengths after the greedy accept must be L0 + n + 1 with
n recomputed from the step's own argmax (bit-exact); idle slots must be untouched
(src/mlx_dspark/batch_engine.py:635-708).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from test_forward_gpu import _compare

pytestmark = pytest.mark.gpu


def _engine(cuda, caps, lengths, seed=0, bits=4, max_rows=96):
    from mlx_dspark_b200.batch_engine import SpecBatch
    from mlx_dspark_b200.target import Target, tiny_config

    cfg = tiny_config(bits=bits)
    t = Target(cfg, seed=seed, slot_caps=caps, max_rows=max_rows)
    eng = SpecBatch(t, max_block=17)
    g = torch.Generator(device=cuda).manual_seed(seed + 1)
    kvs = []
    for L0 in lengths:
        kv = [(torch.randn((cfg.n_kv_heads, L0, cfg.head_dim), device=cuda, generator=g)
               .to(torch.bfloat16),
               torch.randn((cfg.n_kv_heads, L0, cfg.head_dim), device=cuda, generator=g)
               .to(torch.bfloat16)) for _ in range(cfg.n_layers)]
        kvs.append(kv)
        eng.admit(L0, int(torch.randint(0, cfg.vocab, (1,), generator=g, device=cuda)), kv=kv)
    return t, eng, kvs


@pytest.mark.parametrize("bits", [4, 8])
def test_spec_batch_step_matches_per_request_oracle(cuda, oracle, bits):
    caps = [300, 700, 96, 500]
    lengths = [120, 533, 40, 300]
    blocks = [17, 9, 13, 16]          # 55 packed rows: projections in two launches
    t, eng, kvs = _engine(cuda, caps, lengths, seed=bits, bits=bits)
    cfg = t.cfg
    g = torch.Generator(device=cuda).manual_seed(7)
    drafts = torch.randint(0, cfg.vocab, (eng.B, 16), device=cuda, dtype=torch.int32,
                           generator=g)
    pending = eng.pending.clone()
    out = eng.step(drafts, blocks)
    torch.cuda.synchronize()
    cu = out["cu_rows"].cpu().numpy()
    assert list(np.diff(cu)) == blocks
    logits = t.logits[: sum(blocks)].float().cpu().numpy()
    tt = out["tt"][: sum(blocks)].cpu().numpy()
    ow, oc = t.oracle_weights(), t.oracle_config()
    for b, (L0, blk) in enumerate(zip(lengths, blocks)):
        ids = np.concatenate([[int(pending[b])], drafts[b, : blk - 1].cpu().numpy()])
        kc = [np.zeros((cfg.n_kv_heads, caps[b], cfg.head_dim), np.float32) for _ in t.layers]
        vc = [np.zeros((cfg.n_kv_heads, caps[b], cfg.head_dim), np.float32) for _ in t.layers]
        for li, (k, v) in enumerate(kvs[b]):
            kc[li][:, :L0] = k.float().cpu().numpy()
            vc[li][:, :L0] = v.float().cpu().numpy()
        ref_p = oracle.verify_forward(ow, oc, ids, [c.copy() for c in kc],
                                      [c.copy() for c in vc], L0, round_p=True)
        ref = oracle.verify_forward(ow, oc, ids, kc, vc, L0)
        _compare(oracle, logits[cu[b] : cu[b + 1]], ref, ref_p)
        # the block's K/V landed in the request's own slot of the pool
        for li in range(len(t.layers)):
            got_k = t.slot_view(li, b, "k")[:, L0 : L0 + blk].float().cpu().numpy()
            want_k = kc[li][:, L0 : L0 + blk]
            assert float(np.abs(got_k - want_k).max()) <= 2e-2 * float(np.abs(want_k).max())
        # greedy accept from the step's own argmax, bit-exact rollback
        n = 0
        while n < blk - 1 and ids[1 + n] == tt[cu[b] + n]:
            n += 1
        assert int(out["n"][b]) == n
        assert int(out["next"][b]) == int(tt[cu[b] + n])
        assert int(eng.lens[b]) == L0 + n + 1
        assert int(eng.pending[b]) == int(tt[cu[b] + n])


def test_idle_slots_keep_their_state(cuda):
    caps = [200, 200, 200]
    t, eng, _ = _engine(cuda, caps, [50, 60, 70], seed=3)
    eng.retire(1)
    drafts = torch.zeros((eng.B, 16), device=cuda, dtype=torch.int32)
    before = eng.pending.clone()
    out = eng.step(drafts, [9, 9, 9], forced_accept=torch.tensor([3, 3, 3], device=cuda))
    torch.cuda.synchronize()
    assert int(eng.lens[1]) == 0 and int(out["n"][1]) == 0
    assert int(eng.pending[1]) == int(before[1])
    # forced accept: length grows by n + 1 on active slots
    assert int(eng.lens[0]) == 50 + 4 and int(eng.lens[2]) == 70 + 4
    assert list(np.diff(out["cu_rows"].cpu().numpy())) == [9, 0, 9]
    # the freed slot is reused by the next admission
    assert eng.admit(10, 5) == 1


def test_many_steps_lengths_track_accepts(cuda):
    """Repeated steps with seeded accept lengths: every slot's cache length is exactly its
    prefix plus the sum of (accepted + 1) over the steps."""
    caps = [400, 300, 500, 250, 350]
    lengths = [100, 20, 333, 64, 1]
    t, eng, _ = _engine(cuda, caps, lengths, seed=5, max_rows=96)
    rng = np.random.default_rng(0)
    want = list(lengths)
    for _ in range(6):
        blocks = [int(x) for x in rng.integers(8, 17, len(caps))]
        acc = [int(rng.integers(0, b)) for b in blocks]
        drafts = torch.randint(0, t.cfg.vocab, (eng.B, 16), device=cuda, dtype=torch.int32)
        eng.step(drafts, blocks, forced_accept=torch.tensor(acc, device=cuda))
        want = [w + a + 1 for w, a in zip(want, acc)]
    torch.cuda.synchronize()
    assert eng.lens.cpu().tolist() == want


@pytest.mark.parametrize("bits", [4, 8])
def test_spec_batch_step_wide_rows_match_per_request_oracle(cuda, oracle, monkeypatch, bits):
    """More than 64 packed rows: every projection runs once over all rows in the wide-M engine
    (RMSNorm applied to x, tcgen05 product, fused epilogue on the product). Each request's logits
    still match the oracle's single-request forward; the same step through the 32-row launches
    (wide engine switched off) agrees with it within the forward's bar."""
    caps = [300, 700, 96, 500, 260, 410, 180]
    lengths = [120, 533, 40, 300, 17, 222, 99]
    blocks = [17, 9, 13, 16, 12, 15, 11]      # 93 packed rows
    t, eng, kvs = _engine(cuda, caps, lengths, seed=10 + bits, bits=bits, max_rows=128)
    assert t.wide_ws_bytes > 0
    cfg = t.cfg
    g = torch.Generator(device=cuda).manual_seed(8)
    drafts = torch.randint(0, cfg.vocab, (eng.B, 16), device=cuda, dtype=torch.int32,
                           generator=g)
    pending = eng.pending.clone()
    lens0 = eng.lens.clone()
    out = eng.step(drafts, blocks)
    torch.cuda.synchronize()
    R = sum(blocks)
    cu = out["cu_rows"].cpu().numpy()
    logits = t.logits[:R].float().cpu().numpy()
    ow, oc = t.oracle_weights(), t.oracle_config()
    for b, (L0, blk) in enumerate(zip(lengths, blocks)):
        ids = np.concatenate([[int(pending[b])], drafts[b, : blk - 1].cpu().numpy()])
        kc = [np.zeros((cfg.n_kv_heads, caps[b], cfg.head_dim), np.float32) for _ in t.layers]
        vc = [np.zeros((cfg.n_kv_heads, caps[b], cfg.head_dim), np.float32) for _ in t.layers]
        for li, (k, v) in enumerate(kvs[b]):
            kc[li][:, :L0] = k.float().cpu().numpy()
            vc[li][:, :L0] = v.float().cpu().numpy()
        ref_p = oracle.verify_forward(ow, oc, ids, [c.copy() for c in kc],
                                      [c.copy() for c in vc], L0, round_p=True)
        ref = oracle.verify_forward(ow, oc, ids, kc, vc, L0)
        _compare(oracle, logits[cu[b] : cu[b + 1]], ref, ref_p)
    # the same step with the wide engine off (32-row launches): same logits within the bar
    eng.lens.copy_(lens0)
    eng.pending.copy_(pending)
    monkeypatch.setenv("DSPARK_WIDE_MIN_ROWS", "100000")
    eng.step(drafts, blocks)
    torch.cuda.synchronize()
    small = t.logits[:R].float().cpu().numpy()
    rel = float(np.linalg.norm(small - logits) / np.linalg.norm(small))
    assert rel <= 2e-2, rel
