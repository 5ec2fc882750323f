"""K3 / K4 / accept on the GPU: bit-exact against the oracle's restatement of BatchCache,
build_batch_mask, the greedy accept and the ragged packing (src/mlx_dspark/batch_engine.py,
src/mlx_dspark/generate.py:1548-1555)."""

from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

GOLD = json.loads((Path(__file__).parent / "golden" / "reference_goldens.json").read_text())


def test_append_rollback_100_steps(cuda, oracle):
    """BASELINE config 2's cache half: 16-row appends then rollback to an accepted length
    drawn U{0..16}, 100 seeded steps; lengths and cache contents bit-exact."""
    from mlx_dspark_b200.kvcache import BatchCache

    rng = np.random.default_rng(1234)
    B, H, D = 2, 8, 128
    start = [1000, 37]
    init = [(torch.randn(1, H, L, D, device=cuda).to(torch.bfloat16),
             torch.randn(1, H, L, D, device=cuda).to(torch.bfloat16)) for L in start]
    dev = BatchCache.from_rows(init)
    ref = oracle.BatchCacheRef.from_rows([(k.float().cpu().numpy(), v.float().cpu().numpy())
                                          for k, v in init])
    for _ in range(100):
        kn = torch.randn(B, H, 16, D, device=cuda).to(torch.bfloat16)
        vn = torch.randn(B, H, 16, D, device=cuda).to(torch.bfloat16)
        dev.update_and_fetch(kn, vn)
        ref.update_and_fetch(kn.float().cpu().numpy(), vn.float().cpu().numpy())
        acc = rng.integers(0, 17, B)
        ns = [16 - int(a) for a in acc]
        dev.trim(ns)
        ref.trim(ns)
        assert dev.offsets == ref.offsets
        assert dev.lens.tolist() == ref.offsets
    for b in range(B):
        n = ref.offsets[b]
        np.testing.assert_array_equal(dev.keys[b, :, :n].float().cpu().numpy(), ref.keys[b, :, :n])
        np.testing.assert_array_equal(dev.values[b, :, :n].float().cpu().numpy(),
                                      ref.values[b, :, :n])


@pytest.mark.parametrize("case", GOLD["batch_cache"], ids=lambda c: c["name"])
def test_batch_cache_reference_goldens(cuda, case):
    """The reference's own BatchCache goldens, replayed on the device cache."""
    from mlx_dspark_b200.kvcache import BatchCache

    H, D = 2, 8
    c = BatchCache.from_rows([(torch.randn(1, H, L, D, device=cuda),
                               torch.randn(1, H, L, D, device=cuda)) for L in case["lens"]])
    for op in case["ops"]:
        if op[0] == "update":
            T = op[1]
            B = len(case["lens"]) if c.rows is None else c.rows
            k = torch.randn(B, H, T, D, device=cuda)
            K, _ = c.update_and_fetch(k, k)
            if len(op) > 2:
                assert int(K.shape[2]) == op[2]
        elif op[0] == "trim":
            c.trim(op[1])
        elif op[0] == "move":
            c.move_row(op[1], op[2])
        elif op[0] == "rows":
            c.rows = op[1]
        elif op[0] == "expect":
            assert c.offsets == op[1]
            torch.cuda.synchronize()
            assert c.lens.tolist() == op[1]


def test_move_row_copies_live_columns(cuda):
    from mlx_dspark_b200.kvcache import BatchCache

    pairs = [(torch.randn(1, 2, L, 8, device=cuda), torch.randn(1, 2, L, 8, device=cuda))
             for L in (3, 2, 4)]
    c = BatchCache.from_rows(pairs)
    c.move_row(2, 0)
    assert c.offsets == [4, 2, 0]
    assert torch.equal(c.keys[0:1, :, :4], pairs[2][0])
    assert torch.equal(c.values[0:1, :, :4], pairs[2][1])


@pytest.mark.parametrize("case", GOLD["batch_mask"], ids=lambda c: str(c["offsets"]))
def test_batch_mask_goldens(cuda, case):
    from mlx_dspark_b200 import batch_engine

    m = batch_engine.build_batch_mask(case["offsets"], case["T"])
    assert list(m.shape) == case["shape"]
    g = m.to(torch.int32).cpu().tolist()
    for (b, i), row in zip(case["index"], case["rows"]):
        assert g[b][0][i] == row


def test_argmax_accept_rollback(cuda, oracle):
    """Greedy accept over ragged blocks fused with the rollback, vs the oracle; first-index
    tie-breaking like np / mx.argmax."""
    from mlx_dspark_b200 import batch_engine

    rng = np.random.default_rng(5)
    B, V = 6, 1000
    tl = [int(t) for t in rng.integers(1, 17, B)]
    cu = np.concatenate([[0], np.cumsum(tl)]).astype(np.int32)
    R = int(cu[-1])
    logits = rng.normal(0, 1, (R, V)).astype(np.float32)
    logits[0, 7] = logits[0, 9] = 50.0  # tie -> index 7
    logits_b = oracle.round_bf16(logits)
    tt = oracle.argmax_first(logits_b)
    ids = rng.integers(0, V, R).astype(np.int32)
    for b in range(B):  # make a prefix of drafts match the target's argmax
        r0, r1 = cu[b], cu[b + 1]
        n = int(rng.integers(0, r1 - r0))
        ids[r0 + 1 : r0 + 1 + n] = tt[r0 : r0 + n]
    lens0 = rng.integers(100, 200, B).astype(np.int32)
    out = batch_engine.accept(torch.from_numpy(logits_b).to(torch.bfloat16).to(cuda),
                              torch.from_numpy(ids).to(cuda), torch.from_numpy(cu).to(cuda),
                              torch.from_numpy(lens0 + np.array(tl, np.int32)).to(cuda))
    assert out["tt"].cpu().tolist() == tt.tolist()
    assert tt[0] == 7
    for b in range(B):
        r0, r1 = cu[b], cu[b + 1]
        n, committed, trim = oracle.accept(ids[r0 + 1 : r1], tt[r0:r1])
        assert int(out["n"][b]) == n
        assert int(out["next"][b]) == committed[-1]
        assert int(out["lens"][b]) == int(lens0[b]) + n + 1


def test_pack_ragged(cuda, oracle):
    from mlx_dspark_b200 import batch_engine

    rng = np.random.default_rng(8)
    for B in (1, 5, 37, 300):
        bl = rng.integers(8, 17, B).astype(np.int32)
        if B > 3:
            bl[2] = 0  # an idle slot
        kv = rng.integers(0, 5000, B).astype(np.int32)
        so = (np.arange(B, dtype=np.int64) * 123456)
        ids = rng.integers(0, 151936, (B, 16)).astype(np.int32)
        r_max = int(bl.sum()) + 3
        got = batch_engine.pack_ragged(torch.from_numpy(bl).to(cuda), torch.from_numpy(kv).to(cuda),
                                       torch.from_numpy(so).to(cuda), torch.from_numpy(ids).to(cuda),
                                       r_max)
        ref = oracle.pack_ragged(bl, kv, so, ids)
        R = int(ref["cu_rows"][-1])
        assert got["cu_rows"].cpu().tolist() == ref["cu_rows"]
        for key in ("row_pos", "row_kv", "row_req", "ids"):
            assert got[key][:R].cpu().tolist() == ref[key], key
        assert got["kv_len_new"].cpu().tolist() == ref["kv_len_new"]
