"""Column-sharded verify forward (target_tp.TPTarget) on the GPU.

* P = 1 against the oracle's Qwen3 forward (bars as in test_forward_gpu.py): exercises the fused
  QMM entry point, segmented x rows and the gather-based layer sequence on one GPU;
* P = 2 against P = 1 on the same seeded model and cache (two GPUs, skipped with fewer), with
  the gathers fused into the projections' peer stores, over peer memory by separate launches,
  and over NCCL: logits within the bf16 noise of the single-rank
  forward for two blocks in a row, identical on both ranks, identical cache lengths.
"""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch

from test_forward_gpu import _compare, _rel

pytestmark = pytest.mark.gpu


def _fill_cache(t, L0, seed):
    """Seeded full-head K/V prefix; each rank keeps its own heads' slice."""
    g = torch.Generator().manual_seed(seed)
    cfg = t.cfg
    full = []
    for L in t.layers:
        k = torch.randn((cfg.n_kv_heads, L0, cfg.head_dim), generator=g).to(torch.bfloat16)
        v = torch.randn((cfg.n_kv_heads, L0, cfg.head_dim), generator=g).to(torch.bfloat16)
        a, b = t.rank * t.hk, (t.rank + 1) * t.hk
        L["k_cache"][:, :L0].copy_(k[a:b])
        L["v_cache"][:, :L0].copy_(v[a:b])
        full.append((k, v))
    return full


@pytest.mark.parametrize("bits", [4, 8])
def test_tp1_matches_oracle(cuda, oracle, bits):
    from mlx_dspark_b200.target import tiny_config
    from mlx_dspark_b200.target_tp import TPTarget

    cfg = tiny_config(bits=bits)
    t = TPTarget(cfg, 0, 1, kv_cap=1024, seed=bits, max_rows=16)
    L0, R = 300, 16
    full = _fill_cache(t, L0, seed=5)
    ids = torch.randint(0, cfg.vocab, (R,), device=cuda, dtype=torch.int32)
    lens = torch.tensor([L0], dtype=torch.int32, device=cuda)
    logits = t.verify(ids, lens).float().cpu().numpy()
    assert int(lens[0]) == L0 + R
    kc = [np.zeros((cfg.n_kv_heads, 1024, cfg.head_dim), np.float32) for _ in t.layers]
    vc = [np.zeros((cfg.n_kv_heads, 1024, cfg.head_dim), np.float32) for _ in t.layers]
    for li, (k, v) in enumerate(full):
        kc[li][:, :L0] = k.float().numpy()
        vc[li][:, :L0] = v.float().numpy()
    ow, oc = t.oracle_weights(), t.oracle_config()
    ref_p = oracle.verify_forward(ow, oc, ids.cpu().numpy(), [c.copy() for c in kc],
                                  [c.copy() for c in vc], L0, round_p=True)
    ref = oracle.verify_forward(ow, oc, ids.cpu().numpy(), kc, vc, L0)
    _compare(oracle, logits, ref, ref_p)
    out = t.accept_and_rollback(t.b["logits_full"][:R], ids, lens)
    torch.cuda.synchronize()
    assert int(lens[0]) == L0 + int(out["n"][0]) + 1


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _tp_worker(rank, world, port, q, comm):
    import datetime

    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=120))
    try:
        import mlx_dspark_b200  # noqa: F401
        from mlx_dspark_b200 import _lib
        from mlx_dspark_b200.target import tiny_config
        from mlx_dspark_b200.target_tp import TPTarget

        _lib.ensure_init(rank)
        cfg = tiny_config(bits=8)
        t = TPTarget(cfg, rank, world, group=dist.group.WORLD, kv_cap=1024, seed=8,
                     max_rows=16, device=dev, comm=comm)
        _fill_cache(t, 300, seed=5)
        g = torch.Generator().manual_seed(9)
        ids = torch.randint(0, cfg.vocab, (16,), generator=g, dtype=torch.int32).to(dev)
        lens = torch.tensor([300], dtype=torch.int32, device=dev)
        logits = t.verify(ids, lens).float().cpu().numpy()
        out = t.accept_and_rollback(t.b["logits_full"][:16], ids, lens)
        torch.cuda.synchronize()
        ln = int(lens[0])
        # a second block at the same position (its K/V rows overwrite the first's) through the
        # same gather buffers: the peers' completion counters must advance in step
        ids2 = torch.randint(0, cfg.vocab, (16,), generator=g, dtype=torch.int32).to(dev)
        lens.fill_(300)
        logits2 = t.verify(ids2, lens).float().cpu().numpy()
        torch.cuda.synchronize()
        st = _lib.device_status(rank)
        t.close()
        q.put((rank, logits, logits2, ln, int(out["n"][0]), st))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("comm", ["fused", "p2p", "nccl"])
def test_tp2_matches_tp1(cuda, comm):
    import torch.multiprocessing as mp

    from mlx_dspark_b200.target import tiny_config
    from mlx_dspark_b200.target_tp import TPTarget

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_tp_worker, args=(r, 2, port, q, comm)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    for _ in procs:
        rank, logits, logits2, ln, n, st = q.get(timeout=600)
        res[rank] = (logits, logits2, ln, n, st)
    for p in procs:
        p.join(timeout=120)
    cfg = tiny_config(bits=8)
    t = TPTarget(cfg, 0, 1, kv_cap=1024, seed=8, max_rows=16)
    _fill_cache(t, 300, seed=5)
    g = torch.Generator().manual_seed(9)
    ids = torch.randint(0, cfg.vocab, (16,), generator=g, dtype=torch.int32).to(cuda)
    lens = torch.tensor([300], dtype=torch.int32, device=cuda)
    ref = t.verify(ids, lens).float().cpu().numpy()
    ids2 = torch.randint(0, cfg.vocab, (16,), generator=g, dtype=torch.int32).to(cuda)
    lens.fill_(300)
    ref2 = t.verify(ids2, lens).float().cpu().numpy()
    for rank in (0, 1):
        logits, logits2, ln, n, st = res[rank]
        assert st == 0
        assert _rel(logits, ref) <= 1e-2, (rank, _rel(logits, ref))
        assert _rel(logits2, ref2) <= 1e-2, (rank, _rel(logits2, ref2))
        assert ln == 300 + n + 1
    assert np.array_equal(res[0][0], res[1][0])  # every rank holds the same logits
    assert np.array_equal(res[0][1], res[1][1])
