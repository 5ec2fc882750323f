"""Host-side logic of the column-sharded forward (mlx_dspark_b200.target_tp), on CPU.

* every rank's row ranges tile the full matrices exactly once;
* the segmented-row addressing the QMM uses to read an all-gather's [P, M, K/P] output
  (element k of row m at (k // seg) * seg_stride + m * ldx + k % seg) recovers the full rows,
  checked through a real two-rank gloo all-gather.
"""

from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import mlx_dspark_b200  # noqa: F401  (library load only; no GPU call here)
from mlx_dspark_b200.target import QWEN3_32B, tiny_config
from mlx_dspark_b200.target_tp import shard_ranges


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_shard_ranges_tile_the_matrices(world):
    cfg = QWEN3_32B
    H, D, Hq, Hk, I, V = (cfg.hidden, cfg.head_dim, cfg.n_heads, cfg.n_kv_heads,
                          cfg.intermediate, cfg.vocab)
    full = {"q": (0, Hq * D), "k": (Hq * D, (Hq + Hk) * D), "v": ((Hq + Hk) * D, (Hq + 2 * Hk) * D),
            "hidden": (0, H), "inter": (0, I), "vocab": (0, V)}
    for key, (lo, hi) in full.items():
        covered = []
        for r in range(world):
            a, b = shard_ranges(cfg, world, r)[key]
            covered.extend(range(a, b))
        assert covered == list(range(lo, hi)), key


def test_shard_ranges_refuse_uneven_splits():
    with pytest.raises(ValueError):
        shard_ranges(tiny_config(), 3, 0)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _gather_worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    M, K = 5, 24
    full = torch.arange(M * K, dtype=torch.float32).reshape(M, K)
    seg = K // world
    shard = full[:, rank * seg:(rank + 1) * seg].contiguous()
    out = torch.empty(world * M * seg)
    dist.all_gather_into_tensor(out, shard.reshape(-1))
    ok = True
    for m in range(M):
        for k in range(K):
            idx = (k // seg) * (M * seg) + m * seg + k % seg
            ok &= bool(out[idx] == full[m, k])
    q.put((rank, ok))
    dist.destroy_process_group()


def test_segmented_rows_read_an_all_gather_gloo():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gather_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert res == {0: True, 1: True}
