"""dspark_p2p_allgather on one GPU (world = 1): the peer-memory all-gather's copy, completion
counters and round bookkeeping, over several gathers through two buffers of one arena.

With one rank the arena is only this process's own (no IPC mapping): every gather copies the
segment into segment 0 of its buffer, its blocks count themselves on the buffer's flag, block 0
waits for them (all blocks of one launch are resident at once), and the last block advances the
buffer's round. Segment sizes span one block (4 KB) to many (1 MB). The two-rank path is
tests/test_tp_gpu.py::test_tp2_matches_tp1[p2p].
"""

from __future__ import annotations

import ctypes as C

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

FLAGS, COUNTS, DATA = 0, 256, 512


def _arena(nbytes):
    from mlx_dspark_b200 import _lib

    base, handle = C.c_void_p(), (C.c_char * _lib.IPC_HANDLE_BYTES)()
    _lib.check(_lib.lib.dspark_ipc_alloc(nbytes, C.byref(base), handle))
    return base.value


def _view(addr, n):
    from mlx_dspark_b200.target_tp import _device_bytes

    return _device_bytes(addr, n, torch.device("cuda", 0))


def test_single_rank_gathers_copy_and_advance_rounds(cuda):
    from mlx_dspark_b200 import _lib

    _lib.ensure_init(0)
    segs = [4096, 1 << 20]  # bytes: one block, 64 blocks
    offs, off = [], DATA
    for n in segs:
        offs.append(off)
        off += (n + 255) // 256 * 256
    base = _arena(off)
    try:
        arenas = (C.c_void_p * 1)(base)
        g = torch.Generator(device=cuda).manual_seed(3)
        s = torch.cuda.current_stream(cuda).cuda_stream
        for step in range(5):
            for b, n in enumerate(segs):
                src = torch.randint(0, 256, (n,), dtype=torch.uint8, device=cuda, generator=g)
                a = _lib.P2PGatherArgs(C.cast(arenas, C.POINTER(C.c_void_p)), src.data_ptr(), n,
                                       FLAGS, COUNTS, offs[b], 0, 1, b)
                _lib.check(_lib.lib.dspark_p2p_allgather(C.byref(a), s))
                torch.cuda.synchronize()
                assert torch.equal(_view(base + offs[b], n), src), (step, b)
        torch.cuda.synchronize()
        head = _view(base, DATA).cpu().numpy().view(np.uint32)
        nblk = [max(1, min(148, -(-n // 16384))) for n in segs]
        for b in range(len(segs)):
            assert head[FLAGS // 4 + b * 8] == 5 * nblk[b]     # this rank's flag: 5 rounds
            assert head[COUNTS // 4 + b * 2] == 5               # round counter
            assert head[COUNTS // 4 + b * 2 + 1] == 0           # blocks-done counter reset
        assert _lib.device_status(0) == 0
    finally:
        torch.cuda.synchronize()
        _lib.lib.dspark_ipc_free(C.c_void_p(base))


def test_rejects_bad_arguments(cuda):
    from mlx_dspark_b200 import _lib

    _lib.ensure_init(0)
    base = _arena(4096)
    try:
        arenas = (C.c_void_p * 1)(base)
        src = torch.zeros(64, dtype=torch.uint8, device=cuda)
        s = torch.cuda.current_stream(cuda).cuda_stream
        for seg, rank, world, buf in ((40, 0, 1, 0), (64, 1, 1, 0), (64, 0, 9, 0), (64, 0, 1, 8)):
            a = _lib.P2PGatherArgs(C.cast(arenas, C.POINTER(C.c_void_p)), src.data_ptr(), seg,
                                   FLAGS, COUNTS, DATA, rank, world, buf)
            assert _lib.lib.dspark_p2p_allgather(C.byref(a), s) == _lib.ERR_ARG
    finally:
        _lib.lib.dspark_ipc_free(C.c_void_p(base))
