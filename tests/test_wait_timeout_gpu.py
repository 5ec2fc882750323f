"""A bounded device wait that runs out (failure detection, no fault, no hang).

Every kernel wait of the library is bounded by a per-device limit (dspark_set_wait_limit_ns;
2 s by default). Here a peer-memory all-gather is launched as rank 0 of a world of 2 whose
"peer" arena is a second buffer on the same GPU that no kernel ever posts to: the gather's
completion wait for rank 1 can never be satisfied. With a 50 ms limit the launch must return
on its own, leave the timeout code in the device status word, and leave the stream and the
context usable: a normal QMM afterwards matches the oracle and leaves the status clean.
"""

from __future__ import annotations

import ctypes as C
import time

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

K_ERR_WAIT_PEER = 0x105  # DeviceError::kErrWaitPeer (csrc/common.cuh)


def test_gather_wait_runs_out_and_the_device_stays_usable(cuda, oracle):
    from mlx_dspark_b200 import _lib, skinny_qmm

    dev = cuda.index if cuda.index is not None else 0
    assert _lib.device_status(dev) == 0
    seg = 4096
    flags_off, count_off, dst_off = 0, 256, 512
    size = dst_off + 2 * seg
    arenas = [torch.zeros(size, dtype=torch.uint8, device=cuda) for _ in range(2)]
    src = torch.arange(seg, dtype=torch.int32, device=cuda).view(torch.uint8)[:seg].clone()
    ptrs = (C.c_void_p * 2)(arenas[0].data_ptr(), arenas[1].data_ptr())
    args = _lib.P2PGatherArgs(ptrs, src.data_ptr(), seg, flags_off, count_off, dst_off, 0, 2, 0)
    limit_ns = 50_000_000
    _lib.set_wait_limit_ns(dev, limit_ns)
    try:
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        _lib.check(_lib.lib.dspark_p2p_allgather(C.byref(args),
                                                 torch.cuda.current_stream().cuda_stream))
        torch.cuda.synchronize()
        dt = time.perf_counter() - t0
    finally:
        _lib.set_wait_limit_ns(dev, 0)
    # the launch returned by itself after about the limit, and said why
    assert 0.8 * limit_ns / 1e9 <= dt < 1.5, dt
    assert _lib.device_status(dev, clear=True) == K_ERR_WAIT_PEER
    assert _lib.device_status(dev) == 0
    # this rank's own segment landed in both arenas (only the wait for the peer failed)
    for a in arenas:
        assert torch.equal(a[dst_off : dst_off + seg], src)

    # the stream and the context are usable: a normal QMM matches the oracle
    rng = np.random.default_rng(3)
    N, K = 1024, 2048
    wq, sc, bi = oracle.quantize(rng.normal(0, 0.02, (N, K)).astype(np.float32), 4)
    x = oracle.to_bf16(rng.normal(0, 1, (16, K)))
    t = lambda a, dt=None: torch.from_numpy(a).to(cuda)  # noqa: E731
    y = skinny_qmm.qmm(t(x.view(np.int16)).view(torch.bfloat16), t(wq.view(np.int32)),
                       t(sc.view(np.int16)).view(torch.bfloat16),
                       t(bi.view(np.int16)).view(torch.bfloat16), 4)
    ref = oracle.qmm(x, wq, sc, bi, 4)
    err = float(np.abs(y.float().cpu().numpy() - ref).max())
    assert err <= 1e-2 * max(float(np.abs(ref).max()), 1.0)
    assert _lib.device_status(dev) == 0
