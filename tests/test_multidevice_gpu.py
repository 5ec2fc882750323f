"""One process driving two GPUs: the kernels' launch attributes (dynamic shared memory above
48 KB, clusters of up to 16) belong to each device's context, so the library configures every
kernel once per device. QMM and attention run on device 0 and then on device 1 of the same
process and both match the oracle. Skipped with fewer than two GPUs."""

from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_kernels_on_two_devices_in_one_process(oracle):
    import mlx_dspark_b200  # noqa: F401
    from mlx_dspark_b200 import _lib, skinny_qmm
    from mlx_dspark_b200.multirow_attn import multirow_sdpa

    rng = np.random.default_rng(1)
    N, K = 4096, 4096
    wq, sc, bi = oracle.quantize(rng.normal(0, 0.02, (N, K)).astype(np.float32), 4)
    x = oracle.to_bf16(rng.normal(0, 1, (16, K)))
    ref_q = oracle.qmm(x, wq, sc, bi, 4)
    g = torch.Generator().manual_seed(2)
    q = torch.randn((1, 32, 16, 128), generator=g).to(torch.bfloat16)
    k = torch.randn((1, 8, 32768, 128), generator=g).to(torch.bfloat16)
    v = torch.randn((1, 8, 32768, 128), generator=g).to(torch.bfloat16)
    bits = lambda t: t.contiguous().view(torch.int16).numpy().view(np.uint16)  # noqa: E731
    ref_a = oracle.sdpa(bits(q), bits(k), bits(v), 128 ** -0.5, True)
    prev = torch.cuda.current_device()
    try:
        for d in (0, 1):
            dev = torch.device("cuda", d)
            torch.cuda.set_device(dev)
            _lib.ensure_init(d)
            bf = lambda a: torch.from_numpy(a.view(np.int16)).view(torch.bfloat16).to(dev)  # noqa: E731
            y = skinny_qmm.qmm(bf(x), torch.from_numpy(wq.view(np.int32)).to(dev), bf(sc),
                               bf(bi), 4)
            o = multirow_sdpa(q.to(dev), k.to(dev), v.to(dev), scale=128 ** -0.5, causal=True)
            torch.cuda.synchronize(dev)
            eq = float(np.abs(y.float().cpu().numpy() - ref_q).max())
            assert eq <= 1e-2 * float(np.abs(ref_q).max()), (d, eq)
            ea = float(np.abs(o.float().cpu().numpy() - ref_a).max())
            assert ea <= 1e-2 * float(np.abs(ref_a).max()), (d, ea)
            assert _lib.device_status(d) == 0
    finally:
        torch.cuda.set_device(prev)
