"""Wide-M quantized matmul (dspark_qmm_wide, tcgen05) against the oracle.

The reference's wide path computes x @ mx.dequantize(w).T for prefill-width calls
(src/mlx_dspark/wide_gemm.py:1-30): the weights dequantized once (rounded to the activation
type) and a plain GEMM. Here the weights are dequantized into tensor memory per 128-row tile,
rounded once to bf16, and multiplied with up to 256 x rows per MMA in fp32. Bar: max |diff| <=
1e-2 * max |ref| against the oracle's exact fp32 product, at several row counts (tails included),
4- and 8-bit, and a weight-row tail.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _bf(a, dev):
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(torch.bfloat16).to(dev)


@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("M,N,K", [(64, 1024, 4096), (300, 1536, 2048), (768, 4096, 1024),
                                   (257, 1000, 1536), (33, 256, 12288)])
def test_wide_matches_oracle(cuda, oracle, bits, M, N, K):
    from mlx_dspark_b200 import _lib

    rng = np.random.default_rng(M + N + bits)
    wq, sc, bi = oracle.quantize(rng.normal(0, 0.02, (N, K)).astype(np.float32), bits)
    x = oracle.to_bf16(rng.normal(0, 1, (M, K)))
    out = torch.full((M, N + 8), float("nan"), dtype=torch.bfloat16, device=cuda)
    xt, w = _bf(x, cuda), torch.from_numpy(wq.view(np.int32)).to(cuda)
    s, b = _bf(sc, cuda), _bf(bi, cuda)
    _lib.check(_lib.lib.dspark_qmm_wide(xt.data_ptr(), K, M, K, w.data_ptr(), s.data_ptr(),
                                        b.data_ptr(), N, bits, out.data_ptr(), N + 8,
                                        torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    got = out[:, :N].float().cpu().numpy()
    ref = oracle.qmm(x, wq, sc, bi, bits)
    err = float(np.abs(got - ref).max())
    assert err <= 1e-2 * float(np.abs(ref).max()), err
    assert torch.isnan(out[:, N:].float()).all()  # nothing written past the row
    assert _lib.device_status(cuda.index or 0) == 0


def test_wide_refuses_unaligned_k(cuda):
    from mlx_dspark_b200 import _lib

    t = torch.zeros(1 << 16, dtype=torch.int32, device=cuda)
    rc = _lib.lib.dspark_qmm_wide(t.data_ptr(), 576, 64, 576, t.data_ptr(), t.data_ptr(),
                                  t.data_ptr(), 128, 4, t.data_ptr(), 128, None)
    assert rc == _lib.ERR_UNSUPPORTED and "512" in _lib.last_error()


def test_wide_matmul_route_runs_the_kernel(cuda, oracle, monkeypatch):
    """A QuantizedLinear called 300 rows wide inside wide_matmul(64) takes the wide kernel
    (src/mlx_dspark/wide_gemm.py:173-193) and matches the oracle; a 40-row call stays on the
    stock path; verified_shapes admits the shape."""
    from mlx_dspark_b200 import _lib, quant, small_m_qmm, wide_gemm as wg

    rng = np.random.default_rng(3)
    N, K = 1536, 4096
    wq, sc, bi = oracle.quantize(rng.normal(0, 0.02, (N, K)).astype(np.float32), 4)
    mod = small_m_qmm.QuantizedLinear(quant.QWeight(
        torch.from_numpy(wq.view(np.int32)).to(cuda), _bf(sc, cuda), _bf(bi, cuda), 4))
    calls = []
    real = wg.wide
    monkeypatch.setattr(wg, "wide", lambda *a, **k: calls.append(a[0].shape[0]) or real(*a, **k))
    x = oracle.to_bf16(rng.normal(0, 1, (300, K)))
    xt = _bf(x, cuda).reshape(2, 150, K)
    with wg.wide_matmul(64):
        y = mod(xt)
        mod(xt[:, :20])  # 40 rows: below the floor
    assert calls == [300]
    ref = oracle.qmm(x, wq, sc, bi, 4)
    got = y.reshape(300, N).float().cpu().numpy()
    assert float(np.abs(got - ref).max()) <= 1e-2 * float(np.abs(ref).max())
    assert wg.verified_shapes([mod], 64, widths=(256,)) == [wg.shape_key(mod)]
    assert _lib.device_status(cuda.index or 0) == 0
