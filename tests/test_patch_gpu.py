"""The drop-in routes reach the kernels on the GPU.

The reference's verify loop never calls its kernels directly: it runs the model inside
``small_m_matmul(ids)`` (a class patch of ``QuantizedLinear.__call__``,
src/mlx_dspark/small_m_qmm.py:71-106) and ``multirow_attention(cfg)`` (a patch of the SDPA
entry point, src/mlx_dspark/multirow_attn.py:338-370). These tests call a patched layer and the
patched SDPA the way model code does and check that (1) the call went through the kernel route
(the route's function ran and the library launched kernels), (2) the result matches the oracle,
(3) calls outside the gate fall through to the previously installed function.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _bf(a, dev):
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(torch.bfloat16).to(dev)


@pytest.mark.parametrize("bits", [4, 8])
def test_patched_quantized_linear_runs_the_kernel(cuda, oracle, monkeypatch, bits):
    from mlx_dspark_b200 import _lib, quant, skinny_qmm, small_m_qmm

    rng = np.random.default_rng(bits)
    N, K = 1536, 4096
    wq, sc, bi = oracle.quantize(rng.normal(0, 0.02, (N, K)).astype(np.float32), bits)
    bias = oracle.to_bf16(rng.normal(0, 0.1, N))
    mod = small_m_qmm.QuantizedLinear(
        quant.QWeight(torch.from_numpy(wq.view(np.int32)).to(cuda), _bf(sc, cuda), _bf(bi, cuda),
                      bits), bias=_bf(bias, cuda))
    calls = []
    real_call = skinny_qmm.call
    monkeypatch.setattr(skinny_qmm, "call",
                        lambda m, x, rows: calls.append(rows) or real_call(m, x, rows))
    x = oracle.to_bf16(rng.normal(0, 1, (12, K)))
    xt = _bf(x, cuda).reshape(1, 12, K)  # model code passes [B, T, K]
    before = int(_lib.lib.dspark_launch_count())
    with small_m_qmm.small_m_matmul(frozenset({id(mod)})):
        assert small_m_qmm.active()
        y = mod(xt)
    assert not small_m_qmm.active()
    assert calls == [12], "the in-window call must take the kernel route"
    assert int(_lib.lib.dspark_launch_count()) > before
    ref = oracle.round_bf16(oracle.qmm(x, wq, sc, bi, bits)) + oracle.from_bf16(bias)[None]
    got = y.float().cpu().numpy().reshape(12, N)
    assert float(np.abs(got - ref).max()) <= 1e-2 * max(float(np.abs(ref).max()), 1.0)
    # not allow-listed: falls through to the stock call (no skinny route)
    other = small_m_qmm.QuantizedLinear(quant.QWeight(mod.weight, mod.scales, mod.biases, bits))
    with small_m_qmm.small_m_matmul(frozenset({id(mod)})):
        other(xt)
    assert calls == [12]


def test_patched_sdpa_runs_the_kernel(cuda, oracle, monkeypatch):
    from mlx_dspark_b200 import _lib
    from mlx_dspark_b200 import multirow_attn as ma

    g = torch.Generator().manual_seed(4)
    B, Hq, Hk, qL, D, L = 1, 32, 8, 16, 128, 2048
    q = torch.randn((B, Hq, qL, D), generator=g).to(torch.bfloat16)
    k = torch.randn((B, Hk, L, D), generator=g).to(torch.bfloat16)
    v = torch.randn((B, Hk, L, D), generator=g).to(torch.bfloat16)
    bits = lambda t: t.contiguous().view(torch.int16).numpy().view(np.uint16)  # noqa: E731
    ref = oracle.sdpa(bits(q), bits(k), bits(v), D ** -0.5, True)
    calls = []
    real = ma.multirow_sdpa
    monkeypatch.setattr(ma, "multirow_sdpa",
                        lambda *a, **kw: calls.append(kw.get("causal")) or real(*a, **kw))
    cfg = ma.MultirowConfig((ma.default_window(Hq, Hk, D),))
    qd, kd, vd = q.to(cuda), k.to(cuda), v.to(cuda)
    before = int(_lib.lib.dspark_launch_count())
    with ma.multirow_attention(cfg):
        assert ma.active()
        out = ma.sdpa(qd, kd, vd, scale=D ** -0.5, mask="causal")
        # a boolean array mask is not eligible: the stock function serves it
        m = torch.ones((qL, L), dtype=torch.bool, device=cuda)
        out_m = ma.sdpa(qd, kd, vd, scale=D ** -0.5, mask=m)
    assert not ma.active()
    assert calls == [True], calls
    assert int(_lib.lib.dspark_launch_count()) > before
    err = float(np.abs(out.float().cpu().numpy() - ref).max())
    assert err <= 1e-2 * float(np.abs(ref).max()), err
    ref_full = oracle.sdpa(bits(q), bits(k), bits(v), D ** -0.5, False)
    err_m = float(np.abs(out_m.float().cpu().numpy() - ref_full).max())
    assert err_m <= 1e-2 * float(np.abs(ref_full).max()), err_m


def test_patched_sdpa_tree_mask_runs_the_tree_kernel(cuda, oracle):
    from mlx_dspark_b200 import multirow_attn as ma

    g = torch.Generator().manual_seed(5)
    B, Hq, Hk, qL, D, L = 1, 16, 4, 8, 128, 700
    q = torch.randn((B, Hq, qL, D), generator=g).to(torch.bfloat16)
    k = torch.randn((B, Hk, L, D), generator=g).to(torch.bfloat16)
    v = torch.randn((B, Hk, L, D), generator=g).to(torch.bfloat16)
    parent = [-1, 0, 0, 1, 1, 2, 3, 5]
    anc = ma.tree_bits(parent)
    mask = torch.ones((qL, L), dtype=torch.bool, device=cuda)  # identity-matched token
    anc_t = torch.tensor(anc, dtype=torch.int32, device=cuda)
    cfg = ma.MultirowConfig((ma.default_window(Hq, Hk, D),))
    with ma.multirow_attention(cfg), ma.tree_mask(mask, anc_t):
        out = ma.sdpa(q.to(cuda), k.to(cuda), v.to(cuda), scale=D ** -0.5, mask=mask)
    bits = lambda t: t.contiguous().view(torch.int16).numpy().view(np.uint16)  # noqa: E731
    ref = oracle.sdpa(bits(q), bits(k), bits(v), D ** -0.5, False,
                      anc=np.array(anc, dtype=np.uint32))
    err = float(np.abs(out.float().cpu().numpy() - ref).max())
    assert err <= 1e-2 * float(np.abs(ref).max()), err


@pytest.mark.parametrize("sdt", [torch.float16, torch.float32])
def test_fp16_fp32_scales_stay_on_the_stock_path(cuda, oracle, monkeypatch, sdt):
    """A layer whose scales are fp16 / fp32 does not fit the kernel (it reads bf16 scales):
    inside small_m_matmul it is served by the stock dequantize-and-matmul, correctly."""
    from mlx_dspark_b200 import quant, skinny_qmm, small_m_qmm

    rng = np.random.default_rng(5)
    N, K = 256, 1024
    wq, sc, bi = oracle.quantize(rng.normal(0, 0.02, (N, K)).astype(np.float32), 4)
    s32, b32 = oracle.from_bf16(sc), oracle.from_bf16(bi)
    mod = small_m_qmm.QuantizedLinear(quant.QWeight(
        torch.from_numpy(wq.view(np.int32)).to(cuda), torch.from_numpy(s32).to(sdt).to(cuda),
        torch.from_numpy(b32).to(sdt).to(cuda), 4))
    calls = []
    monkeypatch.setattr(skinny_qmm, "call", lambda *a: calls.append(1))
    x = oracle.to_bf16(rng.normal(0, 1, (8, K)))
    with small_m_qmm.small_m_matmul(frozenset({id(mod)})):
        y = mod(_bf(x, cuda))
    assert calls == []
    ref = oracle.qmm(x, wq, sc, bi, 4)  # bf16 scales are exact in fp16 / fp32 here
    assert float(np.abs(y.float().cpu().numpy() - ref).max()) <= 1e-2 * float(np.abs(ref).max())
