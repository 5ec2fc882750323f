"""K1 parity on the GPU: dspark_qmm vs the CPU oracle (mirrors tests/test_small_m_qmm.py).

Tolerance (stated by the build's north star): max|kernel - oracle| <= 1e-2 * max(max|oracle|, 1)
— stricter than the reference's 0.02 gate (src/mlx_dspark/small_m_qmm.py:120). Row-count
invariance is bit-exact (tests/test_small_m_qmm.py:107-119).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

TOL = 1e-2


def _weights(oracle, n, k, bits, seed):
    rng = np.random.default_rng(seed)
    w = rng.normal(0.0, 0.02, (n, k)).astype(np.float32)
    return oracle.quantize(w, bits)


def _to_dev(oracle, wq, sc, bi, dev):
    return (torch.from_numpy(wq.view(np.int32)).to(dev),
            torch.from_numpy(sc.view(np.int16)).view(torch.bfloat16).to(dev),
            torch.from_numpy(bi.view(np.int16)).view(torch.bfloat16).to(dev))


def _x(oracle, m, k, seed, scale=1.0):
    rng = np.random.default_rng(seed + 1000)
    return oracle.to_bf16(rng.normal(0.0, scale, (m, k)))


def _run(cuda, oracle, x_bits, wq, sc, bi, bits):
    from mlx_dspark_b200 import skinny_qmm

    w_d, s_d, b_d = _to_dev(oracle, wq, sc, bi, cuda)
    x = torch.from_numpy(x_bits.view(np.int16)).view(torch.bfloat16).to(cuda)
    y = skinny_qmm.qmm(x, w_d, s_d, b_d, bits)
    torch.cuda.synchronize()
    return y.float().cpu().numpy(), y


def _check(got, ref):
    scale = max(float(np.abs(ref).max()), 1.0)
    diff = float(np.abs(got - ref).max())
    assert diff <= TOL * scale, f"|d|={diff} vs max|y|={scale}"


@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("M", [1, 4, 5, 8, 9, 12, 16])
def test_microbench_shape_matches_oracle(cuda, oracle, bits, M):
    """The BASELINE microbench shape K = N = 4096, x ~ N(0,1), W ~ N(0, 0.02)."""
    K = N = 4096
    wq, sc, bi = _weights(oracle, N, K, bits, seed=bits)
    x = _x(oracle, M, K, seed=M)
    got, _ = _run(cuda, oracle, x, wq, sc, bi, bits)
    _check(got, oracle.qmm(x, wq, sc, bi, bits))


@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("N,K", [(4096, 512), (1024, 4096), (6144, 4096), (4096, 12288),
                                 (5120, 5120), (1024, 5120), (8192, 5120), (64, 512),
                                 (4096, 576), (1024, 640), (520, 1088)])
def test_shapes_window(cuda, oracle, bits, N, K):
    """Every plan family: wide / narrow N, split-K factors, K not a multiple of 512 (scales
    loaded without TMA), N not a multiple of the tile."""
    wq, sc, bi = _weights(oracle, N, K, bits, seed=N + K)
    for M in (1, 7, 16):
        x = _x(oracle, M, K, seed=M, scale=0.1)
        got, _ = _run(cuda, oracle, x, wq, sc, bi, bits)
        _check(got, oracle.qmm(x, wq, sc, bi, bits))


@pytest.mark.parametrize("bits", [4, 8])
def test_32_rows(cuda, oracle, bits):
    K, N = 2048, 2048
    wq, sc, bi = _weights(oracle, N, K, bits, seed=3)
    for M in (17, 24, 32):
        x = _x(oracle, M, K, seed=M)
        got, _ = _run(cuda, oracle, x, wq, sc, bi, bits)
        _check(got, oracle.qmm(x, wq, sc, bi, bits))


@pytest.mark.parametrize("bits", [4, 8])
def test_rows_are_row_count_invariant(cuda, oracle, bits):
    """A row's result does not depend on how many rows ride with it, within a row class
    (1-16 rows: the verify blocks; 17-32 rows): bit-exact. The geometry (split-K and with it
    the summation order) is fixed per weight shape and class."""
    K, N = 4096, 4096
    wq, sc, bi = _weights(oracle, N, K, bits, seed=11)
    x = _x(oracle, 32, K, seed=5)
    _, full16 = _run(cuda, oracle, x[:16], wq, sc, bi, bits)
    _, full32 = _run(cuda, oracle, x, wq, sc, bi, bits)
    for m in (1, 5, 8, 9, 15):
        _, part = _run(cuda, oracle, x[:m], wq, sc, bi, bits)
        assert torch.equal(full16[:m], part), m
    for m in (17, 24):
        _, part = _run(cuda, oracle, x[:m], wq, sc, bi, bits)
        assert torch.equal(full32[:m], part), m


def test_exact_integer_case(cuda, oracle):
    """Known answer: scale 1, bias 0, integer x -> the exact integer product (all exact in
    bf16 / fp32), checks the packing order of every nibble."""
    K, N, M = 1024, 256, 3
    rng = np.random.default_rng(7)
    q = rng.integers(0, 16, (N, K), dtype=np.uint32)
    wq = oracle.pack(q, 4)
    sc = oracle.to_bf16(np.ones((N, K // 64), np.float32))
    bi = oracle.to_bf16(np.zeros((N, K // 64), np.float32))
    xi = np.zeros((M, K), np.float32)
    for m in range(M):  # 16 non-zeros of +-1 per row: |y| <= 240, exact in bf16
        idx = rng.choice(K, 16, replace=False)
        xi[m, idx] = rng.choice([-1.0, 1.0], 16)
    got, _ = _run(cuda, oracle, oracle.to_bf16(xi), wq, sc, bi, 4)
    ref = xi @ q.T.astype(np.float32)
    assert np.abs(ref).max() < 256  # representable exactly in bf16
    np.testing.assert_array_equal(got, ref)


def test_bias_applies(cuda, oracle):
    from mlx_dspark_b200 import skinny_qmm

    K, N = 1024, 512
    wq, sc, bi = _weights(oracle, N, K, 4, seed=2)
    x = _x(oracle, 6, K, seed=2, scale=0.1)
    w_d, s_d, b_d = _to_dev(oracle, wq, sc, bi, cuda)
    bias = (torch.randn(N, device=cuda) * 0.5).to(torch.bfloat16)
    xd = torch.from_numpy(x.view(np.int16)).view(torch.bfloat16).to(cuda)
    y = skinny_qmm.qmm(xd, w_d, s_d, b_d, 4, bias=bias).float().cpu().numpy()
    ref = oracle.round_bf16(oracle.qmm(x, wq, sc, bi, 4)) + bias.float().cpu().numpy()
    _check(y, ref)


def test_rejects_unsupported(cuda):
    from mlx_dspark_b200 import DSparkUnsupported, skinny_qmm

    w = torch.zeros((64, 64), dtype=torch.int32, device=cuda)   # K = 512 at 4 bits
    s = torch.zeros((64, 8), dtype=torch.bfloat16, device=cuda)
    with pytest.raises(DSparkUnsupported):
        skinny_qmm.qmm(torch.zeros((33, 512), dtype=torch.bfloat16, device=cuda), w, s, s, 4)
    with pytest.raises(DSparkUnsupported):
        skinny_qmm.qmm(torch.zeros((2, 512), dtype=torch.bfloat16, device=cuda), w, s, s, 3)


@pytest.mark.parametrize("bits", [4, 8])
def test_deep_k_32_rows(cuda, oracle, bits):
    """17-32 rows on the down-projection shape (K = 12288). There, 32 staged rows of x leave
    shared memory for a high split-K factor only, and the planner may run the rows as two
    16-row launches. Parity with the oracle, and a row's result is the same bits whichever
    count of 17-32 rows rides with it."""
    N, K = 4096, 12288
    wq, sc, bi = _weights(oracle, N, K, bits, seed=21)
    x = _x(oracle, 32, K, seed=9, scale=0.1)
    _, full = _run(cuda, oracle, x, wq, sc, bi, bits)
    ref = oracle.qmm(x, wq, sc, bi, bits)
    _check(full.float().cpu().numpy(), ref)
    for m in (17, 24):
        got, part = _run(cuda, oracle, x[:m], wq, sc, bi, bits)
        _check(got, ref[:m])
        assert torch.equal(full[:m], part), m


def test_deep_k_32_rows_residual_epilogue(cuda, oracle):
    """The residual epilogue (down projection + residual add + the next RMSNorm's per-tile
    sums of squares) at 24 rows on the deep-K shape, through dspark_qmm_fused: rows 16-23
    land at their own output, residual and statistics slots."""
    import ctypes as C

    from mlx_dspark_b200 import _lib
    from mlx_dspark_b200._torch import ptr

    N, K, M, bits = 4096, 12288, 24, 4
    wq, sc, bi = _weights(oracle, N, K, bits, seed=23)
    x = _x(oracle, M, K, seed=4, scale=0.1)
    w_d, s_d, b_d = _to_dev(oracle, wq, sc, bi, cuda)
    xd = torch.from_numpy(x.view(np.int16)).view(torch.bfloat16).to(cuda)
    g = torch.Generator(device=cuda).manual_seed(5)
    resid = (torch.randn((M, N), device=cuda, generator=g) * 0.5).to(torch.bfloat16)
    out = torch.empty((M, N), dtype=torch.bfloat16, device=cuda)
    ntiles = N // 128
    ssq = torch.full((ntiles * 32,), float("nan"), dtype=torch.float32, device=cuda)
    a = _lib.QmmArgs()
    a.x, a.ldx, a.M, a.K, a.N, a.bits = ptr(xd), K, M, K, N, bits
    a.wq, a.scales, a.biases = ptr(w_d), ptr(s_d), ptr(b_d)
    a.out, a.ldo, a.epilogue = ptr(out), N, _lib.EPI_RESID
    a.resid, a.ldr, a.ssq_out, a.ssq_stride, a.eps = ptr(resid), N, ptr(ssq), 32, 1e-6
    _lib.check(_lib.lib.dspark_qmm_fused(C.byref(a), torch.cuda.current_stream(cuda).cuda_stream))
    torch.cuda.synchronize()
    got = out.float().cpu().numpy()
    ref = oracle.round_bf16(oracle.round_bf16(oracle.qmm(x, wq, sc, bi, bits)) +
                            resid.float().cpu().numpy())
    _check(got, ref)
    sums = (got.reshape(M, ntiles, 128) ** 2).sum(axis=2)  # [M, tiles]
    s = ssq.cpu().numpy().reshape(ntiles, 32)
    np.testing.assert_allclose(s[:, :M].T, sums, rtol=5e-3, atol=1e-3)
