"""The allocation-free verify attention entry point (dspark_verify_attn_noalloc).

Callers that cannot allocate device memory — code being captured into a CUDA graph, plugins
whose runtime owns all device memory, paths that must not stall on an allocation — call this
variant, which keeps its scratch in a static device array inside the library. This test calls it
through the C ABI on a shape that needs scratch, twice in a row with different inputs, and checks
each result against the regular entry point (which takes a caller-allocated workspace).

The file is named so that pytest collects it last.
"""

import ctypes as C

import numpy as np
import pytest
import torch

from mlx_dspark_b200 import _lib
from mlx_dspark_b200._torch import elem_strides, ptr, stream_of
from mlx_dspark_b200.multirow_attn import multirow_sdpa

pytestmark = pytest.mark.gpu


def _noalloc(q, k, v, scale, causal):
    B, Hq, qL, D = (int(s) for s in q.shape)
    Hk, L = int(k.shape[1]), int(k.shape[2])
    out = torch.empty_like(q)
    _lib.check(_lib.lib.dspark_verify_attn_noalloc(
        ptr(q), _lib.i64_array(elem_strides(q)), ptr(k), _lib.i64_array(elem_strides(k)),
        ptr(v), _lib.i64_array(elem_strides(v)), B, Hq, Hk, qL, D, L, None, float(scale),
        int(causal), None, ptr(out), _lib.i64_array(elem_strides(out)), stream_of(q)))
    return out


def test_noalloc_matches_the_workspace_entry_point_twice(oracle):
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    _lib.ensure_init(0)
    B, Hq, Hk, qL, D, L = 1, 32, 8, 16, 128, 32768
    ws = int(_lib.lib.dspark_verify_attn_workspace(B, Hq, Hk, qL, D, L))
    assert 0 < ws <= 4 << 20, "the shape must exercise the scratch array and fit it"
    g = torch.Generator(device=dev).manual_seed(11)
    scale = D ** -0.5
    for call in range(2):
        q = torch.randn((B, Hq, qL, D), device=dev, generator=g).to(torch.bfloat16)
        k = torch.randn((B, Hk, L, D), device=dev, generator=g).to(torch.bfloat16)
        v = torch.randn((B, Hk, L, D), device=dev, generator=g).to(torch.bfloat16)
        got = _noalloc(q, k, v, scale, True)
        ref = multirow_sdpa(q, k, v, scale=scale, causal=True)
        torch.cuda.synchronize()
        err = float((got.float() - ref.float()).abs().max())
        tol = 1e-2 * float(ref.float().abs().max())
        assert err <= tol, f"call {call}: max |diff| {err} > {tol}"
        if call == 0:
            # and against the CPU oracle's attention at this 32k-key shape
            bits = lambda t: t.cpu().contiguous().view(torch.int16).numpy().view(np.uint16)  # noqa: E731
            want = oracle.sdpa(bits(q), bits(k), bits(v), scale, True)
            err_o = float(np.abs(got.float().cpu().numpy() - want).max())
            tol_o = 1e-2 * float(np.abs(want).max())
            assert err_o <= tol_o, f"vs oracle: max |diff| {err_o} > {tol_o}"
    assert _lib.device_status(0) == 0


def test_noalloc_refuses_shapes_beyond_its_scratch(monkeypatch):
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    _lib.ensure_init(0)
    # force a split plan whose cross-cluster partials need far more than the static array
    monkeypatch.setenv("DSPARK_ATTN_SPLITS", "64")
    B, Hq, Hk, qL, D, L = 4, 64, 8, 16, 128, 65536
    need = int(_lib.lib.dspark_verify_attn_workspace(B, Hq, Hk, qL, D, L))
    assert need > 4 << 20
    q = torch.zeros((1, 1, 1, 8), dtype=torch.bfloat16, device=dev)
    st = _lib.i64_array([0, 0, 0])
    rc = _lib.lib.dspark_verify_attn_noalloc(ptr(q), st, ptr(q), st, ptr(q), st, B, Hq, Hk, qL,
                                             D, L, None, 0.1, 1, None, ptr(q), st,
                                             stream_of(q))
    assert rc == _lib.ERR_UNSUPPORTED
    assert "static maximum" in _lib.last_error()
