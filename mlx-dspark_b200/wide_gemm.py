"""Wide-M quantized matmul for prefill-width calls: the drop-in for ``wide_gemm``.

Mirrors src/mlx_dspark/wide_gemm.py: :func:`wide_matmul` (``:195-233``) patches
:class:`~.small_m_qmm.QuantizedLinear` at class level so that calls at least ``min_rows`` wide
run ``x @ dequantize(w).T`` (``:173-193``); :func:`active`, :func:`shape_key`,
:func:`quantized_linears`, :func:`widest_quantized_linear`, :func:`verified_shapes` and
``SAFE_MIN_ROWS`` keep their meaning.

Here the product is ``dspark_qmm_wide`` (``csrc/qmm_wide.cu``): the weights are dequantized once
per 128-row tile into tensor memory (rounded to bf16, as MLX's dequantize-to-activation-type
GEMM rounds them) and multiplied with 256 x rows per tcgen05 MMA. Differences a caller can see:

* the product is not bit-identical with the small-M kernels (those fold each group's exact
  integer product with its fp32 scale); :func:`verified_shapes` therefore checks the
  numerics gate of the small-M path (``_REL_TOL``) instead of bit identity;
* there is no CPU row split (the reference's ``cpu_split`` hands rows to the Apple CPU
  through unified memory; a discrete GPU has no such partner), so that argument is refused;
* the kernel needs K % 512 == 0 (groups of 64 loaded 8 at a time); other layers keep the
  stock path.
"""

from __future__ import annotations

import contextlib

import torch

from . import _lib, quant
from . import small_m_qmm as _sm
from ._torch import ptr, require_cuda, stream_of

QuantizedLinear = _sm.QuantizedLinear
SAFE_MIN_ROWS = 64       # below this the 32-row small-M launches are as fast
_REL_TOL = _sm._REL_TOL

_orig_call = QuantizedLinear.__call__
_min_rows = 0            # 0 = inactive
_shapes: frozenset | None = None


def _rows(x: torch.Tensor) -> int:
    return x.numel() // x.shape[-1] if x.shape[-1] else 0


def _in_features(mod) -> int:
    return int(mod["weight"].shape[1]) * 32 // int(mod.bits)


def _eligible(mod) -> bool:
    """Shapes the wide kernel serves: affine 4/8-bit g64 with bf16 scales/biases, K % 512 == 0
    (the reference's affine-only gate, src/mlx_dspark/wide_gemm.py:102-106)."""
    return (isinstance(mod, QuantizedLinear) and getattr(mod, "mode", "affine") == "affine"
            and "biases" in mod and int(mod.bits) in (4, 8) and int(mod.group_size) == 64
            and mod["scales"].dtype == torch.bfloat16 and _in_features(mod) % 512 == 0)


def shape_key(mod) -> str:
    return f"{_in_features(mod)}x{int(mod['weight'].shape[0])}x{int(mod.bits)}"


def wide(x2: torch.Tensor, weight: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor,
         bits: int, out: torch.Tensor | None = None) -> torch.Tensor:
    """``x2 [rows, K] @ dequant(W)^T`` in bf16 through the wide kernel."""
    require_cuda(x2, weight, scales, biases)
    if x2.dtype != torch.bfloat16 or scales.dtype != torch.bfloat16:
        raise _lib.DSparkUnsupported(_lib.ERR_UNSUPPORTED, "bf16 activations and scales only")
    rows, k = int(x2.shape[0]), int(x2.shape[1])
    n = int(weight.shape[0])
    if x2.stride(1) != 1 or (x2.stride(0) * 2) % 16:
        x2 = x2.contiguous()
    if out is None:
        out = torch.empty((rows, n), dtype=torch.bfloat16, device=x2.device)
    _lib.check(_lib.lib.dspark_qmm_wide(ptr(x2), x2.stride(0), rows, k, ptr(weight),
                                        ptr(scales.contiguous()), ptr(biases.contiguous()), n,
                                        int(bits), ptr(out), out.stride(0), stream_of(x2)))
    return out


def _wide_call(self, x):  # src/mlx_dspark/wide_gemm.py:173-193
    if not _eligible(self) or x.dtype != torch.bfloat16:
        return _orig_call(self, x)
    rows = _rows(x)
    if not _min_rows or rows < _min_rows:
        return _orig_call(self, x)
    if _shapes is not None and shape_key(self) not in _shapes:
        return _orig_call(self, x)
    k = x.shape[-1]
    y = wide(x.reshape(rows, k), self["weight"], self["scales"], self["biases"], int(self.bits))
    if "bias" in self:
        y = y + self["bias"]
    return y.reshape(*x.shape[:-1], y.shape[-1])


@contextlib.contextmanager
def wide_matmul(min_rows: int | None, shapes=None, cpu_split: dict | None = None):
    """Route :class:`QuantizedLinear` calls at least ``min_rows`` wide through the wide kernel
    while active (raised to ``SAFE_MIN_ROWS``); ``None`` / 0 is a no-op, nesting is a no-op,
    and the value found at entry is restored on exit, exceptions included. ``shapes`` is an
    allow-list of :func:`shape_key` values (``None``: every eligible shape)."""
    global _min_rows, _shapes
    if cpu_split:
        raise _lib.DSparkUnsupported(_lib.ERR_UNSUPPORTED,
                                     "cpu_split: no CPU row split on a discrete GPU")
    if not min_rows or QuantizedLinear.__call__ is _wide_call:
        yield
        return
    prev = QuantizedLinear.__call__
    _min_rows = max(int(min_rows), SAFE_MIN_ROWS)
    _shapes = None if shapes is None else frozenset(shapes)
    QuantizedLinear.__call__ = _wide_call
    try:
        yield
    finally:
        QuantizedLinear.__call__ = prev
        _min_rows = 0
        _shapes = None


def active() -> bool:
    return QuantizedLinear.__call__ is _wide_call


def quantized_linears(*models):
    """Every eligible :class:`QuantizedLinear` in the given modules (or iterables of them)."""
    for model in models:
        if model is None:
            continue
        mods = model.modules() if isinstance(model, torch.nn.Module) else model
        for mod in mods:
            if _eligible(mod):
                yield mod


def widest_quantized_linear(*models):
    """The eligible layer with the most weight words (a stand-in for the MLP matmuls)."""
    best, size = None, 0
    for mod in quantized_linears(*models):
        n = mod["weight"].numel()
        if n > size:
            best, size = mod, n
    return best


def verified_shapes(models, min_rows: int, widths: tuple[int, ...] = (512, 1024)) -> list[str]:
    """Shape keys whose wide-kernel output matches a torch dequantize-and-matmul within
    ``_REL_TOL`` at ``min_rows`` and each width (the gate of src/mlx_dspark/wide_gemm.py:
    297-320, with the small-M numerics bar instead of bit identity)."""
    ok, seen = [], set()
    for mod in quantized_linears(*([models] if isinstance(models, torch.nn.Module) else models)):
        key = shape_key(mod)
        if key in seen:
            continue
        seen.add(key)
        w = quant.dequantize(quant.QWeight(mod["weight"], mod["scales"], mod["biases"],
                                           int(mod.bits)))
        good = True
        for M in (max(min_rows, SAFE_MIN_ROWS), *widths):
            g = torch.Generator(device=w.device).manual_seed(M)
            x = torch.randn(M, _in_features(mod), device=w.device, generator=g).to(torch.bfloat16)
            ref = x.float() @ w.t()
            got = wide(x, mod["weight"], mod["scales"], mod["biases"], int(mod.bits)).float()
            if float((got - ref).abs().max()) > _REL_TOL * max(float(ref.abs().max()), 1.0):
                good = False
                break
        if good:
            ok.append(key)
    return ok
