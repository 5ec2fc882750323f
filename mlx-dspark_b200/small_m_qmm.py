"""Small-M quantized matmul dispatch: allowlist, window, scoped patch (mirrors
src/mlx_dspark/small_m_qmm.py).

The reference patches ``mlx.nn.QuantizedLinear.__call__`` inside ``small_m_matmul(ids)`` so
allow-listed instances with a row count in their width's window run the skinny kernel
(``:71-106``). Here :class:`QuantizedLinear` is a torch module holding MLX-layout packed
weights on the GPU; its stock ``__call__`` is :func:`~.skinny_qmm.quantized_matmul` (the
same kernel in 32-row launches), and :func:`small_m_matmul` installs the same scoped,
nesting, exception-safe class patch routing in-window calls through
:func:`~.skinny_qmm.call`.

:func:`measure_shapes` keeps the reference's numerics gate (``_REL_TOL``, ``:120``) against a
dequantize-and-matmul computed with torch on the same device; the reference's speed race is
not needed (the kernel is the only quantized matmul here).
"""

from __future__ import annotations

import contextlib

import torch

from . import quant
from . import skinny_qmm as _sk

M4_MIN, M4_MAX = _sk.WINDOW[4]
M8_MIN, M8_MAX = _sk.WINDOW[8]
M_MIN, M_MAX = M8_MIN, M8_MAX

_REL_TOL = 0.02   # max|kernel - reference| <= _REL_TOL * max(max|reference|, 1)


class QuantizedLinear(torch.nn.Module):
    """Affine-quantized linear layer in MLX's packed layout (weight int32/uint32 words,
    bf16 scales/biases, optional bf16 bias). Supports ``mod["weight"]`` style access like
    mlx.nn.Module."""

    def __init__(self, qw: quant.QWeight, bias: torch.Tensor | None = None,
                 group_size: int = quant.GROUP):
        super().__init__()
        self.bits = int(qw.bits)
        self.group_size = int(group_size)
        self.mode = "affine"
        self.register_buffer("weight", qw.wq)
        self.register_buffer("scales", qw.scales)
        self.register_buffer("biases", qw.biases)
        if bias is not None:
            self.register_buffer("bias", bias.to(torch.bfloat16))

    @classmethod
    def from_linear(cls, linear, group_size: int = quant.GROUP, bits: int = 4):
        """Quantize a ``torch.nn.Linear`` (or a weight tensor ``[out, in]``)."""
        if isinstance(linear, torch.Tensor):
            w, b = linear, None
        else:
            w, b = linear.weight.detach(), linear.bias
        if group_size != quant.GROUP or bits not in (4, 8):
            qw = quant.QWeight(torch.zeros(w.shape[0], max(1, w.shape[1] * bits // 32),
                                           dtype=torch.int32, device=w.device),
                               torch.zeros(w.shape[0], max(1, w.shape[1] // group_size),
                                           dtype=torch.bfloat16, device=w.device),
                               torch.zeros(w.shape[0], max(1, w.shape[1] // group_size),
                                           dtype=torch.bfloat16, device=w.device), bits)
            mod = cls(qw, None if b is None else b.detach(), group_size)
            return mod
        return cls(quant.quantize(w, bits, group_size), None if b is None else b.detach(),
                   group_size)

    def __getitem__(self, key: str) -> torch.Tensor:
        if key in ("weight", "scales", "biases", "bias") and hasattr(self, key):
            return getattr(self, key)
        raise KeyError(key)

    def __contains__(self, key: str) -> bool:
        return key in ("weight", "scales", "biases", "bias") and hasattr(self, key)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        bias = self.bias if "bias" in self else None
        if self.scales.dtype != torch.bfloat16 or self.biases.dtype != torch.bfloat16:
            # fp16 / fp32 scales: the kernels read bf16 scales, so these layers keep MLX's stock
            # semantics (w = scale * q + bias in fp32, fp32 accumulation, output in x's type)
            w = quant.dequantize(quant.QWeight(self.weight, self.scales, self.biases, self.bits))
            y = (x.float() @ w.t()).to(x.dtype)
            return y if bias is None else (y + bias.to(y.dtype))
        return _sk.quantized_matmul(x, self.weight, self.scales, self.biases, self.bits, bias)

    def __call__(self, x):  # class attribute the scoped patch swaps
        return self.forward(x)


_orig_call = QuantizedLinear.__call__
_active_ids: frozenset | None = None


def _in_features(mod) -> int:
    return int(mod["weight"].shape[1]) * 32 // int(mod.bits)


def eligible(mod) -> bool:
    """Can this layer's shape/format run on the kernel at all? (small_m_qmm.py:62-64)"""
    return isinstance(mod, QuantizedLinear) and _sk.fits(mod)


def shape_key(mod) -> str:
    return f"{_in_features(mod)}x{int(mod['weight'].shape[0])}b{int(mod.bits)}"


def _mma_call(self, x):  # small_m_qmm.py:71-80
    # an allow-listed layer the kernel cannot read (fp16 / fp32 scales) keeps the stock path
    if (_active_ids is None or id(self) not in _active_ids or x.dtype != torch.bfloat16
            or not _sk.fits(self)):
        return _orig_call(self, x)
    M = 1
    for d in x.shape[:-1]:
        M *= int(d)
    lo, hi = _sk.WINDOW[self.bits]
    if lo <= M <= hi:
        return _sk.call(self, x, M)
    return _orig_call(self, x)


@contextlib.contextmanager
def small_m_matmul(ids: frozenset | None):
    """Route the given :class:`QuantizedLinear` instances (by ``id``) through the kernel for
    forwards inside their width's window. ``None`` / empty is a no-op. Class-level patch that
    restores the value found at entry, so it nests (small_m_qmm.py:83-106)."""
    global _active_ids
    if not ids or QuantizedLinear.__call__ is _mma_call:
        yield
        return
    prev = QuantizedLinear.__call__
    _active_ids = frozenset(ids)
    QuantizedLinear.__call__ = _mma_call
    try:
        yield
    finally:
        QuantizedLinear.__call__ = prev
        _active_ids = None


def active() -> bool:
    return QuantizedLinear.__call__ is _mma_call


def _modules(model):
    if model is None:
        return []
    if isinstance(model, torch.nn.Module):
        return [m for _, m in model.named_modules()]
    return list(model)


def measure_shapes(*models, verbose: bool = False) -> list[str]:
    """Shape keys of eligible layers whose kernel output matches a torch dequantize-and-matmul
    on the same device within ``_REL_TOL`` at the window's edges (the numerics gate of
    small_m_qmm.py:191-207)."""
    groups: dict[str, list] = {}
    for model in models:
        for mod in _modules(model):
            if eligible(mod):
                groups.setdefault(shape_key(mod), []).append(mod)
    won = []
    for key, mods in groups.items():
        mod = mods[0]
        K = _in_features(mod)
        lo, hi = _sk.WINDOW[int(mod.bits)]
        w = quant.dequantize(quant.QWeight(mod.weight, mod.scales, mod.biases, mod.bits))
        ok = True
        for M in sorted({lo, 8, 12, 16, hi}):
            g = torch.Generator(device=mod.weight.device).manual_seed(M)
            x = (torch.randn(M, K, device=mod.weight.device, generator=g) * 0.1).to(torch.bfloat16)
            ref = x.float() @ w.t()
            got = _sk.qmm(x, mod.weight, mod.scales, mod.biases, mod.bits).float()
            diff = (ref - got).abs().max().item()
            if diff > _REL_TOL * max(ref.abs().max().item(), 1.0):
                ok = False
                break
        if verbose:
            print(f"  small-M qmm: {key} {'on' if ok else 'off (numerics)'}", flush=True)
        if ok:
            won.append(key)
    return won


def ids_for_shapes(shapes, *models) -> frozenset:
    """The instance allowlist for :func:`small_m_matmul`, from verified shape keys."""
    keys = set(shapes)
    out = set()
    for model in models:
        for mod in _modules(model):
            if eligible(mod) and shape_key(mod) in keys:
                out.add(id(mod))
    return frozenset(out)
