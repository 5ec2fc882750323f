"""Small-M quantized matmul on B200: the drop-in for ``skinny_qmm`` (K1).

Mirrors src/mlx_dspark/skinny_qmm.py: :func:`qmm` (``:239``), :func:`call` (``:249``),
:func:`plan` / :func:`geometry` (``:214-236``), :func:`fits` (``:174-181``), ``GROUP`` and
``WINDOW``. The arithmetic runs in ``dspark_qmm`` (``csrc/qmm.cu``): weights streamed by TMA
into shared memory, dequantized in registers, tensor-core MMA with the weights as the A
operand, split-K across a thread-block cluster reduced through distributed shared memory.

Differences from the Metal kernel that a caller can see:

* the window is 1-32 rows for both widths (``WINDOW``): on B200 the kernel reads each weight
  once whatever M is, so there is no small-M dead zone to route around;
* results are deterministic and row-count invariant (a row's output does not depend on how
  many rows ride with it), as in the reference;
* there is no CPU path: inputs must be CUDA tensors.
"""

from __future__ import annotations

import ctypes as C

import torch

from . import _lib
from ._torch import ptr, require_cuda, stream_of

GROUP = 64
RT_MAX = 4                          # 8-row tiles per launch (32 rows)
WINDOW = {4: (1, 32), 8: (1, 32)}   # rows served per quantization width


def fits(mod) -> bool:
    """The layout the kernel reads: 4- or 8-bit affine, groups of 64, K % 64 == 0, N % 8 == 0,
    bf16 scales/biases (src/mlx_dspark/skinny_qmm.py:174-181). The reference also accepts fp16
    and fp32 scales; here those layers do not fit (the kernels read bf16 scales and biases, and
    converting them would change the weights), so they stay on the stock path, a torch
    dequantize-and-matmul with MLX's semantics."""
    try:
        w = mod["weight"]
    except (KeyError, TypeError):
        return False
    return (int(getattr(mod, "bits", 0)) in WINDOW and int(getattr(mod, "group_size", 0)) == GROUP
            and getattr(mod, "mode", "affine") == "affine" and "biases" in mod
            and mod["scales"].dtype == torch.bfloat16 and w.ndim == 2
            and (int(w.shape[1]) * 32 // int(mod.bits)) % GROUP == 0 and int(w.shape[0]) % 8 == 0)


def geometry(n: int, k: int, bits: int) -> tuple[int, int]:
    """``(tile_n, split_k)``: output columns per CTA and the split-K factor (cluster size).
    Depends on the weight shape only (never on M)."""
    p = plan(1, n, k, bits)
    return p["tile_n"], p["split_k"]


_plans: dict[tuple[int, int, int], dict] = {}


def plan(rows: int, n: int, k: int, bits: int, dtype=torch.bfloat16) -> dict:
    """Launch geometry for ``rows`` x [n, k] (cached per weight shape)."""
    key = (n, k, bits)
    p = _plans.get(key)
    if p is None:
        out = [C.c_int() for _ in range(4)]
        _lib.check(_lib.lib.dspark_qmm_plan(n, k, bits, *[C.byref(o) for o in out]))
        p = {"tile_n": out[0].value, "split_k": out[1].value, "k_slice": out[2].value,
             "stages": out[3].value}
        _plans[key] = p
    return dict(p, rows=rows, row_tiles=min(RT_MAX, (rows + 7) // 8))


def qmm(x2: torch.Tensor, weight: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor,
        bits: int, _plan=None, out: torch.Tensor | None = None,
        bias: torch.Tensor | None = None) -> torch.Tensor:
    """``x2 [rows, K] @ dequant(W)^T`` for gs64 affine 4/8-bit ``W`` -> bf16 ``[rows, N]``
    (src/mlx_dspark/skinny_qmm.py:239-246). ``weight`` holds the packed uint32 words (as
    int32 or uint32), ``scales`` / ``biases`` are bf16 ``[N, K/64]``."""
    if scales.dtype != torch.bfloat16 or biases.dtype != torch.bfloat16:
        raise _lib.DSparkUnsupported(
            _lib.ERR_UNSUPPORTED, f"scales/biases dtype {scales.dtype}/{biases.dtype} (bf16 only)")
    require_cuda(x2, weight, scales, biases)
    if x2.dtype != torch.bfloat16:
        raise _lib.DSparkUnsupported(_lib.ERR_UNSUPPORTED, f"x dtype {x2.dtype} (bf16 only)")
    rows, k = int(x2.shape[0]), int(x2.shape[1])
    n = int(weight.shape[0])
    if x2.stride(1) != 1:
        x2 = x2.contiguous()
    if out is None:
        out = torch.empty((rows, n), dtype=torch.bfloat16, device=x2.device)
    if bias is not None:
        bias = bias.to(torch.bfloat16).contiguous()
    _lib.check(_lib.lib.dspark_qmm_ex(
        ptr(x2), x2.stride(0), rows, k, ptr(weight), ptr(scales.contiguous()),
        ptr(biases.contiguous()), ptr(bias), n, int(bits), GROUP, ptr(out), out.stride(0),
        stream_of(x2)))
    return out


def quantized_matmul(x: torch.Tensor, weight: torch.Tensor, scales: torch.Tensor,
                     biases: torch.Tensor, bits: int,
                     bias: torch.Tensor | None = None) -> torch.Tensor:
    """``x [..., K] @ dequant(W)^T`` for any number of rows: 32-row launches of the kernel
    (the stock path of :class:`~.small_m_qmm.QuantizedLinear`)."""
    k = x.shape[-1]
    x2 = x.reshape(-1, k)
    rows = int(x2.shape[0])
    n = int(weight.shape[0])
    out = torch.empty((rows, n), dtype=torch.bfloat16, device=x.device)
    lim = WINDOW[int(bits)][1]
    for r0 in range(0, rows, lim):
        r1 = min(rows, r0 + lim)
        qmm(x2[r0:r1], weight, scales, biases, bits, out=out[r0:r1], bias=bias)
    return out.reshape(*x.shape[:-1], n)


def call(mod, x: torch.Tensor, rows: int) -> torch.Tensor:
    """``QuantizedLinear(x)`` through the kernel, launch plan cached on the module
    (src/mlx_dspark/skinny_qmm.py:249-265)."""
    plans = mod.__dict__.get("_dspark_skinny")
    if plans is None:
        plans = {}
        object.__setattr__(mod, "_dspark_skinny", plans)
    k = x.shape[-1]
    p = plans.get(rows)
    if p is None:
        p = plans[rows] = plan(rows, int(mod["weight"].shape[0]), int(k), int(mod.bits))
    bias = mod["bias"] if "bias" in mod else None
    y = qmm(x.reshape(rows, k), mod["weight"], mod["scales"], mod["biases"], int(mod.bits),
            _plan=p, bias=bias)
    return y.reshape(*x.shape[:-1], y.shape[-1])
