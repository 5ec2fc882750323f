"""MLX-layout affine quantization of device tensors (group size 64).

The weight format every kernel here consumes is MLX's affine ``quantize`` output: packed
uint32 ``[N, K*bits/32]`` (LSB-first: 4-bit word j holds k = 8j..8j+7 at bits 4s, 8-bit word
j holds k = 4j..4j+3 at bits 8s — the layout ``skinny_qmm`` reads,
src/mlx_dspark/skinny_qmm.py:97-99, :116-125), bf16 ``scales`` / ``biases`` ``[N, K/64]``,
``w = scale * q + bias``.

:func:`quantize` is the build's own quantizer for random-init weights: per group,
``scale = (max - min) / (2^bits - 1)``, ``bias = min``, ``q = round((w - bias) / scale)``.
(MLX's own edge handling of the group extremes is not reproduced; parity does not depend on
it because the kernels and the checker consume the same packed tensors.) Packed words are
held in ``torch.int32`` tensors carrying the uint32 bit patterns.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

GROUP = 64


@dataclass
class QWeight:
    """A quantized matrix ``[N, K]`` in MLX's packed affine layout."""

    wq: torch.Tensor       # int32 [N, K*bits/32] (uint32 bit patterns)
    scales: torch.Tensor   # bf16 [N, K/64]
    biases: torch.Tensor   # bf16 [N, K/64]
    bits: int

    @property
    def shape(self) -> tuple[int, int]:
        return int(self.wq.shape[0]), int(self.wq.shape[1]) * 32 // self.bits

    @property
    def nbytes(self) -> int:
        return sum(t.numel() * t.element_size() for t in (self.wq, self.scales, self.biases))

    def to(self, device) -> "QWeight":
        return QWeight(self.wq.to(device), self.scales.to(device), self.biases.to(device),
                       self.bits)


def quantize(w: torch.Tensor, bits: int, group_size: int = GROUP) -> QWeight:
    """Quantize a float matrix ``[N, K]`` (any device) into MLX's affine layout."""
    if bits not in (4, 8) or group_size != GROUP:
        raise ValueError(f"only 4/8-bit with group size 64 (got bits={bits}, gs={group_size})")
    w = w.float()
    N, K = w.shape
    if K % group_size:
        raise ValueError(f"K={K} is not a multiple of {group_size}")
    g = w.reshape(N, K // group_size, group_size)
    lo = g.amin(dim=2)
    hi = g.amax(dim=2)
    levels = float((1 << bits) - 1)
    scale = torch.clamp((hi - lo) / levels, min=1e-8)
    q = torch.round((g - lo[..., None]) / scale[..., None]).clamp_(0, levels)
    q = q.to(torch.uint8).reshape(N, K)
    if bits == 4:
        packed = q[:, 0::2] | (q[:, 1::2] << 4)
    else:
        packed = q
    wq = packed.contiguous().view(torch.int32)
    return QWeight(wq, scale.to(torch.bfloat16), lo.to(torch.bfloat16), bits)


def unpack(wq: torch.Tensor, bits: int) -> torch.Tensor:
    per = 32 // bits
    shifts = torch.arange(per, device=wq.device, dtype=torch.int32) * bits
    q = (wq[..., None] >> shifts) & ((1 << bits) - 1)
    return q.reshape(wq.shape[0], -1)


def dequantize(qw: QWeight) -> torch.Tensor:
    """fp32 ``scale * q + bias`` ``[N, K]`` (for tests and weight conversion)."""
    q = unpack(qw.wq, qw.bits).float()
    s = qw.scales.float().repeat_interleave(GROUP, dim=1)
    b = qw.biases.float().repeat_interleave(GROUP, dim=1)
    return s * q + b


def random_qweight(n: int, k: int, bits: int, *, std: float = 0.02, device="cuda",
                   generator: torch.Generator | None = None, chunk_rows: int = 8192) -> QWeight:
    """Quantized ``[n, k]`` matrix of N(0, std^2) weights, generated and quantized in row
    chunks on ``device`` (bounded temporary memory for vocab-sized matrices)."""
    parts = []
    for r0 in range(0, n, chunk_rows):
        r1 = min(n, r0 + chunk_rows)
        w = torch.randn(r1 - r0, k, device=device, generator=generator) * std
        parts.append(quantize(w, bits))
        del w
    if len(parts) == 1:
        return parts[0]
    return QWeight(torch.cat([p.wq for p in parts]), torch.cat([p.scales for p in parts]),
                   torch.cat([p.biases for p in parts]), bits)
