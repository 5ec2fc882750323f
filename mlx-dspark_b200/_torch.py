"""Torch buffer plumbing for the C ABI: pointers, streams, checks."""

from __future__ import annotations

import torch

from . import _lib


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def stream_of(t: torch.Tensor) -> int:
    """The current torch stream handle on ``t``'s device (launches are stream-ordered)."""
    return torch.cuda.current_stream(t.device).cuda_stream


def require_cuda(*ts: torch.Tensor) -> torch.device:
    dev = None
    for t in ts:
        if t is None:
            continue
        if not t.is_cuda:
            raise _lib.DSparkUnsupported(
                _lib.ERR_UNSUPPORTED, f"tensor on {t.device}: dspark kernels run on CUDA only "
                "(there is no CPU path)")
        dev = t.device if dev is None else dev
        if t.device != dev:
            raise _lib.DSparkError(_lib.ERR_ARG, "tensors on different devices")
    assert dev is not None
    _lib.ensure_init(dev.index if dev.index is not None else torch.cuda.current_device())
    return dev


def elem_strides(t: torch.Tensor, n: int = 3) -> list[int]:
    return [int(s) for s in t.stride()[:n]]
