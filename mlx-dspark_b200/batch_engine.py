"""Continuous-batching verify step with ragged packing built on the device (K4).

Mirrors the batched spec round of src/mlx_dspark/batch_engine.py: ``SpecSlots.step``
(``:635-708``) packs each active request's ``[pending] + drafts`` block, runs one verify
forward over all rows, accepts per row with the row-wise cumprod of the argmax match
(``:684-686``) and trims each request's cache by ``cap - n`` (``:692-705``); slots are
admitted / retired without resizing the batch (``:541-633``).

The reference builds the step on the host (Python loops over rows, a padded
``[B, H, Lmax, D]`` cache and a dense boolean mask from :func:`build_batch_mask`). Here one
kernel packs the step (row positions, per-request key counts and cache-slot offsets, packed
token ids) from device-resident per-slot state; the attention reads each request's own slot
with its own length (no padding, no mask), and a second kernel fuses argmax-accept with the
per-request rollback. Requests never need compaction copies: a retired slot is simply not
packed.

:func:`build_batch_mask` is kept (on the device) for checking the packing against the
reference's dense formulation.
"""

from __future__ import annotations

import torch

from . import _lib
from .kvcache import STEP  # noqa: F401  (re-exported like the reference module)
from ._torch import ptr, require_cuda, stream_of


def build_batch_mask(offsets, T: int, device="cuda") -> torch.Tensor:
    """bool ``[B, 1, T, Lcur]`` with ``mask[b, 0, i, j] = j <= offsets[b] + i`` and
    ``Lcur = max(offsets) + T`` (src/mlx_dspark/batch_engine.py:231-239)."""
    off = torch.as_tensor(list(offsets), dtype=torch.int32, device=device)
    require_cuda(off)
    B = int(off.numel())
    lcur = int(max(offsets)) + int(T)
    mask = torch.empty((B, 1, int(T), lcur), dtype=torch.uint8, device=off.device)
    _lib.check(_lib.lib.dspark_batch_mask(ptr(off), B, int(T), lcur, ptr(mask), stream_of(off)))
    return mask.bool()


def pack_ragged(block_len: torch.Tensor, kv_len: torch.Tensor, slot_off: torch.Tensor,
                ids_pad: torch.Tensor, r_max: int, out: dict | None = None) -> dict:
    """Pack one batched verify step on the device (see ``dspark_pack_ragged``)."""
    require_cuda(block_len, kv_len, slot_off, ids_pad)
    B = int(block_len.numel())
    dev = block_len.device
    if out is None:
        out = {"cu_rows": torch.empty(B + 1, dtype=torch.int32, device=dev),
               "row_pos": torch.empty(r_max, dtype=torch.int32, device=dev),
               "row_kv": torch.empty(r_max, dtype=torch.int64, device=dev),
               "row_req": torch.empty(r_max, dtype=torch.int32, device=dev),
               "ids": torch.empty(r_max, dtype=torch.int32, device=dev),
               "kv_len_new": torch.empty(B, dtype=torch.int32, device=dev)}
    _lib.check(_lib.lib.dspark_pack_ragged(
        ptr(block_len), ptr(kv_len), ptr(slot_off), ptr(ids_pad), int(ids_pad.shape[1]), B,
        int(r_max), ptr(out["cu_rows"]), ptr(out["row_pos"]), ptr(out["row_kv"]),
        ptr(out["row_req"]), ptr(out["ids"]), ptr(out["kv_len_new"]), stream_of(block_len)))
    return out


def accept(logits: torch.Tensor, ids: torch.Tensor, cu_rows: torch.Tensor,
           lens: torch.Tensor | None = None) -> dict:
    """Greedy accept of every request's block: ``tt = argmax(logits)`` per row (first index on
    ties), ``n[b]`` = leading drafts of request b equal to ``tt``, ``next[b] = tt[cu[b] + n]``;
    if ``lens`` (tokens cached after the verify's append) is given it is trimmed in place by
    ``cap_b - n_b``. Returns the device tensors ``tt``, ``n``, ``next``, ``lens``."""
    require_cuda(logits, ids, cu_rows)
    R = int(ids.numel())
    B = int(cu_rows.numel()) - 1
    dev = ids.device
    tt = torch.empty(R, dtype=torch.int32, device=dev)
    n = torch.empty(B, dtype=torch.int32, device=dev)
    nxt = torch.empty(B, dtype=torch.int32, device=dev)
    s = stream_of(ids)
    _lib.check(_lib.lib.dspark_argmax(ptr(logits), logits.stride(0), R, int(logits.shape[1]),
                                      ptr(tt), s))
    _lib.check(_lib.lib.dspark_accept(ptr(tt), ptr(ids), ptr(cu_rows), B, ptr(n), ptr(nxt),
                                      ptr(lens), s))
    return {"tt": tt, "n": n, "next": nxt, "lens": lens}
