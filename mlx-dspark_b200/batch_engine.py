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


class SpecBatch:
    """Continuous-batching verify rounds over a :class:`~.target.Target`'s request slots
    (the device-side counterpart of ``SpecSlots``, src/mlx_dspark/batch_engine.py:541-708).

    A request is :meth:`admit`-ted into a free slot with its cached prefix length (and,
    optionally, its K/V prefix); :meth:`step` runs one spec round for every active slot: the
    slots' ``[pending] + drafts`` blocks are packed on the device (``dspark_pack_ragged``), one
    verify forward covers all packed rows (projections in 32-row launches, attention over each
    slot's own keys), and the greedy accept trims every slot's cache by its rejected tail in
    the same kernel. Slots never move: a retired slot simply contributes no rows (the
    reference compacts rows with ``move_row`` instead, ``:609-623``).

    Draft tokens come from the caller (the drafters are outside this path); ``forced_accept``
    replaces the greedy accept count per slot (seeded accept lengths for benchmarking
    random-init weights, whose drafts never match)."""

    def __init__(self, target, max_block: int = 17):
        import ctypes as C

        t = target
        self.t = t
        self.B = t.slots
        self.max_block = int(max_block)
        dev = t.device
        i32 = dict(dtype=torch.int32, device=dev)
        self.lens = torch.zeros(self.B, **i32)           # tokens cached per slot
        self.pending = torch.zeros(self.B, **i32)        # next token to verify per slot
        self.active = [False] * self.B
        self.meta = [None] * self.B
        self.slot_off = torch.tensor([t.slot_offset(b) for b in range(self.B)], dtype=torch.int64,
                                     device=dev)
        R = t.max_rows
        self.buf = {
            "block_len": torch.zeros(self.B, **i32),
            "ids_pad": torch.zeros((self.B, self.max_block), **i32),
            "cu_rows": torch.zeros(self.B + 1, **i32),
            "row_pos": torch.zeros(R, **i32),
            "row_kv": torch.zeros(R, dtype=torch.int64, device=dev),
            "row_req": torch.zeros(R, **i32),
            "ids": torch.zeros(R, **i32),
            "kv_len_new": torch.zeros(self.B, **i32),
            "tt": torch.zeros(R, **i32),
            "n": torch.zeros(self.B, **i32),
            "next": torch.zeros(self.B, **i32),
            "n_rej": torch.zeros(self.B, **i32),
        }
        b, fb = self.buf, t.buf
        # the forward reads the packing straight from this engine's arrays
        self._fwd = _lib.FwdBuffers(
            ptr(fb["h"]), ptr(fb["xq"]), ptr(fb["attn"]), ptr(fb["act"]), ptr(fb["ssq_a"]),
            ptr(fb["ssq_b"]), ptr(fb["inv_freq"]), ptr(b["row_pos"]), ptr(b["row_kv"]),
            ptr(b["kv_len_new"]), ptr(b["cu_rows"]), ptr(b["block_len"]), ptr(self.slot_off),
            ptr(fb["attn_ws"]), fb["attn_ws"].numel(), t.rows_cap,
            ptr(fb["wide_ws"]) if t.wide_ws_bytes else None, t.wide_ws_bytes)
        self._C = C

    @property
    def has_free_slot(self) -> bool:
        return not all(self.active)

    @property
    def n_active(self) -> int:
        return sum(self.active)

    def admit(self, length: int, pending: int, *, kv=None, meta=None) -> int:
        """Claim a free slot for a request whose first ``length`` tokens are cached and whose
        next token to verify is ``pending``; ``kv`` (optional) is a list over layers of
        ``(k, v)`` bf16 ``[Hk, length, D]`` prefixes copied into the slot. Returns the slot."""
        slot = self.active.index(False)
        if length + self.max_block > self.t.slot_caps[slot]:
            raise ValueError(f"slot {slot} holds {self.t.slot_caps[slot]} positions")
        if kv is not None:
            for li, (k, v) in enumerate(kv):
                self.t.slot_view(li, slot, "k")[:, :length].copy_(k)
                self.t.slot_view(li, slot, "v")[:, :length].copy_(v)
        self.lens[slot] = int(length)
        self.pending[slot] = int(pending)
        self.active[slot] = True
        self.meta[slot] = meta
        return slot

    def retire(self, slot: int):
        """Free a slot (its cache length returns to 0); returns the caller's handle."""
        meta = self.meta[slot]
        self.active[slot] = False
        self.meta[slot] = None
        self.lens[slot] = 0
        return meta

    def step(self, drafts: torch.Tensor, block_len: list[int],
             forced_accept: torch.Tensor | None = None) -> dict:
        """One spec round. ``drafts`` int32 ``[B, max_block - 1]`` (row b: slot b's drafts),
        ``block_len[b]`` = 1 + drafts used by slot b (0 for idle slots). Returns the device
        tensors ``n`` (accepted drafts), ``next`` (bonus token), ``tt`` (argmax per packed
        row) and ``cu_rows``; ``lens`` and ``pending`` are updated on the device."""
        t, b = self.t, self.buf
        dev = t.device
        bl = [int(x) if self.active[i] else 0 for i, x in enumerate(block_len)]
        R = sum(bl)
        if R == 0:
            return {"n": b["n"], "next": b["next"], "tt": b["tt"], "cu_rows": b["cu_rows"]}
        if R > t.max_rows:
            raise _lib.DSparkUnsupported(_lib.ERR_UNSUPPORTED, f"{R} rows > {t.max_rows}")
        s = stream_of(self.lens)
        b["block_len"].copy_(torch.tensor(bl, dtype=torch.int32), non_blocking=True)
        b["ids_pad"][:, 0].copy_(self.pending)
        b["ids_pad"][:, 1 : 1 + drafts.shape[1]].copy_(drafts)
        _lib.check(_lib.lib.dspark_pack_ragged(
            ptr(b["block_len"]), ptr(self.lens), ptr(self.slot_off), ptr(b["ids_pad"]),
            self.max_block, self.B, t.max_rows, ptr(b["cu_rows"]), ptr(b["row_pos"]),
            ptr(b["row_kv"]), ptr(b["row_req"]), ptr(b["ids"]), ptr(b["kv_len_new"]), s))
        qL = max(bl)
        L_max = t.kv_cap
        C = self._C
        _lib.check(_lib.lib.dspark_verify_forward(
            C.byref(t._model_c), C.byref(self._fwd), ptr(b["ids"]), R, self.B, qL, L_max,
            ptr(t.logits), t.logits.stride(0), s))
        _lib.check(_lib.lib.dspark_argmax(ptr(t.logits), t.logits.stride(0), R, t.cfg.vocab,
                                          ptr(b["tt"]), s))
        if forced_accept is None:
            _lib.check(_lib.lib.dspark_accept(ptr(b["tt"]), ptr(b["ids"]), ptr(b["cu_rows"]),
                                              self.B, ptr(b["n"]), ptr(b["next"]),
                                              ptr(b["kv_len_new"]), s))
        else:
            blt = torch.tensor(bl, dtype=torch.int32, device=dev)
            n = torch.minimum(forced_accept.to(torch.int32), (blt - 1).clamp(min=0))
            b["n"].copy_(torch.where(blt > 0, n, torch.zeros_like(n)))
            # the bonus token after the forced accept: argmax of the block's row n
            row = (b["cu_rows"][:-1].long() + b["n"].long()).clamp(max=R - 1)
            nxt = b["tt"].gather(0, row)
            b["next"].copy_(torch.where(blt > 0, nxt, torch.full_like(nxt, -1)))
            b["n_rej"].copy_(torch.where(blt > 0, blt - 1 - b["n"], torch.zeros_like(n)))
            _lib.check(_lib.lib.dspark_kv_rollback(ptr(b["kv_len_new"]), ptr(b["n_rej"]),
                                                   self.B, s))
        self.lens.copy_(b["kv_len_new"])
        act = torch.tensor([int(x > 0) for x in bl], dtype=torch.bool, device=dev)
        self.pending.copy_(torch.where(act, b["next"], self.pending))
        return {"n": b["n"], "next": b["next"], "tt": b["tt"], "cu_rows": b["cu_rows"]}


def partition_requests(lengths: list[int], world: int) -> list[list[int]]:
    """Data-parallel request placement: requests (by index) spread over ``world`` ranks so the
    ranks' summed KV lengths stay balanced (longest first onto the least-loaded rank). No
    collective is involved; each rank serves its own list."""
    order = sorted(range(len(lengths)), key=lambda i: -lengths[i])
    load = [0] * world
    out: list[list[int]] = [[] for _ in range(world)]
    for i in order:
        r = min(range(world), key=lambda k: (load[k], k))
        out[r].append(i)
        load[r] += lengths[i]
    return out
