"""Per-row KV cache on the device with in-place rollback (K3).

:class:`BatchCache` mirrors src/mlx_dspark/batch_engine.py:122-224: keys / values
``[B, H, Lbuf, D]``, row b's tokens left-aligned in columns ``0..offsets[b]``, writes at each
row's own offset, ``trim`` as pure per-row metadata clamped at 0 (the next write overwrites
the tail), buffer growth in ``STEP`` columns, slot reuse (``empty`` / ``set_row``) and
retirement compaction (``move_row``), and the active-prefix view ``rows``.

The row writes, trims and row moves run in ``libdspark.so`` (``dspark_kv_append``,
``dspark_kv_rollback``, ``dspark_kv_move_row``); the per-row lengths live on the device in
``lens`` (int32) and a host mirror ``offsets`` is kept for the reference's list-based
interface. Device-side updates (the fused accept + rollback kernel) can be folded back into
the mirror with :meth:`sync_offsets`.
"""

from __future__ import annotations

import ctypes as C

import torch

from . import _lib
from ._torch import elem_strides, ptr, require_cuda, stream_of

STEP = 256


def _round_step(n: int) -> int:
    return ((n + STEP - 1) // STEP) * STEP


class BatchCache:
    """Left-aligned per-row-offset KV cache for one layer (see module docstring)."""

    def __init__(self, keys: torch.Tensor, values: torch.Tensor, offsets):
        require_cuda(keys, values)
        self.keys = keys
        self.values = values
        self.offsets = [int(o) for o in offsets]
        self.lens = torch.tensor(self.offsets, dtype=torch.int32, device=keys.device)
        self.rows: int | None = None

    # -- construction --
    @classmethod
    def from_rows(cls, kv_pairs) -> "BatchCache":
        """Merge per-row ``[1, H, len_b, D]`` (keys, values) into one left-aligned buffer."""
        lens = [int(k.shape[2]) for k, _ in kv_pairs]
        B = len(kv_pairs)
        k0, v0 = kv_pairs[0]
        lbuf = _round_step(max(lens))
        keys = torch.zeros((B, k0.shape[1], lbuf, k0.shape[3]), dtype=k0.dtype, device=k0.device)
        values = torch.zeros((B, v0.shape[1], lbuf, v0.shape[3]), dtype=v0.dtype,
                             device=v0.device)
        for b, (k, v) in enumerate(kv_pairs):
            keys[b : b + 1, :, : lens[b]] = k
            values[b : b + 1, :, : lens[b]] = v
        return cls(keys, values, lens)

    @classmethod
    def empty(cls, capacity: int, n_heads: int, dk: int, dv: int, dtype,
              device="cuda", length: int = STEP) -> "BatchCache":
        """Fixed-capacity cache with every row empty (the slot-reuse form)."""
        lbuf = _round_step(max(1, length))
        return cls(torch.zeros((capacity, n_heads, lbuf, dk), dtype=dtype, device=device),
                   torch.zeros((capacity, n_heads, lbuf, dv), dtype=dtype, device=device),
                   [0] * capacity)

    # -- slot reuse --
    def set_row(self, b: int, keys: torch.Tensor, values: torch.Tensor, offset: int) -> None:
        if offset > self.keys.shape[2]:
            self._grow(_round_step(offset))
        if offset:
            self.keys[b : b + 1, :, :offset] = keys
            self.values[b : b + 1, :, :offset] = values
        self.offsets[b] = int(offset)
        self.lens[b] = int(offset)

    def move_row(self, src: int, dst: int) -> None:
        """Copy row src's live columns onto row dst and vacate src (on the device)."""
        if src == dst:
            return
        n = self.offsets[src]
        _lib.check(_lib.lib.dspark_kv_move_row(
            ptr(self.keys), _lib.i64_array(elem_strides(self.keys)), ptr(self.values),
            _lib.i64_array(elem_strides(self.values)), ptr(self.lens), src, dst,
            int(self.keys.shape[1]), int(self.keys.shape[3]), self.keys.element_size(),
            max(n, 1), stream_of(self.keys)))
        self.offsets[dst] = n
        self.offsets[src] = 0

    # -- interface the attention layers use --
    @property
    def offset(self) -> torch.Tensor:
        n = len(self.offsets) if self.rows is None else self.rows
        return self.lens[:n]

    def update_and_fetch(self, keys: torch.Tensor, values: torch.Tensor):
        """Write each row's ``T`` new tokens at its own offset (one kernel), advance the
        offsets, and return ``[B, H, Lcur, D]`` views with ``Lcur = max(new offsets)``."""
        B, H, T, D = (int(s) for s in keys.shape)
        need = max(o + T for o in self.offsets[:B])
        if need > self.keys.shape[2]:
            self._grow(_round_step(need))
        if keys.stride(3) != 1:
            keys = keys.contiguous()
        if values.stride(3) != 1:
            values = values.contiguous()
        _lib.check(_lib.lib.dspark_kv_append(
            ptr(keys), _lib.i64_array(elem_strides(keys)), ptr(values),
            _lib.i64_array(elem_strides(values)), ptr(self.keys),
            _lib.i64_array(elem_strides(self.keys)), ptr(self.values),
            _lib.i64_array(elem_strides(self.values)), ptr(self.lens), B, H, T, D,
            self.keys.element_size(), int(self.keys.shape[2]), stream_of(keys)))
        for b in range(B):
            self.offsets[b] += T
        lcur = max(self.offsets[:B])
        return self.keys[:B, :, :lcur], self.values[:B, :, :lcur]

    def _grow(self, new_lbuf: int) -> None:
        B, H, L, Dk = self.keys.shape
        nk = torch.zeros((B, H, new_lbuf, Dk), dtype=self.keys.dtype, device=self.keys.device)
        nv = torch.zeros((B, H, new_lbuf, self.values.shape[3]), dtype=self.values.dtype,
                         device=self.values.device)
        nk[:, :, :L] = self.keys
        nv[:, :, :L] = self.values
        self.keys, self.values = nk, nv

    def trim(self, ns) -> None:
        """Roll each row back by ``ns[b]`` tokens — metadata only, on the device."""
        ns = [int(n) for n in ns]
        if not ns:
            return
        n_dev = torch.tensor(ns, dtype=torch.int32, device=self.lens.device)
        _lib.check(_lib.lib.dspark_kv_rollback(ptr(self.lens), ptr(n_dev), len(ns),
                                               stream_of(self.lens)))
        for b, n in enumerate(ns):
            self.offsets[b] = max(0, self.offsets[b] - n)

    def sync_offsets(self) -> list[int]:
        """Refresh the host mirror from the device lengths (after device-side rollback)."""
        self.offsets = [int(x) for x in self.lens.tolist()]
        return self.offsets


def rollback(lens: torch.Tensor, n_rejected: torch.Tensor) -> None:
    """``lens[b] = max(0, lens[b] - n_rejected[b])`` in place on the device
    (Target.rollback / KVCache.trim, src/mlx_dspark/target.py:679-698)."""
    require_cuda(lens, n_rejected)
    _lib.check(_lib.lib.dspark_kv_rollback(ptr(lens), ptr(n_rejected), int(lens.numel()),
                                           stream_of(lens)))


class QuantizedKVCache:
    """A quantized per-row KV cache for one layer (the reference's ``kv_bits`` path,
    src/mlx_dspark/target.py:166-185: mlx-lm's ``QuantizedKVCache(group_size=64, bits)``).

    Keys and values are stored MLX-affine quantized per group of 64 along head_dim: code words
    ``uint32 [B, H, cap, D*bits/32]`` and bf16 scales / biases ``[B, H, cap, D/64]``. ``lens``
    (device int32 ``[B]``) is each row's cached length; :meth:`update` quantizes a block of new
    rows at those lengths (``dspark_kv_append_q``), :meth:`trim` is the same metadata-only
    rollback as the bf16 cache, and :meth:`attention` runs the verify attention over the
    quantized rows (``dspark_verify_attn_q``)."""

    def __init__(self, B: int, H: int, cap: int, D: int, bits: int = 8, device="cuda"):
        if bits not in (4, 8) or D not in (64, 128):
            raise _lib.DSparkUnsupported(_lib.ERR_UNSUPPORTED, f"{bits}-bit KV, head_dim {D}")
        self.B, self.H, self.cap, self.D, self.bits = int(B), int(H), int(cap), int(D), int(bits)
        w = D * bits // 32
        dev = torch.device(device)
        u32 = dict(dtype=torch.int32, device=dev)
        bf = dict(dtype=torch.bfloat16, device=dev)
        self.kq = torch.zeros((B, H, cap, w), **u32)
        self.vq = torch.zeros((B, H, cap, w), **u32)
        self.ks = torch.zeros((B, H, cap, D // 64), **bf)
        self.kb = torch.zeros((B, H, cap, D // 64), **bf)
        self.vs = torch.zeros((B, H, cap, D // 64), **bf)
        self.vb = torch.zeros((B, H, cap, D // 64), **bf)
        self.lens = torch.zeros(B, dtype=torch.int32, device=dev)
        require_cuda(self.kq)
        self._c = _lib.QKV(ptr(self.kq), ptr(self.ks), ptr(self.kb), ptr(self.vq), ptr(self.vs),
                           ptr(self.vb), (C.c_int64 * 3)(*elem_strides(self.kq)),
                           (C.c_int64 * 3)(*elem_strides(self.ks)), self.bits)

    @property
    def offset(self) -> list[int]:
        return [int(x) for x in self.lens.tolist()]

    def update(self, k_new: torch.Tensor, v_new: torch.Tensor) -> None:
        """Quantize ``[B, H, T, D]`` bf16 rows into each row's next T positions."""
        require_cuda(k_new, v_new)
        B, H, T, D = (int(s) for s in k_new.shape)
        _lib.check(_lib.lib.dspark_kv_append_q(
            ptr(k_new), _lib.i64_array(elem_strides(k_new)), ptr(v_new),
            _lib.i64_array(elem_strides(v_new)), C.byref(self._c), ptr(self.lens), B, H, T, D,
            self.cap, stream_of(k_new)))

    def trim(self, n_rejected: torch.Tensor) -> None:
        """``lens -= n_rejected`` clamped at 0 on the device (metadata only)."""
        _lib.check(_lib.lib.dspark_kv_rollback(ptr(self.lens), ptr(n_rejected), self.B,
                                               stream_of(self.lens)))

    def attention(self, q: torch.Tensor, *, scale: float, causal: bool = True,
                  out: torch.Tensor | None = None) -> torch.Tensor:
        """Verify attention of ``q [B, Hq, qL, D]`` (bf16) over each row's ``lens[b]`` cached
        keys (the quantized_scaled_dot_product_attention route of mlx-lm for this cache)."""
        from .multirow_attn import _workspace, workspace_bytes

        require_cuda(q)
        B, Hq, qL, D = (int(s) for s in q.shape)
        if out is None:
            out = torch.empty_like(q)
        L = self.cap
        ws_n = workspace_bytes(Hq, self.H, qL, D, L, B)
        ws = _workspace(q.device, ws_n)
        _lib.check(_lib.lib.dspark_verify_attn_q(
            ptr(q), _lib.i64_array(elem_strides(q)), C.byref(self._c), B, Hq, self.H, qL, D, L,
            ptr(self.lens), float(scale), int(bool(causal)), ptr(out),
            _lib.i64_array(elem_strides(out)), ptr(ws), ws_n, stream_of(q)))
        return out
