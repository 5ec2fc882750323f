"""Multi-row verify attention on B200: the drop-in for ``multirow_attn`` (K2).

Mirrors src/mlx_dspark/multirow_attn.py: :func:`multirow_sdpa` (``:223``), :func:`plan`
(``:204``), :func:`eligible` (``:288``), :class:`Window` / :class:`MultirowConfig`
(``:262-285``), the scoped patch :func:`multirow_attention` (``:352``) with its
:func:`tree_mask` declaration (``:322``), and :func:`active`.

The reference patches ``mx.fast.scaled_dot_product_attention``; here the patched function is
this module's :func:`scaled_dot_product_attention`, which has MLX's semantics (``mask`` is
``None``, ``"causal"`` — bottom-right aligned: query row i of qL sees keys <= L - qL + i — or a
boolean array broadcast to ``[B, H, qL, L]``; optional ``sinks``). Eligible calls go to
``dspark_verify_attn`` (``csrc/attn.cu``); everything else falls through to the function
installed before, by default a torch implementation on the same device.
"""

from __future__ import annotations

import contextlib
import ctypes as C
import math
from dataclasses import dataclass

import torch

from . import _lib
from ._torch import elem_strides, ptr, require_cuda, stream_of

MAX_D = 256
D_SUPPORTED = (64, 128, 256)
_DTYPES = (torch.bfloat16, torch.float16)
_DT_CODE = {torch.bfloat16: 0, torch.float16: 1}  # DSPARK_DTYPE_BF16 / DSPARK_DTYPE_F16


def plan(hq: int, hk: int, q_len: int, d: int, kv_len: int, batch: int = 1) -> dict:
    """Launch geometry: 16-row tiles per CTA (``NRT``), warps splitting each K/V tile
    (``KS``), row groups (``NRG``), key splits merged inside a cluster (``NS``), cluster groups
    merged through the workspace (``NG``), keys per split (``CHUNK``); ``R`` packed rows."""
    out = (C.c_int * 6)()
    _lib.check(_lib.lib.dspark_verify_attn_plan(batch, hq, hk, q_len, d, kv_len, out))
    rows = (hq // hk) * q_len
    return {"R": rows, "NRT": out[0], "KS": out[1], "NRG": out[2], "NS": out[3], "NG": out[4],
            "CHUNK": out[5], "NB": out[3] * out[4]}


def workspace_bytes(hq, hk, q_len, d, kv_len, batch=1) -> int:
    return int(_lib.lib.dspark_verify_attn_workspace(batch, hq, hk, q_len, d, kv_len))


_ws_cache: dict[tuple, torch.Tensor] = {}


def _workspace(device, nbytes: int) -> torch.Tensor | None:
    if nbytes <= 0:
        return None
    key = (device, )
    t = _ws_cache.get(key)
    if t is None or t.numel() < nbytes:
        t = torch.empty(nbytes, dtype=torch.uint8, device=device)
        _ws_cache[key] = t
    return t


def multirow_sdpa(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *, scale: float,
                  causal: bool, tree_anc: torch.Tensor | None = None,
                  kv_len: torch.Tensor | None = None,
                  out: torch.Tensor | None = None) -> torch.Tensor:
    """``scaled_dot_product_attention(q, k, v, scale, mask="causal" if causal else None)`` for
    few-row shapes. ``q [B, Hq, qL, D]``, ``k`` / ``v`` ``[B, Hk, L, D]`` may be strided cache
    views (head_dim contiguous). ``tree_anc`` (uint32/int32 ``[qL]`` or ``[B, qL]``): tree
    verify visibility bits over the last qL keys instead of the causal rule. ``kv_len``
    (int32 ``[B]`` on the device): per-row key counts <= L (ragged rows)."""
    require_cuda(q, k, v)
    if q.dtype not in _DT_CODE or k.dtype != q.dtype or v.dtype != q.dtype:
        raise _lib.DSparkUnsupported(_lib.ERR_UNSUPPORTED,
                                     f"dtypes {q.dtype}/{k.dtype}/{v.dtype} (bf16 or fp16)")
    B, Hq, qL, D = (int(s) for s in q.shape)
    Hk, L = int(k.shape[1]), int(k.shape[2])
    if q.stride(3) != 1:
        q = q.contiguous()
    if out is None:
        out = torch.empty((B, Hq, qL, D), dtype=q.dtype, device=q.device)
    anc = None
    if tree_anc is not None:
        anc = tree_anc.to(device=q.device, dtype=torch.int32).reshape(-1, qL)
        anc = anc.expand(B, qL).contiguous()
        causal = False
    ws_n = workspace_bytes(Hq, Hk, qL, D, L, B)
    ws = _workspace(q.device, ws_n)
    _lib.check(_lib.lib.dspark_verify_attn_dt(
        _DT_CODE[q.dtype], ptr(q), _lib.i64_array(elem_strides(q)), ptr(k),
        _lib.i64_array(elem_strides(k)),
        ptr(v), _lib.i64_array(elem_strides(v)), B, Hq, Hk, qL, D, L, ptr(kv_len),
        float(scale), int(bool(causal)), ptr(anc), ptr(out), _lib.i64_array(elem_strides(out)),
        ptr(ws), ws_n, stream_of(q)))
    return out


# ---------------------------------------------------------------------- stock semantics

def _torch_sdpa(q, k, v, *, scale, mask=None, sinks=None):
    """MLX-semantics SDPA in torch (fp32 math on q's device): the pass-through for calls the
    kernel does not serve (array masks, sinks, wide q, unmeasured shapes)."""
    B, Hq, qL, D = q.shape
    Hk, L = k.shape[1], k.shape[2]
    rep = Hq // Hk
    kk = k.float().repeat_interleave(rep, dim=1)
    vv = v.float().repeat_interleave(rep, dim=1)
    s = torch.einsum("bhqd,bhkd->bhqk", q.float(), kk) * scale
    if isinstance(mask, str) and mask == "causal":
        i = torch.arange(qL, device=q.device)[:, None]
        j = torch.arange(L, device=q.device)[None, :]
        s = s.masked_fill(j > (L - qL) + i, float("-inf"))
    elif mask is not None:
        m = mask.to(q.device)
        if m.dtype == torch.bool:
            s = s.masked_fill(~m, float("-inf"))
        else:
            s = s + m.float()
    if sinks is not None:
        sk = sinks.float().reshape(1, Hq, 1, 1).expand(B, Hq, qL, 1)
        s = torch.cat([s, sk], dim=-1)
        p = torch.softmax(s, dim=-1)[..., :L]
    else:
        p = torch.softmax(s, dim=-1)
    return torch.einsum("bhqk,bhkd->bhqd", p, vv).to(q.dtype)


def scaled_dot_product_attention(q, k, v, *, scale, mask=None, sinks=None, **kw):
    """The attention entry point callers use (MLX semantics). Replaced by
    :func:`multirow_attention` while active."""
    if kw:
        raise TypeError(f"unexpected arguments {sorted(kw)}")
    return _torch_sdpa(q, k, v, scale=scale, mask=mask, sinks=sinks)


_ORIG_SDPA = scaled_dot_product_attention


@dataclass(frozen=True)
class Window:
    """Gate for one attention shape ``(hq, hk, d)``: served when ``min_q <= q_len <= max_q``
    and ``kv_len >= min_kv`` (multirow_attn.py:262-271)."""
    hq: int
    hk: int
    d: int
    min_q: int = 2
    max_q: int = 16
    min_kv: int = 1024


@dataclass(frozen=True)
class MultirowConfig:
    """One :class:`Window` per attention shape the kernel serves (multirow_attn.py:274-285)."""
    windows: tuple[Window, ...] = ()

    def window(self, hq: int, hk: int, d: int) -> Window | None:
        for w in self.windows:
            if w.hq == hq and w.hk == hk and w.d == d:
                return w
        return None


def eligible(q, k, v, mask, sinks, cfg: MultirowConfig) -> bool:
    """Structural + gate check (multirow_attn.py:288-312): unmasked or ``"causal"``, no sinks,
    4-D bf16 tensors of a configured shape, matching head dims in ``D_SUPPORTED``, whole GQA
    groups, q_len / KV length inside the window, head_dim contiguous."""
    if sinks is not None or q.ndim != 4 or k.ndim != 4 or v.ndim != 4:
        return False
    if not (mask is None or (isinstance(mask, str) and mask == "causal")):
        return False
    B, Hq, qL, D = q.shape
    Hk, L = k.shape[1], k.shape[2]
    w = cfg.window(Hq, Hk, D)
    if w is None or not (w.min_q <= qL <= w.max_q and qL <= L) or max(w.min_kv, 16) > L:
        return False
    if q.dtype not in _DTYPES or k.dtype != q.dtype or v.dtype != q.dtype:
        return False
    if k.shape[-1] != D or v.shape[-1] != D or D not in D_SUPPORTED or v.shape[2] != L:
        return False
    if k.stride(3) != 1 or v.stride(3) != 1:
        return False
    return not (Hk == 0 or Hq % Hk or v.shape[1] != Hk or k.shape[0] != B or v.shape[0] != B)


_ACTIVE: MultirowConfig | None = None
_PREV = None
_TREE: tuple | None = None


@contextlib.contextmanager
def tree_mask(mask: torch.Tensor, anc_bits: torch.Tensor):
    """Declare ``mask`` as a tree-verify mask whose last-W-key visibility is ``anc_bits`` (one
    uint32 per row) so calls carrying that exact tensor take the kernel's tree variant
    (multirow_attn.py:322-335). Identity-matched."""
    global _TREE
    prev = _TREE
    _TREE = (mask, anc_bits)
    try:
        yield
    finally:
        _TREE = prev


def _patched_call(q, k, v, *, scale, mask=None, sinks=None, **kw):  # multirow_attn.py:338-349
    cfg = _ACTIVE
    if cfg is not None and not kw:
        tree = _TREE
        if (tree is not None and mask is tree[0] and q.ndim == 4 and q.shape[2] <= 32
                and eligible(q, k, v, None, sinks, cfg)):
            return multirow_sdpa(q, k, v, scale=scale, causal=False, tree_anc=tree[1])
        if eligible(q, k, v, mask, sinks, cfg):
            return multirow_sdpa(q, k, v, scale=scale,
                                 causal=isinstance(mask, str) and q.shape[2] > 1)
    prev = _PREV or _ORIG_SDPA
    return prev(q, k, v, scale=scale, mask=mask, sinks=sinks, **kw)


@contextlib.contextmanager
def multirow_attention(cfg: MultirowConfig | None):
    """Route eligible :func:`scaled_dot_product_attention` calls through the kernel while
    active; everything else falls through to what was installed before. No-op for ``None`` or
    when already installed (multirow_attn.py:352-370)."""
    global _ACTIVE, _PREV, scaled_dot_product_attention
    if cfg is None or scaled_dot_product_attention is _patched_call:
        yield
        return
    prev = scaled_dot_product_attention
    prev_cfg, prev_prev = _ACTIVE, _PREV
    _ACTIVE, _PREV = cfg, prev
    scaled_dot_product_attention = _patched_call
    try:
        yield
    finally:
        scaled_dot_product_attention = prev
        _ACTIVE, _PREV = prev_cfg, prev_prev


def active() -> bool:
    return scaled_dot_product_attention is _patched_call


def sdpa(q, k, v, *, scale, mask=None, sinks=None, **kw):
    """Call whatever :func:`scaled_dot_product_attention` is installed right now."""
    return scaled_dot_product_attention(q, k, v, scale=scale, mask=mask, sinks=sinks, **kw)


def default_window(hq: int, hk: int, d: int) -> Window:
    """The B200 kernel wins from 1 row and short KV, so the default window is wide."""
    return Window(hq, hk, d, min_q=1, max_q=32, min_kv=16)


def tree_bits(parent: list[int]) -> list[int]:
    """Ancestor-or-self bitmasks of a draft tree given parent indices (-1 = root)."""
    bits = []
    for i, p in enumerate(parent):
        b = 1 << i
        while p >= 0:
            b |= 1 << p
            p = parent[p]
        bits.append(b)
    return bits


def _isqrt_scale(d: int) -> float:
    return 1.0 / math.sqrt(d)
