"""CPU oracle for the verify path — TEST INFRASTRUCTURE, never the product.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py`` (its ``cpu_baseline`` leg and
its ``--impl reference`` arm) may import this module, and only to check the CUDA path or
to time the CPU baseline. The product path (``mlx-dspark_b200/``) never calls it.

It restates the reference's algorithm for the hot path (file:line in each docstring):

* MLX affine quantization format and quantized matmul arithmetic (``oracle_qmm`` in C),
* multi-row causal / tree verify attention (``oracle_sdpa`` in C),
* ``BatchCache`` per-row-offset semantics, ``build_batch_mask``, greedy accept + rollback,
  ragged packing (numpy / plain Python),
* the Qwen3 dense verify forward (numpy, composing the above).

Pinning: the integer semantics (BatchCache / mask / trim / accept) are checked against the
golden values in the reference's own tests (``tests/golden/reference_goldens.json``, extracted
from the reference test sources by ``tests/golden/extract_reference_goldens.py``). Numeric
parity of QMM and attention against MLX itself is **unpinned** (MLX cannot be imported
here); those two are pinned by analytic known-answer tests (exact dequantization, one-hot
inputs, closed-form attention cases) in ``tests/test_oracle.py``.
"""

from __future__ import annotations

import ctypes as C
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB = HERE / "liboracle.so"
REF_LIB = HERE / "_ref"  # no compiled reference exists: mlx-dspark is pure Python + Metal

STEP = 256  # BatchCache growth step (src/mlx_dspark/batch_engine.py:38)


# ----------------------------------------------------------------------------- C library

def build() -> Path:
    if not LIB.exists() or LIB.stat().st_mtime < (HERE / "oracle.c").stat().st_mtime:
        subprocess.run(["make", "-C", str(HERE), "liboracle.so"], check=True,
                       capture_output=True)
    return LIB


_lib = None


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        build()
        L = C.CDLL(str(LIB))
        vp, i32, i64, f32 = C.c_void_p, C.c_int, C.c_int64, C.c_float
        L.oracle_qmm.argtypes = [vp, i64, i32, i32, vp, vp, vp, i32, i32, vp, i64]
        L.oracle_qmm.restype = None
        L.oracle_sdpa.argtypes = [vp, vp, vp, vp, vp, vp, i32, i32, i32, i32, i32, i32, f32,
                                  i32, vp, i32, vp]
        L.oracle_sdpa.restype = None
        L.oracle_sdpa_t.argtypes = [vp, vp, vp, vp, vp, vp, i32, i32, i32, i32, i32, i32, f32,
                                    i32, vp, i32, i32, vp]
        L.oracle_sdpa_t.restype = None
        L.oracle_threads.restype = i32
        L.oracle_set_threads.argtypes = [i32]
        _lib = L
    return _lib


def threads() -> int:
    return int(lib().oracle_threads())


def set_threads(n: int) -> None:
    lib().oracle_set_threads(int(n))


# ----------------------------------------------------------------------------- bf16

def to_bf16(a) -> np.ndarray:
    """fp32 -> bf16 bit patterns (uint16), round to nearest even (NaN kept quiet)."""
    a = np.ascontiguousarray(np.asarray(a, dtype=np.float32))
    u = a.view(np.uint32)
    # finite values and infinities stay below 2^32 after the rounding bias; NaN patterns may
    # wrap and are replaced below
    rounded = ((u + np.uint32(0x7FFF) + ((u >> np.uint32(16)) & np.uint32(1)))
               >> np.uint32(16)).astype(np.uint16)
    nan = np.isnan(a)
    if nan.any():
        rounded = np.where(nan, np.uint16(0x7FC0), rounded)
    return rounded


def from_bf16(u) -> np.ndarray:
    return (np.asarray(u, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def round_bf16(a) -> np.ndarray:
    return from_bf16(to_bf16(a))


# ----------------------------------------------------------------------------- quantization

def quantize(w, bits: int, group: int = 64):
    """Affine quantization into MLX's packed layout (the build's own quantizer).

    Per group of 64 along K: scale = (max - min) / (2^bits - 1), bias = min,
    q = round((w - bias) / scale) clamped to [0, 2^bits - 1]; scale and bias stored as bf16.
    Packing is LSB-first uint32 (4-bit: word j holds k = 8j..8j+7 at bits 4s; 8-bit: k = 4j..
    4j+3 at bits 8s), the layout skinny_qmm reads (src/mlx_dspark/skinny_qmm.py:97-99,
    :116-125). Returns (wq uint32 [N, K*bits/32], scales u16 [N, K/64], biases u16).
    """
    w = np.asarray(w, dtype=np.float32)
    N, K = w.shape
    assert K % group == 0 and bits in (4, 8)
    g = w.reshape(N, K // group, group)
    lo = g.min(axis=2)
    hi = g.max(axis=2)
    levels = float((1 << bits) - 1)
    scale = np.maximum((hi - lo) / levels, 1e-8).astype(np.float32)
    q = np.rint((g - lo[..., None]) / scale[..., None])
    q = np.clip(q, 0, levels).astype(np.uint32).reshape(N, K)
    return pack(q, bits), to_bf16(scale), to_bf16(lo)


def pack(q, bits: int) -> np.ndarray:
    q = np.asarray(q, dtype=np.uint32)
    N, K = q.shape
    per = 32 // bits
    q = q.reshape(N, K // per, per)
    shifts = (np.arange(per, dtype=np.uint32) * bits)[None, None, :]
    return np.bitwise_or.reduce(q << shifts, axis=2).astype(np.uint32)


def unpack(wq, bits: int) -> np.ndarray:
    wq = np.asarray(wq, dtype=np.uint32)
    per = 32 // bits
    shifts = (np.arange(per, dtype=np.uint32) * bits)[None, None, :]
    q = (wq[..., None] >> shifts) & np.uint32((1 << bits) - 1)
    return q.reshape(wq.shape[0], -1)


def dequantize(wq, scales, biases, bits: int, group: int = 64) -> np.ndarray:
    """w = scale * q + bias in fp32 (src/mlx_dspark/skinny_qmm.py:13-18)."""
    q = unpack(wq, bits).astype(np.float32)
    N, K = q.shape
    s = np.repeat(from_bf16(scales), group, axis=1)
    b = np.repeat(from_bf16(biases), group, axis=1)
    return s * q + b


# ----------------------------------------------------------------------------- C wrappers

def _ptr(a: np.ndarray) -> int:
    return a.ctypes.data


def qmm(x_bits, wq, scales, biases, bits: int) -> np.ndarray:
    """fp32 [M, N] = x . dequant(W)^T (x as bf16 bit patterns [M, K])."""
    x = np.ascontiguousarray(x_bits, dtype=np.uint16)
    wq = np.ascontiguousarray(wq, dtype=np.uint32)
    sc = np.ascontiguousarray(scales, dtype=np.uint16)
    bi = np.ascontiguousarray(biases, dtype=np.uint16)
    M, K = x.shape
    N = wq.shape[0]
    out = np.empty((M, N), dtype=np.float32)
    lib().oracle_qmm(_ptr(x), K, M, K, _ptr(wq), _ptr(sc), _ptr(bi), N, bits, _ptr(out), N)
    return out


def _strides(a: np.ndarray) -> np.ndarray:
    return np.array([s // a.itemsize for s in a.strides[:3]], dtype=np.int64)


def sdpa(q_bits, k_bits, v_bits, scale: float, causal: bool, anc=None,
         round_p: bool = False, f16: bool = False) -> np.ndarray:
    """fp32 [B, Hq, qL, D]. Inputs are bf16 bit patterns [B, H, rows, D] (``f16``: fp16 bit
    patterns; any strides with D contiguous). ``anc`` (uint32 [B, qL] or [qL]) selects the
    tree-verify rule. ``round_p`` rounds the softmax weights to the input type for the P.V sum
    as the reference kernel does (src/mlx_dspark/multirow_attn.py:136-140); otherwise P stays
    fp32."""
    q = np.asarray(q_bits, dtype=np.uint16)
    k = np.asarray(k_bits, dtype=np.uint16)
    v = np.asarray(v_bits, dtype=np.uint16)
    for a in (q, k, v):
        assert a.strides[3] == 2, "head_dim must be contiguous"
    B, Hq, qL, D = q.shape
    Hk, L = k.shape[1], k.shape[2]
    out = np.empty((B, Hq, qL, D), dtype=np.float32)
    qs, ks, vs = _strides(q), _strides(k), _strides(v)
    a = None
    if anc is not None:
        a = np.ascontiguousarray(np.broadcast_to(np.asarray(anc, dtype=np.uint32), (B, qL)))
    lib().oracle_sdpa_t(_ptr(q), _ptr(qs), _ptr(k), _ptr(ks), _ptr(v), _ptr(vs), B, Hq, Hk, qL,
                        L, D, float(scale), int(bool(causal)),
                        _ptr(a) if a is not None else None, int(bool(round_p)), int(bool(f16)),
                        _ptr(out))
    return out


# ----------------------------------------------------------------------------- batch engine

class BatchCacheRef:
    """Restatement of BatchCache (src/mlx_dspark/batch_engine.py:122-224): left-aligned per-row
    KV ``[B, H, Lbuf, D]``; row b's tokens in columns ``0..offsets[b]``; writes scatter at each
    row's offset; trim is per-row metadata clamped at 0; the buffer grows in STEP columns."""

    def __init__(self, keys, values, offsets):
        self.keys = np.array(keys)
        self.values = np.array(values)
        self.offsets = [int(o) for o in offsets]
        self.rows = None

    @classmethod
    def from_rows(cls, kv_pairs):  # :141-157
        lens = [k.shape[2] for k, _ in kv_pairs]
        B, H, Dk = len(kv_pairs), kv_pairs[0][0].shape[1], kv_pairs[0][0].shape[3]
        Dv = kv_pairs[0][1].shape[3]
        lbuf = _round_step(max(lens))
        keys = np.zeros((B, H, lbuf, Dk), dtype=kv_pairs[0][0].dtype)
        values = np.zeros((B, H, lbuf, Dv), dtype=kv_pairs[0][1].dtype)
        for b, (k, v) in enumerate(kv_pairs):
            keys[b, :, : lens[b]] = k[0]
            values[b, :, : lens[b]] = v[0]
        return cls(keys, values, lens)

    @classmethod
    def empty(cls, capacity, n_heads, dk, dv, dtype=np.float32):  # :159-164
        return cls(np.zeros((capacity, n_heads, STEP, dk), dtype),
                   np.zeros((capacity, n_heads, STEP, dv), dtype), [0] * capacity)

    def set_row(self, b, keys, values, offset):  # :167-175
        if offset > self.keys.shape[2]:
            self._grow(_round_step(offset))
        if offset:
            self.keys[b, :, :offset] = keys[0]
            self.values[b, :, :offset] = values[0]
        self.offsets[b] = offset

    def move_row(self, src, dst):  # :177-185
        n = self.offsets[src]
        if n:
            self.keys[dst, :, :n] = self.keys[src, :, :n]
            self.values[dst, :, :n] = self.values[src, :, :n]
        self.offsets[dst] = n
        self.offsets[src] = 0

    @property
    def offset(self):  # :188-191
        return list(self.offsets if self.rows is None else self.offsets[: self.rows])

    def update_and_fetch(self, keys, values):  # :193-208
        B, _, T, _ = keys.shape
        need = max(o + T for o in self.offsets[:B])
        if need > self.keys.shape[2]:
            self._grow(_round_step(need))
        for b in range(B):
            o = self.offsets[b]
            self.keys[b, :, o : o + T] = keys[b]
            self.values[b, :, o : o + T] = values[b]
            self.offsets[b] = o + T
        lcur = max(self.offsets[:B])
        return self.keys[:B, :, :lcur], self.values[:B, :, :lcur]

    def _grow(self, new_lbuf):  # :210-218
        B, H, L, Dk = self.keys.shape
        nk = np.zeros((B, H, new_lbuf, Dk), self.keys.dtype)
        nv = np.zeros((B, H, new_lbuf, self.values.shape[3]), self.values.dtype)
        nk[:, :, :L] = self.keys
        nv[:, :, :L] = self.values
        self.keys, self.values = nk, nv

    def trim(self, ns):  # :220-224
        for b, n in enumerate(ns):
            self.offsets[b] = max(0, self.offsets[b] - int(n))


def _round_step(n: int) -> int:  # :227-228
    return ((n + STEP - 1) // STEP) * STEP


def build_batch_mask(offsets, T: int) -> np.ndarray:
    """bool [B, 1, T, Lcur], mask[b,0,i,j] = j <= offsets[b] + i (batch_engine.py:231-239)."""
    off = np.asarray(offsets, dtype=np.int64)[:, None, None, None]
    lcur = int(max(offsets)) + T
    i = np.arange(T)[None, None, :, None]
    j = np.arange(lcur)[None, None, None, :]
    return j <= off + i


def ctx_block_mask(lens, k: int) -> np.ndarray:
    """bool [B, 1, k, Lmax + k]: context columns < lens[b] or block columns >= Lmax
    (batch_engine.py:508-518)."""
    lmax = max(lens)
    la = np.asarray(lens)[:, None, None, None]
    j = np.arange(lmax + k)[None, None, None, :]
    m = (j >= lmax) | (j < la)
    return np.broadcast_to(m, (len(lens), 1, k, lmax + k))


def accept(drafts, tt):
    """Greedy accept of one block (src/mlx_dspark/generate.py:1548-1555): n = leading run of
    drafts equal to the target argmax; committed = drafts[:n] + [tt[n]]; trim = cap - n."""
    drafts = [int(d) for d in drafts]
    tt = [int(t) for t in tt]
    match = np.array([d == t for d, t in zip(drafts, tt[: len(drafts)])], dtype=np.int64)
    n = int(np.cumprod(match).sum()) if len(match) else 0
    return n, drafts[:n] + [tt[n]], len(drafts) - n


def argmax_first(logits) -> np.ndarray:
    """argmax along the last axis, first index on ties (np / mx.argmax convention)."""
    return np.argmax(np.asarray(logits, dtype=np.float32), axis=-1).astype(np.int32)


def rollback(lens, n_rejected):
    """lens[b] = max(0, lens[b] - n_rejected[b]) (BatchCache.trim, batch_engine.py:220-224)."""
    return [max(0, int(l) - int(n)) for l, n in zip(lens, n_rejected)]


def pack_ragged(block_len, kv_len, slot_off, ids_pad):
    """Device packing of one batched verify step, restated from SpecSlots.step's host loops
    (src/mlx_dspark/batch_engine.py:677-679, :193-208): packed rows in request order, row
    positions kv_len[b] + i, per-request key counts after the append."""
    block_len = [int(t) for t in block_len]
    cu = [0]
    for t in block_len:
        cu.append(cu[-1] + t)
    row_pos, row_kv, row_req, ids = [], [], [], []
    for b, t in enumerate(block_len):
        for i in range(t):
            row_pos.append(int(kv_len[b]) + i)
            row_kv.append(int(slot_off[b]))
            row_req.append(b)
            ids.append(int(ids_pad[b][i]))
    kv_new = [int(kv_len[b]) + block_len[b] for b in range(len(block_len))]
    return dict(cu_rows=cu, row_pos=row_pos, row_kv=row_kv, row_req=row_req, ids=ids,
                kv_len_new=kv_new)


# ----------------------------------------------------------------------------- dense forward

def rmsnorm(x, w, eps: float) -> np.ndarray:
    """mx.fast.rms_norm: x * rsqrt(mean(x^2) + eps) * w in fp32, rounded to bf16."""
    x = np.asarray(x, dtype=np.float32)
    r = 1.0 / np.sqrt(np.mean(x * x, axis=-1, keepdims=True) + eps)
    return round_bf16(x * r * np.asarray(w, dtype=np.float32))


def rope(x, positions, theta: float) -> np.ndarray:
    """Rotate-half RoPE (mlx nn.RoPE traditional=False): pairs (i, i + D/2), frequency
    theta^(-2i/D), angle = position * frequency; fp32 math, bf16 result. x [..., rows, D]."""
    x = np.asarray(x, dtype=np.float32)
    D = x.shape[-1]
    half = D // 2
    inv = theta ** (-np.arange(half, dtype=np.float64) * 2.0 / D)
    ang = np.asarray(positions, dtype=np.float64)[:, None] * inv[None, :]
    c, s = np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)
    x1, x2 = x[..., :half], x[..., half:]
    return round_bf16(np.concatenate([x1 * c - x2 * s, x1 * s + x2 * c], axis=-1))


def silu_mul(g, u) -> np.ndarray:
    g = np.asarray(g, dtype=np.float32)
    return round_bf16(g / (1.0 + np.exp(-g)) * np.asarray(u, dtype=np.float32))


def qlinear(x_f32, w) -> np.ndarray:
    """bf16 output of a quantized linear: w = dict(wq, scales, biases, bits)."""
    return round_bf16(qmm(to_bf16(x_f32), w["wq"], w["scales"], w["biases"], w["bits"]))


def verify_forward(weights: dict, cfg: dict, ids, kcache: list, vcache: list, L0: int,
                   trace: list | None = None, round_p: bool = False):
    """Qwen3 dense verify forward over one block (Target.verify -> _body_mlxlm + head,
    src/mlx_dspark/target.py:642, :208-221; mlx-lm's qwen3 decoder layer):
    h = embed(ids); per layer: r = attn(rmsnorm(h)); h = h + r; r = mlp(rmsnorm(h));
    h = h + r; logits = lm_head(rmsnorm(h)). Attention: q/k RMSNorm per head, RoPE at
    positions L0 + i, K/V appended to the cache at L0, causal verify attention over
    L0 + M keys. Every op output is rounded to bf16 as MLX's bf16 dataflow does.
    ``round_p`` rounds the attention probabilities to bf16 before P.V (the fused Metal
    kernels' dataflow) instead of keeping them in fp32: the two are equally valid bf16
    dataflows, and the spread between them is the noise floor a GPU forward is judged by.

    weights: numpy arrays from the device model (separate q/k/v/gate/up matrices);
    kcache / vcache: per-layer arrays [Hk, cap, D] (modified in place), either float32 values
    or uint16 bf16 bit patterns (read by the attention without a per-layer conversion; the
    timed CPU baseline keeps its cache that way). Returns fp32 logits [M, vocab]."""
    H, Hq, Hk, D = cfg["hidden"], cfg["n_heads"], cfg["n_kv_heads"], cfg["head_dim"]
    eps, theta = cfg["rms_eps"], cfg["rope_theta"]
    M = len(ids)
    emb = weights["embed"]
    rows = np.asarray(ids, dtype=np.int64)
    h = round_bf16(dequantize(emb["wq"][rows], emb["scales"][rows], emb["biases"][rows],
                              emb["bits"]))
    pos = L0 + np.arange(M)
    L = L0 + M
    for li, lw in enumerate(weights["layers"]):
        x = rmsnorm(h, lw["in_norm"], eps)
        q = qlinear(x, lw["q"]).reshape(M, Hq, D)
        k = qlinear(x, lw["k"]).reshape(M, Hk, D)
        v = qlinear(x, lw["v"]).reshape(M, Hk, D)
        q = rope(rmsnorm(q, lw["q_norm"], eps).transpose(1, 0, 2), pos, theta)  # [Hq, M, D]
        k = rope(rmsnorm(k, lw["k_norm"], eps).transpose(1, 0, 2), pos, theta)
        if kcache[li].dtype == np.uint16:  # bf16 bit-pattern cache
            kcache[li][:, L0:L] = to_bf16(k)
            vcache[li][:, L0:L] = to_bf16(v.transpose(1, 0, 2))
            kb, vb = kcache[li][None, :, :L], vcache[li][None, :, :L]
        else:
            kcache[li][:, L0:L] = k
            vcache[li][:, L0:L] = v.transpose(1, 0, 2)
            kb, vb = to_bf16(kcache[li][:, :L])[None], to_bf16(vcache[li][:, :L])[None]
        o = sdpa(to_bf16(q)[None], kb, vb, D ** -0.5, True, round_p=round_p)[0]
        o = round_bf16(o).transpose(1, 0, 2).reshape(M, Hq * D)
        h = round_bf16(h + qlinear(o, lw["o"]))
        if trace is not None:
            trace.append(("attn", o))
            trace.append(("h_mid", h))
        x = rmsnorm(h, lw["post_norm"], eps)
        a = silu_mul(qlinear(x, lw["gate"]), qlinear(x, lw["up"]))
        h = round_bf16(h + qlinear(a, lw["down"]))
        if trace is not None:
            trace.append(("act", a))
            trace.append(("h", h))
    x = rmsnorm(h, weights["final_norm"], eps)
    lm = weights["lm_head"]
    return qmm(to_bf16(x), lm["wq"], lm["scales"], lm["biases"], lm["bits"])


# ----------------------------------------------------------------------------- quantized KV

def quantize_rows(x, bits: int):
    """Quantize rows [..., D] per group of 64 (the build's affine quantizer, as the device
    append kernel does): returns (codes uint32 [..., D*bits/32], scales u16 bf16 [..., D/64],
    biases u16 bf16). Same rule as :func:`quantize` (fp32 scale for the codes, bf16 storage)."""
    x = np.asarray(x, dtype=np.float32)
    lead, D = x.shape[:-1], x.shape[-1]
    wq, sc, bi = quantize(x.reshape(-1, D), bits)
    return (wq.reshape(*lead, D * bits // 32), sc.reshape(*lead, D // 64),
            bi.reshape(*lead, D // 64))


def sdpa_q(q_bits, kq, ks, kb, vq, vs, vb, bits: int, lens, scale: float, causal: bool):
    """Verify attention over a quantized cache (mlx-lm's quantized SDPA for QuantizedKVCache):
    K / V dequantized exactly in fp32 (scale * q + bias), fp32 softmax. q bf16 bit patterns
    [B, Hq, qL, D]; codes [B, Hk, cap, D*bits/32]; row b sees its first lens[b] keys, causal
    rule key <= lens[b] - qL + i. Returns fp32 [B, Hq, qL, D]."""
    q = from_bf16(np.asarray(q_bits, dtype=np.uint16))
    B, Hq, qL, D = q.shape
    Hk = kq.shape[1]
    G = Hq // Hk
    out = np.zeros((B, Hq, qL, D), np.float32)
    for b in range(B):
        L = int(lens[b])
        for hk in range(Hk):
            K = dequantize(kq[b, hk, :L], ks[b, hk, :L], kb[b, hk, :L], bits)
            V = dequantize(vq[b, hk, :L], vs[b, hk, :L], vb[b, hk, :L], bits)
            for g in range(G):
                s = q[b, hk * G + g] @ K.T * np.float32(scale)
                if causal:
                    j = np.arange(L)[None, :]
                    i = np.arange(qL)[:, None]
                    s = np.where(j <= L - qL + i, s, -np.inf)
                s = s - s.max(axis=1, keepdims=True)
                p = np.exp(s)
                out[b, hk * G + g] = (p / p.sum(axis=1, keepdims=True)) @ V
    return out
