"""Dense Qwen3-shaped verify target on B200 (the caller of K1/K2/K3).

Mirrors the dense branch of src/mlx_dspark/target.py: :meth:`Target.verify` (``:642``: one
forward of ``[anchor] + drafts`` rows returning logits), :meth:`Target.rollback` (``:679-698``:
trim the rejected tail of every layer's cache) and :meth:`Target.make_cache`; the forward is
``_body_mlxlm`` + head (``:208-221``) over mlx-lm's qwen3 decoder.

The whole forward is one C call, ``dspark_verify_forward``, chaining per layer: fused QKV
QMM (input RMSNorm applied while staging x; q/k RMSNorm, RoPE and the KV-cache write in the
epilogue) -> verify attention -> O QMM + residual -> gate/up QMM (post-attention RMSNorm in
the prologue, SwiGLU in the epilogue) -> down QMM + residual; then final norm + lm_head.
Weights are random-init (N(0, 0.02)) and quantized to MLX's affine layout; q/k/v and
gate/up are stored fused (q|k|v rows; gate/up interleaved in blocks of 32 rows) — a load-time
re-layout of the separate MLX matrices that :meth:`Target.oracle_weights` undoes for the
checker.
"""

from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, replace

import torch

from . import _lib, quant
from ._torch import ptr, require_cuda, stream_of


@dataclass(frozen=True)
class Qwen3Config:
    n_layers: int
    hidden: int
    n_heads: int
    n_kv_heads: int
    head_dim: int
    intermediate: int
    vocab: int
    rms_eps: float = 1e-6
    rope_theta: float = 1e6
    bits: int = 4

    @property
    def weight_params(self) -> int:
        H, D = self.hidden, self.head_dim
        per = (H * (self.n_heads + 2 * self.n_kv_heads) * D + self.n_heads * D * H
               + 3 * H * self.intermediate)
        return self.n_layers * per + self.vocab * H

    def weight_bytes(self) -> int:
        """Packed weights + bf16 scales/biases read by one verify forward (embedding rows are
        a gather of R rows and are not counted)."""
        per_param = self.bits / 8 + 4 / 64
        return int(self.weight_params * per_param)


QWEN3_8B = Qwen3Config(36, 4096, 32, 8, 128, 12288, 151936)
QWEN3_32B = Qwen3Config(64, 5120, 64, 8, 128, 25600, 151936, bits=8)


def tiny_config(**kw) -> Qwen3Config:
    """A small config with the real kernels' shape constraints (head_dim 128, hidden and
    intermediate multiples of 512) for parity tests."""
    base = Qwen3Config(2, 1024, 8, 2, 128, 1536, 4096)
    return replace(base, **kw)


def _interleave32(g: quant.QWeight, u: quant.QWeight) -> quant.QWeight:
    def il(a, b):
        n = a.shape[0]
        assert n % 32 == 0
        return torch.stack([a.reshape(n // 32, 32, -1), b.reshape(n // 32, 32, -1)],
                           dim=1).reshape(2 * n, -1).contiguous()
    return quant.QWeight(il(g.wq, u.wq), il(g.scales, u.scales), il(g.biases, u.biases), g.bits)


def _deinterleave32(t: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    n2 = t.shape[0]
    v = t.reshape(n2 // 64, 2, 32, -1)
    return v[:, 0].reshape(n2 // 2, -1), v[:, 1].reshape(n2 // 2, -1)


def _cat(*ws: quant.QWeight) -> quant.QWeight:
    return quant.QWeight(torch.cat([w.wq for w in ws]), torch.cat([w.scales for w in ws]),
                         torch.cat([w.biases for w in ws]), ws[0].bits)


def _qw_struct(w: quant.QWeight) -> _lib.QWeight:
    n, k = w.shape
    return _lib.QWeight(ptr(w.wq), ptr(w.scales), ptr(w.biases), n, k, w.bits)


class Target:
    """Random-init Qwen3-shaped target with a per-slot KV pool and fused verify forward."""

    def __init__(self, cfg: Qwen3Config, *, device="cuda", seed: int = 0, kv_cap: int = 4096,
                 slots: int = 1, max_rows: int = 32, std: float = 0.02,
                 slot_caps: list[int] | None = None):
        """``slot_caps`` (one capacity per slot) switches the KV pools to a position-major
        layout ``[sum(caps), Hk, D]`` where slot b owns positions ``[off_b, off_b + cap_b)``:
        requests of very different lengths then share the pool without each reserving the
        longest one's room. Without it every slot holds ``kv_cap`` positions
        (``[slots, Hk, kv_cap, D]``). A slot's cached length must stay within its capacity
        (the forward's cache write only bounds positions by the largest capacity)."""
        self.cfg = cfg
        self.device = torch.device(device)
        require_cuda(torch.empty(1, device=self.device))
        self.max_rows = int(max_rows)
        if slot_caps is not None:
            self.slot_caps = [int(c) for c in slot_caps]
            self.slots = len(self.slot_caps)
            self.kv_cap = max(self.slot_caps)
            self.position_major = True
            self._slot_base = [0]
            for c in self.slot_caps[:-1]:
                self._slot_base.append(self._slot_base[-1] + c)
        else:
            self.kv_cap = int(kv_cap)
            self.slots = int(slots)
            self.slot_caps = [self.kv_cap] * self.slots
            self.position_major = False
        g = torch.Generator(device=self.device).manual_seed(seed)
        H, D, Hq, Hk, I = cfg.hidden, cfg.head_dim, cfg.n_heads, cfg.n_kv_heads, cfg.intermediate
        bits = cfg.bits
        dev = self.device

        def rq(n, k):
            return quant.random_qweight(n, k, bits, std=std, device=dev, generator=g)

        def norm_w(n):
            return (1.0 + 0.05 * torch.randn(n, device=dev, generator=g)).to(torch.bfloat16)

        self.embed = rq(cfg.vocab, H)
        self.layers = []
        for _ in range(cfg.n_layers):
            q, k, v = rq(Hq * D, H), rq(Hk * D, H), rq(Hk * D, H)
            gate, up = rq(I, H), rq(I, H)
            layer = {
                "qkv": _cat(q, k, v),
                "o": rq(H, Hq * D),
                "gate_up": _interleave32(gate, up),
                "down": rq(H, I),
                "in_norm": norm_w(H), "post_norm": norm_w(H),
                "q_norm": norm_w(D), "k_norm": norm_w(D),
                "k_cache": self._pool(),
                "v_cache": self._pool(),
            }
            self.layers.append(layer)
        self.final_norm = norm_w(H)
        self.lm_head = rq(cfg.vocab, H)
        self._alloc_buffers()
        self._build_structs()

    # ----------------------------------------------------------------- C structs / buffers

    def _pool(self) -> torch.Tensor:
        D, Hk = self.cfg.head_dim, self.cfg.n_kv_heads
        if self.position_major:
            return torch.zeros((sum(self.slot_caps), Hk, D), dtype=torch.bfloat16,
                               device=self.device)
        return torch.zeros((self.slots, Hk, self.kv_cap, D), dtype=torch.bfloat16,
                           device=self.device)

    def kv_strides(self) -> tuple[int, int]:
        """(head stride, position stride) of the pools, in elements."""
        D, Hk = self.cfg.head_dim, self.cfg.n_kv_heads
        return (D, Hk * D) if self.position_major else (self.kv_cap * D, D)

    def slot_view(self, layer: int, slot: int, which: str = "k") -> torch.Tensor:
        """``[Hk, cap, D]`` view of one slot's keys or values."""
        pool = self.layers[layer][f"{which}_cache"]
        if self.position_major:
            b0 = self._slot_base[slot]
            return pool[b0 : b0 + self.slot_caps[slot]].permute(1, 0, 2)
        return pool[slot]

    def _alloc_buffers(self):
        cfg, dev, R = self.cfg, self.device, self.max_rows
        rows_cap = max(32, R)
        H, D, Hq, I = cfg.hidden, cfg.head_dim, cfg.n_heads, cfg.intermediate
        B = self.slots
        e = dict(device=dev)
        self.buf = {
            "h": torch.empty((R, H), dtype=torch.bfloat16, **e),
            "xq": torch.empty((R, Hq * D), dtype=torch.bfloat16, **e),
            "attn": torch.empty((R, Hq * D), dtype=torch.bfloat16, **e),
            "act": torch.empty((R, I), dtype=torch.bfloat16, **e),
            "ssq_a": torch.zeros(1024 * rows_cap, dtype=torch.float32, **e),
            "ssq_b": torch.zeros(1024 * rows_cap, dtype=torch.float32, **e),
            "inv_freq": torch.empty(D // 2, dtype=torch.float32, **e),
            "row_pos": torch.zeros(R, dtype=torch.int32, **e),
            "row_kv": torch.zeros(R, dtype=torch.int64, **e),
            "kv_len": torch.zeros(B, dtype=torch.int32, **e),
            "row_start": torch.zeros(B, dtype=torch.int32, **e),
            "q_len": torch.zeros(B, dtype=torch.int32, **e),
            "kv_off": torch.zeros(B, dtype=torch.int64, **e),
        }
        ws = int(_lib.lib.dspark_verify_attn_workspace(B, Hq, cfg.n_kv_heads, 32, D,
                                                       self.kv_cap))
        self.buf["attn_ws"] = torch.empty(max(ws, 16), dtype=torch.uint8, **e)
        # scratch of the wide-M projections (forwards of 64+ packed rows): normed x + product
        wide = 0
        if R >= 64:
            W = _lib.lib.dspark_qmm_wide_workspace
            qkv_n = (Hq + 2 * cfg.n_kv_heads) * D
            wide = max(W(R, H, qkv_n, _lib.EPI_QKROPE, 1), W(R, Hq * D, H, _lib.EPI_RESID, 0),
                       W(R, H, 2 * I, _lib.EPI_SWIGLU, 1), W(R, I, H, _lib.EPI_RESID, 0),
                       W(R, H, cfg.vocab, _lib.EPI_PLAIN, 1))
        self.buf["wide_ws"] = torch.empty(max(int(wide), 16), dtype=torch.uint8, **e)
        self.wide_ws_bytes = int(wide)
        self.logits = torch.empty((R, cfg.vocab), dtype=torch.bfloat16, **e)
        self.rows_cap = rows_cap

    def _build_structs(self):
        cfg = self.cfg
        D, Hk = cfg.head_dim, cfg.n_kv_heads
        arr = (_lib.Layer * cfg.n_layers)()
        for i, L in enumerate(self.layers):
            arr[i] = _lib.Layer(_qw_struct(L["qkv"]), _qw_struct(L["o"]),
                                _qw_struct(L["gate_up"]), _qw_struct(L["down"]),
                                ptr(L["in_norm"]), ptr(L["post_norm"]), ptr(L["q_norm"]),
                                ptr(L["k_norm"]), ptr(L["k_cache"]), ptr(L["v_cache"]))
        self._layers_c = arr
        k_sh, k_ss = self.kv_strides()
        self._model_c = _lib.Model(cfg.n_layers, cfg.hidden, cfg.n_heads, Hk, D,
                                   cfg.intermediate, cfg.vocab, cfg.rms_eps, cfg.rope_theta,
                                   _qw_struct(self.embed), _qw_struct(self.lm_head),
                                   ptr(self.final_norm), arr,
                                   k_sh, k_ss, k_sh, k_ss, self.kv_cap)
        b = self.buf
        self._buf_c = _lib.FwdBuffers(
            ptr(b["h"]), ptr(b["xq"]), ptr(b["attn"]), ptr(b["act"]), ptr(b["ssq_a"]),
            ptr(b["ssq_b"]), ptr(b["inv_freq"]), ptr(b["row_pos"]), ptr(b["row_kv"]),
            ptr(b["kv_len"]), ptr(b["row_start"]), ptr(b["q_len"]), ptr(b["kv_off"]),
            ptr(b["attn_ws"]), b["attn_ws"].numel(), self.rows_cap,
            ptr(b["wide_ws"]) if self.wide_ws_bytes else None, self.wide_ws_bytes)

    def slot_offset(self, slot: int) -> int:
        """Element offset of a request slot inside each layer's K/V pool."""
        if self.position_major:
            return self._slot_base[slot] * self.cfg.n_kv_heads * self.cfg.head_dim
        return slot * self.cfg.n_kv_heads * self.kv_cap * self.cfg.head_dim

    # ----------------------------------------------------------------- reference API

    def make_cache(self) -> torch.Tensor:
        """Per-slot cached-token counts (device int32 [slots]); the KV pools live in the
        target and are addressed by slot."""
        return torch.zeros(self.slots, dtype=torch.int32, device=self.device)

    def verify(self, ids: torch.Tensor, lens: torch.Tensor, *, L_max: int | None = None,
               logits: torch.Tensor | None = None) -> torch.Tensor:
        """One verify forward of ``ids`` (int32 ``[R]`` = ``[anchor] + drafts``) for slot 0 at
        its cached length ``lens[0]``; appends the block's K/V (``lens[0] += R`` on the
        device) and returns bf16 logits ``[R, vocab]``. Follow with :meth:`rollback` or
        :meth:`accept_and_rollback`. ``L_max`` bounds the key count (default: cache size)."""
        R = int(ids.numel())
        if not 1 <= R <= self.max_rows:
            raise _lib.DSparkUnsupported(_lib.ERR_UNSUPPORTED, f"R={R} rows")
        s = stream_of(ids)
        _lib.check(_lib.lib.dspark_verify_prepare(ptr(lens), R, C.byref(self._buf_c), s))
        out = self.logits if logits is None else logits
        Lm = self.kv_cap if L_max is None else int(L_max)
        _lib.check(_lib.lib.dspark_verify_forward(
            C.byref(self._model_c), C.byref(self._buf_c), ptr(ids), R, 1, R, Lm, ptr(out),
            out.stride(0), s))
        return out[:R]

    def forward_packed(self, ids: torch.Tensor, R: int, B: int, qL_max: int, L_max: int,
                       logits: torch.Tensor | None = None) -> torch.Tensor:
        """Verify forward over ragged packed rows; the packing arrays in ``self.buf`` must be
        filled for the step (see :mod:`.batch_engine`)."""
        out = self.logits if logits is None else logits
        _lib.check(_lib.lib.dspark_verify_forward(
            C.byref(self._model_c), C.byref(self._buf_c), ptr(ids), R, B, qL_max, L_max,
            ptr(out), out.stride(0), stream_of(ids)))
        return out[:R]

    def rollback(self, lens: torch.Tensor, n_rejected: torch.Tensor) -> None:
        """Trim the rejected tail: ``lens -= n_rejected`` (clamped at 0) on the device."""
        _lib.check(_lib.lib.dspark_kv_rollback(ptr(lens), ptr(n_rejected), int(lens.numel()),
                                               stream_of(lens)))

    def accept_and_rollback(self, logits: torch.Tensor, ids: torch.Tensor, lens: torch.Tensor,
                            out: dict | None = None) -> dict:
        """Greedy accept of one verify block fused with the rollback (all on the device):
        ``tt = argmax(logits)``, ``n`` = leading drafts equal to ``tt``, ``next = tt[n]``;
        ``lens`` (advanced to ``L0 + R`` by :meth:`verify`) ends at ``L0 + n + 1``."""
        R = int(ids.numel())
        dev = ids.device
        if out is None:
            out = {"tt": torch.empty(R, dtype=torch.int32, device=dev),
                   "n": torch.empty(1, dtype=torch.int32, device=dev),
                   "next": torch.empty(1, dtype=torch.int32, device=dev),
                   "cu": torch.tensor([0, R], dtype=torch.int32, device=dev)}
        s = stream_of(ids)
        _lib.check(_lib.lib.dspark_argmax(ptr(logits), logits.stride(0), R, self.cfg.vocab,
                                          ptr(out["tt"]), s))
        _lib.check(_lib.lib.dspark_accept(ptr(out["tt"]), ptr(ids), ptr(out["cu"]), 1,
                                          ptr(out["n"]), ptr(out["next"]), ptr(lens), s))
        return out

    # ----------------------------------------------------------------- checker support

    def oracle_weights(self, layers: int | None = None) -> dict:
        """Host numpy copies in the oracle's format (separate q/k/v/gate/up matrices)."""
        import numpy as np

        cfg = self.cfg
        Hq, Hk, D = cfg.n_heads, cfg.n_kv_heads, cfg.head_dim

        def qw(w: quant.QWeight):
            return {"wq": w.wq.cpu().numpy().view(np.uint32),
                    "scales": w.scales.cpu().view(torch.int16).numpy().view(np.uint16),
                    "biases": w.biases.cpu().view(torch.int16).numpy().view(np.uint16),
                    "bits": w.bits}

        def rows(w: quant.QWeight, a, b):
            return quant.QWeight(w.wq[a:b], w.scales[a:b], w.biases[a:b], w.bits)

        def f32(t):
            return t.float().cpu().numpy()

        out = {"embed": qw(self.embed), "lm_head": qw(self.lm_head),
               "final_norm": f32(self.final_norm), "layers": []}
        nq, nk = Hq * D, Hk * D
        for L in self.layers[: (cfg.n_layers if layers is None else layers)]:
            qkv = L["qkv"]
            gu = L["gate_up"]
            gw, uw = _deinterleave32(gu.wq)
            gs, us = _deinterleave32(gu.scales)
            gb, ub = _deinterleave32(gu.biases)
            out["layers"].append({
                "q": qw(rows(qkv, 0, nq)), "k": qw(rows(qkv, nq, nq + nk)),
                "v": qw(rows(qkv, nq + nk, nq + 2 * nk)), "o": qw(L["o"]),
                "gate": qw(quant.QWeight(gw, gs, gb, gu.bits)),
                "up": qw(quant.QWeight(uw, us, ub, gu.bits)), "down": qw(L["down"]),
                "in_norm": f32(L["in_norm"]), "post_norm": f32(L["post_norm"]),
                "q_norm": f32(L["q_norm"]), "k_norm": f32(L["k_norm"]),
            })
        return out

    def oracle_config(self) -> dict:
        c = self.cfg
        return {"hidden": c.hidden, "n_heads": c.n_heads, "n_kv_heads": c.n_kv_heads,
                "head_dim": c.head_dim, "rms_eps": c.rms_eps, "rope_theta": c.rope_theta}


class VerifyGraph:
    """One single-request spec round captured as a CUDA graph (the serving hot loop):
    verify forward of ``R`` rows at the slot's current length, argmax, greedy accept, and the
    rollback of the rejected tail — with no host work between kernels.

    ``ids`` (int32 ``[R]``), ``lens`` (int32 ``[1]``) and, when ``forced_rejects`` is used, the
    rejected count ``n_rej`` (int32 ``[1]``) are static device buffers the graph reads;
    results land in ``tt`` / ``n`` / ``next``. With ``forced_rejects=True`` the cache is
    trimmed by ``n_rej`` (a caller-chosen accept length, e.g. seeded draws for benchmarking
    random-init weights whose drafts never match) instead of by the greedy accept."""

    def __init__(self, target: Target, R: int = 16, *, L_max: int | None = None,
                 forced_rejects: bool = False):
        self.t = target
        self.R = int(R)
        dev = target.device
        self.ids = torch.zeros(self.R, dtype=torch.int32, device=dev)
        self.lens = torch.zeros(1, dtype=torch.int32, device=dev)
        self.n_rej = torch.zeros(1, dtype=torch.int32, device=dev)
        self.out = {"tt": torch.empty(self.R, dtype=torch.int32, device=dev),
                    "n": torch.empty(1, dtype=torch.int32, device=dev),
                    "next": torch.empty(1, dtype=torch.int32, device=dev),
                    "cu": torch.tensor([0, self.R], dtype=torch.int32, device=dev)}
        self.forced = bool(forced_rejects)
        self.L_max = target.kv_cap if L_max is None else int(L_max)
        self.graph = None
        self.launches_per_step = 0

    def _step(self):
        t, R = self.t, self.R
        s = stream_of(self.ids)
        logits = t.verify(self.ids, self.lens, L_max=self.L_max)
        _lib.check(_lib.lib.dspark_argmax(ptr(logits), logits.stride(0), R, t.cfg.vocab,
                                          ptr(self.out["tt"]), s))
        _lib.check(_lib.lib.dspark_accept(
            ptr(self.out["tt"]), ptr(self.ids), ptr(self.out["cu"]), 1, ptr(self.out["n"]),
            ptr(self.out["next"]), None if self.forced else ptr(self.lens), s))
        if self.forced:
            _lib.check(_lib.lib.dspark_kv_rollback(ptr(self.lens), ptr(self.n_rej), 1, s))

    def capture(self) -> "VerifyGraph":
        """Run the step once eagerly (configures every kernel), then capture it. The
        buffers' contents are restored after the warm-up run."""
        saved = self.lens.clone()
        self._step()
        torch.cuda.synchronize(self.t.device)
        self.lens.copy_(saved)
        side = torch.cuda.Stream(device=self.t.device)
        side.wait_stream(torch.cuda.current_stream(self.t.device))
        before = int(_lib.lib.dspark_launch_count())
        with torch.cuda.stream(side):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=side):
                self._step()
        torch.cuda.current_stream(self.t.device).wait_stream(side)
        self.launches_per_step = int(_lib.lib.dspark_launch_count()) - before
        self.graph = g
        return self

    def replay(self) -> None:
        self.graph.replay()
