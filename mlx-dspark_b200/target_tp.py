"""Column-sharded (tensor-parallel) verify forward of a dense Qwen3-shaped target over P GPUs.

For 27B-class targets one GPU's HBM bandwidth is the limit, so every projection's output
columns are split over P ranks (one process per GPU, NCCL over NVLink):

* q/k/v: rank r owns query heads [r*Hq/P, (r+1)*Hq/P) and KV heads [r*Hk/P, ...). The QKV
  launch normalizes, ropes and writes its heads' K/V into the rank's own cache, and the
  verify attention runs over those heads only — attention needs no exchange.
* O, gate/up, down, lm_head: rank r owns 1/P of the output columns (gate/up: 1/P of the
  intermediate units, still interleaved in blocks of 32 so SwiGLU stays in the epilogue).
* Between projections the shards are all-gathered: the attention output before O, the
  updated hidden state (and its per-tile RMSNorm statistics) after O and after down, the
  SwiGLU activations before down, and the vocab-sharded logits at the end. The gathered
  ``[P, M, K/P]`` tensors feed the next projection directly: the QMM reads x as segmented
  rows (``dspark_qmm_fused`` with ``x_seg``), so no transpose copy runs.
* ``comm="nccl"`` (the default, the fastest measured at P = 2) all-gathers with NCCL. The two
  peer-memory transports map every peer's arena through CUDA IPC. ``comm="fused"`` folds three
  of a layer's four gathers into the projections:
  O and down store their hidden shard and its statistics, gate/up its activations, straight
  into segment ``rank`` of every rank's buffer from the epilogue, and count the elements on
  the peers' completion counters; the next projection waits, bounded, on those counters before
  it reads x. The attention output and the logits go through ``dspark_p2p_allgather``, one
  launch that stores a segment into every arena and waits for the peers'. ``comm="p2p"`` uses
  that launch for every gather.

Every rank holds the full embedding and norm weights and computes the same argmax / accept /
rollback, so all ranks' cache lengths stay identical. Weights are generated from one seed as
the full matrices and sliced, so any P yields the same model (the P-independence the parity
tests check). The reference runs 27B targets on one Apple GPU (``src/mlx_dspark/target.py``
dense path, ``:208-221``); this layer has no counterpart there.
"""

from __future__ import annotations

import ctypes as C

import torch

from . import _lib, quant
from ._torch import ptr, require_cuda, stream_of
from .target import Qwen3Config, _interleave32, _qw_struct  # noqa: F401


class _CudaBytes:
    """A device byte range exposed through ``__cuda_array_interface__`` (zero-copy view)."""

    def __init__(self, addr: int, n: int):
        self.__cuda_array_interface__ = {"shape": (n,), "typestr": "|u1", "data": (addr, False),
                                         "version": 3, "strides": None}


def _device_bytes(addr: int, n: int, device) -> torch.Tensor:
    return torch.as_tensor(_CudaBytes(addr, n), device=device)


def _rows(w: quant.QWeight, a: int, b: int) -> quant.QWeight:
    return quant.QWeight(w.wq[a:b].contiguous(), w.scales[a:b].contiguous(),
                         w.biases[a:b].contiguous(), w.bits)


def _cat(*ws: quant.QWeight) -> quant.QWeight:
    return quant.QWeight(torch.cat([w.wq for w in ws]), torch.cat([w.scales for w in ws]),
                         torch.cat([w.biases for w in ws]), ws[0].bits)


def shard_ranges(cfg: Qwen3Config, world: int, rank: int) -> dict:
    """Row ranges of each full weight matrix that rank ``rank`` of ``world`` owns."""
    H, D, Hq, Hk, I, V = (cfg.hidden, cfg.head_dim, cfg.n_heads, cfg.n_kv_heads,
                          cfg.intermediate, cfg.vocab)
    for what, n in (("query heads", Hq), ("kv heads", Hk), ("hidden", H // 128),
                    ("intermediate", I // 32), ("vocab", V // 8)):
        if n % world:
            raise ValueError(f"{what} ({n}) do not split over {world} ranks")
    hq, hk = Hq // world, Hk // world
    return {"q": (rank * hq * D, (rank + 1) * hq * D),
            "k": (Hq * D + rank * hk * D, Hq * D + (rank + 1) * hk * D),
            "v": (Hq * D + Hk * D + rank * hk * D, Hq * D + Hk * D + (rank + 1) * hk * D),
            "hidden": (rank * H // world, (rank + 1) * H // world),
            "inter": (rank * I // world, (rank + 1) * I // world),
            "vocab": (rank * V // world, (rank + 1) * V // world)}


class TPTarget:
    """One rank of a P-way column-sharded target (``group``: the torch.distributed NCCL group;
    ``None`` with ``world == 1``). :meth:`verify` has :meth:`Target.verify`'s contract."""

    def __init__(self, cfg: Qwen3Config, rank: int, world: int, *, group=None, kv_cap: int = 4096,
                 seed: int = 0, std: float = 0.02, max_rows: int = 32, device="cuda",
                 comm: str = "nccl"):
        self.cfg, self.rank, self.world, self.group = cfg, int(rank), int(world), group
        if comm not in ("fused", "p2p", "nccl"):
            raise ValueError(f"comm must be 'fused', 'p2p' or 'nccl', not {comm!r}")
        self.comm = comm if self.world > 1 else "local"
        self._arena, self._peers = None, []
        self.device = torch.device(device)
        require_cuda(torch.empty(1, device=self.device))
        self.kv_cap, self.max_rows = int(kv_cap), int(max_rows)
        P, r = self.world, self.rank
        rg = shard_ranges(cfg, P, r)
        self.ranges = rg
        H, D, Hq, Hk, I = cfg.hidden, cfg.head_dim, cfg.n_heads, cfg.n_kv_heads, cfg.intermediate
        self.hq, self.hk = Hq // P, Hk // P
        dev = self.device
        g = torch.Generator(device=dev).manual_seed(seed)

        def full(n, k):
            return quant.random_qweight(n, k, cfg.bits, std=std, device=dev, generator=g)

        def norm_w(n):
            return (1.0 + 0.05 * torch.randn(n, device=dev, generator=g)).to(torch.bfloat16)

        self.embed = full(cfg.vocab, H)
        self.layers = []
        for _ in range(cfg.n_layers):
            qkv = full((Hq + 2 * Hk) * D, H)
            o = full(H, Hq * D)
            gate, up = full(I, H), full(I, H)
            down = full(H, I)
            a, b = rg["inter"]
            h0, h1 = rg["hidden"]
            layer = {
                "qkv": _cat(_rows(qkv, *rg["q"]), _rows(qkv, *rg["k"]), _rows(qkv, *rg["v"])),
                "o": _rows(o, h0, h1),
                "gate_up": _interleave32(_rows(gate, a, b), _rows(up, a, b)),
                "down": _rows(down, h0, h1),
                "in_norm": norm_w(H), "post_norm": norm_w(H),
                "q_norm": norm_w(D), "k_norm": norm_w(D),
                "k_cache": torch.zeros((self.hk, self.kv_cap, D), dtype=torch.bfloat16, device=dev),
                "v_cache": torch.zeros((self.hk, self.kv_cap, D), dtype=torch.bfloat16, device=dev),
            }
            del qkv, o, gate, up, down
            self.layers.append(layer)
        self.final_norm = norm_w(H)
        lm = full(cfg.vocab, H)
        self.lm_head = _rows(lm, *rg["vocab"])
        del lm
        torch.cuda.empty_cache()
        self._alloc()

    # ------------------------------------------------------------------ buffers

    def _alloc(self):
        cfg, P, R, dev = self.cfg, self.world, self.max_rows, self.device
        H, D, I, V = cfg.hidden, cfg.head_dim, cfg.intermediate, cfg.vocab
        bf = dict(dtype=torch.bfloat16, device=dev)
        self.hs = H // P                       # hidden columns per rank
        self.tiles = self.hs // 128            # RMSNorm statistics entries per rank
        # a rank's hidden shard [R, hs] bf16 and its RMSNorm statistics [tiles, 32] fp32 travel
        # in one buffer (one all-gather): pack = [h shard | statistics]
        self.hbytes = R * self.hs * 2
        self.pack = self.hbytes + self.tiles * 32 * 4
        u8 = dict(dtype=torch.uint8, device=dev)
        # gather destinations: two per kind (alternating: a buffer is rewritten only after the
        # kernels that read it have run on every rank), one for the logits
        self._segs = {"attn": (R * self.hq * D * 2, 2), "pack": (self.pack, 2),
                      "act": (R * (I // P) * 2, 2), "logits": (R * (V // P) * 2, 1)}
        seg = self._alloc_gather_buffers() if self.comm in ("p2p", "fused") else {
            k: [torch.zeros(P * n, **u8) for _ in range(c)] for k, (n, c) in self._segs.items()}
        self.b = {
            "h0": torch.empty((R, H), **bf),                    # embedding output (replicated)
            "pack": torch.zeros(self.pack, **u8),
            "pack_seg": [t.view(P, self.pack) for t in seg["pack"]],
            "xq": torch.empty((R, self.hq * D), **bf),
            "attn": torch.empty((R, self.hq * D), **bf),
            "attn_seg": [t.view(torch.bfloat16).view(P, R, self.hq * D) for t in seg["attn"]],
            "act": torch.empty((R, I // P), **bf),
            "act_seg": [t.view(torch.bfloat16).view(P, R, I // P) for t in seg["act"]],
            "logits": torch.empty((R, V // P), **bf),
            "logits_seg": seg["logits"][0].view(torch.bfloat16).view(P, R, V // P),
            "logits_full": torch.empty((R, V), **bf),
            "ssq0": torch.zeros(1024 * 32, dtype=torch.float32, device=dev),
            "inv_freq": torch.empty(D // 2, dtype=torch.float32, device=dev),
            "row_pos": torch.zeros(R, dtype=torch.int32, device=dev),
            "row_kv": torch.zeros(R, dtype=torch.int64, device=dev),
            "kv_len": torch.zeros(1, dtype=torch.int32, device=dev),
            "row_start": torch.zeros(1, dtype=torch.int32, device=dev),
            "q_len": torch.zeros(1, dtype=torch.int32, device=dev),
            "kv_off": torch.zeros(1, dtype=torch.int64, device=dev),
        }
        b = self.b
        # the split plan (and its workspace) depends on the block height: size for the largest
        ws = max(int(_lib.lib.dspark_verify_attn_workspace(1, self.hq, self.hk, qL, D, L))
                 for qL in range(1, R + 1) for L in (self.kv_cap, max(1, self.kv_cap // 2)))
        b["attn_ws"] = torch.empty(max(ws, 16), dtype=torch.uint8, device=dev)
        # the single-request packing entry fills row_pos / kv_len through this struct
        self._prep = _lib.FwdBuffers(None, None, None, None, None, None, None, ptr(b["row_pos"]),
                                     ptr(b["row_kv"]), ptr(b["kv_len"]), ptr(b["row_start"]),
                                     ptr(b["q_len"]), ptr(b["kv_off"]), None, 0, R)

    # arena layout (identical on every rank): flags uint32 [8][8] at 0, counters uint32 [8][2]
    # at 256, then the gather buffers, 256-byte aligned, [P][segment bytes] each
    _FLAGS_OFF, _COUNT_OFF, _DATA_OFF = 0, 256, 512

    def _alloc_gather_buffers(self) -> dict:
        """One IPC arena per rank holding every gather destination; peers' arenas are mapped
        so that ``dspark_p2p_allgather`` stores straight into them."""
        import torch.distributed as dist

        P = self.world
        self._slots, off = {}, self._DATA_OFF
        for k, (n, c) in self._segs.items():
            for i in range(c):
                self._slots[(k, i)] = (len(self._slots), off, n)
                off += (P * n + 255) // 256 * 256
        base, handle = C.c_void_p(), (C.c_char * _lib.IPC_HANDLE_BYTES)()
        _lib.check(_lib.lib.dspark_ipc_alloc(off, C.byref(base), handle))
        self._arena = base.value
        handles = [None] * P
        dist.all_gather_object(handles, bytes(handle), group=self.group)
        ptrs = []
        for q in range(P):
            if q == self.rank:
                ptrs.append(self._arena)
                continue
            h = (C.c_char * _lib.IPC_HANDLE_BYTES).from_buffer_copy(handles[q])
            peer = C.c_void_p()
            _lib.check(_lib.lib.dspark_ipc_open(h, C.byref(peer)))
            self._peers.append(peer.value)
            ptrs.append(peer.value)
        self._arena_ptrs = (C.c_void_p * P)(*ptrs)
        views = {}
        for (k, i), (_, o, n) in self._slots.items():
            views.setdefault(k, []).append(_device_bytes(self._arena + o, P * n, self.device))
        return views

    def close(self) -> None:
        """Unmap the peers' arenas and free this rank's (after the device is idle)."""
        if self._arena is None:
            return
        torch.cuda.synchronize(self.device)
        for q in self._peers:
            _lib.lib.dspark_ipc_close(C.c_void_p(q))
        self._peers = []
        _lib.lib.dspark_ipc_free(C.c_void_p(self._arena))
        self._arena = None

    def _own(self, kind: str, i: int) -> int:
        """Address of this rank's segment of gather destination (kind, i) in its own arena."""
        _, off, n = self._slots[(kind, i)]
        return self._arena + off + self.rank * n

    def _peer_args(self, a, kind: str, i: int) -> None:
        """Peer stores of a projection's output into destination (kind, i) of every arena."""
        slot = self._slots[(kind, i)][0]
        a.peer_world = self.world
        for q in range(self.world):
            a.peer_delta[q] = self._arena_ptrs[q] - self._arena
        a.peer_flag = self._arena + self._FLAGS_OFF + (slot * 8 + self.rank) * 4

    def _wait_args(self, a, kind: str, i: int, elems: int) -> None:
        """Wait, before x is read, for every rank's ``elems`` elements of destination (kind, i)."""
        slot = self._slots[(kind, i)][0]
        a.wait_flag = self._arena + self._FLAGS_OFF + slot * 8 * 4
        a.wait_world, a.wait_elems = self.world, elems
        a.wait_state = self._arena + self._COUNT_OFF + slot * 2 * 4

    def _gather(self, kind: str, i: int, inp: torch.Tensor) -> None:
        """All-gather this rank's ``inp`` into segment ``rank`` of destination ``(kind, i)``."""
        out = {"attn": self.b["attn_seg"], "pack": self.b["pack_seg"],
               "act": self.b["act_seg"]}.get(kind)
        out = self.b["logits_seg"] if kind == "logits" else out[i]
        if self.comm == "local":
            out.view(-1).copy_(inp.view(-1).view(out.dtype))
        elif self.comm == "fused" and kind in ("pack", "act"):
            return  # the producing projection stored into every rank's buffer itself
        elif self.comm == "nccl":
            import torch.distributed as dist

            dist.all_gather_into_tensor(out.view(-1), inp.view(-1).view(out.dtype), group=self.group)
        else:
            slot, off, n = self._slots[(kind, i)]
            a = _lib.P2PGatherArgs(C.cast(self._arena_ptrs, C.POINTER(C.c_void_p)), inp.data_ptr(), n,
                                   self._FLAGS_OFF,
                                   self._COUNT_OFF, off, self.rank, self.world, slot)
            _lib.check(_lib.lib.dspark_p2p_allgather(C.byref(a), stream_of(inp)))

    def _qmm(self, s, w: quant.QWeight, x, ldx, M, K, epi, out=None, ldo=0, *, x_seg=0,
             x_seg_stride=0, norm_w=None, ssq_in=None, ssq_n=0, ssq_seg=0, ssq_seg_stride=0,
             resid=None, ldr=0, ssq_out=None, n_act=0, layer=None, peer=None, wait=None):
        a = _lib.QmmArgs()
        if peer is not None:
            self._peer_args(a, *peer)
        if wait is not None:
            self._wait_args(a, *wait)
        a.x = x if isinstance(x, int) else ptr(x)
        a.ldx, a.x_seg, a.x_seg_stride = ldx, x_seg, x_seg_stride
        a.M, a.K, a.N, a.bits = M, K, int(w.wq.shape[0]), w.bits
        a.wq, a.scales, a.biases = ptr(w.wq), ptr(w.scales), ptr(w.biases)
        a.out = out if isinstance(out, int) else ptr(out)
        a.ldo, a.epilogue = ldo, epi
        a.norm_w, a.ssq_n, a.ssq_stride = ptr(norm_w), ssq_n, 32
        a.ssq_in = ssq_in if isinstance(ssq_in, int) or ssq_in is None else ptr(ssq_in)
        a.ssq_seg, a.ssq_seg_stride = ssq_seg, ssq_seg_stride

        a.eps = self.cfg.rms_eps
        a.resid = resid if isinstance(resid, int) else ptr(resid)
        a.ldr, a.n_act = ldr, n_act
        a.ssq_out = ssq_out if isinstance(ssq_out, int) else ptr(ssq_out)
        if epi == _lib.EPI_QKROPE:
            b, D = self.b, self.cfg.head_dim
            a.hq, a.hk = self.hq, self.hk
            a.q_norm, a.k_norm, a.inv_freq = ptr(layer["q_norm"]), ptr(layer["k_norm"]), ptr(b["inv_freq"])
            a.q_out, a.ldq = ptr(b["xq"]), self.hq * D
            a.k_cache, a.v_cache = ptr(layer["k_cache"]), ptr(layer["v_cache"])
            a.k_sh, a.k_ss, a.v_sh, a.v_ss = self.kv_cap * D, D, self.kv_cap * D, D
            a.kv_cap = self.kv_cap
            a.row_pos, a.row_kv = ptr(b["row_pos"]), ptr(b["row_kv"])
        _lib.check(_lib.lib.dspark_qmm_fused(C.byref(a), s))

    # ------------------------------------------------------------------ forward

    def verify(self, ids: torch.Tensor, lens: torch.Tensor, *, L_max: int | None = None) -> torch.Tensor:
        """Verify forward of ``ids`` (int32 ``[R]``) at the cached length ``lens[0]`` (advanced
        by R on the device); returns the full bf16 logits ``[R, vocab]`` on every rank."""
        cfg, P, r, b = self.cfg, self.world, self.rank, self.b
        R = int(ids.numel())
        if not 1 <= R <= self.max_rows:
            raise _lib.DSparkUnsupported(_lib.ERR_UNSUPPORTED, f"R={R} rows")
        H, D, Hq, I, V = cfg.hidden, cfg.head_dim, cfg.n_heads, cfg.intermediate, cfg.vocab
        hs, T = self.hs, self.tiles
        s = stream_of(ids)
        _lib.check(_lib.lib.dspark_verify_prepare(ptr(lens), R, C.byref(self._prep), s))
        _lib.check(_lib.lib.dspark_rope_inv_freq(ptr(b["inv_freq"]), D, cfg.rope_theta, s))
        _lib.check(_lib.lib.dspark_embed(ptr(ids), R, ptr(self.embed.wq), ptr(self.embed.scales),
                                         ptr(self.embed.biases), cfg.vocab, H, cfg.bits,
                                         ptr(b["h0"]), ptr(b["ssq0"]), s))
        Lm = self.kv_cap if L_max is None else int(L_max)
        # current hidden state: contiguous (embedding) or the gathered packs [P, pack] (after a
        # gather: rank q's hidden shard at q*pack, its statistics at q*pack + hbytes)
        pk, hb = self.pack, self.hbytes
        loc = b["pack"].data_ptr()
        x, ldx, xseg, xss = b["h0"].data_ptr(), H, 0, 0
        ssq, ssq_n, sseg, ssegs = b["ssq0"].data_ptr(), 1, 0, 0
        resid, ldr = b["h0"][:, r * hs:].data_ptr(), H
        cur = 0
        fz = self.comm == "fused"
        xwait = None  # the gathered hidden state x is waited on (fused gathers, after layer 0)
        q_st = _lib.i64_array([0, D, self.hq * D])
        k_st = _lib.i64_array([0, self.kv_cap * D, D])
        for li, L in enumerate(self.layers):
            j = li & 1  # alternating gather destinations
            self._qmm(s, L["qkv"], x, ldx, R, H, _lib.EPI_QKROPE, x_seg=xseg, x_seg_stride=xss,
                      norm_w=L["in_norm"], ssq_in=ssq, ssq_n=ssq_n, ssq_seg=sseg,
                      ssq_seg_stride=ssegs, layer=L, wait=xwait)
            _lib.check(_lib.lib.dspark_verify_attn(
                ptr(b["xq"]), q_st, ptr(L["k_cache"]), k_st, ptr(L["v_cache"]), k_st, 1, self.hq,
                self.hk, R, D, Lm, ptr(b["kv_len"]), float(D ** -0.5), 1, None, ptr(b["attn"]),
                q_st, ptr(b["attn_ws"]), b["attn_ws"].numel(), s))
            self._gather("attn", j, b["attn"])
            # O: x = all heads' attention ([P, R, hq*D] segments), residual = own hidden shard;
            # the new shard and its statistics land in this rank's pack
            o_out = self._own("pack", cur) if fz else loc
            self._qmm(s, L["o"], b["attn_seg"][j], self.hq * D, R, Hq * D, _lib.EPI_RESID, o_out,
                      hs, x_seg=self.hq * D, x_seg_stride=self.max_rows * self.hq * D,
                      resid=resid, ldr=ldr, ssq_out=o_out + hb,
                      peer=("pack", cur) if fz else None)
            mid = b["pack_seg"][cur]
            self._gather("pack", cur, b["pack"])
            mb = mid.data_ptr()
            # gate/up: post-attention norm over the gathered hidden state, SwiGLU shard
            self._qmm(s, L["gate_up"], mb, hs, R, H, _lib.EPI_SWIGLU,
                      self._own("act", j) if fz else b["act"], I // P,
                      x_seg=hs, x_seg_stride=pk // 2, norm_w=L["post_norm"], ssq_in=mb + hb,
                      ssq_n=P * T, ssq_seg=T, ssq_seg_stride=pk // 4, n_act=I // P,
                      peer=("act", j) if fz else None,
                      wait=("pack", cur, R * hs) if fz else None)
            self._gather("act", j, b["act"])
            # down: x = all activations, residual = own shard of the mid state
            d_out = self._own("pack", cur ^ 1) if fz else loc
            self._qmm(s, L["down"], b["act_seg"][j], I // P, R, I, _lib.EPI_RESID, d_out, hs,
                      x_seg=I // P, x_seg_stride=self.max_rows * (I // P), resid=mb + r * pk,
                      ldr=hs, ssq_out=d_out + hb, peer=("pack", cur ^ 1) if fz else None,
                      wait=("act", j, R * (I // P)) if fz else None)
            cur ^= 1
            nxt = b["pack_seg"][cur]
            self._gather("pack", cur, b["pack"])
            nb = nxt.data_ptr()
            x, ldx, xseg, xss = nb, hs, hs, pk // 2
            ssq, ssq_n, sseg, ssegs = nb + hb, P * T, T, pk // 4
            resid, ldr = nb + r * pk, hs
            xwait = ("pack", cur, R * hs) if fz else None
        # final norm + vocab-sharded lm_head, logits gathered
        self._qmm(s, self.lm_head, x, ldx, R, H, _lib.EPI_PLAIN, b["logits"], V // P, x_seg=xseg,
                  x_seg_stride=xss, norm_w=self.final_norm, ssq_in=ssq, ssq_n=ssq_n,
                  ssq_seg=sseg, ssq_seg_stride=ssegs, wait=xwait)
        self._gather("logits", 0, b["logits"])
        b["logits_full"][:R].view(R, P, V // P).copy_(b["logits_seg"][:, :R].transpose(0, 1))
        return b["logits_full"][:R]

    def accept_and_rollback(self, logits, ids, lens, out=None) -> dict:
        """Greedy accept + rollback, identical on every rank (the ranks' caches stay in step)."""
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

    def oracle_weights(self) -> dict:
        """Host copies of the full weights in the oracle's format (one rank, P == 1 only)."""
        if self.world != 1:
            raise ValueError("the full weights exist on a single rank only when P == 1")
        from .target import Target

        return Target.oracle_weights(self)

    def oracle_config(self) -> dict:
        c = self.cfg
        return {"hidden": c.hidden, "n_heads": c.n_heads, "n_kv_heads": c.n_kv_heads,
                "head_dim": c.head_dim, "rms_eps": c.rms_eps, "rope_theta": c.rope_theta}
