#!/usr/bin/env python
"""Benchmark: verify-block throughput of the Qwen3-8B-shaped 4-bit target, M = 16 rows at 2k
context, on B200.

A step is one speculative verify round of one request: verify forward of 16 rows (the anchor
token + 15 drafts) through all 36 layers and the lm_head, argmax, greedy accept, and the KV
rollback — one CUDA graph of the library's fused kernels. Random-init weights never accept a
random draft, so the rollback follows seeded accept lengths n ~ U{0..15} (the cache grows by
n + 1 per step and is reset to 2048 tokens every 16 steps: mean context ~2.1k).

value      verify-block tokens/s = 16 * steps * n_gpus / max-over-ranks device time, inputs
           resident in HBM (weights 4.26 GB per step, far larger than the 126 MB L2: no flush
           needed).
e2e        same step through the public API (VerifyGraph) with the step's token ids copied
           from pinned host memory and the accept result (argmax row, n, next token) read back
           to pinned host memory every step.
roofline   the dominant kernel (gate/up QMM, ~48% of the bytes of a step), timed live with
           CUDA events over back-to-back launches on all 36 layers' weights: achieved =
           algorithmic bytes per launch / mean launch time vs the measured HBM copy bandwidth.
cpu_baseline  the CPU oracle (C + OpenMP restatement of the same forward) on this host's cores.

Multi-GPU (torchrun, one process per GPU): each rank runs independent requests on its own
replica of the weights (data-parallel requests, no collective in the timed work): weak
scaling. ``--impl reference`` times the reference arm: the CPU restatement of the path (the
reference itself is MLX/Metal-only and cannot run here) on rank 0.

The line also carries, at the same N, the two other multi-GPU configurations: ``tp``
(configs[3]: the Qwen3-32B-shaped 8-bit target at 32k context with every projection
column-sharded over the N ranks and NCCL all-gathers between them, strong scaling; with the
per-GPU HBM fraction and one layer's gathers timed alone) and ``batch`` (configs[4]: 256
requests of the continuous-batching engine partitioned data-parallel over the N ranks). Each
is its own device-timed measurement (max over ranks); ``--no-extras`` skips them.
"""

from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

CTX = 2048
ROWS = 16
METRIC = "verify-block tok/s at Qwen3-8B 4-bit M=16 (2k context)"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=40)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--quick", action="store_true", help="skip e2e/roofline extras")
    ap.add_argument("--no-extras", action="store_true",
                    help="skip the tensor-parallel and batch-engine measurements of the line")
    ap.add_argument("--micro", choices=["qmm", "attn", "attnq", "wide"], default=None,
                    help="run one kernel's microbench alone (ncu small cases)")
    ap.add_argument("--rows", type=int, nargs="+", default=[1, 4, 8, 16])
    ap.add_argument("--bits", type=int, default=4)
    ap.add_argument("--n", type=int, default=4096)
    ap.add_argument("--k", type=int, default=4096)
    ap.add_argument("--copies", type=int, default=48)
    ap.add_argument("--lengths", type=int, nargs="+", default=[1024, 4096, 16384, 32768])
    ap.add_argument("--reps", type=int, default=10)
    ap.add_argument("--batch", action="store_true",
                    help="BASELINE configs[4]: continuous-batching engine, requests split "
                         "data-parallel over the ranks")
    ap.add_argument("--tp", action="store_true",
                    help="BASELINE configs[3]: 32B-shaped 8-bit verify at 32k context, every "
                         "projection column-sharded over the ranks (NCCL all-gathers)")
    ap.add_argument("--tp-context", type=int, default=32768)
    ap.add_argument("--tp-comm", choices=["fused", "p2p", "nccl"], default="nccl",
                    help="--tp gathers: fused into the projections' peer stores, separate "
                         "peer-memory launches (dspark_p2p_allgather), or NCCL")
    ap.add_argument("--batch-requests", type=int, default=256,
                    help="requests in the whole job (256 in configs[4]; their KV is ~151 GB, "
                         "split over the ranks)")
    return ap.parse_args()


def peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": float(d["hbm_gbs"]), "src": "measured"}
    return {"hbm_gbs": 6650.0, "src": "fallback"}


# ----------------------------------------------------------------------------- clocks

class Clocks:
    """nvidia-smi sampled every 200 ms during the timed region."""

    Q = ("pci.bus_id,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, bus_id: str):
        self.bus = bus_id.lower().split(":", 1)[-1]
        self.f = tempfile.NamedTemporaryFile("w+", delete=False, suffix=".csv")
        try:
            self.p = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.Q}",
                                       "--format=csv,noheader,nounits", "-lms", "200"],
                                      stdout=self.f, stderr=subprocess.DEVNULL)
        except OSError:
            self.p = None

    def stop(self) -> dict:
        if self.p is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.p.terminate()
        self.p.wait(timeout=10)
        self.f.flush()
        rows = []
        for line in Path(self.f.name).read_text().splitlines():
            cols = [c.strip() for c in line.split(",")]
            if len(cols) < 9 or cols[0].lower().split(":", 1)[-1] != self.bus:
                continue
            rows.append(cols)
        os.unlink(self.f.name)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        sm = sorted(float(r[1]) for r in rows)
        reasons = set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            for n, v in zip(names, r[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": sm[len(sm) // 2], "sm_max_mhz": float(rows[0][2]),
                "reasons": sorted(reasons), "samples": len(rows),
                "power_w_max": max(float(r[3]) for r in rows if r[3].replace(".", "").isdigit())
                if any(r[3].replace(".", "").isdigit() for r in rows) else None}


# ----------------------------------------------------------------------------- helpers

def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def max_over_ranks(x: float, world: int, dev) -> float:
    if world == 1:
        return x
    import torch
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world: int):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def _config(world: int) -> dict:
    """The workload both arms report."""
    return {"workload": "qwen3-8b-shape 4-bit verify, 16-row blocks at 2k context "
                        "(BASELINE configs[2])",
            "model": "Qwen3-8B-shaped (36 layers, hidden 4096, inter 12288, GQA 32/8, "
                     "head_dim 128, vocab 151936), random init",
            "global_batch": world, "rows_per_block": ROWS, "seq_len": CTX,
            "parallelism": f"dp{world} (independent requests per GPU)",
            "l2": "inputs larger than L2 (4.26 GB of weights per step)",
            "accept": "seeded accept lengths U{0..15}; cache reset to 2048 every 16 steps"}


def host_model(seed: int = 0):
    """The Qwen3-8B-shaped 4-bit model for the CPU restatement, built on the host in MLX's
    packed layout: all 36 layers, the full embedding and lm_head (4.26 GB packed). Codes are
    uniform 4-bit words and each group's bf16 scale / bias lies in the range that N(0, 0.02)
    weights quantize to (scale ~ 0.0065, bias ~ -7.5 scale): the same bytes and arithmetic per
    step as the device model, generated in seconds instead of quantizing 7.6 B floats. Returns
    (weights, oracle config, K caches, V caches, ids) with 2k random bf16 keys / values cached
    (as bf16 bit patterns, the oracle's conversion-free cache form)."""
    sys.path.insert(0, str(ROOT / "oracle"))
    import numpy as np

    import oracle  # CPU restatement: checker / baseline only

    from mlx_dspark_b200.target import QWEN3_8B as c

    rng = np.random.default_rng(seed)
    # 256 bf16 scale / bias values in the quantized-N(0, 0.02) range, picked per group
    sc_tab = oracle.to_bf16(np.linspace(0.0055, 0.0075, 256, dtype=np.float32))
    bi_tab = oracle.to_bf16(-7.5 * np.linspace(0.005, 0.008, 256, dtype=np.float32))

    def qw(n, k):
        wq = rng.integers(0, 1 << 32, size=(n, k // 8), dtype=np.uint32)
        si = rng.integers(0, 256, size=(n, k // 64), dtype=np.uint8)
        bj = rng.integers(0, 256, size=(n, k // 64), dtype=np.uint8)
        return {"wq": wq, "scales": sc_tab[si], "biases": bi_tab[bj], "bits": 4}

    def nw(n):
        return oracle.round_bf16(1 + 0.05 * rng.standard_normal(n).astype(np.float32))

    H, I, Hq, Hk, D = c.hidden, c.intermediate, c.n_heads, c.n_kv_heads, c.head_dim
    layers = [{"q": qw(Hq * D, H), "k": qw(Hk * D, H), "v": qw(Hk * D, H), "o": qw(H, Hq * D),
               "gate": qw(I, H), "up": qw(I, H), "down": qw(H, I), "in_norm": nw(H),
               "post_norm": nw(H), "q_norm": nw(D), "k_norm": nw(D)}
              for _ in range(c.n_layers)]
    W = {"embed": qw(c.vocab, H), "lm_head": qw(c.vocab, H), "final_norm": nw(H),
         "layers": layers}
    ocfg = {"hidden": H, "n_heads": Hq, "n_kv_heads": Hk, "head_dim": D, "rms_eps": c.rms_eps,
            "rope_theta": c.rope_theta}
    kc = [oracle.to_bf16(rng.standard_normal((Hk, CTX + ROWS, D), dtype=np.float32))
          for _ in range(c.n_layers)]
    vc = [oracle.to_bf16(rng.standard_normal((Hk, CTX + ROWS, D), dtype=np.float32))
          for _ in range(c.n_layers)]
    ids = rng.integers(0, c.vocab, ROWS)
    return W, ocfg, kc, vc, ids


def cpu_threads() -> int:
    """Every host thread this process may run on (torchrun sets OMP_NUM_THREADS=1 per rank;
    the CPU arm runs on rank 0 alone and takes all of them)."""
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def cpu_forward_times(steps: int, warmup: int, seed: int = 0) -> dict:
    """Time the CPU restatement's full verify forward (embed, all 36 layers, final norm,
    lm_head) of one 16-row block at 2k context, ``warmup`` untimed + ``steps`` timed, on every
    host thread. Wall time per step, no extrapolation."""
    sys.path.insert(0, str(ROOT / "oracle"))
    import numpy as np

    import oracle  # CPU restatement: checker / baseline only

    oracle.build()
    oracle.set_threads(cpu_threads())
    cores = oracle.threads()
    t0 = time.perf_counter()
    W, ocfg, kc, vc, ids = host_model(seed)
    t_build = time.perf_counter() - t0
    times = []
    for i in range(warmup + steps):
        t0 = time.perf_counter()
        oracle.verify_forward(W, ocfg, ids, kc, vc, CTX)
        dt = time.perf_counter() - t0
        if i >= warmup:
            times.append(dt)
    secs = float(np.mean(times))
    return {"seconds_per_block": secs, "seconds_total": float(np.sum(times)), "cores": cores,
            "build_s": round(t_build, 1),
            "sample": (f"CPU restatement (C/OpenMP oracle + numpy) of the full verify forward, "
                       f"{ROWS} rows at {CTX} context: embed, all 36 layers, lm_head; {steps} "
                       f"timed blocks after {warmup} warm-up, mean {secs:.3f} s per block on "
                       f"{cores} threads")}


# ----------------------------------------------------------------------------- our arm

def run_ours(args):
    import numpy as np
    import torch

    world, rank, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    group = _dist_setup(world, dev)
    import mlx_dspark_b200  # noqa: F401
    from mlx_dspark_b200 import _lib
    from mlx_dspark_b200.target import QWEN3_8B, Target, VerifyGraph

    _lib.ensure_init(local)
    cfg = QWEN3_8B
    t = Target(cfg, kv_cap=4096, seed=1 + rank, max_rows=32)
    g = torch.Generator(device=dev).manual_seed(7 + rank)
    for L in t.layers:
        L["k_cache"][0, :, :CTX] = torch.randn(L["k_cache"][0, :, :CTX].shape, device=dev,
                                               generator=g).to(torch.bfloat16)
        L["v_cache"][0, :, :CTX] = torch.randn(L["v_cache"][0, :, :CTX].shape, device=dev,
                                               generator=g).to(torch.bfloat16)
    vg = VerifyGraph(t, ROWS, L_max=CTX + ROWS * 17, forced_rejects=True)
    vg.lens.fill_(CTX)
    vg.capture()
    total = args.warmup + args.steps
    rng = np.random.default_rng(1234 + rank)
    acc = rng.integers(0, ROWS, total)                   # accepted drafts n ~ U{0..15}
    ids_all = torch.randint(0, cfg.vocab, (total, ROWS), device=dev, dtype=torch.int32,
                            generator=g)
    nrej_all = torch.from_numpy((ROWS - 1 - acc).astype(np.int32)).to(dev)

    def step(i):
        if i % 16 == 0:
            vg.lens.fill_(CTX)
        vg.ids.copy_(ids_all[i])
        vg.n_rej.copy_(nrej_all[i : i + 1])
        vg.replay()

    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()
    pr = torch.cuda.get_device_properties(dev)
    bus = (f"{getattr(pr, 'pci_domain_id', 0):08x}:{getattr(pr, 'pci_bus_id', 0):02x}:"
           f"{getattr(pr, 'pci_device_id', 0):02x}.0")
    barrier(world)
    clk = Clocks(bus)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(args.warmup, total):
        step(i)
    e1.record()
    torch.cuda.synchronize()
    clocks = clk.stop()
    ms = e0.elapsed_time(e1)
    ms = max_over_ranks(ms, world, dev)
    barrier(world)
    st = _lib.device_status(local)
    secs = ms / 1e3
    value = world * args.steps * ROWS / secs
    committed = world * float((acc[args.warmup:] + 1).sum()) / secs
    weight_bytes = cfg.weight_bytes()
    kv_bytes = 2 * cfg.n_layers * cfg.n_kv_heads * cfg.head_dim * 2 * (CTX + 60)
    step_bytes = weight_bytes + kv_bytes

    out = {"metric": METRIC, "value": round(value, 1), "unit": "tok/s", "n_gpus": world,
           "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 4),
           "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
           "data": "synthetic (random-init N(0,0.02) weights quantized MLX-affine 4-bit g64; "
                   "random tokens; random bf16 KV prefix)",
           "config": _config(world),
           "blocks_per_s": round(world * args.steps / secs, 2),
           "committed_tok_s": round(committed, 1),
           "hbm_bytes_per_step": step_bytes,
           "step_hbm_gbs": round(step_bytes * args.steps / secs / 1e9, 1),
           "gpu_launches": vg.launches_per_step * args.steps,
           "launches_per_step": vg.launches_per_step,
           "clocks": clocks, "device_status": st}
    pk = peaks()
    out["step_roofline_frac"] = round(out["step_hbm_gbs"] / pk["hbm_gbs"], 3)

    if not args.quick:
        out["e2e"] = e2e(vg, ids_all, nrej_all, args, world, dev)
        out["roofline"] = roofline(t, dev, pk)
        out["qmm_microbench"] = qmm_microbench(dev, pk)
        out["attn_microbench"] = attn_microbench(dev, pk)
        out["wide_microbench"] = wide_microbench(dev)
        out["attn_q_microbench"] = attn_q_microbench(dev, pk)
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        try:
            cb = cpu_forward_times(steps=2, warmup=1)
            out["cpu_baseline"] = {"value": round(ROWS / cb["seconds_per_block"], 3),
                                   "unit": "tok/s", "cores": cb["cores"], "kind": "port",
                                   "sample": cb["sample"]}
        except Exception as e:  # noqa: BLE001 — the baseline must not sink the bench line
            out["cpu_baseline"] = {"value": None, "error": f"{type(e).__name__}: {e}"}
    vg.graph = None
    if not args.quick and not args.no_extras:
        # the other two multi-GPU configurations, at this job's N: tensor parallelism (configs[3],
        # strong scaling) and the data-parallel batch engine; every rank runs both
        del vg, t
        torch.cuda.empty_cache()
        out["tp"] = tp_measure(8, 3, world, rank, dev, group)
        out["batch"] = batch_measure(256, 6, 2, world, rank, dev)
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(out), flush=True)


def e2e(vg, ids_all, nrej_all, args, world, dev) -> dict:
    """Verify rounds through the public API with host buffers: per step, H2D of the block's
    ids from pinned memory, the graph, and D2H of (argmax row, n, next token) + sync."""
    import torch

    R = vg.R
    host_ids = torch.empty((args.steps, R), dtype=torch.int32).pin_memory()
    host_ids.copy_(ids_all[args.warmup :].cpu())
    host_out = torch.empty((R + 2,), dtype=torch.int32).pin_memory()
    s = torch.cuda.current_stream(dev)

    def one(i, ids_row):
        if i % 16 == 0:
            vg.lens.fill_(CTX)
        vg.ids.copy_(ids_row, non_blocking=True)
        vg.n_rej.copy_(nrej_all[(args.warmup + i) % nrej_all.numel()].view(1))
        vg.replay()
        host_out[:R].copy_(vg.out["tt"], non_blocking=True)
        host_out[R : R + 1].copy_(vg.out["n"], non_blocking=True)
        host_out[R + 1 : R + 2].copy_(vg.out["next"], non_blocking=True)
        s.synchronize()

    for i in range(min(3, args.steps)):
        one(i, host_ids[i])
    barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record()
    for i in range(args.steps):
        one(i, host_ids[i])
    e1.record()
    torch.cuda.synchronize()
    ms = max_over_ranks(e0.elapsed_time(e1), world, dev)
    return {"value": round(world * args.steps * R / (ms / 1e3), 1), "unit": "tok/s",
            "h2d_bytes_per_step": R * 4, "d2h_bytes_per_step": (R + 2) * 4,
            "ms_per_step": round(ms / args.steps, 4)}


def _qmm_bytes(n, k, m, bits):
    return n * k * bits // 8 + n * (k // 64) * 4 + m * k * 2 + m * n * 2


# DRAM bytes (read + write) of one launch of the step's gate/up instance (RMSNorm prologue,
# SwiGLU epilogue, 16 rows), from an ncu capture of the verify step itself:
#   python bench.py --steps 3 --warmup 3 --quick --no-cpu-baseline --no-extras
#   ncu --clock-control none --kernel-name-base demangled -k "regex:qmm_st_kernel<\\(int\\)4, \\(int\\)2, \\(int\\)2"
#       -s 8 -c 1 --section SpeedOfLight --section MemoryWorkloadAnalysis <the same command>
# dram__bytes.sum.per_second 1.886593 TB/s x gpu__time_duration.sum 30.208 us (cold, under ncu)
GATEUP_SWIGLU_TRAFFIC = 56_990_201


def roofline(t, dev, pk) -> dict:
    """Dominant kernel: the step's gate/up QMM instance (N = 24576, K = 4096, 16 rows, RMSNorm
    prologue from per-tile statistics, SwiGLU epilogue), launched back to back on all 36 layers'
    weights (2 GB, no L2 reuse), CUDA events on the launching stream."""
    import ctypes as C

    import torch

    from mlx_dspark_b200 import _lib
    from mlx_dspark_b200._torch import ptr

    cfg = t.cfg
    H, I = cfg.hidden, cfg.intermediate
    g = torch.Generator(device=dev).manual_seed(2)
    x = torch.randn((ROWS, H), device=dev, generator=g).to(torch.bfloat16)
    ssq = (x.float() ** 2).reshape(ROWS, H // 128, 128).sum(-1).t().contiguous()  # [tiles, rows]
    act = torch.empty((ROWS, I), dtype=torch.bfloat16, device=dev)
    args = []
    for L in t.layers:
        w = L["gate_up"]
        a = _lib.QmmArgs()
        a.x, a.ldx, a.M, a.K, a.N, a.bits = ptr(x), H, ROWS, H, 2 * I, w.bits
        a.wq, a.scales, a.biases = ptr(w.wq), ptr(w.scales), ptr(w.biases)
        a.out, a.ldo, a.epilogue, a.n_act = ptr(act), I, _lib.EPI_SWIGLU, I
        a.norm_w, a.ssq_in, a.ssq_n, a.ssq_stride = ptr(L["post_norm"]), ptr(ssq), H // 128, ROWS
        a.eps = cfg.rms_eps
        args.append(a)

    def burst():
        s = torch.cuda.current_stream(dev).cuda_stream
        for a in args:
            _lib.check(_lib.lib.dspark_qmm_fused(C.byref(a), s))

    per = _graph_time(burst, 10, dev) / len(args)
    nbytes = _qmm_bytes(2 * I, H, ROWS, cfg.bits)
    ach = nbytes / per / 1e9
    return {"kernel": "qmm_st_kernel<4, 2, EPI_SWIGLU> (gate/up 24576x4096, 4-bit, 16 rows, "
                      "RMSNorm prologue)", "bound": "hbm",
            "achieved": round(ach, 1), "peak": pk["hbm_gbs"], "unit": "GB/s",
            "frac": round(ach / pk["hbm_gbs"], 3), "traffic": GATEUP_SWIGLU_TRAFFIC,
            "algorithmic_bytes_per_launch": nbytes, "us_per_launch": round(per * 1e6, 2),
            "peak_source": pk["src"]}


def _graph_time(burst, reps: int, dev) -> float:
    """Seconds per replay of ``burst`` captured in a CUDA graph (3 untimed replays, then
    ``reps`` timed back to back with CUDA events on the replay stream)."""
    import torch

    burst()
    side = torch.cuda.Stream(device=dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(side):
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr, stream=side):
            burst()
    torch.cuda.current_stream(dev).wait_stream(side)
    for _ in range(3):
        gr.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        gr.replay()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / reps / 1e3


def qmm_microbench(dev, pk, rows=(1, 4, 8, 16), bits=4, n=4096, k=4096, copies=48,
                   reps=10) -> dict:
    """K = N = 4096, 4-bit, M in {1, 4, 8, 16}; ``copies`` distinct weight
    copies (48: ~450 MB, > 3x L2) rotated back to back inside a CUDA graph."""
    import torch

    from mlx_dspark_b200 import quant, skinny_qmm

    g = torch.Generator(device=dev).manual_seed(0)
    ws = [quant.random_qweight(n, k, bits, device=dev, generator=g) for _ in range(copies)]
    res = {}
    for M in rows:
        x = torch.randn((M, k), device=dev, generator=g).to(torch.bfloat16)
        out = torch.empty((M, n), dtype=torch.bfloat16, device=dev)

        def burst():
            for w in ws:
                skinny_qmm.qmm(x, w.wq, w.scales, w.biases, bits, out=out)

        per = _graph_time(burst, reps, dev) / len(ws)
        gbs = _qmm_bytes(n, k, M, bits) / per / 1e9
        res[f"M{M}"] = {"us": round(per * 1e6, 3), "gbs": round(gbs, 1),
                        "frac": round(gbs / pk["hbm_gbs"], 3)}
    return res


def wide_microbench(dev, rows=(256, 1024, 3072), n=24576, k=4096, bits=4, reps=5) -> dict:
    """The wide-M engine (dspark_qmm_wide, tcgen05) at the gate/up shape of the Qwen3-8B-shaped
    model for batch-engine row counts: TFLOP/s against the measured cuBLAS bf16 peak
    (MEASURED_PEAKS.json, burst figure for a kernel timed alone). Compute-bound from ~256 rows
    (the weights are re-read from L2 by every 256-row x tile, not from HBM)."""
    import torch

    from mlx_dspark_b200 import quant, wide_gemm

    p = ROOT / "MEASURED_PEAKS.json"
    peak = float(json.loads(p.read_text())["bf16_tflops"]) if p.exists() else 1590.0
    g = torch.Generator(device=dev).manual_seed(3)
    w = quant.random_qweight(n, k, bits, device=dev, generator=g)
    res = {"shape": f"{n}x{k} {bits}-bit", "peak_tflops": peak,
           "peak_source": "measured" if p.exists() else "fallback"}
    for M in rows:
        x = torch.randn((M, k), device=dev, generator=g).to(torch.bfloat16)
        out = torch.empty((M, n), dtype=torch.bfloat16, device=dev)

        def burst():
            for _ in range(4):
                wide_gemm.wide(x, w.wq, w.scales, w.biases, bits, out=out)

        per = _graph_time(burst, reps, dev) / 4
        tf = 2.0 * M * n * k / per / 1e12
        res[f"M{M}"] = {"us": round(per * 1e6, 2), "tflops": round(tf, 1),
                        "frac": round(tf / peak, 3)}
    return res


def attn_microbench(dev, pk, lengths=(1024, 4096, 16384, 32768), reps=10) -> dict:
    """GQA 32/8, head_dim 128, 16 causal query rows over a bf16 cache of
    L keys, scale 1/sqrt(128); distinct K/V copies rotated so at least ~400 MB (> 3x L2) is
    streamed per replay. Algorithmic bytes = K + V + q + out = 4096 L + 262144."""
    import torch

    from mlx_dspark_b200.multirow_attn import multirow_sdpa

    g = torch.Generator(device=dev).manual_seed(0)
    res = {}
    for L in lengths:
        nbytes = 4096 * L + 262144
        copies = max(3, -(-400_000_000 // nbytes))
        q = torch.randn((1, 32, 16, 128), device=dev, generator=g).to(torch.bfloat16)
        kv = [(torch.randn((1, 8, L, 128), device=dev, generator=g).to(torch.bfloat16),
               torch.randn((1, 8, L, 128), device=dev, generator=g).to(torch.bfloat16))
              for _ in range(copies)]
        out = torch.empty_like(q)

        def burst():
            for k, v in kv:
                multirow_sdpa(q, k, v, scale=128 ** -0.5, causal=True, out=out)

        per = _graph_time(burst, reps, dev) / copies
        gbs = nbytes / per / 1e9
        res[f"L{L}"] = {"us": round(per * 1e6, 3), "gbs": round(gbs, 1),
                        "frac": round(gbs / pk["hbm_gbs"], 3)}
        del kv
    return res


def attn_q_microbench(dev, pk, lengths=(2048, 32768), bits=(8, 4), reps=10) -> dict:
    """Verify attention over a quantized KV cache (the reference's kv_bits, mlx-lm's
    QuantizedKVCache, group 64): GQA 32/8, head_dim 128, 16 causal rows. Algorithmic bytes =
    K + V codes and their bf16 scales / biases + q + out = 8 * L * 2 * (128 * bits / 8 + 8) +
    262144; distinct caches rotated so that >= ~400 MB streams per replay (> 3x L2)."""
    import torch

    from mlx_dspark_b200.kvcache import QuantizedKVCache

    g = torch.Generator(device=dev).manual_seed(5)
    res = {}
    for nb in bits:
        for L in lengths:
            nbytes = 8 * L * 2 * (128 * nb // 8 + 8) + 262144
            copies = max(3, -(-400_000_000 // nbytes))
            q = torch.randn((1, 32, 16, 128), device=dev, generator=g).to(torch.bfloat16)
            caches = []
            for _ in range(copies):
                c = QuantizedKVCache(1, 8, L, 128, nb, device=dev)
                kv = torch.randn((1, 8, L, 128), device=dev, generator=g).to(torch.bfloat16)
                c.update(kv, kv)
                caches.append(c)
            out = torch.empty_like(q)

            def burst():
                for c in caches:
                    c.attention(q, scale=128 ** -0.5, causal=True, out=out)

            per = _graph_time(burst, reps, dev) / copies
            gbs = nbytes / per / 1e9
            res[f"b{nb}_L{L}"] = {"us": round(per * 1e6, 3), "gbs": round(gbs, 1),
                                  "frac": round(gbs / pk["hbm_gbs"], 3), "bytes": nbytes}
            del caches
    return res


def run_micro(args):
    """``--micro qmm|attn``: one kernel's microbench alone (the small cases profiled with ncu).
    Prints one JSON line."""
    import torch

    import mlx_dspark_b200  # noqa: F401
    from mlx_dspark_b200 import _lib

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    _lib.ensure_init(0)
    pk = peaks()
    if args.micro == "qmm":
        r = qmm_microbench(dev, pk, rows=tuple(args.rows), bits=args.bits, n=args.n, k=args.k,
                           copies=args.copies, reps=args.reps)
        cfg = {"bits": args.bits, "n": args.n, "k": args.k, "copies": args.copies}
    elif args.micro == "attnq":
        r = attn_q_microbench(dev, pk, lengths=tuple(args.lengths), bits=(args.bits,),
                              reps=args.reps)
        cfg = {"hq": 32, "hk": 8, "qL": 16, "d": 128, "kv_bits": args.bits}
    elif args.micro == "wide":
        r = wide_microbench(dev, rows=tuple(args.rows), n=args.n, k=args.k, bits=args.bits,
                            reps=args.reps)
        cfg = {"bits": args.bits, "n": args.n, "k": args.k}
    else:
        r = attn_microbench(dev, pk, lengths=tuple(args.lengths), reps=args.reps)
        cfg = {"hq": 32, "hk": 8, "qL": 16, "d": 128}
    print(json.dumps({"micro": args.micro, "config": cfg, "peak_gbs": pk["hbm_gbs"],
                      "peak_source": pk["src"], "result": r,
                      "device_status": _lib.device_status(0)}), flush=True)


def _dist_setup(world: int, dev, timeout_s: int = 300):
    if world > 1:
        import datetime

        import torch.distributed as dist

        if not dist.is_initialized():
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=timeout_s),
                                    device_id=dev)
        return dist.group.WORLD
    return None


def batch_measure(n_req: int, steps: int, warmup: int, world: int, rank: int, dev) -> dict:
    """``n_req`` requests (prompt lengths log-uniform 256-16k, seeded)
    placed data-parallel over the ranks by summed KV length (no collective in the data path);
    each step every request verifies a block of U{8..16} rows and keeps a seeded accept length
    U{0..block-1} (random-init weights never accept a random draft). Value = committed tokens
    per second over the whole job (sum of accepted + 1), device-timed, max over ranks."""
    import numpy as np
    import torch

    from mlx_dspark_b200 import _lib
    from mlx_dspark_b200.batch_engine import SpecBatch, partition_requests
    from mlx_dspark_b200.target import QWEN3_8B, Target

    rng = np.random.default_rng(2024)
    lengths = [int(x) for x in np.exp(rng.uniform(np.log(256), np.log(16384), n_req))]
    mine = partition_requests(lengths, world)[rank]
    total = warmup + steps
    my_len = [lengths[i] for i in mine]
    caps = [L + 17 * (total + 1) for L in my_len]
    B = len(mine)
    t = Target(QWEN3_8B, seed=1 + rank, slot_caps=caps, max_rows=max(32, 16 * B))
    g = torch.Generator(device=dev).manual_seed(11 + rank)
    for L in t.layers:  # random K/V prefixes
        for name in ("k_cache", "v_cache"):
            pool = L[name]
            for r0 in range(0, pool.shape[0], 1 << 16):
                r1 = min(pool.shape[0], r0 + (1 << 16))
                pool[r0:r1].normal_(generator=g)
    eng = SpecBatch(t, max_block=17)
    for L0 in my_len:
        eng.admit(L0, int(rng.integers(0, QWEN3_8B.vocab)))
    blocks = rng.integers(8, 17, (total, B))
    accs = np.array([[int(rng.integers(0, b)) for b in row] for row in blocks])
    drafts = torch.randint(0, QWEN3_8B.vocab, (total, B, 16), device=dev, dtype=torch.int32,
                           generator=g)
    acc_dev = torch.from_numpy(accs.astype(np.int32)).to(dev)
    launches0 = int(_lib.lib.dspark_launch_count())

    def step(i):
        eng.step(drafts[i], [int(x) for x in blocks[i]], forced_accept=acc_dev[i])

    for i in range(warmup):
        step(i)
    torch.cuda.synchronize()
    barrier(world)
    l0 = int(_lib.lib.dspark_launch_count())
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(warmup, total):
        step(i)
    e1.record()
    torch.cuda.synchronize()
    launches = int(_lib.lib.dspark_launch_count()) - l0
    ms = max_over_ranks(e0.elapsed_time(e1), world, dev)
    committed = float((accs[warmup:] + 1).sum())
    rows = float(blocks[warmup:].sum())
    kv_bytes = 2 * QWEN3_8B.n_layers * QWEN3_8B.n_kv_heads * QWEN3_8B.head_dim * 2 * sum(my_len)
    if world > 1:
        import torch.distributed as dist

        tot = torch.tensor([committed, rows], dtype=torch.float64, device=dev)
        dist.all_reduce(tot)
        committed, rows = float(tot[0]), float(tot[1])
    secs = ms / 1e3
    st = _lib.device_status(dev.index)
    del eng, t, drafts
    torch.cuda.empty_cache()
    _ = launches0
    return {"metric": "batch-engine committed tok/s (Qwen3-8B 4-bit, continuous batching)",
            "value": round(committed / secs, 1), "unit": "tok/s", "n_gpus": world,
            "steps": steps, "warmup": warmup, "ms_per_step": round(ms / steps, 3),
            "scaling": "strong",
            "config": {"workload": f"BASELINE configs[4] at {n_req} requests (prompts "
                                   "log-uniform 256-16k, blocks U{8..16}, accepts U{0..block-1})",
                       "requests": n_req, "requests_rank0": B,
                       "parallelism": f"dp{world} (requests partitioned by KV length)"},
            "verify_rows_per_s": round(rows / secs, 1), "rank0_kv_gb": round(kv_bytes / 1e9, 2),
            "gpu_launches_rank0": launches, "device_status": st}


def run_batch(args):
    """``--batch``: the batch-engine measurement alone (prints its JSON line)."""
    import torch

    world, rank, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    _dist_setup(world, dev)
    import mlx_dspark_b200  # noqa: F401
    from mlx_dspark_b200 import _lib

    _lib.ensure_init(local)
    out = batch_measure(int(args.batch_requests), args.steps, args.warmup, world, rank, dev)
    out.update(higher_is_better=True, vs_baseline=None, dtype="bf16",
               data="synthetic (random-init weights, random K/V prefixes, seeded blocks/accepts)")
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(out), flush=True)


def tp_measure(steps: int, warmup: int, world: int, rank: int, dev, group, *, context: int = 32768,
               comm: str = "nccl") -> dict:
    """Qwen3-32B-shaped 8-bit target (64 layers, hidden 5120, GQA 64/8),
    one request verifying 16-row blocks at ``context`` tokens, projections column-sharded over
    the ranks with all-gathers between them (mlx_dspark_b200.target_tp; NCCL by default). A step =
    verify forward + argmax + accept + rollback to a seeded accept length, captured in one CUDA
    graph (collectives included). value = verified rows per second of the one request (strong
    scaling: the same work at every N). Also: the gathers' own cost, timed with CUDA events
    around one layer's four gathers (eager, the same buffers and sizes)."""
    import numpy as np
    import torch

    from mlx_dspark_b200 import _lib
    from mlx_dspark_b200.target import QWEN3_32B
    from mlx_dspark_b200.target_tp import TPTarget

    cfg, ctx, R = QWEN3_32B, int(context), ROWS
    t = TPTarget(cfg, rank, world, group=group, kv_cap=ctx + R * 18, seed=1, max_rows=R,
                 device=dev, comm=comm)
    g = torch.Generator(device=dev).manual_seed(7)
    for L in t.layers:
        L["k_cache"][:, :ctx].normal_(generator=g)
        L["v_cache"][:, :ctx].normal_(generator=g)
    total = warmup + steps
    rng = np.random.default_rng(99)
    acc = rng.integers(0, R, total)
    ids_all = torch.randint(0, cfg.vocab, (total, R), device=dev, dtype=torch.int32, generator=g)
    nrej_all = torch.from_numpy((R - 1 - acc).astype(np.int32)).to(dev)
    ids = torch.zeros(R, dtype=torch.int32, device=dev)
    lens = torch.tensor([ctx], dtype=torch.int32, device=dev)
    nrej = torch.zeros(1, dtype=torch.int32, device=dev)
    out = {"tt": torch.empty(R, dtype=torch.int32, device=dev),
           "next": torch.empty(1, dtype=torch.int32, device=dev),
           "cu": torch.tensor([0, R], dtype=torch.int32, device=dev)}

    def body():
        logits = t.verify(ids, lens)
        s = torch.cuda.current_stream(dev).cuda_stream
        _lib.check(_lib.lib.dspark_argmax(logits.data_ptr(), logits.stride(0), R, cfg.vocab,
                                          out["tt"].data_ptr(), s))
        _lib.check(_lib.lib.dspark_accept(out["tt"].data_ptr(), ids.data_ptr(),
                                          out["cu"].data_ptr(), 1, None, out["next"].data_ptr(),
                                          None, s))
        _lib.check(_lib.lib.dspark_kv_rollback(lens.data_ptr(), nrej.data_ptr(), 1, s))

    body()  # configure every kernel once, then capture the step
    torch.cuda.synchronize()
    lens.fill_(ctx)
    side = torch.cuda.Stream(device=dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    before = int(_lib.lib.dspark_launch_count())
    with torch.cuda.stream(side):
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=side):
            body()
    torch.cuda.current_stream(dev).wait_stream(side)
    launches = int(_lib.lib.dspark_launch_count()) - before

    def step(i):
        if i % 16 == 0:
            lens.fill_(ctx)
        ids.copy_(ids_all[i])
        nrej.copy_(nrej_all[i : i + 1])
        graph.replay()

    for i in range(warmup):
        step(i)
    torch.cuda.synchronize()
    barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(warmup, total):
        step(i)
    e1.record()
    torch.cuda.synchronize()
    ms = max_over_ranks(e0.elapsed_time(e1), world, dev)
    # one layer's four gathers (attention output, hidden pack, activations, hidden pack), eager
    b = t.b
    gather_us = None
    if t.comm in ("nccl", "p2p", "local"):
        def gathers():
            t._gather("attn", 0, b["attn"])
            t._gather("pack", 0, b["pack"])
            t._gather("act", 0, b["act"])
            t._gather("pack", 1, b["pack"])

        for _ in range(3):
            gathers()
        torch.cuda.synchronize()
        barrier(world)
        g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        g0.record()
        for _ in range(20):
            gathers()
        g1.record()
        torch.cuda.synchronize()
        gather_us = max_over_ranks(g0.elapsed_time(g1) * 1e3 / 20, world, dev)
    secs = ms / 1e3
    w_bytes = cfg.weight_bytes() / world
    kv_bytes = 2 * cfg.n_layers * (cfg.n_kv_heads // world) * cfg.head_dim * 2 * (ctx + 8 * R)
    pk = peaks()
    per_gpu_gbs = (w_bytes + kv_bytes) / (ms / steps / 1e3) / 1e9
    st = _lib.device_status(dev.index)
    del graph
    t.close()
    del t
    torch.cuda.empty_cache()
    n_gathers = 4 * cfg.n_layers + 1 if world > 1 else 0
    return {"metric": "verify-block tok/s at Qwen3-32B-shaped 8-bit M=16 (32k context), "
                      "tensor-parallel", "value": round(steps * R / secs, 1), "unit": "tok/s",
            "n_gpus": world, "steps": steps, "warmup": warmup,
            "ms_per_step": round(ms / steps, 4), "scaling": "strong",
            "config": {"workload": f"qwen3-32b-shape 8-bit verify, 16-row blocks at {ctx} "
                                   "context (BASELINE configs[3])",
                       "parallelism": f"tp{world} (column-sharded projections, heads per rank, "
                                      + {"nccl": "NCCL all-gathers)",
                                         "p2p": "peer-memory all-gathers)",
                                         "fused": "gathers fused into the projections' peer "
                                                  "stores)",
                                         "local": "no collectives)"}[t_comm(world, comm)]},
            "per_gpu_hbm_bytes_per_step": int(w_bytes + kv_bytes),
            "per_gpu_hbm_gbs": round(per_gpu_gbs, 1),
            "per_gpu_hbm_frac": round(per_gpu_gbs / pk["hbm_gbs"], 3),
            "gathers_per_block": n_gathers,
            "one_layer_gathers_us": None if gather_us is None else round(gather_us, 2),
            "gathers_us_per_block_est": None if gather_us is None or world == 1
            else round(gather_us * cfg.n_layers, 1),
            "gpu_launches": launches * steps, "device_status": st}


def t_comm(world: int, comm: str) -> str:
    return comm if world > 1 else "local"


def run_tp(args):
    """``--tp``: the tensor-parallel measurement alone (prints its JSON line)."""
    import torch

    world, rank, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    group = _dist_setup(world, dev)
    import mlx_dspark_b200  # noqa: F401
    from mlx_dspark_b200 import _lib

    _lib.ensure_init(local)
    res = tp_measure(args.steps, args.warmup, world, rank, dev, group,
                     context=int(args.tp_context), comm=args.tp_comm)
    res.update(higher_is_better=True, vs_baseline=None, dtype="bf16",
               data="synthetic (random-init N(0,0.02) weights quantized MLX-affine 8-bit g64; "
                    "random tokens; random bf16 KV prefix)")
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(res), flush=True)


# ----------------------------------------------------------------------------- reference arm

def run_reference(args):
    """The reference arm: mlx-dspark's own path is MLX + Metal (Apple GPU) and MLX cannot be
    installed here, so the arm times the CPU restatement of the same arithmetic (the oracle:
    C/OpenMP quantized matmul and attention, numpy glue) on every host thread, on rank 0 only.
    Each step is one full verify forward of the Qwen3-8B-shaped 4-bit model (all 36 layers),
    16 rows at 2k context, timed by wall clock."""
    world, rank, _ = dist_env()
    if rank != 0:
        return
    cb = cpu_forward_times(steps=args.steps, warmup=args.warmup)
    secs = cb["seconds_per_block"]
    value = ROWS / secs
    out = {"metric": METRIC, "value": round(value, 3), "unit": "tok/s", "n_gpus": world,
           "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(secs * 1e3, 2),
           "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
           "data": "synthetic (random packed 4-bit weights, random tokens / KV)",
           "config": _config(world),
           "impl": "reference",
           "cpu_baseline": {"value": round(value, 3), "unit": "tok/s", "cores": cb["cores"],
                            "kind": "port", "sample": cb["sample"]},
           "e2e": {"value": round(value, 3), "unit": "tok/s", "h2d_bytes_per_step": 0,
                   "d2h_bytes_per_step": 0},
           "timed_s": round(cb["seconds_total"], 2), "build_s": cb["build_s"],
           "note": "mlx-dspark's own path is MLX/Metal (Apple GPU) and MLX is not installable "
                   "here; the arm runs the CPU restatement of the same arithmetic"}
    print(json.dumps(out), flush=True)


def main():
    args = parse()
    if args.micro:
        run_micro(args)
    elif args.batch:
        run_batch(args)
    elif args.tp:
        run_tp(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
