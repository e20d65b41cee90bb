#!/usr/bin/env python
"""nanoGPT f32 training throughput (tokens/s) on B200 through the malus C ABI.

Workload: BASELINE.json configs[3], the Karpathy char-nanoGPT shape (V=65,
L=6, H=6, C=384, T=256, batch 64 per GPU, f32, AdamW lr=1e-3 b2=0.99),
random-init N(0,0.02) weights (seeded Philox, as the reference) and uniform
random token ids from a seed (synthetic; no dataset).  One step = forward +
backward + (N>1: all-reduce of the fused gradient buffer) + AdamW.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl malus|reference]

N>1 runs under torchrun, one process per GPU; per-GPU batch is fixed (weak
scaling); value = all ranks' tokens / max-over-ranks device time.
`--impl reference` times the CPU restatement of the reference's step (the
oracle; the Rust/Metal reference cannot run here) on the host cores.
"""
from __future__ import annotations

import argparse
import ctypes as C
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

C4 = dict(vocab=65, n_layer=6, n_head=6, n_embd=384, block_size=256, batch=64)
# GPT-2-small shape (a parity config of the survey; measured on request, not the contract line)
C5 = dict(vocab=50304, n_layer=12, n_head=12, n_embd=768, block_size=1024, batch=8, tied=True)
WORKLOADS = {"c4": (C4, "C4 Karpathy char-nanoGPT: V65 L6 H6 C384 T256, batch 64/GPU"),
             "c5": (C5, "C5 GPT-2-small shape: V50304 L12 H12 C768 T1024, batch 8/GPU, tied head")}
OPT = dict(lr=1e-3, beta1=0.9, beta2=0.99, eps=1e-8, wd=0.01)
METRIC = "nanoGPT f32 train tokens/s"
PEAKS = ROOT / "MEASURED_PEAKS.json"


def peaks():
    if PEAKS.exists():
        d = json.loads(PEAKS.read_text())
        return d["hbm_gbs"], d["bf16_tflops"], d.get("bf16_tflops_sustained"), "measured"
    return 6650.0, 1590.0, 1400.0, "fallback"


def step_flops(cfg) -> float:
    """Algorithmic matmul FLOPs of one fwd+bwd step (2MNK per GEMM, x3 for bwd)."""
    V, L, H, C_, T, B = (cfg[k] for k in ("vocab", "n_layer", "n_head", "n_embd", "block_size", "batch"))
    M = B * T
    per_layer = 2 * M * C_ * C_ * 4 + 2 * M * C_ * 4 * C_ * 2 + 2 * 2 * B * T * T * C_
    fwd = L * per_layer + 2 * M * C_ * V
    return 3.0 * fwd


class ClockSampler:
    """nvidia-smi clocks/throttle reasons sampled during the timed region."""

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.proc = None
        self.out = None

    def __enter__(self):
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.idx}", f"--query-gpu={q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.lines = []
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except FileNotFoundError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.t.join(timeout=2)

    def summary(self):
        if not self.proc or not self.lines:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                smax = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax,
                "reasons": sorted(reasons), "samples": len(sm)}


def traffic_from_profiles(kernel: str, workload: str, mode: int):
    """DRAM bytes (read + write) per launch of `kernel` from the committed ncu
    capture of this bench command (profiles/roofline_traffic.json).  The capture
    is of the default workload's fused step; other workloads get None."""
    p = ROOT / "profiles" / "roofline_traffic.json"
    if p.exists() and workload == "c4" and mode == 1:
        d = json.loads(p.read_text())
        e = d.get(kernel)
        return e.get("bytes_per_launch") if isinstance(e, dict) else e
    return None


def cpu_baseline_port(cfg, steps=2, sample_batch=8):
    """The oracle (CPU restatement of the reference step) on all host cores."""
    from oracle import pyoracle as O
    threads = O.set_threads(os.cpu_count())
    c = dict(cfg, batch=sample_batch)
    g = O.Gpt(**c, **OPT)
    rng = np.random.default_rng(99)
    m = sample_batch * cfg["block_size"]
    x = rng.integers(0, cfg["vocab"], m).astype(np.int32)
    y = rng.integers(0, cfg["vocab"], m).astype(np.int32)
    g.step(x, y)  # warm-up (allocation, first touch)
    t0 = time.perf_counter()
    for _ in range(steps):
        g.step(x, y)
    dt = time.perf_counter() - t0
    g.close()
    return {"value": steps * m / dt, "unit": "tokens/s", "cores": threads, "kind": "port",
            "sample": f"{steps} steps of the C4 model with batch {sample_batch} x {cfg['block_size']} "
                      f"tokens ({m} tokens/step) on the oracle's OpenMP loops"}


def c2_cpu_ops(threads: int):
    """The C2 op shapes through the oracle (the reference's CPU path restated) on
    `threads` host threads: {op name: seconds} (best of 2 after one warm-up)."""
    from oracle import pyoracle as O
    O.set_threads(threads)
    rng = np.random.default_rng(0)
    n = 8192
    x = rng.standard_normal((n, n), dtype=np.float32)
    y = rng.standard_normal((n, n), dtype=np.float32)
    a = rng.standard_normal((65536, 768), dtype=np.float32)
    g = rng.standard_normal((65536, 768), dtype=np.float32)
    lg = rng.standard_normal((65536, 65), dtype=np.float32)
    tg = rng.integers(0, 65, 65536).astype(np.int32)
    wte = rng.standard_normal((65, 768), dtype=np.float32)
    de = rng.standard_normal((65536, 768), dtype=np.float32)
    pa = rng.standard_normal(10_000_000, dtype=np.float32)
    ga = rng.standard_normal(10_000_000, dtype=np.float32)
    ma, va = np.zeros_like(pa), np.zeros_like(pa)
    sm = O.softmax(a, 1)
    ly, lv = O.layernorm(a, 1)
    _, probs = O.xent(lg, tg)
    cases = {
        "add 8192^2": lambda: O.broadcast(0, x, y),
        "mul 8192^2": lambda: O.broadcast(2, x, y),
        "scalar*tensor 8192^2": lambda: O.broadcast(2, x, np.array([1.5], np.float32)),
        "sigmoid 8192^2": lambda: O.unary("sigmoid", x),
        "gelu 8192^2": lambda: O.unary("gelu", x),
        "exp 8192^2": lambda: O.unary("exp", x),
        "row sum 8192^2": lambda: O.reduce(0, x, 1),
        "col sum 8192^2": lambda: O.reduce(0, x, 0),
        "softmax 65536x768": lambda: O.softmax(a, 1),
        "softmax bwd 65536x768": lambda: O.softmax_bwd(sm, g, 1),
        "layernorm 65536x768": lambda: O.layernorm(a, 1),
        "layernorm bwd 65536x768": lambda: O.layernorm_bwd(ly, lv, g, 1),
        "cross_entropy fwd 65536x65": lambda: O.xent(lg, tg),
        "cross_entropy bwd 65536x65": lambda: O.xent_bwd(probs, tg, 1.0),
        "embedding fwd 65x768, 65536 ids": lambda: O.embedding(wte, tg),
        "embedding bwd 65x768, 65536 ids": lambda: O.embedding_bwd(de, tg, 65),
        "AdamW 10M params": lambda: O.adamw(pa, ga, ma, va, 1e-3, 0.9, 0.95, 1e-8, 0.1, 1),
    }
    out = {}
    for name, fn in cases.items():
        fn()
        best = float("inf")
        for _ in range(2):
            t0 = time.perf_counter()
            fn()
            best = min(best, time.perf_counter() - t0)
        out[name] = best
    return out


def run_ops(args):
    """C2 op microbench: each op on the GPU (CUDA events, median of --reps) beside
    the oracle's CPU path on 1 thread and on all host threads; GB/s = algorithmic
    bytes / time."""
    from malus_b200 import opbench
    rows, peaks = opbench.run(reps=20, verbose=False)
    ncpu = os.cpu_count() or 1
    cpu1 = c2_cpu_ops(1)
    cpun = c2_cpu_ops(ncpu)
    for r in rows:
        if r["op"] in cpu1:
            r["cpu1_gbs"] = round(r["bytes"] / cpu1[r["op"]] / 1e9, 2)
            r["cpun_gbs"] = round(r["bytes"] / cpun[r["op"]] / 1e9, 2)
    print(json.dumps({"metric": "C2 op microbench", "unit": "GB/s", "peaks": peaks, "cpu_threads": ncpu,
                      "ops": rows}))
    print(f"| op | GPU ms | GPU GB/s | of HBM | f32 TF/s (tf32 pipe) | CPU 1-thread GB/s | CPU {ncpu}-thread GB/s |")
    print("|---|---:|---:|---:|---:|---:|---:|")
    for r in rows:
        tf = f"{r['f32_tflops']} ({r['frac_tf32']})" if "f32_tflops" in r else ""
        print(f"| {r['op']} | {r['ms']} | {r['gbs']} | {r['frac_hbm']} | {tf} | {r.get('cpu1_gbs', '')} | "
              f"{r.get('cpun_gbs', '')} |")


def run_reference(args, rank, world):
    if rank != 0:
        return
    from oracle import pyoracle as O
    threads = O.set_threads(os.cpu_count())
    sample_batch = 4
    c = dict(C4, batch=sample_batch)
    g = O.Gpt(**c, **OPT)
    rng = np.random.default_rng(5)
    m = sample_batch * C4["block_size"]
    for _ in range(args.warmup):
        g.step(rng.integers(0, 65, m).astype(np.int32), rng.integers(0, 65, m).astype(np.int32))
    t0 = time.perf_counter()
    for _ in range(args.steps):
        g.step(rng.integers(0, 65, m).astype(np.int32), rng.integers(0, 65, m).astype(np.int32))
    dt = time.perf_counter() - t0
    g.close()
    v = args.steps * m / dt
    line = {"impl": "reference", "metric": METRIC, "value": v, "unit": "tokens/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * dt / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic uniform token ids from a seed; N(0,0.02) Philox init",
            "config": {"workload": "C4 Karpathy char-nanoGPT (V65 L6 H6 C384 T256), CPU sample of "
                                   f"batch {sample_batch} per step", "global_batch": sample_batch,
                       "seq_len": 256, "parallelism": "cpu"},
            "cpu_baseline": {"value": v, "unit": "tokens/s", "cores": threads, "kind": "port",
                             "sample": f"batch {sample_batch} x 256 tokens per step on the oracle "
                                       "(CPU restatement of the reference step; the Rust/Metal "
                                       "reference cannot build or run on this box)"},
            "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="malus", choices=["malus", "reference"])
    ap.add_argument("--mode", type=int, default=int(os.environ.get("MALUS_BENCH_MODE", "1")))
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--ops", action="store_true", help="C2 op microbench (GPU and CPU oracle)")
    ap.add_argument("--workload", default="c4", choices=sorted(WORKLOADS),
                    help="c4 (the contract line) or c5 (GPT-2-small shape, on request)")
    ap.add_argument("--graph", type=int, default=int(os.environ.get("MALUS_BENCH_GRAPH", "1")),
                    help="replay the fused step as one CUDA graph (mode 1)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    if args.ops:
        if rank == 0:
            run_ops(args)
        return

    import torch
    import torch.distributed as dist
    import malus_b200 as M

    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device("cuda", local))
    lib = M.load()
    lib.malus_set_device(local)
    if world > 1:
        from malus_b200.dist import init_data_parallel
        init_data_parallel(lib, rank, world, timeout_ms=120000)

    cfg, workload_name = WORKLOADS[args.workload]
    cfg = dict(cfg)
    model = M.GPT(**cfg, **OPT, mode=args.mode, use_graph=args.graph, seed=0)
    m = cfg["batch"] * cfg["block_size"]
    rng = np.random.default_rng(1000 + rank)
    nb = args.steps + args.warmup
    xs = rng.integers(0, cfg["vocab"], (nb, m)).astype(np.int32)
    ys = rng.integers(0, cfg["vocab"], (nb, m)).astype(np.int32)
    xd = torch.from_numpy(xs).cuda()
    yd = torch.from_numpy(ys).cuda()
    mstream = torch.cuda.ExternalStream(lib.malus_stream())

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(v: float) -> float:
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    for i in range(args.warmup):
        lib.malus_gpt_step_device(model.h, xd[i].data_ptr(), yd[i].data_ptr())
    lib.gpu_barrier()

    # ---------------- device-timed throughput (inputs resident in HBM) ----------------
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)

    def timed_steps():
        barrier()
        torch.cuda.synchronize()
        lib.gpu_barrier()
        ev0.record(mstream)
        for i in range(args.steps):
            j = args.warmup + i
            lib.malus_gpt_step_device(model.h, xd[j].data_ptr(), yd[j].data_ptr())
        ev1.record(mstream)
        lib.gpu_barrier()
        torch.cuda.synchronize()
        return max_over_ranks(ev0.elapsed_time(ev1))

    launches0 = lib.malus_launch_count()
    with ClockSampler(local) as clk:
        dt_ms = timed_steps()
    launches = lib.malus_launch_count() - launches0
    barrier()
    loss_last = lib.malus_gpt_last_loss(model.h)
    value = world * args.steps * m / (dt_ms / 1e3)

    # ---------------- roofline: the same K steps again, every GEMM bracketed by
    # CUDA events on the runtime stream (the events cost a few percent, so the
    # throughput above is taken without them)
    lib.malus_prof_enable(1)
    dt_prof_ms = timed_steps()
    cnt, ms_k, fl_k, by_k = C.c_int64(), C.c_double(), C.c_double(), C.c_double()
    lib.malus_prof_report(0, C.byref(cnt), C.byref(ms_k), C.byref(fl_k), C.byref(by_k))
    lib.malus_prof_enable(0)
    hbm, bf16, bf16_sus, peak_src = peaks()
    roofline = None
    if cnt.value:
        per_launch_ms = ms_k.value / cnt.value
        algo = fl_k.value / cnt.value / (per_launch_ms / 1e3) / 1e12   # 2MNK f32 flops per launch / time
        tf32_peak = 0.5 * (bf16_sus or bf16)            # tf32 runs at half the bf16 rate on tcgen05
        f32_peak = tf32_peak / 3.0                      # 3xTF32: three tf32 products per f32 product
        roofline = {"bound": "tensor", "kernel": "k_gemm_tc (3xTF32 tcgen05)",
                    "achieved": round(algo, 2), "peak": round(f32_peak, 2), "unit": "TFLOP/s",
                    "frac": round(algo / f32_peak, 4),
                    "traffic": traffic_from_profiles("k_gemm_tc", args.workload, args.mode),
                    "algorithmic_bytes_per_launch": round(by_k.value / cnt.value),
                    "launches_per_step": cnt.value / args.steps,
                    "gemm_share_of_step": round(ms_k.value / dt_prof_ms, 4) if world == 1 else None,
                    "executed_tf32_tflops": round(3.0 * algo, 2),
                    "profiled_pass_ms_per_step": round(dt_prof_ms / args.steps, 4),
                    "note": f"achieved = algorithmic f32 2MNK per launch / mean launch time (CUDA events on the "
                            f"runtime stream around every GEMM, over a second pass of the same K steps); "
                            f"peak = {peak_src} sustained bf16 dense ({bf16_sus or bf16}) "
                            "x 1/2 (tf32 rate) / 3 (3xTF32 products per f32 product)"}

    # ---------------- end to end through the public API (host buffers) ----------------
    barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for i in range(args.steps):
        j = (args.warmup + i) % nb
        model.step(xs[j], ys[j])        # H2D ids, step, D2H loss (synchronous)
    e2e_s = max_over_ranks(time.perf_counter() - t0)
    e2e = {"value": world * args.steps * m / e2e_s, "unit": "tokens/s",
           "h2d_bytes_per_step": 2 * m * 4, "d2h_bytes_per_step": 4}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline_port(cfg)

    model.close()
    if world > 1:
        lib.malus_dp_destroy()
    if rank == 0:
        line = {"metric": METRIC, "value": round(value, 1), "unit": "tokens/s", "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dt_ms / args.steps, 4),
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
                "data": f"synthetic: uniform token ids in [0,{cfg['vocab']}) from a seed; N(0,0.02) Philox init",
                "config": {"workload": workload_name,
                           "model": "char-nanoGPT" if args.workload == "c4" else "nanoGPT (GPT-2-small shape)",
                           "global_batch": cfg["batch"] * world,
                           "seq_len": cfg["block_size"], "parallelism": f"dp{world}",
                           "mode": "fused" if args.mode == 1 else "tape",
                           "cuda_graph": bool(args.graph and args.mode == 1),
                           "l2": "working set (activations, several GB) exceeds the 126 MB L2"},
                "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e, "gpu_launches": int(launches),
                "clocks": clk.summary(), "loss_last": loss_last,
                "algorithmic_tflops_per_step": round(step_flops(cfg) / 1e12, 4)}
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
