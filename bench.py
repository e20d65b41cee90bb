#!/usr/bin/env python
"""nanoGPT f32 training throughput (tokens/s) on B200 through the malus C ABI.

Workload: benchmark config C4, the Karpathy char-nanoGPT shape (V=65,
L=6, H=6, C=384, T=256, batch 64 per GPU, f32, AdamW lr=1e-3 b2=0.99),
random-init N(0,0.02) weights (seeded Philox, as the reference) and uniform
random token ids from a seed (synthetic; no dataset).  One step = forward +
backward + (N>1: all-reduce of the fused gradient buffer) + AdamW.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl malus|reference]

The headline `value` is the compiled step (mode 1, one CUDA graph per step).
At N=1 the same line also carries
  * `tape`: the reference's own call sequence (examples/nanogpt_modular.ml
    through RuntimeSymbols, the stdlib host functions and the tape, mode 0),
    captured once as a CUDA graph and replayed, on the same C4 workload;
  * `c5`: the GPT-2-small shape (config C5) through the compiled step.
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
# GPT-2-small shape (a parity config of the survey; measured as the line's `c5` object)
C5 = dict(vocab=50304, n_layer=12, n_head=12, n_embd=768, block_size=1024, batch=8, tied=True)
WORKLOADS = {"c4": (C4, "C4 Karpathy char-nanoGPT: V65 L6 H6 C384 T256, batch 64/GPU"),
             "c5": (C5, "C5 GPT-2-small shape: V50304 L12 H12 C768 T1024, batch 8/GPU, tied head")}
OPT = dict(lr=1e-3, beta1=0.9, beta2=0.99, eps=1e-8, wd=0.01)
METRIC = "nanoGPT f32 train tokens/s"
PEAKS = ROOT / "MEASURED_PEAKS.json"
# sequences per CPU step (both CPU legs): 2048 of the 16384 tokens of a C4 step
# (MALUS_BENCH_CPU_BATCH shrinks it for the CPU test suite)
CPU_SAMPLE_BATCH = int(os.environ.get("MALUS_BENCH_CPU_BATCH", "8"))
L2_NOTE = "working set (activations, several GB) exceeds the 126 MB L2"


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


def workload_config(workload: str, world: int) -> dict:
    """The `config` object of both arms' lines (same keys and values)."""
    cfg, name = WORKLOADS[workload]
    return {"workload": name,
            "model": "char-nanoGPT" if workload == "c4" else "nanoGPT (GPT-2-small shape)",
            "global_batch": cfg["batch"] * world, "seq_len": cfg["block_size"],
            "parallelism": f"dp{world}", "l2": L2_NOTE}


class ClockSampler:
    """nvidia-smi clocks/throttle reasons sampled every 50 ms while under load."""

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.proc = None
        self.lines = []

    def __enter__(self):
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.idx}", f"--query-gpu={q}",
                                          "--format=csv,noheader,nounits", "-lms", "50"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
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
                "reasons": sorted(reasons), "samples": len(sm), "period_ms": 50}


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


def _oracle_tokens_per_s(cfg, threads: int, steps: int, warmup: int, seed: int):
    """Time `steps` oracle training steps (batch CPU_SAMPLE_BATCH of the C4
    model) on `threads` host threads; returns (tokens/s, seconds, threads used)."""
    from oracle import pyoracle as O
    used = O.set_threads(threads)
    c = dict(cfg, batch=CPU_SAMPLE_BATCH)
    g = O.Gpt(**c, **OPT)
    rng = np.random.default_rng(seed)
    m = CPU_SAMPLE_BATCH * cfg["block_size"]

    def ids():
        return rng.integers(0, cfg["vocab"], m).astype(np.int32)

    for _ in range(warmup):
        g.step(ids(), ids())
    t0 = time.perf_counter()
    for _ in range(steps):
        g.step(ids(), ids())
    dt = time.perf_counter() - t0
    g.close()
    return steps * m / dt, dt, used


def cpu_baseline_port(cfg, steps=2):
    """The oracle (CPU restatement of the reference step) on all host cores, and
    one step on a single thread beside it."""
    v, _, threads = _oracle_tokens_per_s(cfg, os.cpu_count() or 1, steps, 1, 99)
    v1, dt1, _ = _oracle_tokens_per_s(cfg, 1, 1, 0, 98)
    m = CPU_SAMPLE_BATCH * cfg["block_size"]
    return {"value": v, "unit": "tokens/s", "cores": threads, "kind": "port",
            "sample": f"{steps} steps of the C4 model with batch {CPU_SAMPLE_BATCH} x {cfg['block_size']} "
                      f"tokens ({m} tokens/step) on the oracle's OpenMP loops",
            "single_thread": {"value": v1, "unit": "tokens/s", "cores": 1,
                              "sample": f"1 step of batch {CPU_SAMPLE_BATCH} on one thread ({dt1:.1f} s)"}}


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
    rows, peaks_ = opbench.run(reps=20, verbose=False)
    ncpu = os.cpu_count() or 1
    cpu1 = c2_cpu_ops(1)
    cpun = c2_cpu_ops(ncpu)
    for r in rows:
        if r["op"] in cpu1:
            r["cpu1_gbs"] = round(r["bytes"] / cpu1[r["op"]] / 1e9, 2)
            r["cpun_gbs"] = round(r["bytes"] / cpun[r["op"]] / 1e9, 2)
    print(json.dumps({"metric": "C2 op microbench", "unit": "GB/s", "peaks": peaks_, "cpu_threads": ncpu,
                      "ops": rows}))
    print(f"| op | GPU ms | GPU GB/s | of HBM | f32 TF/s (tf32 pipe) | CPU 1-thread GB/s | CPU {ncpu}-thread GB/s |")
    print("|---|---:|---:|---:|---:|---:|---:|")
    for r in rows:
        tf = f"{r['f32_tflops']} ({r['frac_tf32']})" if "f32_tflops" in r else ""
        print(f"| {r['op']} | {r['ms']} | {r['gbs']} | {r['frac_hbm']} | {tf} | {r.get('cpu1_gbs', '')} | "
              f"{r.get('cpun_gbs', '')} |")


def run_reference(args, rank, world):
    """The reference arm: the oracle step (the reference's CPU path restated) on
    all host threads, on rank 0 only; each step is a batch-8 sample of the C4
    step.  A single-thread step is timed beside it."""
    if rank != 0:
        return
    v, dt, threads = _oracle_tokens_per_s(C4, os.cpu_count() or 1, args.steps, args.warmup, 5)
    v1, dt1, _ = _oracle_tokens_per_s(C4, 1, 1, 0, 6)
    m = CPU_SAMPLE_BATCH * C4["block_size"]
    line = {"impl": "reference", "metric": METRIC, "value": v, "unit": "tokens/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * dt / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic uniform token ids from a seed; N(0,0.02) Philox init",
            "config": workload_config("c4", world),
            "cpu_baseline": {"value": v, "unit": "tokens/s", "cores": threads, "kind": "port",
                             "sample": f"each step: batch {CPU_SAMPLE_BATCH} x 256 tokens ({m} of the C4 step's "
                                       "16384) on the oracle (CPU restatement of the reference step; the "
                                       "Rust/Metal reference cannot build or run on this box)",
                             "single_thread": {"value": v1, "unit": "tokens/s", "cores": 1,
                                               "sample": f"1 step of batch {CPU_SAMPLE_BATCH} on one thread "
                                                         f"({dt1:.1f} s)"}},
            "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


class Runner:
    """Times one (workload, mode) on this rank's GPU: the device-timed pass with
    inputs resident, an optional profiled pass for the GEMM roofline, and the
    end-to-end pass through malus_gpt_step with host ids."""

    def __init__(self, lib, torch, dist, world, rank):
        self.lib, self.torch, self.dist, self.world, self.rank = lib, torch, dist, world, rank
        self.mstream = torch.cuda.ExternalStream(lib.malus_stream())

    def barrier(self):
        if self.world > 1:
            self.dist.barrier()

    def max_over_ranks(self, v: float) -> float:
        if self.world == 1:
            return v
        t = self.torch.tensor([v], dtype=self.torch.float64, device="cuda")
        self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return float(t.item())

    def measure(self, workload, mode, graph, steps, warmup, roofline=True, clocks=None):
        import malus_b200 as M
        torch, lib = self.torch, self.lib
        cfg = dict(WORKLOADS[workload][0])
        model = M.GPT(**cfg, **OPT, mode=mode, use_graph=graph, seed=0)
        m = cfg["batch"] * cfg["block_size"]
        rng = np.random.default_rng(1000 + self.rank)
        nb = steps + warmup
        xs = rng.integers(0, cfg["vocab"], (nb, m)).astype(np.int32)
        ys = rng.integers(0, cfg["vocab"], (nb, m)).astype(np.int32)
        xd = torch.from_numpy(xs).cuda()
        yd = torch.from_numpy(ys).cuda()
        for i in range(warmup):
            lib.malus_gpt_step_device(model.h, xd[i].data_ptr(), yd[i].data_ptr())
        lib.gpu_barrier()
        ev0 = torch.cuda.Event(enable_timing=True)
        ev1 = torch.cuda.Event(enable_timing=True)

        def timed_steps():
            self.barrier()
            torch.cuda.synchronize()
            lib.gpu_barrier()
            ev0.record(self.mstream)
            for i in range(steps):
                j = warmup + i
                lib.malus_gpt_step_device(model.h, xd[j].data_ptr(), yd[j].data_ptr())
            ev1.record(self.mstream)
            lib.gpu_barrier()
            torch.cuda.synchronize()
            return self.max_over_ranks(ev0.elapsed_time(ev1))

        launches0 = lib.malus_launch_count()
        if clocks is not None:
            clocks.__enter__()
        dt_ms = timed_steps()
        launches = lib.malus_launch_count() - launches0
        self.barrier()
        loss_last = lib.malus_gpt_last_loss(model.h)
        out = {"value": round(self.world * steps * m / (dt_ms / 1e3), 1),
               "ms_per_step": round(dt_ms / steps, 4), "gpu_launches": int(launches),
               "loss_last": loss_last}

        # roofline: the same K steps again, every GEMM bracketed by CUDA events on
        # the runtime stream (the events cost a few percent, so `value` is taken
        # without them)
        if roofline:
            lib.malus_prof_enable(1)
            dt_prof_ms = timed_steps()
            cnt, ms_k, fl_k, by_k = C.c_int64(), C.c_double(), C.c_double(), C.c_double()
            lib.malus_prof_report(0, C.byref(cnt), C.byref(ms_k), C.byref(fl_k), C.byref(by_k))
            if self.world > 1:
                out["dp"] = self._dp_report(lib, steps, dt_prof_ms)
            out["kernels"] = self._kernel_table(lib, steps, dt_prof_ms)
            lib.malus_prof_enable(0)
            out["roofline"] = self._gemm_roofline(cnt.value, ms_k.value, fl_k.value, by_k.value, dt_prof_ms,
                                                  steps, workload, mode)

        # end to end through the public API (host ids in, host loss out)
        self.barrier()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for i in range(steps):
            j = (warmup + i) % nb
            model.step(xs[j], ys[j])        # H2D ids, step, D2H loss (synchronous)
        e2e_s = self.max_over_ranks(time.perf_counter() - t0)
        if clocks is not None:
            clocks.__exit__(None, None, None)
        out["e2e"] = {"value": self.world * steps * m / e2e_s, "unit": "tokens/s",
                      "h2d_bytes_per_step": 2 * m * 4, "d2h_bytes_per_step": 4}
        model.close()
        del xd, yd
        torch.cuda.empty_cache()
        return out

    def _kernel_table(self, lib, steps, dt_prof_ms):
        """The compiled step's non-GEMM kernels from the profiled pass: per label,
        launches and ms per step, share of the step, and achieved GB/s =
        algorithmic bytes (one read of each input, one write of each output) /
        CUDA-event time, as a fraction of the measured HBM copy peak."""
        need = lib.malus_prof_kernels(None, 0)
        if need <= 0:
            return []
        buf = C.create_string_buffer(need + 1)
        lib.malus_prof_kernels(buf, need + 1)
        hbm = peaks()[0]
        rows = []
        for ln in buf.value.decode().splitlines():
            name, n, ms, by = ln.split("\t")
            n, ms, by = int(n), float(ms), float(by)
            gbs = by / (ms / 1e3) / 1e9 if ms else 0.0
            rows.append({"kernel": name, "launches_per_step": n / steps, "ms_per_step": round(ms / steps, 4),
                         "share_of_step": round(ms / dt_prof_ms, 4), "gbs": round(gbs, 1),
                         "frac_hbm": round(gbs / hbm, 3)})
        return sorted(rows, key=lambda r: -r["ms_per_step"])

    def _dp_report(self, lib, steps, dt_prof_ms):
        """The gradient all-reduces of the profiled pass (this rank): their time on
        the collective stream, the part the main stream waited for at the join
        (not hidden by the backward pass), and the bus bandwidth NCCL reached."""
        n, ms, _, by = C.c_int64(), C.c_double(), C.c_double(), C.c_double()
        lib.malus_prof_report(3, C.byref(n), C.byref(ms), None, C.byref(by))
        nj, msj = C.c_int64(), C.c_double()
        lib.malus_prof_report(4, C.byref(nj), C.byref(msj), None, None)
        w = self.world
        bus = 2.0 * (w - 1) / w * by.value / (ms.value / 1e3) / 1e9 if ms.value else None
        return {"allreduce_calls_per_step": n.value / steps,
                "allreduce_ms_per_step": round(ms.value / steps, 4),
                "exposed_ms_per_step": round(msj.value / steps, 4),
                "payload_mb_per_step": round(by.value / steps / 1e6, 2),
                "bus_gbs": round(bus, 1) if bus else None,
                "profiled_step_ms": round(dt_prof_ms / steps, 4),
                "note": "rank 0's profiled pass (eager): allreduce_ms_per_step spans each all-reduce on the "
                        "collective stream from its gradients being ready to its completion, overlapped with the "
                        "backward (bus_gbs is payload over that span, so it reflects contention for SMs, not "
                        "link bandwidth); exposed_ms_per_step is the main stream's wait at the join"}

    def _gemm_roofline(self, cnt, ms_k, fl_k, by_k, dt_prof_ms, steps, workload, mode):
        if not cnt:
            return None
        _, bf16, bf16_sus, peak_src = peaks()
        per_launch_ms = ms_k / cnt
        algo = fl_k / cnt / (per_launch_ms / 1e3) / 1e12   # 2MNK f32 flops per launch / time
        # tf32 runs at half the bf16 rate on tcgen05; 3xTF32 issues three tf32
        # products per f32 product.  `peak` uses the burst bf16 figure (the
        # GEMMs run at full clock in the short timed region); the sustained
        # (power-capped, seconds-long) figure is reported beside it.
        f32_burst = 0.5 * bf16 / 3.0
        f32_sus = 0.5 * (bf16_sus or bf16) / 3.0
        return {"bound": "tensor", "kernel": "k_gemm_tc (3xTF32 tcgen05)",
                "achieved": round(algo, 2), "peak": round(f32_burst, 2), "unit": "TFLOP/s",
                "frac": round(algo / f32_burst, 4), "frac_burst": round(algo / f32_burst, 4),
                "frac_sustained": round(algo / f32_sus, 4),
                "peak_sustained": round(f32_sus, 2),
                "traffic": traffic_from_profiles("k_gemm_tc", workload, mode),
                "algorithmic_bytes_per_launch": round(by_k / cnt),
                "launches_per_step": cnt / steps,
                "gemm_share_of_step": round(ms_k / dt_prof_ms, 4) if self.world == 1 else None,
                "executed_tf32_tflops": round(3.0 * algo, 2),
                "profiled_pass_ms_per_step": round(dt_prof_ms / steps, 4),
                "note": f"achieved = algorithmic f32 2MNK per launch / mean launch time (CUDA events on the "
                        f"runtime stream around every GEMM, over a second pass of the same K steps); "
                        f"peak = {peak_src} burst bf16 dense ({bf16}) x 1/2 (tf32 rate) / 3 (3xTF32 "
                        f"products per f32 product); peak_sustained the same from the sustained figure "
                        f"({bf16_sus})"}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="malus", choices=["malus", "reference"])
    ap.add_argument("--mode", type=int, default=int(os.environ.get("MALUS_BENCH_MODE", "1")),
                    help="headline path: 1 compiled step, 0 the reference's call sequence (tape)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extras", action="store_true", help="skip the `tape` and `c5` objects")
    ap.add_argument("--ops", action="store_true", help="C2 op microbench (GPU and CPU oracle)")
    ap.add_argument("--workload", default="c4", choices=sorted(WORKLOADS),
                    help="headline workload: c4 (the contract line) or c5")
    ap.add_argument("--graph", type=int, default=int(os.environ.get("MALUS_BENCH_GRAPH", "1")),
                    help="replay each step as one CUDA graph")
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

    run = Runner(lib, torch, dist, world, rank)
    clk = ClockSampler(local)
    head = run.measure(args.workload, args.mode, args.graph, args.steps, args.warmup, roofline=True, clocks=clk)
    extras = {}
    if world == 1 and not args.no_extras:
        if not (args.workload == "c4" and args.mode == 0):
            t = run.measure("c4", 0, 1, args.steps, args.warmup, roofline=False)
            t["path"] = ("the reference's call sequence (nanogpt_modular.ml through RuntimeSymbols, stdlib "
                         "host functions, tape backward, AdamW), captured once as a CUDA graph and replayed")
            t["of_headline"] = round(t["value"] / head["value"], 4) if args.workload == "c4" else None
            extras["tape"] = t
        if args.workload != "c5":
            c5 = run.measure("c5", 1, 1, max(3, min(args.steps, 20)), 3, roofline=True)
            c5["config"] = workload_config("c5", world)
            extras["c5"] = c5

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline_port(C4 if args.workload == "c4" else C5)

    if world > 1:
        lib.malus_dp_destroy()
    if rank == 0:
        cfg = WORKLOADS[args.workload][0]
        line = {"metric": METRIC, "value": head["value"], "unit": "tokens/s", "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": head["ms_per_step"],
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
                "data": f"synthetic: uniform token ids in [0,{cfg['vocab']}) from a seed; N(0,0.02) Philox init",
                "config": workload_config(args.workload, world),
                "path": {"mode": "fused" if args.mode == 1 else "tape", "cuda_graph": bool(args.graph)},
                "roofline": head.get("roofline"), "cpu_baseline": cpu, "e2e": head["e2e"],
                "gpu_launches": head["gpu_launches"], "clocks": clk.summary(), "loss_last": head["loss_last"],
                **({"dp": head["dp"]} if "dp" in head else {}),
                **({"kernels": head["kernels"]} if head.get("kernels") else {}),
                "algorithmic_tflops_per_step": round(step_flops(cfg) / 1e12, 4), **extras}
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
