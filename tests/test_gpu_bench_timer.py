"""GPU: the warm-median step timer bench_step_begin / bench_step_end /
bench_report (crates/malus-runtime/src/bench.rs:12-70).

Semantics checked: dormant until bench_enable (begin/end record nothing); a
step is host-clock time from begin to end, and end waits for the GPU inside
the timed region; an end without a begin records nothing; the report is the
median of the steps after the first three (mean of the middle two for an even
count), -1 with fewer than four steps; bench_report_range gives the same
steps' min and max; bench_reset disables the timer and forgets the steps."""
import ctypes as C
import time

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def report(rt):
    n = C.c_int64()
    med = rt.bench_report(C.byref(n))
    lo, hi = C.c_double(), C.c_double()
    rt.bench_report_range(C.byref(lo), C.byref(hi))
    return med, n.value, lo.value, hi.value


def step(rt, seconds):
    rt.bench_step_begin()
    time.sleep(seconds)
    rt.bench_step_end()


def test_dormant_until_enabled(rt):
    rt.bench_reset()
    for _ in range(6):
        step(rt, 0.001)
    assert report(rt)[:2] == (-1.0, 0)


def test_warm_median_and_range(rt):
    rt.bench_reset()
    rt.bench_enable()
    for _ in range(3):
        step(rt, 0.060)                     # warm-up steps: excluded
    rt.bench_step_end()                     # an end without a begin: nothing recorded
    for s in (0.010, 0.040, 0.020, 0.030):
        step(rt, s)
    med, n, lo, hi = report(rt)
    assert n == 4
    assert 25.0 <= med < 25.0 + 8.0          # (20 + 30) / 2 ms, plus call overhead
    assert 10.0 <= lo < 18.0 and 40.0 <= hi < 48.0
    step(rt, 0.050)                          # odd count: the middle step
    med, n, _, _ = report(rt)
    assert n == 5 and 30.0 <= med < 38.0
    rt.bench_reset()
    assert report(rt)[:2] == (-1.0, 0)
    step(rt, 0.001)                          # reset also disabled the timer
    assert report(rt)[:2] == (-1.0, 0)


def test_step_end_waits_for_the_gpu(M, rt):
    """Work queued inside the step (asynchronous on the runtime stream) is
    inside the timed region: the recorded step is at least as long as the same
    work timed alone with a host synchronisation."""
    a = M.Tensor.from_numpy(np.random.default_rng(0).standard_normal((8192, 8192), dtype=np.float32))
    b = M.Tensor.from_numpy(np.random.default_rng(1).standard_normal((8192, 8192), dtype=np.float32))

    def work():
        outs = [rt.tensor_matmul(a.h, b.h) for _ in range(4)]
        return outs

    for h in work():
        rt.tensor_release(h)
    rt.gpu_barrier()
    t0 = time.perf_counter()
    outs = work()
    rt.gpu_barrier()
    alone_ms = 1e3 * (time.perf_counter() - t0)
    for h in outs:
        rt.tensor_release(h)

    rt.bench_reset()
    rt.bench_enable()
    for _ in range(4):
        rt.bench_step_begin()
        outs = work()
        rt.bench_step_end()
        for h in outs:
            rt.tensor_release(h)
    med, n, _, _ = report(rt)
    rt.bench_reset()
    assert n == 1
    assert med >= 0.8 * alone_ms, (med, alone_ms)
