"""Per-op microbenchmark (the C2 op shapes of the benchmark configs) through the C ABI.

Each op runs on seeded N(0,1) inputs of the configured shape; the timing is
the median of `--reps` launches bracketed by CUDA events on the runtime's own
stream, after one warm-up, and the inputs (>= 17 MB, mostly far above the
126 MB L2 for the 8192^2 ops) are reused across repetitions.  Achieved GB/s =
algorithmic bytes (one read of each input, one write of each output) / time;
GEMM rows report f32-algorithmic TFLOP/s (2MNK) and the executed tf32 rate
(3x for 3xTF32).

  python -m malus_b200.opbench [--only NAME] [--reps N] [--json]
"""
from __future__ import annotations

import argparse
import ctypes as C
import json
import statistics
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))
import malus_b200 as M  # noqa: E402

F = 4


def _peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d["hbm_gbs"], d["bf16_tflops"] * 0.5, "measured"
    return 6650.0, 795.0, "fallback"


class Bench:
    def __init__(self, reps):
        import torch
        self.torch = torch
        self.lib = M.load()
        self.reps = reps
        self.stream = torch.cuda.ExternalStream(self.lib.malus_stream())
        self.keep = []

    def T(self, a):
        t = M.Tensor.from_numpy(a)
        self.keep.append(t)
        return t

    def time(self, fn):
        torch = self.torch
        out = fn()
        if out:
            self.lib.tensor_release(out)
        self.lib.gpu_barrier()
        ts = []
        for _ in range(self.reps):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(self.stream)
            out = fn()
            e1.record(self.stream)
            self.lib.gpu_barrier()
            ts.append(e0.elapsed_time(e1))
            if out:
                self.lib.tensor_release(out)
        return statistics.median(ts)


def cases(b: Bench, rng):
    lib = b.lib
    n = 8192
    x = b.T(rng.standard_normal((n, n), dtype=np.float32))
    y = b.T(rng.standard_normal((n, n), dtype=np.float32))
    s = b.T(np.array([0.5], np.float32))
    E = n * n * F
    ids = (C.c_uint64 * 3)(7001, 7002, 7003)
    nm = (C.c_char_p * 3)(b"malus_mul_scalar", b"sigmoid", b"exp")
    lib.malus_runtime_init(ids, nm, 3)
    yield "add 8192^2", lambda: lib.__broadcast_add_fwd(x.h, y.h), 3 * E, 0
    yield "mul 8192^2", lambda: lib.__broadcast_mul_fwd(x.h, y.h), 3 * E, 0
    yield "scalar*tensor 8192^2", lambda: lib.kernel_dispatch(7001, (C.c_int64 * 2)(x.h, s.h), 2), 2 * E, 0
    yield "sigmoid 8192^2", lambda: lib.kernel_dispatch(7002, (C.c_int64 * 1)(x.h), 1), 2 * E, 0
    yield "gelu 8192^2", lambda: lib.__gelu_fwd(x.h), 2 * E, 0
    yield "exp 8192^2", lambda: lib.kernel_dispatch(7003, (C.c_int64 * 1)(x.h), 1), 2 * E, 0
    yield "row sum 8192^2", lambda: lib.__reduce_sum_fwd(x.h, 1, 0), E + n * F, 0
    yield "col sum 8192^2", lambda: lib.__reduce_sum_fwd(x.h, 0, 0), E + n * F, 0
    r, c = 65536, 768
    a = b.T(rng.standard_normal((r, c), dtype=np.float32))
    g = b.T(rng.standard_normal((r, c), dtype=np.float32))
    yield "softmax 65536x768", lambda: lib.__softmax_fwd(a.h, 1), 2 * r * c * F, 0
    sm = M.Tensor(lib.__softmax_fwd(a.h, 1))
    b.keep.append(sm)
    yield "softmax bwd 65536x768", lambda: lib.__softmax_bwd(sm.h, g.h, 1), 3 * r * c * F, 0
    # the attention scores of the reference's call sequence at C4: (QK^T * scale) + causal
    # mask, deferred, read by the softmax ([384, 256, 256]; the mask stays in L2)
    z, t = 384, 256
    qk = b.T(rng.standard_normal((z, t, t), dtype=np.float32))
    sc1 = b.T(np.array([[0.125]], np.float32))
    mask = b.T(np.where(np.arange(t)[None, :] > np.arange(t)[:, None], -1e9, 0).astype(np.float32))
    scaled = lib.__broadcast_mul_fwd(qk.h, sc1.h)
    masked = M.Tensor(lib.__broadcast_add_fwd(scaled, mask.h))
    lib.tensor_release(scaled)
    b.keep.append(masked)
    yield "softmax (x*s+mask deferred) 98304x256", lambda: lib.__softmax_fwd(masked.h, 2), 2 * z * t * t * F, 0
    yield "softmax 98304x256", lambda: lib.__softmax_fwd(qk.h, 2), 2 * z * t * t * F, 0

    def ln():
        box = lib.__layernorm_fwd(a.h, 1)
        yh, vh = M.tuple_fields(box)
        lib.tensor_release(vh)
        return yh
    yield "layernorm 65536x768", ln, 2 * r * c * F + r * F, 0
    box = lib.__layernorm_fwd(a.h, 1)
    yh, vh = M.tuple_fields(box)
    yt, vt = M.Tensor(yh), M.Tensor(vh)
    b.keep += [yt, vt]
    yield "layernorm bwd 65536x768", lambda: lib.__layernorm_bwd(yt.h, vt.h, g.h, 1), 3 * r * c * F, 0
    nt, v = 65536, 65
    lg = b.T(rng.standard_normal((nt, v), dtype=np.float32))
    tg = b.T(rng.integers(0, v, nt).astype(np.int32))

    def xent():
        box = lib.__cross_entropy_fwd(lg.h, tg.h)
        lh, ph = M.tuple_fields(box)
        lib.tensor_release(ph)
        return lh
    yield "cross_entropy fwd 65536x65", xent, 2 * nt * v * F + nt * 4, 0
    box = lib.__cross_entropy_fwd(lg.h, tg.h)
    lh, ph = M.tuple_fields(box)
    lt, pt = M.Tensor(lh), M.Tensor(ph)
    one = b.T(np.array([1.0], np.float32))
    b.keep += [lt, pt]
    yield "cross_entropy bwd 65536x65", lambda: lib.__cross_entropy_bwd(pt.h, tg.h, one.h), 2 * nt * v * F + nt * 4, 0
    wte = b.T(rng.standard_normal((65, 768), dtype=np.float32))
    eid = b.T(rng.integers(0, 65, 65536).astype(np.int32))
    de = b.T(rng.standard_normal((65536, 768), dtype=np.float32))
    yield "embedding fwd 65x768, 65536 ids", lambda: lib.__embedding_fwd(wte.h, eid.h), 65536 * 768 * F + 65536 * 4, 0
    yield "embedding bwd 65x768, 65536 ids", lambda: lib.__embedding_bwd(wte.h, eid.h, de.h), 65536 * 768 * F + 65536 * 4 + 65 * 768 * F, 0
    npar = 10_000_000
    arrs = [b.T(rng.standard_normal(npar, dtype=np.float32)) for _ in range(2)] + \
           [b.T(np.zeros(npar, np.float32)) for _ in range(2)]
    hp = lambda i: (C.c_int64 * 1)(arrs[i].h)

    def adamw():
        lib.malus_adamw_multi(hp(0), hp(1), hp(2), hp(3), 1, 1e-3, 0.9, 0.95, 1e-8, 0.1, 1, 1.0)
        return 0
    yield "AdamW 10M params", adamw, 7 * npar * F, 0
    # GEMM shapes of the C4 step (M = 64*256 tokens)
    for (mm, kk, nn, label) in [(16384, 384, 384, "QKV/O proj"), (16384, 384, 1536, "MLP up"),
                                (16384, 1536, 384, "MLP down"), (16384, 384, 65, "LM head")]:
        A = b.T(rng.standard_normal((mm, kk), dtype=np.float32))
        W = b.T(rng.standard_normal((kk, nn), dtype=np.float32))
        yield f"matmul {mm}x{kk}x{nn} ({label})", (lambda A=A, W=W: lib.tensor_matmul(A.h, W.h)), \
            (mm * kk + kk * nn + mm * nn) * F, 2.0 * mm * nn * kk
    yield from plane_cases(b, rng)
    Q = b.T(rng.standard_normal((384, 256, 64), dtype=np.float32))
    Kt = b.T(rng.standard_normal((384, 64, 256), dtype=np.float32))
    yield "bmm 384x256x64x256 (QK^T)", lambda: lib.tensor_matmul(Q.h, Kt.h), \
        (2 * 384 * 256 * 64 + 384 * 256 * 256) * F, 2.0 * 384 * 256 * 256 * 64


def plane_cases(b: Bench, rng):
    """The fused step's GEMMs at the C4 shapes, on pre-split tf32 planes through
    malus_tc_gemm (operands and outputs exactly as the step lays them out)."""
    lib = b.lib
    Mt, Cc, H, T, hs = 16384, 384, 6, 256, 64
    C4, Bz = 4 * Cc, 64

    def buf(*shape, rand=True):
        a = rng.standard_normal(shape, dtype=np.float32) * 0.1 if rand else np.zeros(shape, np.float32)
        return lib.malus_tensor_data(b.T(a).h)

    def op(rows, cols, mn, nz=1, zmode=0, seg=0):
        return M.TcOperand(buf(nz, rows, cols), buf(nz, rows, cols), rows, cols, cols, nz, rows * cols,
                           int(mn), zmode, seg)

    def L(d1=0, s1=0, d2=0, s2=0, s3=0):
        return M.TcLayout(d1, s1, d2, s2, s3)

    def prob(Mm, N, K, batch, a, bb, epi=0, oz=None, om=None, on=None, out=False, planes=False, aux=False,
             alpha=1.0):
        q = M.TcProblem()
        q.M, q.N, q.K, q.batch, q.a, q.b, q.epi = Mm, N, K, batch, a, bb, epi
        q.oz, q.om, q.on = oz or L(), om or L(s3=N), on or L(s3=1)
        n_out = Mm * N * batch
        q.out = buf(n_out, rand=False) if out else None
        if planes:
            q.out_hi, q.out_lo = buf(n_out, rand=False), buf(n_out, rand=False)
        q.aux = buf(n_out) if aux else None
        q.alpha, q.beta = alpha, 0.0
        return q

    def run(q):
        lib.malus_tc_gemm(C.byref(q))
        return 0

    def nbytes(q, Mm, N, K, batch, n_out_arrays, aux):
        return (8 * (Mm * K + N * K) * batch + 4 * Mm * N * batch * (n_out_arrays + int(aux)))

    cases_ = [
        ("tc QKV (planes out, head fold)", prob(Mt, 3 * Cc, Cc, 1, op(Mt, Cc, False),
                                                op(Cc, Cc, True, 3, 3, Cc), planes=True,
                                                om=L(T, H * T * hs, 0, 0, hs),
                                                on=L(Cc, Bz * H * T * hs, hs, T * hs, 1)), (Mt, 3 * Cc, Cc, 1, 2, False)),
        ("tc attn S=QK^T (f32 out)", prob(T, T, hs, Bz * H, op(T, hs, False, Bz * H, 1),
                                          op(T, hs, False, Bz * H, 1), out=True, oz=L(s3=T * T),
                                          om=L(s3=T), alpha=0.125), (T, T, hs, Bz * H, 1, False)),
        ("tc attn O=PV (planes, unfold)", prob(T, hs, T, Bz * H, op(T, T, False, Bz * H, 1),
                                               op(T, hs, True, Bz * H, 1), planes=True,
                                               oz=L(H, T * Cc, 0, 0, hs), om=L(s3=Cc)), (T, hs, T, Bz * H, 2, False)),
        ("tc proj + residual", prob(Mt, Cc, Cc, 1, op(Mt, Cc, False), op(Cc, Cc, True), epi=1, out=True,
                                    aux=True), (Mt, Cc, Cc, 1, 1, True)),
        ("tc MLP up + GELU", prob(Mt, C4, Cc, 1, op(Mt, Cc, False), op(Cc, C4, True), epi=2, out=True,
                                  planes=True), (Mt, C4, Cc, 1, 3, False)),
        ("tc MLP down + residual", prob(Mt, Cc, C4, 1, op(Mt, C4, False), op(C4, Cc, True), epi=1,
                                        out=True, aux=True), (Mt, Cc, C4, 1, 1, True)),
        ("tc GELU backward", prob(Mt, C4, Cc, 1, op(Mt, Cc, False), op(C4, Cc, False), epi=3, planes=True,
                                  aux=True), (Mt, C4, Cc, 1, 2, True)),
        ("tc dW1 = xn^T dh (split-K)", prob(Cc, C4, Mt, 1, op(Mt, Cc, True), op(Mt, C4, True), out=True),
         (Cc, C4, Mt, 1, 1, False)),
    ]
    for name, q, (Mm, N, K, batch, nout, aux) in cases_:
        yield name, (lambda q=q: run(q)), nbytes(q, Mm, N, K, batch, nout, aux), 2.0 * Mm * N * K * batch
    # fused causal attention at the C4 shape: q|k|v planes in, O planes and row
    # statistics out (the step's form; P planes are not written)
    qh, ql = buf(3, Bz, H, T, hs), buf(3, Bz, H, T, hs)
    oh, ol = buf(Mt, Cc, rand=False), buf(Mt, Cc, rand=False)
    st = buf(Bz * H * T, 2, rand=False)

    def attn():
        lib.malus_attn_fwd(qh, ql, Bz, H, T, hs, C.c_float(0.125), None, None, oh, ol, st)
        return 0
    causal = 0.5 * (1 + 128 / T)   # score entries up to each query's 128-wide tile
    yield ("attn fwd fused (causal, C4)", attn,
           8 * 3 * Mt * Cc + 8 * Mt * Cc + 8 * Bz * H * T,
           2.0 * 2 * Bz * H * T * T * hs * 0.5)
    # the fused step's form at T = 256: P planes written for the GEMM backward
    # (score entries up to each query's 128-wide tile)
    ph, pl = buf(Bz * H, T, T, rand=False), buf(Bz * H, T, T, rand=False)
    pbytes = 8 * Bz * H * T * T * causal

    def attn_p():
        lib.malus_attn_fwd(qh, ql, Bz, H, T, hs, C.c_float(0.125), ph, pl, oh, ol, st)
        return 0

    def attn_p_recompute():
        prev = lib.malus_attn_set_resident(0)
        attn_p()
        lib.malus_attn_set_resident(prev)
        return 0
    yield ("attn fwd fused + P planes (C4 step)", attn_p,
           8 * 3 * Mt * Cc + 8 * Mt * Cc + 8 * Bz * H * T + pbytes,
           2.0 * 2 * Bz * H * T * T * hs * 0.5)
    yield ("attn fwd + P planes, scores recomputed", attn_p_recompute,
           8 * 3 * Mt * Cc + 8 * Mt * Cc + 8 * Bz * H * T + pbytes,
           2.0 * 2 * Bz * H * T * T * hs * 0.5)
    # backward: dq | dk | dv planes from q|k|v, dO and O planes and the statistics
    dh, dl = buf(Bz * H, T, hs), buf(Bz * H, T, hs)
    dw = buf(Bz * H * T, rand=False)
    gh, gl = buf(3, Mt, Cc, rand=False), buf(3, Mt, Cc, rand=False)
    attn()
    lib.gpu_barrier()

    def attn_bwd():
        lib.malus_attn_bwd(qh, ql, dh, dl, oh, ol, st, dw, Bz, H, T, hs, C.c_float(0.125), gh, gl)
        return 0
    yield ("attn bwd fused (causal, C4)", attn_bwd,
           8 * 3 * Mt * Cc + 8 * 2 * Mt * Cc + 8 * 3 * Mt * Cc + 12 * Bz * H * T,
           2.0 * 5 * Bz * H * T * T * hs * 0.5)


def run(only: str | None = None, reps: int = 20, verbose: bool = True) -> tuple[list[dict], dict]:
    """Time every case (or those whose name contains `only`); returns (rows, peaks)."""
    hbm, tf32, src = _peaks()
    b = Bench(reps)
    rng = np.random.default_rng(0)
    rows = []
    for name, fn, nbytes, flops in cases(b, rng):
        if only and only not in name:
            continue
        ms = b.time(fn)
        row = {"op": name, "ms": round(ms, 4), "bytes": nbytes, "gbs": round(nbytes / ms / 1e6, 1),
               "frac_hbm": round(nbytes / ms / 1e6 / hbm, 3)}
        if flops:
            row["flops"] = flops
            row["f32_tflops"] = round(flops / ms / 1e9, 1)
            row["tf32_executed_tflops"] = round(3 * flops / ms / 1e9, 1)
            row["frac_tf32"] = round(3 * flops / ms / 1e9 / tf32, 3)
        rows.append(row)
        if verbose:
            print(f"{name:42s} {ms:9.4f} ms  {row['gbs']:8.1f} GB/s ({row['frac_hbm']:.2f} of HBM)"
                  + (f"  {row['f32_tflops']:6.1f} f32-TF/s, tf32 pipe {row['frac_tf32']:.2f}" if flops else ""),
                  flush=True)
    return rows, {"hbm_gbs": hbm, "tf32_tflops": tf32, "source": src}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--only", default=None)
    ap.add_argument("--reps", type=int, default=20)
    ap.add_argument("--json", action="store_true")
    args = ap.parse_args()
    rows, peaks = run(args.only, args.reps, verbose=not args.json)
    if args.json:
        print(json.dumps({"peaks": peaks, "ops": rows}))


if __name__ == "__main__":
    main()
