"""GPU: the plane-level tcgen05 GEMM (malus_tc_gemm) against float64 numpy:
every epilogue, the head fold/unfold output maps, N- and K-segmented
operands, batching, and all four operand major-ness combinations."""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

_LIVE = []


@pytest.fixture(autouse=True)
def _free():
    yield
    _LIVE.clear()


def dev(M, a):
    t = M.Tensor.from_numpy(np.ascontiguousarray(a, np.float32))
    _LIVE.append(t)
    return t


def ptr(lib, t):
    return lib.malus_tensor_data(t.h)


def planes(M, lib, x):
    """x: [nz, rows, cols] or [rows, cols] -> (hi, lo, pitch) device planes."""
    x = np.asarray(x, np.float32)
    if x.ndim == 2:
        x = x[None]
    nz, rows, cols = x.shape
    pitch = (cols + 3) // 4 * 4
    src = dev(M, x)
    hi = dev(M, np.zeros((nz, rows, pitch), np.float32))
    lo = dev(M, np.zeros((nz, rows, pitch), np.float32))
    lib.malus_tf32_split(ptr(lib, src), rows, cols, cols, nz, rows * cols, ptr(lib, hi), ptr(lib, lo), pitch)
    return hi, lo, pitch, nz, rows, cols


def operand(M, lib, x, mn_major, zmode=0, seg=0):
    hi, lo, pitch, nz, rows, cols = planes(M, lib, x)
    return M.TcOperand(ptr(lib, hi), ptr(lib, lo), rows, cols, pitch, nz, rows * pitch,
                       int(mn_major), zmode, seg)


def lay(d1=0, s1=0, d2=0, s2=0, s3=0):
    """index i -> (i//d1)*s1 + ((i%d1)//d2)*s2 + (i%d2)*s3 (d = 0 skips a level)"""
    import malus_b200 as M
    return M.TcLayout(d1, s1, d2, s2, s3)


def run(M, lib, Mm, N, K, batch, a, b, epi=0, oz=None, om=None, on=None, out=None, out_hi=None,
        out_lo=None, aux=None, alpha=1.0, beta=0.0, causal=0):
    p = M.TcProblem()
    p.M, p.N, p.K, p.batch = Mm, N, K, batch
    p.a, p.b = a, b
    p.epi = epi
    p.oz = oz or lay()
    p.om = om or lay(s3=N)
    p.on = on or lay(s3=1)
    p.out = ptr(lib, out) if out is not None else None
    p.out_hi = ptr(lib, out_hi) if out_hi is not None else None
    p.out_lo = ptr(lib, out_lo) if out_lo is not None else None
    p.aux = ptr(lib, aux) if aux is not None else None
    p.alpha, p.beta = alpha, beta
    p.causal = causal
    lib.malus_tc_gemm(C.byref(p))


def err(got, ref, a, b):
    scale = np.abs(a.astype(np.float64)) @ np.abs(b.astype(np.float64))
    return float(np.max(np.abs(got - ref) / np.maximum(scale, 1e-30)))


@pytest.mark.parametrize("a_mn,b_mn", [(False, False), (False, True), (True, False), (True, True)])
@pytest.mark.parametrize("Mm,N,K", [(300, 200, 130), (512, 384, 384), (1024, 65, 384), (129, 1536, 64),
                                    (32, 16, 16), (32, 32, 16), (64, 16, 32), (40, 24, 20),
                                    (3200, 1536, 96)])   # a full grid of 192-wide tiles
def test_majors(M, rt, rng, a_mn, b_mn, Mm, N, K):
    A = rng.standard_normal((Mm, K)).astype(np.float32)
    B = rng.standard_normal((K, N)).astype(np.float32)
    ao = operand(M, rt, A.T if a_mn else A, a_mn)
    bo = operand(M, rt, B if b_mn else B.T, b_mn)
    out = dev(M, np.zeros((Mm, N)))
    run(M, rt, Mm, N, K, 1, ao, bo, out=out)
    ref = A.astype(np.float64) @ B
    assert err(out.numpy(), ref, A, B) < 1e-4


def test_store_beta_and_planes(M, rt, rng):
    A = rng.standard_normal((256, 128)).astype(np.float32)
    B = rng.standard_normal((128, 256)).astype(np.float32)
    C0 = rng.standard_normal((256, 256)).astype(np.float32)
    out = dev(M, C0)
    hi = dev(M, np.zeros((256, 256)))
    lo = dev(M, np.zeros((256, 256)))
    run(M, rt, 256, 256, 128, 1, operand(M, rt, A, False), operand(M, rt, B, True), out=out,
        out_hi=hi, out_lo=lo, alpha=0.5, beta=1.0)
    ref = 0.5 * (A.astype(np.float64) @ B) + C0
    got = out.numpy()
    assert err(got, ref, A, B) < 1e-4
    assert np.max(np.abs(hi.numpy().astype(np.float64) + lo.numpy() - got)) <= 1e-6 * np.max(np.abs(got))


def test_planes_only_output(M, rt, rng):
    """out = NULL: only the tf32 planes of the product are written."""
    A = rng.standard_normal((256, 128)).astype(np.float32)
    B = rng.standard_normal((128, 192)).astype(np.float32)
    hi = dev(M, np.zeros((256, 192)))
    lo = dev(M, np.zeros((256, 192)))
    run(M, rt, 256, 192, 128, 1, operand(M, rt, A, False), operand(M, rt, B, True), out=None,
        out_hi=hi, out_lo=lo)
    got = hi.numpy().astype(np.float64) + lo.numpy()
    assert err(got, A.astype(np.float64) @ B, A, B) < 1e-4


@pytest.mark.parametrize("Mm,N,K", [(384, 512, 128), (3200, 1536, 96)])   # 128- and 192-wide tiles
def test_residual_gelu_gelubwd(M, rt, rng, Mm, N, K):
    A = rng.standard_normal((Mm, K)).astype(np.float32) * 0.5
    B = rng.standard_normal((K, N)).astype(np.float32) * 0.5
    ref = A.astype(np.float64) @ B
    R = rng.standard_normal((Mm, N)).astype(np.float32)
    ao, bo = operand(M, rt, A, False), operand(M, rt, B, True)
    out = dev(M, np.zeros((Mm, N)))
    resid = dev(M, R)
    run(M, rt, Mm, N, K, 1, ao, bo, epi=1, out=out, aux=resid)
    assert err(out.numpy() - R, ref, A, B) < 2e-4
    pre = dev(M, np.zeros((Mm, N)))
    hi, lo = dev(M, np.zeros((Mm, N))), dev(M, np.zeros((Mm, N)))
    run(M, rt, Mm, N, K, 1, ao, bo, epi=2, out=pre, out_hi=hi, out_lo=lo)
    assert err(pre.numpy(), ref, A, B) < 1e-4
    g = 0.5 * ref * (1 + np.tanh(0.7978845608028654 * (ref + 0.044715 * ref ** 3)))
    assert np.max(np.abs(hi.numpy().astype(np.float64) + lo.numpy() - g)) < 1e-4
    X = rng.standard_normal((Mm, N)).astype(np.float32)
    xs = dev(M, X)
    d = dev(M, np.zeros((Mm, N)))
    run(M, rt, Mm, N, K, 1, ao, bo, epi=3, out=d, out_hi=hi, out_lo=lo, aux=xs)
    x = X.astype(np.float64)
    t = np.tanh(0.7978845608028654 * (x + 0.044715 * x ** 3))
    gp = 0.7978845608028654 * (1 + 3 * 0.044715 * x * x)
    dref = ref * (0.5 * (1 + t) + 0.5 * x * (1 - t * t) * gp)
    assert np.max(np.abs(d.numpy() - dref) / (np.abs(A) @ np.abs(B) + 1e-9)) < 2e-4


@pytest.mark.parametrize("Bsz,T,H,hs", [(4, 64, 6, 64), (4, 32, 4, 16)])
def test_qkv_nseg_with_head_fold(M, rt, rng, Bsz, T, H, hs):
    """x[M,C] @ [Wq|Wk|Wv] (three separate [C,C] slices) written as [3][B][H][T][hs]."""
    Cc, Mm = H * hs, Bsz * T
    X = rng.standard_normal((Mm, Cc)).astype(np.float32)
    W = rng.standard_normal((3, Cc, Cc)).astype(np.float32)
    ao = operand(M, rt, X, False)
    bo = operand(M, rt, W, True, zmode=3, seg=Cc)      # MN-major, N segmented over slices
    out = dev(M, np.zeros((3, Bsz, H, T, hs)))
    # m = b*T + t -> b*H*T*hs + t*hs ; n = j*C + h*hs + d -> j*B*H*T*hs + h*T*hs + d
    run(M, rt, Mm, 3 * Cc, Cc, 1, ao, bo, out=out, om=lay(T, H * T * hs, 0, 0, hs),
        on=lay(Cc, Bsz * H * T * hs, hs, T * hs, 1))
    got = out.numpy()
    for j in range(3):
        ref = (X.astype(np.float64) @ W[j]).reshape(Bsz, T, H, hs).transpose(0, 2, 1, 3)
        scale = (np.abs(X.astype(np.float64)) @ np.abs(W[j])).reshape(Bsz, T, H, hs).transpose(0, 2, 1, 3)
        assert np.max(np.abs(got[j] - ref) / scale) < 1e-4
    # N-segmented B into a plain [M, 3C] output
    out2 = dev(M, np.zeros((Mm, 3 * Cc)))
    run(M, rt, Mm, 3 * Cc, Cc, 1, ao, bo, out=out2)
    ref2 = np.concatenate([X.astype(np.float64) @ W[j] for j in range(3)], axis=1)
    Wcat = np.concatenate([W[j] for j in range(3)], axis=1)
    assert err(out2.numpy(), ref2, X, Wcat) < 1e-4


def test_kseg_sum_of_products(M, rt, rng):
    """dx = sum_j dq_j @ W_j^T with dq [3][M][C] and W [3][C][C] as K segments."""
    Mm, Cc = 256, 384
    DQ = rng.standard_normal((3, Mm, Cc)).astype(np.float32)
    W = rng.standard_normal((3, Cc, Cc)).astype(np.float32)
    ao = operand(M, rt, DQ, False, zmode=2, seg=Cc)    # K-major, K segmented
    bo = operand(M, rt, W, False, zmode=2, seg=Cc)     # B^T rows = n: W_j[n][c] K-major
    out = dev(M, np.zeros((Mm, Cc)))
    run(M, rt, Mm, Cc, 3 * Cc, 1, ao, bo, out=out)
    A = np.concatenate([DQ[j] for j in range(3)], axis=1)
    Bm = np.concatenate([W[j].T for j in range(3)], axis=0)
    ref = A.astype(np.float64) @ Bm
    assert err(out.numpy(), ref, A, Bm) < 1e-4


def test_batched_with_unfold(M, rt, rng):
    """P[BH,T,T] @ V[BH,T,hs] written straight into the [B*T, H*hs] layout."""
    Bsz, H, T, hs = 2, 3, 128, 64
    P = rng.standard_normal((Bsz * H, T, T)).astype(np.float32)
    V = rng.standard_normal((Bsz * H, T, hs)).astype(np.float32)
    ao = operand(M, rt, P, False, zmode=1)
    bo = operand(M, rt, V, True, zmode=1)              # V stored [K=T][N=hs]: MN-major
    out = dev(M, np.zeros((Bsz * T, H * hs)))
    # z = b*H + h -> b*T*H*hs + h*hs ; m = t -> t*H*hs ; n = d
    run(M, rt, T, hs, T, Bsz * H, ao, bo, out=out, oz=lay(H, T * H * hs, 0, 0, hs), om=lay(s3=H * hs),
        on=lay(s3=1))
    ref = np.einsum("ztk,zkd->ztd", P.astype(np.float64), V).reshape(Bsz, H, T, hs).transpose(0, 2, 1, 3)
    scale = np.einsum("ztk,zkd->ztd", np.abs(P).astype(np.float64), np.abs(V)).reshape(Bsz, H, T, hs).transpose(0, 2, 1, 3)
    assert np.max(np.abs(out.numpy().reshape(Bsz, T, H, hs) - ref) / scale) < 1e-4


@pytest.mark.parametrize("side", ["a", "b"])
@pytest.mark.parametrize("mn", [False, True])
@pytest.mark.parametrize("seg,nseg", [(64, 3), (96, 3), (32, 5)])
def test_mnseg_tiles_straddle_segments(M, rt, rng, side, mn, seg, nseg):
    """M- or N-segmented operands whose segments are narrower than a 128-wide tile."""
    K, other = 80, 200
    S = rng.standard_normal((nseg, seg, K)).astype(np.float32)    # segment j: rows j*seg.. of the MN x K matrix
    full = np.concatenate(list(S), axis=0)                        # [nseg*seg, K]
    X = rng.standard_normal((other, K)).astype(np.float32)
    stored = np.ascontiguousarray(S.transpose(0, 2, 1)) if mn else S   # MN-major: [K][seg] per segment
    so = operand(M, rt, stored, mn, zmode=3, seg=seg)
    if side == "a":
        xo = operand(M, rt, X.T, True)                            # B: [K][N] MN-major
        Mm, N, A, B = nseg * seg, other, full, X.T
        out = dev(M, np.zeros((Mm, N)))
        run(M, rt, Mm, N, K, 1, so, xo, out=out)
    else:
        xo = operand(M, rt, X, False)                             # A: [M][K] K-major
        Mm, N, A, B = other, nseg * seg, X, full.T
        out = dev(M, np.zeros((Mm, N)))
        run(M, rt, Mm, N, K, 1, xo, so, out=out)
    assert err(out.numpy(), A.astype(np.float64) @ B, A, B) < 1e-4


@pytest.mark.parametrize("Mm,N,K", [(384, 1536, 16384), (65, 384, 16384), (384, 384, 4096), (200, 100, 2000)])
def test_splitk_weight_gradient_shapes(M, rt, rng, Mm, N, K):
    """dW = X^T dY: few output tiles and a long K are computed as K slices; the
    slices are summed in a fixed order, so two runs agree bit for bit."""
    X = rng.standard_normal((K, Mm)).astype(np.float32)
    D = rng.standard_normal((K, N)).astype(np.float32)
    ao = operand(M, rt, X, True)           # A = X^T: X stored [K][M], MN-major
    bo = operand(M, rt, D, True)           # B = dY stored [K][N], MN-major
    out = dev(M, np.zeros((Mm, N)))
    run(M, rt, Mm, N, K, 1, ao, bo, out=out)
    got = out.numpy()
    A = X.T
    assert err(got, A.astype(np.float64) @ D, A, D) < 1e-4
    out2 = dev(M, np.zeros((Mm, N)))
    run(M, rt, Mm, N, K, 1, ao, bo, out=out2)
    assert np.array_equal(got, out2.numpy())


def test_splitk_nseg_output_and_epilogues(M, rt, rng):
    """Split-K with the dWqkv output map (N segments into three [C][C] slices),
    alpha/beta, and the residual / GELU / GELU-backward epilogues."""
    Cc, K = 96, 8192
    X = rng.standard_normal((K, Cc)).astype(np.float32) * 0.1
    D = rng.standard_normal((3, K, Cc)).astype(np.float32) * 0.1
    ao = operand(M, rt, X, True)
    bo = operand(M, rt, D, True, zmode=3, seg=Cc)
    out = dev(M, np.zeros((3, Cc, Cc)))
    run(M, rt, Cc, 3 * Cc, K, 1, ao, bo, out=out, om=lay(s3=Cc), on=lay(Cc, Cc * Cc, 0, 0, 1))
    for j in range(3):
        assert err(out.numpy()[j], X.T.astype(np.float64) @ D[j], X.T, D[j]) < 1e-4
    B = D[0]
    ref = X.T.astype(np.float64) @ B
    bo1 = operand(M, rt, B, True)
    C0 = rng.standard_normal((Cc, Cc)).astype(np.float32)
    o = dev(M, C0)
    run(M, rt, Cc, Cc, K, 1, ao, bo1, out=o, alpha=0.5, beta=2.0)
    assert err(o.numpy() - 2.0 * C0, 0.5 * ref, X.T, B) < 2e-4
    R = dev(M, C0)
    o = dev(M, np.zeros((Cc, Cc)))
    run(M, rt, Cc, Cc, K, 1, ao, bo1, epi=1, out=o, aux=R)
    assert err(o.numpy() - C0, ref, X.T, B) < 2e-4
    hi, lo = dev(M, np.zeros((Cc, Cc))), dev(M, np.zeros((Cc, Cc)))
    run(M, rt, Cc, Cc, K, 1, ao, bo1, epi=2, out=o, out_hi=hi, out_lo=lo)
    g = 0.5 * ref * (1 + np.tanh(0.7978845608028654 * (ref + 0.044715 * ref ** 3)))
    assert np.max(np.abs(hi.numpy().astype(np.float64) + lo.numpy() - g)) < 1e-4 * np.max(np.abs(ref))
    run(M, rt, Cc, Cc, K, 1, ao, bo1, epi=3, out=o, out_hi=hi, out_lo=lo, aux=R)
    x = C0.astype(np.float64)
    t = np.tanh(0.7978845608028654 * (x + 0.044715 * x ** 3))
    gp = 0.7978845608028654 * (1 + 3 * 0.044715 * x * x)
    dref = ref * (0.5 * (1 + t) + 0.5 * x * (1 - t * t) * gp)
    scale = (np.abs(X.T).astype(np.float64) @ np.abs(B)) * np.max(np.abs(0.5 * (1 + t) + 0.5 * x * (1 - t * t) * gp))
    assert np.max(np.abs(o.numpy() - dref) / scale) < 2e-4


def test_splitk_batched(M, rt, rng):
    """Batched problems with one tile each and a long K also take K slices."""
    Z, Mm, N, K = 3, 64, 48, 4096
    A = rng.standard_normal((Z, Mm, K)).astype(np.float32)
    B = rng.standard_normal((Z, K, N)).astype(np.float32)
    ao = operand(M, rt, A, False, zmode=1)
    bo = operand(M, rt, B, True, zmode=1)
    out = dev(M, np.zeros((Z, Mm, N)))
    run(M, rt, Mm, N, K, Z, ao, bo, out=out, oz=lay(s3=Mm * N))
    for z in range(Z):
        assert err(out.numpy()[z], A[z].astype(np.float64) @ B[z], A[z], B[z]) < 1e-4


@pytest.mark.parametrize("T,hs", [(256, 64), (200, 48), (384, 32)])
@pytest.mark.parametrize("a_mn", [False, True])
def test_causal_triangular_a(M, rt, rng, T, hs, a_mn):
    """Attention-shaped batched GEMMs whose A is triangular: the K range stops at
    (lower) or starts from (upper) the diagonal; results equal the full product."""
    Z = 3
    for mode, tri in ((2, np.tril), (3, np.triu)):
        A = tri(rng.standard_normal((Z, T, T)).astype(np.float32))
        B = rng.standard_normal((Z, T, hs)).astype(np.float32)
        ao = operand(M, rt, A.transpose(0, 2, 1) if a_mn else A, a_mn, zmode=1)
        bo = operand(M, rt, B, True, zmode=1)
        out = dev(M, np.zeros((Z, T, hs)))
        run(M, rt, T, hs, T, Z, ao, bo, out=out, oz=lay(s3=T * hs), om=lay(s3=hs), causal=mode)
        for z in range(Z):
            assert err(out.numpy()[z], A[z].astype(np.float64) @ B[z], A[z], B[z]) < 1e-4, mode


@pytest.mark.parametrize("T", [256, 200, 384])
def test_causal_output_tiles(M, rt, rng, T):
    """Only tiles reaching the lower triangle are computed; every element on or
    below the diagonal is exact, and skipped tiles are left untouched."""
    Z, hs = 2, 64
    Q = rng.standard_normal((Z, T, hs)).astype(np.float32)
    Kt = rng.standard_normal((Z, T, hs)).astype(np.float32)
    qo = operand(M, rt, Q, False, zmode=1)
    ko = operand(M, rt, Kt, False, zmode=1)
    sentinel = np.full((Z, T, T), 7.0, np.float32)
    out = dev(M, sentinel)
    run(M, rt, T, T, hs, Z, qo, ko, out=out, oz=lay(s3=T * T), om=lay(s3=T), alpha=0.125, causal=1)
    got = out.numpy()
    low = np.tril(np.ones((T, T), bool))
    for z in range(Z):
        ref = 0.125 * (Q[z].astype(np.float64) @ Kt[z].T)
        scale = 0.125 * (np.abs(Q[z]).astype(np.float64) @ np.abs(Kt[z]).T)
        assert np.max((np.abs(got[z] - ref) / scale)[low]) < 1e-4
        for tm in range(0, T, 128):
            for tn in range(0, T, 128):
                if tn > tm + 127:
                    assert np.all(got[z, tm:tm + 128, tn:tn + 128] == 7.0)


def test_softmax_backward_epilogue(M, rt, rng):
    """dS = scale * P * (dO V^T - D) in the GEMM epilogue, P read from its tf32
    planes, D per row, causal tiles only (the fused attention backward)."""
    Z, T, hs, scale = 3, 256, 64, 0.125
    S = rng.standard_normal((Z, T, T)) + np.triu(np.full((T, T), -np.inf), 1)
    P = np.exp(S - S.max(-1, keepdims=True))
    P = (P / P.sum(-1, keepdims=True)).astype(np.float32)
    dO = rng.standard_normal((Z, T, hs)).astype(np.float32)
    V = rng.standard_normal((Z, T, hs)).astype(np.float32)
    D = np.einsum("ztd,ztd->zt", dO.astype(np.float64), np.einsum("ztk,zkd->ztd", P.astype(np.float64), V))
    p_hi, p_lo, _, _, _, _ = planes(M, rt, P)
    Dd = dev(M, D.astype(np.float32))
    hi, lo = dev(M, np.zeros((Z, T, T))), dev(M, np.zeros((Z, T, T)))
    p = M.TcProblem()
    p.M, p.N, p.K, p.batch = T, T, hs, Z
    p.a, p.b = operand(M, rt, dO, False, zmode=1), operand(M, rt, V, False, zmode=1)
    p.epi = 4
    p.oz, p.om, p.on = lay(s3=T * T), lay(s3=T), lay(s3=1)
    p.out_hi, p.out_lo = ptr(rt, hi), ptr(rt, lo)
    p.aux, p.aux_lo, p.rowv = ptr(rt, p_hi), ptr(rt, p_lo), ptr(rt, Dd)
    p.alpha, p.beta, p.causal = scale, 0.0, 1
    rt.malus_tc_gemm(C.byref(p))
    got = hi.numpy().astype(np.float64) + lo.numpy()
    dP = np.einsum("ztd,zkd->ztk", dO.astype(np.float64), V)
    ref = scale * P * (dP - D[..., None])
    bound = scale * P * (np.einsum("ztd,zkd->ztk", np.abs(dO).astype(np.float64), np.abs(V)) + np.abs(D)[..., None])
    low = np.tril(np.ones((T, T), bool))
    assert np.max((np.abs(got - ref) / np.maximum(bound, 1e-30))[:, low]) < 1e-5


def test_splitk_256_wide_tiles_epilogues(M, rt, rng):
    """Split-K problem with N % 256 == 0 (the 256-wide tile): plain store,
    residual, GELU (f32 + planes) and GELU-backward epilogues after the
    deterministic reduction."""
    Mm, N, K = 256, 512, 8192
    A = rng.standard_normal((K, Mm)).astype(np.float32) * 0.1
    B = rng.standard_normal((K, N)).astype(np.float32) * 0.1
    ao, bo = operand(M, rt, A, True), operand(M, rt, B, True)
    ref = A.T.astype(np.float64) @ B
    out = dev(M, np.zeros((Mm, N)))
    run(M, rt, Mm, N, K, 1, ao, bo, out=out)
    assert err(out.numpy(), ref, A.T, B) < 1e-4
    R = rng.standard_normal((Mm, N)).astype(np.float32)
    rs = dev(M, R)
    run(M, rt, Mm, N, K, 1, ao, bo, epi=1, out=out, aux=rs)
    assert err(out.numpy() - R, ref, A.T, B) < 2e-4
    hi, lo = dev(M, np.zeros((Mm, N))), dev(M, np.zeros((Mm, N)))
    run(M, rt, Mm, N, K, 1, ao, bo, epi=2, out=out, out_hi=hi, out_lo=lo)
    g = 0.5 * ref * (1 + np.tanh(0.7978845608028654 * (ref + 0.044715 * ref ** 3)))
    assert np.max(np.abs(hi.numpy().astype(np.float64) + lo.numpy() - g)) < 1e-4 * np.max(np.abs(ref))
    run(M, rt, Mm, N, K, 1, ao, bo, epi=3, out=out, out_hi=hi, out_lo=lo, aux=rs)
    x = R.astype(np.float64)
    t = np.tanh(0.7978845608028654 * (x + 0.044715 * x ** 3))
    gp = 0.7978845608028654 * (1 + 3 * 0.044715 * x * x)
    dref = ref * (0.5 * (1 + t) + 0.5 * x * (1 - t * t) * gp)
    assert np.max(np.abs(out.numpy() - dref) / (np.abs(A.T) @ np.abs(B) + 1e-9)) < 2e-4


@pytest.mark.parametrize("lo_first", [False, True])
@pytest.mark.parametrize("a_mn,b_mn", [(False, True), (True, False), (False, False)])
def test_paired_plane_loads_either_order(M, rt, rng, lo_first, a_mn, b_mn):
    """Both planes of an operand in one buffer, hi then lo or lo then hi: the
    paired-plane load (one box per stage for both planes, based at the lower
    address) must put each plane where the MMA reads it."""
    Mm, N, K = 1024, 1536, 96

    def op_in_one_buffer(x, mn):
        rows, cols = x.shape
        both = dev(M, np.zeros((2, rows, cols)))
        src = dev(M, x)
        base = ptr(rt, both)
        first, second = base, base + rows * cols * 4
        hi, lo = (second, first) if lo_first else (first, second)
        rt.malus_tf32_split(ptr(rt, src), rows, cols, cols, 1, rows * cols, hi, lo, cols)
        return M.TcOperand(hi, lo, rows, cols, cols, 1, rows * cols, int(mn), 0, 0)

    A = rng.standard_normal((Mm, K)).astype(np.float32)
    B = rng.standard_normal((K, N)).astype(np.float32)
    ao = op_in_one_buffer(np.ascontiguousarray(A.T) if a_mn else A, a_mn)
    bo = op_in_one_buffer(B if b_mn else np.ascontiguousarray(B.T), b_mn)
    out = dev(M, np.zeros((Mm, N)))
    run(M, rt, Mm, N, K, 1, ao, bo, out=out)
    assert err(out.numpy(), A.astype(np.float64) @ B, A, B) < 1e-4


# ---- CTA pairs: problems whose M is whole 256-row tiles, unsplit and
# non-causal, run as 2-CTA clusters (one M = 256 MMA per k-step, each CTA
# loading its 128 rows of A and half of the tile's B columns).  These tests
# put the GEMM in pair mode 1 (every eligible shape as pairs, whatever the
# epilogue and K) and pick shapes that are eligible: 192-wide tiles (full
# grid), 128-wide tiles with depth 32, ragged N and K edges, batching, segments.
@pytest.fixture
def pairs_all(rt):
    assert rt.malus_gemm_pair_clusters() > 0
    prev = rt.malus_gemm_pair_mode(1)
    yield
    rt.malus_gemm_pair_mode(prev)


@pytest.mark.parametrize("a_mn,b_mn", [(False, False), (False, True), (True, False), (True, True)])
@pytest.mark.parametrize("Mm,N,K", [(4096, 1152, 384), (1024, 1536, 96), (512, 200, 72)])
def test_pair_majors(M, rt, rng, pairs_all, a_mn, b_mn, Mm, N, K):
    A = rng.standard_normal((Mm, K)).astype(np.float32)
    B = rng.standard_normal((K, N)).astype(np.float32)
    ao = operand(M, rt, A.T if a_mn else A, a_mn)
    bo = operand(M, rt, B if b_mn else B.T, b_mn)
    out = dev(M, np.zeros((Mm, N)))
    run(M, rt, Mm, N, K, 1, ao, bo, out=out)
    assert err(out.numpy(), A.astype(np.float64) @ B, A, B) < 1e-4


def test_pair_epilogues(M, rt, rng, pairs_all):
    """Residual add (192 x 16 tiles) and GELU / GELU backward with tf32 output
    planes (192 x 32 tiles) on 256-row pair tiles."""
    test_residual_gelu_gelubwd(M, rt, rng, 4096, 1536, 96)


def test_pair_batched(M, rt, rng, pairs_all):
    Z, Mm, N, K = 6, 256, 128, 256
    A = rng.standard_normal((Z, Mm, K)).astype(np.float32)
    B = rng.standard_normal((Z, K, N)).astype(np.float32)
    ao = operand(M, rt, A, False, zmode=1)
    bo = operand(M, rt, B, True, zmode=1)              # [K][N] per batch: MN-major
    out = dev(M, np.zeros((Z, Mm, N)))
    run(M, rt, Mm, N, K, Z, ao, bo, out=out, oz=lay(s3=Mm * N))
    ref = np.einsum("zmk,zkn->zmn", A.astype(np.float64), B)
    scale = np.einsum("zmk,zkn->zmn", np.abs(A).astype(np.float64), np.abs(B))
    assert np.max(np.abs(out.numpy() - ref) / scale) < 1e-4


@pytest.mark.parametrize("side", ["a", "b"])
@pytest.mark.parametrize("mn", [False, True])
def test_pair_mnseg(M, rt, rng, pairs_all, side, mn):
    """Segmented operands on pair tiles: B's 96-wide segments straddle the two
    CTAs' 64-column halves; A's 96-row segments straddle the 128-row halves."""
    K, seg = 80, 96
    nseg = 8 if side == "a" else 3
    other = 200 if side == "a" else 512
    S = rng.standard_normal((nseg, seg, K)).astype(np.float32)
    full = np.concatenate(list(S), axis=0)
    X = rng.standard_normal((other, K)).astype(np.float32)
    stored = np.ascontiguousarray(S.transpose(0, 2, 1)) if mn else S
    so = operand(M, rt, stored, mn, zmode=3, seg=seg)
    if side == "a":
        xo = operand(M, rt, X.T, True)
        Mm, N, A, B = nseg * seg, other, full, X.T
        out = dev(M, np.zeros((Mm, N)))
        run(M, rt, Mm, N, K, 1, so, xo, out=out)
    else:
        xo = operand(M, rt, X, False)
        Mm, N, A, B = other, nseg * seg, X, full.T
        out = dev(M, np.zeros((Mm, N)))
        run(M, rt, Mm, N, K, 1, xo, so, out=out)
    assert err(out.numpy(), A.astype(np.float64) @ B, A, B) < 1e-4


def test_pair_clusters_resident(M, rt):
    """On a B200 every TPC can hold one CTA pair of the GEMM: 74 pairs (148 SMs)."""
    n = rt.malus_gemm_pair_clusters()
    assert 1 <= n <= 74


def test_pair_mode_hook(M, rt):
    prev = rt.malus_gemm_pair_mode(0)
    try:
        assert rt.malus_gemm_pair_clusters() == 0
        assert rt.malus_gemm_pair_mode(7) == 0        # any other value selects the measured rule
        assert rt.malus_gemm_pair_mode(-1) == -1
    finally:
        rt.malus_gemm_pair_mode(prev)


@pytest.mark.parametrize("mode", [0, 1])
def test_pair_mode_same_result(M, rt, rng, mode):
    """The same product as pairs and as single CTAs agrees to the tf32x3 error
    (the per-element arithmetic is the same; only the CTA that computes a row
    changes)."""
    A = rng.standard_normal((2048, 384)).astype(np.float32)
    B = rng.standard_normal((384, 1152)).astype(np.float32)
    ao, bo = operand(M, rt, A, False), operand(M, rt, B, True)
    outs = []
    prev = rt.malus_gemm_pair_mode(mode)
    try:
        for m in (mode, 1 - mode):
            rt.malus_gemm_pair_mode(m)
            out = dev(M, np.zeros((2048, 1152)))
            run(M, rt, 2048, 1152, 384, 1, ao, bo, out=out)
            outs.append(out.numpy())
    finally:
        rt.malus_gemm_pair_mode(prev)
    assert np.array_equal(outs[0], outs[1])
