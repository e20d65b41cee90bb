"""GPU parity: every kernel behind the C ABI against the CPU oracle on seeded
inputs.  Tolerances (the parity bars of this path): gather/indexing bit-exact;
elementwise and reductions <= 1e-5 relative (reductions normalised by
sum|x|, the bound of the reference's own sequential f32 order); matmul
<= 1e-4 relative normalised by sum_k |a_ik * b_kj|."""
import ctypes as C

import numpy as np
import pytest

from conftest import rel_err

pytestmark = pytest.mark.gpu


_LIVE = []  # keeps inline-created tensors alive until the test ends


@pytest.fixture(autouse=True)
def _release_live():
    yield
    _LIVE.clear()


def T(M, a):
    t = M.Tensor.from_numpy(np.asarray(a))
    _LIVE.append(t)
    return t


def H(M, h):
    t = M.Tensor(h)
    _LIVE.append(t)
    return t


def sarr(shape):
    return (C.c_size_t * max(1, len(shape)))(*shape), len(shape)


# ------------------------------------------------------------ elementwise
@pytest.mark.parametrize("op,fn", [(0, "__broadcast_add_fwd"), (1, "__broadcast_sub_fwd"),
                                   (2, "__broadcast_mul_fwd"), (3, "__broadcast_div_fwd")])
@pytest.mark.parametrize("sa,sb", [((1001,), (1001,)), ((64, 384), (384,)), ((384,), (64, 384)),
                                   ((24, 16, 16), (16, 16)), ((24, 16, 16), (1, 1)),
                                   ((4, 8), (8,)), ((1, 4), (3, 4)), ((33, 1), (33, 7)),
                                   ((5, 1, 3), (1, 4, 1)), ((0, 3), (3,))])
def test_broadcast_binops(M, rt, orc, rng, op, fn, sa, sb):
    a = rng.standard_normal(sa).astype(np.float32)
    b = rng.standard_normal(sb).astype(np.float32)
    if op == 3:
        b = np.where(np.abs(b) < 0.1, 0.5, b).astype(np.float32)
    ta, tb_ = T(M, a), T(M, b)
    out = H(M, getattr(rt, fn)(ta.h, tb_.h))
    ref = orc.broadcast(op, a, b)
    got = out.numpy()
    assert got.shape == ref.shape
    np.testing.assert_array_equal(got, ref)  # IEEE add/sub/mul/div: bit-exact


def test_broadcast_golden_cases(M, rt):
    out = H(M, rt.__broadcast_add_fwd(T(M, np.ones((4, 8), np.float32)).h,
                                      T(M, np.arange(1, 9, dtype=np.float32)).h))
    assert np.all(out.numpy() == np.arange(2, 10, dtype=np.float32)[None])
    out = H(M, rt.__broadcast_sub_fwd(T(M, np.array([[1, 2, 3, 4]], np.float32)).h,
                                      T(M, np.ones((3, 4), np.float32)).h))
    assert out.numpy().shape == (3, 4) and np.all(out.numpy() == np.array([0, 1, 2, 3], np.float32))


UNARY = ["relu", "sigmoid", "tanh", "exp", "log", "sqrt", "abs"]


@pytest.mark.parametrize("name", UNARY)
def test_unary_builtins_via_kernel_dispatch(M, rt, orc, rng, name):
    ids = (C.c_uint64 * 1)(100 + UNARY.index(name))
    nm = (C.c_char_p * 1)(name.encode())
    rt.malus_runtime_init(ids, nm, 1)
    x = rng.standard_normal(4099).astype(np.float32) * 3
    if name in ("log", "sqrt"):
        x = np.abs(x) + 0.01
    tx = T(M, x)
    hs = (C.c_int64 * 1)(tx.h)
    out = H(M, rt.kernel_dispatch(100 + UNARY.index(name), hs, 1)).numpy()
    ref = orc.unary(name, x)
    assert rel_err(out, ref, np.maximum(np.abs(ref), 1.0)) < 1e-5   # rtol = atol = 1e-5


@pytest.mark.parametrize("name,op", [("malus_add_scalar", lambda x, s: x + s),
                                     ("malus_sub_scalar", lambda x, s: x - s),
                                     ("malus_rsub_scalar", lambda x, s: s - x),
                                     ("malus_mul_scalar", lambda x, s: x * s),
                                     ("malus_div_scalar", lambda x, s: x / s),
                                     ("malus_rdiv_scalar", lambda x, s: s / x)])
def test_scalar_builtins(M, rt, rng, name, op):
    kid = 200 + abs(hash(name)) % 1000
    rt.malus_runtime_init((C.c_uint64 * 1)(kid), (C.c_char_p * 1)(name.encode()), 1)
    x = (rng.standard_normal(1027) + 3).astype(np.float32)
    s = np.array([0.35355], np.float32)
    tx, ts = T(M, x), T(M, s)
    out = H(M, rt.kernel_dispatch(kid, (C.c_int64 * 2)(tx.h, ts.h), 2)).numpy()
    np.testing.assert_array_equal(out, op(x, s[0]).astype(np.float32))


def test_same_shape_builtins(M, rt, rng):
    rt.malus_runtime_init((C.c_uint64 * 2)(300, 301), (C.c_char_p * 2)(b"malus_add", b"malus_div"), 2)
    a = rng.standard_normal(515).astype(np.float32)
    b = rng.standard_normal(515).astype(np.float32) + 5
    ta, tb_ = T(M, a), T(M, b)
    np.testing.assert_array_equal(H(M, rt.kernel_dispatch(300, (C.c_int64 * 2)(ta.h, tb_.h), 2)).numpy(), a + b)
    np.testing.assert_array_equal(H(M, rt.kernel_dispatch(301, (C.c_int64 * 2)(ta.h, tb_.h), 2)).numpy(), a / b)


@pytest.mark.parametrize("name,fn,pos", [("sigmoid", "__sigmoid_bwd", True), ("relu", "__relu_bwd", False),
                                         ("tanh", "__tanh_bwd", True), ("sqrt", "__sqrt_bwd", True),
                                         ("abs", "__abs_bwd", False), ("gelu", "__gelu_bwd", False)])
def test_unary_vjps(M, rt, orc, rng, name, fn, pos):
    x = rng.standard_normal(3001).astype(np.float32)
    if pos:
        x = (np.abs(x) * 0.4 + 0.05).astype(np.float32)
    g = rng.standard_normal(3001).astype(np.float32)
    out = H(M, getattr(rt, fn)(T(M, x).h, T(M, g).h)).numpy()
    ref = orc.unary_bwd(name, x, g)
    assert rel_err(out, ref, np.maximum(np.abs(ref), 1.0)) < 1e-5   # rtol = atol = 1e-5


def test_gelu_forward(M, rt, orc, rng):
    x = (rng.standard_normal((64, 1536)) * 2).astype(np.float32)
    out = H(M, rt.__gelu_fwd(T(M, x).h)).numpy()
    ref = orc.unary("gelu", x)
    assert rel_err(out, ref, np.maximum(np.abs(ref), 1.0)) < 1e-5   # rtol = atol = 1e-5


# ------------------------------------------------------------ reductions
@pytest.mark.parametrize("shape,axis", [((2, 3), 0), ((2, 3), 1), ((257, 513), 0), ((257, 513), 1),
                                        ((16384, 384), 0), ((8, 8192), 1), ((8192, 8), 0),
                                        ((6, 5, 7), 1), ((3, 2100), 1), ((1, 70000), 1), ((5,), 0)])
@pytest.mark.parametrize("op,fn", [(0, "__reduce_sum_fwd"), (1, "__reduce_mean_fwd"),
                                   (2, "__reduce_max_fwd"), (3, "__reduce_var_fwd")])
def test_reductions(M, rt, orc, rng, shape, axis, op, fn):
    x = rng.standard_normal(shape).astype(np.float32)
    for keep in (0, 1):
        out = H(M, getattr(rt, fn)(T(M, x).h, axis, keep)).numpy()
        ref = orc.reduce(op, x, axis, bool(keep))
        assert out.shape == ref.shape
        if op == 2:
            np.testing.assert_array_equal(out, ref)
        elif op == 3:
            assert rel_err(out, ref, np.maximum(np.abs(ref), 1e-3)) < 1e-4
        else:
            n = shape[axis]
            scale = np.sum(np.abs(x), axis=axis, keepdims=bool(keep)).reshape(ref.shape)
            if op == 1:
                scale = scale / n
            assert rel_err(out, ref, scale) < 1e-5


def test_reduce_all_sum(M, rt, rng):
    for n in (1, 7, 1024, 100003):
        x = rng.standard_normal(n).astype(np.float32)
        out = H(M, rt.__reduce_all_sum_fwd(T(M, x).h)).numpy()
        assert out.shape == (1,)
        assert abs(float(out[0]) - float(np.sum(x.astype(np.float64)))) <= 1e-5 * float(np.sum(np.abs(x)))


# --------------------------------------------------------- softmax / LN
@pytest.mark.parametrize("shape,axis", [((24, 64, 64), 2), ((4, 256, 256), 2), ((300, 65), 1),
                                        ((8, 50304), 1), ((3, 2000), 1), ((5, 7, 3), 1), ((7, 9), 0)])
def test_softmax_fwd_bwd(M, rt, orc, rng, shape, axis):
    x = (rng.standard_normal(shape) * 3).astype(np.float32)
    s = H(M, rt.__softmax_fwd(T(M, x).h, axis))
    ref = orc.softmax(x, axis)
    # long rows: the reference's sequential f32 sum itself drifts ~n*eps, so the
    # bar is an f64 evaluation (the oracle is checked against it at its own bound)
    x64 = x.astype(np.float64)
    e = np.exp(x64 - x64.max(axis=axis, keepdims=True))
    ref64 = e / e.sum(axis=axis, keepdims=True)
    assert rel_err(s.numpy(), ref64, np.max(ref64)) < 1e-5
    assert rel_err(ref, ref64, np.max(ref64)) < 1e-7 * shape[axis]
    g = rng.standard_normal(shape).astype(np.float32)
    dx = H(M, rt.__softmax_bwd(s.h, T(M, g).h, axis)).numpy()
    dref = orc.softmax_bwd(s.numpy(), g, axis)
    scale = np.max(np.abs(ref * g)) + 1e-6
    assert rel_err(dx, dref, scale) < 1e-5


def test_softmax_masked_rows(M, rt, rng):
    # causal masking with -1e9 must give exact zeros above the diagonal
    T_ = 32
    x = rng.standard_normal((2, T_, T_)).astype(np.float32)
    x = x + np.triu(np.full((T_, T_), -1e9, np.float32), 1)
    s = H(M, rt.__softmax_fwd(T(M, x).h, 2)).numpy()
    assert np.all(s[:, np.triu_indices(T_, 1)[0], np.triu_indices(T_, 1)[1]] == 0)


@pytest.mark.parametrize("shape,axis", [((64, 128), 1), ((1024, 384), 1), ((16, 768), 1),
                                        ((9, 1000), 1), ((5, 2500), 1), ((6, 10), 0), ((2, 5), 1)])
def test_layernorm_fwd_bwd(M, rt, orc, rng, shape, axis):
    x = (rng.standard_normal(shape) * 2 + 0.5).astype(np.float32)
    box = rt.__layernorm_fwd(T(M, x).h, axis)
    yh, vh = M.tuple_fields(box)
    y, var = H(M, yh), H(M, vh)
    yref, vref = orc.layernorm(x, axis)
    assert var.numpy().shape == vref.shape
    assert rel_err(y.numpy(), yref, np.maximum(np.abs(yref), 1.0)) < 1e-5
    assert rel_err(var.numpy(), vref) < 1e-5
    g = rng.standard_normal(shape).astype(np.float32)
    dx = H(M, rt.__layernorm_bwd(y.h, var.h, T(M, g).h, axis)).numpy()
    dref = orc.layernorm_bwd(yref, vref, g, axis)
    assert rel_err(dx, dref, np.max(np.abs(dref))) < 1e-5


# --------------------------------------------------------- cross-entropy
@pytest.mark.parametrize("n,v,dt", [(64, 65, np.int32), (1000, 65, np.int64), (16, 50304, np.int32),
                                    (3, 1500, np.int32)])
def test_cross_entropy(M, rt, orc, rng, n, v, dt):
    logits = (rng.standard_normal((n, v)) * 2).astype(np.float32)
    t = rng.integers(0, v, n).astype(dt)
    box = rt.__cross_entropy_fwd(T(M, logits).h, T(M, t).h)
    lh, ph = M.tuple_fields(box)
    loss, probs = H(M, lh), H(M, ph)
    lref, pref = orc.xent(logits, t.astype(np.int32))
    assert abs(float(loss.numpy()[0]) - float(lref[0])) <= 1e-5 * abs(float(lref[0]))
    assert rel_err(probs.numpy(), pref, np.max(pref)) < 1e-5
    dout = np.array([0.7], np.float32)
    dx = H(M, rt.__cross_entropy_bwd(probs.h, T(M, t).h, T(M, dout).h)).numpy()
    dref = orc.xent_bwd(pref, t.astype(np.int32), 0.7)
    assert rel_err(dx, dref, np.max(np.abs(dref))) < 1e-5


# ---------------------------------------------------------------- embedding
@pytest.mark.parametrize("dt", [np.int32, np.int64])
def test_embedding_golden(M, rt, dt):
    w = np.arange(12, dtype=np.float32).reshape(4, 3)
    idx = np.array([1, 0, 2], dt)
    out = H(M, rt.__embedding_fwd(T(M, w).h, T(M, idx).h)).numpy()
    np.testing.assert_array_equal(out.ravel(), w[idx].ravel())
    dw = H(M, rt.__embedding_bwd(T(M, np.ones((4, 2), np.float32)).h,
                                 T(M, np.array([0, 2, 1, 0], dt)).h,
                                 T(M, np.ones((4, 2), np.float32)).h)).numpy()
    np.testing.assert_array_equal(dw.ravel(), np.array([2, 2, 1, 1, 1, 1, 0, 0], np.float32))


@pytest.mark.parametrize("n,V,D,mode", [(16384, 65, 384, "uniform"), (3000, 50304, 96, "uniform"),
                                        (5000, 7, 33, "same"), (1, 10, 4, "uniform"),
                                        (2049, 256, 128, "uniform"), (65536, 65, 64, "uniform")])
def test_embedding_parity(M, rt, orc, rng, n, V, D, mode):
    w = rng.standard_normal((V, D)).astype(np.float32)
    idx = (rng.integers(0, V, n) if mode == "uniform" else np.full(n, V - 1)).astype(np.int32)
    out = H(M, rt.__embedding_fwd(T(M, w).h, T(M, idx).h)).numpy()
    np.testing.assert_array_equal(out, w[idx])   # gather: bit-exact
    g = rng.standard_normal((n, D)).astype(np.float32)
    dw1 = H(M, rt.__embedding_bwd(T(M, w).h, T(M, idx).h, T(M, g).h)).numpy()
    dw2 = H(M, rt.__embedding_bwd(T(M, w).h, T(M, idx).h, T(M, g).h)).numpy()
    np.testing.assert_array_equal(dw1, dw2)      # deterministic
    # the segmented sum adds each id's rows in token order from 0.0f, as the
    # oracle's scatter-add does: bit-exact
    np.testing.assert_array_equal(dw1, orc.embedding_bwd(g, idx, V))


def test_embedding_empty(M, rt):
    w = np.ones((5, 4), np.float32)
    idx = np.zeros(0, np.int32)
    dw = H(M, rt.__embedding_bwd(T(M, w).h, T(M, idx).h, T(M, np.zeros((0, 4), np.float32)).h)).numpy()
    assert dw.shape == (5, 4) and np.all(dw == 0)


# ------------------------------------------------------------------ permute
@pytest.mark.parametrize("shape,perm", [((4, 16, 6, 64), (0, 2, 1, 3)), ((24, 64, 32), (0, 2, 1)),
                                        ((5, 7), (1, 0)), ((3, 4, 5, 6), (3, 1, 0, 2)),
                                        ((2, 3, 4), (2, 0, 1)), ((33, 65), (1, 0))])
def test_permute(M, rt, orc, rng, shape, perm):
    x = rng.standard_normal(shape).astype(np.float32)
    p = (C.c_size_t * len(perm))(*perm)
    out = H(M, rt.tensor_permute(T(M, x).h, p, len(perm))).numpy()
    np.testing.assert_array_equal(out, np.transpose(x, perm))
    np.testing.assert_array_equal(out, orc.permute(x, perm))


def test_permute_normalisation(M, rt, rng):
    x = rng.standard_normal((3, 4)).astype(np.float32)
    out = H(M, rt.tensor_permute(T(M, x).h, None, 0)).numpy()       # 0 args: 2-D transpose
    np.testing.assert_array_equal(out, x.T)
    x3 = rng.standard_normal((2, 3, 4)).astype(np.float32)
    out = H(M, rt.tensor_permute(T(M, x3).h, (C.c_size_t * 2)(0, 2), 2)).numpy()  # swap
    np.testing.assert_array_equal(out, np.swapaxes(x3, 0, 2))
    out = H(M, rt.tensor_permute(T(M, x).h, (C.c_size_t * 2)(0, 1), 2)).numpy()   # 2 args = swap
    np.testing.assert_array_equal(out, x.T)


def test_reshape_aliases(M, rt, rng):
    x = rng.standard_normal((6, 4)).astype(np.float32)
    t = T(M, x)
    s, n = sarr((2, 3, 4))
    r = H(M, rt.tensor_reshape(t.h, s, n))
    assert r.shape == (2, 3, 4)
    assert rt.malus_tensor_data(r.h) == rt.malus_tensor_data(t.h)
    t.close()                     # the alias keeps the storage alive
    np.testing.assert_array_equal(r.numpy(), x.reshape(2, 3, 4))


# ------------------------------------------------------------------- matmul
def _mm_scale(a, b):
    return np.abs(a.astype(np.float64)) @ np.abs(b.astype(np.float64))


@pytest.mark.parametrize("sa,sb", [((2, 3), (3, 2)), ((4, 2), (2, 8)), ((37, 19), (19, 23)),
                                   ((256, 384), (384, 384)), ((1000, 128), (128, 65)),
                                   ((512, 384), (384, 1536)), ((300, 1536), (1536, 384)),
                                   ((384, 130), (130, 200))])
def test_matmul_2d(M, rt, orc, rng, sa, sb):
    a = rng.standard_normal(sa).astype(np.float32)
    b = rng.standard_normal(sb).astype(np.float32)
    out = H(M, rt.tensor_matmul(T(M, a).h, T(M, b).h)).numpy()
    ref = orc.matmul(a, b)
    assert rel_err(out, ref, _mm_scale(a, b)) < 1e-4


def test_matmul_small_is_bit_exact(M, rt, orc, rng):
    a = rng.standard_normal((4, 2)).astype(np.float32)
    b = rng.standard_normal((2, 8)).astype(np.float32)
    out = H(M, rt.tensor_matmul(T(M, a).h, T(M, b).h)).numpy()
    np.testing.assert_array_equal(out, orc.matmul(a, b))


def test_matmul_golden(M, rt):
    a = np.array([[1, 2, 3], [4, 5, 6]], np.float32)
    b = np.array([[1, 0], [0, 1], [1, 0]], np.float32)
    np.testing.assert_array_equal(H(M, rt.tensor_matmul(T(M, a).h, T(M, b).h)).numpy(), [[4, 2], [10, 5]])


@pytest.mark.parametrize("sa,sb", [((24, 64, 32), (24, 32, 64)), ((24, 64, 64), (24, 64, 32)),
                                   ((6, 256, 64), (6, 64, 256)), ((3, 130, 64), (3, 64, 70))])
def test_matmul_batched(M, rt, orc, rng, sa, sb):
    a = rng.standard_normal(sa).astype(np.float32)
    b = rng.standard_normal(sb).astype(np.float32)
    out = H(M, rt.tensor_matmul(T(M, a).h, T(M, b).h)).numpy()
    ref = orc.matmul(a, b)
    scale = np.stack([_mm_scale(a[i], b[i]) for i in range(a.shape[0])])
    assert rel_err(out, ref, scale) < 1e-4


def test_matmul_3x2(M, rt, orc, rng):
    a = rng.standard_normal((4, 64, 128)).astype(np.float32)
    b = rng.standard_normal((128, 96)).astype(np.float32)
    out = H(M, rt.tensor_matmul(T(M, a).h, T(M, b).h)).numpy()
    ref = orc.matmul(a, b)
    scale = np.stack([_mm_scale(a[i], b) for i in range(4)])
    assert rel_err(out, ref, scale) < 1e-4


@pytest.mark.parametrize("sa,sb", [((512, 384), (384, 384)), ((700, 128), (128, 65)),
                                   ((8, 256, 64), (8, 64, 256)), ((8, 256, 256), (8, 256, 64)),
                                   ((4, 64, 128), (128, 96)), ((37, 19), (19, 23))])
def test_matmul_vjps(M, rt, orc, rng, sa, sb):
    a = rng.standard_normal(sa).astype(np.float32)
    b = rng.standard_normal(sb).astype(np.float32)
    ta, tbb = T(M, a), T(M, b)
    c = H(M, rt.tensor_matmul(ta.h, tbb.h))
    g = rng.standard_normal(c.shape).astype(np.float32)
    tg = T(M, g)
    da = H(M, rt.__matmul_bwd_a(ta.h, tbb.h, tg.h)).numpy()
    db = H(M, rt.__matmul_bwd_b(ta.h, tbb.h, tg.h)).numpy()
    bt = np.swapaxes(b, -1, -2)
    if b.ndim == 2:
        da_ref = orc.matmul(g.reshape(-1, g.shape[-1]), np.ascontiguousarray(b.T)).reshape(a.shape)
        a2 = a.reshape(-1, a.shape[-1])
        db_ref = orc.matmul(np.ascontiguousarray(a2.T), g.reshape(-1, g.shape[-1]))
        sa_ = _mm_scale(g.reshape(-1, g.shape[-1]), b.T).reshape(a.shape)
        sb_ = _mm_scale(a2.T, g.reshape(-1, g.shape[-1]))
    else:
        da_ref = orc.matmul(g, np.ascontiguousarray(bt))
        db_ref = orc.matmul(np.ascontiguousarray(np.swapaxes(a, 1, 2)), g)
        sa_ = np.stack([_mm_scale(g[i], bt[i]) for i in range(a.shape[0])])
        sb_ = np.stack([_mm_scale(a[i].T, g[i]) for i in range(a.shape[0])])
    assert da.shape == a.shape and db.shape == b.shape
    assert rel_err(da, da_ref, sa_) < 1e-4
    assert rel_err(db, db_ref, sb_) < 1e-4


# ------------------------------------------------------------------ AdamW
def test_adamw_bit_exact(M, rt, orc, rng):
    n = 10007
    p = rng.standard_normal(n).astype(np.float32)
    g = rng.standard_normal(n).astype(np.float32)
    m = np.zeros(n, np.float32)
    v = np.zeros(n, np.float32)
    tp, tg, tm, tv = T(M, p), T(M, g), T(M, m), T(M, v)
    arr = lambda h: (C.c_int64 * 1)(h)
    for step in (1, 2, 3):
        rt.malus_adamw_multi(arr(tp.h), arr(tg.h), arr(tm.h), arr(tv.h), 1, 1e-3, 0.9, 0.99, 1e-8, 0.1, step, 1.0)
        orc.adamw(p, g, m, v, 1e-3, 0.9, 0.99, 1e-8, 0.1, step)
    np.testing.assert_array_equal(tp.numpy(), p)
    np.testing.assert_array_equal(tm.numpy(), m)
    np.testing.assert_array_equal(tv.numpy(), v)


# ------------------------------------------------------------ RNG & mask
def test_randn_matches_oracle(M, rt, orc):
    rt.malus_rng_reset(5)
    s, n = sarr((17, 33))
    a = H(M, rt.tensor_randn(s, n)).numpy()
    np.testing.assert_array_equal(a, orc.randn((17, 33), 5))
    assert rt.malus_rand_int(65) == orc.rand_int(65, 6)
    assert rt.malus_rand_uniform() == np.float32(orc.rand_uniform(7))


def test_causal_mask(M, rt):
    m = H(M, rt.tensor_causal_mask(5)).numpy()
    ref = np.triu(np.full((5, 5), -1e9, np.float32), 1)
    np.testing.assert_array_equal(m, ref)


def test_alloc_zeros_ones_and_get(M, rt):
    s, n = sarr((3, 5))
    z = H(M, rt.tensor_alloc_zeros_gpu(s, n))
    o = H(M, rt.tensor_alloc_ones_gpu(s, n))
    assert np.all(z.numpy() == 0) and np.all(o.numpy() == 1)
    assert rt.malus_tensor_get_f32(o.h, 7) == 1.0
    s0, n0 = sarr((0,))
    e = H(M, rt.tensor_alloc_zeros_gpu(s0, n0))
    assert rt.tensor_len(e.h) == 0


def test_buffer_freeze(M, rt):
    b = rt.malus_buffer_i32(5)
    for i in range(5):
        rt.malus_buffer_set_i32(b, i, 10 * i)
    t = H(M, rt.malus_buffer_freeze_i32(b))
    rt.malus_buffer_free(b)
    np.testing.assert_array_equal(t.numpy(), np.arange(0, 50, 10, dtype=np.int32))


def test_no_device_error_word(M, rt):
    assert rt.malus_device_error() == 0
