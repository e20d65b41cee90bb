"""GPU: every stdlib kernel name that kernel_dispatch_v2 binds natively,
launched exactly as its .ml host function launches it (grid, threadgroup,
out= shape with trailing-zero sentinels stripped, uniforms packed 4 bytes each
in declaration order), against the oracle or the kernel's own formula.

Sources of the launch conventions (crates/malus-stdlib/stdlib/):
softmax.ml:30-40, layernorm.ml:59-72, reduce_{sum,mean,max,var}.ml (the
(ndim, axis, keepdim) out= branches), reduce_all.ml:9-12, gelu.ml:12-14,
cross_entropy.ml:18-28, embedding.ml:18-23, broadcast_binop.ml:82-112,
permute.ml:21-126, backward/reduce_bwd.ml:22-38,
backward/transformer_bwd.ml:6-98, backward/unary_bwd.ml:6-91.
Bars: gathers, permutes, fills, masks and sign selections bit-exact;
elementwise arithmetic within 1e-5 relative; reductions within 1e-5 of sum|x|."""
import ctypes as C
import itertools
import struct

import numpy as np
import pytest

from conftest import rel_err

pytestmark = pytest.mark.gpu

NAMES = ["__softmax_kernel", "__layernorm_kernel", "__layernorm_var_kernel", "__reduce_sum_kernel",
         "__reduce_mean_kernel", "__reduce_max_kernel", "__reduce_var_kernel", "__expand_axis_kernel",
         "__gelu_kernel", "__gelu_bwd_kernel", "__cross_entropy_nll_kernel", "__cross_entropy_bwd_kernel",
         "__embedding_kernel", "__embedding_bwd_kernel", "__transpose_2d_kernel", "__permute_3d_kernel",
         "__permute_nd_kernel", "__scale_kernel", "__fill_like_kernel", "__eq_kernel",
         "__sigmoid_bwd_kernel", "__relu_bwd_kernel", "__tanh_bwd_kernel", "__sqrt_bwd_kernel",
         "__abs_bwd_kernel", "__rsqrt_eps_kernel", "__broadcast_add_kernel", "__broadcast_sub_kernel",
         "__broadcast_mul_kernel", "__broadcast_div_kernel"]
BASE_ID = 880000


@pytest.fixture(scope="module")
def kid(rt):
    ids = (C.c_uint64 * len(NAMES))(*[BASE_ID + i for i in range(len(NAMES))])
    nm = (C.c_char_p * len(NAMES))(*[n.encode() for n in NAMES])
    rt.malus_runtime_init(ids, nm, len(NAMES))
    return {n: BASE_ID + i for i, n in enumerate(NAMES)}


def pack(*uniforms):
    """Uniforms as codegen-cpu packs them: 4 bytes each, i32 for ints, f32 for floats."""
    b = b"".join(struct.pack("<f", u) if isinstance(u, float) else struct.pack("<i", u) for u in uniforms)
    return C.create_string_buffer(b, len(b)), len(b)


def v2(M, rt, kid, name, inputs, grid, tg, out=None, uniforms=()):
    """kernel_dispatch_v2 as the JIT lowers `name[grid=, tg=, out=](inputs..., uniforms...)`."""
    ts = [M.Tensor.from_numpy(a) for a in inputs]
    hs = (C.c_int64 * len(ts))(*[t.h for t in ts])
    g = (C.c_size_t * 3)(*grid)
    t = (C.c_size_t * 3)(*tg)
    dims = list(out or [])
    while dims and dims[-1] == 0:          # trailing literal 0s are sentinels (codegen-cpu lib.rs:2225-2240)
        dims.pop()
    od = (C.c_size_t * max(1, len(dims)))(*dims)
    ub, nb = pack(*uniforms) if uniforms else (None, 0)
    h = rt.kernel_dispatch_v2(kid[name], hs, len(ts), g, t, od, len(dims), 0, ub, nb)
    return M.Tensor(h).numpy()


def groups(shape, axis):
    outer = int(np.prod(shape[:axis])) if axis else 1
    inner = int(np.prod(shape[axis + 1:])) if axis + 1 < len(shape) else 1
    return outer, shape[axis], inner


@pytest.mark.parametrize("shape,axis", [((4, 37, 5), 1), ((8, 300), 1), ((64, 3), 0), ((2, 3, 129), 2)])
def test_softmax_kernel(M, rt, kid, orc, rng, shape, axis):
    x = rng.standard_normal(shape).astype(np.float32) * 3
    outer, a, inner = groups(shape, axis)
    got = v2(M, rt, kid, "__softmax_kernel", [x], [outer * inner, 1, 1], [a, 1, 1], None, (a, inner))
    assert got.shape == shape
    assert rel_err(got, orc.softmax(x, axis), np.abs(orc.softmax(x, axis)) + 1e-6) < 1e-5


@pytest.mark.parametrize("shape,axis", [((16, 96), 1), ((3, 50, 4), 1), ((40, 6), 0)])
def test_layernorm_kernels(M, rt, kid, orc, rng, shape, axis):
    x = (rng.standard_normal(shape) * 2 + 0.5).astype(np.float32)
    outer, a, inner = groups(shape, axis)
    y = v2(M, rt, kid, "__layernorm_kernel", [x], [outer * inner, 1, 1], [a, 1, 1], None, (a, inner, 1e-5))
    var = v2(M, rt, kid, "__layernorm_var_kernel", [x], [outer * inner, 1, 1], [a, 1, 1], None,
             (a, inner, 1e-5))
    ry, rv = orc.layernorm(x, axis)
    # x - mean cancels near the group mean: relative to max(|y|, 1) (y is O(1) by construction)
    assert rel_err(y, ry, np.maximum(np.abs(ry), 1.0)) < 1e-5
    # layernorm.ml:35-57: the per-group variance written at every element of the group
    assert rel_err(var, np.broadcast_to(rv, shape), np.broadcast_to(rv, shape)) < 1e-5


def reduce_out_shape(shape, axis, keepdim):
    """The out= literal of reduce_*.ml's (ndim, axis, keepdim) branches."""
    if len(shape) == 1:
        return [1, 0, 0]
    rest = [d for i, d in enumerate(shape) if i != axis]
    if keepdim:
        return [1 if i == axis else d for i, d in enumerate(shape)] + [0] * (3 - len(shape))
    return rest + [0] * (3 - len(rest))


@pytest.mark.parametrize("op,name", [(0, "__reduce_sum_kernel"), (1, "__reduce_mean_kernel"),
                                     (2, "__reduce_max_kernel"), (3, "__reduce_var_kernel")])
@pytest.mark.parametrize("shape,axis,keepdim", [((1000,), 0, 0), ((7, 900), 1, 0), ((600, 9), 0, 1),
                                                ((5, 6, 70), 1, 0), ((5, 6, 70), 2, 1), ((3, 300, 4), 0, 0)])
def test_reduce_kernels(M, rt, kid, orc, rng, op, name, shape, axis, keepdim):
    x = rng.standard_normal(shape).astype(np.float32)
    outer, a, inner = groups(shape, axis)
    grid = [1, 1, 1] if len(shape) == 1 else [outer * inner, 1, 1]
    got = v2(M, rt, kid, name, [x], grid, [a, 1, 1], reduce_out_shape(shape, axis, keepdim), (a, inner))
    ref = orc.reduce(op, x, axis, bool(keepdim))
    assert got.size == ref.size
    scale = np.sum(np.abs(x), axis=axis).ravel() / (a if op in (1,) else 1)
    if op == 3:
        scale = np.sum(x.astype(np.float64) ** 2, axis=axis).ravel() / a + 1e-6
    if op == 2:
        np.testing.assert_array_equal(got.ravel(), ref.ravel())   # max is a selection
    else:
        assert rel_err(got.ravel(), ref.ravel(), scale) < 1e-5


def test_reduce_all_sum_via_reduce_sum_kernel(M, rt, kid, rng):
    x = rng.standard_normal((33, 31)).astype(np.float32)
    n = x.size
    got = v2(M, rt, kid, "__reduce_sum_kernel", [x], [1, 1, 1], [n, 1, 1], [1, 0, 0], (n, 1))
    assert got.shape == (1,)
    assert abs(float(got[0]) - float(np.sum(x, dtype=np.float64))) < 1e-5 * float(np.sum(np.abs(x)))


@pytest.mark.parametrize("shape,axis", [((6,), 0), ((5, 7), 0), ((5, 7), 1), ((3, 4, 5), 1)])
def test_expand_axis_kernel(M, rt, kid, rng, shape, axis):
    outer, a, inner = groups(shape, axis)
    small = rng.standard_normal(outer * inner).astype(np.float32)
    got = v2(M, rt, kid, "__expand_axis_kernel", [small], [outer * a * inner, 1, 1], [1, 1, 1],
             list(shape) + [0] * (3 - len(shape)), (a, inner))
    ref = np.broadcast_to(small.reshape(outer, 1, inner), (outer, a, inner)).reshape(shape)
    np.testing.assert_array_equal(got, ref)


def test_gelu_kernels(M, rt, kid, orc, rng):
    x = (rng.standard_normal(5000) * 3).astype(np.float32)
    g = rng.standard_normal(5000).astype(np.float32)
    y = v2(M, rt, kid, "__gelu_kernel", [x], [x.size, 1, 1], [1, 1, 1])
    ry = orc.unary("gelu", x)
    # 1 + tanh(.) cancels for large negative x: relative to max(|gelu(x)|, |x|)
    assert rel_err(y, ry, np.maximum(np.abs(ry), np.abs(x)) + 1e-6) < 1e-5
    dx = v2(M, rt, kid, "__gelu_bwd_kernel", [x, g], [x.size, 1, 1], [1, 1, 1])
    rdx = orc.unary_bwd("gelu", x, g)
    # the derivative is O(1) but passes through zero near x = -0.75: relative to |dout|
    assert rel_err(dx, rdx, np.abs(g) + 1e-6) < 1e-5


@pytest.mark.parametrize("dt", [np.int32, np.int64])
def test_cross_entropy_kernels(M, rt, kid, orc, rng, dt):
    n, V = 300, 65
    logits = rng.standard_normal((n, V)).astype(np.float32)
    t = rng.integers(0, V, n).astype(dt)
    _, probs = orc.xent(logits, t.astype(np.int32))
    nll = v2(M, rt, kid, "__cross_entropy_nll_kernel", [probs, t], [n, 1, 1], [1, 1, 1], [n, 0, 0], (V,))
    ref = -np.log(probs[np.arange(n), t].astype(np.float64))
    assert rel_err(nll, ref, np.abs(ref)) < 1e-6
    dout0 = 0.75
    n_f = np.float32(0.0)
    for _ in range(n):                       # transformer_bwd.ml:67-74: n_f counted up in f32
        n_f = np.float32(n_f + np.float32(1.0))
    scale = float(np.float32(dout0) / n_f)
    dx = v2(M, rt, kid, "__cross_entropy_bwd_kernel", [probs, t], [n * V, 1, 1], [1, 1, 1], None, (V, scale))
    onehot = np.zeros((n, V), np.float32)
    onehot[np.arange(n), t] = 1.0
    np.testing.assert_array_equal(dx, (probs - onehot) * np.float32(scale))   # same two f32 ops


@pytest.mark.parametrize("dt", [np.int32, np.int64])
def test_embedding_kernels(M, rt, kid, orc, rng, dt):
    V, D, n = 65, 48, 777
    w = rng.standard_normal((V, D)).astype(np.float32)
    idx = rng.integers(0, V, n).astype(dt)
    out = v2(M, rt, kid, "__embedding_kernel", [w, idx], [n * D, 1, 1], [1, 1, 1], [n, D, 0], (D,))
    np.testing.assert_array_equal(out, w[idx])
    g = rng.standard_normal((n, D)).astype(np.float32)
    dw = v2(M, rt, kid, "__embedding_bwd_kernel", [g, idx], [V * D, 1, 1], [1, 1, 1], [V, D, 0], (n, D))
    np.testing.assert_array_equal(dw, orc.embedding_bwd(g, idx.astype(np.int32), V))


def test_permute_kernels(M, rt, kid, rng):
    x2 = rng.standard_normal((33, 65)).astype(np.float32)
    t2 = v2(M, rt, kid, "__transpose_2d_kernel", [x2], [x2.size, 1, 1], [1, 1, 1], [65, 33, 0])
    np.testing.assert_array_equal(t2, x2.T)
    x3 = rng.standard_normal((4, 5, 6)).astype(np.float32)
    for p in itertools.permutations(range(3)):
        os_ = [x3.shape[k] for k in p]
        got = v2(M, rt, kid, "__permute_3d_kernel", [x3], [x3.size, 1, 1], [1, 1, 1], os_,
                 (p[0], p[1], p[2], os_[1], os_[2]))
        np.testing.assert_array_equal(got, np.transpose(x3, p))
    x4 = rng.standard_normal((2, 3, 4, 5)).astype(np.float32)
    for p in [(0, 2, 1, 3), (3, 1, 0, 2), (1, 0, 3, 2)]:
        os_ = [x4.shape[k] for k in p] + [0] * 4
        got = v2(M, rt, kid, "__permute_nd_kernel", [x4], [x4.size, 1, 1], [1, 1, 1], os_,
                 tuple(p) + (0, 0, 0, 0))
        np.testing.assert_array_equal(got, np.transpose(x4, p))


def test_unary_helper_kernels(M, rt, kid, rng):
    x = rng.standard_normal(4097).astype(np.float32)
    x[::7] = 0.0
    y = x.copy()
    y[::3] = rng.standard_normal(y[::3].size).astype(np.float32)
    g = rng.standard_normal(4097).astype(np.float32)
    n = [x.size, 1, 1]
    one = [1, 1, 1]
    np.testing.assert_array_equal(v2(M, rt, kid, "__scale_kernel", [x], n, one, None, (-0.375,)),
                                  x * np.float32(-0.375))
    np.testing.assert_array_equal(v2(M, rt, kid, "__fill_like_kernel", [x], n, one, None, (2.5,)),
                                  np.full_like(x, 2.5))
    np.testing.assert_array_equal(v2(M, rt, kid, "__eq_kernel", [x, y], n, one),
                                  (x == y).astype(np.float32))
    np.testing.assert_array_equal(v2(M, rt, kid, "__relu_bwd_kernel", [x, g], n, one),
                                  np.where(x > 0, g, np.float32(0)))
    np.testing.assert_array_equal(v2(M, rt, kid, "__abs_bwd_kernel", [x, g], n, one),
                                  np.where(x > 0, g, np.where(x < 0, -g, np.float32(0))))
    s = (1 / (1 + np.exp(-x.astype(np.float64)))).astype(np.float32)
    ref = g.astype(np.float64) * s * (1.0 - s)
    assert rel_err(v2(M, rt, kid, "__sigmoid_bwd_kernel", [s, g], n, one), ref, np.abs(ref) + 1e-7) < 1e-5
    t = np.tanh(x).astype(np.float32)
    ref = g.astype(np.float64) * (1.0 - t.astype(np.float64) ** 2)
    # 1 - t*t cancels as |t| -> 1: relative to |dout|
    assert rel_err(v2(M, rt, kid, "__tanh_bwd_kernel", [t, g], n, one), ref, np.abs(g) + 1e-7) < 1e-5
    q = (np.abs(x) + 0.5).astype(np.float32)
    ref = g.astype(np.float64) / (2.0 * q)
    assert rel_err(v2(M, rt, kid, "__sqrt_bwd_kernel", [q, g], n, one), ref, np.abs(ref)) < 1e-5
    ref = 1.0 / np.sqrt(q.astype(np.float64) + 1e-5)
    assert rel_err(v2(M, rt, kid, "__rsqrt_eps_kernel", [q], n, one, None, (1e-5,)), ref, ref) < 1e-5


@pytest.mark.parametrize("op,name", [(0, "__broadcast_add_kernel"), (1, "__broadcast_sub_kernel"),
                                     (2, "__broadcast_mul_kernel"), (3, "__broadcast_div_kernel")])
@pytest.mark.parametrize("sa,sb", [((6, 10), (10,)), ((4, 5, 6), (5, 1)), ((4, 5, 6), (4, 5, 6)),
                                   ((3, 8), (1, 1)), ((2, 3, 4), (1, 3, 1))])
def test_broadcast_kernels(M, rt, kid, rng, op, name, sa, sb):
    """broadcast_binop.ml:10-80: out has a's shape (out_ndim 0 inherits input 0),
    b is projected through its strides with size-1 dims pinned to index 0."""
    a = rng.standard_normal(sa).astype(np.float32)
    b = (rng.standard_normal(sb) + (3.0 if op == 3 else 0.0)).astype(np.float32)
    got = v2(M, rt, kid, name, [a, b], [a.size, 1, 1], [1, 1, 1])
    fn = [np.add, np.subtract, np.multiply, np.divide][op]
    np.testing.assert_array_equal(got, fn(a, np.broadcast_to(b, sa)).astype(np.float32))
