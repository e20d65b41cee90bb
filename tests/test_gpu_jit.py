"""GPU: user kernels registered as MSL source (the reference's runtime_init
contract), compiled by NVRTC, launched through kernel_dispatch /
kernel_dispatch_v2 with the reference's buffer / TensorMeta / uniform layout."""
import ctypes as C
import struct

import numpy as np
import pytest

import msl_kernels as K

pytestmark = pytest.mark.gpu
_LIVE = []


@pytest.fixture(autouse=True)
def _free():
    yield
    _LIVE.clear()


def T(M, a):
    t = M.Tensor.from_numpy(np.ascontiguousarray(a, np.float32))
    _LIVE.append(t)
    return t


def register(rt, kid, src):
    rt.malus_runtime_init((C.c_uint64 * 1)(kid), (C.c_char_p * 1)(src.encode()), 1)


def v2(M, rt, kid, ins, grid, tg, uniforms=b""):
    hs = (C.c_int64 * len(ins))(*[t.h for t in ins])
    g = (C.c_size_t * 3)(*grid)
    b = (C.c_size_t * 3)(*tg)
    ub = C.create_string_buffer(uniforms, max(1, len(uniforms)))
    out = M.Tensor(rt.kernel_dispatch_v2(kid, hs, len(ins), g, b, None, 0, -1, ub, len(uniforms)))
    _LIVE.append(out)
    return out.numpy()


def test_implicit_kernels(M, rt, rng):
    n = 100003                       # not a multiple of the block: the guard matters
    a, b = rng.standard_normal(n).astype(np.float32), rng.standard_normal(n).astype(np.float32)
    ta, tb_ = T(M, a), T(M, b)
    for kid, src, ref in [(5001, K.ADD, a + b),
                          (5002, K.RELU_BWD, a * (b > 0)),
                          (5003, K.SIGMOID_BWD, (a * b) * (np.float32(1) - b)),
                          (5004, K.SIGMOID, 1.0 / (1.0 + np.exp(-a.astype(np.float64))))]:
        register(rt, kid, src)
        args = [ta] if src is K.SIGMOID else [ta, tb_]
        h = rt.kernel_dispatch(kid, (C.c_int64 * len(args))(*[t.h for t in args]), len(args))
        got = M.Tensor(h).numpy()
        np.testing.assert_allclose(got, ref, rtol=1e-6, atol=1e-7, err_msg=str(kid))


def test_scalar_builtin(M, rt, rng):
    a = rng.standard_normal(4097).astype(np.float32)
    register(rt, 5010, K.MUL_SCALAR)
    ta, ts = T(M, a), T(M, np.array([1.5], np.float32))
    got = M.Tensor(rt.kernel_dispatch(5010, (C.c_int64 * 2)(ta.h, ts.h), 2)).numpy()
    np.testing.assert_array_equal(got, a * np.float32(1.5))


def test_explicit_gelu_thread_id(M, rt, rng):
    n = 5000
    x = rng.standard_normal(n).astype(np.float32)
    register(rt, 5020, K.GELU)
    got = v2(M, rt, 5020, [T(M, x)], ((n + 255) // 256, 1, 1), (256, 1, 1))
    xd = x.astype(np.float64)
    ref = 0.5 * xd * (1 + np.tanh(0.7978846 * (xd + 0.044715 * xd ** 3)))
    np.testing.assert_allclose(got, ref, rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("rows,cols", [(64, 100), (7, 512), (1, 1)])
def test_explicit_softmax_shared_barriers_uniforms(M, rt, rng, rows, cols):
    x = rng.standard_normal((rows, cols)).astype(np.float32)
    register(rt, 5030, K.SOFTMAX)
    got = v2(M, rt, 5030, [T(M, x)], (rows, 1, 1), (cols, 1, 1), struct.pack("<i", cols))
    e = np.exp(x.astype(np.float64) - x.max(1, keepdims=True))
    np.testing.assert_allclose(got, e / e.sum(1, keepdims=True), rtol=1e-5, atol=1e-7)


def test_explicit_layernorm_strided_rsqrt(M, rt, rng):
    rows, cols = 33, 384
    x = rng.standard_normal((rows, cols)).astype(np.float32)
    register(rt, 5040, K.LAYERNORM)
    got = v2(M, rt, 5040, [T(M, x)], (rows, 1, 1), (cols, 1, 1), struct.pack("<iff", cols, 1.0 / cols, 1e-5))
    xd = x.astype(np.float64)
    ref = (xd - xd.mean(1, keepdims=True)) / np.sqrt(xd.var(1, keepdims=True) + 1e-5)
    np.testing.assert_allclose(got, ref, rtol=1e-4, atol=1e-5)


def test_same_source_compiles_once(M, rt):
    for kid in (5101, 5102, 5103):
        register(rt, kid, K.ADD)       # cached by source: three ids, one module
    a = T(M, np.ones(10, np.float32))
    for kid in (5101, 5102, 5103):
        out = M.Tensor(rt.kernel_dispatch(kid, (C.c_int64 * 2)(a.h, a.h), 2)).numpy()
        assert np.all(out == 2)
