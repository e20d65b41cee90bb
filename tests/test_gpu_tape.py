"""GPU: the autograd tape through the C ABI, against the reference's own
backward-rule tests (crates/malus-runtime/src/tests.rs:466-866, 1102-1160,
1421-1461) and the XOR example (examples/xor.ml) driven op by op the way
the JIT drives the runtime."""
import ctypes as C
import json
from pathlib import Path

import numpy as np
import pytest

from conftest import rel_err

pytestmark = pytest.mark.gpu
G = json.loads((Path(__file__).parent / "golden" / "reference_golden.json").read_text())

ADD, SUB, MUL, DIV, SIGMOID, RELU, ABS, SUM, TRANSPOSE, MATMUL = 1, 2, 3, 4, 5, 6, 11, 12, 13, 0


_LIVE = []  # keeps tensors alive until the test ends (inline temporaries would be freed early)


def T(M, a, leaf=False, rt=None):
    t = M.Tensor.from_numpy(np.asarray(a, np.float32))
    _LIVE.append(t)
    if leaf:
        rt.tape_register_leaf(t.h)
    return t


def grad(M, rt, t):
    return M.Tensor(rt.tape_get_grad(t.h)).numpy()


@pytest.fixture(autouse=True)
def reset(rt):
    rt.malus_tape_reset()
    yield
    rt.malus_tape_reset()
    _LIVE.clear()


@pytest.mark.parametrize("name,tag", [("backward_add", ADD), ("backward_sub", SUB),
                                      ("backward_mul", MUL), ("backward_div", DIV)])
def test_binop_backward_golden(M, rt, name, tag):
    g = G[name]
    a, b = T(M, g["a"], True, rt), T(M, g["b"], True, rt)
    fn = {ADD: rt.__broadcast_add_fwd, SUB: rt.__broadcast_sub_fwd, MUL: rt.__broadcast_mul_fwd,
          DIV: rt.__broadcast_div_fwd}[tag]
    out = M.Tensor(fn(a.h, b.h))
    rt.tape_record_binop(tag, a.h, b.h, out.h)
    rt.backward(out.h)
    np.testing.assert_allclose(grad(M, rt, a), g["ga"], rtol=1e-6)
    np.testing.assert_allclose(grad(M, rt, b), g["gb"], rtol=1e-6)


@pytest.mark.parametrize("name,tag", [("backward_relu", RELU), ("backward_abs", ABS)])
def test_unary_backward_golden(M, rt, name, tag):
    g = G[name]
    x = T(M, g["x"], True, rt)
    out = T(M, np.zeros(len(g["x"])))
    rt.tape_record_unary(tag, x.h, out.h)
    rt.backward(out.h)
    np.testing.assert_array_equal(grad(M, rt, x), np.array(g["gx"], np.float32))


def test_sum_and_transpose_backward(M, rt):
    x = T(M, [1, 2, 3], True, rt)
    s = M.Tensor(rt.__reduce_all_sum_fwd(x.h))
    rt.tape_record_unary(SUM, x.h, s.h)
    rt.backward(s.h)
    np.testing.assert_array_equal(grad(M, rt, x), [1, 1, 1])
    y = T(M, [[1, 2], [3, 4]], True, rt)
    out = T(M, [[1, 3], [2, 4]])
    rt.tape_record_unary(TRANSPOSE, y.h, out.h)   # no dims: 2-D transpose
    rt.backward(out.h)
    gy = grad(M, rt, y)
    assert gy.shape == (2, 2) and np.all(gy == 1)


def test_matmul_backward_golden(M, rt):
    g = G["backward_matmul"]
    a, b = T(M, g["a"], True, rt), T(M, g["b"], True, rt)
    out = M.Tensor(rt.tensor_matmul(a.h, b.h))
    rt.tape_record_binop(MATMUL, a.h, b.h, out.h)
    rt.backward(out.h)
    ga, gb = grad(M, rt, a), grad(M, rt, b)
    assert ga.shape == (2, 3) and gb.shape == (3, 2)
    np.testing.assert_allclose(ga[0], g["ga_row0"], rtol=1e-5)


def test_embedding_vjp_golden(M, rt):
    g = G["embedding_vjp"]
    w = T(M, np.ones((g["vocab"], g["dim"])), True, rt)
    idx = M.Tensor.from_numpy(np.array(g["idx"], np.int32))
    out = M.Tensor(rt.__embedding_fwd(w.h, idx.h))
    rt.tape_record_embedding(24, w.h, idx.h, out.h)
    loss = M.Tensor(rt.__reduce_all_sum_fwd(out.h))
    rt.tape_record_unary(SUM, out.h, loss.h)
    rt.backward(loss.h)
    np.testing.assert_array_equal(grad(M, rt, w).ravel(), np.array(g["gw"], np.float32))


def test_broadcast_add_backward(M, rt):
    a = T(M, np.ones((1, 3)), True, rt)
    b = T(M, np.ones((2, 3)), True, rt)
    out = M.Tensor(rt.__broadcast_add_fwd(a.h, b.h))
    rt.tape_record_binop(ADD, a.h, b.h, out.h)
    loss = M.Tensor(rt.__reduce_all_sum_fwd(out.h))
    rt.tape_record_unary(SUM, out.h, loss.h)
    rt.backward(loss.h)
    ga, gb = grad(M, rt, a), grad(M, rt, b)
    assert ga.shape == (1, 3) and np.all(ga == 2)
    assert gb.shape == (2, 3) and np.all(gb == 1)


def test_accumulate_and_zero_grad(M, rt):
    a = T(M, [3.0], True, rt)
    for _ in range(2):
        out = M.Tensor(rt.__scale_fwd(a.h, 1.0))
        rt.tape_record_unary(SUM, a.h, out.h)
        rt.backward(out.h)
    np.testing.assert_array_equal(grad(M, rt, a), [2.0])
    rt.tape_zero_grad((C.c_int64 * 1)(a.h), 1)
    np.testing.assert_array_equal(grad(M, rt, a), [0.0])


def test_pause_records_nothing(M, rt):
    a, b = T(M, [1, 2], True, rt), T(M, [3, 4], True, rt)
    rt.tape_pause()
    out = M.Tensor(rt.__broadcast_add_fwd(a.h, b.h))
    rt.tape_record_binop(ADD, a.h, b.h, out.h)
    rt.tape_resume()
    rt.backward(out.h)
    assert np.all(grad(M, rt, a) == 0) and np.all(grad(M, rt, b) == 0)


def test_leaf_registry_dies_with_tensor(M, rt):
    a = T(M, [1.0], True, rt)
    out = M.Tensor(rt.__scale_fwd(a.h, 2.0))
    rt.tape_record_unary(SUM, a.h, out.h)
    rt.backward(out.h)
    lv, gr = C.c_int64(), C.c_int64()
    rt.malus_tape_registry_lens(C.byref(lv), C.byref(gr))
    assert lv.value == 1 and gr.value == 1
    a.close()
    rt.malus_tape_registry_lens(C.byref(lv), C.byref(gr))
    assert lv.value == 0 and gr.value == 0


def test_refcounts_balance_over_backward(M, rt, rng):
    # metal_integration.rs:1086-1139: per-step retain/release balance is constant
    x = T(M, rng.standard_normal((8, 16)), True, rt)
    w = T(M, rng.standard_normal((16, 4)), True, rt)
    deltas = []
    for _ in range(3):
        r0, l0, a0 = (C.c_int64() for _ in range(3))
        rt.malus_rc_counts(C.byref(r0), C.byref(l0), C.byref(a0))
        y = M.Tensor(rt.tensor_matmul(x.h, w.h))
        rt.tape_record_binop(MATMUL, x.h, w.h, y.h)
        s = M.Tensor(rt.__reduce_all_sum_fwd(y.h))
        rt.tape_record_unary(SUM, y.h, s.h)
        rt.backward(s.h)
        y.close(); s.close()
        rt.tape_zero_grad((C.c_int64 * 2)(x.h, w.h), 2)
        r1, l1, a1 = (C.c_int64() for _ in range(3))
        rt.malus_rc_counts(C.byref(r1), C.byref(l1), C.byref(a1))
        deltas.append((a1.value - a0.value) + (r1.value - r0.value) - (l1.value - l0.value))
    assert deltas[0] == deltas[1] == deltas[2] == 0


def _register_xor_kernels(rt, msl=False):
    if msl:     # the sources codegen-gpu emits, compiled by NVRTC
        import msl_kernels as K
        names = [K.SIGMOID.encode(), K.MUL_SCALAR.encode(), K.SIGMOID_BWD.encode()]
    else:       # native kernels bound by name
        names = [b"sigmoid", b"malus_mul_scalar", b"sigmoid_backward"]
    rt.malus_runtime_init((C.c_uint64 * 3)(900, 901, 902), (C.c_char_p * 3)(*names), 3)


@pytest.mark.parametrize("msl", [False, True], ids=["native", "nvrtc"])
def test_xor_through_the_abi(M, rt, orc, msl):
    """examples/xor.ml, 10k full-batch SGD steps, every op a C-ABI call; the
    three kernels bound natively or compiled from their MSL by NVRTC."""
    _register_xor_kernels(rt, msl)
    L = rt
    f = lambda a: M.Tensor.from_numpy(np.asarray(a, np.float32))
    x = f([[0, 0], [0, 1], [1, 0], [1, 1]])
    tgt = f([[0], [1], [1], [0]])
    ones41 = f([[1], [1], [1], [1]])
    w1 = f([[0.5, -0.6, 0.7, -0.4, 0.3, -0.5, 0.6, -0.3], [-0.4, 0.5, -0.6, 0.7, -0.3, 0.4, -0.5, 0.6]])
    b1 = f([[0.1, -0.1, 0.1, -0.1, 0.1, -0.1, 0.1, -0.1]])
    w2 = f([[0.6], [-0.5], [0.4], [-0.6], [0.5], [-0.4], [0.6], [-0.5]])
    b2 = f([[0.0]])
    lr = f([1.5])
    two = f([2.0])
    W = [w1.h, b1.h, w2.h, b2.h]
    own = lambda h: h  # handles we release explicitly
    rel = L.tensor_release

    def disp(kid, *hs):
        return L.kernel_dispatch(kid, (C.c_int64 * len(hs))(*hs), len(hs))

    def tr(h):
        return L.tensor_permute(h, None, 0)

    loss_h = 0
    out = 0
    for step in range(10000):
        z1a = L.tensor_matmul(x.h, W[0]); z1b = L.tensor_matmul(ones41.h, W[1])
        z1 = L.__broadcast_add_fwd(z1a, z1b); rel(z1a); rel(z1b)
        h = disp(900, z1); rel(z1)
        z2a = L.tensor_matmul(h, W[2]); z2b = L.tensor_matmul(ones41.h, W[3])
        z2 = L.__broadcast_add_fwd(z2a, z2b); rel(z2a); rel(z2b)
        if out:
            rel(out)
        out = disp(900, z2); rel(z2)
        diff = L.__broadcast_sub_fwd(out, tgt.h)
        sq = L.__broadcast_mul_fwd(diff, diff)
        if loss_h:
            rel(loss_h)
        loss_h = L.__reduce_all_sum_fwd(sq); rel(sq)
        dout = disp(901, diff, two.h); rel(diff)
        dz2 = disp(902, dout, out); rel(dout)
        hT = tr(h); dw2 = L.tensor_matmul(hT, dz2); rel(hT)
        oT = tr(ones41.h); db2 = L.tensor_matmul(oT, dz2)
        w2T = tr(W[2]); dh = L.tensor_matmul(dz2, w2T); rel(w2T); rel(dz2)
        dz1 = disp(902, dh, h); rel(dh); rel(h)
        xT = tr(x.h); dw1 = L.tensor_matmul(xT, dz1); rel(xT)
        db1 = L.tensor_matmul(oT, dz1); rel(oT); rel(dz1)
        new = []
        for p, g in zip(W, [dw1, db1, dw2, db2]):
            s = disp(901, g, lr.h); rel(g)
            n = L.__broadcast_sub_fwd(p, s); rel(s)
            new.append(n)
        for i in (0, 1, 2, 3):
            if step > 0:
                rel(W[i])
        W = new
    loss = L.malus_tensor_get_f32(loss_h, 0)
    preds = M.Tensor(out).numpy().ravel()
    g = G["xor_10k"]
    oloss, opreds = orc.xor_train(10000, 1.5)
    assert abs(loss - g["loss"]) / g["loss"] < g["rtol"]
    assert rel_err(preds, g["preds"]) < g["rtol"]
    assert abs(loss - oloss) / oloss < 1e-3
    assert rel_err(preds, opreds) < 1e-4
    rel(loss_h)
    for hnd in W:
        rel(hnd)
