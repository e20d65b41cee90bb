"""GPU: deferred products x * s (s a one-element tensor) and (x * s) + m (m of
x's trailing shape), as the attention scores are scaled and masked in
nanogpt_modular.ml:53-58, and the deferred gradients of leaves read by one
node (the scale and mask leaves).

The deferred result must be indistinguishable from the eager ops: bit-equal
values when read on the host, through a softmax (which reads it fused), as a
GEMM operand (whose split applies the multiply), after a reshape or permute,
and in the VJPs that produce one (mul_bwd_a) or alias a gradient (add_bwd,
sub_bwd).  Small tensors are never deferred (results equal either way)."""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def T(M, a):
    return M.Tensor.from_numpy(np.ascontiguousarray(a))


def np_of(M, h):
    return M.Tensor(h, owned=False).numpy()


@pytest.fixture
def scores(rng):
    Z, T_ = 24, 256
    qk = (rng.standard_normal((Z, T_, T_)) * 4).astype(np.float32)
    s = np.array([[0.125]], np.float32)
    mask = np.where(np.arange(T_)[None, :] > np.arange(T_)[:, None], np.float32(-1e9), np.float32(0))
    return qk, s, mask.astype(np.float32)


def test_scaled_and_masked_values(M, rt, scores):
    qk, s, mask = scores
    tq, ts, tm = T(M, qk), T(M, s), T(M, mask)
    sc = rt.__broadcast_mul_fwd(tq.h, ts.h)
    ms = rt.__broadcast_add_fwd(sc, tm.h)
    want_sc = qk * s[0, 0]
    want_ms = want_sc + mask
    np.testing.assert_array_equal(np_of(M, ms), want_ms)
    np.testing.assert_array_equal(np_of(M, sc), want_sc)
    for h in (sc, ms):
        rt.tensor_release(h)


def test_softmax_of_deferred_scores_equals_eager(M, rt, scores):
    qk, s, mask = scores
    tq, ts, tm = T(M, qk), T(M, s), T(M, mask)
    sc = rt.__broadcast_mul_fwd(tq.h, ts.h)
    ms = rt.__broadcast_add_fwd(sc, tm.h)
    fused = M.Tensor(rt.__softmax_fwd(ms, 2)).numpy()
    eager_in = T(M, qk * s[0, 0] + mask)
    eager = M.Tensor(rt.__softmax_fwd(eager_in.h, 2)).numpy()
    np.testing.assert_array_equal(fused, eager)
    assert np.all(np.triu(fused[0], 1) == 0.0)          # the masked half is exactly zero
    for h in (sc, ms):
        rt.tensor_release(h)


def test_scaled_gemm_operand_equals_eager(M, rt, rng):
    a = rng.standard_normal((96, 256, 128)).astype(np.float32)
    b = rng.standard_normal((96, 128, 64)).astype(np.float32)
    s = np.array([[0.3]], np.float32)
    ta, tb_, ts = T(M, a), T(M, b), T(M, s)
    sa = rt.__broadcast_mul_fwd(ta.h, ts.h)
    got = M.Tensor(rt.tensor_matmul(sa, tb_.h)).numpy()
    ea = T(M, a * s[0, 0])
    want = M.Tensor(rt.tensor_matmul(ea.h, tb_.h)).numpy()
    np.testing.assert_array_equal(got, want)
    # both VJPs with the deferred operand as the incoming gradient
    g = rng.standard_normal((96, 256, 64)).astype(np.float32)
    tg, ts2 = T(M, g), T(M, np.array([[1.7]], np.float32))
    sg = rt.__broadcast_mul_fwd(tg.h, ts2.h)
    eg = T(M, g * np.float32(1.7))
    for fn in (rt.__matmul_bwd_a, rt.__matmul_bwd_b):
        np.testing.assert_array_equal(M.Tensor(fn(ta.h, tb_.h, sg)).numpy(),
                                      M.Tensor(fn(ta.h, tb_.h, eg.h)).numpy())
    rt.tensor_release(sa)
    rt.tensor_release(sg)


def test_reshape_and_permute_of_deferred(M, rt, rng):
    x = rng.standard_normal((64, 32, 48)).astype(np.float32)
    s = np.array([2.5], np.float32)
    tx, ts = T(M, x), T(M, s)
    sx = rt.__broadcast_mul_fwd(tx.h, ts.h)
    dims = (C.c_size_t * 2)(64 * 32, 48)
    r = rt.tensor_reshape(sx, dims, 2)
    np.testing.assert_array_equal(np_of(M, r), (x * s[0]).reshape(64 * 32, 48))
    p = (C.c_size_t * 3)(2, 0, 1)
    pt = rt.tensor_permute(sx, p, 3)
    np.testing.assert_array_equal(np_of(M, pt), np.transpose(x * s[0], (2, 0, 1)))
    for h in (sx, r, pt):
        rt.tensor_release(h)


def test_vjps_that_alias_or_defer(M, rt, rng):
    g = rng.standard_normal((128, 1024)).astype(np.float32)
    a = rng.standard_normal((128, 1024)).astype(np.float32)
    s = np.array([[0.7]], np.float32)
    tg, ta, ts = T(M, g), T(M, a), T(M, s)
    da = rt.__add_bwd_a(tg.h, ta.h)
    db = rt.__sub_bwd_b(tg.h, ta.h)
    dm = rt.__mul_bwd_a(tg.h, ta.h, ts.h)
    tg.close()                                           # the aliases keep the data alive
    np.testing.assert_array_equal(np_of(M, da), g)
    np.testing.assert_array_equal(np_of(M, db), -g)
    np.testing.assert_array_equal(np_of(M, dm), g * s[0, 0])
    small = T(M, rng.standard_normal((4, 4)).astype(np.float32))
    ds = rt.__mul_bwd_a(small.h, small.h, ts.h)           # small: eager either way
    np.testing.assert_array_equal(np_of(M, ds), small.numpy() * s[0, 0])
    for h in (da, db, dm, ds):
        rt.tensor_release(h)


MUL_TAG, ADD_TAG, SUM_TAG = 3, 1, 12


def _score_graph(M, rt, x, s, m):
    """loss = sum((x * s) + m) recorded on the tape (the attention scale/mask shape)."""
    y = rt.__broadcast_mul_fwd(x.h, s.h)
    rt.tape_record_binop(MUL_TAG, x.h, s.h, y)
    z = rt.__broadcast_add_fwd(y, m.h)
    rt.tape_record_binop(ADD_TAG, y, m.h, z)
    loss = rt.__reduce_all_sum_fwd(z)
    rt.tape_record_unary(SUM_TAG, z, loss)
    for h in (y, z):
        rt.tensor_release(h)
    return loss


def test_deferred_leaf_gradients(M, rt, rng):
    """The scale and mask leaves' gradients: evaluated when the leaf outlives the
    tape (same values as the eager VJPs), dropped unevaluated when the tape held
    the last reference."""
    rt.malus_tape_reset()
    x = T(M, rng.standard_normal((16, 64, 64)).astype(np.float32))
    s = T(M, np.array([[0.5]], np.float32))
    m = T(M, rng.standard_normal((64, 64)).astype(np.float32))
    for t in (x, s, m):
        rt.tape_register_leaf(t.h)
    loss = _score_graph(M, rt, x, s, m)
    rt.backward(loss)
    rt.tensor_release(loss)
    gs = M.Tensor(rt.tape_get_grad(s.h)).numpy()
    gm = M.Tensor(rt.tape_get_grad(m.h)).numpy()
    gx = M.Tensor(rt.tape_get_grad(x.h)).numpy()
    xs = x.numpy().astype(np.float64)
    assert gs.shape == (1, 1) and abs(gs[0, 0] - xs.sum()) <= 1e-5 * np.abs(xs).sum()
    np.testing.assert_array_equal(gm, np.full((64, 64), 16.0, np.float32))
    np.testing.assert_array_equal(gx, np.full(xs.shape, 0.5, np.float32))
    # the same graph with the scale and mask held only by the tape
    rt.malus_tape_reset()
    s2 = M.Tensor.from_numpy(np.array([[0.5]], np.float32))
    m2 = M.Tensor.from_numpy(rng.standard_normal((64, 64)).astype(np.float32))
    rt.tape_register_leaf(x.h)
    rt.tape_register_leaf(s2.h)
    rt.tape_register_leaf(m2.h)
    loss = _score_graph(M, rt, x, s2, m2)
    s2.close()
    m2.close()
    rt.backward(loss)
    rt.tensor_release(loss)
    leaves, grads = C.c_int64(), C.c_int64()
    rt.malus_tape_registry_lens(C.byref(leaves), C.byref(grads))
    assert (leaves.value, grads.value) == (1, 1)           # only x remains, with its gradient
    np.testing.assert_array_equal(M.Tensor(rt.tape_get_grad(x.h)).numpy(), np.full(xs.shape, 0.5, np.float32))
    rt.malus_tape_reset()


def test_gain_vector_products_equal_eager(M, rt, orc, rng):
    """The layernorm gain x * w (w along the last dim), its VJPs and its reads:
    a GEMM operand (the split applies w), the layernorm VJP (reads dout * w
    fused), and the gain gradient (column sums of dout * y in one pass) are
    bit-equal to the eager products."""
    m_, c_ = 2048, 384
    y = rng.standard_normal((m_, c_)).astype(np.float32)
    w = (1.0 + 0.1 * rng.standard_normal(c_)).astype(np.float32)
    wq = rng.standard_normal((c_, 3 * c_)).astype(np.float32)
    ty, tw, twq = T(M, y), T(M, w), T(M, wq)
    xn = rt.__broadcast_mul_fwd(ty.h, tw.h)
    np.testing.assert_array_equal(np_of(M, xn), y * w)              # host read (materialised)
    xn2 = rt.__broadcast_mul_fwd(ty.h, tw.h)                          # a fresh deferred product
    ex = T(M, y * w)
    np.testing.assert_array_equal(M.Tensor(rt.tensor_matmul(xn2, twq.h)).numpy(),
                                  M.Tensor(rt.tensor_matmul(ex.h, twq.h)).numpy())
    g = rng.standard_normal((m_, 3 * c_)).astype(np.float32)
    tg = T(M, g)
    np.testing.assert_array_equal(M.Tensor(rt.__matmul_bwd_b(xn2, twq.h, tg.h)).numpy(),
                                  M.Tensor(rt.__matmul_bwd_b(ex.h, twq.h, tg.h)).numpy())
    # backward of xn = y * w: d_y deferred (dout * w), read by the layernorm VJP
    x = (rng.standard_normal((m_, c_)) * 2 + 0.3).astype(np.float32)
    ly, lv = orc.layernorm(x, 1)
    dout = rng.standard_normal((m_, c_)).astype(np.float32)
    tly, tlv, td = T(M, ly), T(M, lv), T(M, dout)
    dy = rt.__mul_bwd_a(td.h, tly.h, tw.h)
    tdw = T(M, dout * w)                                              # the eager product
    np.testing.assert_array_equal(M.Tensor(rt.__layernorm_bwd(tly.h, tlv.h, dy, 1)).numpy(),
                                  M.Tensor(rt.__layernorm_bwd(tly.h, tlv.h, tdw.h, 1)).numpy())
    np.testing.assert_array_equal(np_of(M, dy), dout * w)
    # the gain gradient: column sums of dout * y, bit-equal to summing the product
    dw = M.Tensor(rt.__mul_bwd_b(td.h, tly.h, tw.h)).numpy()
    prod = T(M, dout * ly)
    ones_c = T(M, np.zeros(c_, np.float32))
    ref = M.Tensor(rt.__sum_to_shape_bwd(prod.h, ones_c.h)).numpy()
    np.testing.assert_array_equal(dw, ref)
    assert np.allclose(dw, (dout.astype(np.float64) * ly).sum(axis=0), rtol=0, atol=1e-5 * np.abs(dout * ly).sum(axis=0).max())
    for h in (xn, xn2, dy):
        rt.tensor_release(h)


def test_causal_zero_gemms_equal_full(M, rt, rng):
    """softmax(qk * s + causal mask) is exactly 0 above the diagonal, and so is
    its VJP; GEMMs that read them as their A operand (P V, P^T dO, dS K) skip
    those K blocks.  The results equal the same GEMMs on untagged copies of the
    same values (the skipped products are exact zeros)."""
    Z, T_, hs = 24, 256, 64
    qk = (rng.standard_normal((Z, T_, T_)) * 3).astype(np.float32)
    v = rng.standard_normal((Z, T_, hs)).astype(np.float32)
    g = rng.standard_normal((Z, T_, hs)).astype(np.float32)
    tq, tv, tg = T(M, qk), T(M, v), T(M, g)
    ts = T(M, np.array([[0.125]], np.float32))
    mask = rt.tensor_causal_mask(T_)
    sc = rt.__broadcast_mul_fwd(tq.h, ts.h)
    ms = rt.__broadcast_add_fwd(sc, mask)
    p = rt.__softmax_fwd(ms, 2)
    pn = np_of(M, p)
    assert np.all(pn[:, np.triu_indices(T_, 1)[0], np.triu_indices(T_, 1)[1]] == 0.0)
    tp_plain = T(M, pn)                                   # the same values, no tag
    np.testing.assert_array_equal(M.Tensor(rt.tensor_matmul(p, tv.h)).numpy(),
                                  M.Tensor(rt.tensor_matmul(tp_plain.h, tv.h)).numpy())
    np.testing.assert_array_equal(M.Tensor(rt.__matmul_bwd_b(p, tv.h, tg.h)).numpy(),
                                  M.Tensor(rt.__matmul_bwd_b(tp_plain.h, tv.h, tg.h)).numpy())
    # the clipped products above cached only the planes they read; P as the
    # B operand of an unclipped product needs (and gets) all of them
    xw = T(M, rng.standard_normal((Z, hs, T_)).astype(np.float32))
    np.testing.assert_array_equal(M.Tensor(rt.tensor_matmul(xw.h, p)).numpy(),
                                  M.Tensor(rt.tensor_matmul(xw.h, tp_plain.h)).numpy())
    dp = T(M, rng.standard_normal((Z, T_, T_)).astype(np.float32))
    ds = rt.__softmax_bwd(p, dp.h, 2)
    dsn = np_of(M, ds)
    # the VJP of a tagged P skips the zero half: the same values as over an untagged copy
    np.testing.assert_array_equal(dsn, M.Tensor(rt.__softmax_bwd(tp_plain.h, dp.h, 2)).numpy())
    assert np.all(dsn[:, np.triu_indices(T_, 1)[0], np.triu_indices(T_, 1)[1]] == 0.0)
    dsc = rt.__mul_bwd_a(ds, tq.h, ts.h)                  # deferred ds * s, still zero above the diagonal
    plain = T(M, dsn * np.float32(0.125))
    qq = T(M, rng.standard_normal((Z, T_, hs)).astype(np.float32))   # scores = Q @ K^T
    kk = T(M, rng.standard_normal((Z, T_, hs)).astype(np.float32))
    kt = rt.tensor_permute(kk.h, (C.c_size_t * 3)(0, 2, 1), 3)
    np.testing.assert_array_equal(M.Tensor(rt.__matmul_bwd_a(qq.h, kt, dsc)).numpy(),
                                  M.Tensor(rt.__matmul_bwd_a(qq.h, kt, plain.h)).numpy())
    # dS itself (tagged, unscaled) as the A of a clipped product: its planes are
    # split only where the 128-row tiles read them
    ds_plain = T(M, dsn)
    np.testing.assert_array_equal(M.Tensor(rt.tensor_matmul(ds, kk.h)).numpy(),
                                  M.Tensor(rt.tensor_matmul(ds_plain.h, kk.h)).numpy())
    for h in (mask, sc, ms, p, ds, dsc, kt):
        rt.tensor_release(h)


def test_gelu_results_carry_their_planes(M, rt, rng):
    """GELU and its VJP at a GEMM's output (the MLP's pre-activation) write the
    tf32 planes of their large results as they store them, for the GEMMs that
    read them next (the MLP's down product and both VJPs of the up product).  Those GEMMs equal the same GEMMs over copies of the
    values, whose planes the operand split makes."""
    m_, c4, c_ = 2048, 1536, 384
    w2 = rng.standard_normal((c4, c_)).astype(np.float32)
    g2 = rng.standard_normal((m_, c_)).astype(np.float32)
    dh_in = rng.standard_normal((m_, c4)).astype(np.float32)
    xn = rng.standard_normal((m_, c_)).astype(np.float32)
    w1 = (rng.standard_normal((c_, c4)) * 0.1).astype(np.float32)
    tw2, tg2, tdh, txn, tw1 = (T(M, a) for a in (w2, g2, dh_in, xn, w1))
    tx = M.Tensor(rt.tensor_matmul(txn.h, tw1.h))          # the pre-activation: a GEMM's output
    h = rt.__gelu_fwd(tx.h)
    d = rt.__gelu_bwd(tx.h, tdh.h)
    got = [M.Tensor(rt.tensor_matmul(h, tw2.h)).numpy(), M.Tensor(rt.__matmul_bwd_b(h, tw2.h, tg2.h)).numpy(),
           M.Tensor(rt.__matmul_bwd_a(txn.h, tw1.h, d)).numpy(), M.Tensor(rt.__matmul_bwd_b(txn.h, tw1.h, d)).numpy()]
    hc, dc = T(M, np_of(M, h)), T(M, np_of(M, d))
    ref = [M.Tensor(rt.tensor_matmul(hc.h, tw2.h)).numpy(), M.Tensor(rt.__matmul_bwd_b(hc.h, tw2.h, tg2.h)).numpy(),
           M.Tensor(rt.__matmul_bwd_a(txn.h, tw1.h, dc.h)).numpy(),
           M.Tensor(rt.__matmul_bwd_b(txn.h, tw1.h, dc.h)).numpy()]
    for a, b in zip(got, ref):
        np.testing.assert_array_equal(a, b)
    for hh in (h, d):
        rt.tensor_release(hh)
