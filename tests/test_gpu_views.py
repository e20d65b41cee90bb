"""GPU: strided views (permute, reshapes of permuted tensors) and the GEMM
operand-plane cache.

A permute returns a view of its input's storage; reshapes of views stay views
where the memory allows (up to two radices per dimension); GEMMs read views
through their strides when they split operands; any other consumer sees
contiguous data (the view is materialised once).  Checked against numpy:
the attention head fold and unfold of nanogpt_modular.ml:48-60 through
tensor_matmul and both matmul VJPs, views read by host reads, elementwise ops
and reductions, reshapes that are and are not expressible as views, i32 views,
and operand planes reused across GEMMs (and dropped when the data changes)."""
import ctypes as C

import numpy as np
import pytest

from conftest import rel_err

pytestmark = pytest.mark.gpu


def T(M, a):
    return M.Tensor.from_numpy(np.ascontiguousarray(a))


def H(M, h):
    return M.Tensor(h)


def perm(rt, t, p):
    arr = (C.c_size_t * len(p))(*p)
    return rt.tensor_permute(t.h if hasattr(t, "h") else t, arr, len(p))


def reshape(rt, h, shape):
    arr = (C.c_size_t * len(shape))(*shape)
    return rt.tensor_reshape(h, arr, len(shape))


def mm_close(got, a, b):
    ref = np.matmul(a.astype(np.float64), b.astype(np.float64))
    scale = np.matmul(np.abs(a).astype(np.float64), np.abs(b).astype(np.float64))
    return rel_err(got, ref, scale)


def fold(rt, x, B, T_, H_, hs):
    """[B*T, C] -> reshape [B,T,H,hs] -> permute (0,2,1,3) -> reshape [B*H, T, hs]."""
    r = reshape(rt, x, [B, T_, H_, hs])
    p = perm(rt, r, [0, 2, 1, 3])
    out = reshape(rt, p, [B * H_, T_, hs])
    rt.tensor_release(r)
    rt.tensor_release(p)
    return out


def unfold(rt, y, B, T_, H_, hs):
    """[B*H, T, hs] -> reshape [B,H,T,hs] -> permute (0,2,1,3) -> reshape [B*T, C]."""
    r = reshape(rt, y, [B, H_, T_, hs])
    p = perm(rt, r, [0, 2, 1, 3])
    out = reshape(rt, p, [B * T_, H_ * hs])
    rt.tensor_release(r)
    rt.tensor_release(p)
    return out


@pytest.mark.parametrize("B,T_,H_,hs", [(2, 128, 3, 64), (4, 64, 4, 32), (1, 96, 2, 48)])
def test_attention_fold_through_matmuls(M, rt, rng, B, T_, H_, hs):
    C_ = H_ * hs
    q = rng.standard_normal((B * T_, C_)).astype(np.float32)
    k = rng.standard_normal((B * T_, C_)).astype(np.float32)
    v = rng.standard_normal((B * T_, C_)).astype(np.float32)
    tq, tk, tv = T(M, q), T(M, k), T(M, v)
    Q = fold(rt, tq.h, B, T_, H_, hs)
    K = fold(rt, tk.h, B, T_, H_, hs)
    V = fold(rt, tv.h, B, T_, H_, hs)
    Kt = perm(rt, K, [0, 2, 1])
    nq = q.reshape(B, T_, H_, hs).transpose(0, 2, 1, 3).reshape(B * H_, T_, hs)
    nk = k.reshape(B, T_, H_, hs).transpose(0, 2, 1, 3).reshape(B * H_, T_, hs)
    nv = v.reshape(B, T_, H_, hs).transpose(0, 2, 1, 3).reshape(B * H_, T_, hs)
    s = H(M, rt.tensor_matmul(Q, Kt))
    assert mm_close(s.numpy(), nq, nk.transpose(0, 2, 1)) < 1e-4
    p = rng.standard_normal((B * H_, T_, T_)).astype(np.float32)
    tp = T(M, p)
    av = rt.tensor_matmul(tp.h, V)
    assert mm_close(H(M, rt.tensor_matmul(tp.h, V)).numpy(), p, nv) < 1e-4
    ao = unfold(rt, av, B, T_, H_, hs)
    w = rng.standard_normal((C_, C_)).astype(np.float32)
    tw = T(M, w)
    proj = H(M, rt.tensor_matmul(ao, tw.h))
    nav = np.matmul(p.astype(np.float64), nv)
    nao = nav.reshape(B, H_, T_, hs).transpose(0, 2, 1, 3).reshape(B * T_, C_)
    assert rel_err(proj.numpy(), nao @ w, np.abs(nao) @ np.abs(w)) < 2e-4
    # the view itself, read on the host and by an elementwise op, is the unfolded data
    np.testing.assert_allclose(H(M, rt.__broadcast_add_fwd(ao, ao)).numpy(), 2 * nao, rtol=2e-5, atol=1e-4)
    for h in (Q, K, V, Kt, av, ao):
        rt.tensor_release(h)


@pytest.mark.parametrize("B,T_,H_,hs", [(2, 128, 3, 64), (4, 64, 2, 32)])
def test_matmul_vjps_with_view_operands(M, rt, rng, B, T_, H_, hs):
    """matmul_bwd_a / _b where the saved operands and the incoming gradient are
    views (the gradients of the head-folded Q, K, V flow back through the
    inverse permutes)."""
    C_ = H_ * hs
    a = rng.standard_normal((B * T_, C_)).astype(np.float32)
    g = rng.standard_normal((B * H_, T_, T_)).astype(np.float32)
    ta, tg = T(M, a), T(M, g)
    A = fold(rt, ta.h, B, T_, H_, hs)                 # [BH, T, hs] view
    At = perm(rt, A, [0, 2, 1])                       # [BH, hs, T] view
    na = a.reshape(B, T_, H_, hs).transpose(0, 2, 1, 3).reshape(B * H_, T_, hs)
    # S = A @ At ; dA_left = dS @ At^T, dAt = A^T @ dS
    da = H(M, rt.__matmul_bwd_a(A, At, tg.h)).numpy()
    assert mm_close(da, g, na) < 1e-4
    dat = H(M, rt.__matmul_bwd_b(A, At, tg.h)).numpy()
    assert mm_close(dat, na.transpose(0, 2, 1), g) < 1e-4
    # a gradient that is itself a view: dX [B*T, C] unfolded from a [BH, T, hs] tensor,
    # through both VJPs of X @ W
    y = rng.standard_normal((B * H_, T_, hs)).astype(np.float32)
    ty = T(M, y)
    dX = unfold(rt, ty.h, B, T_, H_, hs)
    ny = y.reshape(B, H_, T_, hs).transpose(0, 2, 1, 3).reshape(B * T_, C_)
    w = rng.standard_normal((C_, 3 * C_)).astype(np.float32)
    x = rng.standard_normal((B * T_, C_)).astype(np.float32)
    tw, tx = T(M, w), T(M, x)
    gw = rng.standard_normal((B * T_, 3 * C_)).astype(np.float32)
    tgw = T(M, gw)
    # dY of Y = X @ W where X's gradient is the view: dX @ ...
    d1 = H(M, rt.__matmul_bwd_a(tx.h, tw.h, tgw.h)).numpy()
    assert mm_close(d1, gw, w.T) < 1e-4
    w2 = rng.standard_normal((C_, C_)).astype(np.float32)
    tw2 = T(M, w2)
    d2 = H(M, rt.__matmul_bwd_a(tx.h, tw2.h, dX)).numpy()       # dX (view) @ W2^T
    assert mm_close(d2, ny, w2.T) < 1e-4
    d3 = H(M, rt.__matmul_bwd_b(tx.h, tw2.h, dX)).numpy()       # X^T @ dX (view)
    assert mm_close(d3, x.T, ny) < 1e-4
    # a transposed-gradient view (the K path: d(K^T) permuted back), read MN-major
    kt = rng.standard_normal((B * H_, hs, T_)).astype(np.float32)
    tkt = T(M, kt)
    dk = perm(rt, tkt.h, [0, 2, 1])
    dk4 = reshape(rt, dk, [B, H_, T_, hs])
    dk4p = perm(rt, dk4, [0, 2, 1, 3])
    dkf = reshape(rt, dk4p, [B * T_, C_])
    nk = kt.transpose(0, 2, 1).reshape(B, H_, T_, hs).transpose(0, 2, 1, 3).reshape(B * T_, C_)
    d4 = H(M, rt.__matmul_bwd_a(tx.h, tw2.h, dkf)).numpy()
    assert mm_close(d4, nk, w2.T) < 1e-4
    d5 = H(M, rt.__matmul_bwd_b(tx.h, tw2.h, dkf)).numpy()
    assert mm_close(d5, x.T, nk) < 1e-4
    np.testing.assert_array_equal(M.Tensor(dkf, owned=False).numpy(), nk)   # host read of the view
    for h in (A, At, dX, dk, dk4, dk4p, dkf):
        rt.tensor_release(h)


def test_reshapes_of_views(M, rt, rng):
    x = rng.standard_normal((2, 3, 4)).astype(np.float32)
    tx = T(M, x)
    # flatten of a 2-D transpose: one two-radix dim
    y = rng.standard_normal((6, 4)).astype(np.float32)
    ty = T(M, y)
    t1 = perm(rt, ty.h, [1, 0])
    f1 = reshape(rt, t1, [24])
    np.testing.assert_array_equal(H(M, f1).numpy(), y.T.reshape(24))
    # flatten of a full reversal: three atoms, not a view -> materialised
    t2 = perm(rt, tx.h, [2, 1, 0])
    f2 = reshape(rt, t2, [24])
    np.testing.assert_array_equal(H(M, f2).numpy(), x.transpose(2, 1, 0).reshape(24))
    # split and merge that stay views
    t3 = perm(rt, tx.h, [1, 0, 2])                      # [3, 2, 4]
    f3 = reshape(rt, t3, [3, 8])
    np.testing.assert_array_equal(H(M, f3).numpy(), x.transpose(1, 0, 2).reshape(3, 8))
    f4 = reshape(rt, t3, [3, 2, 2, 2])
    np.testing.assert_array_equal(H(M, f4).numpy(), x.transpose(1, 0, 2).reshape(3, 2, 2, 2))
    # a view of a view, then a reduction and a softmax over it
    t5 = perm(rt, t3, [2, 0, 1])                        # [4, 3, 2]
    ref5 = x.transpose(1, 0, 2).transpose(2, 0, 1)
    got = H(M, rt.__reduce_sum_fwd(t5, 1, 0)).numpy()
    assert rel_err(got, ref5.sum(axis=1), np.abs(ref5).sum(axis=1)) < 1e-6
    sm = H(M, rt.__softmax_fwd(t5, 2)).numpy()
    e = np.exp(ref5 - ref5.max(axis=2, keepdims=True))
    np.testing.assert_allclose(sm, e / e.sum(axis=2, keepdims=True), rtol=1e-6)
    assert rt.tensor_ndim(t5) == 3 and [rt.tensor_dim(t5, i) for i in range(3)] == [4, 3, 2]
    for h in (t1, t2, t3, t5):
        rt.tensor_release(h)


def test_int_view_materialises_for_a_gather(M, rt, rng):
    ids = rng.integers(0, 7, (5, 4)).astype(np.int32)
    w = rng.standard_normal((7, 8)).astype(np.float32)
    ti, tw = T(M, ids), T(M, w)
    it = perm(rt, ti.h, [1, 0])
    flat = reshape(rt, it, [20])
    out = H(M, rt.__embedding_fwd(tw.h, flat)).numpy()
    np.testing.assert_array_equal(out, w[ids.T.reshape(20)])
    rt.tensor_release(it)
    rt.tensor_release(flat)


def test_plane_cache_reuse_and_invalidation(M, rt, rng):
    """The same operand in several GEMMs reuses its planes; a host write or an
    AdamW update in place drops them, so later GEMMs see the new data."""
    a = rng.standard_normal((512, 256)).astype(np.float32)
    w = rng.standard_normal((256, 384)).astype(np.float32)
    ta, tw = T(M, a), T(M, w)
    r1 = H(M, rt.tensor_matmul(ta.h, tw.h)).numpy()
    r2 = H(M, rt.tensor_matmul(ta.h, tw.h)).numpy()
    np.testing.assert_array_equal(r1, r2)
    assert mm_close(r1, a, w) < 1e-4
    w2 = rng.standard_normal((256, 384)).astype(np.float32)
    rt.malus_tensor_write(tw.h, w2.ctypes.data_as(C.c_void_p), w2.nbytes)
    assert mm_close(H(M, rt.tensor_matmul(ta.h, tw.h)).numpy(), a, w2) < 1e-4
    g = rng.standard_normal(w2.shape).astype(np.float32)
    m = np.zeros_like(w2)
    v = np.zeros_like(w2)
    tg, tm, tv = T(M, g), T(M, m), T(M, v)
    hs = [(C.c_int64 * 1)(x.h) for x in (tw, tg, tm, tv)]
    rt.malus_adamw_multi(hs[0], hs[1], hs[2], hs[3], 1, 1e-2, 0.9, 0.99, 1e-8, 0.0, 1, 1.0)
    w3 = tw.numpy()
    assert not np.array_equal(w3, w2)
    assert mm_close(H(M, rt.tensor_matmul(ta.h, tw.h)).numpy(), a, w3) < 1e-4
