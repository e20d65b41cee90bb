"""GPU: the fused causal attention kernels against a float64 reference of the
reference's attention block (scale, -1e9 causal mask, softmax, P V) and of its
VJP chain (bmm VJPs, softmax VJP, the scale)."""
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


def ptr(rt, t):
    return rt.malus_tensor_data(t.h)


@pytest.mark.parametrize("B,H,T,hs", [(2, 3, 256, 64), (1, 2, 128, 32), (2, 2, 384, 64), (3, 1, 256, 32)])
def test_attn_fwd_matches_reference(M, rt, rng, B, H, T, hs):
    qkv = (rng.standard_normal((3, B, H, T, hs)) * 0.5).astype(np.float32)
    src = dev(M, qkv)
    hi, lo = dev(M, np.zeros_like(qkv)), dev(M, np.zeros_like(qkv))
    rows = 3 * B * H * T
    rt.malus_tf32_split(ptr(rt, src), rows, hs, hs, 1, 0, ptr(rt, hi), ptr(rt, lo), hs)
    p_hi, p_lo = dev(M, np.zeros((B * H, T, T))), dev(M, np.zeros((B * H, T, T)))
    o_hi, o_lo = dev(M, np.zeros((B * T, H * hs))), dev(M, np.zeros((B * T, H * hs)))
    scale = 1.0 / np.sqrt(hs)
    stats = dev(M, np.zeros((B * H * T, 2)))
    rc = rt.malus_attn_fwd(ptr(rt, hi), ptr(rt, lo), B, H, T, hs, np.float32(scale), ptr(rt, p_hi),
                           ptr(rt, p_lo), ptr(rt, o_hi), ptr(rt, o_lo), ptr(rt, stats))
    assert rc == 0
    assert rt.malus_device_error() == 0
    q, k, v = (qkv[i].astype(np.float64).reshape(B * H, T, hs) for i in range(3))
    s = np.einsum("ztd,zkd->ztk", q, k) * np.float32(scale)
    s = s + np.triu(np.full((T, T), -np.inf), 1)
    m = s.max(-1, keepdims=True)
    p = np.exp(s - m)
    l = p.sum(-1, keepdims=True)
    p /= l
    o = np.einsum("ztk,zkd->ztd", p, v)
    st = stats.numpy().reshape(B * H, T, 2)
    # row max in base-2 units (scores times log2 e)
    assert np.max(np.abs(st[..., 0] - m[..., 0] * np.log2(np.e))) < 1e-5 * (1 + np.abs(m).max())
    assert np.max(np.abs(st[..., 1] * l[..., 0] - 1)) < 2e-6
    got_p = p_hi.numpy().astype(np.float64) + p_lo.numpy()
    lower = np.tril(np.ones((T, T), bool))
    assert np.max(np.abs(got_p - p)[:, lower]) < 2e-6
    got_o = (o_hi.numpy().astype(np.float64) + o_lo.numpy()).reshape(B, T, H, hs).transpose(0, 2, 1, 3)
    ref_o = o.reshape(B, H, T, hs)
    scale_o = np.einsum("ztk,zkd->ztd", p, np.abs(v)).reshape(B, H, T, hs)
    assert np.max(np.abs(got_o - ref_o) / scale_o) < 1e-5


@pytest.mark.parametrize("B,H,T,hs,with_p", [(2, 3, 256, 64, 1), (2, 3, 256, 64, 0), (1, 2, 128, 32, 1),
                                             (2, 2, 384, 64, 1), (3, 1, 256, 32, 0), (1, 1, 384, 32, 1)])
def test_resident_scores_kernel_equals_recomputing_kernel(M, rt, rng, B, H, T, hs, with_p):
    """For T <= 384 the scores of a query tile stay in tensor memory and are
    computed once; the kernel that recomputes them per pass must give the same
    bits (same products in the same order, same softmax expressions)."""
    qkv = (rng.standard_normal((3, B, H, T, hs)) * 0.7).astype(np.float32)
    src = dev(M, qkv)
    hi, lo = dev(M, np.zeros_like(qkv)), dev(M, np.zeros_like(qkv))
    rt.malus_tf32_split(ptr(rt, src), 3 * B * H * T, hs, hs, 1, 0, ptr(rt, hi), ptr(rt, lo), hs)
    scale = np.float32(1.0 / np.sqrt(hs))
    outs = []
    prev = rt.malus_attn_set_resident(1)
    try:
        for resident in (1, 0):
            rt.malus_attn_set_resident(resident)
            p_hi, p_lo = dev(M, np.zeros((B * H, T, T))), dev(M, np.zeros((B * H, T, T)))
            o_hi, o_lo = dev(M, np.zeros((B * T, H * hs))), dev(M, np.zeros((B * T, H * hs)))
            stats = dev(M, np.zeros((B * H * T, 2)))
            pp = (ptr(rt, p_hi), ptr(rt, p_lo)) if with_p else (None, None)
            assert rt.malus_attn_fwd(ptr(rt, hi), ptr(rt, lo), B, H, T, hs, scale, *pp, ptr(rt, o_hi),
                                     ptr(rt, o_lo), ptr(rt, stats)) == 0
            assert rt.malus_device_error() == 0
            outs.append([t.numpy() for t in (p_hi, p_lo, o_hi, o_lo, stats)])
    finally:
        rt.malus_attn_set_resident(prev)
    for a, b in zip(*outs):
        np.testing.assert_array_equal(a, b)
    assert np.all(np.isfinite(outs[0][2]))


def test_attn_fwd_rejects_unsupported_shapes(M, rt):
    z = dev(M, np.zeros(16, np.float32))
    zp = ptr(rt, z)
    assert rt.malus_attn_fwd(zp, zp, 1, 1, 96, 64, 0.125, zp, zp, zp, zp, None) == -1
    assert rt.malus_attn_fwd(zp, zp, 1, 1, 128, 48, 0.125, zp, zp, zp, zp, None) == -1
    assert rt.malus_attn_bwd(zp, zp, zp, zp, zp, zp, zp, zp, 1, 1, 96, 64, 0.125, zp, zp) == -1
    assert rt.malus_attn_bwd(zp, zp, zp, zp, zp, zp, zp, zp, 1, 1, 128, 48, 0.125, zp, zp) == -1


def split(M, rt, a, cols):
    """tf32 hi/lo planes of a float32 array (rows x cols)."""
    src = dev(M, a)
    hi, lo = dev(M, np.zeros_like(a)), dev(M, np.zeros_like(a))
    rows = a.size // cols
    rt.malus_tf32_split(ptr(rt, src), rows, cols, cols, 1, 0, ptr(rt, hi), ptr(rt, lo), cols)
    return hi, lo


@pytest.mark.parametrize("B,H,T,hs", [(2, 3, 256, 64), (1, 2, 128, 32), (2, 2, 384, 64), (1, 1, 512, 32)])
def test_attn_bwd_matches_reference(M, rt, rng, B, H, T, hs):
    """dq, dk, dv from the fused backward (P recomputed from the forward's row
    statistics, no P planes written) against float64 VJPs of the block."""
    qkv = (rng.standard_normal((3, B, H, T, hs)) * 0.5).astype(np.float32)
    dO = rng.standard_normal((B, H, T, hs)).astype(np.float32)
    hi, lo = split(M, rt, qkv, hs)
    dh, dl = split(M, rt, dO, hs)
    C = H * hs
    o_hi, o_lo = dev(M, np.zeros((B * T, C))), dev(M, np.zeros((B * T, C)))
    stats = dev(M, np.zeros((B * H * T, 2)))
    scale = 1.0 / np.sqrt(hs)
    assert rt.malus_attn_fwd(ptr(rt, hi), ptr(rt, lo), B, H, T, hs, np.float32(scale), None, None,
                             ptr(rt, o_hi), ptr(rt, o_lo), ptr(rt, stats)) == 0
    D = dev(M, np.zeros(B * H * T))
    g_hi, g_lo = dev(M, np.zeros((3, B * T, C))), dev(M, np.zeros((3, B * T, C)))
    assert rt.malus_attn_bwd(ptr(rt, hi), ptr(rt, lo), ptr(rt, dh), ptr(rt, dl), ptr(rt, o_hi), ptr(rt, o_lo),
                             ptr(rt, stats), ptr(rt, D), B, H, T, hs, np.float32(scale), ptr(rt, g_hi),
                             ptr(rt, g_lo)) == 0
    assert rt.malus_device_error() == 0
    q, k, v = (qkv[i].astype(np.float64).reshape(B * H, T, hs) for i in range(3))
    do = dO.astype(np.float64).reshape(B * H, T, hs)
    s = np.einsum("ztd,zkd->ztk", q, k) * np.float32(scale)
    s = s + np.triu(np.full((T, T), -np.inf), 1)
    p = np.exp(s - s.max(-1, keepdims=True))
    p /= p.sum(-1, keepdims=True)
    dp = np.einsum("ztd,zkd->ztk", do, v)
    dd = (dp * p).sum(-1, keepdims=True)
    ds = p * (dp - dd) * np.float32(scale)
    ref = [np.einsum("ztk,zkd->ztd", ds, k), np.einsum("ztk,ztd->zkd", ds, q), np.einsum("ztk,ztd->zkd", p, do)]
    mag = p * (np.abs(dp) + np.abs(dd)) * np.float32(scale)
    bound = [np.einsum("ztk,zkd->ztd", mag, np.abs(k)), np.einsum("ztk,ztd->zkd", mag, np.abs(q)),
             np.einsum("ztk,ztd->zkd", p, np.abs(do))]
    got = (g_hi.numpy().astype(np.float64) + g_lo.numpy()).reshape(3, B, T, H, hs).transpose(0, 1, 3, 2, 4)
    np.testing.assert_allclose(D.numpy().reshape(B * H, T), dd[..., 0], rtol=1e-4, atol=1e-5)
    for i, name in enumerate(("dq", "dk", "dv")):
        g = got[i].reshape(B * H, T, hs)
        err = np.abs(g - ref[i]) / (bound[i] + 1e-30)
        assert np.max(err) < 2e-5, (name, np.max(err))
        assert np.linalg.norm(g - ref[i]) / np.linalg.norm(ref[i]) < 1e-5, name
