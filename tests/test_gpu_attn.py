"""GPU: the fused causal attention forward kernel against a float64 reference
of the reference's attention block (scale, -1e9 causal mask, softmax, P V)."""
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
    rc = rt.malus_attn_fwd(ptr(rt, hi), ptr(rt, lo), B, H, T, hs, np.float32(scale), ptr(rt, p_hi),
                           ptr(rt, p_lo), ptr(rt, o_hi), ptr(rt, o_lo))
    assert rc == 0
    assert rt.malus_device_error() == 0
    q, k, v = (qkv[i].astype(np.float64).reshape(B * H, T, hs) for i in range(3))
    s = np.einsum("ztd,zkd->ztk", q, k) * np.float32(scale)
    s = s + np.triu(np.full((T, T), -np.inf), 1)
    p = np.exp(s - s.max(-1, keepdims=True))
    p /= p.sum(-1, keepdims=True)
    o = np.einsum("ztk,zkd->ztd", p, v)
    got_p = p_hi.numpy().astype(np.float64) + p_lo.numpy()
    lower = np.tril(np.ones((T, T), bool))
    assert np.max(np.abs(got_p - p)[:, lower]) < 2e-6
    got_o = (o_hi.numpy().astype(np.float64) + o_lo.numpy()).reshape(B, T, H, hs).transpose(0, 2, 1, 3)
    ref_o = o.reshape(B, H, T, hs)
    scale_o = np.einsum("ztk,zkd->ztd", p, np.abs(v)).reshape(B, H, T, hs)
    assert np.max(np.abs(got_o - ref_o) / scale_o) < 1e-5


def test_attn_fwd_rejects_unsupported_shapes(M, rt):
    z = dev(M, np.zeros(16, np.float32))
    assert rt.malus_attn_fwd(ptr(rt, z), ptr(rt, z), 1, 1, 96, 64, 0.125, ptr(rt, z), ptr(rt, z), ptr(rt, z),
                             ptr(rt, z)) == -1
    assert rt.malus_attn_fwd(ptr(rt, z), ptr(rt, z), 1, 1, 128, 48, 0.125, ptr(rt, z), ptr(rt, z), ptr(rt, z),
                             ptr(rt, z)) == -1
