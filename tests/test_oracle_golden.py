"""CPU: pin the oracle against the reference's own known answers
(tests/golden/reference_golden.json, transcribed with file:line citations)."""
import json
from pathlib import Path

import numpy as np
import pytest

from conftest import rel_err

G = json.loads((Path(__file__).parent / "golden" / "reference_golden.json").read_text())


def test_matmul_golden(orc):
    g = G["matmul_2x3_3x2"]
    np.testing.assert_array_equal(orc.matmul(g["a"], g["b"]), np.array(g["out"], np.float32))
    g = G["matmul_ones"]
    out = orc.matmul(np.ones(g["a_shape"]), np.ones(g["b_shape"]))
    assert np.all(out == g["value"])


def test_broadcast_golden(orc):
    g = G["broadcast_rank_expansion"]
    out = orc.broadcast(0, np.full(g["a_shape"], g["a_fill"]), np.array(g["b"]))
    assert out.shape == (4, 8)
    assert np.all(out == np.array(g["row"], np.float32)[None, :])
    g = G["broadcast_sub_row"]
    out = orc.broadcast(1, np.array(g["a"]), np.full(g["b_shape"], g["b_fill"]))
    assert out.shape == (3, 4)
    assert np.all(out == np.array(g["out_row"], np.float32)[None, :])


@pytest.mark.parametrize("name,op,axis,keep", [
    ("reduce_sum_axis0", 0, 0, False), ("reduce_sum_axis1_keepdim", 0, 1, True),
    ("reduce_mean_axis0", 1, 0, False), ("reduce_max_axis1", 2, 1, False),
    ("reduce_var_axis0", 3, 0, False)])
def test_reduce_golden(orc, name, op, axis, keep):
    g = G[name]
    out = orc.reduce(op, np.array(g["x"]), axis, keep)
    np.testing.assert_allclose(out, np.array(g["out"], np.float32), rtol=1e-6)


def test_embedding_golden(orc):
    w = np.arange(12, dtype=np.float32).reshape(4, 3)
    for k in ("embedding_fwd_i32", "embedding_fwd_i64"):
        g = G[k]
        np.testing.assert_array_equal(orc.embedding(w, g["idx"]).ravel(), np.array(g["out"], np.float32))
    g = G["embedding_vjp"]
    dw = orc.embedding_bwd(np.ones((len(g["idx"]), g["dim"])), g["idx"], g["vocab"])
    np.testing.assert_array_equal(dw.ravel(), np.array(g["gw"], np.float32))


def test_vjp_golden(orc):
    # softmax/layernorm VJPs against central finite differences of the oracle forward
    rng = np.random.default_rng(0)
    x = rng.standard_normal((3, 7)).astype(np.float64)
    w = rng.standard_normal((3, 7))
    def f_sm(z):
        return float(np.sum(orc.softmax(z, 1).astype(np.float64) * w))
    s = orc.softmax(x, 1)
    an = orc.softmax_bwd(s, w, 1)
    eps = 1e-2
    for i, j in [(0, 0), (1, 3), (2, 6)]:
        zp, zm = x.copy(), x.copy()
        zp[i, j] += eps
        zm[i, j] -= eps
        fd = (f_sm(zp) - f_sm(zm)) / (2 * eps)
        assert abs(fd - an[i, j]) < 2e-3
    y, var = orc.layernorm(x, 1)
    an = orc.layernorm_bwd(y, var, w, 1)
    def f_ln(z):
        return float(np.sum(orc.layernorm(z, 1)[0].astype(np.float64) * w))
    for i, j in [(0, 1), (2, 5)]:
        zp, zm = x.copy(), x.copy()
        zp[i, j] += eps
        zm[i, j] -= eps
        fd = (f_ln(zp) - f_ln(zm)) / (2 * eps)
        assert abs(fd - an[i, j]) < 5e-3


def test_xor_readme_golden(orc):
    g = G["xor_10k"]
    loss, preds = orc.xor_train(10000, 1.5)
    assert abs(loss - g["loss"]) / g["loss"] < g["rtol"]
    assert rel_err(preds, g["preds"]) < g["rtol"]


def test_philox_randn_properties(orc):
    # metal.rs:1715-1737: N(0,1); deterministic per call index; distinct keys differ
    a = orc.randn((64, 64), 0)
    b = orc.randn((64, 64), 0)
    c = orc.randn((64, 64), 1)
    np.testing.assert_array_equal(a, b)
    assert not np.array_equal(a, c)
    assert abs(float(a.mean())) < 0.1 and abs(float(a.std()) - 1) < 0.05
    ints = [orc.rand_int(65, k) for k in range(2000)]
    assert min(ints) == 0 and max(ints) == 64
    u = [orc.rand_uniform(k) for k in range(100)]
    assert all(0.0 <= v < 1.0 for v in u)


def test_gelu_constants(orc):
    x = np.linspace(-5, 5, 101).astype(np.float32)
    y = orc.unary("gelu", x).astype(np.float64)
    xd = x.astype(np.float64)
    ref = 0.5 * xd * (1 + np.tanh(0.7978845608028654 * (xd + 0.044715 * xd ** 3)))
    assert np.max(np.abs(y - ref)) < 1e-5


def test_adamw_matches_composed_numpy(orc):
    rng = np.random.default_rng(3)
    p = rng.standard_normal(1000).astype(np.float32)
    g = rng.standard_normal(1000).astype(np.float32)
    m = np.zeros(1000, np.float32)
    v = np.zeros(1000, np.float32)
    p0 = p.copy()
    orc.adamw(p, g, m, v, 1e-3, 0.9, 0.99, 1e-8, 0.1, 1)
    f = np.float32
    gg = g + f(0.1) * p0
    mm = f(0.9) * f(0) + f(1 - np.float32(0.9)) * gg
    vv = f(0.99) * f(0) + (f(1 - np.float32(0.99)) * gg) * gg
    bc1 = f(1) - np.power(f(0.9), f(1))
    bc2 = f(1) - np.power(f(0.99), f(1))
    pp = p0 - (f(1e-3) * (mm / bc1)) / (np.sqrt(vv / bc2) + f(1e-8))
    np.testing.assert_array_equal(p, pp.astype(np.float32))


def test_gpt_oracle_loss_decreases(orc):
    # reference metal_integration.rs:1385-1432: loss[9] < 0.9 * loss[0] on a fixed batch
    g = orc.Gpt(65, 1, 2, 32, 16, 4, lr=3e-3)
    rng = np.random.default_rng(0)
    x = rng.integers(0, 65, 64)
    y = rng.integers(0, 65, 64)
    losses = [g.step(x, y) for _ in range(10)]
    g.close()
    assert losses[9] < 0.9 * losses[0]
    assert abs(losses[0] - np.log(65)) < 0.2
