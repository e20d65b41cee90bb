"""GPU: the runtime's graph capture API (malus_graph_begin/end/replay/destroy)
and the tape-mode training step captured through it."""
import os
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parent.parent
_LIVE = []


@pytest.fixture(autouse=True)
def _free():
    yield
    _LIVE.clear()


def dev(M, a):
    t = M.Tensor.from_numpy(np.ascontiguousarray(a, np.float32))
    _LIVE.append(t)
    return t


def gelu(x):
    return 0.5 * x * (1 + np.tanh(0.7978845608028654 * (x + 0.044715 * x ** 3)))


def test_capture_and_replay_with_new_inputs(M, rt, rng):
    """matmul -> broadcast add -> GELU captured once; each replay after a
    malus_tensor_write of new inputs gives the new result."""
    a0 = rng.standard_normal((64, 48)).astype(np.float32)
    b = rng.standard_normal((48, 32)).astype(np.float32)
    bias = rng.standard_normal((1, 32)).astype(np.float32)
    a, bt, bb = dev(M, a0), dev(M, b), dev(M, bias)

    def seq():
        c = rt.tensor_matmul(a.h, bt.h)
        d = rt.__broadcast_add_fwd(c, bb.h)
        rt.tensor_release(c)
        e = rt.__gelu_fwd(d)
        rt.tensor_release(d)
        return e

    rt.tensor_release(seq())          # sizes every workspace before the capture
    rt.gpu_barrier()
    assert rt.malus_graph_begin() == 0
    e = seq()
    gid = rt.malus_graph_end()
    assert gid > 0
    out = M.Tensor(e)
    for _ in range(3):
        a_new = rng.standard_normal((64, 48)).astype(np.float32)
        rt.malus_tensor_write(a.h, a_new.ctypes.data, a_new.nbytes)
        assert rt.malus_graph_replay(gid) == 0
        ref = gelu(a_new.astype(np.float64) @ b + bias)
        np.testing.assert_allclose(out.numpy(), ref, rtol=1e-4, atol=1e-4)
    assert rt.malus_graph_replay(gid + 1000) == -1
    # the graph's buffers stay out of the pool while it exists: a tensor made
    # after the output is released does not get the output's buffer
    ptr = rt.malus_tensor_data(e)
    del out
    other = dev(M, np.zeros((64, 32)))
    assert rt.malus_tensor_data(other.h) != ptr
    assert rt.malus_graph_replay(gid) == 0   # still valid: writes its own buffers only
    rt.gpu_barrier()
    assert not np.any(other.numpy())
    assert rt.malus_graph_destroy(gid) == 0
    assert rt.malus_graph_destroy(gid) == -1


def test_host_read_inside_a_capture_aborts():
    """A host read between malus_graph_begin and malus_graph_end is an error the
    runtime reports (panic-only error model), not a silent wrong capture."""
    code = ("import numpy as np, malus_b200 as M\n"
            "rt = M.load()\n"
            "t = M.Tensor.from_numpy(np.ones((4, 4), np.float32))\n"
            "rt.malus_graph_begin()\n"
            "rt.malus_tensor_get_f32(t.h, 0)\n")
    r = subprocess.run([sys.executable, "-c", code], cwd=ROOT, capture_output=True, text=True, timeout=120)
    assert r.returncode != 0
    assert "during graph capture" in r.stderr, r.stderr[-2000:]


@pytest.mark.parametrize("tied", [False, True])
def test_tape_step_graph_matches_eager_bitwise(M, tied):
    """The reference's per-step call sequence (tape mode) captured through the
    graph API after one eager step and replayed: same losses and parameters,
    bit for bit, as launching every call (AdamW's step counter lives on the
    device, so every replay is a new step)."""
    sys.path.insert(0, str(ROOT / "tests"))
    from test_gpu_gpt import batches
    cfg = dict(vocab=65, n_layer=2, n_head=4, n_embd=64, block_size=32, batch=4)
    a = M.GPT(**cfg, lr=1e-3, mode=0, use_graph=0, tied=tied)
    b = M.GPT(**cfg, lr=1e-3, mode=0, use_graph=1, tied=tied)
    for x, y in batches(cfg, 6, seed=3):
        la, lb = a.step(x, y), b.step(x, y)
        assert la == lb, (la, lb)
    for pa, pb in zip(a.params(), b.params()):
        assert np.array_equal(pa, pb)
    a.close()
    b.close()
