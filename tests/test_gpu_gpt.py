"""GPU: the nanoGPT training step (malus_gpt_*) against the CPU oracle's
restatement of the same step, from identical seeded initial weights and
token ids.  Bar: loss curves within 0.5% per step."""
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TOY = dict(vocab=65, n_layer=2, n_head=4, n_embd=64, block_size=32, batch=4)
C3 = dict(vocab=65, n_layer=4, n_head=4, n_embd=128, block_size=64, batch=16)
# shapes the fused attention kernels take (T % 128 == 0; hs 64 and 32)
A128 = dict(vocab=65, n_layer=2, n_head=2, n_embd=128, block_size=128, batch=2)
A256 = dict(vocab=65, n_layer=1, n_head=4, n_embd=128, block_size=256, batch=2)


def batches(cfg, n, seed=7):
    rng = np.random.default_rng(seed)
    m = cfg["batch"] * cfg["block_size"]
    return [(rng.integers(0, cfg["vocab"], m).astype(np.int32),
             rng.integers(0, cfg["vocab"], m).astype(np.int32)) for _ in range(n)]


def check_params(pg, po, lr):
    """Parameters after several AdamW steps.  Adam moves an element by about
    lr * g / (|g| + eps); an element whose gradient cancels to within rounding of
    zero takes a step of up to ~lr in either direction, and in a model with
    millions of elements a few always do.  So: each tensor within 1e-4 normwise,
    at most 1e-4 of the elements off by more than a quarter step, none by more
    than two steps.  Gradients themselves are checked tightly in
    test_gradients_match_oracle."""
    for i, (a, b) in enumerate(zip(pg, po)):
        d = np.abs(a.ravel().astype(np.float64) - b)
        assert np.linalg.norm(d) / np.linalg.norm(b) < 1e-4, (i, np.linalg.norm(d) / np.linalg.norm(b))
        assert np.mean(d > 0.25 * lr) <= 1e-4, (i, np.mean(d > 0.25 * lr))
        assert d.max() < 2 * lr, (i, d.max())


def run_pair(M, orc, cfg, steps, mode, lr=3e-4, tied=False, use_graph=0, **opt):
    """opt: optimizer / init settings (beta1, beta2, eps, wd, ...) given to both sides."""
    orc.set_threads(os.cpu_count())
    g = M.GPT(**cfg, tied=tied, lr=lr, mode=mode, use_graph=use_graph, **opt)
    o = orc.Gpt(**cfg, tied=tied, lr=lr, **opt)
    init_g = g.params()
    init_o = o.params()
    for a, b in zip(init_g, init_o):
        np.testing.assert_array_equal(a.ravel(), b)   # identical Philox init
    lg, lo = [], []
    for x, y in batches(cfg, steps):
        lg.append(g.step(x, y))
        lo.append(o.step(x, y))
    pg, po = g.params(), o.params()
    g.close()
    o.close()
    return np.array(lg), np.array(lo), pg, po


@pytest.mark.parametrize("tied", [False, True])
def test_tape_mode_matches_oracle(M, orc, tied):
    lg, lo, pg, po = run_pair(M, orc, TOY, 8, mode=0, lr=1e-3, tied=tied)
    assert np.all(np.abs(lg - lo) / lo < 5e-3), (lg, lo)
    assert abs(lg[0] - lo[0]) / lo[0] < 1e-5
    check_params(pg, po, lr=1e-3)


def test_tape_mode_c3_loss_curve(M, orc):
    # 200 steps: the loss-curve bar (<= 0.5 % per step over 200 steps)
    steps = int(os.environ.get("MALUS_C3_STEPS", "200"))
    lg, lo, _, _ = run_pair(M, orc, C3, steps, mode=0, lr=3e-4)
    assert np.max(np.abs(lg - lo) / lo) < 5e-3, (lg, lo)


def test_tape_mode_loss_decreases(M):
    # reference metal_integration.rs:1385-1432: loss[9] < 0.9*loss[0] on a repeated batch
    g = M.GPT(**TOY, lr=3e-3, mode=0)
    x, y = batches(TOY, 1)[0]
    losses = [g.step(x, y) for _ in range(10)]
    g.close()
    assert losses[9] < 0.9 * losses[0]


@pytest.mark.parametrize("tied", [False, True])
def test_fused_mode_matches_oracle(M, orc, tied):
    lg, lo, pg, po = run_pair(M, orc, TOY, 8, mode=1, lr=1e-3, tied=tied)
    assert np.all(np.abs(lg - lo) / lo < 5e-3), (lg, lo)
    assert abs(lg[0] - lo[0]) / lo[0] < 1e-5
    check_params(pg, po, lr=1e-3)


def test_fused_mode_c3_loss_curve(M, orc):
    steps = int(os.environ.get("MALUS_C3_STEPS", "200"))
    lg, lo, _, _ = run_pair(M, orc, C3, steps, mode=1, lr=3e-4, use_graph=1)
    assert np.max(np.abs(lg - lo) / lo) < 5e-3, (lg, lo)
    assert lg[-1] < lg[0]                       # it trains


def test_fused_graph_c4_architecture(M, orc):
    """The bench's architecture (V65 L6 H6 C384 T256) through the fused step as a
    CUDA graph, at batch 2 so the CPU oracle finishes in seconds."""
    cfg = dict(vocab=65, n_layer=6, n_head=6, n_embd=384, block_size=256, batch=2)
    steps = int(os.environ.get("MALUS_C4_STEPS", "5"))
    lg, lo, pg, po = run_pair(M, orc, cfg, steps, mode=1, lr=1e-3, use_graph=1, wd=0.01, beta2=0.99)
    assert abs(lg[0] - lo[0]) / lo[0] < 1e-5, (lg, lo)
    assert np.max(np.abs(lg - lo) / lo) < 5e-3, (lg, lo)
    check_params(pg, po, lr=1e-3)


def test_fused_and_tape_modes_agree(M):
    cfg = dict(vocab=65, n_layer=2, n_head=2, n_embd=128, block_size=128, batch=2)
    a = M.GPT(**cfg, lr=1e-3, mode=0)
    b = M.GPT(**cfg, lr=1e-3, mode=1)
    for x, y in batches(cfg, 5, seed=11):
        la, lb = a.step(x, y), b.step(x, y)
        assert abs(la - lb) / la < 1e-4, (la, lb)
    check_params(b.params(), [p.ravel().astype(np.float64) for p in a.params()], lr=1e-3)
    a.close()
    b.close()


@pytest.mark.parametrize("mode", [0, 1])
@pytest.mark.parametrize("tied", [False, True])
@pytest.mark.parametrize("cfg", [TOY, C3, A128, A256], ids=["toy", "c3", "attn128", "attn256"])
def test_gradients_match_oracle(M, orc, cfg, tied, mode):
    """Every parameter's first-step gradient against the oracle's, normwise per tensor."""
    orc.set_threads(os.cpu_count())
    g = M.GPT(**cfg, tied=tied, lr=1e-3, mode=mode)
    o = orc.Gpt(**cfg, tied=tied, lr=1e-3)
    x, y = batches(cfg, 1)[0]
    g.step(x, y)
    o.step(x, y)
    for i, (a, b) in enumerate(zip(g.grads(), o.grads())):
        e = np.max(np.abs(a.ravel().astype(np.float64) - b)) / np.max(np.abs(b))
        assert e < 3e-5, (i, e)
    g.close()
    o.close()


@pytest.mark.parametrize("T", [64, 128])
@pytest.mark.parametrize("tied", [False, True])
def test_graph_replay_matches_eager_bitwise(M, tied, T):
    """The fused step captured once as a CUDA graph and replayed gives the same
    bits as launching it eagerly (same kernels, same arguments; the AdamW bias
    corrections come from a device step counter).  T = 128 runs the fused
    attention kernels, which are deterministic (no atomics)."""
    cfg = dict(vocab=65, n_layer=2, n_head=4, n_embd=128, block_size=T, batch=4)
    a = M.GPT(**cfg, lr=1e-3, mode=1, use_graph=0, tied=tied)
    b = M.GPT(**cfg, lr=1e-3, mode=1, use_graph=1, tied=tied)
    for x, y in batches(cfg, 6, seed=5):
        la, lb = a.step(x, y), b.step(x, y)
        assert la == lb, (la, lb)
    for pa, pb in zip(a.params(), b.params()):
        assert np.array_equal(pa, pb)
    a.close()
    b.close()


def test_graph_step_matches_oracle(M, orc):
    lg, lo, pg, po = run_pair(M, orc, TOY, 8, mode=1, lr=1e-3, use_graph=1)
    assert np.all(np.abs(lg - lo) / lo < 5e-3), (lg, lo)
    assert abs(lg[0] - lo[0]) / lo[0] < 1e-5
    check_params(pg, po, lr=1e-3)


def test_fused_wide_vocab_tied_matches_oracle(M, orc):
    """C5's vocabulary (50304, tied head) through the fused step: the block-per-row
    cross-entropy, the 50304-row LM head GEMMs and the large-vocab embedding VJP;
    other dimensions small so the oracle keeps up."""
    cfg = dict(vocab=50304, n_layer=1, n_head=2, n_embd=128, block_size=128, batch=2)
    lg, lo, pg, po = run_pair(M, orc, cfg, 3, mode=1, lr=1e-3, tied=True, use_graph=1)
    assert abs(lg[0] - lo[0]) / lo[0] < 1e-5, (lg, lo)
    assert np.max(np.abs(lg - lo) / lo) < 5e-3, (lg, lo)
    check_params(pg, po, lr=1e-3)


@pytest.mark.parametrize("tied", [False, True])
@pytest.mark.parametrize("cfg", [A128, A256], ids=["attn128", "attn256"])
def test_fused_attention_backward_gradients_match_oracle(M, orc, cfg, tied, monkeypatch):
    """The step with the fused attention backward (P recomputed from the
    forward's row statistics, MALUS_ATTN_BWD=1): first-step gradients against
    the oracle's, as for the GEMM backward."""
    monkeypatch.setenv("MALUS_ATTN_BWD", "1")
    orc.set_threads(os.cpu_count())
    g = M.GPT(**cfg, tied=tied, lr=1e-3, mode=1)
    o = orc.Gpt(**cfg, tied=tied, lr=1e-3)
    x, y = batches(cfg, 1)[0]
    g.step(x, y)
    o.step(x, y)
    for i, (a, b) in enumerate(zip(g.grads(), o.grads())):
        e = np.max(np.abs(a.ravel().astype(np.float64) - b)) / np.max(np.abs(b))
        assert e < 3e-5, (i, e)
    g.close()
    o.close()


def test_fused_attention_backward_graph_c4_architecture(M, orc, monkeypatch):
    """C4's architecture with the fused attention backward, replayed as a graph:
    losses and parameters track the oracle; graph replay is bitwise equal to
    eager launches."""
    monkeypatch.setenv("MALUS_ATTN_BWD", "1")
    cfg = dict(vocab=65, n_layer=6, n_head=6, n_embd=384, block_size=256, batch=2)
    lg, lo, pg, po = run_pair(M, orc, cfg, 4, mode=1, lr=1e-3, use_graph=1, wd=0.01, beta2=0.99)
    assert abs(lg[0] - lo[0]) / lo[0] < 1e-5, (lg, lo)
    assert np.max(np.abs(lg - lo) / lo) < 5e-3, (lg, lo)
    check_params(pg, po, lr=1e-3)
    small = dict(vocab=65, n_layer=2, n_head=4, n_embd=128, block_size=128, batch=4)
    a = M.GPT(**small, lr=1e-3, mode=1, use_graph=0)
    b = M.GPT(**small, lr=1e-3, mode=1, use_graph=1)
    for x, y in batches(small, 5, seed=5):
        la, lb = a.step(x, y), b.step(x, y)
        assert la == lb, (la, lb)
    for pa, pb in zip(a.params(), b.params()):
        assert np.array_equal(pa, pb)
    a.close()
    b.close()
