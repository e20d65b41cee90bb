"""GPU data parallelism (needs >= 2 GPUs; skipped otherwise).

* parity: 2 ranks x batch B agree with 1 GPU x batch 2B on the concatenated
  tokens (same math; only the summation order differs), for the fused step
  (per-layer gradient buckets) and for the tape replay (the backward walk
  averages each bucket of registered parameter gradients as soon as it is
  final, malus_dp_register_leaves), each eager and as a CUDA graph;
* a rank leaving between steps is detected on the host before the next
  step's collectives (no NCCL kernel waits for it), NVLS off."""
import os
import socket
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parent.parent
WORKER = ROOT / "tests" / "dp_worker.py"


def ngpu() -> int:
    import torch
    return torch.cuda.device_count()


needs2 = pytest.mark.skipif("ngpu() < 2", reason="needs 2 GPUs")


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def torchrun(mode, out, steps=3, timeout=240, graph=0, model_mode=1):
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    env.pop("MALUS_DEVICE", None)          # each rank binds its LOCAL_RANK
    cmd = ["timeout", "-k", "30", str(timeout), sys.executable, "-m", "torch.distributed.run",
           "--nnodes=1", "--nproc-per-node=2", "--master-addr", "127.0.0.1", "--master-port",
           str(free_port()), str(WORKER), "--mode", mode, "--out", str(out), "--steps", str(steps),
           "--graph", str(graph), "--model-mode", str(model_mode)]
    r = subprocess.run(cmd, env=env, cwd=ROOT, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]


@needs2
@pytest.mark.parametrize("graph", [0, 1])
@pytest.mark.parametrize("model_mode", [1, 0], ids=["fused", "tape"])
def test_dp2_matches_single_gpu_double_batch(M, tmp_path, graph, model_mode):
    from malus_b200.dist import shard_tokens
    sys.path.insert(0, str(ROOT / "tests"))
    from dp_worker import CFG
    steps = 4
    torchrun("parity", tmp_path, steps, graph=graph, model_mode=model_mode)
    l0, l1 = np.load(tmp_path / "losses0.npy"), np.load(tmp_path / "losses1.npy")
    p2 = np.load(tmp_path / "params0.npz")
    m = CFG["batch"] * CFG["block_size"]
    x0, y0 = shard_tokens(11, 0, CFG["vocab"], m, steps)
    x1, y1 = shard_tokens(11, 1, CFG["vocab"], m, steps)
    big = dict(CFG, batch=2 * CFG["batch"])
    g = M.GPT(**big, lr=1e-3, mode=model_mode)
    ls = [g.step(np.concatenate([x0[s], x1[s]]), np.concatenate([y0[s], y1[s]])) for s in range(steps)]
    p1 = g.params()
    g.close()
    for s in range(steps):
        assert abs(ls[s] - 0.5 * (l0[s] + l1[s])) / ls[s] < 1e-5, (s, ls, l0, l1)
    lr = 1e-3
    for i, a in enumerate(p1):
        b = p2[f"arr_{i}"]
        d = a.astype(np.float64) - b
        assert np.max(np.abs(d)) < 0.25 * lr, (i, np.max(np.abs(d)))
        assert np.linalg.norm(d) / np.linalg.norm(b) < 1e-4


@needs2
def test_departed_rank_detected_before_next_collective(tmp_path):
    torchrun("leave", tmp_path, timeout=180)
    assert (tmp_path / "rank1.txt").read_text() == "left after step 0"
    r0 = (tmp_path / "rank0.txt").read_text()
    assert r0.startswith("peerlost:") and "left before step 1" in r0, r0
