"""Data-parallel host logic on CPU: NCCL-id exchange, token shards, step
liveness (a departed or silent rank is reported before the next step's
collectives), and the fused-buffer layout / all-reduce buckets of the step,
exercised with world-size-2 gloo process groups.  No GPU is touched."""
import ctypes as C
import os
import socket
import sys
import time
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))

C4 = dict(vocab=65, n_layer=6, n_head=6, n_embd=384, block_size=256, batch=64)
C5 = dict(vocab=50304, n_layer=12, n_head=12, n_embd=768, block_size=1024, batch=8)


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port):
    import torch.distributed as dist
    from datetime import timedelta
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, timeout=timedelta(seconds=20))
    return dist


def _worker_unique_id(rank, world, port, out):
    dist = _init(rank, world, port)
    from malus_b200.dist import exchange_unique_id
    made = []

    def make():
        made.append(1)
        return bytes(np.random.default_rng(123).integers(0, 256, 128, dtype=np.uint8))

    idb = exchange_unique_id(make, rank)
    np.save(os.path.join(out, f"id{rank}.npy"), np.frombuffer(idb, np.uint8))
    np.save(os.path.join(out, f"made{rank}.npy"), np.array([len(made)]))
    dist.destroy_process_group()


def _worker_liveness(rank, world, port, out, mode):
    dist = _init(rank, world, port)
    from malus_b200.dist import Liveness, PeerLost
    store = dist.distributed_c10d._get_default_store()
    live = Liveness(store, rank, world, timeout_s=2.0, prefix="t")
    result = "ok"
    try:
        for step in range(4):
            if rank == 1 and step == 2 and mode != "all":
                if mode == "leave":
                    live.leave()
                result = "left"
                break          # rank 1 exits between steps; nothing in flight
            live.check(step)
    except PeerLost as e:
        result = f"peerlost:{step}:{e}"
    with open(os.path.join(out, f"live{rank}.txt"), "w") as f:
        f.write(result)
    # no collective after a loss: the process group is torn down locally
    if mode == "all":
        dist.destroy_process_group()


def spawn(fn, *args, world=2):
    import torch.multiprocessing as mp
    mp.start_processes(fn, args=(world,) + args, nprocs=world, start_method="spawn", join=True)


def test_unique_id_exchange(tmp_path):
    spawn(_worker_unique_id, free_port(), str(tmp_path))
    a, b = np.load(tmp_path / "id0.npy"), np.load(tmp_path / "id1.npy")
    assert a.shape == (128,) and np.array_equal(a, b)
    assert int(np.load(tmp_path / "made0.npy")[0]) == 1       # only rank 0 makes the id
    assert int(np.load(tmp_path / "made1.npy")[0]) == 0


def test_liveness_all_ranks_present(tmp_path):
    spawn(_worker_liveness, free_port(), str(tmp_path), "all")
    assert (tmp_path / "live0.txt").read_text() == "ok"
    assert (tmp_path / "live1.txt").read_text() == "ok"


@pytest.mark.parametrize("mode", ["leave", "silent"])
def test_liveness_detects_departed_rank(tmp_path, mode):
    t0 = time.monotonic()
    spawn(_worker_liveness, free_port(), str(tmp_path), mode)
    r0 = (tmp_path / "live0.txt").read_text()
    assert (tmp_path / "live1.txt").read_text() == "left"
    assert r0.startswith("peerlost:2:"), r0          # detected before step 2's collectives
    if mode == "leave":
        assert "left" in r0
    else:
        assert "did not reach step 2" in r0
    assert time.monotonic() - t0 < 60


def test_shards_distinct_and_reproducible():
    from malus_b200.dist import shard_tokens
    x0, y0 = shard_tokens(7, 0, 65, 4096, 3)
    x1, _ = shard_tokens(7, 1, 65, 4096, 3)
    x0b, y0b = shard_tokens(7, 0, 65, 4096, 3)
    assert x0.dtype == np.int32 and x0.shape == (3, 4096)
    assert np.array_equal(x0, x0b) and np.array_equal(y0, y0b)
    assert not np.array_equal(x0, x1)
    assert x0.min() >= 0 and x0.max() < 65


def layout(M, cfg, tied=False):
    lib = M.load()
    g = M.GptConfig(cfg["vocab"], cfg["n_layer"], cfg["n_head"], cfg["n_embd"], cfg["block_size"],
                    cfg["batch"], int(tied), 1e-3, 0.9, 0.99, 1e-8, 0.01, 0.02, 1, 0, 0)
    n = lib.malus_gpt_layout(C.byref(g), None, None, 0, None)
    offs, sizes, total = (C.c_int64 * n)(), (C.c_int64 * n)(), C.c_int64()
    assert lib.malus_gpt_layout(C.byref(g), offs, sizes, n, C.byref(total)) == n
    nb = lib.malus_gpt_dp_buckets(C.byref(g), None, None, 0)
    lo, hi = (C.c_int64 * nb)(), (C.c_int64 * nb)()
    assert lib.malus_gpt_dp_buckets(C.byref(g), lo, hi, nb) == nb
    return list(offs), list(sizes), total.value, list(zip(lo, hi))


@pytest.mark.parametrize("cfg,tied", [(C4, False), (C4, True), (C5, True)])
def test_layout_and_buckets(M, cfg, tied):
    offs, sizes, total, buckets = layout(M, cfg, tied)
    Cc, V, T, Lr = cfg["n_embd"], cfg["vocab"], cfg["block_size"], cfg["n_layer"]
    per_layer = 2 * Cc + 4 * Cc * Cc + 8 * Cc * Cc
    expect = Lr * per_layer + V * Cc + T * Cc + Cc + (0 if tied else Cc * V)
    assert sum(sizes) == expect
    assert len(sizes) == 8 * Lr + (3 if tied else 4)
    assert all(o % 64 == 0 for o in offs)                       # 256-byte aligned slices
    assert all(offs[i] + sizes[i] <= offs[i + 1] for i in range(len(offs) - 1))
    assert offs[-1] + sizes[-1] <= total
    # buckets: one per layer (last layer first) then the top; disjoint; every
    # parameter slice in exactly one bucket
    assert len(buckets) == Lr + 1
    for l in range(Lr):
        lo, hi = buckets[Lr - 1 - l]
        assert lo == offs[8 * l] and hi == offs[8 * l + 7] + sizes[8 * l + 7]
    covered = np.zeros(total, np.int32)
    for lo, hi in buckets:
        covered[lo:hi] += 1
    assert covered.max() == 1
    for o, s in zip(offs, sizes):
        assert covered[o:o + s].min() == 1


def test_c4_buffer_size(M):
    _, sizes, total, _ = layout(M, C4)
    assert abs(sum(sizes) - 10.77e6) / 10.77e6 < 0.01              # ≈ 10.77 M parameters
    assert abs(total * 4 / 1e6 - 43.1) < 0.3                        # ≈ 43.1 MB per fused buffer


def _worker_bucket_allreduce(rank, world, port, out):
    """The bucketed sum-all-reduce followed by 1/world equals the mean of the
    ranks' gradients exactly once per element (gloo stands in for NCCL)."""
    dist = _init(rank, world, port)
    import torch
    import malus_b200 as M
    _, _, total, buckets = layout(M, dict(vocab=65, n_layer=2, n_head=2, n_embd=64, block_size=32, batch=2))
    g = torch.from_numpy(np.random.default_rng(rank).standard_normal(total).astype(np.float32))
    mine = g.clone()
    for lo, hi in buckets:
        view = g[lo:hi]
        dist.all_reduce(view)
    g.mul_(1.0 / world)
    np.save(os.path.join(out, f"g{rank}.npy"), g.numpy())
    np.save(os.path.join(out, f"mine{rank}.npy"), mine.numpy())
    dist.destroy_process_group()


def test_bucketed_allreduce_is_mean(tmp_path):
    spawn(_worker_bucket_allreduce, free_port(), str(tmp_path))
    g0, g1 = np.load(tmp_path / "g0.npy"), np.load(tmp_path / "g1.npy")
    m0, m1 = np.load(tmp_path / "mine0.npy"), np.load(tmp_path / "mine1.npy")
    _, _, _, buckets = layout(__import__("malus_b200"), dict(vocab=65, n_layer=2, n_head=2, n_embd=64,
                                                              block_size=32, batch=2))
    assert np.array_equal(g0, g1)
    inside = np.zeros(g0.size, bool)
    for lo, hi in buckets:
        inside[lo:hi] = True
    np.testing.assert_allclose(g0[inside], ((m0 + m1) / 2)[inside], rtol=1e-6, atol=1e-7)
