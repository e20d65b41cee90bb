"""Data parallelism, host side: one process per GPU.

The training step all-reduces its gradients over NCCL inside the library
(`malus_dp_*`, dp.cu: one communicator, per-layer buckets issued as soon as a
layer's backward is done, AdamW applies 1/world).  This module holds what
surrounds that on the host:

* `init_data_parallel` — rank 0 makes the 128-byte NCCL unique id, the other
  ranks receive it over torch.distributed, every rank joins the communicator
  with a bounded wait;
* `shard_tokens` — per-rank token ids from rank-offset seeds (the batch is per
  GPU, so the job weak-scales and each rank's data is reproducible);
* `Liveness` — before a step every rank posts its step number in the
  rendezvous store and waits, bounded, for every peer's; a rank that has left
  (clean exit: a `left` key) or stopped answering is reported as `PeerLost` on
  the host before any collective of that step is launched, so no NCCL kernel
  is left waiting for it.

The reference has no multi-device layer; the bucket layout it would all-reduce
is `malus_gpt_dp_buckets` (host-only, tested without a GPU).
"""
from __future__ import annotations

import ctypes as C
import time
from datetime import timedelta

import numpy as np


class PeerLost(RuntimeError):
    """A data-parallel peer left or did not reach the same step in time."""


def exchange_unique_id(make_id, rank: int, group=None) -> bytes:
    """Rank 0 calls `make_id()` (128 bytes); every rank returns rank 0's bytes."""
    import torch.distributed as dist
    obj = [make_id() if rank == 0 else None]
    dist.broadcast_object_list(obj, src=0, group=group)
    idb = obj[0]
    if not isinstance(idb, (bytes, bytearray)) or len(idb) != 128:
        raise RuntimeError("malformed NCCL unique id received")
    return bytes(idb)


def nccl_id_maker(lib):
    def make() -> bytes:
        buf = (C.c_uint8 * 128)()
        if lib.malus_dp_unique_id(buf) != 0:
            raise RuntimeError("ncclGetUniqueId failed")
        return bytes(buf)
    return make


def init_data_parallel(lib, rank: int, world: int, timeout_ms: int = 60000, group=None) -> None:
    """Join the library's NCCL communicator (no-op for world 1)."""
    if world <= 1:
        return
    idb = exchange_unique_id(nccl_id_maker(lib), rank, group)
    rc = lib.malus_dp_init(rank, world, (C.c_uint8 * 128)(*idb), timeout_ms)
    if rc != 0:
        raise RuntimeError(f"malus_dp_init failed on rank {rank}: {rc}")


def shard_tokens(seed: int, rank: int, vocab: int, tokens_per_step: int, steps: int):
    """(x, y) int32 arrays [steps, tokens_per_step] for one rank: uniform ids
    from a generator keyed by (seed, rank)."""
    rng = np.random.default_rng([seed, rank])
    xs = rng.integers(0, vocab, (steps, tokens_per_step)).astype(np.int32)
    ys = rng.integers(0, vocab, (steps, tokens_per_step)).astype(np.int32)
    return xs, ys


class Liveness:
    """Step-level liveness through a torch.distributed store.

    `check(step)` posts `<prefix>/live/<step>/<rank>` and polls until every
    rank's key of that step exists; a `<prefix>/left/<r>` key (posted by
    `leave()`) or the timeout raises `PeerLost`."""

    def __init__(self, store, rank: int, world: int, timeout_s: float = 30.0, prefix: str = "malus",
                 poll_s: float = 0.005):
        self.store, self.rank, self.world = store, rank, world
        self.timeout_s, self.prefix, self.poll_s = timeout_s, prefix, poll_s

    def _live(self, step: int, r: int) -> str:
        return f"{self.prefix}/live/{step}/{r}"

    def _left(self, r: int) -> str:
        return f"{self.prefix}/left/{r}"

    def check(self, step: int) -> None:
        if self.world <= 1:
            return
        self.store.set(self._live(step, self.rank), "1")
        peers = [r for r in range(self.world) if r != self.rank]
        t0 = time.monotonic()
        while True:
            if all(self.store.check([self._live(step, r)]) for r in peers):
                return
            gone = [r for r in peers if self.store.check([self._left(r)])]
            if gone:
                raise PeerLost(f"rank {self.rank}: rank(s) {gone} left before step {step}")
            if time.monotonic() - t0 > self.timeout_s:
                missing = [r for r in peers if not self.store.check([self._live(step, r)])]
                raise PeerLost(f"rank {self.rank}: rank(s) {missing} did not reach step {step} "
                               f"within {self.timeout_s:.1f} s")
            time.sleep(self.poll_s)

    def leave(self) -> None:
        """Announce a clean exit (between steps, nothing in flight)."""
        self.store.set(self._left(self.rank), "1")


def store_timeout(seconds: float) -> timedelta:
    return timedelta(seconds=seconds)
