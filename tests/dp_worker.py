"""One data-parallel rank for tests/test_gpu_dp.py (run under torchrun).

  parity: a few training steps (fused, or the tape replay whose backward
          averages each bucket of parameter gradients as soon as it is final)
          on this rank's token shard; writes its losses and (rank 0) the final
          parameters.
  leave:  rank 1 finishes step 0 and leaves between steps (nothing in flight);
          rank 0 must learn of it on the host (Liveness) before launching any
          collective of step 1, abort its communicator locally and report.
"""
import argparse
import os
import sys
from datetime import timedelta
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))

CFG = dict(vocab=65, n_layer=2, n_head=4, n_embd=128, block_size=64, batch=4)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--mode", choices=["parity", "leave"], required=True)
    ap.add_argument("--out", required=True)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--graph", type=int, default=0)
    ap.add_argument("--model-mode", type=int, default=1)   # 0: tape (per-leaf bucketed all-reduce), 1: fused
    args = ap.parse_args()
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))

    import torch.distributed as dist
    import malus_b200 as M
    from malus_b200.dist import Liveness, PeerLost, init_data_parallel, shard_tokens

    dist.init_process_group("gloo", timeout=timedelta(seconds=60))
    lib = M.load()
    lib.malus_set_device(local)
    init_data_parallel(lib, rank, world, timeout_ms=30000)
    live = Liveness(dist.distributed_c10d._get_default_store(), rank, world, timeout_s=20.0,
                    prefix="dpw")
    m = CFG["batch"] * CFG["block_size"]
    xs, ys = shard_tokens(11, rank, CFG["vocab"], m, args.steps)
    g = M.GPT(**CFG, lr=1e-3, mode=args.model_mode, use_graph=args.graph)
    out = Path(args.out)
    if args.mode == "parity":
        losses = []
        for s in range(args.steps):
            live.check(s)
            losses.append(g.step(xs[s], ys[s]))
        np.save(out / f"losses{rank}.npy", np.array(losses))
        if rank == 0:
            np.savez(out / "params0.npz", *g.params())
        live.check(args.steps)            # nobody leaves while a peer may still be in a step
        g.close()
        lib.malus_dp_destroy()
        dist.destroy_process_group()
        return
    # leave
    live.check(0)
    g.step(xs[0], ys[0])                  # returns after this step's collectives completed
    if rank == 1:
        live.leave()
        g.close()
        lib.malus_dp_abort()
        (out / "rank1.txt").write_text("left after step 0")
        return
    try:
        live.check(1)
        g.step(xs[1], ys[1])
        result = "no failure detected"
    except PeerLost as e:
        lib.malus_dp_abort()
        result = f"peerlost: {e}"
    (out / "rank0.txt").write_text(result)
    g.close()


if __name__ == "__main__":
    main()
