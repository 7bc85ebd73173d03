"""One rank of the two-GPU sharded-acceptance test (launched by
tests/test_gpu_tp.py): every rank builds the same seeded inputs, keeps its
vocabulary shard, runs the NCCL exchange and checks that its accepted paths
equal the unsharded kernel's."""
import datetime
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

from parallel_tree_spec_b200 import kernels as K  # noqa: E402
from parallel_tree_spec_b200 import workload as wl  # noqa: E402


def main():
    rank, world = int(sys.argv[1]), int(sys.argv[2])
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        V = 128256
        rng = np.random.default_rng(5)
        trees = [wl.make_tree(rng, 8, 8, V) for _ in range(4)]
        x = np.concatenate([wl.make_logits(rng, t, V, plant=0.8, soft=True) for t in trees], 0)
        x[1, :] = x[1, 0]
        indptr, par, tok, dp = wl.stack_trees(trees)
        d = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
        xt = torch.from_numpy(x.view(np.int16)).to(dev).view(torch.bfloat16)
        step = V // world
        lo, hi = rank * step, (V if rank == world - 1 else (rank + 1) * step)
        got = K.accept_sharded(xt[:, lo:hi], lo, V, d(indptr), d(par), d(tok), d(dp), temperature=0.9, seed=3,
                               offset=1)
        ref = K.accept_traversal(xt, d(indptr), d(par), d(tok), d(dp), temperature=0.9, seed=3, offset=1)
        ok = torch.equal(got[2], ref[2])
        for b in range(len(trees)):
            n = int(ref[2][b, 0])
            ok = ok and torch.equal(got[0][b, :n], ref[0][b, :n]) and torch.equal(got[1][b, :n], ref[1][b, :n])
        torch.cuda.synchronize()
    finally:
        dist.destroy_process_group()
    sys.exit(0 if ok else 1)


if __name__ == "__main__":
    main()
