"""CPU, two gloo ranks: the multi-rank host paths.

* The vocabulary-sharded acceptance's exchange.  Every rank builds the same
  seeded logits and keeps one vocabulary shard; the partials, token logits
  and tie indices cross ranks through ``kernels.gather_shards`` (the
  function ``kernels.accept_sharded`` and ``bench.py --tp`` exchange with),
  and the oracle's shard merge must then reproduce the whole-row argmax, the
  target probabilities Mb and the accepted paths of the unsharded oracle, on
  every rank.  The GPU kernels of the same steps are checked against the
  unsharded kernels in test_gpu_tp.py.
* ``bench.over_ranks``: the max / min over ranks behind the benchmark's
  slowest-rank timing.
* A rank that leaves before the exchange: the other rank's
  ``gather_shards`` ends with an error within the process group's short
  timeout instead of waiting for good (the failure is made on the host; no
  kernel is involved).
"""
import datetime
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import accept as acc
from oracle.philox import UniformStream

WORLD = 2
V = 5000
BOUNDS = [0, 2049, V]                                    # unequal shards


def _inputs():
    from parallel_tree_spec_b200 import workload as wl
    rng = np.random.default_rng(17)
    trees = [wl.make_tree(rng, 4, 4, V) for _ in range(4)]
    x = np.concatenate([wl.make_logits(rng, t, V, plant=0.8, soft=True) for t in trees], 0)
    # every value equal: the max is in both shards, the smaller index wins
    x[1, :] = x[1, 0]
    # the max only in the second shard, the bf16 value just below it everywhere else: both round to
    # the same probability, so the argmax is the first column of the first shard
    m = np.float32(2.0 ** -10)
    x[5, :] = acc.f32_to_bf16_bits(acc._prev_bf16(np.array([m], np.float32)))[0]
    x[5, 3000:3010] = acc.f32_to_bf16_bits(np.array([m], np.float32))[0]
    # a max of 0: the value below it is the smallest negative bf16
    x[9, :] = acc.f32_to_bf16_bits(np.array([-1.0], np.float32))[0]
    x[9, 4000] = 0
    indptr = np.zeros(len(trees) + 1, dtype=np.int64)
    indptr[1:] = np.cumsum([t.size for t in trees])
    par = np.concatenate([t.parents for t in trees]).astype(np.int64)
    tok = np.concatenate([t.tokens for t in trees]).astype(np.int64)
    dp = np.concatenate([t.draft_probs for t in trees]).astype(np.float32)
    return x, indptr, par, tok, dp


def _sharded_stats(x, shard, indptr, par, tok, T):
    from parallel_tree_spec_b200.kernels import gather_shards
    lo, hi = BOUNDS[shard], BOUNDS[shard + 1]
    parts, tk = acc.shard_partials(x[:, lo:hi], lo, indptr, par, tok, T)
    m, s, first, flag, tm = acc.merge_shards(gather_shards(torch.from_numpy(parts)).numpy(),
                                             gather_shards(torch.from_numpy(tk)).numpy())
    ties = gather_shards(torch.from_numpy(acc.shard_ties(x[:, lo:hi], lo, m, s, flag, T))).numpy()
    assert ties.shape == (WORLD, x.shape[0])
    return acc.merged_row_argmax(first, flag, ties), acc.merged_mb(indptr, par, m, s, tm), flag


def _rank_main(rank, port):
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=WORLD,
                            timeout=datetime.timedelta(seconds=60))
    try:
        import bench
        assert bench.over_ranks([rank + 1.0, -rank], "max", "cpu") == [float(WORLD), 0.0]
        assert bench.over_ranks([rank + 1.0, -rank], "min", "cpu") == [1.0, float(1 - WORLD)]

        from parallel_tree_spec_b200.kernels import gather_shards
        x, indptr, par, tok, dp = _inputs()
        # shards in vocabulary order over the ranks, then reversed
        for T, shard in ((1.0, rank), (0.8, rank), (1.0, WORLD - 1 - rank)):
            am, mb, flag = _sharded_stats(x, shard, indptr, par, tok, T)
            ref_am, probs = acc.row_stats(x, T)
            assert np.array_equal(am, ref_am), np.nonzero(am != ref_am)
            assert flag[5] and flag[9] and not flag[1]
            assert am[1] == 0 and am[5] == 0 and am[9] == 4000
            for b in range(len(indptr) - 1):
                lo, hi = int(indptr[b]), int(indptr[b + 1])
                p, t = par[lo:hi], tok[lo:hi]
                ref_mb = acc.mb_from_probs(p, t, probs[lo:hi])
                assert np.array_equal(mb[lo + 1:hi], ref_mb[1:]), b
                if T == 1.0:
                    assert acc.greedy_walk(p, t, am[lo:hi]) == acc.greedy_walk(p, t, ref_am[lo:hi]), b
                got = acc.traversal_walk(p, t, dp[lo:hi], mb[lo:hi], am[lo:hi], UniformStream(3, 1, b))
                ref = acc.traversal_walk(p, t, dp[lo:hi], ref_mb, ref_am[lo:hi], UniformStream(3, 1, b))
                assert got == ref, b
            # every rank merged the same statistics
            everyone = gather_shards(torch.from_numpy(am)).numpy()
            assert all(np.array_equal(everyone[0], everyone[k]) for k in range(WORLD))
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.timeout(300)
def test_sharded_exchange_and_rank_reductions_two_gloo_ranks():
    mp.start_processes(_rank_main, args=(_free_port(),), nprocs=WORLD, start_method="spawn", join=True)


def _leaver_main(rank, port):
    import time
    # a long rendezvous timeout (spawned ranks import torch at different speeds), a short one for the exchange
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=WORLD,
                            timeout=datetime.timedelta(seconds=120))
    group = dist.new_group(list(range(WORLD)), timeout=datetime.timedelta(seconds=5))
    dist.barrier()
    if rank == 1:
        dist.destroy_process_group()                     # leaves between steps, before the exchange
        return
    from parallel_tree_spec_b200.kernels import gather_shards
    t0 = time.monotonic()
    try:
        gather_shards(torch.arange(8, dtype=torch.int32), group)
    except Exception:                                    # gloo: peer closed or timed out
        raised = True
    else:
        raised = False
    elapsed = time.monotonic() - t0
    assert raised, "the exchange completed without its peer"
    assert elapsed < 60.0, elapsed


@pytest.mark.timeout(300)
def test_exchange_with_a_rank_that_left_raises_instead_of_waiting():
    mp.start_processes(_leaver_main, args=(_free_port(),), nprocs=WORLD, start_method="spawn", join=True)


def test_gather_shards_without_a_process_group_is_one_shard():
    from parallel_tree_spec_b200.kernels import gather_shards
    t = torch.arange(6).view(3, 2)
    assert not dist.is_initialized()
    assert torch.equal(gather_shards(t), t.unsqueeze(0))
