"""GPU parity of the vocabulary-sharded (tensor-parallel) acceptance.

The sharded path (per-shard partials -> all-gather -> merge in shard order ->
tie exchange -> walk) must give the same accepted paths as the unsharded
kernels and the oracle.  One GPU emulates the shards (each shard is a column
slice of the same logits, the all-gather is a stack); a two-process NCCL run
covers the real exchange when two GPUs are visible.
"""
import os
import socket
import subprocess
import sys

import numpy as np
import pytest
import torch

from oracle import accept as acc
from parallel_tree_spec_b200 import kernels as K
from parallel_tree_spec_b200 import workload as wl

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _inputs(seed, n_trees, vocab, width=8, depth=8, constant_rows=0):
    rng = np.random.default_rng(seed)
    trees = [wl.make_tree(rng, width, depth, vocab) for _ in range(n_trees)]
    logits = [wl.make_logits(rng, t, vocab, plant=0.8, soft=True) for t in trees]
    x = np.concatenate(logits, 0)
    # rows of one repeated value: every token ties, the argmax needs the exchange
    for r in range(constant_rows):
        x[3 * r + 1, :] = x[3 * r + 1, 0]
    indptr, par, tok, dp = wl.stack_trees(trees)
    d = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(DEV)
    xt = torch.from_numpy(x.view(np.int16)).to(DEV).view(torch.bfloat16)
    return trees, x, xt, d(indptr), d(par), d(tok), d(dp)


def _sharded(xt, shards, indptr, par, tok, dp, T, seed, offset, bounds=None):
    """The sharded pipeline with the all-gathers emulated by stacking."""
    V = xt.shape[1]
    if bounds is None:
        step = V // shards
        bounds = [k * step for k in range(shards)] + [V]
    parts, toks = [], []
    for k in range(shards):
        p, t = K.accept_shard_partials(xt[:, bounds[k]:bounds[k + 1]], bounds[k], indptr, par, tok, T)
        parts.append(p)
        toks.append(t)
    stats, tokm = K.accept_merge_shards(torch.stack(parts), torch.stack(toks))
    ties = torch.stack([K.accept_shard_ties(xt[:, bounds[k]:bounds[k + 1]], bounds[k], stats, T)
                        for k in range(shards)])
    return K.accept_walk_merged(stats, tokm, ties, V, indptr, par, tok, dp, seed=seed, offset=offset)


def _same(a, b, B):
    ot, oh, oc = (t.cpu().numpy() for t in a)
    rt, rh, rc = (t.cpu().numpy() for t in b)
    assert np.array_equal(oc, rc), (oc, rc)
    for i in range(B):
        n = int(rc[i, 0])
        assert np.array_equal(ot[i, :n], rt[i, :n]) and np.array_equal(oh[i, :n], rh[i, :n]), i


@pytest.mark.parametrize("shards,T", [(2, 1.0), (8, 1.0), (8, 0.8)])
def test_sharded_matches_unsharded_traversal_and_greedy(shards, T):
    V = 128256
    trees, x, xt, indptr, par, tok, dp = _inputs(31 + shards, 6, V, constant_rows=2)
    B = len(trees)
    ref = K.accept_traversal(xt, indptr, par, tok, dp, temperature=T, seed=9, offset=2)
    got = _sharded(xt, shards, indptr, par, tok, dp, T, 9, 2)
    _same(got, ref, B)
    ref_g = K.accept_greedy(xt, indptr, par, tok)
    got_g = _sharded(xt, shards, indptr, par, tok, None, 1.0, 0, 0)
    _same(got_g, ref_g, B)


def test_sharded_unaligned_shards_and_oracle():
    """Shard widths that are not multiples of 8 take the per-chunk kernel;
    the greedy result is checked against the oracle as well."""
    V = 20000
    trees, x, xt, indptr, par, tok, dp = _inputs(7, 5, V, width=4, depth=5, constant_rows=1)
    bounds = [0, 6667, 13331, V]
    got = _sharded(xt, 3, indptr, par, tok, None, 1.0, 0, 0, bounds)
    ot, oh, oc = (t.cpu().numpy() for t in got)
    lo = 0
    for b, t in enumerate(trees):
        am, _ = acc.row_stats(x[lo:lo + t.size])
        s, h, tl, al = acc.greedy_walk(t.parents, t.tokens, am)
        n = int(oc[b, 0])
        assert ot[b, :n].tolist() == s and oh[b, :n].tolist() == list(h), b
        lo += t.size


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_sharded_over_nccl_two_ranks():
    env = dict(os.environ, MASTER_ADDR="127.0.0.1", MASTER_PORT=str(_free_port()), NCCL_NVLS_ENABLE="0")
    script = os.path.join(ROOT, "tests", "tp_worker.py")
    procs = [subprocess.Popen([sys.executable, script, str(r), "2"], env=env, cwd=ROOT) for r in range(2)]
    codes = [p.wait(timeout=300) for p in procs]
    assert codes == [0, 0], codes
