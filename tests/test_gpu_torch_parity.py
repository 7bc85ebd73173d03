"""Acceptance arithmetic against the reference's own computation on the GPU.

The reference takes its probabilities from ``torch.softmax`` of the logits in
their own dtype on the device: ``_sample_probs(logits)`` for greedy
verification (``verification.py:55,213``) and ``_sample_probs(logits / T)``
for traversal (``verification.py:310-311``); the greedy choice is the first
index of the largest bf16 probability, the traversal's Mb is
``probs[parent, token]`` (``verification.py:349``).  The golden vectors pin
the kernels to the reference run on the CPU; this test measures them against
torch's CUDA softmax over about a million config-2-shaped rows
([1040, 128256] bf16 N(0, 3) batches), a tenth of them adversarial:

* near-uniform rows (N(0, 1e-3)), where many values share the largest rounded
  probability and the first-index rule decides;
* rows whose maximum appears several times;
* rows with child tokens planted at and just below the maximum.

It prints the mismatch counts of the per-row argmax and the per-node Mb, and
the accepted-path mismatch rate of traversal walks on a sample of the trees
(the kernel's walk against the oracle's walk fed with torch's Mb and argmax
and the same Philox draws).  Argmax mismatches must be zero.
"""
import os

import numpy as np
import pytest
import torch

from oracle import accept as acc
from oracle.philox import UniformStream
from parallel_tree_spec_b200 import kernels as K
from parallel_tree_spec_b200 import workload as wl

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
V = 128256
BATCHES = int(os.environ.get("PTS_PARITY_BATCHES", "960"))     # x 1040 rows
PATH_SAMPLE_BATCHES = 24


def _trees(seed):
    rng = np.random.default_rng(seed)
    trees = [wl.make_tree(rng, 8, 8, V) for _ in range(16)]
    indptr, par, tok, dp = wl.stack_trees(trees)
    d = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(DEV)
    parent_row = np.full(len(par), -1, np.int64)
    for b in range(16):
        lo = indptr[b]
        for i in range(indptr[b + 1] - lo):
            if par[lo + i] >= 0:
                parent_row[lo + i] = lo + par[lo + i]
    return trees, d(indptr), d(par), d(tok), d(dp), parent_row


def _logits(g, parent_row, tok):
    R = parent_row.shape[0]
    x = torch.randn(R, V, generator=g, device=DEV) * 3.0
    kind = torch.randint(0, 40, (R,), generator=g, device=DEV)
    flat = kind == 0                                           # near-uniform rows
    x[flat] = torch.randn(int(flat.sum()), V, generator=g, device=DEV) * 1e-3
    x = x.to(torch.bfloat16)
    dup = (kind == 1).nonzero().reshape(-1)                    # the maximum several times
    if dup.numel():
        m = x[dup].amax(dim=1, keepdim=True)
        cols = torch.randint(0, V, (dup.numel(), 4), generator=g, device=DEV)
        x[dup.unsqueeze(1), cols] = m.expand(-1, 4)
    # child tokens at the maximum and one bf16 step below it
    child = torch.from_numpy(np.nonzero(parent_row >= 0)[0]).to(DEV)
    pr = torch.from_numpy(parent_row[parent_row >= 0]).to(DEV)
    pick = torch.rand(child.numel(), generator=g, device=DEV) < 0.2
    child, pr = child[pick], pr[pick]
    m = x[pr].amax(dim=1)
    below = (m.view(torch.int16) - torch.where(m > 0, 1, -1).to(torch.int16)).view(torch.bfloat16)
    vals = torch.where(torch.rand(child.numel(), generator=g, device=DEV) < 0.5, m, below)
    x[pr, tok[child].long()] = vals
    return x


@pytest.mark.parametrize("method,temperature", [("exact", 1.0), ("traversal", 0.8)])
@torch.no_grad()
def test_row_argmax_and_mb_against_torch_softmax_on_cuda(method, temperature):
    trees, indptr, par, tok, dp, parent_row = _trees(11)
    g = torch.Generator(device=DEV)
    g.manual_seed(1234 if method == "exact" else 4321)
    nonroot = torch.from_numpy(np.nonzero(parent_row >= 0)[0]).to(DEV)
    prow = torch.from_numpy(parent_row[parent_row >= 0]).to(DEV)
    rows = am_bad = mb_bad = nodes = 0
    walks = path_bad = 0
    worst = 0.0
    for it in range(BATCHES):
        x = _logits(g, parent_row, tok)
        if method == "exact":
            ot, oh, oc = K.accept_greedy(x, indptr, par, tok, max_nodes=65)
        else:
            ot, oh, oc = K.accept_traversal(x, indptr, par, tok, dp, temperature=temperature, seed=9, offset=it,
                                            max_nodes=65)
        am, mb = K.accept_row_stats(x, indptr, par, tok, temperature=temperature)
        p = torch.softmax(x if temperature == 1.0 else x / temperature, dim=-1)   # the reference's arithmetic
        ref_am = p.argmax(dim=-1)
        ref_mb = p[prow, tok[nonroot].long()].float()
        rows += x.shape[0]
        am_bad += int((am.long() != ref_am).sum())
        d = (mb[nonroot] - ref_mb).abs()
        mb_bad += int((d != 0).sum())
        worst = max(worst, float((d / ref_mb.clamp_min(1e-30)).max()))
        nodes += nonroot.numel()
        if method == "traversal" and it < PATH_SAMPLE_BATCHES:
            ram, rmb = ref_am.cpu().numpy(), np.zeros(x.shape[0], np.float32)
            rmb[nonroot.cpu().numpy()] = ref_mb.cpu().numpy()
            oc_h, ot_h, oh_h = oc.cpu().numpy(), ot.cpu().numpy(), oh.cpu().numpy()
            ip = indptr.cpu().numpy()
            for b, t in enumerate(trees):
                lo, hi = ip[b], ip[b + 1]
                mbb = rmb[lo:hi].copy()
                mbb[0] = 1.0
                s, h, tl, al, _ = acc.traversal_walk(t.parents, t.tokens, t.draft_probs, mbb, ram[lo:hi],
                                                     UniformStream(9, it, b))
                n = int(oc_h[b, 0])
                walks += 1
                path_bad += int((ot_h[b, :n].tolist(), oh_h[b, :n].tolist()) != (list(s), list(h)))
    print(f"\n[torch-parity] {method} T={temperature}: rows {rows}, argmax mismatches {am_bad}; nodes {nodes}, "
          f"Mb mismatches {mb_bad} (rate {mb_bad / max(nodes, 1):.3e}, worst relative {worst:.3e})"
          + (f"; traversal paths {walks}, mismatches {path_bad}" if walks else ""))
    assert am_bad == 0
    assert mb_bad <= nodes // 1000
    assert path_bad <= max(1, walks // 100)
