"""The lm_head GEMM with the acceptance statistics in its epilogue.

* pts_lmhead_logits (tcgen05 GEMM) against an fp32 matmul of the same bf16
  operands, ragged row and vocabulary tiles;
* pts_lmhead_accept (no logits in memory) against the unfused path, the same
  GEMM writing bf16 logits followed by the acceptance kernels: accepted tokens,
  hidden indices and counts equal, greedy and traversal at T = 1 and 0.8, on
  config-2-shaped hidden states (16 trees of 65 rows, hidden 4096, vocabulary
  128256) whose draft tokens are taken from the top of their parents' rows so
  that paths are long;
* rows whose argmax is a rounding tie: all-zero hidden rows (every logit 0,
  settled from the per-tile candidate lists), and near-constant rows with more
  tied values in a tile than the lists keep (reported as -4, redone from
  materialised logits by the Python wrapper).
"""
import numpy as np
import pytest
import torch

from parallel_tree_spec_b200 import kernels as K
from parallel_tree_spec_b200 import workload as wl

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _gen(R, V, H, seed, hidden_scale=1.0):
    g = torch.Generator(device=DEV)
    g.manual_seed(seed)
    hidden = (torch.randn(R, H, generator=g, device=DEV) * hidden_scale).to(torch.bfloat16)
    weight = (torch.randn(V, H, generator=g, device=DEV) * (3.0 / H ** 0.5)).to(torch.bfloat16)
    return hidden, weight


def test_logits_against_fp32_matmul_ragged_tiles():
    R, V, H = 300, 4224, 512
    hidden, weight = _gen(R, V, H, 1)
    got = K.lmhead_logits(hidden, weight).float()
    ref = hidden.float() @ weight.float().t()
    err = (got - ref).abs()
    # bf16 output: half an ulp of the value plus fp32 summation-order noise
    tol = ref.abs() * 2.0 ** -8 + 1e-3
    assert bool((err <= tol).all()), float((err - tol).max())
    assert got.shape == (R, V)


def _trees_from_logits(x, B, width, depth, seed):
    """Beam-shaped trees whose child tokens are the top-ranked tokens of their
    parent row (the first child the row's argmax), so greedy and traversal
    accept along them."""
    rng = np.random.default_rng(seed)
    V = x.shape[1]
    n = 1 + width * depth
    order = torch.argsort(x.float(), dim=1, descending=True)[:, :16].cpu().numpy()
    trees = []
    for b in range(B):
        t = wl.make_tree(rng, width, depth, V)
        tok = t.tokens.copy()
        used = {}
        for i in range(1, n):
            pr = b * n + int(t.parents[i])
            k = used.get(pr, 0)
            tok[i] = int(order[pr, k])
            used[pr] = k + 1
        trees.append(wl.DraftTree(t.parents, tok, t.draft_probs, t.levels))
    return trees


def _unfused(hidden, weight, ind, par, tok, dp, method, temperature, n):
    x = K.lmhead_logits(hidden, weight)
    if method == "exact":
        return K.accept_greedy(x, ind, par, tok, max_nodes=n)
    return K.accept_traversal(x, ind, par, tok, dp, temperature=temperature, seed=3, offset=1, max_nodes=n)


def _same(a, b):
    (t1, h1, c1), (t2, h2, c2) = a, b
    assert torch.equal(c1, c2)
    for r in range(c1.shape[0]):
        n = int(c1[r, 0])
        assert torch.equal(t1[r, :n], t2[r, :n]) and torch.equal(h1[r, :n], h2[r, :n]), r


@pytest.mark.parametrize("method,temperature", [("exact", 1.0), ("traversal", 1.0), ("traversal", 0.8)])
def test_fused_matches_unfused_config2_shape(method, temperature):
    B, width, depth, V, H = 16, 8, 8, 128256, 4096
    n = 1 + width * depth
    hidden, weight = _gen(B * n, V, H, 7)
    trees = _trees_from_logits(K.lmhead_logits(hidden, weight), B, width, depth, 11)
    indptr, par, tok, dp = wl.stack_trees(trees)
    d = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(DEV)
    ind, par, tok, dp = d(indptr), d(par), d(tok), d(dp)
    ref = _unfused(hidden, weight, ind, par, tok, dp, method, temperature, n)
    got = K.lmhead_accept(hidden, weight, ind, par, tok, dp, method=method, temperature=temperature, seed=3,
                          offset=1, max_nodes=n, fallback=False)
    torch.cuda.synchronize()
    assert int((got[2][:, 0] < 0).sum()) == 0
    _same(got, ref)
    if method == "exact":
        assert float(ref[2][:, 2].float().mean()) >= 1.0      # paths longer than the root's child


def test_rounding_ties_from_candidate_lists_and_fallback():
    B, width, depth, V, H = 4, 3, 3, 8192, 512
    n = 1 + width * depth
    hidden, weight = _gen(B * n, V, H, 21)
    hidden[3] = 0                                             # every logit 0: the first index wins the tie
    hidden[n + 2] = 0
    rows_flat = [2 * n, 2 * n + 1, 3 * n + 4]                 # near-constant rows: many tied values per tile
    for r in rows_flat:
        hidden[r] = (hidden[r].float() * 1e-4).to(torch.bfloat16)
    x = K.lmhead_logits(hidden, weight)
    trees = _trees_from_logits(x, B, width, depth, 5)
    indptr, par, tok, dp = wl.stack_trees(trees)
    d = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(DEV)
    ind, par, tok, dp = d(indptr), d(par), d(tok), d(dp)
    for method in ("exact", "traversal"):
        ref = _unfused(hidden, weight, ind, par, tok, dp, method, 1.0, n)
        raw = K.lmhead_accept(hidden, weight, ind, par, tok, dp, method=method, seed=3, offset=1, max_nodes=n,
                              fallback=False)
        c = raw[2][:, 0].cpu()
        assert int(c[0]) >= 0 and int(c[1]) >= 0               # zero rows: settled on the device
        assert int(c[2]) == -4 and int(c[3]) == -4             # near-constant rows: reported
        got = K.lmhead_accept(hidden, weight, ind, par, tok, dp, method=method, seed=3, offset=1, max_nodes=n)
        _same(got, ref)
    # the zero rows' argmax is column 0 in the row statistics as well
    am, _ = K.accept_row_stats(x, ind, par, tok)
    assert int(am[3]) == 0 and int(am[n + 2]) == 0
