"""GPU parity: fused acceptance kernel vs the reference's golden outputs and
the oracle.  Accepted tokens, hidden indices and counts must be bit-exact."""
import numpy as np
import pytest
import torch

from oracle import accept as acc
from oracle.philox import UniformStream
from parallel_tree_spec_b200 import kernels as K
from parallel_tree_spec_b200 import workload as wl
from tests.golden_inputs import checked_inputs

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def bf16(bits: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16)


def run_batch(trees, logits_bits, method, eos=None, T=1.0, seed=0, offset=0, max_nodes=None):
    indptr, par, tok, dp = wl.stack_trees(trees)
    x = bf16(np.concatenate(logits_bits, 0)).to(DEV)
    args = (x, torch.from_numpy(indptr).to(DEV), torch.from_numpy(par).to(DEV), torch.from_numpy(tok).to(DEV))
    if method == "exact":
        ot, oh, oc = K.accept_greedy(*args, eos_token_id=eos, max_nodes=max_nodes)
    else:
        ot, oh, oc = K.accept_traversal(*args, torch.from_numpy(dp).to(DEV), eos_token_id=eos, temperature=T,
                                        seed=seed, offset=offset, max_nodes=max_nodes)
    ot, oh, oc = ot.cpu().numpy(), oh.cpu().numpy(), oc.cpu().numpy()
    res = []
    for b in range(len(trees)):
        n = int(oc[b, 0])
        res.append(dict(tokens=ot[b, :n].tolist(), hidden=oh[b, :n].tolist(), total_len=int(oc[b, 1]),
                        accept_len=int(oc[b, 2]), node=int(oc[b, 3])))
    return res


def filler(vocab, rng):
    t = wl.make_tree(rng, 0, 0, vocab)
    return t, wl.make_logits(rng, t, vocab)


def test_golden_acceptance_cases(accept_golden):
    """Every golden case, placed at its Philox request index in a batch padded
    with root-only trees."""
    rng = np.random.default_rng(0)
    for rec in accept_golden:
        c = rec["case"]
        t, x = checked_inputs(rec)
        req = c.get("request", 0) if c["method"] == "traversal" else 0
        trees, logits = [], []
        for _ in range(req):
            ft, fx = filler(c["vocab"], rng)
            trees.append(ft)
            logits.append(fx)
        trees.append(t)
        logits.append(x)
        out = run_batch(trees, logits, c["method"], eos=c.get("eos_value"), T=c.get("temperature", 1.0),
                        seed=c.get("philox_seed", 0), offset=c.get("philox_offset", 0))[req]
        assert out["tokens"] == rec["tokens"], c
        assert out["hidden"] == rec["hidden"], c
        assert (out["total_len"], out["accept_len"]) == (rec["total_len"], rec["accept_len"]), c


@pytest.mark.parametrize("method,T,plant,max_nodes", [("exact", 1.0, 0.7, None), ("exact", 1.0, 0.0, None),
                                                      ("traversal", 1.0, 1.0, None), ("traversal", 0.8, 1.0, None),
                                                      ("traversal", 1.0, 0.0, None), ("exact", 1.0, 0.7, 65),
                                                      ("traversal", 1.0, 1.0, 65), ("traversal", 0.8, 1.0, 65)])
def test_batched_full_vocab_vs_oracle(method, T, plant, max_nodes):
    """Benchmark shape: 16 trees of 65 rows over a 128256 vocabulary; with
    max_nodes = 65 (the tree size, as the benchmark and the drop-in module
    pass it) traversal streams the internal rows in depth-first order and
    walks on CTAs of their own."""
    rng = np.random.default_rng(11 + int(plant * 10) + int(T * 100))
    V = 128256
    trees = [wl.make_tree(rng, 8, 8, V) for _ in range(16)]
    logits = [wl.make_logits(rng, t, V, plant=plant, soft=(method == "traversal")) for t in trees]
    seed, offset = 1234, 77
    out = run_batch(trees, logits, method, T=T, seed=seed, offset=offset, max_nodes=max_nodes)
    accepted = 0
    for b, (t, x) in enumerate(zip(trees, logits)):
        am, p = acc.row_stats(x, T if method == "traversal" else 1.0)
        if method == "exact":
            s, h, tl, al = acc.greedy_walk(t.parents, t.tokens, am)
        else:
            mb = acc.mb_from_probs(t.parents, t.tokens, p)
            s, h, tl, al, _ = acc.traversal_walk(t.parents, t.tokens, t.draft_probs, mb, am,
                                                 UniformStream(seed, offset, b))
        assert out[b]["tokens"] == s and out[b]["hidden"] == h, (b, out[b], s, h)
        assert (out[b]["total_len"], out[b]["accept_len"]) == (tl, al)
        accepted += al
    if plant > 0:
        assert accepted > 0


@pytest.mark.parametrize("shapes,V", [
    ([(8, 8)] * 40, 8192),            # 40 requests: every CTA streams and walks (depth-first order)
    ([(8, 8)] * 70, 4096),            # 4550 rows: internal rows in row order
    ([(1, 64)] * 12, 4096),           # 65-deep chains: keys longer than 64 bits
    ([(16, 8), (1, 64), (4, 3), (0, 0), (8, 8), (2, 30)] * 4, 4096),   # ragged sizes, 129-node trees
])
def test_traversal_stream_orders_vs_oracle(shapes, V):
    """Traversal beyond the benchmark shape, with max_nodes = the largest
    tree: the stream orders and walker placements of the persistent kernel."""
    rng = np.random.default_rng(len(shapes) * 31 + V)
    trees = [wl.make_tree(rng, w, d, V) for w, d in shapes]
    logits = [wl.make_logits(rng, t, V, plant=1.0, soft=True) for t in trees]
    seed, offset = 99, 3
    mn = max(len(t.parents) for t in trees)
    out = run_batch(trees, logits, "traversal", seed=seed, offset=offset, max_nodes=mn)
    for b, (t, x) in enumerate(zip(trees, logits)):
        am, p = acc.row_stats(x, 1.0)
        mb = acc.mb_from_probs(t.parents, t.tokens, p)
        s, h, tl, al, _ = acc.traversal_walk(t.parents, t.tokens, t.draft_probs, mb, am,
                                             UniformStream(seed, offset, b))
        assert out[b]["tokens"] == s and out[b]["hidden"] == h, (b, out[b], s, h)
        assert (out[b]["total_len"], out[b]["accept_len"]) == (tl, al)


def test_near_tie_rows_vs_oracle():
    """Tiny logits: many distinct values round to the same bf16 probability,
    so the argmax must come from the rounded probabilities (the rescan path)."""
    rng = np.random.default_rng(5)
    V = 50000
    trees = [wl.make_tree(rng, 4, 3, V) for _ in range(6)]
    logits = [wl.make_logits(rng, t, V, sigma=0.01) for t in trees]
    out = run_batch(trees, logits, "exact")
    n_tie_rows = 0
    for b, (t, x) in enumerate(zip(trees, logits)):
        am, p = acc.row_stats(x)
        raw = np.argmax(acc.bf16_bits_to_f32(x), axis=-1)
        n_tie_rows += int(np.count_nonzero(raw != am))
        s, h, tl, al = acc.greedy_walk(t.parents, t.tokens, am)
        assert out[b]["tokens"] == s and out[b]["hidden"] == h
    assert n_tie_rows > 0          # the case really exercises rounded-probability ties


def test_unaligned_vocab_and_stride():
    """Odd vocabulary (scalar load path) and a padded row stride."""
    rng = np.random.default_rng(9)
    V = 1001
    trees = [wl.make_tree(rng, 3, 3, V) for _ in range(3)]
    logits = [wl.make_logits(rng, t, V, plant=0.8) for t in trees]
    indptr, par, tok, dp = wl.stack_trees(trees)
    x = np.concatenate(logits, 0)
    padded = np.zeros((x.shape[0], 1040), np.uint16)
    padded[:, :V] = x
    xt = bf16(padded).to(DEV)[:, :V]
    ot, oh, oc = K.accept_greedy(xt, torch.from_numpy(indptr).to(DEV), torch.from_numpy(par).to(DEV),
                                 torch.from_numpy(tok).to(DEV))
    oc = oc.cpu().numpy()
    for b, (t, xb) in enumerate(zip(trees, logits)):
        am, _ = acc.row_stats(xb)
        s, h, tl, al = acc.greedy_walk(t.parents, t.tokens, am)
        n = int(oc[b, 0])
        assert ot[b, :n].cpu().tolist() == s and oh[b, :n].cpu().tolist() == h


def test_repeated_calls_reuse_workspace():
    """Counters in the shared workspace are reset on every call."""
    rng = np.random.default_rng(2)
    V = 4096
    trees = [wl.make_tree(rng, 4, 4, V) for _ in range(4)]
    logits = [wl.make_logits(rng, t, V, plant=0.9) for t in trees]
    a = run_batch(trees, logits, "exact")
    for _ in range(3):
        assert run_batch(trees, logits, "exact") == a


def test_bad_arguments_raise():
    x = torch.zeros(4, 16, dtype=torch.bfloat16, device=DEV)
    ind = torch.tensor([0, 4], dtype=torch.int32, device=DEV)
    par = torch.tensor([-1, 0, 0, 1], dtype=torch.int32, device=DEV)
    tok = torch.tensor([0, 1, 2, 3], dtype=torch.int32, device=DEV)
    with pytest.raises(ValueError):
        K.accept_traversal(x, ind, par, tok, torch.ones(4, device=DEV), temperature=0.0)
    with pytest.raises(ValueError):
        K.accept_greedy(x.cpu(), ind, par, tok)


@pytest.mark.parametrize("method,B,max_nodes", [("traversal", 16, 65), ("traversal", 30, 65), ("exact", 16, 65),
                                                ("traversal", 6, None)])
def test_accept_with_compaction_matches_separate_launch(method, B, max_nodes):
    """Acceptance with compact= (each walk compacts its request's KV in the
    same launch) = acceptance, then pts_kv_compact: the same outputs, pool
    bytes and new lengths, over a 2-layer pool with scattered pages."""
    rng = np.random.default_rng(B * 3 + (max_nodes or 0))
    V = 16384
    trees = [wl.make_tree(rng, 8, 8, V) for _ in range(B)]
    logits = [wl.make_logits(rng, t, V, plant=1.0, soft=(method == "traversal")) for t in trees]
    indptr, par, tok, dp = wl.stack_trees(trees)
    x = bf16(np.concatenate(logits, 0)).to(DEV)
    L, Hkv, D, pl = 2, 2, 64, 16
    prefix = rng.integers(0, 100, size=B)
    kv_len = prefix + np.array([t.size for t in trees])
    npages = (kv_len + pl - 1) // pl
    P = int(npages.sum()) + 5
    perm = rng.permutation(P)[:int(npages.sum())].astype(np.int32)
    pind = torch.from_numpy(np.concatenate([[0], np.cumsum(npages)]).astype(np.int32)).to(DEV)
    pidx = torch.from_numpy(perm).to(DEV)
    offs = torch.from_numpy(prefix.astype(np.int32)).to(DEV)
    pool0 = torch.randint(-2 ** 15, 2 ** 15, (L, P, 2, pl, Hkv, D), dtype=torch.int16,
                          generator=torch.Generator().manual_seed(B)).view(torch.bfloat16).to(DEV)
    args = (x, torch.from_numpy(indptr).to(DEV), torch.from_numpy(par).to(DEV), torch.from_numpy(tok).to(DEV))
    kw = dict(max_nodes=max_nodes)
    if method == "traversal":
        args = args + (torch.from_numpy(dp).to(DEV),)
        kw.update(seed=21, offset=4)
    fn = K.accept_traversal if method == "traversal" else K.accept_greedy
    # separate launches
    pool_a = pool0.clone()
    ot_a, oh_a, oc_a = fn(*args, **kw)
    nl_a = torch.zeros(B, dtype=torch.int32, device=DEV)
    lp_a = torch.zeros(B, dtype=torch.int32, device=DEV)
    K.kv_compact(pool_a, pind, pidx, oh_a, oc_a, offs, nl_a, lp_a)
    # fused
    pool_b = pool0.clone()
    nl_b = torch.zeros(B, dtype=torch.int32, device=DEV)
    lp_b = torch.zeros(B, dtype=torch.int32, device=DEV)
    ca = K.kv_compact_args(pool_b, pind, pidx, offs, nl_b, lp_b)
    ot_b, oh_b, oc_b = fn(*args, **kw, compact=ca)
    torch.cuda.synchronize()
    assert torch.equal(oc_a, oc_b)
    for b in range(B):
        n = int(oc_a[b, 0])
        assert torch.equal(ot_a[b, :n], ot_b[b, :n]) and torch.equal(oh_a[b, :n], oh_b[b, :n])
    assert torch.equal(nl_a, nl_b) and torch.equal(lp_a, lp_b)
    assert torch.equal(pool_a.view(torch.int16), pool_b.view(torch.int16))
    assert int((oc_a[:, 0] > 1).sum()) > 0          # some paths really move rows


@pytest.mark.parametrize("shapes,V,eos_at", [
    ([(8, 8)] * 16, 128256, None),                  # the benchmark shape
    ([(8, 8)] * 16, 16384, 3),                      # EOS on an accepted path
    ([(8, 8)] * 40, 16384, None),                   # 40 requests: fewer CTAs per request
    ([(1, 24)] * 3, 40000, None),                   # chains (24 rows each), three requests
    ([(16, 8), (1, 30), (4, 3), (0, 0), (8, 8), (2, 12)] * 3, 50000, None),   # ragged, root-only trees
    ([(4, 4)] * 200, 8192, None),                   # more requests than SMs
])
def test_greedy_step_reduces_path_rows_on_demand(shapes, V, eos_at):
    """The compacting greedy call reduces only the rows on each accepted path
    (the path chain).  Tokens, hidden indices, counts, new lengths and pool
    bytes must equal the greedy call without compaction (every row streamed)
    followed by pts_kv_compact, and the oracle's greedy walk."""
    rng = np.random.default_rng(len(shapes) * 7 + V)
    trees = [wl.make_tree(rng, w, d, V) for w, d in shapes]
    logits = [wl.make_logits(rng, t, V, plant=0.9) for t in trees]
    B = len(trees)
    indptr, par, tok, dp = wl.stack_trees(trees)
    eos = None
    if eos_at is not None:
        # the token request eos_at's walk accepts first (its root row's argmax, planted on a child):
        # that walk stops on EOS after one node, with no bonus row
        am0, _ = acc.row_stats(logits[eos_at], 1.0)
        eos = int(am0[0])
    x = bf16(np.concatenate(logits, 0)).to(DEV)
    mn = max(t.size for t in trees)
    args = (x, torch.from_numpy(indptr).to(DEV), torch.from_numpy(par).to(DEV), torch.from_numpy(tok).to(DEV))
    L, Hkv, D, pl = 2, 2, 64, 16
    prefix = rng.integers(0, 40, size=B)
    kv_len = prefix + np.array([t.size for t in trees])
    npages = (kv_len + pl - 1) // pl
    P = int(npages.sum()) + 3
    perm = rng.permutation(P)[:int(npages.sum())].astype(np.int32)
    pind = torch.from_numpy(np.concatenate([[0], np.cumsum(npages)]).astype(np.int32)).to(DEV)
    pidx = torch.from_numpy(perm).to(DEV)
    offs = torch.from_numpy(prefix.astype(np.int32)).to(DEV)
    pool0 = torch.randint(-2 ** 15, 2 ** 15, (L, P, 2, pl, Hkv, D), dtype=torch.int16,
                          generator=torch.Generator().manual_seed(B)).view(torch.bfloat16).to(DEV)
    for rep in range(2):                           # twice: the request slots and counters start clean each call
        pool_a, pool_b = pool0.clone(), pool0.clone()
        nl_a, lp_a, nl_b, lp_b = (torch.zeros(B, dtype=torch.int32, device=DEV) for _ in range(4))
        ot_a, oh_a, oc_a = K.accept_greedy(*args, eos_token_id=eos, max_nodes=mn)
        K.kv_compact(pool_a, pind, pidx, oh_a, oc_a, offs, nl_a, lp_a)
        ca = K.kv_compact_args(pool_b, pind, pidx, offs, nl_b, lp_b)
        ot_b, oh_b, oc_b = K.accept_greedy(*args, eos_token_id=eos, max_nodes=mn, compact=ca)
        torch.cuda.synchronize()
        assert torch.equal(oc_a, oc_b)
        for b in range(B):
            n = int(oc_a[b, 0])
            assert torch.equal(ot_a[b, :n], ot_b[b, :n]) and torch.equal(oh_a[b, :n], oh_b[b, :n]), b
        assert torch.equal(nl_a, nl_b) and torch.equal(lp_a, lp_b)
        assert torch.equal(pool_a.view(torch.int16), pool_b.view(torch.int16))
    ot_b, oh_b, oc_b = ot_b.cpu().numpy(), oh_b.cpu().numpy(), oc_b.cpu().numpy()
    for b in (0, B // 2, B - 1):
        t = trees[b]
        am, _ = acc.row_stats(logits[b], 1.0)
        s, h, tl, al = acc.greedy_walk(t.parents, t.tokens, am, eos)
        n = int(oc_b[b, 0])
        assert list(ot_b[b, :n]) == s and list(oh_b[b, :n]) == h and (int(oc_b[b, 1]), int(oc_b[b, 2])) == (tl, al)
    assert int(oc_b[:, 2].sum()) > 0                      # some paths accepted
    if eos_at is not None:
        s, h, tl, al = acc.greedy_walk(trees[eos_at].parents, trees[eos_at].tokens,
                                       acc.row_stats(logits[eos_at], 1.0)[0], eos)
        assert int(oc_b[eos_at, 0]) == len(s) and list(ot_b[eos_at, :len(s)]) == s
        if al == 1:
            assert s[-1] == eos and len(s) == 1           # stopped on EOS: no bonus token
