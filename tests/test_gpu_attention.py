"""GPU parity: tcgen05 tree attention vs an fp32 torch reference and the oracle.

Tolerance (bf16 in/out): max-abs 2e-2 and mean-abs 1e-3 against fp32.
"""
import math

import numpy as np
import pytest
import torch

from oracle import attention as att
from parallel_tree_spec_b200 import kernels as K
from parallel_tree_spec_b200 import workload as wl

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
MAX_ABS, MEAN_ABS = 2e-2, 1e-3


def make_case(seed, trees, prefixes, Hq=32, Hkv=8, D=128, pl=16, extra_pages=7):
    g = torch.Generator(device="cpu").manual_seed(seed)
    kv_lens = [p + t.size for p, t in zip(prefixes, trees)]
    n_pages = [(L + pl - 1) // pl for L in kv_lens]
    P = sum(n_pages) + extra_pages
    perm = torch.randperm(P, generator=g).tolist()
    tables, cur = [], 0
    for n in n_pages:
        tables.append(perm[cur:cur + n])
        cur += n
    layer = (torch.randn(P, 2, pl, Hkv, D, generator=g) / math.sqrt(D)).to(torch.bfloat16)
    T = sum(t.size for t in trees)
    q = torch.randn(T, Hq, D, generator=g).to(torch.bfloat16)
    return dict(trees=trees, prefixes=prefixes, kv_lens=kv_lens, tables=tables, layer=layer, q=q, Hq=Hq, Hkv=Hkv,
                D=D, pl=pl)


def torch_reference(c):
    """Dense fp32 masked attention per request (on the GPU)."""
    q, layer = c["q"].to(DEV).float(), c["layer"].to(DEV).float()
    g = c["Hq"] // c["Hkv"]
    outs, q0 = [], 0
    for t, pre, L, tb in zip(c["trees"], c["prefixes"], c["kv_lens"], c["tables"]):
        n = t.size
        idx = torch.tensor(tb, device=DEV)
        k = layer[idx, 0].reshape(-1, c["Hkv"], c["D"])[:L]
        v = layer[idx, 1].reshape(-1, c["Hkv"], c["D"])[:L]
        k = k.repeat_interleave(g, dim=1)
        v = v.repeat_interleave(g, dim=1)
        mask = torch.from_numpy(att.tree_mask(t.parents, pre)).to(DEV)
        s = torch.einsum("nhd,lhd->hnl", q[q0:q0 + n], k) / math.sqrt(c["D"])
        s = s.masked_fill(~mask[None], float("-inf"))
        outs.append(torch.einsum("hnl,lhd->nhd", torch.softmax(s, -1), v))
        q0 += n
    return torch.cat(outs, 0)


def run_kernel(c):
    trees = c["trees"]
    indptr, par, _, _ = wl.stack_trees(trees)
    qo = torch.from_numpy(indptr).to(DEV)
    words = K.mask_words_for(max(t.size for t in trees))
    bits = K.tree_mask_from_parents(torch.from_numpy(par).to(DEV), qo, words)
    pind = torch.tensor(np.cumsum([0] + [len(t) for t in c["tables"]]), dtype=torch.int32, device=DEV)
    pidx = torch.tensor(sum(c["tables"], []), dtype=torch.int32, device=DEV)
    last = torch.tensor([(L - 1) % c["pl"] + 1 for L in c["kv_lens"]], dtype=torch.int32, device=DEV)
    out = K.tree_attention(c["q"].to(DEV), c["layer"].to(DEV), qo, pind, pidx, last, bits,
                           max(t.size for t in trees), max(c["kv_lens"]))
    torch.cuda.synchronize()
    return out


def check(out, ref):
    d = (out.float() - ref).abs()
    assert torch.isfinite(out.float()).all()
    assert d.max().item() <= MAX_ABS, d.max().item()
    assert d.mean().item() <= MEAN_ABS, d.mean().item()


def test_small_ragged_vs_oracle():
    rng = np.random.default_rng(0)
    trees = [wl.make_tree(rng, 3, 4, 100), wl.make_tree(rng, 8, 8, 100), wl.make_tree(rng, 0, 0, 100)]
    c = make_case(1, trees, [37, 100, 5])
    out = run_kernel(c)
    q = c["q"].float().numpy()
    layer = c["layer"].float().numpy()
    masks = [att.tree_mask(t.parents, p) for t, p in zip(trees, c["prefixes"])]
    indptr = np.cumsum([0] + [t.size for t in trees])
    ref = att.tree_attention(q, layer, c["tables"], c["kv_lens"], indptr, masks, 1 / math.sqrt(128))
    check(out.cpu(), torch.from_numpy(ref).float())


@pytest.mark.parametrize("prefix", [0, 1, 16, 31, 32, 33, 255, 1000])
def test_prefix_lengths(prefix):
    """Partial last pages, odd page counts (zero-filled missing page) and
    blocks that straddle the prefix/tree boundary."""
    rng = np.random.default_rng(prefix)
    trees = [wl.make_tree(rng, 8, 8, 100), wl.make_tree(rng, 4, 3, 100)]
    c = make_case(prefix + 3, trees, [prefix, prefix + 7])
    check(run_kernel(c), torch_reference(c))


def test_large_tree_two_groups():
    """129-node tree: 516 query rows, five 128-row tiles in two CTA groups."""
    rng = np.random.default_rng(7)
    trees = [wl.make_tree(rng, 16, 8, 100), wl.make_tree(rng, 8, 8, 100)]
    c = make_case(5, trees, [300, 64])
    check(run_kernel(c), torch_reference(c))


def test_chain_is_causal_prefill():
    """A chain tree with no prefix is a causal prefill."""
    rng = np.random.default_rng(3)
    trees = [wl.make_tree(rng, 1, 127, 100), wl.make_tree(rng, 1, 40, 100)]
    c = make_case(9, trees, [0, 0])
    check(run_kernel(c), torch_reference(c))


@pytest.mark.parametrize("Hq,Hkv", [(32, 8), (8, 8), (16, 2)])
def test_gqa_groups(Hq, Hkv):
    rng = np.random.default_rng(Hq * 10 + Hkv)
    trees = [wl.make_tree(rng, 8, 8, 100) for _ in range(3)]
    c = make_case(11, trees, [200, 150, 90], Hq=Hq, Hkv=Hkv)
    check(run_kernel(c), torch_reference(c))


def test_benchmark_shape():
    """16 requests, 4096-token prefix, 65-row trees, Hq=32, Hkv=8, D=128."""
    rng = np.random.default_rng(2)
    trees = [wl.make_tree(rng, 8, 8, 100) for _ in range(16)]
    c = make_case(0, trees, [4096] * 16, extra_pages=0)
    check(run_kernel(c), torch_reference(c))


def test_repeat_is_deterministic():
    rng = np.random.default_rng(4)
    trees = [wl.make_tree(rng, 8, 8, 100) for _ in range(4)]
    c = make_case(4, trees, [500] * 4)
    a = run_kernel(c)
    b = run_kernel(c)
    assert torch.equal(a, b)
