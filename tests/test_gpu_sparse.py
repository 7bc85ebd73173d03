"""GPU parity of the per-KV-head sparse page sets (long-prefix requests).

Page key sums and the page selection must equal the oracle's exactly (the
same fp32 operations in the same order); tree attention over the per-head
page tables is checked against the float64 oracle and fp32 torch within the
attention tolerance (2e-2 max-abs, 1e-3 mean-abs).
"""
import math

import numpy as np
import pytest
import torch

from oracle import pages as opg
from parallel_tree_spec_b200 import kernels as K
from parallel_tree_spec_b200 import workload as wl

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
MAX_ABS, MEAN_ABS = 2e-2, 1e-3


def _case(seed, prefixes, widths_depths, Hq=32, Hkv=8, D=128, pl=16):
    rng = np.random.default_rng(seed)
    trees = [wl.make_tree(rng, w, d, 1000) for w, d in widths_depths]
    kv_lens = [p + t.size for p, t in zip(prefixes, trees)]
    npg = [(L + pl - 1) // pl for L in kv_lens]
    P = sum(npg) + 5
    perm = rng.permutation(P)
    indptr = np.concatenate([[0], np.cumsum(npg)]).astype(np.int32)
    indices = perm[: indptr[-1]].astype(np.int32)
    layer = wl._bf16_bits((rng.standard_normal((P, 2, pl, Hkv, D)) / math.sqrt(D)).astype(np.float32))
    # make some pages stand out for some heads
    for i in rng.choice(indptr[-1], size=indptr[-1] // 5, replace=False):
        layer[indices[i], 0, :, rng.integers(0, Hkv)] = wl._bf16_bits(
            (rng.standard_normal((pl, D)) * 0.5).astype(np.float32))
    qo = np.concatenate([[0], np.cumsum([t.size for t in trees])]).astype(np.int32)
    q = wl._bf16_bits(rng.standard_normal((int(qo[-1]), Hq, D)).astype(np.float32))
    last = np.asarray([(L - 1) % pl + 1 for L in kv_lens], np.int32)
    return dict(trees=trees, kv_lens=kv_lens, indptr=indptr, indices=indices, layer=layer, qo=qo, q=q, last=last,
                Hq=Hq, Hkv=Hkv, D=D)


def _dbf(a):
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).to(DEV).view(torch.bfloat16)


def _di(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV)


def test_select_pages_matches_oracle_and_attention_over_head_pages():
    c = _case(3, [4100, 1500, 300, 2053], [(8, 8), (4, 6), (3, 3), (16, 4)])
    layer = _dbf(c["layer"])
    ks = K.page_key_sums(layer, _di(c["indices"]))
    ks_ref = opg.page_key_sums(c["layer"], c["indices"])
    assert np.array_equal(ks.cpu().numpy(), ks_ref)
    n_first, n_top, n_last = 4, 24, 8
    hi, hx, hl = K.select_pages(ks, _di(c["indptr"]), _di(c["indices"]), _di(c["last"]), _dbf(c["q"]), _di(c["qo"]),
                                c["Hkv"], n_first=n_first, n_top=n_top, n_last=n_last)
    ri, rx, rl = opg.select_pages(ks_ref, c["indptr"], c["indices"], c["last"], c["q"], c["qo"], c["Hq"], c["Hkv"],
                                  n_first=n_first, n_top=n_top, n_last=n_last)
    hi_np = hi.cpu().numpy()
    assert np.array_equal(hi_np, ri)
    assert np.array_equal(hx.cpu().numpy()[: hi_np[-1]], rx)
    assert np.array_equal(hl.cpu().numpy(), rl)
    # attention over the per-head tables
    parents = [t.parents for t in c["trees"]]
    qo = _di(c["qo"])
    par = _di(np.concatenate(parents).astype(np.int32))
    n_max = max(t.size for t in c["trees"])
    bits = K.tree_mask_from_parents(par, qo, K.mask_words_for(n_max))
    max_kv = int(np.max(np.diff(hi_np))) * 16
    out = K.tree_attention_head_pages(_dbf(c["q"]), layer, qo, hi, hx, hl, bits, n_max, max_kv)
    ref = opg.tree_attention_head_pages(wl._bf16_f32(c["q"]), wl._bf16_f32(c["layer"]), ri, rx, rl, c["qo"],
                                        parents, 1 / math.sqrt(c["D"]))
    err = np.abs(out.float().cpu().numpy() - ref)
    assert err.max() <= MAX_ABS and err.mean() <= MEAN_ABS, (err.max(), err.mean())


def test_head_pages_equal_shared_tables_when_nothing_is_dropped():
    """With every page selected, per-head tables reproduce pts_tree_attn_run."""
    c = _case(11, [700, 1234], [(8, 8), (4, 4)])
    layer = _dbf(c["layer"])
    ks = K.page_key_sums(layer, _di(c["indices"]))
    hi, hx, hl = K.select_pages(ks, _di(c["indptr"]), _di(c["indices"]), _di(c["last"]), _dbf(c["q"]), _di(c["qo"]),
                                c["Hkv"], n_first=4, n_top=1000, n_last=8)
    qo = _di(c["qo"])
    par = _di(np.concatenate([t.parents for t in c["trees"]]).astype(np.int32))
    n_max = max(t.size for t in c["trees"])
    bits = K.tree_mask_from_parents(par, qo, K.mask_words_for(n_max))
    a = K.tree_attention_head_pages(_dbf(c["q"]), layer, qo, hi, hx, hl, bits, n_max, max(c["kv_lens"]))
    b = K.tree_attention(_dbf(c["q"]), layer, qo, _di(c["indptr"]), _di(c["indices"]), _di(c["last"]), bits, n_max,
                         max(c["kv_lens"]))
    assert torch.equal(a, b)
