"""Draft beam search on the GPU.

* ``pts_beam_select`` against the oracle's restatement of the reference's
  scoring and top-K (``oracle/beam.py``): scores, flat indices and step
  probabilities bit for bit, first step (no cumulative scores) and decode
  steps, T = 1 and 0.8, rows with planted ties (the smaller flat index wins);
* ``pts_kv_copy_pages`` against torch's indexed copy;
* ``parallel_tree_spec_b200.beam_search.beam_search`` with the deterministic
  stand-in model against the reference's own run of the same search
  (``tests/golden/beam.json``): every decode step's page table, the tree, the
  free pages and the pool's bytes.
"""
import hashlib
import json
import os

import numpy as np
import pytest
import torch

from oracle import beam as ob
from oracle.accept import f32_to_bf16_bits
from parallel_tree_spec_b200 import beam_search as pbs
from parallel_tree_spec_b200 import kernels as K
from parallel_tree_spec_b200.cache_manager import KvCachePool, RequestKvCache
from tests import beam_fixture as bf

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "beam.json")
LAYERS, HEADS, DIM = 2, 2, 8


def _rows(seed, rows, vocab, sigma=3.0, ties=False):
    rng = np.random.default_rng(seed)
    bits = f32_to_bf16_bits((rng.standard_normal((rows, vocab)) * sigma).astype(np.float32))
    if ties:                                       # equal maxima inside a row and across rows
        for r in range(rows):
            cols = rng.choice(vocab, 3, replace=False)
            bits[r, cols] = f32_to_bf16_bits(np.float32(12.0))
        bits[:, :4] = f32_to_bf16_bits(np.float32(12.0))
    return bits


@pytest.mark.parametrize("rows,vocab,T,with_cum,ties", [
    (1, 1000, 1.0, False, False), (1, 128256, 0.8, False, False), (4, 32000, 1.0, True, False),
    (8, 128256, 1.0, True, False), (16, 4096, 0.8, True, False), (6, 700, 1.0, True, True),
    (3, 2048, 1.0, False, True),
])
def test_beam_select_matches_oracle(rows, vocab, T, with_cum, ties):
    k = min(rows, 16) if with_cum else min(8, vocab)
    bits = _rows(rows * 1000 + vocab, rows, vocab, ties=ties)
    x = bf.bits_to_bf16(bits).to(DEV)
    if with_cum:
        rng = np.random.default_rng(7)
        cum = (-rng.random(rows) * 5).astype(np.float32)
        if ties:
            cum[:] = np.float32(-1.5)
        s, idx, p = K.beam_select(x, k, T, torch.from_numpy(cum).to(DEV))
        rs, rpar, rtok, rp = ob.step_select(bits, [float(v) for v in cum], T, k)
        ridx = rpar * vocab + rtok
    else:
        s, idx, p = K.beam_select(x, k, T)
        p_all = ob.row_probs(bits, T).reshape(-1)
        ridx = ob._order(p_all)[:k]
        rs, rp = p_all[ridx], p_all[ridx]
    assert idx.cpu().numpy().tolist() == [int(v) for v in ridx]
    assert np.array_equal(s.cpu().numpy().view(np.uint32), np.float32(rs).view(np.uint32))
    assert np.array_equal(p.cpu().numpy().view(np.uint32), np.float32(rp).view(np.uint32))


def test_kv_copy_pages_matches_indexed_copy():
    g = torch.Generator(device=DEV).manual_seed(3)
    pool = torch.randn(3, 20, 2, 16, 4, 32, generator=g, device=DEV).to(torch.bfloat16)
    ref = pool.clone()
    src, dst = [1, 7, 4], [9, 2, 15]
    for a, b in zip(src, dst):
        ref[:, b, :, :11] = ref[:, a, :, :11]
    K.kv_copy_pages(pool, torch.tensor(src, device=DEV), torch.tensor(dst, device=DEV), 11)
    assert torch.equal(pool, ref)


def _golden():
    with open(GOLDEN) as f:
        return json.load(f)


@pytest.mark.parametrize("idx", range(6))
def test_beam_search_matches_reference_run(idx):
    rec = _golden()[idx]
    c = rec["case"]
    pool = KvCachePool(c["max_pages"], LAYERS, HEADS, DIM, c["page_len"], torch.bfloat16, torch.device(DEV))
    pool.cache_data.copy_(bf.bits_to_bf16(bf.initial_pool_bits(rec["seed"], tuple(pool.cache_data.shape))).to(DEV))
    req = RequestKvCache(pool, c["page_len"], c["prompt"])
    pre = bf.bits_to_bf16(bf.step_logits_bits([rec["prompt_token"]], [c["prompt"] - 1], c["vocab"],
                                              c["sigma"])).unsqueeze(0).to(DEV)
    model = bf.FakeModel(c["vocab"], c["sigma"], c["page_len"]).to(DEV)
    cfg = pbs.BeamSearchConfig(topk_len=c["K"], max_depth=c["depth"], temperature=c["temperature"])
    ids = torch.tensor([[rec["prompt_token"]]], dtype=torch.long, device=DEV)
    tree, times, runner = pbs.beam_search(model, req, ids, cfg, bf.FakeWrapper(), prefilled_logits=pre)
    torch.cuda.synchronize()
    assert list(req.kv_page_indices) == rec["prompt_pages"]
    assert model.records == rec["steps"]
    assert [(-1 if n.parent is None else n.parent) for n in tree.nodes] == rec["parents"]
    assert [n.token_id for n in tree.nodes] == rec["tokens"]
    assert [n.depth for n in tree.nodes] == rec["depths"]
    assert np.array_equal(np.float32([n.cumulative_probability for n in tree.nodes]), np.float32(rec["probs"]))
    assert pool.free_page_mask.nonzero().squeeze(1).tolist() == rec["free_pages"]
    digest = hashlib.sha1(pool.cache_data.contiguous().view(torch.int16).cpu().numpy().tobytes()).hexdigest()
    assert digest == rec["pool_sha1"]
    assert len(times) == c["depth"] and runner is None
