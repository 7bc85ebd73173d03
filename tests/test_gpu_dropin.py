"""GPU parity through the drop-in modules, called the way the reference's
callers call them: ``verify_tree_exact`` / ``verify_tree_traversal`` on a Tree
and a logits tensor, ``RequestKvCache.reorder_cache_with_offset`` on a pool,
and ``BeFlashinferWrapper.prepareAttention`` / ``computeAttention`` after
``getKvCacheBatchPosition`` (``target_tree_decode``, verification.py:119-178)."""
import hashlib
import math
import os

import numpy as np
import pytest
import torch

from oracle import attention as att
from parallel_tree_spec_b200 import cache_manager as cm
from parallel_tree_spec_b200 import verification as ver
from parallel_tree_spec_b200 import workload as wl
from parallel_tree_spec_b200.attention_wrapper import POS_ENCODING_MODE, BeFlashinferWrapper
from parallel_tree_spec_b200.tree import Tree
from tests.conftest import GOLDEN
from tests.golden_inputs import checked_inputs

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def bf16_dev(bits: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16).to(DEV)


def test_verify_functions_match_reference_golden(accept_golden):
    """Every golden case that sits at request index 0 of its Philox stream,
    through the reference-shaped single-tree functions."""
    seen = 0
    for rec in accept_golden:
        c = rec["case"]
        if c["method"] == "traversal" and c.get("request", 0) != 0:
            continue
        w, x = checked_inputs(rec)
        tree = Tree.from_arrays(w.parents, w.tokens, w.draft_probs)
        logits = bf16_dev(x).unsqueeze(0)                                   # [1, N, V] like the model output
        if c["method"] == "exact":
            s, h, tl, al = ver.verify_tree_exact(tree, logits, eos_token_id=c.get("eos_value"))
        else:
            ver.set_traversal_seed(c.get("philox_seed", 0), c.get("philox_offset", 0))
            s, h, tl, al = ver.verify_tree_traversal(tree, logits, eos_token_id=c.get("eos_value"),
                                                     temperature=c.get("temperature", 1.0))
            assert s.device == logits.device and h.device == logits.device
        assert s.dtype == torch.long and s.shape[0] == 1
        assert s[0].tolist() == rec["tokens"], c
        assert h.tolist() == rec["hidden"], c
        assert (tl, al) == (rec["total_len"], rec["accept_len"]), c
        seen += 1
    assert seen >= 30


def test_verify_trees_batch_matches_single_calls():
    """The batched entry point gives each tree what the single-tree call gives."""
    rng = np.random.default_rng(3)
    V = 4096
    ws = [wl.make_tree(rng, 3, 4, V) for _ in range(5)]
    xs = [wl.make_logits(rng, w, V, plant=0.8) for w in ws]
    trees = [Tree.from_arrays(w.parents, w.tokens, w.draft_probs) for w in ws]
    batch = ver.verify_trees(trees, bf16_dev(np.concatenate(xs, 0)), "exact")
    for t, x, (s, h, tl, al) in zip(trees, xs, batch):
        s1, h1, tl1, al1 = ver.verify_tree_exact(t, bf16_dev(x))
        assert torch.equal(s.cpu(), s1.cpu()) and torch.equal(h.cpu(), h1.cpu()) and (tl, al) == (tl1, al1)
    with pytest.raises(ValueError):
        ver.verify_trees(trees, bf16_dev(np.concatenate(xs, 0)), "sideways")


def _sha1(a: np.ndarray) -> str:
    h = hashlib.sha1()
    h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def test_request_reorder_matches_reference_golden(reorder_golden):
    """RequestKvCache.reorder_cache_with_offset on the reference's own pools
    (cache_manager.py:196-213): bytes, lengths, page list and free mask."""
    for i, rec in enumerate(reorder_golden):
        L, max_pages, _, pl, H, D = rec["shape"]
        dtype = torch.bfloat16 if rec["dtype"] == "bfloat16" else torch.float32
        before = np.load(os.path.join(GOLDEN, f"reorder_{i}_before.npy"))
        pool = cm.KvCachePool(max_pages, L, H, D, pl, dtype, DEV)
        view = torch.int16 if dtype == torch.bfloat16 else torch.int32
        pool.cache_data.view(view).copy_(torch.from_numpy(before.view(np.int16 if dtype == torch.bfloat16 else np.int32)))
        req = cm.RequestKvCache(pool, pl, rec["prompt"])
        req.increment(rec["n_tree"])
        assert req.kv_page_indices == rec["pages_before"], i
        req.reorder_cache_with_offset(torch.tensor(rec["path"], dtype=torch.long), offset=rec["offset"])
        torch.cuda.synchronize()
        after = pool.cache_data.view(view).cpu().numpy().view(before.dtype)
        assert _sha1(after) == rec["sha1_after"], i
        assert (req.kv_len, req.kv_last_page_len, req.kv_page_indices) == (rec["kv_len"], rec["last_page_len"],
                                                                          rec["pages_after"]), i
        assert pool.free_page_mask.tolist() == rec["free_mask"], i


@pytest.mark.parametrize("use_bool_mask", [True, False])
def test_wrapper_tree_attention_vs_fp32(use_bool_mask):
    """KvCachePool + RequestKvCache + getKvCacheBatchPosition("tree") +
    BeFlashinferWrapper, as target_tree_decode drives them, against a dense
    fp32 masked softmax over the same pages."""
    rng = np.random.default_rng(9)
    g = torch.Generator(device="cpu").manual_seed(9)
    Hq, Hkv, D, pl, L = 8, 2, 128, 16, 2
    prefixes = [37, 130, 16]
    n = 15
    pool = cm.KvCachePool(64, L, Hkv, D, pl, torch.bfloat16, DEV)
    pool.cache_data.copy_((torch.randn(pool.cache_data.shape, generator=g) / math.sqrt(D)).to(torch.bfloat16))
    ws = [wl.make_tree(rng, 2, 3, 500, full=True) for _ in prefixes]
    trees = [Tree.from_arrays(w.parents, w.tokens, w.draft_probs) for w in ws]
    reqs = []
    for p in prefixes:
        r = cm.RequestKvCache(pool, pl, p)
        r.increment(n)                                                      # the tree's slots (target_tree_decode)
        reqs.append(r)
    bp = cm.getKvCacheBatchPosition(reqs, "tree", DEV, treeTokens=n)
    wrapper = BeFlashinferWrapper(Hq, Hkv, Hq * D, pl, device=DEV)
    if use_bool_mask:
        mask = torch.cat([t.create_attention_mask(prefix_length=p).reshape(-1) for t, p in zip(trees, prefixes)])
        wrapper.prepareAttention("tree", bp, pl, POS_ENCODING_MODE.NONE, torch.bfloat16, attention_mask=mask)
    else:
        parents = torch.tensor(np.concatenate([w.parents for w in ws]), dtype=torch.int32, device=DEV)
        wrapper.set_tree_masks(parents, bp, n)
    T = n * len(prefixes)
    q = torch.randn(T, Hq * D, generator=g).to(torch.bfloat16).to(DEV)
    k = (torch.randn(T, Hkv * D, generator=g) / math.sqrt(D)).to(torch.bfloat16).to(DEV)
    v = torch.randn(T, Hkv * D, generator=g).to(torch.bfloat16).to(DEV)
    layer = 1
    qh, kh, vh = wrapper.reshape_qkv_for_attention(q, k, v, bp)          # as FiLlamaAttention.forward does
    out = wrapper.computeAttention(qh, kh, vh, pool.cache_data[layer], "tree", bp, None, layer)
    torch.cuda.synchronize()
    assert out.shape == (T, Hq * D)
    # reference: the appended tree K/V must now sit at slots prefix .. prefix+n-1
    cache = pool.cache_data[layer].float()
    qf = q.float().view(T, Hq, D)
    gsz = Hq // Hkv
    refs = []
    for b, (r, p, w) in enumerate(zip(reqs, prefixes, ws)):
        idx = torch.tensor(r.kv_page_indices, device=DEV)
        kk = cache[idx, 0].reshape(-1, Hkv, D)[: p + n]
        vv = cache[idx, 1].reshape(-1, Hkv, D)[: p + n]
        assert torch.equal(kk[p:].to(torch.bfloat16), k[b * n:(b + 1) * n].view(n, Hkv, D))
        kk, vv = kk.repeat_interleave(gsz, 1), vv.repeat_interleave(gsz, 1)
        m = torch.from_numpy(att.tree_mask(w.parents, p)).to(DEV)
        s = torch.einsum("nhd,lhd->hnl", qf[b * n:(b + 1) * n], kk) / math.sqrt(D)
        s = s.masked_fill(~m[None], float("-inf"))
        refs.append(torch.einsum("hnl,lhd->nhd", torch.softmax(s, -1), vv).reshape(n, Hq * D))
    ref = torch.cat(refs)
    d = (out.float() - ref).abs()
    assert d.max().item() <= 2e-2 and d.mean().item() <= 1e-3, (d.max().item(), d.mean().item())


def _rotate_half(x):
    h = x.shape[-1] // 2
    return torch.cat((-x[..., h:], x[..., :h]), dim=-1)


def test_wrapper_applies_rope_in_the_append():
    """computeAttention(..., position_embeddings=(cos, sin)) with q, k before
    the rotary embedding = the reference's order (apply_rotary_pos_emb in the
    model, then computeAttention): the same output and cache bytes."""
    g = torch.Generator(device="cpu").manual_seed(4)
    rng = np.random.default_rng(4)
    Hq, Hkv, D, pl, L = 8, 2, 128, 16, 1
    prefixes, n = [50, 17], 13
    runs = []
    for fused in (False, True):
        pool = cm.KvCachePool(32, L, Hkv, D, pl, torch.bfloat16, DEV)
        pool.cache_data.copy_((torch.randn(pool.cache_data.shape, generator=torch.Generator().manual_seed(1))
                               / math.sqrt(D)).to(torch.bfloat16))
        reqs = []
        for p in prefixes:
            r = cm.RequestKvCache(pool, pl, p)
            r.increment(n)
            reqs.append(r)
        bp = cm.getKvCacheBatchPosition(reqs, "tree", DEV, treeTokens=n)
        wrapper = BeFlashinferWrapper(Hq, Hkv, Hq * D, pl, device=DEV)
        ws = [wl.make_tree(np.random.default_rng(7), 4, 3, 500) for _ in prefixes]
        assert all(w.size == n for w in ws)
        parents = torch.tensor(np.concatenate([w.parents for w in ws]), dtype=torch.int32, device=DEV)
        wrapper.set_tree_masks(parents, bp, n)
        T = n * len(prefixes)
        gg = torch.Generator().manual_seed(11)
        q = torch.randn(T, Hq, D, generator=gg).to(torch.bfloat16).to(DEV)
        k = (torch.randn(T, Hkv, D, generator=gg) / math.sqrt(D)).to(torch.bfloat16).to(DEV)
        v = torch.randn(T, Hkv, D, generator=gg).to(torch.bfloat16).to(DEV)
        pos = torch.cat([torch.arange(p, p + n) for p in prefixes]).float()
        inv = 1.0 / (500000.0 ** (torch.arange(0, D, 2).float() / D))
        emb = torch.cat([pos[:, None] * inv[None]] * 2, dim=-1)
        cos, sin = emb.cos().to(torch.bfloat16).to(DEV), emb.sin().to(torch.bfloat16).to(DEV)
        if fused:
            out = wrapper.computeAttention(q, k, v, pool.cache_data[0], "tree", bp, None, 0,
                                           position_embeddings=(cos, sin))
        else:
            qr = q * cos[:, None] + _rotate_half(q) * sin[:, None]
            kr = k * cos[:, None] + _rotate_half(k) * sin[:, None]
            out = wrapper.computeAttention(qr, kr, v, pool.cache_data[0], "tree", bp, None, 0)
        torch.cuda.synchronize()
        runs.append((out.clone(), pool.cache_data.clone()))
    assert torch.equal(runs[0][0].view(torch.int16), runs[1][0].view(torch.int16))
    assert torch.equal(runs[0][1].view(torch.int16), runs[1][1].view(torch.int16))
