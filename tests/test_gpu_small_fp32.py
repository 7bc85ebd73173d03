"""The reference's small fp32 configuration on the GPU path.

* fp32 acceptance against the reference's own outputs on fp32 logits
  (accept_f32.json), accepted paths bit-exact;
* the SIMT attention kernel (fp32 and bf16 caches, head_dim 64) against the
  float64 oracle;
* one verify step of a 2-layer Llama-architecture fp32 model (hidden 256, 4
  query / 2 KV heads, head_dim 64, SwiGLU 688, vocab 1024, weights N(0, 0.02)
  seed 0; a 128-token prefix in 16-token pages; a 15-node binary tree) driven
  through the drop-in modules the way target_tree_decode drives them
  (verification.py:119-178): prefill and tree attention through
  BeFlashinferWrapper, greedy acceptance through verify_tree_exact, KV
  compaction through RequestKvCache.reorder_cache_with_offset.  It is checked
  against a dense fp32 forward of the same weights over the prefix and the
  tree (tree rows see the prefix and their ancestors).
"""
import json
import math
import os

import numpy as np
import pytest
import torch

from oracle import accept as acc
from oracle import attention as att
from oracle.philox import UniformStream
from parallel_tree_spec_b200 import cache_manager as cm
from parallel_tree_spec_b200 import kernels as K
from parallel_tree_spec_b200 import verification as ver
from parallel_tree_spec_b200 import workload as wl
from parallel_tree_spec_b200.attention_wrapper import POS_ENCODING_MODE, BeFlashinferWrapper
from parallel_tree_spec_b200.tree import Tree
from tests.conftest import GOLDEN
from tests.golden_inputs import checked_inputs

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def test_fp32_acceptance_matches_reference_golden():
    with open(os.path.join(GOLDEN, "accept_f32.json")) as f:
        recs = json.load(f)
    rng = np.random.default_rng(0)
    for rec in recs:
        c = rec["case"]
        t, x = checked_inputs(rec)
        req = c.get("request", 0) if c["method"] == "traversal" else 0
        trees, xs = [], []
        for _ in range(req):                                  # fillers up to the case's Philox request index
            f = wl.make_tree(rng, 0, 0, c["vocab"])
            trees.append(f)
            xs.append(rng.standard_normal((1, c["vocab"])).astype(np.float32))
        trees.append(t)
        xs.append(x)
        indptr, par, tok, dp = wl.stack_trees(trees)
        d = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(DEV)
        xt = d(np.concatenate(xs).astype(np.float32))
        if c["method"] == "exact":
            ot, oh, oc = K.accept_greedy(xt, d(indptr), d(par), d(tok), eos_token_id=c.get("eos_value"))
        else:
            ot, oh, oc = K.accept_traversal(xt, d(indptr), d(par), d(tok), d(dp), eos_token_id=c.get("eos_value"),
                                            temperature=c["temperature"], seed=c["philox_seed"],
                                            offset=c.get("philox_offset", 0))
        n = int(oc[req, 0])
        got = (ot[req, :n].tolist(), oh[req, :n].tolist(), int(oc[req, 1]), int(oc[req, 2]))
        assert got == (rec["tokens"], rec["hidden"], rec["total_len"], rec["accept_len"]), c


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_simt_attention_head_dim_64(dtype):
    rng = np.random.default_rng(4)
    Hq, Hkv, D, pl = 4, 2, 64, 16
    trees = [wl.make_tree(rng, 2, 3, 100, full=True), wl.make_tree(rng, 3, 2, 100)]
    prefixes = [128, 37]
    kv_lens = [p + t.size for p, t in zip(prefixes, trees)]
    npg = [(L + pl - 1) // pl for L in kv_lens]
    perm = rng.permutation(sum(npg) + 3)
    tables = [perm[:npg[0]].tolist(), perm[npg[0]:npg[0] + npg[1]].tolist()]
    layer = (rng.standard_normal((sum(npg) + 3, 2, pl, Hkv, D)) / math.sqrt(D)).astype(np.float32)
    T = sum(t.size for t in trees)
    q = rng.standard_normal((T, Hq, D)).astype(np.float32)
    tl = torch.from_numpy(layer).to(dtype).to(DEV)
    tq = torch.from_numpy(q).to(dtype).to(DEV)
    indptr, par, _, _ = wl.stack_trees(trees)
    qo = torch.from_numpy(indptr).to(DEV)
    bits = K.tree_mask_from_parents(torch.from_numpy(par).to(DEV), qo, 1)
    i32 = lambda v: torch.tensor(v, dtype=torch.int32, device=DEV)
    out = K.tree_attention(tq, tl, qo, i32([0, npg[0], npg[0] + npg[1]]), i32(sum(tables, [])),
                           i32([(L - 1) % pl + 1 for L in kv_lens]), bits, max(t.size for t in trees), max(kv_lens))
    masks = [att.tree_mask(t.parents, p) for t, p in zip(trees, prefixes)]
    ref = att.tree_attention(tq.float().cpu().numpy(), tl.float().cpu().numpy(), tables, kv_lens, indptr, masks,
                             1 / math.sqrt(D))
    err = np.abs(out.float().cpu().numpy() - ref)
    tol = (1e-5, 1e-6) if dtype == torch.float32 else (2e-2, 1e-3)
    assert err.max() <= tol[0] and err.mean() <= tol[1], (err.max(), err.mean())


# ------------------------------------------------------------------ 2-layer model
def _model():
    from transformers import LlamaConfig, LlamaForCausalLM
    cfg = LlamaConfig(vocab_size=1024, hidden_size=256, intermediate_size=688, num_hidden_layers=2,
                      num_attention_heads=4, num_key_value_heads=2, head_dim=64, initializer_range=0.02,
                      max_position_embeddings=512, rms_norm_eps=1e-6, tie_word_embeddings=False)
    torch.manual_seed(0)
    return LlamaForCausalLM(cfg).to(torch.float32).to(DEV).eval()


def _layers(model, ids, pos, attend):
    """The model's own modules with attention supplied by ``attend(layer, q, k,
    v)`` (q [T, Hq, D], k/v [T, Hkv, D] after RoPE) -> logits [T, V]."""
    from transformers.models.llama.modeling_llama import apply_rotary_pos_emb
    m = model.model
    c = model.config
    D = c.head_dim
    h = m.embed_tokens(ids)
    cos, sin = m.rotary_emb(h[None], pos[None])
    T = ids.shape[0]
    for li, layer in enumerate(m.layers):
        a = layer.self_attn
        x = layer.input_layernorm(h)
        q = a.q_proj(x).view(T, -1, D).transpose(0, 1)[None]
        k = a.k_proj(x).view(T, -1, D).transpose(0, 1)[None]
        v = a.v_proj(x).view(T, -1, D)
        q, k = apply_rotary_pos_emb(q, k, cos, sin)
        o = attend(li, q[0].transpose(0, 1).contiguous(), k[0].transpose(0, 1).contiguous(), v.contiguous())
        h = h + a.o_proj(o.reshape(T, -1))
        h = h + layer.mlp(layer.post_attention_layernorm(h))
    return model.lm_head(m.norm(h))


def _dense(model, ids, pos, mask):
    """Dense fp32 attention with a boolean [S, S] mask; also returns K/V."""
    kv = {}

    def attend(li, q, k, v):
        g = q.shape[1] // k.shape[1]
        kv[li] = (k, v)
        s = torch.einsum("thd,shd->hts", q, k.repeat_interleave(g, 1)) / math.sqrt(q.shape[-1])
        s = s.masked_fill(~mask[None], float("-inf"))
        return torch.einsum("hts,shd->thd", torch.softmax(s, -1), v.repeat_interleave(g, 1))

    return _layers(model, ids, pos, attend), kv


@torch.no_grad()
def test_two_layer_fp32_model_verify_step_and_compaction():
    model = _model()
    P, pl, Hkv, D = 128, 16, 2, 64
    g = torch.Generator().manual_seed(1)
    prompt = torch.randint(0, 1024, (P,), generator=g).to(DEV)
    # the tree: a binary depth-3 tree rooted at the last prompt token whose
    # first branch follows the model's own greedy tokens (so greedy verification
    # accepts along it); the other tokens are random
    w = wl.make_tree(np.random.default_rng(2), 2, 3, 1024, full=True, root_token=int(prompt[-1]))
    tokens = w.tokens.copy()
    depth = w.depths()
    path = [0, 1, 3, 7]                                       # first child at every level (BFS numbering)
    causal = torch.ones(P, P, dtype=torch.bool, device=DEV).tril()
    for k in range(1, len(path)):
        ids = torch.cat([prompt, torch.tensor(tokens[path[:k]], device=DEV)])
        pos = torch.cat([torch.arange(P, device=DEV), P - 1 + torch.arange(k, device=DEV)])
        S = P + k
        mask = torch.zeros(S, S, dtype=torch.bool, device=DEV)
        mask[:P, :P] = causal
        mask[P:, :P] = True
        mask[P:, P:] = torch.ones(k, k, dtype=torch.bool, device=DEV).tril()
        logits, _ = _dense(model, ids, pos, mask)
        tokens[path[k]] = int(logits[-1].argmax())
    tree = Tree.from_arrays(w.parents, tokens, w.draft_probs)
    n = tree.current_size

    # ---- the drop-in path: prefill, tree decode, verify, compaction
    pool = cm.KvCachePool(32, 2, Hkv, D, pl, torch.float32, DEV)
    req = cm.RequestKvCache(pool, pl, P)
    wrapper = BeFlashinferWrapper(4, Hkv, 256, pl, device=DEV)
    bp = cm.getKvCacheBatchPosition([req], "prefill", DEV)
    wrapper.prepareAttention("prefill", bp, pl, POS_ENCODING_MODE.NONE, torch.float32)
    attend = lambda li, q, k, v: wrapper.computeAttention(q, k, v, pool.cache_data[li], "prefill", bp, None, li)
    _layers(model, prompt, torch.arange(P, device=DEV), attend)
    req.increment(n)
    bp = cm.getKvCacheBatchPosition([req], "tree", DEV, treeTokens=n)
    wrapper.prepareAttention("tree", bp, pl, POS_ENCODING_MODE.NONE, torch.float32,
                             attention_mask=tree.create_attention_mask(prefix_length=P))
    tids = torch.tensor(tokens, device=DEV)
    tpos = torch.tensor(P - 1 + depth, device=DEV)
    attend = lambda li, q, k, v: wrapper.computeAttention(q, k, v, pool.cache_data[li], "tree", bp, None, li)
    logits = _layers(model, tids, tpos, attend)
    s, h, tl, al = ver.verify_tree_exact(tree, logits)
    req.reorder_cache_with_offset(h, offset=P + 1)
    torch.cuda.synchronize()

    # ---- dense fp32 reference over prefix + tree
    S = P + n
    mask = torch.zeros(S, S, dtype=torch.bool, device=DEV)
    mask[:P, :P] = causal
    mask[P:, :P] = True
    mask[P:, P:] = torch.from_numpy(att.ancestor_mask(w.parents)).to(DEV)
    ref_logits, kv = _dense(model, torch.cat([prompt, tids]), torch.cat([torch.arange(P, device=DEV), tpos]), mask)
    assert (logits - ref_logits[P:]).abs().max().item() < 1e-4
    am, _ = acc.row_stats_f32(ref_logits[P:].cpu().numpy())
    rs, rh, rtl, ral = acc.greedy_walk(w.parents, tokens, am)
    assert (s.reshape(-1).tolist(), h.tolist(), tl, al) == (rs, list(rh), rtl, ral)
    assert al == 3                                            # the planted branch is accepted
    # compacted KV: slot P + i holds tree node h[i]'s K/V in every layer
    for li in range(2):
        k_ref, v_ref = kv[li]
        idx = torch.tensor(req.kv_page_indices, device=DEV)
        kk = pool.cache_data[li][idx, 0].reshape(-1, Hkv, D)
        vv = pool.cache_data[li][idx, 1].reshape(-1, Hkv, D)
        for i, node in enumerate(h.tolist()):
            assert torch.allclose(kk[P + i], k_ref[P + node], atol=1e-5)
            assert torch.allclose(vv[P + i], v_ref[P + node], atol=1e-5)
    assert req.kv_len == P + len(h)
