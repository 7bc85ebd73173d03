"""The reference's 2-layer fp32 configuration through the reference's own call sequence.

Nothing below calls a kernel directly.  A Hugging Face ``LlamaForCausalLM``
(hidden 256, 4 query / 2 KV heads, head_dim 64, SwiGLU 688, vocab 1024,
weights N(0, 0.02) from seed 0) is patched with
``apply_flashinfer_kernel_to_llama`` and then driven as the reference's
experiment drives its target (``experiment.py:265-310,392-403``):

* prefill: ``RequestKvCache.increment`` -> ``getKvCacheBatchPosition(mode="tree")``
  -> ``prepareAttention("prefill")`` -> ``model(..., kvCachePool=,
  batch_position=, mode="prefill", flashinferWrapper=)``;
* the draft tree (binary, 15 nodes) is grown the way the reference's beam
  search and ``add_nodes`` grow it: the first level and the last level by
  appending to ``tree.nodes`` and bumping ``tree.current_size``
  (``beam_search.py:441-447,570-579``), the middle level with ``add_nodes``;
* ``verify_draft_tree`` -> ``target_tree_decode`` -> the patched model
  forward -> ``FiLlamaAttention.forward`` -> ``computeAttention``
  (``verification.py:119-178,531-588``, ``flashinfer/attention.py:56-101``);
* ``RequestKvCache.reorder_cache_with_offset`` with the accepted indices.

The tree logits are checked against a dense fp32 forward of the same weights
(prefix causal, tree rows see the prefix and their ancestors), the
``VerifyResult`` against the oracle's walks on those dense logits, and the
compacted cache against the dense model's K/V of the accepted nodes.
"""
import math

import numpy as np
import pytest
import torch

from oracle import accept as acc
from oracle import attention as att
from oracle.philox import UniformStream
from parallel_tree_spec_b200 import verification as ver
from parallel_tree_spec_b200.flashinfer import (BeFlashinferWrapper, KvCachePool, RequestKvCache,
                                                apply_flashinfer_kernel_to_llama, getKvCacheBatchPosition)
from parallel_tree_spec_b200.tree import Tree, TreeNode
from tests.test_gpu_small_fp32 import _dense

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
P, PAGE, HKV, D, V = 128, 16, 2, 64, 1024


def _patched_model():
    from transformers import LlamaConfig, LlamaForCausalLM
    cfg = LlamaConfig(vocab_size=V, hidden_size=256, intermediate_size=688, num_hidden_layers=2,
                      num_attention_heads=4, num_key_value_heads=HKV, head_dim=D, initializer_range=0.02,
                      max_position_embeddings=512, rms_norm_eps=1e-6, tie_word_embeddings=False)
    torch.manual_seed(0)
    model = LlamaForCausalLM(cfg).to(torch.float32).to(DEV).eval()
    apply_flashinfer_kernel_to_llama(model)
    return model


def _prefill(model, pool, wrapper, prompt):
    """The reference experiment's target prefill (``experiment.py:276-310``)."""
    req = RequestKvCache(kvCachePool=pool, page_len=PAGE, seq_init_len=0)
    req.increment(P)
    bp = getKvCacheBatchPosition(request_kv_caches=[req], mode="tree", device=DEV, treeTokens=P)
    wrapper.prepareAttention("prefill", bp, PAGE, "NONE", pool.cache_data[0].dtype)
    out = model(prompt.unsqueeze(0), position_ids=torch.arange(P, device=DEV).unsqueeze(0), past_key_values=None,
                use_cache=False, kvCachePool=pool, batch_position=bp, mode="prefill", flashinferWrapper=wrapper)
    return req, out.logits[0]


def _grow_tree(tokens, probs):
    """A 15-node binary tree, BFS numbered, built through the producer paths
    the reference uses.  tokens/probs: per node, node 0 = root."""
    tree = Tree(torch.tensor(tokens[0]))
    for i in (1, 2):                                         # beam_search.py:441-447
        new_idx = tree.current_size
        tree.nodes[0].children.append(new_idx)
        tree.nodes.append(TreeNode(parent=0, token_id=int(tokens[i]), cumulative_probability=float(probs[i]),
                                   depth=1))
        tree.current_size += 1
    tree.available_leaves = [1, 2]
    tree.add_nodes(torch.from_numpy(np.asarray(tokens[3:7]))[None, None],            # tree.py:78-121
                   torch.from_numpy(np.asarray(probs[3:7]))[None, None], torch.tensor([[[0, 0, 1, 1]]]))
    for i in range(7, 15):                                   # beam_search.py:570-579
        parent = 3 + (i - 7) // 2
        new_idx = tree.current_size
        tree.nodes[parent].children.append(new_idx)
        tree.nodes.append(TreeNode(parent=parent, token_id=int(tokens[i]), cumulative_probability=float(probs[i]),
                                   depth=tree.nodes[parent].depth + 1))
        tree.current_size += 1
    return tree


PARENTS = np.array([-1, 0, 0, 1, 1, 2, 2, 3, 3, 4, 4, 5, 5, 6, 6])
DEPTHS = np.array([0, 1, 1, 2, 2, 2, 2, 3, 3, 3, 3, 3, 3, 3, 3])


def _planted_tokens(model, prompt):
    """Random tree tokens whose first branch (nodes 0, 1, 3, 7) follows the
    model's own greedy choices, so greedy verification accepts along it."""
    rng = np.random.default_rng(2)
    tokens = rng.integers(0, V, size=15)
    tokens[0] = int(prompt[-1])
    path = [0, 1, 3, 7]
    for k in range(1, len(path)):
        ids = torch.cat([prompt, torch.tensor(tokens[path[:k]], device=DEV)])
        pos = torch.cat([torch.arange(P, device=DEV), P - 1 + torch.arange(k, device=DEV)])
        S = P + k
        mask = torch.ones(S, S, dtype=torch.bool, device=DEV).tril()
        logits, _ = _dense(model, ids, pos, mask)
        tokens[path[k]] = int(logits[-1].argmax())
    probs = rng.dirichlet(np.full(15, 0.5)).astype(np.float32)
    probs[0] = 1.0
    return tokens, probs


def _dense_tree(model, prompt, tokens):
    S = P + 15
    mask = torch.zeros(S, S, dtype=torch.bool, device=DEV)
    mask[:P, :P] = torch.ones(P, P, dtype=torch.bool, device=DEV).tril()
    mask[P:, :P] = True
    mask[P:, P:] = torch.from_numpy(att.ancestor_mask(PARENTS)).to(DEV)
    ids = torch.cat([prompt, torch.tensor(tokens, device=DEV)])
    pos = torch.cat([torch.arange(P, device=DEV), torch.from_numpy(P - 1 + DEPTHS).to(DEV)])
    logits, kv = _dense(model, ids, pos, mask)
    return logits[P:], kv


@pytest.mark.parametrize("method", ["exact", "traversal"])
@torch.no_grad()
def test_config1_verify_draft_tree_through_reference_call_sites(method):
    model = _patched_model()
    g = torch.Generator().manual_seed(1)
    prompt = torch.randint(0, V, (P,), generator=g).to(DEV)
    tokens, probs = _planted_tokens(model, prompt)
    tree = _grow_tree(tokens, probs)
    assert tree.current_size == 15 and [n.parent if n.parent is not None else -1 for n in tree.nodes] == \
        PARENTS.tolist()

    pool = KvCachePool(max_pages=32, num_layers=2, num_heads=HKV, head_dim=D, page_len=PAGE, dtype=torch.float32,
                       device=DEV)
    wrapper = BeFlashinferWrapper(num_attention_heads=4, num_key_value_heads=HKV, hidden_size=256, page_len=PAGE,
                                  device=DEV)
    req, prefill_logits = _prefill(model, pool, wrapper, prompt)

    captured = []
    hook = model.lm_head.register_forward_hook(lambda m, i, o: captured.append(o.detach().clone()))
    seed, offset = 1234, 7
    ver.set_traversal_seed(seed, offset)
    res = ver.verify_draft_tree(target_model=model, flashinfer_wrapper=wrapper, tree=tree, request_kv_cache=req,
                                position_offset=P - 1, device=DEV, eos_token_id=None, verification_method=method,
                                temperature=1.0)
    hook.remove()
    assert isinstance(res, ver.VerifyResult) and res.verify_time > 0.0
    req.reorder_cache_with_offset(res.hidden_indices, offset=P + 1)
    torch.cuda.synchronize()

    # the logits the verification saw equal a dense forward over prefix + tree
    ref_logits, kv = _dense_tree(model, prompt, tokens)
    assert len(captured) == 1
    tree_logits = captured[0][0]
    assert (tree_logits - ref_logits).abs().max().item() < 1e-4
    # prefill through the patched model equals the dense causal forward too
    dense_prefill, _ = _dense(model, prompt, torch.arange(P, device=DEV),
                              torch.ones(P, P, dtype=torch.bool, device=DEV).tril())
    assert (prefill_logits - dense_prefill).abs().max().item() < 1e-4

    # the accepted path equals the oracle's walk over the logits the kernel read
    x = tree_logits.cpu().numpy()
    am, p = acc.row_stats_f32(x)
    if method == "exact":
        rs, rh, rtl, ral = acc.greedy_walk(PARENTS, tokens, am)
        assert ral == 3                                      # the planted branch
    else:
        mb = acc.mb_from_probs(PARENTS, tokens, p)
        rs, rh, rtl, ral, _ = acc.traversal_walk(PARENTS, tokens, probs, mb, am, UniformStream(seed, offset, 0))
    assert res.sampled_tokens.dtype == torch.long and tuple(res.sampled_tokens.shape) == (1, len(rs))
    assert (res.sampled_tokens.reshape(-1).tolist(), res.hidden_indices.tolist(), res.total_len, res.accept_len) \
        == (list(rs), list(rh), rtl, ral)

    # compaction: slot P + i holds the K/V of accepted node hidden[i] in every layer
    hidden = res.hidden_indices.tolist()
    assert req.kv_len == P + len(hidden)
    assert len(req.kv_page_indices) == math.ceil(req.kv_len / PAGE)
    idx = torch.tensor(req.kv_page_indices, device=DEV)
    for li in range(2):
        k_ref, v_ref = kv[li]
        kk = pool.cache_data[li][idx, 0].reshape(-1, HKV, D)
        vv = pool.cache_data[li][idx, 1].reshape(-1, HKV, D)
        assert torch.allclose(kk[:P], k_ref[:P], atol=1e-5) and torch.allclose(vv[:P], v_ref[:P], atol=1e-5)
        for i, node in enumerate(hidden):
            assert torch.allclose(kk[P + i], k_ref[P + node], atol=1e-5)
            assert torch.allclose(vv[P + i], v_ref[P + node], atol=1e-5)
