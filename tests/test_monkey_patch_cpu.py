"""The model-side drop-in on CPU: ``apply_flashinfer_kernel_to_llama`` and the
patched forwards (``flashinfer/monkey_patch.py:95-123``,
``flashinfer/modeling_llama.py:23-116``, ``flashinfer/attention.py:56-101``).

A stand-in wrapper records what ``FiLlamaAttention.forward`` hands to
``computeAttention`` and answers with dense causal attention, so the patched
model must reproduce the unpatched Hugging Face forward.  No kernel runs."""
import math

import pytest
import torch

from parallel_tree_spec_b200.flashinfer import apply_flashinfer_kernel_to_llama
from parallel_tree_spec_b200.flashinfer.attention_wrapper import POS_ENCODING_MODE


class _RecordingWrapper:
    def __init__(self, hq, hkv, d):
        self.hq, self.hkv, self.d = hq, hkv, d
        self.calls = []

    def reshape_qkv_for_attention(self, q, k, v, batch_position):
        return q.view(-1, self.hq, self.d), k.view(-1, self.hkv, self.d), v.view(-1, self.hkv, self.d)

    def computeAttention(self, q, k, v, cacheData, mode, batchPosition, rotaryParams, layer_idx,
                         appendBatchPosition=None):
        self.calls.append(dict(layer=layer_idx, mode=mode, bp=batchPosition, cache=cacheData,
                               pos_mode=rotaryParams.pos_encoding_mode, shapes=(q.shape, k.shape, v.shape)))
        T, g = q.shape[0], self.hq // self.hkv
        kk, vv = k.repeat_interleave(g, 1), v.repeat_interleave(g, 1)
        s = torch.einsum("thd,shd->hts", q, kk) / math.sqrt(self.d)
        s = s.masked_fill(~torch.ones(T, T, dtype=torch.bool).tril()[None], float("-inf"))
        return torch.einsum("hts,shd->thd", torch.softmax(s, -1), vv).reshape(T, -1)


class _Pool:
    def __init__(self, layers):
        self.cache_data = [torch.zeros(1) + i for i in range(layers)]


@torch.no_grad()
def test_patched_llama_forward_routes_attention_through_the_wrapper():
    from transformers import LlamaConfig, LlamaForCausalLM
    cfg = LlamaConfig(vocab_size=128, hidden_size=64, intermediate_size=96, num_hidden_layers=2,
                      num_attention_heads=4, num_key_value_heads=2, head_dim=16, max_position_embeddings=64,
                      tie_word_embeddings=False, attn_implementation="eager")
    torch.manual_seed(0)
    model = LlamaForCausalLM(cfg).eval()
    ids = torch.randint(0, 128, (1, 9))
    pos = torch.arange(9).unsqueeze(0)
    ref = model(ids, position_ids=pos).logits

    apply_flashinfer_kernel_to_llama(model)
    wrapper, pool, bp = _RecordingWrapper(4, 2, 16), _Pool(2), object()
    out = model(ids, position_ids=pos, past_key_values=None, use_cache=False, kvCachePool=pool, batch_position=bp,
                mode="tree", flashinferWrapper=wrapper)
    assert torch.allclose(out.logits, ref, atol=1e-5)
    assert [c["layer"] for c in wrapper.calls] == [0, 1]
    for li, c in enumerate(wrapper.calls):
        assert c["mode"] == "tree" and c["bp"] is bp and c["cache"] is pool.cache_data[li]
        assert c["pos_mode"] == POS_ENCODING_MODE.NONE
        assert [tuple(s) for s in c["shapes"]] == [(9, 4, 16), (9, 2, 16), (9, 2, 16)]


def test_patch_rejects_other_attention_modules():
    from parallel_tree_spec_b200.flashinfer.monkey_patch import _patch_attention_module
    with pytest.raises(ValueError):
        _patch_attention_module(torch.nn.Linear(2, 2))
