"""Llama attention through ``BeFlashinferWrapper`` (``flashinfer/attention.py:31-101``).

``FiLlamaAttention.forward`` is bound onto the attention modules of a Hugging
Face Llama model by ``apply_flashinfer_kernel_to_llama``.  Per layer it
projects q/k/v, applies the model's rotary embedding, hands token-major
``[tokens, heads, head_dim]`` rows to ``computeAttention`` (which appends
this layer's k/v to the paged cache and runs the tree-masked attention on the
device) and projects the output.  The paged-cache arguments arrive as the
keyword arguments the patched model forward passes down
(``flashinferWrapper``, ``kvCachePool``, ``mode``, ``batch_position`` and
optionally ``append_batch_position``).
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch
from torch import nn
from transformers.models.llama.modeling_llama import apply_rotary_pos_emb

from ..attention_wrapper import POS_ENCODING_MODE, AttentionRotaryParams


class FiLlamaAttention(nn.Module):
    """Llama attention layer over the paged KV cache (``flashinfer/attention.py:31-53``)."""

    def __init__(self, config, layer_idx: int):
        super().__init__()
        self.config = config
        self.layer_idx = layer_idx
        self.head_dim = getattr(config, "head_dim", None) or config.hidden_size // config.num_attention_heads
        self.num_key_value_groups = config.num_attention_heads // config.num_key_value_heads
        self.scaling = self.head_dim ** -0.5
        self.attention_dropout = config.attention_dropout
        self.is_causal = True
        bias = config.attention_bias
        hq, hkv = config.num_attention_heads * self.head_dim, config.num_key_value_heads * self.head_dim
        self.q_proj = nn.Linear(config.hidden_size, hq, bias=bias)
        self.k_proj = nn.Linear(config.hidden_size, hkv, bias=bias)
        self.v_proj = nn.Linear(config.hidden_size, hkv, bias=bias)
        self.o_proj = nn.Linear(hq, config.hidden_size, bias=bias)

    def forward(self, hidden_states: torch.Tensor, position_embeddings: Tuple[torch.Tensor, torch.Tensor],
                attention_mask: Optional[torch.Tensor] = None, past_key_value=None,
                cache_position: Optional[torch.LongTensor] = None, **kwargs) -> Tuple[torch.Tensor, None]:
        """``hidden_states`` [batch, tokens, hidden] -> ([batch, tokens, hidden], None)
        (``flashinfer/attention.py:56-101``).  ``attention_mask`` is ignored:
        the mask was planned by ``prepareAttention``."""
        wrapper = kwargs["flashinferWrapper"]
        pool = kwargs.get("kvCachePool")
        mode = kwargs.get("mode", "prefill")
        batch_position = kwargs.get("batch_position")
        append_position = kwargs.get("append_batch_position")
        lead = hidden_states.shape[:-1]
        D = self.head_dim

        def by_head(proj):                                   # [batch, heads, tokens, D], as the rotary helper takes it
            return proj(hidden_states).view(*lead, -1, D).transpose(1, 2)

        cos, sin = position_embeddings
        q, k = apply_rotary_pos_emb(by_head(self.q_proj), by_head(self.k_proj), cos, sin)
        v = self.v_proj(hidden_states).view(*lead, -1, D)
        # token-major rows [batch, tokens, heads, D]: one row per token, the cache's order
        q, k, v = wrapper.reshape_qkv_for_attention(q.transpose(1, 2).contiguous(), k.transpose(1, 2).contiguous(),
                                                    v.contiguous(), batch_position)
        out = wrapper.computeAttention(q, k, v, pool.cache_data[self.layer_idx], mode, batch_position,
                                       AttentionRotaryParams(pos_encoding_mode=POS_ENCODING_MODE.NONE),
                                       self.layer_idx, appendBatchPosition=append_position)
        return self.o_proj(out.reshape(*lead, -1)), None
