"""Model forwards without the dense causal mask (``flashinfer/modeling_llama.py:23-116``).

The tree mask lives in the attention plan (``BeFlashinferWrapper.prepareAttention``),
so the base model skips Hugging Face's ``create_causal_mask`` and passes the
paged-cache keyword arguments (``kvCachePool``, ``batch_position``, ``mode``,
``flashinferWrapper``, ...) through every decoder layer to its attention.
Both functions are bound onto model instances by
``apply_flashinfer_kernel_to_llama``.
"""
from __future__ import annotations

from typing import Optional, Union

import torch
from transformers.cache_utils import DynamicCache
from transformers.modeling_outputs import BaseModelOutputWithPast, CausalLMOutputWithPast


def llama_model_forward(self, input_ids: Optional[torch.LongTensor] = None,
                        attention_mask: Optional[torch.Tensor] = None,
                        position_ids: Optional[torch.LongTensor] = None, past_key_values=None,
                        inputs_embeds: Optional[torch.FloatTensor] = None,
                        cache_position: Optional[torch.LongTensor] = None, use_cache: Optional[bool] = None,
                        **kwargs) -> BaseModelOutputWithPast:
    """``LlamaModel.forward`` with no causal-mask construction
    (``flashinfer/modeling_llama.py:23-76``)."""
    if (input_ids is None) == (inputs_embeds is None):
        raise ValueError("You must specify exactly one of input_ids or inputs_embeds")
    h = self.embed_tokens(input_ids) if inputs_embeds is None else inputs_embeds
    if use_cache and past_key_values is None:
        past_key_values = DynamicCache(config=self.config)
    if cache_position is None:
        seen = past_key_values.get_seq_length() if past_key_values is not None else 0
        cache_position = torch.arange(seen, seen + h.shape[1], device=h.device)
    if position_ids is None:
        position_ids = cache_position.unsqueeze(0)
    rotary = self.rotary_emb(h, position_ids)
    for layer in self.layers[: self.config.num_hidden_layers]:
        h = layer(h, attention_mask=None, position_ids=position_ids, past_key_values=past_key_values,
                  cache_position=cache_position, position_embeddings=rotary, **kwargs)
    return BaseModelOutputWithPast(last_hidden_state=self.norm(h), past_key_values=past_key_values)


def llama_causal_lm_forward(self, input_ids: Optional[torch.LongTensor] = None,
                            attention_mask: Optional[torch.Tensor] = None,
                            position_ids: Optional[torch.LongTensor] = None, past_key_values=None,
                            inputs_embeds: Optional[torch.FloatTensor] = None,
                            labels: Optional[torch.LongTensor] = None, use_cache: Optional[bool] = None,
                            cache_position: Optional[torch.LongTensor] = None,
                            logits_to_keep: Union[int, torch.Tensor] = 0, **kwargs) -> CausalLMOutputWithPast:
    """``LlamaForCausalLM.forward``: base model, then ``lm_head`` over the kept
    positions (``flashinfer/modeling_llama.py:79-116``)."""
    out = self.model(input_ids=input_ids, attention_mask=attention_mask, position_ids=position_ids,
                     past_key_values=past_key_values, inputs_embeds=inputs_embeds, use_cache=use_cache,
                     cache_position=cache_position, **kwargs)
    keep = slice(-logits_to_keep, None) if isinstance(logits_to_keep, int) else logits_to_keep
    logits = self.lm_head(out.last_hidden_state[:, keep, :])
    loss = None
    if labels is not None:
        loss = self.loss_function(logits=logits, labels=labels, vocab_size=self.config.vocab_size, **kwargs)
    return CausalLMOutputWithPast(loss=loss, logits=logits, past_key_values=out.past_key_values,
                                  hidden_states=out.hidden_states, attentions=out.attentions)
