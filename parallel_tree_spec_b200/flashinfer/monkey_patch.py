"""Patch a Hugging Face Llama model to run its attention over the paged cache
(``flashinfer/monkey_patch.py:95-123``).

``apply_flashinfer_kernel_to_llama(model)`` binds ``FiLlamaAttention.forward``
onto every decoder layer's attention module and the mask-free forwards of
``modeling_llama`` onto the base model and its causal-LM wrapper, so that
``model(input_ids, position_ids=..., kvCachePool=..., batch_position=...,
mode=..., flashinferWrapper=...)`` runs each layer's attention through
``BeFlashinferWrapper.computeAttention``.  ``rms_norm=True`` keeps the model's
own RMSNorm modules: the reference swaps in FlashInfer's fused norm there,
which is outside the verification path and is not replaced by this package.
"""
from __future__ import annotations

from typing import Callable

import torch.nn as nn
from transformers.models.llama.modeling_llama import LlamaAttention

from .attention import FiLlamaAttention
from .modeling_llama import llama_causal_lm_forward, llama_model_forward


def _bind_method_to_module(module: nn.Module, method_name: str, new_method: Callable) -> None:
    """Give one module instance its own bound ``method_name``."""
    module.__dict__[method_name] = new_method.__get__(module, module.__class__)


def _patch_attention_module(module: nn.Module) -> None:
    if isinstance(module, FiLlamaAttention):
        return
    if not isinstance(module, LlamaAttention):
        raise ValueError(f"Unsupported attention module type: {type(module)}")
    _bind_method_to_module(module, "forward", FiLlamaAttention.forward)


def apply_flashinfer_kernel_to_llama(model: nn.Module, attention: bool = True, rms_norm: bool = True) -> None:
    """Patch ``model`` (a loaded ``LlamaForCausalLM`` or ``LlamaModel``) in place."""
    if not attention:
        return
    base = getattr(model, getattr(model, "base_model_prefix", "model"), model)
    _bind_method_to_module(base, "forward", llama_model_forward)
    if base is not model:
        _bind_method_to_module(model, "forward", llama_causal_lm_forward)
    for layer in base.layers:
        _patch_attention_module(layer.self_attn)
