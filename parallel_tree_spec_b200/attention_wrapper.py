"""Paged attention wrapper, interface of the reference's ``flashinfer/attention_wrapper.py``.

``BeFlashinferWrapper`` keeps the reference's constructor and methods
(``attention_wrapper.py:53-262``): ``prepareAttention`` once per step (shared
by every layer), then per layer ``computeAttention`` = append the new K/V to
the paged cache + attention over it.  Behind it:

* mode "tree" with a custom mask: the boolean mask ``[1, 1, N, prefix + N]``
  (``tree.py:167-194``) is packed on the device into per-row ancestor
  bitmasks (``pts_tree_mask_from_bool``); a mask whose prefix columns are not
  all true is rejected with ``ValueError``;
* mode "tree"/"prefill" without a mask and mode "decode": causal rows;
* append: ``pts_kv_append``; attention: ``pts_tree_attn_run_any``.

No FlashInfer, no CPU path.  bf16 caches with head_dim 128, 16-token pages
and GQA groups up to 16 run on the tcgen05 kernel; fp32 caches and other
head dims (multiples of 32 up to 256) on the SIMT kernel.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from enum import Enum
from typing import Optional, Tuple

import torch

from . import kernels as K
from .cache_manager import KvCacheBatchPosition

FLASH_INFER_SUPPORTED_DIMS = [64, 128, 256]


class POS_ENCODING_MODE(Enum):
    ROPE_LLAMA = "ROPE_LLAMA"
    ALIBI = "ALIBI"
    NONE = "NONE"


@dataclass(frozen=True)
class AttentionRotaryParams:
    causal: bool = True
    pos_encoding_mode: POS_ENCODING_MODE = POS_ENCODING_MODE.ROPE_LLAMA
    rope_scale: float = 1.0
    rope_theta: float = 1.0e4


def find_padded_head_dim(head_dim: int) -> int:
    for dim in FLASH_INFER_SUPPORTED_DIMS:
        if head_dim <= dim:
            return dim
    raise ValueError(f"Head dimension {head_dim} too large (max {FLASH_INFER_SUPPORTED_DIMS[-1]})")


class BeFlashinferWrapper:
    """Paged attention for prefill, decode and tree (custom mask) modes."""

    def __init__(self, num_attention_heads: int, num_key_value_heads: int, hidden_size: int, page_len: int,
                 device: Optional[torch.device] = None):
        self.hidden_size = hidden_size
        self.num_attention_heads = num_attention_heads
        self.num_key_value_heads = num_key_value_heads
        self.head_dim = hidden_size // num_attention_heads
        self._head_padded_dim = find_padded_head_dim(self.head_dim)
        self.page_len = page_len
        self.group_size = num_attention_heads // num_key_value_heads
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self._plan = None

    def init_cuda_graph_decode(self, K: int, max_num_pages: int, device: torch.device):
        """``attention_wrapper.py:95-107`` rebuilds FlashInfer's decode wrapper
        over fixed index buffers before graph capture.  The kernels here read
        the page tables on the device and keep no host plan state a graph
        would freeze, so there is nothing to rebuild."""
        return None

    # ------------------------------------------------------------------ plan
    def prepareAttention(self, mode: str, batch_position: KvCacheBatchPosition, page_len: int, pos_encoding_mode,
                         dtype: torch.dtype, attention_mask: Optional[torch.Tensor] = None):
        """Plan the next forward pass (``attention_wrapper.py:113-170``)."""
        if mode not in ("tree", "prefill", "decode"):
            raise ValueError(f"Invalid attention mode: {mode}")
        if page_len != self.page_len:
            raise ValueError(f"page_len {page_len} differs from the wrapper's {self.page_len}")
        bp = batch_position
        if bp.host_qo_lens is not None:
            qo_lens, kv_lens = list(bp.host_qo_lens), list(bp.host_kv_lens)
        else:
            qo = bp.seq_indptr.cpu().tolist()
            pind = bp.kv_page_indptr.cpu().tolist()
            last = bp.kv_last_page_len.cpu().tolist()
            qo_lens = [qo[i + 1] - qo[i] for i in range(len(qo) - 1)]
            kv_lens = [(pind[i + 1] - pind[i] - 1) * page_len + last[i] for i in range(len(last))]
        bits, words = None, 1
        if mode == "tree" and attention_mask is not None:
            words = K.mask_words_for(max(qo_lens))
            m = attention_mask.to(self.device, non_blocking=True).reshape(-1)
            mind = [0]
            for n, L in zip(qo_lens, kv_lens):
                mind.append(mind[-1] + n * L)
            if m.numel() != mind[-1]:
                raise ValueError(f"attention_mask has {m.numel()} entries, expected {mind[-1]} "
                                 "(sum over requests of rows x kv_len)")
            dev_i32 = lambda x: torch.tensor(x, dtype=torch.int32, device=self.device)
            bits = K.tree_mask_from_bool(m, bp.seq_indptr, dev_i32(mind), dev_i32(kv_lens), words)
        self._plan = dict(mode=mode, bp=bp, bits=bits, words=words, max_qo=max(qo_lens), max_kv=max(kv_lens),
                          dtype=dtype)

    def set_tree_masks(self, parents: torch.Tensor, batch_position: KvCacheBatchPosition, max_nodes: int):
        """Plan tree mode straight from the parent arrays (no boolean mask,
        no host sync): ``parents`` int32 [sum N], local indices per request."""
        words = K.mask_words_for(max_nodes)
        bits = K.tree_mask_from_parents(parents, batch_position.seq_indptr, words)
        bp = batch_position
        self._plan = dict(mode="tree", bp=bp, bits=bits, words=words, max_qo=max(bp.host_qo_lens),
                          max_kv=max(bp.host_kv_lens), dtype=torch.bfloat16)

    # --------------------------------------------------------------- helpers
    def reshape_qkv_for_attention(self, q, k, v, batchPosition: KvCacheBatchPosition):
        return (q.view(-1, self.num_attention_heads, self.head_dim),
                k.view(-1, self.num_key_value_heads, self.head_dim),
                v.view(-1, self.num_key_value_heads, self.head_dim))

    def append_kv_cache(self, q, k, v, batch_position: KvCacheBatchPosition, paged_kv_cache: torch.Tensor,
                        page_len: int):
        """Write k/v at the batch positions (``attention_wrapper.py:201-212``)."""
        K.kv_append(k, v, paged_kv_cache, batch_position.batch_indices, batch_position.positions,
                    batch_position.kv_page_indptr, batch_position.kv_page_indices)

    # --------------------------------------------------------------- compute
    def computeAttention(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, cacheData: torch.Tensor, mode: str,
                         batchPosition: KvCacheBatchPosition, rotaryParams: AttentionRotaryParams, layer_idx: int,
                         appendBatchPosition: Optional[KvCacheBatchPosition] = None,
                         position_embeddings: Optional[Tuple[torch.Tensor, torch.Tensor]] = None):
        """Append K/V, then attention with the planned mask; returns
        [tokens, hidden] (``attention_wrapper.py:218-252``).  With
        ``position_embeddings`` = (cos, sin) [tokens, D] (the model's, for
        these tokens), q and k are taken before the rotary embedding and the
        append applies it (to k on its way into the cache, to q for the
        attention), replacing the model's ``apply_rotary_pos_emb`` call."""
        if mode not in ("prefill", "tree", "decode"):
            raise ValueError(f"Invalid attention mode: {mode}")
        plan = self._plan
        if plan is None:
            raise RuntimeError("prepareAttention must be called before computeAttention")
        append_pos = appendBatchPosition if appendBatchPosition is not None else batchPosition
        if position_embeddings is not None:
            cos, sin = position_embeddings
            D = cacheData.shape[-1]
            q = K.kv_append_rope(q.reshape(q.shape[0], -1, D), k.reshape(k.shape[0], -1, D),
                                 v.reshape(v.shape[0], -1, D), cos.reshape(-1, D), sin.reshape(-1, D), cacheData,
                                 append_pos.batch_indices, append_pos.positions, append_pos.kv_page_indptr,
                                 append_pos.kv_page_indices)
        else:
            self.append_kv_cache(q, k, v, append_pos, cacheData, self.page_len)
        bp = plan["bp"]
        out = K.tree_attention(q.contiguous(), cacheData, bp.seq_indptr, bp.kv_page_indptr, bp.kv_page_indices,
                               bp.kv_last_page_len, plan["bits"], plan["max_qo"], plan["max_kv"],
                               sm_scale=1.0 / math.sqrt(self._head_padded_dim))
        return out.view(-1, self.hidden_size)
