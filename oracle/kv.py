"""Paged-KV oracle: batch positions, append, compaction.

Restates (parallel_tree_spec, ``src/parallel_tree_spec/flashinfer``):

* ``batch_positions``    -- ``getKvCacheBatchPosition(mode="tree")``
  (``cache_manager.py:216-280``) with FlashInfer's
  ``get_batch_indices_positions`` rule ``position = seq_len - append_len + i``
  applied per request (the reference builds one append segment, which is the
  same thing for a single request).
* ``append``             -- ``flashinfer.append_paged_kv_cache`` as called at
  ``attention_wrapper.py:201-212`` (NHD layout).
* ``pool_reorder_flat``  -- ``KvCachePool.reorder_cache_with_offset``
  (``cache_manager.py:103-140``): flat physical slot ``offset+idx[i]`` is
  copied to ``offset+i`` in every layer, K and V, all reads before all writes.
* ``request_reorder``    -- ``RequestKvCache.reorder_cache_with_offset``
  (``cache_manager.py:196-213``): offset decremented by one, then the copy
  follows the request's page table (logical slots); identical to the flat
  rule when the request owns physical pages 0..n-1 in order.

* ``rope_bf16``          -- ``apply_rotary_pos_emb`` as the reference's model
  applies it to q and k before the append (``flashinfer/attention.py:83``):
  ``x * cos + rotate_half(x) * sin`` in the activation dtype, each torch
  elementwise op rounding its fp32 result to bf16.

Pools are NumPy arrays ``[L, max_pages, 2, page_len, Hkv, D]`` of any dtype
(bf16 kept as uint16 bits): every operation here is a bit copy.
"""
from __future__ import annotations

import math
from typing import List, Sequence

import numpy as np


def batch_positions(kv_lens: Sequence[int], append_lens: Sequence[int]):
    """Per appended token: (batch index, absolute position)."""
    bi, pos = [], []
    for b, (L, n) in enumerate(zip(kv_lens, append_lens)):
        for i in range(n):
            bi.append(b)
            pos.append(L - n + i)
    return np.asarray(bi, dtype=np.int32), np.asarray(pos, dtype=np.int32)


def slot_of(page_indices: Sequence[int], page_len: int, pos: int):
    return int(page_indices[pos // page_len]), pos % page_len


def append(layer: np.ndarray, k: np.ndarray, v: np.ndarray, page_tables: List[Sequence[int]],
           batch_idx: np.ndarray, positions: np.ndarray) -> None:
    """Write k/v rows ([T, Hkv, D]) into one layer ``[max_pages, 2, page_len, Hkv, D]``."""
    page_len = layer.shape[2]
    for t in range(k.shape[0]):
        pg, sl = slot_of(page_tables[int(batch_idx[t])], page_len, int(positions[t]))
        layer[pg, 0, sl] = k[t]
        layer[pg, 1, sl] = v[t]


def pool_reorder_flat(cache: np.ndarray, beam_idx: Sequence[int], offset: int) -> None:
    """``KvCachePool.reorder_cache_with_offset`` on flat physical slots."""
    L, P, _, pl, H, D = cache.shape
    idx = np.asarray(beam_idx, dtype=np.int64)
    old = idx + offset
    new = np.arange(offset, offset + len(idx), dtype=np.int64)
    for kv in (0, 1):
        flat = cache[:, :, kv].reshape(L, P * pl, H, D)
        gathered = flat[:, old].copy()
        flat[:, new] = gathered
        cache[:, :, kv] = flat.reshape(L, P, pl, H, D)


def request_reorder(cache: np.ndarray, page_indices: List[int], kv_len: int, beam_idx: Sequence[int],
                    offset: int):
    """``RequestKvCache.reorder_cache_with_offset`` following the page table.

    Returns (new_kv_len, new_last_page_len, kept_page_indices, freed_pages).
    """
    pl = cache.shape[3]
    if offset != 0:
        offset -= 1                                               # :200-201
    idx = [int(i) for i in beam_idx]
    src = [slot_of(page_indices, pl, offset + i) for i in idx]
    dst = [slot_of(page_indices, pl, offset + j) for j in range(len(idx))]
    rows = [cache[:, pg, :, sl].copy() for (pg, sl) in src]
    for (pg, sl), r in zip(dst, rows):
        cache[:, pg, :, sl] = r
    new_len = offset + len(idx)                                   # :203
    last = 0 if new_len == 0 else (new_len - 1) % pl + 1          # :204-207
    need = math.ceil(new_len / pl) if new_len > 0 else 0          # :208
    kept = list(page_indices[:need])
    freed = list(page_indices[need:]) if len(page_indices) > need else []
    return new_len, last, kept, freed


def _bf16_to_f32(bits: np.ndarray) -> np.ndarray:
    return (bits.astype(np.uint32) << 16).view(np.float32)


def _f32_to_bf16(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even fp32 -> bf16 bits (finite inputs)."""
    u = x.astype(np.float32).view(np.uint32)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def rope_bf16(x_bits: np.ndarray, cos_bits: np.ndarray, sin_bits: np.ndarray) -> np.ndarray:
    """x [..., T, H, D], cos / sin [T, D], all bf16 bits: x * cos +
    rotate_half(x) * sin with rotate_half(x) = cat(-x[D/2:], x[:D/2]); every
    product and the sum rounded to bf16 (products of two bf16 values and the
    fp32 sum are what torch computes before rounding)."""
    x = _bf16_to_f32(x_bits)
    c = _bf16_to_f32(cos_bits)[:, None, :]
    s = _bf16_to_f32(sin_bits)[:, None, :]
    h = x.shape[-1] // 2
    rot = np.concatenate([-x[..., h:], x[..., :h]], axis=-1)
    p1 = _bf16_to_f32(_f32_to_bf16((x * c).astype(np.float32)))
    p2 = _bf16_to_f32(_f32_to_bf16((rot * s).astype(np.float32)))
    return _f32_to_bf16((p1 + p2).astype(np.float32))
