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
