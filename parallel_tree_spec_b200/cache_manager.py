"""Paged KV cache manager, interface of the reference's ``flashinfer/cache_manager.py``.

``KvCachePool`` / ``RequestKvCache`` / ``KvCacheBatchPosition`` /
``getKvCacheBatchPosition`` keep the reference's constructors, attributes and
tensor layout (``cache_data[L, max_pages, 2, page_len, Hkv, D]``, host-side
free-page mask with first-fit allocation, ``cache_manager.py:23-213``).  The
device work goes through libpts_b200:

* ``getKvCacheBatchPosition`` computes append batch indices / positions with
  ``pts_batch_positions``, one append segment per request (the reference
  builds a single segment, ``cache_manager.py:263-271``, which is the same
  thing for one request);
* ``reorder_cache_with_offset`` moves only the accepted rows with
  ``pts_kv_compact`` instead of cloning the whole pool twice
  (``cache_manager.py:130-140``).  The pool-level method addresses flat
  physical slots like the reference; the request-level method follows the
  request's page table, which is identical whenever the request owns
  physical pages 0..n-1 in order (the only case in which the reference's
  flat-slot arithmetic addresses the request's own pages).
"""
from __future__ import annotations

import math
from typing import List

import numpy as np
import torch

from . import kernels as K


class KvCacheBatchPosition:
    """Batch descriptor (``cache_manager.py:23-48``).  Also keeps host copies
    of the per-request lengths so planning needs no device sync."""

    def __init__(self, seq_indptr, kv_page_indptr, kv_page_indices, kv_last_page_len, batch_indices, positions):
        self.seq_indptr = seq_indptr
        self.kv_page_indptr = kv_page_indptr
        self.kv_page_indices = kv_page_indices
        self.kv_last_page_len = kv_last_page_len
        self.batch_indices = batch_indices
        self.positions = positions
        self.host_qo_lens = None
        self.host_kv_lens = None

    def print_info(self):
        for k in ("seq_indptr", "kv_page_indptr", "kv_page_indices", "kv_last_page_len", "batch_indices", "positions"):
            print(f"  {k + ':':<18}{getattr(self, k)}")


class KvCachePool:
    """Device pool of fixed-size pages (``cache_manager.py:51-140``)."""

    def __init__(self, max_pages: int, num_layers: int, num_heads: int, head_dim: int, page_len: int,
                 dtype: torch.dtype, device):
        self.cache_data = torch.zeros(num_layers, max_pages, 2, page_len, num_heads, head_dim, dtype=dtype,
                                      device=device)
        self.num_layers = num_layers
        self.device = device
        self.max_pages = max_pages
        self.page_len = page_len
        self.num_heads = num_heads
        self.head_dims = head_dim
        self.dtype = dtype
        self.free_page_mask = torch.ones(max_pages, dtype=torch.bool, device="cpu")
        self._identity_pages = None

    def reset(self):
        self.cache_data.zero_()
        self.free_page_mask.fill_(True)

    def num_free_pages(self):
        return self.free_page_mask.sum().item()

    def allocate(self, num_pages: int) -> List[int]:
        """First-fit allocation (``cache_manager.py:89-97``)."""
        free = self.free_page_mask.nonzero()
        assert len(free) >= num_pages, f"Out of cache pages: asked {num_pages}, only {len(free)} free"
        got = free[:num_pages]
        self.free_page_mask[got] = False
        return got.squeeze(1).tolist()

    def deallocate(self, kv_page_indices: List[int]):
        self.free_page_mask[kv_page_indices] = True

    def _compact(self, pages: List[int], beam_idx: torch.Tensor, base: int):
        dev = self.cache_data.device
        idx = torch.as_tensor(beam_idx, device=dev).to(torch.int32).reshape(1, -1)
        n = idx.shape[1]
        if n == 0:
            return
        if pages is None:
            if self._identity_pages is None:
                self._identity_pages = torch.arange(self.max_pages, dtype=torch.int32, device=dev)
            pidx = self._identity_pages
        else:
            pidx = torch.as_tensor(pages, dtype=torch.int32, device=dev)
        pind = torch.tensor([0, pidx.numel()], dtype=torch.int32, device=dev)
        counts = torch.tensor([n], dtype=torch.int32, device=dev)
        offs = torch.tensor([base], dtype=torch.int32, device=dev)
        K.kv_compact(self.cache_data, pind, pidx, idx, counts, offs)

    def reorder_cache_with_offset(self, beam_idx: torch.LongTensor, offset: int = 0, num_new_tokens: int = 0):
        """Flat physical slot ``offset + beam_idx[i]`` -> ``offset + i`` in every
        layer, K and V (``cache_manager.py:103-140``)."""
        self._compact(None, beam_idx, offset)


class RequestKvCache:
    """Per-request page list and length (``cache_manager.py:143-213``)."""

    def __init__(self, kvCachePool: KvCachePool, page_len: int, seq_init_len: int):
        self.kvCachePool = kvCachePool
        self.page_len = page_len
        n = math.ceil(seq_init_len / page_len) if seq_init_len > 0 else 0
        self.kv_last_page_len = seq_init_len - (n - 1) * page_len if n > 0 else 0
        self.kv_page_indices = kvCachePool.allocate(n) if n > 0 else []
        self.kv_len = seq_init_len
        self.is_released = False

    def get_seq_length(self):
        return self.kv_len

    def increment(self, num_tokens: int = 1):
        if num_tokens <= 0:
            return
        if len(self.kv_page_indices) == 0:
            self.kv_page_indices.extend(self.kvCachePool.allocate(1))
            self.kv_last_page_len = 0
        self.kv_len += num_tokens
        self.kv_last_page_len += num_tokens
        while self.kv_last_page_len > self.page_len:
            self.kv_last_page_len -= self.page_len
            self.kv_page_indices.extend(self.kvCachePool.allocate(1))

    def decrement(self, num_tokens: int = 1):
        if num_tokens <= 0:
            return
        num_tokens = min(num_tokens, self.kv_len)
        self.kv_len -= num_tokens
        need = math.ceil(self.kv_len / self.page_len) if self.kv_len > 0 else 0
        while len(self.kv_page_indices) > need:
            self.kvCachePool.deallocate([self.kv_page_indices.pop()])
        self.kv_last_page_len = 0 if self.kv_len == 0 else (self.kv_len - 1) % self.page_len + 1

    def release(self):
        if not self.is_released:
            self.kvCachePool.deallocate(self.kv_page_indices)
            self.is_released = True

    def reorder_cache_with_offset(self, beam_idx: torch.LongTensor, offset: int = 0, num_new_tokens: int = 0):
        """Keep the accepted rows: slot ``offset-1 + beam_idx[i]`` ->
        ``offset-1 + i`` through this request's page table, then truncate."""
        if offset != 0:
            offset -= 1
        self.kvCachePool._compact(self.kv_page_indices, beam_idx, offset)
        self.kv_len = offset + int(torch.as_tensor(beam_idx).numel())
        self.kv_last_page_len = 0 if self.kv_len == 0 else (self.kv_len - 1) % self.page_len + 1
        need = math.ceil(self.kv_len / self.page_len) if self.kv_len > 0 else 0
        if len(self.kv_page_indices) > need:
            self.kvCachePool.deallocate(self.kv_page_indices[need:])
            self.kv_page_indices = self.kv_page_indices[:need]


def getKvCacheBatchPosition(request_kv_caches: List[RequestKvCache], mode: str, device,
                            treeTokens: int = 0) -> KvCacheBatchPosition:
    """Batch descriptor for ``mode`` in {"prefill", "decode", "tree"}
    (``cache_manager.py:216-280``)."""
    pages, page_indptr, seq_indptr, last, kv_lens, app = [], [0], [0], [], [], []
    for r in request_kv_caches:
        pages.extend(r.kv_page_indices)
        page_indptr.append(page_indptr[-1] + len(r.kv_page_indices))
        last.append(r.kv_last_page_len)
        kv_lens.append(r.kv_len)
        if mode == "prefill":
            n = r.kv_len
        elif mode == "decode":
            n = 1
        elif mode == "tree":
            n = treeTokens
        else:
            raise ValueError(f"Invalid mode: {mode}")
        app.append(n)
        seq_indptr.append(seq_indptr[-1] + n)
    i32 = lambda x: torch.tensor(x, dtype=torch.int32, device=device)
    seq = i32(seq_indptr)
    bp = KvCacheBatchPosition(seq, i32(page_indptr), i32(pages), i32(last), None, None)
    bp.batch_indices, bp.positions = K.batch_positions(seq, i32(kv_lens), seq_indptr[-1])
    bp.host_qo_lens = app
    bp.host_kv_lens = kv_lens
    return bp
