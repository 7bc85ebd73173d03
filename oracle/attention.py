"""Tree-masked paged attention oracle (float64).

Restates what the reference asks FlashInfer for on the tree path
(``flashinfer/attention_wrapper.py:131-144,250-252``): a batch prefill over a
paged NHD cache with ``custom_mask``, ``causal=False``, no positional encoding
(RoPE is applied before the append, ``flashinfer/attention.py:74,83-84``) and
``sm_scale = 1/sqrt(head_dim)``.  The mask is the one ``Tree.create_attention_mask``
builds (``tree.py:167-194``): every query row sees the whole prefix and the
tree rows that are its ancestors or itself.  GQA maps query head ``h`` to
KV head ``h // (Hq // Hkv)``.

The arithmetic is FlashInfer's (third party), so this restatement is pinned
only through the mask builder: attention parity is "unpinned" beyond the
2e-2 max-abs / 1e-3 mean-abs tolerance.
"""
from __future__ import annotations

from typing import List, Sequence

import numpy as np


def ancestor_mask(parents: Sequence[int]) -> np.ndarray:
    """[N, N] bool, row i True at i and its ancestors (``tree.py:180-187``)."""
    n = len(parents)
    m = np.zeros((n, n), dtype=bool)
    for i in range(n):
        m[i, i] = True
        p = int(parents[i])
        while p >= 0:
            m[i, p] = True
            p = int(parents[p])
    return m


def tree_mask(parents: Sequence[int], prefix: int) -> np.ndarray:
    """[N, prefix + N] bool, prefix columns all True (``tree.py:188-194``)."""
    a = ancestor_mask(parents)
    return np.concatenate([np.ones((len(parents), prefix), dtype=bool), a], axis=1)


def gather_kv(layer: np.ndarray, page_indices: Sequence[int], kv_len: int):
    """Logical KV rows of one request: ([kv_len, Hkv, D], [kv_len, Hkv, D])."""
    pl = layer.shape[2]
    pages = np.asarray(page_indices, dtype=np.int64)
    k = layer[pages, 0].reshape(-1, *layer.shape[3:])[:kv_len]
    v = layer[pages, 1].reshape(-1, *layer.shape[3:])[:kv_len]
    return k, v


def tree_attention(q: np.ndarray, layer: np.ndarray, page_tables: List[Sequence[int]],
                   kv_lens: Sequence[int], qo_indptr: Sequence[int], masks: List[np.ndarray],
                   sm_scale: float) -> np.ndarray:
    """q: [sum N, Hq, D] float; layer: [max_pages, 2, page_len, Hkv, D] float;
    masks[b]: [N_b, kv_len_b] bool.  Returns float64 [sum N, Hq, D]."""
    Hq, D = q.shape[1], q.shape[2]
    Hkv = layer.shape[3]
    g = Hq // Hkv
    out = np.zeros(q.shape, dtype=np.float64)
    for b in range(len(kv_lens)):
        lo, hi = int(qo_indptr[b]), int(qo_indptr[b + 1])
        k, v = gather_kv(layer, page_tables[b], int(kv_lens[b]))
        k = k.astype(np.float64)
        v = v.astype(np.float64)
        mk = masks[b]
        for h in range(Hq):
            kh = k[:, h // g]
            vh = v[:, h // g]
            s = (q[lo:hi, h].astype(np.float64) @ kh.T) * sm_scale
            s = np.where(mk, s, -np.inf)
            s = s - s.max(axis=1, keepdims=True)
            e = np.exp(s)
            p = e / e.sum(axis=1, keepdims=True)
            out[lo:hi, h] = p @ vh
    return out
