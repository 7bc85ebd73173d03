"""Sparse page-set oracle (test infrastructure): page key sums, per-KV-head
page selection and tree attention over per-head page tables.

Restates the selection the library computes for long-prefix requests: per
(request, KV head) the first ``n_first`` and last ``n_last`` full prefix
pages, the ``n_top`` middle pages of highest score ``qbar . key_sum`` (ties
to the earlier page) and every page from the first one holding a tree token.
It follows the page-importance rule of the reference's sparse attention
(``sparse_attention/pillar.py:149-216``: ``q . k`` aggregated per page, top-k
plus a recent window), which the reference uses for the draft's decode with
one page set for all heads; it has no per-head counterpart there, so this
selection is parity unpinned (restated, not checked against the reference).
The fp32 arithmetic is replayed operation by operation: sequential sums,
then the lane-wise dot products and a butterfly over 32 lanes.
"""
from __future__ import annotations

from typing import List, Sequence

import numpy as np

from .accept import bf16_bits_to_f32
from .attention import ancestor_mask

F32 = np.float32


def page_key_sums(layer_bits: np.ndarray, page_ids: Sequence[int]) -> np.ndarray:
    """Sum of the 16 keys of each page, per KV head: float32 [n, Hkv, D]."""
    k = bf16_bits_to_f32(layer_bits[np.asarray(page_ids, dtype=np.int64), 0])   # [n, pl, Hkv, D]
    acc = np.zeros((k.shape[0],) + k.shape[2:], dtype=F32)
    for t in range(k.shape[1]):
        acc = (acc + k[:, t]).astype(F32)
    return acc


def _score(qbar: np.ndarray, ks: np.ndarray) -> F32:
    lanes = np.zeros(32, dtype=F32)
    for lane in range(32):
        d = 4 * lane
        s = F32(qbar[d] * ks[d])
        for j in range(1, 4):
            s = F32(s + F32(qbar[d + j] * ks[d + j]))
        lanes[lane] = s
    for o in (16, 8, 4, 2, 1):
        lanes = (lanes + lanes[np.arange(32) ^ o]).astype(F32)
    return lanes[0]


def select_pages(key_sums, page_indptr, page_indices, last_page_len, q_bits, qo_indptr, Hq, Hkv,
                 page_len=16, n_first=4, n_top=64, n_last=8):
    """Returns (head_indptr [B*Hkv+1], head_indices, head_last_page_len [B*Hkv])."""
    g = Hq // Hkv
    B = len(page_indptr) - 1
    indptr, out, last = [0], [], []
    for b in range(B):
        p0, p1 = int(page_indptr[b]), int(page_indptr[b + 1])
        n_pages = p1 - p0
        n_nodes = int(qo_indptr[b + 1]) - int(qo_indptr[b])
        kv_len = (n_pages - 1) * page_len + int(last_page_len[b]) if n_pages else 0
        F = min(max(0, kv_len - n_nodes) // page_len, n_pages)
        root = bf16_bits_to_f32(q_bits[int(qo_indptr[b])])          # [Hq, D]
        for h in range(Hkv):
            if F <= n_first + n_top + n_last:
                sel = list(range(n_pages))
            else:
                s = np.zeros(128, dtype=F32)
                for j in range(g):
                    s = (s + root[h * g + j]).astype(F32)
                qbar = (s / F32(g)).astype(F32)
                mid = range(n_first, F - n_last)
                scores = [_score(qbar, key_sums[p0 + i, h]) for i in mid]
                order = sorted(range(len(scores)), key=lambda k: (-float(scores[k]), k))
                top = sorted(order[:n_top])
                sel = list(range(n_first)) + [n_first + k for k in top] + list(range(F - n_last, n_pages))
            out.extend(int(page_indices[p0 + i]) for i in sel)
            indptr.append(len(out))
            last.append(int(last_page_len[b]))
    return np.asarray(indptr, np.int32), np.asarray(out, np.int32), np.asarray(last, np.int32)


def tree_attention_head_pages(q: np.ndarray, layer: np.ndarray, head_indptr, head_indices, head_last,
                              qo_indptr, parents: List[Sequence[int]], sm_scale: float,
                              page_len: int = 16) -> np.ndarray:
    """Masked attention where KV head h of request b reads its own page list;
    the tree occupies the last N slots of every list.  float64 out."""
    Hq, D = q.shape[1], q.shape[2]
    Hkv = layer.shape[3]
    g = Hq // Hkv
    out = np.zeros(q.shape, dtype=np.float64)
    for b in range(len(qo_indptr) - 1):
        lo, hi = int(qo_indptr[b]), int(qo_indptr[b + 1])
        n = hi - lo
        anc = ancestor_mask(parents[b])
        for h in range(Hkv):
            t = b * Hkv + h
            pages = np.asarray(head_indices[head_indptr[t]:head_indptr[t + 1]], dtype=np.int64)
            L = (len(pages) - 1) * page_len + int(head_last[t])
            k = layer[pages, 0, :, h].reshape(-1, D)[:L].astype(np.float64)
            v = layer[pages, 1, :, h].reshape(-1, D)[:L].astype(np.float64)
            mask = np.concatenate([np.ones((n, L - n), dtype=bool), anc], axis=1)
            for j in range(g):
                s = (q[lo:hi, h * g + j].astype(np.float64) @ k.T) * sm_scale
                s = np.where(mask, s, -np.inf)
                e = np.exp(s - s.max(axis=1, keepdims=True))
                out[lo:hi, h * g + j] = (e / e.sum(axis=1, keepdims=True)) @ v
    return out
