"""Device operations: torch tensors in, C-ABI calls out.

Every function here validates shapes and dtypes, takes raw device pointers
from CUDA tensors and launches on the current torch stream.  Nothing falls
back to another implementation: a missing library or a non-CUDA tensor
raises.
"""
from __future__ import annotations

import ctypes as C
import math
import os
from typing import Dict, Optional, Tuple

import torch

from . import _lib

_WS: Dict[Tuple[int, int, str], torch.Tensor] = {}


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _need_cuda(*ts: torch.Tensor) -> torch.device:
    dev = ts[0].device
    for t in ts:
        if t.device.type != "cuda":
            raise ValueError("tensors must be on a CUDA device (this path has no CPU implementation)")
        if t.device != dev:
            raise ValueError("all tensors must be on the same device")
    return dev


def _i32(t: torch.Tensor, name: str) -> torch.Tensor:
    if t.dtype != torch.int32:
        t = t.to(torch.int32)
    if not t.is_contiguous():
        t = t.contiguous()
    return t


def workspace(device: torch.device, kind: str, nbytes: int) -> torch.Tensor:
    """A scratch buffer per device, current stream and kind (256-byte aligned),
    grown on demand.  Calls on one stream run in order and share it; calls on
    different streams get different buffers, so they may overlap."""
    index = device.index if device.index is not None else torch.cuda.current_device()
    key = (index, _stream(torch.device("cuda", index)), kind)
    buf = _WS.get(key)
    if buf is None or buf.numel() < nbytes:
        buf = torch.zeros(max(nbytes, 256), dtype=torch.uint8, device=device)
        _WS[key] = buf
    return buf


# ------------------------------------------------------------------ acceptance
def _accept_common(logits, row_indptr, parents, tokens):
    if logits.dtype not in (torch.bfloat16, torch.float32) or logits.dim() != 2:
        raise ValueError("logits must be a 2-D bf16 or fp32 tensor [rows, vocab]")
    if logits.stride(1) != 1:
        raise ValueError("logits rows must be contiguous")
    dev = _need_cuda(logits, row_indptr, parents, tokens)
    return dev, _i32(row_indptr, "row_indptr"), _i32(parents, "parents"), _i32(tokens, "tokens")


def kv_compact_args(pool: torch.Tensor, page_indptr: torch.Tensor, page_indices: torch.Tensor,
                    offsets: torch.Tensor, new_kv_len: Optional[torch.Tensor] = None,
                    new_last_page_len: Optional[torch.Tensor] = None):
    """The ``compact=`` argument of the acceptance functions: compact the
    accepted paths of ``pool`` [L, max_pages, 2, page_len, Hkv, D] in the same
    launch (``kv_compact`` with the acceptance's hidden indices and counts).
    The index tensors must stay alive until the launch has run."""
    _need_cuda(pool, page_indptr, page_indices, offsets)
    if pool.dim() != 6 or pool.shape[2] != 2 or not pool.is_contiguous():
        raise ValueError("pool must be a contiguous [L, max_pages, 2, page_len, Hkv, D] tensor")
    L, P, _, pl, H, D = pool.shape
    keep = [_i32(page_indptr, "indptr"), _i32(page_indices, "indices"), _i32(offsets, "offsets")]
    for t in (new_kv_len, new_last_page_len):
        if t is not None and (t.dtype != torch.int32 or not t.is_contiguous()):
            raise ValueError("new_kv_len / new_last_page_len must be contiguous int32")
    args = _lib.KvCompactArgs(pool.data_ptr(), L, P, pl, H, D, pool.element_size(), keep[0].data_ptr(),
                              keep[1].data_ptr(), keep[2].data_ptr(),
                              new_kv_len.data_ptr() if new_kv_len is not None else None,
                              new_last_page_len.data_ptr() if new_last_page_len is not None else None)
    args._keep = keep
    return args


def accept_greedy(logits: torch.Tensor, row_indptr: torch.Tensor, parents: torch.Tensor, tokens: torch.Tensor,
                  eos_token_id: Optional[int] = None, max_nodes: Optional[int] = None,
                  out: Optional[Tuple[torch.Tensor, torch.Tensor, torch.Tensor]] = None, compact=None):
    """Greedy acceptance (``verify_tree_exact``) for a batch of trees.

    Returns (tokens [B, S] int32, hidden [B, S] int32, counts [B, 4] int32)
    with counts = (n_out, total_len, accept_len, accepted_node).  With
    ``compact`` (from ``kv_compact_args``, bf16 logits) the same launch also
    compacts the accepted paths' KV.
    """
    dev, row_indptr, parents, tokens = _accept_common(logits, row_indptr, parents, tokens)
    B = row_indptr.numel() - 1
    R, V = logits.shape
    mn = int(max_nodes) if max_nodes is not None else R
    mn = min(mn, _lib.PTS_MAX_TREE_NODES)
    if out is None:
        ot = torch.empty(B, mn, dtype=torch.int32, device=dev)
        oh = torch.empty(B, mn, dtype=torch.int32, device=dev)
        oc = torch.empty(B, 4, dtype=torch.int32, device=dev)
    else:
        ot, oh, oc = out
    wsz = _lib.lib().pts_accept_workspace_size(R, V)
    ws = workspace(dev, "accept", wsz)
    eos = -1 if eos_token_id is None else int(eos_token_id)
    if compact is not None:
        if logits.dtype != torch.bfloat16:
            raise ValueError("compact takes bf16 logits in this build")
        _lib.call("pts_accept_greedy_compact", logits.data_ptr(), logits.stride(0), row_indptr.data_ptr(),
                  parents.data_ptr(), tokens.data_ptr(), B, R, V, mn, eos, ot.data_ptr(), oh.data_ptr(),
                  oc.data_ptr(), ot.shape[1], ws.data_ptr(), ws.numel(), C.byref(compact), _stream(dev))
        return ot, oh, oc
    fn = "pts_accept_greedy_f32" if logits.dtype == torch.float32 else "pts_accept_greedy"
    _lib.call(fn, logits.data_ptr(), logits.stride(0), row_indptr.data_ptr(), parents.data_ptr(),
              tokens.data_ptr(), B, R, V, mn, eos, ot.data_ptr(), oh.data_ptr(), oc.data_ptr(), ot.shape[1],
              ws.data_ptr(), ws.numel(), _stream(dev))
    return ot, oh, oc


def accept_traversal(logits: torch.Tensor, row_indptr: torch.Tensor, parents: torch.Tensor, tokens: torch.Tensor,
                     draft_probs: torch.Tensor, eos_token_id: Optional[int] = None, temperature: float = 1.0,
                     top_p: float = 1.0, do_sample: bool = False, seed: int = 0, offset: int = 0,
                     max_nodes: Optional[int] = None,
                     out: Optional[Tuple[torch.Tensor, torch.Tensor, torch.Tensor]] = None, compact=None):
    """Traversal verification (``verify_tree_traversal``) for a batch of trees;
    the per-iteration uniform of request b is Philox stream (seed, offset, b).
    With ``compact`` (from ``kv_compact_args``, bf16 logits) the same launch
    also compacts the accepted paths' KV."""
    dev, row_indptr, parents, tokens = _accept_common(logits, row_indptr, parents, tokens)
    if draft_probs.dtype != torch.float32:
        draft_probs = draft_probs.to(torch.float32)
    draft_probs = draft_probs.contiguous()
    _need_cuda(logits, draft_probs)
    B = row_indptr.numel() - 1
    R, V = logits.shape
    mn = int(max_nodes) if max_nodes is not None else R
    mn = min(mn, _lib.PTS_MAX_TREE_NODES)
    if out is None:
        ot = torch.empty(B, mn, dtype=torch.int32, device=dev)
        oh = torch.empty(B, mn, dtype=torch.int32, device=dev)
        oc = torch.empty(B, 4, dtype=torch.int32, device=dev)
    else:
        ot, oh, oc = out
    wsz = _lib.lib().pts_accept_workspace_size(R, V)
    ws = workspace(dev, "accept", wsz)
    if logits.dtype == torch.float32:
        if top_p < 1.0 or do_sample or compact is not None:
            raise ValueError("top_p < 1, do_sample and compact take bf16 logits in this build")
        _lib.call("pts_accept_traversal_f32", logits.data_ptr(), logits.stride(0), row_indptr.data_ptr(),
                  parents.data_ptr(), tokens.data_ptr(), draft_probs.data_ptr(), B, R, V, mn,
                  -1 if eos_token_id is None else int(eos_token_id), float(temperature), int(seed) & (2 ** 64 - 1),
                  int(offset) & (2 ** 64 - 1), ot.data_ptr(), oh.data_ptr(), oc.data_ptr(), ot.shape[1],
                  ws.data_ptr(), ws.numel(), _stream(dev))
        return ot, oh, oc
    args = (logits.data_ptr(), logits.stride(0), row_indptr.data_ptr(), parents.data_ptr(), tokens.data_ptr(),
            draft_probs.data_ptr(), B, R, V, mn, -1 if eos_token_id is None else int(eos_token_id),
            float(temperature), float(top_p), 1 if do_sample else 0, int(seed) & (2 ** 64 - 1),
            int(offset) & (2 ** 64 - 1), ot.data_ptr(), oh.data_ptr(), oc.data_ptr(), ot.shape[1], ws.data_ptr(),
            ws.numel())
    if compact is not None:
        _lib.call("pts_accept_traversal_compact", *args, C.byref(compact), _stream(dev))
    else:
        _lib.call("pts_accept_traversal", *args, _stream(dev))
    return ot, oh, oc


# ------------------------------------------------- vocabulary-sharded acceptance
def accept_row_stats(logits: torch.Tensor, row_indptr: torch.Tensor, parents: torch.Tensor, tokens: torch.Tensor,
                     temperature: float = 1.0) -> Tuple[torch.Tensor, torch.Tensor]:
    """(argmax [rows] int32, Mb [rows] float32) that the most recent bf16
    acceptance call on the current stream computed for these inputs (same
    logits, trees and temperature, no top-p): each row's argmax of its rounded
    softmax and each node's probability under its parent's row."""
    dev, row_indptr, parents, tokens = _accept_common(logits, row_indptr, parents, tokens)
    if logits.dtype != torch.bfloat16:
        raise ValueError("accept_row_stats takes bf16 logits")
    R, V = logits.shape
    B = row_indptr.numel() - 1
    ws = workspace(dev, "accept", _lib.lib().pts_accept_workspace_size(R, V))
    am = torch.empty(R, dtype=torch.int32, device=dev)
    mb = torch.empty(R, dtype=torch.float32, device=dev)
    _lib.call("pts_accept_export_row_stats", ws.data_ptr(), ws.numel(), logits.data_ptr(), logits.stride(0),
              row_indptr.data_ptr(), parents.data_ptr(), tokens.data_ptr(), B, R, V, float(temperature),
              am.data_ptr(), mb.data_ptr(), _stream(dev))
    return am, mb


# ------------------------------------------------------------------ lm_head
def _lmhead_args(hidden: torch.Tensor, weight: torch.Tensor):
    dev = _need_cuda(hidden, weight)
    if hidden.dtype != torch.bfloat16 or weight.dtype != torch.bfloat16:
        raise ValueError("hidden and weight must be bf16")
    if hidden.dim() != 2 or weight.dim() != 2 or hidden.shape[1] != weight.shape[1]:
        raise ValueError("hidden [rows, H] and weight [vocab, H] with the same H")
    return dev, hidden.contiguous(), weight.contiguous()


def lmhead_logits(hidden: torch.Tensor, weight: torch.Tensor) -> torch.Tensor:
    """bf16 logits [rows, vocab] = hidden x weight^T on the tensor cores."""
    dev, hidden, weight = _lmhead_args(hidden, weight)
    R, H = hidden.shape
    V = weight.shape[0]
    out = torch.empty(R, V, dtype=torch.bfloat16, device=dev)
    _lib.call("pts_lmhead_logits", hidden.data_ptr(), weight.data_ptr(), R, V, H, out.data_ptr(), out.stride(0),
              _stream(dev))
    return out


def lmhead_accept(hidden: torch.Tensor, weight: torch.Tensor, row_indptr: torch.Tensor, parents: torch.Tensor,
                  tokens: torch.Tensor, draft_probs: Optional[torch.Tensor] = None, method: str = "exact",
                  eos_token_id: Optional[int] = None, temperature: float = 1.0, seed: int = 0, offset: int = 0,
                  max_nodes: Optional[int] = None, fallback: bool = True):
    """Acceptance straight from the hidden states: the lm_head GEMM with the
    acceptance statistics in its epilogue (no logits in memory), then the
    walks.  Returns (tokens, hidden, counts) like accept_greedy /
    accept_traversal.  With ``fallback`` a request whose rounding tie could
    not be settled from the statistics (counts = -4) is redone from
    materialised logits."""
    dev, hidden, weight = _lmhead_args(hidden, weight)
    row_indptr, parents, tokens = _i32(row_indptr, "indptr"), _i32(parents, "parents"), _i32(tokens, "tokens")
    _need_cuda(hidden, row_indptr, parents, tokens)
    if method not in ("exact", "traversal"):
        raise ValueError(f"Unknown verification method: {method!r} (expected 'traversal' or 'exact')")
    trav = method == "traversal"
    if trav:
        if draft_probs is None:
            raise ValueError("traversal needs draft_probs")
        draft_probs = draft_probs.to(torch.float32).contiguous()
    R, H = hidden.shape
    V = weight.shape[0]
    B = row_indptr.numel() - 1
    mn = min(int(max_nodes) if max_nodes is not None else R, _lib.PTS_MAX_TREE_NODES)
    ot = torch.empty(B, mn, dtype=torch.int32, device=dev)
    oh = torch.empty(B, mn, dtype=torch.int32, device=dev)
    oc = torch.empty(B, 4, dtype=torch.int32, device=dev)
    ws = workspace(dev, "lmhead", _lib.lib().pts_lmhead_workspace_size(R, V))
    _lib.call("pts_lmhead_accept", hidden.data_ptr(), weight.data_ptr(), R, V, H, row_indptr.data_ptr(),
              parents.data_ptr(), tokens.data_ptr(), draft_probs.data_ptr() if trav else None, B, mn,
              -1 if eos_token_id is None else int(eos_token_id), 1 if trav else 0, float(temperature),
              int(seed) & (2 ** 64 - 1), int(offset) & (2 ** 64 - 1), ot.data_ptr(), oh.data_ptr(), oc.data_ptr(),
              ot.shape[1], ws.data_ptr(), ws.numel(), _stream(dev))
    if fallback and bool((oc[:, 0] == -4).any()):
        x = lmhead_logits(hidden, weight)
        if trav:
            rt, rh, rc = accept_traversal(x, row_indptr, parents, tokens, draft_probs, eos_token_id=eos_token_id,
                                          temperature=temperature, seed=seed, offset=offset, max_nodes=mn)
        else:
            rt, rh, rc = accept_greedy(x, row_indptr, parents, tokens, eos_token_id=eos_token_id, max_nodes=mn)
        redo = oc[:, 0] == -4
        ot[redo], oh[redo], oc[redo] = rt[redo], rh[redo], rc[redo]
    return ot, oh, oc


def accept_shard_partials(logits_shard: torch.Tensor, vocab_offset: int, row_indptr: torch.Tensor,
                          parents: torch.Tensor, tokens: torch.Tensor, temperature: float = 1.0):
    """Step 1 of the sharded acceptance: ``logits_shard`` [rows, Vs] bf16 is
    this rank's vocabulary columns (any row stride).  Returns (partials
    [rows, 2] int64 holding 16-byte records, token logits [rows] f32)."""
    if logits_shard.dtype != torch.bfloat16 or logits_shard.dim() != 2 or logits_shard.stride(1) != 1:
        raise ValueError("logits_shard must be a 2-D bf16 tensor with contiguous rows")
    dev, row_indptr, parents, tokens = _accept_common(logits_shard, row_indptr, parents, tokens)
    R, Vs = logits_shard.shape
    parts = torch.empty(R, 2, dtype=torch.int64, device=dev)
    tok = torch.empty(R, dtype=torch.float32, device=dev)
    ws = workspace(dev, "accept_shard", _lib.lib().pts_accept_workspace_size(R, Vs))
    _lib.call("pts_accept_shard_partials", logits_shard.data_ptr(), logits_shard.stride(0), row_indptr.data_ptr(),
              parents.data_ptr(), tokens.data_ptr(), row_indptr.numel() - 1, R, Vs, int(vocab_offset),
              float(temperature), parts.data_ptr(), tok.data_ptr(), ws.data_ptr(), ws.numel(), _stream(dev))
    return parts, tok


def accept_merge_shards(parts_all: torch.Tensor, tok_all: torch.Tensor):
    """Step 3: ``parts_all`` [shards, rows, 2] int64, ``tok_all`` [shards, rows]
    f32 (all-gathered in shard order) -> (row statistics [rows, 4] int32
    holding 16-byte records, merged token logits [rows] f32)."""
    dev = _need_cuda(parts_all, tok_all)
    K, R = tok_all.shape
    stats = torch.empty(R, 4, dtype=torch.int32, device=dev)
    tok = torch.empty(R, dtype=torch.float32, device=dev)
    _lib.call("pts_accept_merge_shards", parts_all.contiguous().data_ptr(), tok_all.contiguous().data_ptr(), K, R,
              stats.data_ptr(), tok.data_ptr(), _stream(dev))
    return stats, tok


def accept_shard_ties(logits_shard: torch.Tensor, vocab_offset: int, stats: torch.Tensor,
                      temperature: float = 1.0) -> torch.Tensor:
    """Step 4: per tied row the first index of this shard holding the row's
    largest rounded probability (INT_MAX elsewhere), [rows] int32."""
    dev = _need_cuda(logits_shard, stats)
    R, Vs = logits_shard.shape
    first = torch.empty(R, dtype=torch.int32, device=dev)
    _lib.call("pts_accept_shard_ties", logits_shard.data_ptr(), logits_shard.stride(0), R, Vs, int(vocab_offset),
              float(temperature), stats.data_ptr(), first.data_ptr(), _stream(dev))
    return first


def accept_walk_merged(stats: torch.Tensor, tok: torch.Tensor, ties_all: torch.Tensor, vocab: int,
                       row_indptr: torch.Tensor, parents: torch.Tensor, tokens: torch.Tensor,
                       draft_probs: Optional[torch.Tensor] = None, eos_token_id: Optional[int] = None,
                       seed: int = 0, offset: int = 0, max_nodes: Optional[int] = None):
    """Step 6: greedy (``draft_probs`` None) or traversal walks from merged
    statistics; same outputs as ``accept_greedy`` / ``accept_traversal``."""
    dev = _need_cuda(stats, tok, ties_all, row_indptr, parents, tokens)
    row_indptr, parents, tokens = _i32(row_indptr, "a"), _i32(parents, "b"), _i32(tokens, "c")
    B = row_indptr.numel() - 1
    R = tok.numel()
    mn = min(int(max_nodes) if max_nodes is not None else R, _lib.PTS_MAX_TREE_NODES)
    ot = torch.empty(B, mn, dtype=torch.int32, device=dev)
    oh = torch.empty(B, mn, dtype=torch.int32, device=dev)
    oc = torch.empty(B, 4, dtype=torch.int32, device=dev)
    dp = None
    if draft_probs is not None:
        dp = draft_probs.to(torch.float32).contiguous()
    _lib.call("pts_accept_walk_merged", stats.data_ptr(), tok.data_ptr(), ties_all.contiguous().data_ptr(),
              ties_all.shape[0], row_indptr.data_ptr(), parents.data_ptr(), tokens.data_ptr(),
              dp.data_ptr() if dp is not None else None, B, R, int(vocab), mn,
              -1 if eos_token_id is None else int(eos_token_id), int(seed) & (2 ** 64 - 1),
              int(offset) & (2 ** 64 - 1), ot.data_ptr(), oh.data_ptr(), oc.data_ptr(), mn, _stream(dev))
    return ot, oh, oc


def gather_shards(t: torch.Tensor, group=None) -> torch.Tensor:
    """All-gather ``t`` from every rank of ``group`` into [ranks, *t.shape],
    rank r's tensor at index r (rank order is shard order).  One collective
    into one buffer; NCCL for CUDA tensors, gloo for CPU tensors.  Without an
    initialised process group the result is ``t`` itself as the one shard."""
    import torch.distributed as dist
    if not (dist.is_available() and dist.is_initialized()):
        return t.unsqueeze(0)
    K = dist.get_world_size(group)
    t = t.contiguous()
    out = torch.empty(K * t.shape[0], *t.shape[1:], dtype=t.dtype, device=t.device)
    dist.all_gather_into_tensor(out, t, group=group)
    return out.view(K, *t.shape)


def accept_sharded(logits_shard: torch.Tensor, vocab_offset: int, vocab: int, row_indptr: torch.Tensor,
                   parents: torch.Tensor, tokens: torch.Tensor, draft_probs: Optional[torch.Tensor] = None,
                   group=None, eos_token_id: Optional[int] = None, temperature: float = 1.0, seed: int = 0,
                   offset: int = 0, max_nodes: Optional[int] = None):
    """Tensor-parallel acceptance on one rank of ``group`` (torch.distributed,
    NCCL): the shard partials and the tie indices are all-gathered, every
    rank merges in shard order and walks; all ranks return the same paths."""
    parts, tok = accept_shard_partials(logits_shard, vocab_offset, row_indptr, parents, tokens, temperature)
    stats, tokm = accept_merge_shards(gather_shards(parts, group), gather_shards(tok, group))
    ties_all = gather_shards(accept_shard_ties(logits_shard, vocab_offset, stats, temperature), group)
    return accept_walk_merged(stats, tokm, ties_all, vocab, row_indptr, parents, tokens, draft_probs,
                              eos_token_id, seed, offset, max_nodes)


# ------------------------------------------------------------------ paged KV
def batch_positions(append_indptr: torch.Tensor, seq_lens: torch.Tensor, num_tokens: int):
    dev = _need_cuda(append_indptr, seq_lens)
    append_indptr, seq_lens = _i32(append_indptr, "append_indptr"), _i32(seq_lens, "seq_lens")
    bi = torch.empty(num_tokens, dtype=torch.int32, device=dev)
    pos = torch.empty(num_tokens, dtype=torch.int32, device=dev)
    _lib.call("pts_batch_positions", append_indptr.data_ptr(), seq_lens.data_ptr(), append_indptr.numel() - 1,
              num_tokens, bi.data_ptr(), pos.data_ptr(), _stream(dev))
    return bi, pos


def kv_append(k: torch.Tensor, v: torch.Tensor, kv_layer: torch.Tensor, batch_indices: torch.Tensor,
              positions: torch.Tensor, page_indptr: torch.Tensor, page_indices: torch.Tensor) -> None:
    """Scatter k/v [T, Hkv, D] into one layer [max_pages, 2, page_len, Hkv, D]."""
    dev = _need_cuda(k, v, kv_layer, batch_indices, positions, page_indptr, page_indices)
    if kv_layer.dim() != 5 or kv_layer.shape[1] != 2:
        raise ValueError("kv_layer must be [max_pages, 2, page_len, Hkv, D]")
    if not kv_layer.is_contiguous():
        raise ValueError("kv_layer must be contiguous")
    P, _, pl, H, D = kv_layer.shape
    if k.dtype != kv_layer.dtype or v.dtype != kv_layer.dtype:
        raise ValueError("k/v dtype must match the cache dtype")
    k = k.reshape(k.shape[0], H * D) if k.stride(-1) == 1 and k[0].is_contiguous() else k.contiguous().reshape(-1, H * D)
    v = v.reshape(v.shape[0], H * D) if v.stride(-1) == 1 and v[0].is_contiguous() else v.contiguous().reshape(-1, H * D)
    _lib.call("pts_kv_append", k.data_ptr(), v.data_ptr(), k.stride(0), v.stride(0), kv_layer.data_ptr(),
              _i32(batch_indices, "bi").data_ptr(), _i32(positions, "pos").data_ptr(),
              _i32(page_indptr, "indptr").data_ptr(), _i32(page_indices, "indices").data_ptr(), k.shape[0], H, D, pl,
              P, kv_layer.element_size(), _stream(dev))


def kv_append_rope(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor,
                   kv_layer: torch.Tensor, batch_indices: torch.Tensor, positions: torch.Tensor,
                   page_indptr: torch.Tensor, page_indices: torch.Tensor,
                   q_out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``kv_append`` with the rotary embedding: q [T, Hq, D] and k/v
    [T, Hkv, D] before RoPE, cos/sin [T, D] their position embeddings; k is
    rotated into the cache and the rotated q is returned."""
    dev = _need_cuda(q, k, v, cos, sin, kv_layer, batch_indices, positions, page_indptr, page_indices)
    if kv_layer.dim() != 5 or kv_layer.shape[1] != 2 or not kv_layer.is_contiguous():
        raise ValueError("kv_layer must be a contiguous [max_pages, 2, page_len, Hkv, D] tensor")
    P, _, pl, H, D = kv_layer.shape
    dt = kv_layer.dtype
    if any(t.dtype != dt for t in (q, k, v, cos, sin)):
        raise ValueError("q, k, v, cos and sin must have the cache dtype")
    T = q.shape[0]
    rows = lambda t, w: t.reshape(T, w) if t.stride(-1) == 1 and t[0].is_contiguous() else t.contiguous().reshape(T, w)
    q2, k2, v2 = rows(q, q.shape[1] * D), rows(k, H * D), rows(v, H * D)
    cos2, sin2 = rows(cos, D), rows(sin, D)
    if cos2.stride(0) != sin2.stride(0):
        cos2, sin2 = cos2.contiguous(), sin2.contiguous()
    if q_out is None:
        q_out = torch.empty(T, q.shape[1], D, dtype=dt, device=dev)
    _lib.call("pts_kv_append_rope", q2.data_ptr(), q2.stride(0), q_out.data_ptr(), q.shape[1], k2.data_ptr(),
              v2.data_ptr(), k2.stride(0), v2.stride(0), cos2.data_ptr(), sin2.data_ptr(), cos2.stride(0),
              kv_layer.data_ptr(), _i32(batch_indices, "bi").data_ptr(), _i32(positions, "pos").data_ptr(),
              _i32(page_indptr, "indptr").data_ptr(), _i32(page_indices, "indices").data_ptr(), T, H, D, pl, P,
              kv_layer.element_size(), _stream(dev))
    return q_out


def kv_compact(pool: torch.Tensor, page_indptr: torch.Tensor, page_indices: torch.Tensor,
               accepted: torch.Tensor, accepted_counts: torch.Tensor, offsets: torch.Tensor,
               new_kv_len: Optional[torch.Tensor] = None, new_last_page_len: Optional[torch.Tensor] = None) -> None:
    """For request b copy slot offsets[b] + accepted[b, i] -> offsets[b] + i,
    i < accepted_counts[b, 0], in every layer of ``pool``
    [L, max_pages, 2, page_len, Hkv, D].  ``accepted`` is [B, S] int32 and
    ``accepted_counts`` [B] or [B, C] (first column used), which is what the
    acceptance kernels return."""
    dev = _need_cuda(pool, page_indptr, page_indices, accepted, accepted_counts, offsets)
    if pool.dim() != 6 or pool.shape[2] != 2 or not pool.is_contiguous():
        raise ValueError("pool must be a contiguous [L, max_pages, 2, page_len, Hkv, D] tensor")
    L, P, _, pl, H, D = pool.shape
    accepted = _i32(accepted, "accepted")
    if accepted.dim() != 2:
        raise ValueError("accepted must be [B, S]")
    counts = _i32(accepted_counts, "counts")
    cstride = 1 if counts.dim() == 1 else counts.stride(0)
    B, S = accepted.shape
    _lib.call("pts_kv_compact", pool.data_ptr(), L, P, pl, H, D, pool.element_size(),
              _i32(page_indptr, "a").data_ptr(), _i32(page_indices, "b").data_ptr(), accepted.data_ptr(),
              accepted.stride(0), counts.data_ptr(), cstride, _i32(offsets, "e").data_ptr(), B, S,
              new_kv_len.data_ptr() if new_kv_len is not None else None,
              new_last_page_len.data_ptr() if new_last_page_len is not None else None, _stream(dev))


# ------------------------------------------------------------------ attention
def mask_words_for(max_nodes: int) -> int:
    return max(1, math.ceil(max_nodes / 64))


def tree_mask_from_parents(parents: torch.Tensor, qo_indptr: torch.Tensor, mask_words: int) -> torch.Tensor:
    dev = _need_cuda(parents, qo_indptr)
    parents, qo_indptr = _i32(parents, "parents"), _i32(qo_indptr, "qo_indptr")
    T = parents.numel()
    bits = torch.empty(T, mask_words, dtype=torch.int64, device=dev)
    _lib.call("pts_tree_mask_from_parents", parents.data_ptr(), qo_indptr.data_ptr(), qo_indptr.numel() - 1, T,
              mask_words, bits.data_ptr(), _stream(dev))
    return bits


def tree_prepare(parents: torch.Tensor, qo_indptr: torch.Tensor, mask_words: int,
                 seq_lens: Optional[torch.Tensor] = None):
    """One launch per tree step: ancestor bitmasks [T, mask_words] and, with
    ``seq_lens``, the append batch indices and positions of the tree tokens."""
    dev = _need_cuda(parents, qo_indptr)
    parents, qo_indptr = _i32(parents, "parents"), _i32(qo_indptr, "qo_indptr")
    T = parents.numel()
    bits = torch.empty(T, mask_words, dtype=torch.int64, device=dev)
    bi = pos = None
    if seq_lens is not None:
        bi = torch.empty(T, dtype=torch.int32, device=dev)
        pos = torch.empty(T, dtype=torch.int32, device=dev)
    _lib.call("pts_tree_prepare", parents.data_ptr(), qo_indptr.data_ptr(),
              _i32(seq_lens, "seq_lens").data_ptr() if seq_lens is not None else None, qo_indptr.numel() - 1,
              mask_words, bits.data_ptr(), bi.data_ptr() if bi is not None else None,
              pos.data_ptr() if pos is not None else None, _stream(dev))
    return bits, bi, pos


def tree_prepare_append(parents: torch.Tensor, qo_indptr: torch.Tensor, mask_words: int, seq_lens: torch.Tensor,
                        k: torch.Tensor, v: torch.Tensor, kv_layer: torch.Tensor, page_indptr: torch.Tensor,
                        page_indices: torch.Tensor):
    """``tree_prepare`` with positions and ``kv_append`` of the tree tokens'
    k/v [T, Hkv, D] into one layer [max_pages, 2, page_len, Hkv, D], in one
    launch.  Returns (bits, batch_indices, positions)."""
    dev = _need_cuda(parents, qo_indptr, seq_lens, k, v, kv_layer, page_indptr, page_indices)
    if kv_layer.dim() != 5 or kv_layer.shape[1] != 2 or not kv_layer.is_contiguous():
        raise ValueError("kv_layer must be a contiguous [max_pages, 2, page_len, Hkv, D] tensor")
    P, _, pl, H, D = kv_layer.shape
    if k.dtype != kv_layer.dtype or v.dtype != kv_layer.dtype:
        raise ValueError("k/v dtype must match the cache dtype")
    parents, qo_indptr = _i32(parents, "parents"), _i32(qo_indptr, "qo_indptr")
    T = parents.numel()
    if k.shape[0] != T or v.shape[0] != T:
        raise ValueError("k and v need one row per tree token")
    k = k.reshape(T, H * D) if k.stride(-1) == 1 and k[0].is_contiguous() else k.contiguous().reshape(-1, H * D)
    v = v.reshape(T, H * D) if v.stride(-1) == 1 and v[0].is_contiguous() else v.contiguous().reshape(-1, H * D)
    bits = torch.empty(T, mask_words, dtype=torch.int64, device=dev)
    bi = torch.empty(T, dtype=torch.int32, device=dev)
    pos = torch.empty(T, dtype=torch.int32, device=dev)
    _lib.call("pts_tree_prepare_append", parents.data_ptr(), qo_indptr.data_ptr(), _i32(seq_lens, "seq_lens").data_ptr(),
              qo_indptr.numel() - 1, mask_words, bits.data_ptr(), bi.data_ptr(), pos.data_ptr(), k.data_ptr(),
              v.data_ptr(), k.stride(0), v.stride(0), kv_layer.data_ptr(), _i32(page_indptr, "indptr").data_ptr(),
              _i32(page_indices, "indices").data_ptr(), T, H, D, pl, P, kv_layer.element_size(), _stream(dev))
    return bits, bi, pos


def tree_prepare_append_rope(parents: torch.Tensor, qo_indptr: torch.Tensor, mask_words: int,
                             seq_lens: torch.Tensor, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                             cos: torch.Tensor, sin: torch.Tensor, kv_layer: torch.Tensor, page_indptr: torch.Tensor,
                             page_indices: torch.Tensor, q_out: Optional[torch.Tensor] = None):
    """``tree_prepare_append`` with the rotary embedding applied on the way:
    q [T, Hq, D], k/v [T, Hkv, D] are the tree tokens' projections before
    RoPE and cos/sin [T, D] their position embeddings (the model's
    ``position_embeddings``).  k is rotated into the cache and q into
    ``q_out``.  Returns (bits, batch_indices, positions, q_out)."""
    dev = _need_cuda(parents, qo_indptr, seq_lens, q, k, v, cos, sin, kv_layer, page_indptr, page_indices)
    if kv_layer.dim() != 5 or kv_layer.shape[1] != 2 or not kv_layer.is_contiguous():
        raise ValueError("kv_layer must be a contiguous [max_pages, 2, page_len, Hkv, D] tensor")
    P, _, pl, H, D = kv_layer.shape
    dt = kv_layer.dtype
    if any(t.dtype != dt for t in (q, k, v, cos, sin)):
        raise ValueError("q, k, v, cos and sin must have the cache dtype")
    parents, qo_indptr = _i32(parents, "parents"), _i32(qo_indptr, "qo_indptr")
    T = parents.numel()
    if q.dim() != 3 or q.shape[0] != T or q.shape[2] != D or k.shape[0] != T or v.shape[0] != T:
        raise ValueError("q [T, Hq, D] and k, v [T, Hkv, D] need one row per tree token")
    rows = lambda t, w: t.reshape(T, w) if t.stride(-1) == 1 and t[0].is_contiguous() else t.contiguous().reshape(T, w)
    q2, k2, v2 = rows(q, q.shape[1] * D), rows(k, H * D), rows(v, H * D)
    cos2, sin2 = rows(cos, D), rows(sin, D)
    if cos2.stride(0) != sin2.stride(0):
        cos2, sin2 = cos2.contiguous(), sin2.contiguous()
    if q_out is None:
        q_out = torch.empty(T, q.shape[1], D, dtype=dt, device=dev)
    bits = torch.empty(T, mask_words, dtype=torch.int64, device=dev)
    bi = torch.empty(T, dtype=torch.int32, device=dev)
    pos = torch.empty(T, dtype=torch.int32, device=dev)
    _lib.call("pts_tree_prepare_append_rope", parents.data_ptr(), qo_indptr.data_ptr(),
              _i32(seq_lens, "seq_lens").data_ptr(), qo_indptr.numel() - 1, mask_words, bits.data_ptr(),
              bi.data_ptr(), pos.data_ptr(), q2.data_ptr(), q2.stride(0), q_out.data_ptr(), q.shape[1],
              k2.data_ptr(), v2.data_ptr(), k2.stride(0), v2.stride(0), cos2.data_ptr(), sin2.data_ptr(),
              cos2.stride(0), kv_layer.data_ptr(), _i32(page_indptr, "indptr").data_ptr(),
              _i32(page_indices, "indices").data_ptr(), T, H, D, pl, P, kv_layer.element_size(), _stream(dev))
    return bits, bi, pos, q_out


def tree_mask_from_bool(mask: torch.Tensor, qo_indptr: torch.Tensor, mask_indptr: torch.Tensor,
                        kv_lens: torch.Tensor, mask_words: int, total_q: Optional[int] = None,
                        check: bool = True) -> torch.Tensor:
    """Pack a flattened boolean tree mask into per-row ancestor bitmasks.
    With ``check`` the prefix columns are verified on the device and a
    non-tree mask raises ValueError (one device-to-host read)."""
    dev = _need_cuda(mask, qo_indptr, mask_indptr, kv_lens)
    if mask.dtype != torch.bool:
        mask = mask.to(torch.bool)
    mask = mask.contiguous()
    qo_indptr = _i32(qo_indptr, "qo")
    if total_q is None:
        total_q = int(qo_indptr[-1].item())
    bad = torch.zeros(1, dtype=torch.int32, device=dev)
    bits = torch.empty(total_q, mask_words, dtype=torch.int64, device=dev)
    _lib.call("pts_tree_mask_from_bool", mask.data_ptr(), qo_indptr.data_ptr(), _i32(mask_indptr, "mi").data_ptr(),
              _i32(kv_lens, "kl").data_ptr(), qo_indptr.numel() - 1, total_q, mask_words, bits.data_ptr(),
              bad.data_ptr(), _stream(dev))
    if check and int(bad.item()) != 0:
        raise ValueError("custom mask is not a tree mask: a prefix column is masked out")
    return bits


def tree_attention(q: torch.Tensor, kv_layer: torch.Tensor, qo_indptr: torch.Tensor, page_indptr: torch.Tensor,
                   page_indices: torch.Tensor, last_page_len: torch.Tensor, mask_bits: Optional[torch.Tensor],
                   max_qo_len: int, max_kv_len: int, sm_scale: Optional[float] = None,
                   out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Tree-masked paged attention: q [T, Hq, D], kv_layer [P, 2, page_len, Hkv, D],
    both bf16 or both fp32; ``mask_bits`` None means causal rows.  bf16 with
    head_dim 128 and 16-token pages runs on the tensor cores, other shapes
    on the SIMT kernel."""
    dev = _need_cuda(q, kv_layer, qo_indptr, page_indptr, page_indices, last_page_len,
                     *([mask_bits] if mask_bits is not None else []))
    if q.dtype not in (torch.bfloat16, torch.float32) or kv_layer.dtype != q.dtype:
        raise ValueError("tree attention takes bf16 or fp32 queries and a cache of the same type")
    if not q.is_contiguous() or not kv_layer.is_contiguous():
        raise ValueError("q and kv_layer must be contiguous")
    T, Hq, D = q.shape
    P, _, pl, Hkv, D2 = kv_layer.shape
    if D2 != D:
        raise ValueError("head_dim mismatch between q and cache")
    B = qo_indptr.numel() - 1
    if out is None:
        out = torch.empty_like(q)
    scale = float(sm_scale) if sm_scale is not None else 1.0 / math.sqrt(D)
    wsz = _lib.lib().pts_tree_attn_workspace_size(B, T, Hq, D, int(max_kv_len))
    ws = workspace(dev, "attn", max(wsz, 256))
    _lib.call("pts_tree_attn_run_any", q.data_ptr(), kv_layer.data_ptr(), _i32(qo_indptr, "qo").data_ptr(),
              _i32(page_indptr, "pi").data_ptr(), _i32(page_indices, "px").data_ptr(),
              _i32(last_page_len, "lp").data_ptr(), mask_bits.data_ptr() if mask_bits is not None else None,
              mask_bits.shape[1] if mask_bits is not None else 1, out.data_ptr(), B, T,
              int(max_qo_len), int(max_kv_len), Hq, Hkv, D, pl, P, scale, q.element_size(), ws.data_ptr(),
              ws.numel(), _stream(dev))
    if _CHECK_ATTENTION:
        check_attention(dev)
    return out


# PTS_B200_CHECK=1: read the attention kernels' error word after every call
# (synchronises the stream; for debugging).
_CHECK_ATTENTION = os.environ.get("PTS_B200_CHECK", "0") not in ("", "0")


def check_attention(device: Optional[torch.device] = None) -> None:
    """Raise if an attention launch on the current stream gave up waiting
    (pts_tree_attn_check: synchronises the stream, then clears the error)."""
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    ws = workspace(dev, "attn", 256)
    status = C.c_int(0)
    _lib.call("pts_tree_attn_check", ws.data_ptr(), C.addressof(status), _stream(dev))
    if status.value != 0:
        raise RuntimeError(f"tree attention gave up waiting (error {status.value}); its output is not valid")


def set_wait_limit(cycles: int) -> int:
    """Process-wide limit (SM clocks) on the kernels' waits; <= 0 restores the
    default.  Returns the previous limit."""
    return int(_lib.lib().pts_set_wait_limit(int(cycles)))


ATTN_SCHEDULE_AUTO, ATTN_SCHEDULE_PER_UNIT, ATTN_SCHEDULE_BALANCED = 0, 1, 2


def set_attention_schedule(mode: int) -> int:
    """Process-wide attention schedule (pts_tree_attn_set_schedule): 0 chooses
    per launch, 1 one CTA per (request, KV head, row group), 2 balanced block
    ranges over one CTA per SM.  Returns the previous choice."""
    prev = int(_lib.lib().pts_tree_attn_set_schedule(int(mode)))
    if prev < 0:
        raise ValueError(f"attention schedule {mode}: expected 0, 1 or 2")
    return prev


# ------------------------------------------------------------ sparse page sets
def page_key_sums(kv_layer: torch.Tensor, page_ids: torch.Tensor) -> torch.Tensor:
    """Per page and KV head the fp32 sum of its keys: [n, Hkv, D] float32
    (a page summary computed once, when the page is full)."""
    dev = _need_cuda(kv_layer, page_ids)
    P, _, pl, H, D = kv_layer.shape
    ids = _i32(page_ids, "page_ids")
    out = torch.empty(ids.numel(), H, D, dtype=torch.float32, device=dev)
    _lib.call("pts_page_key_sums", kv_layer.data_ptr(), ids.data_ptr(), ids.numel(), H, D, pl, out.data_ptr(),
              _stream(dev))
    return out


def select_pages(key_sums: torch.Tensor, page_indptr: torch.Tensor, page_indices: torch.Tensor,
                 last_page_len: torch.Tensor, q: torch.Tensor, qo_indptr: torch.Tensor, num_kv_heads: int,
                 n_first: int = 4, n_top: int = 64, n_last: int = 8, page_len: int = 16,
                 max_prefix_pages: Optional[int] = None):
    """Per-(request, KV head) sparse page tables for pts_tree_attn_run_head_pages:
    the first ``n_first`` and last ``n_last`` full prefix pages, the ``n_top``
    middle pages of highest root-query . key-sum score, and the pages that
    hold the tree.  ``key_sums`` is aligned with ``page_indices``.  Returns
    (head_indptr [B*Hkv+1], head_indices, head_last_page_len [B*Hkv])."""
    dev = _need_cuda(key_sums, page_indptr, page_indices, last_page_len, q, qo_indptr)
    page_indptr, page_indices = _i32(page_indptr, "a"), _i32(page_indices, "b")
    B = page_indptr.numel() - 1
    T, Hq, D = q.shape
    if max_prefix_pages is None:
        max_prefix_pages = int((page_indptr[1:] - page_indptr[:-1]).max().item())
    indptr = torch.empty(B * num_kv_heads + 1, dtype=torch.int32, device=dev)
    indices = torch.empty(num_kv_heads * page_indices.numel(), dtype=torch.int32, device=dev)
    last = torch.empty(B * num_kv_heads, dtype=torch.int32, device=dev)
    _lib.call("pts_select_pages", key_sums.data_ptr(), page_indptr.data_ptr(), page_indices.data_ptr(),
              _i32(last_page_len, "c").data_ptr(), q.data_ptr(), _i32(qo_indptr, "d").data_ptr(), B, Hq,
              num_kv_heads, D, page_len, n_first, n_top, n_last, int(max_prefix_pages), indptr.data_ptr(),
              indices.data_ptr(), last.data_ptr(), _stream(dev))
    return indptr, indices, last


def tree_attention_head_pages(q: torch.Tensor, kv_layer: torch.Tensor, qo_indptr: torch.Tensor,
                              head_indptr: torch.Tensor, head_indices: torch.Tensor, head_last: torch.Tensor,
                              mask_bits: Optional[torch.Tensor], max_qo_len: int, max_kv_len: int,
                              sm_scale: Optional[float] = None, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Tree attention where KV head h of request b reads its own page list
    (index b * Hkv + h); the tree occupies the last N slots of every list."""
    dev = _need_cuda(q, kv_layer, qo_indptr, head_indptr, head_indices, head_last)
    T, Hq, D = q.shape
    P, _, pl, Hkv, _ = kv_layer.shape
    B = qo_indptr.numel() - 1
    if out is None:
        out = torch.empty_like(q)
    scale = float(sm_scale) if sm_scale is not None else 1.0 / math.sqrt(D)
    # the same workspace as tree_attention, so the two choose their schedule alike
    wsz = _lib.lib().pts_tree_attn_workspace_size(B, T, Hq, D, int(max_kv_len))
    ws = workspace(dev, "attn", max(wsz, 256))
    _lib.call("pts_tree_attn_run_head_pages", q.data_ptr(), kv_layer.data_ptr(), _i32(qo_indptr, "qo").data_ptr(),
              _i32(head_indptr, "hi").data_ptr(), _i32(head_indices, "hx").data_ptr(),
              _i32(head_last, "hl").data_ptr(), mask_bits.data_ptr() if mask_bits is not None else None,
              mask_bits.shape[1] if mask_bits is not None else 1, out.data_ptr(), B, T, int(max_qo_len),
              int(max_kv_len), Hq, Hkv, D, pl, P, scale, ws.data_ptr(), ws.numel(), _stream(dev))
    return out


# ------------------------------------------------------------ draft beam search
def beam_select(logits: torch.Tensor, k: int, temperature: float = 1.0,
                cum_log_probs: Optional[torch.Tensor] = None):
    """The beam search's per-step selection (``beam_search.py:549-561``):
    the k best of ``cum[:, None] + log(softmax(logits / T) + 1e-10)`` over the
    flattened [rows, vocab] scores, or with ``cum_log_probs`` None the k best
    probabilities of the rows (the first step, ``:432-433``).  Returns
    (scores fp32 [k], flat indices int64 [k], probabilities fp32 [k]), best
    first, ties to the smaller flat index."""
    dev = _need_cuda(logits)
    if logits.dim() != 2 or logits.dtype not in (torch.bfloat16, torch.float32):
        raise ValueError("logits must be a 2-D bf16 or fp32 tensor [rows, vocab]")
    if logits.stride(1) != 1:
        logits = logits.contiguous()
    rows, vocab = logits.shape
    cum_ptr = None
    if cum_log_probs is not None:
        _need_cuda(logits, cum_log_probs)
        cum_log_probs = cum_log_probs.to(torch.float32).contiguous()
        if cum_log_probs.numel() != rows:
            raise ValueError("cum_log_probs needs one value per row")
        cum_ptr = cum_log_probs.data_ptr()
    score = torch.empty(k, dtype=torch.float32, device=dev)
    index = torch.empty(k, dtype=torch.int64, device=dev)
    prob = torch.empty(k, dtype=torch.float32, device=dev)
    nbytes = _lib.lib().pts_beam_select_workspace_size(rows, k)
    ws = workspace(dev, "beam", max(nbytes, 256))
    _lib.call("pts_beam_select", logits.data_ptr(), logits.stride(0), logits.element_size(), rows, vocab,
              float(temperature), cum_ptr, k, score.data_ptr(), index.data_ptr(), prob.data_ptr(), ws.data_ptr(),
              ws.numel(), _stream(dev))
    return score, index, prob


def kv_copy_pages(cache_data: torch.Tensor, src_pages: torch.Tensor, dst_pages: torch.Tensor, tokens: int) -> None:
    """Copy-on-write copies of one decode step (``beam_search.py:92-96``):
    ``cache_data[:, dst, :, :tokens] = cache_data[:, src, :, :tokens]`` for
    every pair, in one launch.  ``cache_data``: the pool [L, P, 2, page, H, D]."""
    dev = _need_cuda(cache_data, src_pages, dst_pages)
    if cache_data.dim() != 6 or not cache_data.is_contiguous():
        raise ValueError("cache_data must be a contiguous [layers, pages, 2, page_len, heads, dim] tensor")
    L, P, _, page_len, H, D = cache_data.shape
    src, dst = _i32(src_pages, "src_pages"), _i32(dst_pages, "dst_pages")
    if src.numel() != dst.numel():
        raise ValueError("src_pages and dst_pages differ in length")
    _lib.call("pts_kv_copy_pages", cache_data.data_ptr(), L, P, page_len, H * D * cache_data.element_size(),
              src.data_ptr(), dst.data_ptr(), src.numel(), int(tokens), _stream(dev))
