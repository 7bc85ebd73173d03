"""Tree verification, interface of the reference's ``verification.py``.

Same functions, arguments and return values as ``parallel_tree_spec.verification``
(``verification.py:32-588``): ``VerifyResult``, ``prepare_tree_inputs``,
``target_tree_decode``, ``verify_tree_exact``, ``verify_tree_traversal``,
``verify_draft_tree``.  Acceptance runs as one fused kernel over the bf16
logits on the device (``pts_accept_greedy`` / ``pts_accept_traversal``); only
the tree's flat columns go to the device and only the accepted path comes
back.  ``verify_trees`` verifies a whole batch of trees in one launch.

Stochastic draws: where the reference calls ``torch.rand(1)`` once per loop
iteration (``verification.py:396``), the kernel uses the Philox4x32-10
stream of (seed, offset, request): ``set_traversal_seed`` fixes the seed
(default ``torch.initial_seed()``) and every call advances the offset, so
successive calls draw fresh uniforms.  Given the same uniforms the accepted
path is the reference's, bit for bit.

Limits of this build: bf16 or fp32 logits on a CUDA device (top-p and
sampled bonuses with bf16), ``root_ind == 0`` and
``skip_nodes == 0`` (the only values the reference's own caller passes,
``verification.py:569-576``), sibling tokens distinct (the reference's greedy
walk fails on duplicates, ``verification.py:245-246``).
"""
from __future__ import annotations

import time
from dataclasses import dataclass
from typing import List, Optional, Sequence, Tuple

import numpy as np
import torch

from . import kernels as K
from .attention_wrapper import BeFlashinferWrapper
from .cache_manager import KvCachePool, RequestKvCache, getKvCacheBatchPosition
from .tree import Tree, tree_columns


@dataclass
class VerifyResult:
    """Result of one draft-verify cycle (``verification.py:32-39``)."""
    sampled_tokens: torch.Tensor
    hidden_indices: torch.Tensor
    total_len: int
    accept_len: int
    verify_time: float


_stream_state = {"seed": None, "offset": 0}


def set_traversal_seed(seed: int, offset: int = 0) -> None:
    """Fix the Philox seed (and starting offset) of traversal verification."""
    _stream_state["seed"] = int(seed)
    _stream_state["offset"] = int(offset)


def _next_stream() -> Tuple[int, int]:
    seed = _stream_state["seed"] if _stream_state["seed"] is not None else torch.initial_seed()
    off = _stream_state["offset"]
    _stream_state["offset"] = off + 1
    return int(seed), int(off)


def _sample_probs(logits: torch.Tensor) -> torch.Tensor:
    """Softmax over the last dim (``verification.py:46-55``)."""
    return torch.softmax(logits, dim=-1)


def _verify_step_greedy(probs: torch.Tensor, children_token_ids: torch.Tensor):
    """Argmax of ``probs`` and whether a child carries it (``verification.py:58-77``)."""
    tok = probs.argmax()
    if torch.any(tok == children_token_ids):
        return tok, None
    return None, tok


def prepare_tree_inputs(tree: Tree, position_offset: int, device, skip_nodes: int = 0):
    """(input ids [N], position ids = depth + offset [N], mask [1, 1, N, offset+1+N])
    (``verification.py:84-112``)."""
    data = tree.get_tree_data(skip_nodes)
    ids = data["token_ids"].to(device)
    pos = (data["depths"] + position_offset).to(device)
    mask = tree.create_attention_mask(prefix_length=position_offset + 1, skip_nodes=skip_nodes, device=device)
    return ids, pos, mask


@torch.no_grad()
def target_tree_decode(target_model: torch.nn.Module, flashinfer_wrapper: BeFlashinferWrapper, tree: Tree,
                       request_kv_cache: RequestKvCache, position_offset: int, device) -> torch.Tensor:
    """Target forward over the draft tree with tree attention; logits [1, N, V]
    (``verification.py:119-178``)."""
    pool = request_kv_cache.kvCachePool
    n = tree.current_size
    ids, pos, mask = prepare_tree_inputs(tree, position_offset=position_offset, device=device)
    request_kv_cache.increment(n)
    bp = getKvCacheBatchPosition(request_kv_caches=[request_kv_cache], mode="tree", device=device, treeTokens=n)
    flashinfer_wrapper.prepareAttention("tree", bp, pool.page_len, "NONE", pool.cache_data[0].dtype,
                                        attention_mask=mask)
    out = target_model(input_ids=ids.unsqueeze(0), past_key_values=None, position_ids=pos.unsqueeze(0),
                       use_cache=False, kvCachePool=pool, batch_position=bp, mode="tree",
                       flashinferWrapper=flashinfer_wrapper)
    return out.logits


# ------------------------------------------------------------------ device glue
def _rows(logits: torch.Tensor) -> torch.Tensor:
    x = logits.reshape(-1, logits.shape[-1])
    if x.device.type != "cuda":
        raise ValueError("logits must be on a CUDA device (this path has no CPU implementation)")
    if x.dtype not in (torch.bfloat16, torch.float32):
        raise ValueError(f"logits must be bf16 or fp32 (got {x.dtype})")
    if x.stride(-1) != 1:
        x = x.contiguous()
    return x


_staging = {}


def _pinned(device, n: int) -> torch.Tensor:
    """A pinned host staging buffer per device, grown on demand.  Before it is
    refilled, the host waits for the copy that last read it."""
    key = str(device)
    entry = _staging.get(key)
    if entry is not None and entry[1] is not None:
        entry[1].synchronize()
    if entry is None or entry[0].numel() < n:
        entry = (torch.empty(max(n, 4096), dtype=torch.int32, pin_memory=True), None)
        _staging[key] = entry
    return entry[0]


def _copied(device, d: torch.Tensor) -> None:
    """Mark the staging buffer of ``device`` as read by the copy just enqueued."""
    ev = torch.cuda.Event()
    ev.record(torch.cuda.current_stream(d.device))
    _staging[str(device)] = (_staging[str(device)][0], ev)


def _tree_columns(trees: Sequence, device):
    """Row pointers, parents, tokens and draft probabilities of a batch of
    trees (read through ``get_tree_data()``), moved to ``device`` in one copy."""
    cols = [tree_columns(t) for t in trees]
    sizes = [c[0].shape[0] for c in cols]
    indptr = np.zeros(len(trees) + 1, dtype=np.int32)
    indptr[1:] = np.cumsum(sizes)
    B, T = len(trees), int(indptr[-1])
    total = B + 1 + 3 * T
    host = _pinned(device, total)
    h = host.numpy()
    h[: B + 1] = indptr
    o = B + 1
    h[o:o + T] = np.concatenate([c[0] for c in cols])
    h[o + T:o + 2 * T] = np.concatenate([c[1] for c in cols])
    h[o + 2 * T:o + 3 * T] = np.concatenate([c[2] for c in cols]).view(np.int32)
    d = host[:total].to(device, non_blocking=True)
    _copied(device, d)
    return (d[: B + 1], d[o:o + T], d[o + T:o + 2 * T], d[o + 2 * T:o + 3 * T].view(torch.float32), max(sizes))


def _check_args(root_ind: int, skip_nodes: int):
    if root_ind != 0 or skip_nodes != 0:
        raise ValueError("this build verifies from the root with skip_nodes=0 "
                         f"(got root_ind={root_ind}, skip_nodes={skip_nodes})")


def _results(ot, oh, oc, device_out):
    ot, oh, oc = ot.cpu(), oh.cpu(), oc.cpu()
    res = []
    for b in range(oc.shape[0]):
        n = int(oc[b, 0])
        if n == -3:
            raise RuntimeError(f"acceptance of tree {b} timed out waiting for its rows' statistics")
        if n < 0:
            raise ValueError(f"tree {b} is malformed (parents must precede children, root first)")
        toks = ot[b, :n].to(torch.long).unsqueeze(0)
        hid = oh[b, :n].to(torch.long)
        if device_out is not None:
            toks, hid = toks.to(device_out), hid.to(device_out)
        res.append((toks, hid, int(oc[b, 1]), int(oc[b, 2])))
    return res


def verify_trees(trees: Sequence[Tree], logits: torch.Tensor, method: str = "traversal",
                 eos_token_id: Optional[int] = None, temperature: float = 1.0, seed: Optional[int] = None,
                 offset: Optional[int] = None, top_p: float = 1.0, do_sample: bool = False) -> List[tuple]:
    """Verify a batch of trees in one launch.  ``logits``: [sum N, V] (trees
    back to back) or [B, N, V] bf16 on the device.  Returns one
    (sampled_tokens [1, L], hidden_indices [L], total_len, accept_len) per tree."""
    x = _rows(logits)
    indptr, par, tok, dp, max_n = _tree_columns(trees, x.device)
    if method == "exact":
        ot, oh, oc = K.accept_greedy(x, indptr, par, tok, eos_token_id=eos_token_id, max_nodes=max_n)
    elif method == "traversal":
        if seed is None or offset is None:
            s0, o0 = _next_stream()
            seed = s0 if seed is None else seed
            offset = o0 if offset is None else offset
        ot, oh, oc = K.accept_traversal(x, indptr, par, tok, dp, eos_token_id=eos_token_id, temperature=temperature,
                                        top_p=top_p, do_sample=do_sample, seed=seed, offset=offset, max_nodes=max_n)
    else:
        raise ValueError(f"Unknown verification method: {method!r} (expected 'traversal' or 'exact')")
    return _results(ot, oh, oc, None)


@torch.no_grad()
def verify_tree_exact(tree: Tree, logits: torch.Tensor, root_ind: int = 0, eos_token_id: Optional[int] = None,
                      skip_nodes: int = 0):
    """Greedy argmax matching along the tree (``verification.py:185-268``)."""
    _check_args(root_ind, skip_nodes)
    x = _rows(logits)
    if x.shape[0] != tree.current_size:
        raise ValueError(f"logits have {x.shape[0]} rows for a tree of {tree.current_size} nodes")
    return verify_trees([tree], x, "exact", eos_token_id=eos_token_id)[0]


@torch.no_grad()
def verify_tree_traversal(tree: Tree, logits: torch.Tensor, root_ind: int = 0, eos_token_id: Optional[int] = None,
                          skip_nodes: int = 0, do_sample: bool = False, temperature: float = 1.0):
    """Traversal verification (``verification.py:275-524``); outputs on
    ``logits.device`` like the reference."""
    _check_args(root_ind, skip_nodes)
    x = _rows(logits)
    if x.shape[0] != tree.current_size:
        raise ValueError(f"logits have {x.shape[0]} rows for a tree of {tree.current_size} nodes")
    s, h, tl, al = verify_trees([tree], x, "traversal", eos_token_id=eos_token_id, temperature=temperature,
                                do_sample=do_sample)[0]
    return s.to(logits.device), h.to(logits.device), tl, al


@torch.no_grad()
def verify_draft_tree(target_model: torch.nn.Module, flashinfer_wrapper: BeFlashinferWrapper, tree: Tree,
                      request_kv_cache: RequestKvCache, position_offset: int, device,
                      eos_token_id: Optional[int] = None, verification_method: str = "traversal",
                      temperature: float = 1.0) -> VerifyResult:
    """Target tree decode + verification (``verification.py:531-588``)."""
    t0 = time.perf_counter()
    logits = target_tree_decode(target_model, flashinfer_wrapper, tree, request_kv_cache, position_offset, device)
    if verification_method == "traversal":
        s, h, tl, al = verify_tree_traversal(tree, logits, root_ind=0, eos_token_id=eos_token_id,
                                             temperature=temperature)
    elif verification_method == "exact":
        s, h, tl, al = verify_tree_exact(tree, logits, root_ind=0, eos_token_id=eos_token_id)
    else:
        raise ValueError(f"Unknown verification method: {verification_method!r} (expected 'traversal' or 'exact')")
    return VerifyResult(sampled_tokens=s, hidden_indices=h, total_len=tl, accept_len=al,
                        verify_time=time.perf_counter() - t0)
