"""Acceptance oracle: softmax over bf16 logits, greedy walk, traversal walk.

Restates the reference (parallel_tree_spec, ``src/parallel_tree_spec``):

* ``row_probs``      -- ``_sample_probs`` (``verification.py:46-55``) on
  bf16 logits, optionally divided by the temperature first
  (``verification.py:310``), rounded to bf16 as torch does.
* ``greedy_walk``    -- ``verify_tree_exact`` (``verification.py:185-268``)
  with ``_verify_step_greedy`` (``verification.py:58-77``).
* ``traversal_walk`` -- ``verify_tree_traversal`` (``verification.py:275-524``),
  replaying its fp32-tensor / fp64-scalar operation order.

bf16 arrays are held as ``uint16`` bit patterns.  Temperature scaling follows
torch's CUDA path for ``bf16_tensor / python_float`` (multiply by the fp32
reciprocal, round to bf16), because the reference computes it on the GPU.
Sums over sibling sets run left to right in fp32.
"""
from __future__ import annotations

from typing import Iterable, List, Optional, Sequence

import numpy as np

EPS = 1e-8
EPS32 = np.float32(1e-8)


# --------------------------------------------------------------------- bf16
def f32_to_bf16_bits(x) -> np.ndarray:
    """Round float32 to bf16 (round-to-nearest-even), return uint16 bits."""
    x = np.asarray(x, dtype=np.float32)
    b = x.view(np.uint32).astype(np.uint64)
    nan = np.isnan(x)
    r = ((b + np.uint64(0x7FFF) + ((b >> np.uint64(16)) & np.uint64(1))) >> np.uint64(16)).astype(np.uint16)
    if np.any(nan):
        r = np.where(nan, np.uint16(0x7FC0), r)
    return r


def bf16_bits_to_f32(b) -> np.ndarray:
    b = np.asarray(b, dtype=np.uint16)
    return (b.astype(np.uint32) << np.uint32(16)).view(np.float32)


def round_bf16(x) -> np.ndarray:
    return bf16_bits_to_f32(f32_to_bf16_bits(x))


# ------------------------------------------------------------------ softmax
def scale_logits(row_bits: np.ndarray, temperature: float) -> np.ndarray:
    """``logits / temperature`` as torch computes it for a CUDA bf16 tensor
    (``verification.py:310``): x * fp32(1/fp32(T)), rounded to bf16.
    Returns float32 values (exactly bf16-representable)."""
    x = bf16_bits_to_f32(row_bits)
    if temperature == 1.0:
        return x
    inv = np.float32(1.0) / np.float32(temperature)
    return round_bf16(x * inv)


def row_probs(row_bits: np.ndarray, temperature: float = 1.0) -> np.ndarray:
    """bf16-rounded softmax of one or more rows (last axis), float32 values.

    exp is evaluated in float64 and rounded to float32, the row sum is taken
    in float64 and rounded to float32, and the quotient is an fp32 division
    rounded to bf16 -- the arithmetic of torch's softmax for bf16 input
    (fp32 accumulate, bf16 output) up to the last-ulp summation order.
    """
    x = scale_logits(row_bits, temperature)
    m = x.max(axis=-1, keepdims=True)
    e = np.exp((x - m).astype(np.float64)).astype(np.float32)
    s = e.astype(np.float64).sum(axis=-1, keepdims=True).astype(np.float32)
    return round_bf16(e / s)


def row_stats(logits_bits: np.ndarray, temperature: float = 1.0):
    """Per-row argmax over the rounded probabilities, plus the probability
    rows themselves.  ``logits_bits``: uint16 [rows, V]."""
    p = row_probs(logits_bits, temperature)
    return np.argmax(p, axis=-1).astype(np.int64), p


# ------------------------------------------------------------- tree helpers
def children_lists(parents: Sequence[int]) -> List[List[int]]:
    """Children of every node in ascending index order, which is the order
    ``Tree.add_nodes`` appends them (``tree.py:108-119``)."""
    n = len(parents)
    ch: List[List[int]] = [[] for _ in range(n)]
    for i in range(n):
        p = int(parents[i])
        if p >= 0:
            ch[p].append(i)
    return ch


def depths_of(parents: Sequence[int]) -> np.ndarray:
    d = np.zeros(len(parents), dtype=np.int64)
    for i in range(len(parents)):
        p = int(parents[i])
        d[i] = 0 if p < 0 else d[p] + 1
    return d


# ------------------------------------------------------------------- greedy
def greedy_walk(parents, tokens, row_argmax, eos: Optional[int] = None, root: int = 0):
    """``verify_tree_exact`` (``verification.py:185-268``).

    Returns (sampled_tokens list, hidden_indices list, total_len, accept_len).
    """
    ch = children_lists(parents)
    sampled: List[int] = []
    hidden: List[int] = []
    total_len = 0
    accept_len = 0
    cur = int(root)
    bonus = None
    while len(ch[cur]) > 0:                                  # :232
        total_len += 1
        tok = int(row_argmax[cur])                           # :73
        match = [c for c in ch[cur] if int(tokens[c]) == tok]
        if match:                                            # :74, :237
            bonus = None
            accept_len += 1
            sampled.append(tok)
            hidden.append(cur)
            if eos is not None and tok == int(eos):          # :242
                break
            cur = match[0]                                   # :245
            if len(ch[cur]) == 0:                            # :249
                break
        else:
            bonus = tok
            break
    if not sampled or eos is None or sampled[-1] != int(eos):   # :257
        if bonus is None:
            bonus = int(row_argmax[cur])                     # :260-262
        sampled.append(bonus)
        hidden.append(cur)
    return sampled, hidden, total_len, accept_len


# ---------------------------------------------------------------- traversal
def _sum_f32(v: np.ndarray) -> np.float32:
    acc = np.float32(0.0)
    for x in v:
        acc = np.float32(acc + x)
    return acc


def _ratio(mb: np.ndarray, ms: np.ndarray) -> np.ndarray:
    out = np.zeros_like(mb)
    ok = ms > EPS32
    out[ok] = mb[ok] / ms[ok]
    return out


def traversal_walk(parents, tokens, draft_probs, mb_init, row_argmax, uniforms,
                   eos: Optional[int] = None, bonus_sampler=None):
    """``verify_tree_traversal`` (``verification.py:275-524``), skip_nodes=0.

    parents, tokens: per-node int arrays (root = node 0, parent -1).
    draft_probs: per-node draft probability (``cumulative_probability``),
        stored as float32 like ``t_cum_probs`` (``:320,332``).
    mb_init: per-node float32 target probability of the node's token under
        its parent's row (``:349``); entry 0 is ignored.
    row_argmax: per-row argmax of the rounded probabilities (bonus, ``:511``).
    uniforms: object with ``next()`` returning float32 (``torch.rand(1)``).
    bonus_sampler: optional callable(node) -> token for ``do_sample=True``.
    Returns (sampled_tokens, hidden_indices, total_len, accept_len, draws).
    """
    n = len(parents)
    ch = children_lists(parents)
    par = [int(p) for p in parents]
    dep = depths_of(par)

    Mb = np.zeros(n, dtype=np.float32)
    Mb[0] = 1.0
    Ms = np.zeros(n, dtype=np.float32)
    Ms[0] = 1.0
    for i in range(1, n):
        Mb[i] = np.float32(mb_init[i])                               # :349
        Ms[i] = np.float32(draft_probs[i])                           # :353
    pa = np.zeros(n, dtype=np.float32)
    pa[0] = 1.0
    maxd = int(dep.max()) if n else 0
    for d in range(1, maxd + 1):                                     # :359-371
        idx = np.nonzero(dep == d)[0]
        if idx.size == 0:
            continue
        pp = pa[[par[i] for i in idx]]
        r = _ratio(Mb[idx], Ms[idx])
        pa[idx] = np.minimum((pp * r).astype(np.float32), np.float32(1.0))

    valid = np.ones(n, dtype=bool)
    accepted = 0
    draws = 0
    while True:                                                      # :377
        curr = 0
        while True:
            fc = None
            for c in ch[curr]:
                if valid[c]:
                    fc = c
                    break
            if fc is None:
                break
            curr = fc
        cand = curr
        if not valid[cand]:
            break
        p_val = float(pa[cand])                                      # :395
        eta = float(uniforms.next())                                 # :396
        draws += 1
        if eta < p_val:
            accepted = cand
            break
        valid[cand] = False                                          # :403
        old_ms_rej = float(Ms[cand])
        Ms[cand] = 0.0
        parent = par[cand]
        if parent == -1:                                             # :408
            accepted = 0
            break
        sibs = ch[parent]
        if len(sibs) == 0:
            continue
        active = [c for c in sibs if valid[c]]
        if not active:                                               # :417
            continue
        p_old = float(pa[parent])                                    # :422
        p_old32 = np.float32(p_old)
        ms_denom = 1.0 - old_ms_rej
        if ms_denom < EPS:
            ms_denom = EPS
        mbs = Mb[sibs].copy()
        mss = Ms[sibs].copy()
        t = np.maximum((p_old32 * mbs).astype(np.float32) - mss, np.float32(0.0)).astype(np.float32)
        S_tree = float(_sum_f32(t))                                  # :432
        S_outside = p_old * (1.0 - float(_sum_f32(mbs)))            # :433
        S = S_tree + S_outside
        if S < EPS:
            S = EPS
        p_new = S / (S + 1.0 - p_old)                                # :439
        pa[parent] = np.float32(p_new)
        act = np.array(active, dtype=np.int64)
        sib_mbs = Mb[act].copy()
        sib_mss = Ms[act].copy()
        new_ms = (sib_mss / np.float32(ms_denom)).astype(np.float32)  # :445
        new_mb = (np.maximum((p_old32 * sib_mbs).astype(np.float32) - sib_mss, np.float32(0.0))
                  / np.float32(S)).astype(np.float32)                # :446
        Ms[act] = new_ms
        Mb[act] = new_mb
        old_mb_rej = float(Mb[cand])                                 # :451
        Mb[cand] = np.float32(max(p_old * old_mb_rej - old_ms_rej, 0.0) / S)
        r = _ratio(new_mb, new_ms)                                   # :455-458
        pa[act] = np.minimum((np.float32(p_new) * r).astype(np.float32), np.float32(1.0))
        queue = list(active)                                         # :461-477
        while queue:
            u = queue.pop(0)
            p_u = pa[u]
            vc = [c for c in ch[u] if valid[c]]
            if vc:
                vca = np.array(vc, dtype=np.int64)
                r = _ratio(Mb[vca], Ms[vca])
                pa[vca] = np.minimum((p_u * r).astype(np.float32), np.float32(1.0))
                queue.extend(vc)

    path = []                                                        # :480-485
    curr = accepted
    while curr != -1:
        path.append(curr)
        curr = par[curr]
    path.reverse()
    sampled: List[int] = []
    hidden: List[int] = []
    for i in range(1, len(path)):                                    # :490-497
        tok = int(tokens[path[i]])
        sampled.append(tok)
        hidden.append(path[i])
        if eos is not None and tok == int(eos):
            break
    if not (sampled and eos is not None and sampled[-1] == int(eos)):   # :500-515
        if bonus_sampler is not None:
            bonus = int(bonus_sampler(accepted))
        else:
            bonus = int(row_argmax[accepted])
        sampled.append(bonus)
        hidden.append(accepted)
    total_len = len(sampled)
    accept_len = max(0, total_len - 1)
    return sampled, hidden, total_len, accept_len, draws


def mb_from_probs(parents, tokens, probs: np.ndarray) -> np.ndarray:
    """Mb[i] = probs[parent(i), token(i)] (``verification.py:349``)."""
    n = len(parents)
    mb = np.zeros(n, dtype=np.float32)
    mb[0] = 1.0
    for i in range(1, n):
        mb[i] = probs[int(parents[i]), int(tokens[i])]
    return mb


def verify_batch(logits_bits: np.ndarray, row_indptr: Sequence[int], parents, tokens,
                 method: str = "exact", eos: Optional[int] = None, temperature: float = 1.0,
                 draft_probs=None, seed: int = 0, offset: int = 0):
    """Reference acceptance for a batch of trees laid out back to back.

    logits_bits: uint16 [rows, V]; row_indptr: [B+1]; parents: per-row local
    parent (-1 root); tokens: per-row token id.  Returns a list of dicts.
    """
    from .philox import UniformStream
    out = []
    B = len(row_indptr) - 1
    for b in range(B):
        lo, hi = int(row_indptr[b]), int(row_indptr[b + 1])
        par = np.asarray(parents[lo:hi], dtype=np.int64)
        tok = np.asarray(tokens[lo:hi], dtype=np.int64)
        t = temperature if method == "traversal" else 1.0
        am, p = row_stats(logits_bits[lo:hi], t)
        if method == "exact":
            s, h, tl, al = greedy_walk(par, tok, am, eos)
            out.append(dict(tokens=s, hidden=h, total_len=tl, accept_len=al, argmax=am))
        elif method == "traversal":
            mb = mb_from_probs(par, tok, p)
            us = UniformStream(seed, offset, b)
            s, h, tl, al, nd = traversal_walk(par, tok, np.asarray(draft_probs[lo:hi], np.float32),
                                              mb, am, us, eos)
            out.append(dict(tokens=s, hidden=h, total_len=tl, accept_len=al, argmax=am, mb=mb, draws=nd))
        else:
            raise ValueError(f"Unknown verification method: {method!r} (expected 'traversal' or 'exact')")
    return out


# ------------------------------------------- top-p target and sampled bonus
# Neither exists in the reference's acceptance (it takes softmax rows as they
# are and the bonus by argmax unless do_sample draws it with torch.multinomial,
# verification.py:508-511); these restate the rules the library states in
# include/pts_b200.h (pts_accept_traversal), so their parity is unpinned.
def _expf(d: np.ndarray) -> np.ndarray:
    return np.exp(np.asarray(d, dtype=np.float32).astype(np.float64)).astype(np.float32)


def nucleus(row_bits: np.ndarray, temperature: float, top_p: float, m: float, s: float):
    """(t*, s_N): the smallest logit value of the nucleus and its fp32 mass.
    Cumulative mass from the top over distinct values: count * expf(v - m)
    summed in float64, until it reaches top_p * s."""
    x = scale_logits(row_bits, temperature)
    vals, counts = np.unique(x, return_counts=True)
    target = float(np.float32(top_p)) * float(np.float32(s))
    cum = 0.0
    for v, c in zip(vals[::-1], counts[::-1]):
        cum += float(c) * float(_expf(np.float32(v) - np.float32(m)))
        if cum >= target:
            return np.float32(v), np.float32(cum)
    return np.float32(-np.inf), np.float32(cum)


def nucleus_probs(row_bits: np.ndarray, temperature: float, m: float, t: float, s_n: float) -> np.ndarray:
    """p'(x) = bf16(expf(x - m) / s_N) inside the nucleus (x >= t*), else 0."""
    x = scale_logits(row_bits, temperature)
    p = round_bf16((_expf(x - np.float32(m)) / np.float32(s_n)).astype(np.float32))
    return np.where(x >= t, p, np.float32(0.0)).astype(np.float32)


def sample_inverse_cdf(p: np.ndarray, u: float, segments: int = 1024) -> int:
    """First index whose running fp64 sum exceeds u * total; the sums run over
    ``segments`` consecutive segments (sequential inside each), then over the
    segment sums in order."""
    V = p.shape[0]
    per = (V + segments - 1) // segments
    p64 = p.astype(np.float64)
    local = np.zeros(segments, dtype=np.float64)
    for i in range(segments):
        seg = p64[min(i * per, V):min((i + 1) * per, V)]
        if seg.size:
            local[i] = np.cumsum(seg)[-1]
    excl = np.zeros(segments, dtype=np.float64)
    total = 0.0
    for i in range(segments):
        excl[i] = total
        total += local[i]
    target = float(np.float32(u)) * total
    for i in range(segments):
        if excl[i] <= target < excl[i] + local[i]:
            cum = excl[i]
            for e in range(min(i * per, V), min((i + 1) * per, V)):
                if p[e] > 0:
                    cum += float(p64[e])
                    if cum > target:
                        return e
    nz = np.nonzero(p > 0)[0]
    return int(nz[-1]) if nz.size else -1


# --------------------------------------------------------------- fp32 logits
def scale_logits_f32(x: np.ndarray, temperature: float) -> np.ndarray:
    """``logits / temperature`` for fp32 logits as the device computes it
    (multiply by the fp32 reciprocal; ``verification.py:310``)."""
    x = np.asarray(x, dtype=np.float32)
    if temperature == 1.0:
        return x
    return (x * (np.float32(1.0) / np.float32(temperature))).astype(np.float32)


def row_stats_f32(x: np.ndarray, temperature: float = 1.0):
    """fp32 softmax rows (``verification.py:46-55`` on fp32 logits): exp in
    float64 rounded to fp32, row sum in float64 rounded to fp32, p = e / s in
    fp32; argmax = first index of the largest p.  Returns (argmax, probs)."""
    x = scale_logits_f32(x, temperature)
    m = x.max(axis=-1, keepdims=True)
    e = np.exp((x - m).astype(np.float32).astype(np.float64)).astype(np.float32)
    s = e.astype(np.float64).sum(axis=-1, keepdims=True).astype(np.float32)
    p = (e / s).astype(np.float32)
    return np.argmax(p, axis=-1).astype(np.int64), p


# ------------------------------------------------------- vocabulary shards
# The library's tensor-parallel acceptance splits the vocabulary over ranks
# (include/pts_b200.h, pts_accept_shard_partials .. pts_accept_walk_merged).
# The reference has no sharded form, so these restate the exchange itself:
# per-shard partials, the merge in shard order, the exchange of tie indices.
# The merged statistics must reproduce row_stats and mb_from_probs of whole
# rows (verification.py:46-55, :349); tests check exactly that.
INT_MAX = 2 ** 31 - 1


def _exp_rounded(d: np.ndarray) -> np.ndarray:
    """fp32 exp of an fp32 difference, as row_probs evaluates it."""
    return np.exp(np.asarray(d, dtype=np.float32).astype(np.float64)).astype(np.float32)


def shard_partials(shard_bits: np.ndarray, vocab_offset: int, row_indptr, parents, tokens,
                   temperature: float = 1.0):
    """One shard's partials.  ``shard_bits``: uint16 [rows, Vs], vocabulary
    columns vocab_offset .. vocab_offset + Vs - 1 of every row.

    Returns (parts [rows, 3] float64: the shard's max m_k, the float64 sum of
    fp32 exp(x - m_k), the first global index of m_k; tok [rows] float32:
    node i's token logit in its parent's row if this shard holds the token,
    else -inf, and -inf for tree roots)."""
    x = scale_logits(shard_bits, temperature)
    R, Vs = x.shape
    m = x.max(axis=-1)
    s = _exp_rounded(x - m[:, None]).astype(np.float64).sum(axis=-1)
    first = np.argmax(x, axis=-1) + int(vocab_offset)
    parts = np.stack([m.astype(np.float64), s, first.astype(np.float64)], axis=-1)
    tok = np.full(R, -np.inf, dtype=np.float32)
    for b in range(len(row_indptr) - 1):
        lo, hi = int(row_indptr[b]), int(row_indptr[b + 1])
        for i in range(lo, hi):
            p, t = int(parents[i]), int(tokens[i]) - int(vocab_offset)
            if p >= 0 and 0 <= t < Vs:
                tok[i] = x[lo + p, t]
    return parts, tok


def _prev_bf16(v: np.ndarray) -> np.ndarray:
    """The largest bf16 value below each (bf16-exact, finite) value."""
    bits = f32_to_bf16_bits(v).astype(np.int64)
    out = np.where(v > 0, bits - 1, np.where(v < 0, bits + 1, 0x8001))
    return bf16_bits_to_f32(out.astype(np.uint16))


def merge_shards(parts_all: np.ndarray, tok_all: np.ndarray):
    """Merge partials gathered in shard order: parts_all [shards, rows, 3],
    tok_all [shards, rows].  Returns (m [rows] f32, s [rows] f32, smallest
    index of the max over the shards holding it [rows] int64, tie flag [rows]
    bool, token logit [rows] f32).

    s = sum_k s_k exp(m_k - m) in float64, rounded to fp32.  A row is flagged
    when the largest bf16 value below its max still rounds to the max's
    probability bf16(1 / s): only then can an index before the first max hold
    the largest rounded probability, and the shards settle it."""
    mk = parts_all[..., 0]
    m = mk.max(axis=0)
    s = (parts_all[..., 1] * np.exp(mk - m)).sum(axis=0).astype(np.float32)
    first = np.where(mk == m, parts_all[..., 2], np.inf).min(axis=0).astype(np.int64)
    m32 = m.astype(np.float32)
    qmax = round_bf16(np.float32(1.0) / s)
    flag = round_bf16(_exp_rounded(_prev_bf16(m32) - m32) / s) == qmax
    return m32, s, first, flag, tok_all.max(axis=0).astype(np.float32)


def shard_ties(shard_bits: np.ndarray, vocab_offset: int, m: np.ndarray, s: np.ndarray, flag: np.ndarray,
               temperature: float = 1.0) -> np.ndarray:
    """Per flagged row the first global index of this shard whose rounded
    probability equals the row's largest, bf16(1 / s); INT_MAX elsewhere."""
    x = scale_logits(shard_bits, temperature)
    p = round_bf16(_exp_rounded(x - m[:, None]) / s[:, None])
    hit = p == round_bf16(np.float32(1.0) / s)[:, None]
    got = np.where(hit.any(axis=-1), np.argmax(hit, axis=-1) + int(vocab_offset), INT_MAX)
    return np.where(flag, got, INT_MAX).astype(np.int64)


def merged_row_argmax(first: np.ndarray, flag: np.ndarray, ties_all: np.ndarray) -> np.ndarray:
    """The rows' argmax: the smallest tie index over all shards where flagged."""
    return np.where(flag, ties_all.min(axis=0), first).astype(np.int64)


def merged_mb(row_indptr, parents, m: np.ndarray, s: np.ndarray, tok: np.ndarray) -> np.ndarray:
    """Mb per node (mb_from_probs) from the merged statistics: the rounded
    probability bf16(exp(x - m) / s) of the node's token logit x in its
    parent's row; 1 for tree roots."""
    mb = np.ones(len(tok), dtype=np.float32)
    for b in range(len(row_indptr) - 1):
        lo, hi = int(row_indptr[b]), int(row_indptr[b + 1])
        for i in range(lo, hi):
            p = int(parents[i])
            if p >= 0:
                r = lo + p
                mb[i] = round_bf16(_exp_rounded(np.float32(tok[i]) - m[r]) / s[r])
    return mb
