"""Draft beam-search oracle (test infrastructure): the selection arithmetic and
the copy-on-write page management of the reference's ``beam_search``
(``beam_search.py:315-616``), restated with NumPy.

* ``initial_select``   -- ``torch.softmax(logits / T).topk(K)`` and
  ``torch.log(topk_probs)`` of the prompt's last row (``:432-433, 461``).
* ``step_select``      -- ``cum[:, None] + torch.log(probs + 1e-10)``,
  flattened, ``topk(K)``, with each pick's ``probs[parent, tok]``
  (``:549-561``).  Probabilities are the bf16-rounded softmax of
  ``oracle.accept.row_probs``; ``probs + 1e-10`` and ``log`` round to bf16
  (torch's bf16 arithmetic); ``cum + log`` is an fp32 add.  Ties are broken
  by the smaller (flat) index.
* ``run_beam_search``  -- the decode loop's page bookkeeping (``:468-604``):
  pages are handed out lowest index first (``KvCachePool.allocate``,
  ``flashinfer/cache_manager.py:88-96``); copy-on-write of a shared partial
  page copies its first ``off`` slots of every layer; children share their
  parent's pages by reference count; released nodes give back pages whose
  count reaches zero; at the end every page outside the prompt goes back.

The model is a pair of callables (logits and appended K/V rows of a token at a
position), so the same deterministic stand-in drives the reference, this
restatement and the CUDA path.
"""
from __future__ import annotations

import hashlib
from typing import Callable, Dict, List

import numpy as np

from oracle.accept import bf16_bits_to_f32, f32_to_bf16_bits, round_bf16, row_probs


def _log_bf16(a: np.ndarray) -> np.ndarray:
    """torch.log of a bf16 tensor: fp32 log rounded to bf16."""
    return round_bf16(np.log(a.astype(np.float64)).astype(np.float32))


def _order(scores: np.ndarray) -> np.ndarray:
    """Indices by descending score, ties by ascending index."""
    return np.lexsort((np.arange(scores.size), -scores.astype(np.float64)))


def initial_select(prefill_bits: np.ndarray, K: int, temperature: float):
    """(token ids, bf16 probabilities as float32, cum log-probs as floats)."""
    p = row_probs(prefill_bits.reshape(1, -1), temperature)[0]
    ids = _order(p)[:K]
    return ids.astype(np.int64), p[ids], [float(v) for v in _log_bf16(p[ids])]


def step_scores(logits_bits: np.ndarray, cum: List[float], temperature: float):
    """(flat fp32 scores [K*V], bf16 probability rows [K, V] as float32)."""
    p = row_probs(logits_bits, temperature)
    lp = _log_bf16(round_bf16(p + np.float32(1e-10)))
    c = np.asarray(cum, dtype=np.float32)[:, None]
    return (c + lp).astype(np.float32).reshape(-1), p


def step_select(logits_bits: np.ndarray, cum: List[float], temperature: float, K: int):
    """(scores [K] fp32, parent rows [K], tokens [K], step probs [K])."""
    scores, p = step_scores(logits_bits, cum, temperature)
    V = logits_bits.shape[1]
    top = _order(scores)[:K]
    par, tok = top // V, top % V
    return scores[top], par.astype(np.int64), tok.astype(np.int64), p[par, tok]


def has_ties(scores: np.ndarray, K: int) -> bool:
    """Equal values among the K + 1 largest."""
    top = np.sort(scores.astype(np.float64))[::-1][: K + 1]
    return len(set(top.tolist())) < len(top)


class _Pool:
    """A paged pool [L, P, 2, page, H, D] of bf16 bits with the reference's
    allocation order."""

    def __init__(self, bits: np.ndarray):
        self.data = bits.copy()
        self.free = np.ones(bits.shape[1], bool)

    def allocate(self, n: int) -> List[int]:
        idx = np.nonzero(self.free)[0][:n]
        assert len(idx) == n, "out of cache pages"
        self.free[idx] = False
        return [int(i) for i in idx]

    def deallocate(self, pages):
        self.free[list(pages)] = True


def run_beam_search(pool_bits: np.ndarray, page_len: int, prompt_len: int, prompt_token: int,
                    prefill_bits: np.ndarray, K: int, depth: int, temperature: float,
                    logits_fn: Callable, kv_fn: Callable) -> Dict:
    """The reference's beam search on a stand-in model; returns the records
    ``tests/golden/gen_beam_golden.py`` writes."""
    pool = _Pool(pool_bits)
    n0 = -(-prompt_len // page_len) if prompt_len > 0 else 0
    prompt_pages = pool.allocate(n0)                              # RequestKvCache(pool, page, prompt)
    parents, tokens, probs, depths = [-1], [prompt_token], [1.0], [0]
    children: List[List[int]] = [[]]

    def add(parent, tok, prob):
        children[parent].append(len(parents))
        parents.append(parent)
        tokens.append(int(tok))
        probs.append(float(prob))
        depths.append(depths[parent] + 1)
        children.append([])
        return len(parents) - 1

    ids, p0, cum = initial_select(prefill_bits, K, temperature)
    node_pages: Dict[int, List[int]] = {}
    ref: Dict[int, int] = {}
    beam = []
    for i in range(K):                                            # :438-452
        nd = add(0, ids[i], p0[i])
        node_pages[nd] = list(prompt_pages)
        for pg in prompt_pages:
            ref[pg] = ref.get(pg, 0) + 1
        beam.append(nd)
    steps = []
    pos = prompt_len
    for _ in range(depth - 1):                                    # :465
        off, pli = pos % page_len, pos // page_len
        uniq = list(set(beam))                                    # the reference's order of a set of ints
        if off == 0:                                              # :471-475
            new = pool.allocate(len(uniq))
            for nd, pg in zip(uniq, new):
                node_pages[nd].append(pg)
                ref[pg] = 1
        else:                                                     # :476-485
            for nd in uniq:
                wp = node_pages[nd][pli]
                if ref[wp] > 1:
                    np_ = pool.allocate(1)[0]
                    pool.data[:, np_, :, :off] = pool.data[:, wp, :, :off]
                    ref[wp] -= 1
                    if ref[wp] == 0:
                        pool.deallocate([wp])
                        del ref[wp]
                    node_pages[nd][pli] = np_
                    ref[np_] = 1
        pages_list = [node_pages[beam[k]] for k in range(K)]
        indptr = [0]
        flat = []
        for pgs in pages_list:
            flat.extend(pgs)
            indptr.append(len(flat))
        btoks = [tokens[beam[k]] for k in range(K)]
        steps.append(dict(tokens=btoks, positions=[pos] * K, indptr=indptr, indices=flat,
                          last_page_len=[pos % page_len + 1] * K))
        rows = logits_fn(btoks, [pos] * K)                        # the model's decode step
        for k in range(K):                                        # its KV append
            pg = pages_list[k][pos // page_len]
            pool.data[:, pg, :, pos % page_len] = kv_fn(btoks[k], pos)
        sc, par, tok, sp = step_select(rows, cum, temperature, K)
        seen: Dict[tuple, int] = {}
        new_beam = []
        for i in range(K):                                        # :563-591
            pn = beam[int(par[i])]
            key = (pn, int(tok[i]))
            if key in seen:
                nn = seen[key]
            else:
                ex = next((c for c in children[pn] if tokens[c] == int(tok[i])), -1)
                if ex != -1 and ex in node_pages:
                    nn = ex
                else:
                    nn = add(pn, tok[i], sp[i])
                    node_pages[nn] = list(node_pages[pn])
                    for pg in node_pages[nn]:
                        ref[pg] += 1
                seen[key] = nn
            new_beam.append(nn)
        for old in set(beam):                                     # :593-603
            free = []
            for pg in node_pages[old]:
                ref[pg] -= 1
                if ref[pg] == 0:
                    free.append(pg)
                    del ref[pg]
            for pg in free:
                pool.deallocate([pg])
            del node_pages[old]
        beam = new_beam
        cum = [float(v) for v in sc]
        pos += 1
    keep = set(prompt_pages)                                      # :607-614
    release = set()
    for pgs in node_pages.values():
        for pg in pgs:
            if pg not in keep:
                release.add(pg)
    for pg in release:
        pool.deallocate([pg])
    digest = hashlib.sha1(np.ascontiguousarray(pool.data).view(np.int16).tobytes()).hexdigest()
    return dict(prompt_pages=prompt_pages, steps=steps, parents=parents, tokens=tokens, probs=probs, depths=depths,
                free_pages=[int(i) for i in np.nonzero(pool.free)[0]], pool_sha1=digest)


def reference_has_ties(rec: Dict, case: Dict, records: List[Dict]) -> bool:
    """Ties among the K + 1 best flat scores of any decode step of a recorded
    run (the logits recomputed from the recorded tokens and positions)."""
    from tests import beam_fixture as bf
    K, T = case["K"], case["temperature"]
    pre = bf.step_logits_bits([rec["prompt_token"]], [case["prompt"] - 1], case["vocab"], case["sigma"])
    _, _, cum = initial_select(pre, K, T)
    for r in records:
        rows = bf.step_logits_bits(r["tokens"], r["positions"], case["vocab"], case["sigma"])
        scores, _ = step_scores(rows, cum, T)
        if has_ties(scores, K):
            return True
        cum = [float(v) for v in scores[_order(scores)[:K]]]
    return False
