"""Seeded synthetic workloads for the tree-verification step.

The reference measures on real checkpoints and prompts; here seeded synthetic
inputs with the benchmark's shapes stand in for them:

* draft trees shaped like beam-search output (``beam_search.py:437-604``):
  a root plus ``depth`` levels of ``width`` nodes, each node of level d
  picking its parent uniformly from level d-1, BFS numbering
  (``parent[i] < i``), token ids distinct among siblings;
* per-node draft probabilities: every parent owns a top-32 token set with
  Dirichlet(0.1) masses, its children take the highest-mass tokens of that
  set and carry their mass as ``cumulative_probability``;
* target logits ``N(0, sigma)`` rounded to bf16, optionally "planted" so that
  a row's argmax (or a large share of its mass) falls on a child token and
  accepted paths are long.

Everything is NumPy with ``numpy.random.default_rng`` so the same seed gives
the same inputs on every machine.  bf16 arrays are ``uint16`` bit patterns.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import List, Optional

import numpy as np


def _bf16_bits(x: np.ndarray) -> np.ndarray:
    x = np.asarray(x, dtype=np.float32)
    b = x.view(np.uint32).astype(np.uint64)
    return ((b + np.uint64(0x7FFF) + ((b >> np.uint64(16)) & np.uint64(1))) >> np.uint64(16)).astype(np.uint16)


def _bf16_f32(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << np.uint32(16)).view(np.float32)


@dataclass
class DraftTree:
    """Flat BFS representation of one draft tree (root = node 0)."""
    parents: np.ndarray            # int64 [N], -1 for the root
    tokens: np.ndarray             # int64 [N]
    draft_probs: np.ndarray        # float32 [N], root 1.0
    levels: List[np.ndarray] = field(default_factory=list)   # node ids per depth

    @property
    def size(self) -> int:
        return int(self.parents.shape[0])

    def depths(self) -> np.ndarray:
        d = np.zeros(self.size, dtype=np.int64)
        for i in range(1, self.size):
            d[i] = d[self.parents[i]] + 1
        return d


def make_tree(rng: np.random.Generator, width: int, depth: int, vocab: int,
              topk: int = 32, alpha: float = 0.1, full: bool = False,
              root_token: Optional[int] = None) -> DraftTree:
    """Beam-shaped tree: ``depth`` levels of ``width`` nodes (``full=True``
    gives a complete ``width``-ary tree instead)."""
    topk = min(topk, vocab)
    parents = [-1]
    tokens = [int(rng.integers(0, vocab)) if root_token is None else int(root_token)]
    probs = [1.0]
    levels = [np.array([0])]
    cand: dict = {}

    def candidates(p):
        if p not in cand:
            toks = rng.choice(vocab, size=topk, replace=False)
            mass = rng.dirichlet(np.full(topk, alpha))
            order = np.argsort(-mass, kind="stable")
            cand[p] = [toks[order].tolist(), mass[order].tolist(), 0]
        return cand[p]

    for d in range(1, depth + 1):
        prev = levels[-1]
        if full:
            par = np.repeat(prev, width)
        elif d == 1:
            par = np.zeros(width, dtype=np.int64)
        else:
            par = rng.choice(prev, size=width, replace=True)
        ids = []
        for p in par:
            p = int(p)
            c = candidates(p)
            j = c[2]
            c[2] += 1
            parents.append(p)
            tokens.append(int(c[0][j]))
            probs.append(float(c[1][j]))
            ids.append(len(parents) - 1)
        levels.append(np.array(ids))
    return DraftTree(np.asarray(parents, dtype=np.int64), np.asarray(tokens, dtype=np.int64),
                     np.asarray(probs, dtype=np.float32), levels)


def make_logits(rng: np.random.Generator, tree: DraftTree, vocab: int, sigma: float = 3.0,
                plant: float = 0.0, soft: bool = False) -> np.ndarray:
    """bf16 bits [N, V] drawn N(0, sigma).

    ``plant``: probability that a row with children gets one child token
    forced to be its unique argmax (row max + 2..4).  With ``soft`` the other
    children of that row also get logits near the row max, so traversal
    verification sees large target probabilities on draft tokens.
    """
    n = tree.size
    x = (rng.standard_normal((n, vocab), dtype=np.float32) * np.float32(sigma))
    bits = _bf16_bits(x)
    if plant > 0.0:
        vals = _bf16_f32(bits)
        ch = [[] for _ in range(n)]
        for i in range(1, n):
            ch[tree.parents[i]].append(i)
        for r in range(n):
            if not ch[r] or rng.random() >= plant:
                continue
            m = float(vals[r].max())
            c = ch[r][int(rng.integers(0, len(ch[r])))]
            if soft:
                for o in ch[r]:
                    if o != c:
                        vals[r, tree.tokens[o]] = m + float(rng.normal(0.0, 1.5)) - 1.0
            vals[r, tree.tokens[c]] = m + 2.0 + 2.0 * float(rng.random())
        bits = _bf16_bits(vals)
    return bits


def stack_trees(trees: List[DraftTree]):
    """Concatenate trees: (row_indptr int32 [B+1], parents int32, tokens int32,
    draft_probs float32), parents local to each tree."""
    indptr = np.zeros(len(trees) + 1, dtype=np.int32)
    for i, t in enumerate(trees):
        indptr[i + 1] = indptr[i] + t.size
    par = np.concatenate([t.parents for t in trees]).astype(np.int32)
    tok = np.concatenate([t.tokens for t in trees]).astype(np.int32)
    dp = np.concatenate([t.draft_probs for t in trees]).astype(np.float32)
    return indptr, par, tok, dp
