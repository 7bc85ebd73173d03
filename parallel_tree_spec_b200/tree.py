"""Draft tree (host side), interface of the reference's ``tree.py``.

Same classes, methods and return types as ``parallel_tree_spec.tree``
(``tree.py:17-230``): ``TreeNode``, ``Tree.add_nodes`` (level-by-level BFS
append, batch 1), ``get_tree_data``, ``create_attention_mask``,
``find_child_index``, ``get_children_indices`` ...  Nodes are stored as flat
columns (parent, token, probability, depth) instead of one Python object per
node, so the device path reads them as arrays without a per-node loop:
``as_arrays()`` returns the int32/float32 columns the kernels consume, and
``create_attention_mask`` builds the ancestor matrix with one vectorised pass
per depth.
"""
from __future__ import annotations

from typing import Dict, List, Optional

import numpy as np
import torch


class TreeNode:
    """One node (``tree.py:17-47``); a view onto the tree's columns."""

    __slots__ = ("parent", "children", "depth", "token_id", "cumulative_probability", "has_been_sampled")

    def __init__(self, parent: Optional[int], token_id: int, cumulative_probability: float, depth: int):
        self.parent = parent
        self.children: List[int] = []
        self.depth = depth
        self.token_id = token_id
        self.cumulative_probability = cumulative_probability
        self.has_been_sampled = False

    def __repr__(self):
        return (f"TreeNode(token_id={self.token_id}, prob={self.cumulative_probability:.4f}, "
                f"depth={self.depth}, parent={self.parent})")


class Tree:
    """Draft token tree with parent links (``tree.py:50-230``)."""

    def __init__(self, root_token_id, prob_dtype: torch.dtype = torch.float32):
        self.prob_dtype = prob_dtype
        tok = root_token_id.item() if isinstance(root_token_id, torch.Tensor) else root_token_id
        self._parent: List[int] = [-1]
        self._token: List[int] = [int(tok)]
        self._prob: List[float] = [1.0]
        self._depth: List[int] = [0]
        self._children: List[List[int]] = [[]]
        self._sampled: List[bool] = [False]
        self.available_leaves: List[int] = [0]
        self._arrays = None

    # ----------------------------------------------------------- construction
    @property
    def current_size(self) -> int:
        return len(self._parent)

    def _node(self, i: int) -> TreeNode:
        n = TreeNode(None if self._parent[i] < 0 else self._parent[i], self._token[i], self._prob[i], self._depth[i])
        n.children = list(self._children[i])
        n.has_been_sampled = self._sampled[i]
        return n

    @property
    def nodes(self) -> List[TreeNode]:
        """Snapshot of all nodes as ``TreeNode`` objects."""
        return [self._node(i) for i in range(self.current_size)]

    def add_nodes(self, token_ids: torch.Tensor, token_probs: torch.Tensor, local_parent_indices: torch.Tensor):
        """Append ``total_depth`` levels; level entries name their parent by its
        position in ``available_leaves`` (``tree.py:78-121``)."""
        batch_size, total_depth, num_samples = token_ids.shape
        assert batch_size == 1, "Currently only batch_size=1 is supported."
        pidx = local_parent_indices.to("cpu").tolist()
        toks = token_ids.to("cpu").tolist()
        probs = token_probs.to("cpu").tolist()
        for d in range(total_depth):
            for leaf in self.available_leaves:
                self._sampled[leaf] = True
            base = self.current_size
            new_leaves = []
            for i, (p, t, pr) in enumerate(zip(pidx[0][d], toks[0][d], probs[0][d])):
                parent = self.available_leaves[p]
                self._parent.append(parent)
                self._token.append(int(t))
                self._prob.append(float(pr))
                self._depth.append(self._depth[parent] + 1)
                self._children.append([])
                self._sampled.append(False)
                self._children[parent].append(base + i)
                new_leaves.append(base + i)
            self.available_leaves = new_leaves
        self._arrays = None

    @classmethod
    def from_arrays(cls, parents, tokens, probs=None, prob_dtype: torch.dtype = torch.float32) -> "Tree":
        """Build from flat BFS columns (``parent[i] < i``, root parent -1)."""
        parents = [int(p) for p in parents]
        tokens = [int(t) for t in tokens]
        t = cls(tokens[0], prob_dtype)
        probs = [1.0] * len(parents) if probs is None else [float(p) for p in probs]
        for i in range(1, len(parents)):
            p = parents[i]
            if not 0 <= p < i:
                raise ValueError(f"parent[{i}] = {p} is not an earlier node")
            t._parent.append(p)
            t._token.append(tokens[i])
            t._prob.append(probs[i])
            t._depth.append(t._depth[p] + 1)
            t._children.append([])
            t._sampled.append(False)
            t._children[p].append(i)
        maxd = max(t._depth)
        t.available_leaves = [i for i in range(len(parents)) if t._depth[i] == maxd]
        return t

    # ----------------------------------------------------------------- access
    def get_node(self, node_index: int) -> TreeNode:
        if node_index < 0 or node_index >= self.current_size:
            raise IndexError(f"Node index {node_index} out of bounds for tree size {self.current_size}.")
        return self._node(node_index)

    def get_children_indices(self, node_index) -> torch.Tensor:
        if isinstance(node_index, torch.Tensor):
            node_index = node_index.item()
        return torch.tensor(self._children[node_index], dtype=torch.long, device="cpu")

    def get_children_ids(self, node_index: int) -> torch.Tensor:
        return torch.tensor([self._token[c] for c in self._children[node_index]], dtype=torch.long, device="cpu")

    def find_child_index(self, node_index: int, match_token_id: int) -> int:
        for c in self._children[node_index]:
            if self._token[c] == match_token_id:
                return c
        return -1

    def get_tree_data(self, skip_nodes: int = 0) -> Dict[str, torch.Tensor]:
        s = slice(skip_nodes, None)
        return {
            "token_ids": torch.tensor(self._token[s], dtype=torch.long, device="cpu"),
            "cumulative_probabilities": torch.tensor(self._prob[s], dtype=self.prob_dtype, device="cpu"),
            "depths": torch.tensor(self._depth[s], dtype=torch.long, device="cpu"),
            "parent_indices": torch.tensor(self._parent[s], dtype=torch.long, device="cpu"),
        }

    def as_arrays(self):
        """(parents int32, tokens int32, draft_probs float32, depths int32) NumPy
        columns, cached until the tree changes."""
        if self._arrays is None:
            self._arrays = (np.asarray(self._parent, dtype=np.int32), np.asarray(self._token, dtype=np.int32),
                            np.asarray(self._prob, dtype=np.float32), np.asarray(self._depth, dtype=np.int32))
        return self._arrays

    def get_depth(self) -> int:
        return max(self._depth, default=0)

    def size(self) -> int:
        return self.current_size

    def create_attention_mask(self, prefix_length: int = 0, skip_nodes: int = 0, device: str = "cpu") -> torch.Tensor:
        """[1, 1, N, prefix_length + N] bool: all prefix columns, plus each
        node's ancestors and itself (``tree.py:167-194``)."""
        n = self.current_size
        if n == 0:
            return torch.empty((1, 1, 0, prefix_length), dtype=self.prob_dtype, device=device)
        par = np.asarray(self._parent, dtype=np.int64)
        dep = np.asarray(self._depth, dtype=np.int64)
        anc = np.zeros((n, n), dtype=bool)
        order = np.argsort(dep, kind="stable")
        for i in order:                                    # parents before children
            if par[i] >= 0:
                anc[i] = anc[par[i]]
            anc[i, i] = True
        m = torch.from_numpy(anc).to(device)
        if prefix_length > 0:
            m = torch.cat([torch.ones((n, prefix_length), dtype=torch.bool, device=device), m], dim=1)
        return m[skip_nodes:, :].unsqueeze(0).unsqueeze(0)

    def print(self, tokenizer=None, show_token_id: bool = True, show_probability: bool = True):
        def label(i):
            parts = []
            if show_token_id:
                parts.append(repr(tokenizer.decode([self._token[i]])) if tokenizer else str(self._token[i]))
            if show_probability:
                parts.append(f"({self._prob[i]:.4f})")
            return " ".join(parts)

        def rec(i, prefix):
            ch = self._children[i]
            for k, c in enumerate(ch):
                last = k == len(ch) - 1
                print(prefix + ("└── " if last else "├── ") + label(c))
                rec(c, prefix + ("    " if last else "│   "))

        print(label(0))
        rec(0, "")

    def __repr__(self):
        return f"Tree(num_nodes={self.current_size}, device='cpu')"
