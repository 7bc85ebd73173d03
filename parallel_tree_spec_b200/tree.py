"""Draft tree (host side), interface of the reference's ``tree.py``.

Same classes, attributes, methods and return types as
``parallel_tree_spec.tree`` (``tree.py:17-230``).  ``Tree.nodes`` is a live
list of ``TreeNode`` objects and ``Tree.current_size`` a plain attribute, so a
producer that grows the tree by hand works unchanged: the reference's beam
search appends nodes with ``tree.nodes[parent].children.append(i)``,
``tree.nodes.append(node)`` and ``tree.current_size += 1``
(``beam_search.py:444-447,574-579``), and ``add_nodes`` appends whole levels.

The device path reads a tree only through ``get_tree_data()``, the method
both this class and the reference's class provide (``tree_columns``), so the
verification functions accept a tree of either class.  The ancestor mask is
built with one vectorised row copy per node instead of a walk up the parent
chain of every node.
"""
from __future__ import annotations

from typing import Dict, List, Optional, Tuple

import numpy as np
import torch


class TreeNode:
    """One draft node (``tree.py:17-47``)."""

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

    __slots__ = ("prob_dtype", "nodes", "current_size", "available_leaves")

    def __init__(self, root_token_id, prob_dtype: torch.dtype = torch.float32):
        self.prob_dtype = prob_dtype
        tok = root_token_id.item() if isinstance(root_token_id, torch.Tensor) else root_token_id
        self.nodes: List[TreeNode] = [TreeNode(None, tok, 1.0, 0)]
        self.current_size = 1
        self.available_leaves: List[int] = [0]

    # ----------------------------------------------------------- construction
    def add_nodes(self, token_ids: torch.Tensor, token_probs: torch.Tensor, local_parent_indices: torch.Tensor):
        """Append ``total_depth`` levels [1, total_depth, samples]; entry i of a
        level names its parent by position in ``available_leaves``, and the
        level's nodes become the new leaves (``tree.py:78-121``)."""
        batch_size, total_depth, _ = token_ids.shape
        assert batch_size == 1, "Currently only batch_size=1 is supported."
        pidx = local_parent_indices.to("cpu").tolist()[0]
        toks = token_ids.to("cpu").tolist()[0]
        probs = token_probs.to("cpu").tolist()[0]
        for level in range(total_depth):
            for leaf in self.available_leaves:
                self.nodes[leaf].has_been_sampled = True
            first = self.current_size
            leaves = []
            for i, (p, t, pr) in enumerate(zip(pidx[level], toks[level], probs[level])):
                parent = self.available_leaves[p]
                self.nodes[parent].children.append(first + i)
                self.nodes.append(TreeNode(parent, t, pr, self.nodes[parent].depth + 1))
                leaves.append(first + i)
            self.current_size += len(leaves)
            self.available_leaves = leaves

    @classmethod
    def from_arrays(cls, parents, tokens, probs=None, prob_dtype: torch.dtype = torch.float32) -> "Tree":
        """Build from flat columns in BFS numbering (``parent[i] < i``, root
        parent -1); the deepest nodes become ``available_leaves``."""
        parents = [int(p) for p in parents]
        tokens = [int(t) for t in tokens]
        probs = [1.0] * len(parents) if probs is None else [float(p) for p in probs]
        t = cls(tokens[0], prob_dtype)
        for i in range(1, len(parents)):
            p = parents[i]
            if not 0 <= p < i:
                raise ValueError(f"parent[{i}] = {p} is not an earlier node")
            t.nodes[p].children.append(i)
            t.nodes.append(TreeNode(p, tokens[i], probs[i], t.nodes[p].depth + 1))
        t.current_size = len(parents)
        deepest = max(n.depth for n in t.nodes)
        t.available_leaves = [i for i, n in enumerate(t.nodes) if n.depth == deepest]
        return t

    # ----------------------------------------------------------------- access
    def get_node(self, node_index: int) -> TreeNode:
        if node_index < 0 or node_index >= self.current_size:
            raise IndexError(f"Node index {node_index} out of bounds for tree size {self.current_size}.")
        return self.nodes[node_index]

    def get_children_indices(self, node_index) -> torch.Tensor:
        if isinstance(node_index, torch.Tensor):
            node_index = node_index.item()
        return torch.tensor(self.nodes[node_index].children, dtype=torch.long, device="cpu")

    def get_children_ids(self, node_index: int) -> torch.Tensor:
        return torch.tensor([self.nodes[c].token_id for c in self.nodes[node_index].children], dtype=torch.long,
                            device="cpu")

    def find_child_index(self, node_index: int, match_token_id: int) -> int:
        """First child carrying ``match_token_id``, or -1."""
        for c in self.nodes[node_index].children:
            if self.nodes[c].token_id == match_token_id:
                return c
        return -1

    def get_tree_data(self, skip_nodes: int = 0) -> Dict[str, torch.Tensor]:
        """Flat columns of every node in ``nodes`` (``tree.py:145-159``)."""
        nodes = self.nodes[skip_nodes:]
        return {
            "token_ids": torch.tensor([n.token_id for n in nodes], dtype=torch.long, device="cpu"),
            "cumulative_probabilities": torch.tensor([n.cumulative_probability for n in nodes],
                                                     dtype=self.prob_dtype, device="cpu"),
            "depths": torch.tensor([n.depth for n in nodes], dtype=torch.long, device="cpu"),
            "parent_indices": torch.tensor([-1 if n.parent is None else n.parent for n in nodes], dtype=torch.long,
                                           device="cpu"),
        }

    def get_depth(self) -> int:
        return max((n.depth for n in self.nodes), default=0)

    def size(self) -> int:
        return self.current_size

    def create_attention_mask(self, prefix_length: int = 0, skip_nodes: int = 0, device: str = "cpu") -> torch.Tensor:
        """[1, 1, N, prefix_length + N] bool, N = ``current_size``: every prefix
        column, plus each node's ancestors and itself (``tree.py:167-194``)."""
        n = self.current_size
        if n == 0:
            return torch.empty((1, 1, 0, prefix_length), dtype=self.prob_dtype, device=device)
        par = [-1 if self.nodes[i].parent is None else self.nodes[i].parent for i in range(n)]
        anc = np.zeros((n, n), dtype=bool)
        if all(p < i for i, p in enumerate(par)):
            for i, p in enumerate(par):                      # a parent's row is complete before its children's
                if p >= 0:
                    anc[i] = anc[p]
                anc[i, i] = True
        else:
            for i in range(n):
                anc[i, i] = True
                p = par[i]
                while p >= 0:
                    anc[i, p] = True
                    p = par[p]
        m = torch.from_numpy(anc).to(device)
        if prefix_length > 0:
            m = torch.cat([torch.ones((n, prefix_length), dtype=torch.bool, device=device), m], dim=1)
        return m[skip_nodes:, :].unsqueeze(0).unsqueeze(0)

    def print(self, tokenizer=None, show_token_id: bool = True, show_probability: bool = True):
        def label(i):
            node = self.nodes[i]
            parts = []
            if show_token_id:
                parts.append(repr(tokenizer.decode([node.token_id])) if tokenizer else str(node.token_id))
            if show_probability:
                parts.append(f"({node.cumulative_probability:.4f})")
            return " ".join(parts)

        def rec(i, prefix):
            ch = self.nodes[i].children
            for k, c in enumerate(ch):
                last = k == len(ch) - 1
                print(prefix + ("└── " if last else "├── ") + label(c))
                rec(c, prefix + ("    " if last else "│   "))

        print(label(0))
        rec(0, "")

    def __repr__(self):
        return f"Tree(num_nodes={self.current_size}, device='cpu')"


def tree_columns(tree) -> Tuple[np.ndarray, np.ndarray, np.ndarray, np.ndarray]:
    """(parents int32, tokens int32, draft_probs float32, depths int32) of a
    tree, read through ``get_tree_data()`` (``tree.py:145-159``), so a tree of
    the reference's own ``Tree`` class works as well as this module's."""
    d = tree.get_tree_data()
    return (d["parent_indices"].numpy().astype(np.int32), d["token_ids"].numpy().astype(np.int32),
            d["cumulative_probabilities"].to(torch.float32).numpy(), d["depths"].numpy().astype(np.int32))
