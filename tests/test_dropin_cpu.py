"""Host-side parts of the drop-in modules, on CPU: the Tree mirror against the
reference's golden masks, page bookkeeping of KvCachePool / RequestKvCache,
and the reference's error behaviour (no GPU needed, no kernel is called)."""
import numpy as np
import pytest
import torch

from oracle import attention as att
from parallel_tree_spec_b200 import cache_manager as cm
from parallel_tree_spec_b200 import verification as ver
from parallel_tree_spec_b200 import workload as wl
from parallel_tree_spec_b200.tree import Tree, TreeNode, tree_columns


def test_tree_mask_matches_reference_golden(mask_golden):
    """Tree.create_attention_mask gives the reference's bits (tree.py:167-194)."""
    for rec in mask_golden:
        t = Tree.from_arrays(rec["parents"], list(range(len(rec["parents"]))))
        m = t.create_attention_mask(prefix_length=rec["prefix"])
        assert list(m.shape) == rec["shape"]
        flat = m.reshape(-1).numpy().astype(bool)
        bits = np.unpackbits(np.asarray(rec["packed"], np.uint8))[: flat.size].astype(bool)
        assert np.array_equal(flat, bits)


def test_tree_columns_depths_and_children():
    rng = np.random.default_rng(5)
    w = wl.make_tree(rng, 4, 5, 1000)
    t = Tree.from_arrays(w.parents, w.tokens, w.draft_probs)
    par, tok, prob, _ = tree_columns(t)
    assert np.array_equal(par, w.parents) and np.array_equal(tok, w.tokens)
    assert np.allclose(prob[1:], w.draft_probs[1:])
    data = t.get_tree_data()
    depth = np.zeros(len(w.parents), np.int64)
    for i in range(1, len(w.parents)):
        depth[i] = depth[w.parents[i]] + 1
    assert np.array_equal(np.asarray(data["depths"]).reshape(-1), depth)
    for i in range(t.current_size):
        kids = [c for c in range(len(w.parents)) if w.parents[c] == i]
        assert t.get_children_indices(i).tolist() == kids
        assert t.get_children_ids(i).tolist() == [int(w.tokens[c]) for c in kids]
    assert t.get_depth() == int(depth.max())
    assert np.array_equal(t.create_attention_mask(prefix_length=9)[0, 0].numpy(), att.tree_mask(w.parents, 9))


def test_tree_add_nodes_levels():
    """add_nodes appends levels whose entries name a parent by its position in
    the current leaves (tree.py:78-121)."""
    t = Tree(7)
    t.add_nodes(torch.tensor([[[11, 12]]]), torch.tensor([[[0.6, 0.3]]]), torch.tensor([[[0, 0]]]))
    t.add_nodes(torch.tensor([[[21, 22, 23]]]), torch.tensor([[[0.5, 0.2, 0.9]]]), torch.tensor([[[0, 1, 1]]]))
    par, tok, _, _ = tree_columns(t)
    assert par.tolist() == [-1, 0, 0, 1, 2, 2]
    assert tok.tolist() == [7, 11, 12, 21, 22, 23]
    assert t.available_leaves == [3, 4, 5]
    assert t.find_child_index(2, 23) == 5


def test_tree_grown_like_the_reference_producer():
    """The reference's beam search grows trees by hand: it appends to
    ``tree.nodes``, extends a parent's ``children`` and bumps
    ``tree.current_size`` (beam_search.py:441-447,570-579).  The columns,
    the mask and the node accessors follow those edits."""
    t = Tree(torch.tensor(5))
    for tok in (10, 11):
        i = t.current_size
        t.nodes[0].children.append(i)
        t.nodes.append(TreeNode(parent=0, token_id=tok, cumulative_probability=0.25, depth=1))
        t.current_size += 1
    t.available_leaves = [1, 2]
    t.add_nodes(torch.tensor([[[20, 21]]]), torch.tensor([[[0.5, 0.125]]]), torch.tensor([[[1, 1]]]))
    i = t.current_size
    t.nodes[3].children.append(i)
    t.nodes.append(TreeNode(parent=3, token_id=30, cumulative_probability=0.75, depth=3))
    t.current_size += 1
    par, tok, prob, dep = tree_columns(t)
    assert par.tolist() == [-1, 0, 0, 2, 2, 3]
    assert tok.tolist() == [5, 10, 11, 20, 21, 30]
    assert prob.tolist() == [1.0, 0.25, 0.25, 0.5, 0.125, 0.75]
    assert dep.tolist() == [0, 1, 1, 2, 2, 3]
    assert t.find_child_index(2, 21) == 4 and t.get_node(5).token_id == 30
    assert t.get_children_ids(2).tolist() == [20, 21]
    assert np.array_equal(t.create_attention_mask(prefix_length=3)[0, 0].numpy(), att.tree_mask(par, 3))


class _ForeignTree:
    """A tree of another class that offers only the reference's interface
    (``nodes``, ``current_size``, ``get_tree_data``), as the reference's own
    ``Tree`` does."""

    def __init__(self, parents, tokens):
        self.current_size = len(parents)
        self._p, self._t = list(parents), list(tokens)

    def get_tree_data(self, skip_nodes: int = 0):
        n = len(self._p)
        return {"token_ids": torch.tensor(self._t, dtype=torch.long),
                "cumulative_probabilities": torch.full((n,), 0.5, dtype=torch.float32),
                "depths": torch.tensor(wl.DraftTree(np.asarray(self._p), np.asarray(self._t),
                                                    np.ones(n, np.float32)).depths()),
                "parent_indices": torch.tensor(self._p, dtype=torch.long)}


def test_tree_columns_read_any_tree_through_get_tree_data():
    par, tok, prob, dep = tree_columns(_ForeignTree([-1, 0, 0, 1], [4, 5, 6, 7]))
    assert par.dtype == np.int32 and par.tolist() == [-1, 0, 0, 1]
    assert tok.tolist() == [4, 5, 6, 7] and prob.tolist() == [0.5] * 4 and dep.tolist() == [0, 1, 1, 2]


def test_tree_errors():
    t = Tree.from_arrays([-1, 0, 0], [1, 2, 3])
    with pytest.raises(IndexError):
        t.get_node(3)
    with pytest.raises(ValueError):
        Tree.from_arrays([-1, 2, 0], [1, 2, 3])


def test_pool_and_request_page_bookkeeping():
    pool = cm.KvCachePool(10, 1, 2, 8, 16, torch.bfloat16, "cpu")
    a = cm.RequestKvCache(pool, 16, 37)                       # 3 pages, 5 tokens on the last
    assert (a.kv_page_indices, a.kv_last_page_len, a.kv_len) == ([0, 1, 2], 5, 37)
    a.increment(30)                                           # 67 tokens: 5 pages, 3 on the last
    assert (len(a.kv_page_indices), a.kv_last_page_len, a.kv_len) == (5, 3, 67)
    b = cm.RequestKvCache(pool, 16, 16)
    assert b.kv_page_indices == [5] and b.kv_last_page_len == 16
    a.decrement(20)                                           # 47 tokens: 3 pages
    assert (len(a.kv_page_indices), a.kv_last_page_len) == (3, 15)
    assert pool.num_free_pages() == 10 - 3 - 1
    with pytest.raises(AssertionError):                       # cache_manager.py:92
        pool.allocate(100)
    a.release()
    b.release()
    assert pool.num_free_pages() == 10


def test_reference_error_types():
    """Unknown modes and methods raise ValueError; CPU logits are refused
    (this path has no CPU implementation)."""
    pool = cm.KvCachePool(4, 1, 2, 8, 16, torch.bfloat16, "cpu")
    r = cm.RequestKvCache(pool, 16, 5)
    with pytest.raises(ValueError):
        cm.getKvCacheBatchPosition([r], "sideways", "cpu")
    t = Tree.from_arrays([-1, 0], [1, 2])
    x = torch.zeros(2, 32, dtype=torch.bfloat16)
    with pytest.raises(ValueError):
        ver.verify_tree_exact(t, x)
    with pytest.raises(ValueError):
        ver.verify_tree_traversal(t, x)
    with pytest.raises(ValueError):
        ver.verify_tree_exact(t, x, root_ind=1)


def test_acceptance_timeout_and_malformed_counts_map_to_exceptions():
    """A walk that gave up waiting for its rows reports count -3 and a
    malformed tree -1; the host turns them into RuntimeError / ValueError."""
    ot = torch.zeros(2, 4, dtype=torch.int32)
    oh = torch.zeros(2, 4, dtype=torch.int32)
    oc = torch.tensor([[1, 1, 0, 0], [-3, 0, 0, 0]], dtype=torch.int32)
    with pytest.raises(RuntimeError):
        ver._results(ot, oh, oc, None)
    oc[1, 0] = -1
    with pytest.raises(ValueError):
        ver._results(ot, oh, oc, None)
