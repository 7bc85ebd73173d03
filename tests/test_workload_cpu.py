"""CPU: the seeded synthetic workload has the shape the benchmark states
(beam-shaped trees in BFS order, distinct sibling tokens, Dirichlet draft
masses, planted argmaxes) and is the same for the same seed."""
import numpy as np

from oracle import accept as acc
from parallel_tree_spec_b200 import workload as wl


def test_beam_shaped_trees():
    rng = np.random.default_rng(3)
    for _ in range(20):
        t = wl.make_tree(rng, 8, 8, 128256)
        assert t.size == 65 and t.parents[0] == -1 and t.draft_probs[0] == 1.0
        assert all(0 <= t.parents[i] < i for i in range(1, t.size))          # BFS numbering
        d = t.depths()
        assert [int((d == k).sum()) for k in range(9)] == [1] + [8] * 8        # 8 nodes per level
        assert all(d[i] == d[t.parents[i]] + 1 for i in range(1, t.size))
        for p in range(t.size):
            kids = np.nonzero(t.parents == p)[0]
            toks = t.tokens[kids]
            assert len(set(toks.tolist())) == len(toks)                       # distinct siblings
            mass = t.draft_probs[kids]
            assert np.all(mass > 0) and mass.sum() <= 1.0 + 1e-6
            assert np.all(np.diff(mass) <= 0)                                 # highest mass first
        assert np.all((t.tokens >= 0) & (t.tokens < 128256))


def test_planted_rows_put_the_argmax_on_a_child():
    rng = np.random.default_rng(4)
    t = wl.make_tree(rng, 4, 4, 4096)
    x = wl.make_logits(rng, t, 4096, plant=1.0)
    am, _ = acc.row_stats(x)
    for r in range(t.size):
        kids = np.nonzero(t.parents == r)[0]
        if kids.size:
            assert am[r] in set(t.tokens[kids].tolist()), r


def test_same_seed_same_inputs():
    a = [wl.make_tree(np.random.default_rng(9), 8, 8, 1000) for _ in range(2)]
    assert all(np.array_equal(getattr(a[0], f), getattr(a[1], f)) for f in ("parents", "tokens", "draft_probs"))
    x0 = wl.make_logits(np.random.default_rng(1), a[0], 1000, plant=0.7, soft=True)
    x1 = wl.make_logits(np.random.default_rng(1), a[1], 1000, plant=0.7, soft=True)
    assert x0.dtype == np.uint16 and np.array_equal(x0, x1)
    indptr, par, tok, dp = wl.stack_trees(a)
    assert indptr.tolist() == [0, 65, 130] and par.dtype == np.int32 and dp.dtype == np.float32
