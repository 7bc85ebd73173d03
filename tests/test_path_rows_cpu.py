"""CPU: the rows whose statistics a verification walk reads, restated on the
oracle.  The greedy path chain (pts_accept_greedy_compact) reduces only the
rows of the root and of each accepted node, and the top-p nucleus pass skips
leaf rows when no bonus is sampled; both rely on the reference's walks never
reading any other row.  These tests replace every other row of the logits
with unrelated values and check that the walks' outputs do not change
(verification.py:185-268 for greedy, 275-524 for traversal)."""
import numpy as np
import pytest

from oracle import accept as acc
from oracle.philox import UniformStream
from parallel_tree_spec_b200 import workload as wl

V = 4096


def _case(seed, width, depth, plant):
    rng = np.random.default_rng(seed)
    t = wl.make_tree(rng, width, depth, V)
    x = wl.make_logits(rng, t, V, plant=plant, soft=True)
    return rng, t, x


def _scramble(rng, x, keep):
    """The rows outside ``keep`` replaced by fresh N(0, 3) logits (bf16 bits)."""
    y = x.copy()
    other = [r for r in range(x.shape[0]) if r not in keep]
    if other:
        y[other] = wl._bf16_bits((rng.standard_normal((len(other), x.shape[1])) * 3.0).astype(np.float32))
    return y


@pytest.mark.parametrize("seed,width,depth,plant,eos_first", [
    (1, 8, 8, 0.9, False), (2, 8, 8, 0.3, False), (3, 4, 4, 1.0, False), (4, 1, 12, 1.0, False),
    (5, 8, 8, 0.9, True), (6, 0, 0, 0.0, False), (7, 16, 3, 0.8, False)])
def test_greedy_walk_reads_only_its_path_rows(seed, width, depth, plant, eos_first):
    rng, t, x = _case(seed, width, depth, plant)
    am, _ = acc.row_stats(x, 1.0)
    eos = int(am[0]) if eos_first else None
    s, h, tl, al = acc.greedy_walk(t.parents, t.tokens, am, eos)
    # the rows read: each output's node (the root, then each accepted node)
    keep = set(int(v) for v in h) | {0}
    assert len(keep) <= al + 1
    for _ in range(3):
        am2, _ = acc.row_stats(_scramble(rng, x, keep), 1.0)
        assert acc.greedy_walk(t.parents, t.tokens, am2, eos) == (s, h, tl, al)


@pytest.mark.parametrize("seed,width,depth,plant,temperature", [
    (11, 8, 8, 1.0, 1.0), (12, 8, 8, 0.0, 1.0), (13, 4, 5, 1.0, 0.8), (14, 1, 10, 1.0, 1.0),
    (15, 16, 3, 1.0, 1.0)])
def test_traversal_walk_reads_internal_rows_and_the_bonus_row(seed, width, depth, plant, temperature):
    rng, t, x = _case(seed, width, depth, plant)
    am, p = acc.row_stats(x, temperature)
    mb = acc.mb_from_probs(t.parents, t.tokens, p)
    s, h, tl, al, _ = acc.traversal_walk(t.parents, t.tokens, t.draft_probs, mb, am,
                                         UniformStream(seed, 2, 0))
    internal = {0} | set(int(v) for v in t.parents[1:] if v >= 0)
    accepted = int(h[-1]) if h else 0
    keep = internal | {accepted}
    for _ in range(3):
        am2, p2 = acc.row_stats(_scramble(rng, x, keep), temperature)
        mb2 = acc.mb_from_probs(t.parents, t.tokens, p2)
        out = acc.traversal_walk(t.parents, t.tokens, t.draft_probs, mb2, am2, UniformStream(seed, 2, 0))
        assert out[:4] == (s, h, tl, al)


def test_scrambling_a_read_row_changes_the_walks():
    """Control: the checks above are not vacuous; scrambling the rows the walks
    do read changes their outputs."""
    changed_g = changed_t = 0
    for seed in range(20, 30):
        rng, t, x = _case(seed, 8, 8, 1.0)
        am, p = acc.row_stats(x, 1.0)
        g = acc.greedy_walk(t.parents, t.tokens, am, None)
        am2, _ = acc.row_stats(_scramble(rng, x, set()), 1.0)
        changed_g += acc.greedy_walk(t.parents, t.tokens, am2, None) != g
        mb = acc.mb_from_probs(t.parents, t.tokens, p)
        tr = acc.traversal_walk(t.parents, t.tokens, t.draft_probs, mb, am, UniformStream(seed, 2, 0))[:4]
        internal = set(int(v) for v in t.parents[1:] if v >= 0) - {0}
        am3, p3 = acc.row_stats(_scramble(rng, x, set(range(x.shape[0])) - internal), 1.0)
        mb3 = acc.mb_from_probs(t.parents, t.tokens, p3)
        tr3 = acc.traversal_walk(t.parents, t.tokens, t.draft_probs, mb3, am3, UniformStream(seed, 2, 0))[:4]
        changed_t += tr3 != tr
    assert changed_g >= 5 and changed_t >= 3
