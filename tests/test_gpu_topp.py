"""GPU parity of traversal acceptance with a top-p target distribution and
with a sampled bonus token, against the oracle's restatement of the rules
stated in include/pts_b200.h (no counterpart in the reference: parity
unpinned, restated exactly)."""
import numpy as np
import pytest
import torch

from oracle import accept as acc
from oracle.philox import UniformStream, traversal_uniforms
from parallel_tree_spec_b200 import kernels as K
from parallel_tree_spec_b200 import workload as wl

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
MAXN = 1024      # PTS_MAX_TREE_NODES: the bonus draw is uniform 2 * MAXN of the request's stream


def _row_ms(row_bits, T):
    x = acc.scale_logits(row_bits, T)
    m = np.float32(x.max())
    e = np.exp((x - m).astype(np.float64)).astype(np.float32)
    return m, np.float32(e.astype(np.float64).sum())


def _oracle(trees, logits, T, top_p, do_sample, seed, offset):
    out = []
    for b, (t, x) in enumerate(zip(trees, logits)):
        am, _ = acc.row_stats(x, T)
        probs = []
        for r in range(t.size):
            m, s = _row_ms(x[r], T)
            if top_p < 1.0:
                th, sn = acc.nucleus(x[r], T, top_p, m, s)
            else:
                th, sn = np.float32(-np.inf), s
            probs.append(acc.nucleus_probs(x[r], T, m, th, sn))
        mb = acc.mb_from_probs(t.parents, t.tokens, np.stack(probs))
        sampler = None
        if do_sample:
            u = traversal_uniforms(seed, offset, b, 2 * MAXN + 1)[2 * MAXN]
            sampler = lambda node: acc.sample_inverse_cdf(probs[node], u)
        s_, h, tl, al, _ = acc.traversal_walk(t.parents, t.tokens, t.draft_probs, mb, am,
                                             UniformStream(seed, offset, b), bonus_sampler=sampler)
        out.append((s_, list(h)))
    return out


@pytest.mark.parametrize("top_p,T,do_sample", [(0.9, 1.0, False), (0.5, 0.8, False), (1.0, 1.0, True),
                                               (0.9, 1.0, True)])
def test_topp_and_sampled_bonus_match_oracle(top_p, T, do_sample):
    V = 32000
    rng = np.random.default_rng(17)
    trees = [wl.make_tree(rng, 4, 5, V) for _ in range(5)] + [wl.make_tree(rng, 2, 3, V)]
    logits = [wl.make_logits(rng, t, V, sigma=2.0, plant=0.9, soft=True) for t in trees]
    indptr, par, tok, dp = wl.stack_trees(trees)
    x = torch.from_numpy(np.concatenate(logits).view(np.int16)).to(DEV).view(torch.bfloat16)
    d = lambda a: torch.from_numpy(a).to(DEV)
    ot, oh, oc = K.accept_traversal(x, d(indptr), d(par), d(tok), d(dp), temperature=T, top_p=top_p,
                                    do_sample=do_sample, seed=123, offset=4)
    ot, oh, oc = ot.cpu().numpy(), oh.cpu().numpy(), oc.cpu().numpy()
    ref = _oracle(trees, logits, T, top_p, do_sample, 123, 4)
    for b, (s_, h) in enumerate(ref):
        n = int(oc[b, 0])
        assert ot[b, :n].tolist() == s_ and oh[b, :n].tolist() == h, (b, ot[b, :n].tolist(), s_)


def test_topp_changes_acceptance_and_sampling_varies_with_the_stream():
    """A narrow nucleus removes mass from draft tokens outside it; sampled
    bonuses differ across Philox offsets while argmax bonuses do not."""
    V = 16000
    rng = np.random.default_rng(5)
    trees = [wl.make_tree(rng, 4, 4, V) for _ in range(8)]
    logits = [wl.make_logits(rng, t, V, sigma=1.0) for t in trees]
    indptr, par, tok, dp = wl.stack_trees(trees)
    x = torch.from_numpy(np.concatenate(logits).view(np.int16)).to(DEV).view(torch.bfloat16)
    d = lambda a: torch.from_numpy(a).to(DEV)
    bon = []
    for off in range(4):
        ot, oh, oc = K.accept_traversal(x, d(indptr), d(par), d(tok), d(dp), do_sample=True, seed=1, offset=off)
        bon.append([int(ot[b, int(oc[b, 0]) - 1]) for b in range(len(trees))])
    assert len({tuple(v) for v in bon}) > 1
