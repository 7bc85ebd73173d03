"""GPU: the verification step's C-ABI calls capture into a CUDA graph.

None of them syncs with the host or allocates, so a server can capture a whole
step (tree preparation with the KV append, tree attention, acceptance with
the KV compaction) once and replay it.  Kernel arguments are frozen at capture
time; the Philox offset among them, so a replay draws the same uniforms as the
captured call.  The test replays a captured step and checks every output and
the cache bytes against the same step run eagerly.
"""
import numpy as np
import pytest
import torch

from parallel_tree_spec_b200 import kernels as K
from parallel_tree_spec_b200 import workload as wl

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _inputs(seed=0):
    rng = np.random.default_rng(seed)
    B, Hq, Hkv, D, pl, V = 4, 8, 2, 128, 16, 4096
    trees = [wl.make_tree(rng, 4, 4, V) for _ in range(B)]
    indptr, par, tok, dp = wl.stack_trees(trees)
    T = int(indptr[-1])
    n = max(t.size for t in trees)
    prefix = rng.integers(40, 300, size=B)
    seq = prefix + np.array([t.size for t in trees])
    npages = (seq + pl - 1) // pl
    P = int(npages.sum()) + 4
    perm = rng.permutation(P)[:int(npages.sum())].astype(np.int32)
    g = torch.Generator().manual_seed(seed)
    d = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(DEV)
    x = dict(
        B=B, n=n, T=T, words=K.mask_words_for(n), kv_max=int(seq.max()),
        par=d(par), qo=d(indptr), tok=d(tok), dp=d(dp),
        seq=d(seq.astype(np.int32)), offs=d(prefix.astype(np.int32)),
        pind=d(np.concatenate([[0], np.cumsum(npages)]).astype(np.int32)), pidx=d(perm),
        last=d(((seq - 1) % pl + 1).astype(np.int32)),
        q=torch.randn(T, Hq, D, generator=g).to(torch.bfloat16).to(DEV),
        k=(torch.randn(T, Hkv, D, generator=g) / D ** 0.5).to(torch.bfloat16).to(DEV),
        v=(torch.randn(T, Hkv, D, generator=g) / D ** 0.5).to(torch.bfloat16).to(DEV),
        pool=(torch.randn(1, P, 2, pl, Hkv, D, generator=g) / D ** 0.5).to(torch.bfloat16).to(DEV),
    )
    logits = np.concatenate([wl.make_logits(rng, t, V, plant=1.0, soft=True) for t in trees], 0)
    x["logits"] = torch.from_numpy(logits.view(np.int16)).view(torch.bfloat16).to(DEV)
    return x


def _step(x, cargs):
    layer = x["pool"][0]
    bits, bi, pos = K.tree_prepare_append(x["par"], x["qo"], x["words"], x["seq"], x["k"], x["v"], layer,
                                          x["pind"], x["pidx"])
    out = K.tree_attention(x["q"], layer, x["qo"], x["pind"], x["pidx"], x["last"], bits, x["n"], x["kv_max"])
    ot, oh, oc = K.accept_traversal(x["logits"], x["qo"], x["par"], x["tok"], x["dp"], seed=5, offset=9,
                                    max_nodes=x["n"], compact=cargs)
    return bits, pos, out, ot, oh, oc


def test_verification_step_replays_from_a_cuda_graph():
    x = _inputs()
    new_len = torch.zeros(x["B"], dtype=torch.int32, device=DEV)
    cargs = K.kv_compact_args(x["pool"], x["pind"], x["pidx"], x["offs"], new_len)
    pool0 = x["pool"].clone()
    eager = [t.clone() for t in _step(x, cargs)]
    eager_pool, eager_len = x["pool"].clone(), new_len.clone()
    # warm up on a side stream, as torch's capture expects, then capture
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        _step(x, cargs)
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):                         # workspaces are per stream: the capture stream's
        outs = _step(x, cargs)                            # come from the graph's memory pool
    for _ in range(2):
        x["pool"].copy_(pool0)
        new_len.zero_()
        graph.replay()
        torch.cuda.synchronize()
        for name, a, b in zip(("bits", "positions", "attention", "counts"), outs[:3] + outs[5:], eager[:3] + eager[5:]):
            assert torch.equal(a, b), name
        # tokens and hidden indices: the first counts[b, 0] entries of each row are written, the rest is
        # whatever the buffer held
        for r in range(x["B"]):
            k = int(eager[5][r, 0])
            assert torch.equal(outs[3][r, :k], eager[3][r, :k]) and torch.equal(outs[4][r, :k], eager[4][r, :k])
        assert torch.equal(x["pool"].view(torch.int16), eager_pool.view(torch.int16))
        assert torch.equal(new_len, eager_len)
    assert int(eager[5][:, 2].sum()) > 0                   # some paths accepted, so compaction moved rows
