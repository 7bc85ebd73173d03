"""pts_accept_traversal_noalloc gives the same results as pts_accept_traversal.

Some callers of this library cannot allocate device memory for a workspace: a
host program that only receives device pointers from another runtime and has
no allocator of its own, or a server that plans its device memory once at
start-up and may not call cudaMalloc afterwards.  For them the library keeps
the acceptance kernel's scratch in a fixed device array and exposes
pts_accept_traversal_noalloc.  These tests call it through the C ABI, twice in
a row (the second call must not see the first call's counters), and compare
with the workspace entry point.  The file name makes pytest collect it last.
"""
import numpy as np
import pytest
import torch

from parallel_tree_spec_b200 import _lib
from parallel_tree_spec_b200 import kernels as K
from parallel_tree_spec_b200 import workload as wl

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _inputs(seed, n_trees, vocab):
    rng = np.random.default_rng(seed)
    trees = [wl.make_tree(rng, 8, 8, vocab) for _ in range(n_trees)]
    logits = np.concatenate([wl.make_logits(rng, t, vocab, plant=1.0, soft=True) for t in trees])
    indptr, par, tok, dp = wl.stack_trees(trees)
    x = torch.from_numpy(logits.view(np.int16)).to(DEV).view(torch.bfloat16)
    dev = lambda a: torch.from_numpy(a).to(DEV)
    return x, dev(indptr), dev(par), dev(tok), dev(dp), trees


@pytest.mark.parametrize("top_p,do_sample", [(1.0, 0), (0.9, 0), (1.0, 1), (0.9, 1)])
def test_noalloc_matches_workspace_entry_point_on_two_calls(top_p, do_sample):
    """Plain traversal, the top-p target and the sampled bonus: the last three
    run the statistics, nucleus, walk and bonus kernels on the shared array."""
    V = 128256
    x, ind, par, tok, dp, trees = _inputs(21, 6, V)
    B, R, N = len(trees), x.shape[0], max(t.size for t in trees)
    ref_t, ref_h, ref_c = K.accept_traversal(x, ind, par, tok, dp, temperature=0.9, top_p=top_p,
                                             do_sample=bool(do_sample), seed=77, offset=3, max_nodes=N)
    lib = _lib.lib()
    for _ in range(2):
        ot = torch.full((B, N), -5, dtype=torch.int32, device=DEV)
        oh = torch.full((B, N), -5, dtype=torch.int32, device=DEV)
        oc = torch.full((B, 4), -5, dtype=torch.int32, device=DEV)
        rc = lib.pts_accept_traversal_noalloc(x.data_ptr(), x.stride(0), ind.data_ptr(), par.data_ptr(),
                                              tok.data_ptr(), dp.data_ptr(), B, R, V, N, -1, 0.9, top_p, do_sample,
                                              77, 3,
                                              ot.data_ptr(), oh.data_ptr(), oc.data_ptr(), N,
                                              torch.cuda.current_stream().cuda_stream)
        assert rc == 0, lib.pts_last_error().decode()
        torch.cuda.synchronize()
        assert torch.equal(oc, ref_c)
        for b in range(B):
            n = int(ref_c[b, 0])
            assert torch.equal(ot[b, :n], ref_t[b, :n]) and torch.equal(oh[b, :n], ref_h[b, :n])


def test_noalloc_rejects_inputs_above_its_fixed_scratch():
    lib = _lib.lib()
    x = torch.zeros(8, dtype=torch.bfloat16, device=DEV)
    i32 = torch.zeros(8, dtype=torch.int32, device=DEV)
    f32 = torch.zeros(8, dtype=torch.float32, device=DEV)
    rc = lib.pts_accept_traversal_noalloc(x.data_ptr(), 262144, i32.data_ptr(), i32.data_ptr(), i32.data_ptr(),
                                          f32.data_ptr(), 1, 60000, 262144, 8, -1, 1.0, 1.0, 0, 0, 0,
                                          i32.data_ptr(), i32.data_ptr(), i32.data_ptr(), 8,
                                          torch.cuda.current_stream().cuda_stream)
    assert rc == _lib.PTS_ERR_CAPACITY
    assert "scratch" in lib.pts_last_error().decode()
