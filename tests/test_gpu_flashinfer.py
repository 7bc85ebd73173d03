"""Tree attention against the reference's own attention kernel.

The reference runs tree attention through FlashInfer's
BatchPrefillWithPagedKVCacheWrapper with a custom boolean mask
(flashinfer/attention_wrapper.py:131-144,250-252).  FlashInfer is installed as a
library in this image (it builds its kernel on first use); the test runs it on
the benchmark shape and on a ragged batch, with the same queries, paged cache
and tree masks as this library's kernel, and compares the outputs with the
attention tolerance (2e-2 max-abs, 1e-3 mean-abs).  Skipped where FlashInfer
cannot be imported or built.
"""
import math

import numpy as np
import pytest
import torch

from oracle import attention as oatt
from parallel_tree_spec_b200 import kernels as K
from parallel_tree_spec_b200 import workload as wl
from tests.test_gpu_attention import MAX_ABS, MEAN_ABS, make_case, run_kernel

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _flashinfer():
    try:
        import flashinfer
        return flashinfer
    except Exception as e:                                    # not importable in this environment
        pytest.skip(f"flashinfer unavailable: {e}")


def _flashinfer_tree_attention(fi, c):
    trees = c["trees"]
    indptr, _, _, _ = wl.stack_trees(trees)
    i32 = lambda v: torch.as_tensor(np.asarray(v), dtype=torch.int32, device=DEV)
    qo = i32(indptr)
    pind = i32(np.cumsum([0] + [len(t) for t in c["tables"]]))
    pidx = i32(sum(c["tables"], []))
    last = i32([(L - 1) % c["pl"] + 1 for L in c["kv_lens"]])
    mask = torch.cat([torch.from_numpy(oatt.tree_mask(t.parents, p).reshape(-1))
                      for t, p in zip(trees, c["prefixes"])]).to(DEV)
    ws = torch.empty(256 << 20, dtype=torch.int8, device=DEV)
    w = fi.BatchPrefillWithPagedKVCacheWrapper(ws, kv_layout="NHD")
    try:
        w.plan(qo, pind, pidx, last, c["Hq"], c["Hkv"], c["D"], c["pl"], custom_mask=mask,
               q_data_type=torch.bfloat16, kv_data_type=torch.bfloat16,
               sm_scale=1.0 / math.sqrt(c["D"]))
    except Exception as e:                                    # its kernel could not be built here
        pytest.skip(f"flashinfer could not build its prefill kernel: {e}")
    return w.run(c["q"].to(DEV), c["layer"].to(DEV))


@pytest.mark.parametrize("shape", ["benchmark", "ragged"])
def test_tree_attention_matches_flashinfer_custom_mask(shape):
    fi = _flashinfer()
    rng = np.random.default_rng(17)
    if shape == "benchmark":
        trees = [wl.make_tree(rng, 8, 8, 1000) for _ in range(16)]
        c = make_case(5, trees, [4096] * 16)
    else:
        trees = [wl.make_tree(rng, 8, 8, 1000), wl.make_tree(rng, 3, 4, 1000), wl.make_tree(rng, 16, 8, 1000)]
        c = make_case(6, trees, [1000, 37, 2500])
    ours = run_kernel(c).float()
    ref = _flashinfer_tree_attention(fi, c).float()
    d = (ours - ref).abs()
    assert d.max().item() <= MAX_ABS and d.mean().item() <= MEAN_ABS, (d.max().item(), d.mean().item())
