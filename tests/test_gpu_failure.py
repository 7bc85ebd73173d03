"""Failure handling on the GPU without a fault.

Every wait of the attention kernel on other warps or on its copies is bounded.
Here the limit is cut to 200 SM clocks, far below the time the first K/V copy
takes, so waits run out on purpose: the kernel must record an error, drain its
own tensor-core work and copies, free TMEM and return, the host must read the
error (pts_tree_attn_check), and the same context must then compute a correct
result once the default limit is back.
"""
import pytest
import torch

from parallel_tree_spec_b200 import kernels as K
from parallel_tree_spec_b200 import workload as wl
from tests.test_gpu_attention import MAX_ABS, MEAN_ABS, make_case, run_kernel, torch_reference

pytestmark = pytest.mark.gpu


def _case():
    import numpy as np
    rng = np.random.default_rng(12)
    trees = [wl.make_tree(rng, 8, 8, 1000) for _ in range(4)]
    return make_case(31, trees, [1000, 777, 64, 1500])


def test_attention_wait_runs_out_is_reported_and_the_context_recovers():
    c = _case()
    K.check_attention()                                      # nothing pending before the test
    prev = K.set_wait_limit(200)
    try:
        run_kernel(c)
        with pytest.raises(RuntimeError):
            K.check_attention()
    finally:
        K.set_wait_limit(prev)
    out = run_kernel(c)
    K.check_attention()                                      # no error with the default limit
    err = (out.float() - torch_reference(c)).abs()
    assert err.max().item() <= MAX_ABS and err.mean().item() <= MEAN_ABS


def test_normal_launch_leaves_no_error():
    c = _case()
    run_kernel(c)
    K.check_attention()
    assert K.set_wait_limit(0) == K.set_wait_limit(0)        # the default is reported back unchanged
