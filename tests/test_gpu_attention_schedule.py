"""GPU parity of the attention kernel's two schedules.

With a workspace of pts_tree_attn_workspace_size bytes and the balanced
schedule chosen, the kernel runs one CTA per SM over equal ranges of KV
blocks; the CTAs that share a unit cut by a range boundary write partial
results, which a second kernel merges in CTA order.  With a 256-byte workspace
it runs one CTA per (request, KV head, row group).  Both must match the fp32
reference within the attention tolerance and each other closely, and the
balanced schedule must give the same bits on every run.
"""
import math

import numpy as np
import pytest
import torch

from parallel_tree_spec_b200 import _lib
from parallel_tree_spec_b200 import kernels as K
from parallel_tree_spec_b200 import workload as wl
from tests.test_gpu_attention import DEV, check, make_case, torch_reference

pytestmark = pytest.mark.gpu


def _launch(c, ws):
    trees = c["trees"]
    indptr, par, _, _ = wl.stack_trees(trees)
    qo = torch.from_numpy(indptr).to(DEV)
    words = K.mask_words_for(max(t.size for t in trees))
    bits = K.tree_mask_from_parents(torch.from_numpy(par).to(DEV), qo, words)
    pind = torch.tensor(np.cumsum([0] + [len(t) for t in c["tables"]]), dtype=torch.int32, device=DEV)
    pidx = torch.tensor(sum(c["tables"], []), dtype=torch.int32, device=DEV)
    last = torch.tensor([(L - 1) % c["pl"] + 1 for L in c["kv_lens"]], dtype=torch.int32, device=DEV)
    q, layer = c["q"].to(DEV), c["layer"].to(DEV)
    out = torch.empty_like(q)
    T, Hq, D = q.shape
    P, _, pl, Hkv, _ = layer.shape
    _lib.call("pts_tree_attn_run", q.data_ptr(), layer.data_ptr(), qo.data_ptr(), pind.data_ptr(), pidx.data_ptr(),
              last.data_ptr(), bits.data_ptr(), bits.shape[1], out.data_ptr(), len(trees), T,
              max(t.size for t in trees), max(c["kv_lens"]), Hq, Hkv, D, pl, P, 1.0 / math.sqrt(D), ws.data_ptr(),
              ws.numel(), torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    return out


def _full_workspace():
    n = _lib.lib().pts_tree_attn_workspace_size(1, 1, 32, 128, 1)
    assert n > 256, "the balanced schedule needs the SM count of the device"
    return torch.zeros(n, dtype=torch.uint8, device=DEV)


def _cases():
    rng = np.random.default_rng(21)
    yield "ragged", make_case(21, [wl.make_tree(rng, 8, 8, 100) for _ in range(5)], [3000, 17, 900, 64, 2000])
    rng = np.random.default_rng(22)
    yield "one_request_long", make_case(22, [wl.make_tree(rng, 8, 8, 100)], [8000])
    rng = np.random.default_rng(23)
    yield "two_row_groups", make_case(23, [wl.make_tree(rng, 16, 8, 100), wl.make_tree(rng, 8, 8, 100)], [1500, 700])
    rng = np.random.default_rng(24)
    yield "gqa_16_2", make_case(24, [wl.make_tree(rng, 8, 8, 100) for _ in range(3)], [1200, 2500, 333], Hq=16,
                                Hkv=2)
    rng = np.random.default_rng(25)
    yield "many_short", make_case(25, [wl.make_tree(rng, 4, 3, 100) for _ in range(40)],
                                  [int(x) for x in rng.integers(0, 300, 40)])


@pytest.mark.parametrize("name,case", list(_cases()), ids=[n for n, _ in _cases()])
def test_balanced_and_unit_per_cta_agree(name, case):
    ref = torch_reference(case)
    small = torch.zeros(256, dtype=torch.uint8, device=DEV)
    a = _launch(case, small)                                 # one CTA per unit
    ws = _full_workspace()
    prev = K.set_attention_schedule(K.ATTN_SCHEDULE_BALANCED)
    try:
        b = _launch(case, ws)                                # balanced ranges, split units merged
        c2 = _launch(case, ws)
    finally:
        K.set_attention_schedule(prev)
    check(a, ref)
    check(b, ref)
    assert (a.float() - b.float()).abs().max().item() <= 1.6e-2
    assert torch.equal(b, c2)                               # same bits on a second run
    assert int(ws[:4].view(torch.int32).item()) == 0        # no wait gave up

