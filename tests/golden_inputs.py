"""Regenerate the inputs of a golden case from its seeds (no reference needed)."""
import hashlib

import numpy as np

from parallel_tree_spec_b200 import workload as wl


def sha1(*arrays) -> str:
    h = hashlib.sha1()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def case_inputs(c):
    rng = np.random.default_rng(c["seed"])
    t = wl.make_tree(rng, c["width"], c["depth"], c["vocab"], full=c.get("full", False))
    x = wl.make_logits(rng, t, c["vocab"], sigma=c["sigma"], plant=c["plant"], soft=c.get("soft", False))
    if c.get("const_rows"):
        x[: c["const_rows"]] = wl._bf16_bits(np.zeros((1, c["vocab"]), np.float32))
    if c.get("dtype") == "f32":
        x = (wl._bf16_f32(x) + rng.standard_normal(x.shape).astype(np.float32) * np.float32(1e-3)).astype(np.float32)
        if c.get("const_rows"):
            x[: c["const_rows"]] = 0.0
    return t, x


def checked_inputs(rec):
    t, x = case_inputs(rec["case"])
    assert sha1(t.parents, t.tokens, t.draft_probs, x) == rec["sha1"], "input generator drifted"
    return t, x
