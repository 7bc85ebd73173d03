"""Generate golden vectors by running the reference's own functions.

Run in a container that has the reference checked out (it is not needed
afterwards; the committed fixtures travel instead):

    python tests/golden/gen_golden.py --ref <checkout>/src
    PTS_REFERENCE_SRC=<checkout>/src python tests/golden/gen_golden.py

where ``<checkout>/src`` is the directory holding the reference's
``parallel_tree_spec`` package.

For every case the inputs are regenerated from seeds by
``parallel_tree_spec_b200.workload`` (NumPy, machine independent); the
fixture stores the seeds, SHA-1 digests of the generated inputs and the
reference's outputs:

* ``verify_tree_exact``     (``verification.py:185-268``)
* ``verify_tree_traversal`` (``verification.py:275-524``) with ``torch.rand``
  replaced by the Philox uniform stream of ``oracle.philox``
* the per-row argmax and per-node target probability that the reference's
  ``_sample_probs`` produces (``verification.py:46-55,349``)
* ``RequestKvCache.reorder_cache_with_offset`` / ``KvCachePool.reorder_cache_with_offset``
  (``cache_manager.py:103-140,196-213``) on small CPU pools
* ``Tree.create_attention_mask`` (``tree.py:167-194``)
* the same acceptance functions on fp32 logits (``accept_f32.json``; the
  logits are the bf16 generator's values plus a seeded fp32 perturbation)

``--f32-only`` writes ``accept_f32.json`` alone.
"""
from __future__ import annotations

import argparse
import hashlib
import json
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from parallel_tree_spec_b200 import workload as wl  # noqa: E402
from oracle.philox import traversal_uniforms  # noqa: E402


def sha1(*arrays) -> str:
    h = hashlib.sha1()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def bits_to_torch_bf16(bits: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(bits.astype(np.uint16).view(np.int16).copy()).view(torch.bfloat16)


def ref_tree(Tree, t: wl.DraftTree):
    tree = Tree(int(t.tokens[0]))
    for d in range(1, len(t.levels)):
        ids = t.levels[d]
        prev = list(t.levels[d - 1])
        local = [prev.index(int(t.parents[i])) for i in ids]
        tree.add_nodes(torch.tensor([[list(t.tokens[ids])]], dtype=torch.long),
                       torch.tensor([[list(t.draft_probs[ids].astype(np.float64))]], dtype=torch.float64),
                       torch.tensor([[local]], dtype=torch.long))
    return tree


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


def run_accept_case(mods, c):
    Tree, verification = mods
    t, x = case_inputs(c)
    tree = ref_tree(Tree, t)
    logits = (torch.from_numpy(x.copy()) if c.get("dtype") == "f32" else bits_to_torch_bf16(x)).unsqueeze(0)
    eos = c.get("eos")
    if eos == "planted":
        # an accepted-path token when the tree is planted: the root's first child
        eos = int(t.tokens[1]) if t.size > 1 else None
    c["eos_value"] = eos
    T = c.get("temperature", 1.0)
    scaled = logits / T if (c["method"] == "traversal" and T != 1.0) else logits
    probs = verification._sample_probs(scaled).squeeze(0)
    argmax = probs.argmax(dim=-1).tolist()
    mb = [1.0] + [float(probs[int(t.parents[i]), int(t.tokens[i])]) for i in range(1, t.size)]
    rec = dict(case=c, sha1=sha1(t.parents, t.tokens, t.draft_probs, x), ref_argmax=argmax)
    if c["method"] == "exact":
        s, h, tl, al = verification.verify_tree_exact(tree, logits, eos_token_id=eos)
    else:
        us = traversal_uniforms(c["philox_seed"], c.get("philox_offset", 0), c.get("request", 0), 4 * t.size + 8)
        calls = [0]
        orig = torch.rand

        def fake_rand(*a, **k):
            u = float(us[calls[0]])
            calls[0] += 1
            return torch.tensor([u], dtype=torch.float32)

        torch.rand = fake_rand
        try:
            s, h, tl, al = verification.verify_tree_traversal(tree, logits, eos_token_id=eos, temperature=T)
        finally:
            torch.rand = orig
        rec["draws"] = calls[0]
        rec["ref_mb_f32"] = mb
    rec.update(tokens=[int(v) for v in s.reshape(-1).tolist()], hidden=[int(v) for v in h.tolist()],
               total_len=int(tl), accept_len=int(al))
    return rec


def accept_cases():
    cases = []
    seed = 100
    shapes = [
        dict(width=4, depth=4, vocab=1024),
        dict(width=8, depth=8, vocab=1024),
        dict(width=2, depth=3, vocab=1024, full=True),
        dict(width=1, depth=6, vocab=1024),
        dict(width=0, depth=0, vocab=1024),
        dict(width=16, depth=8, vocab=2048),
        dict(width=3, depth=2, vocab=4096, full=True),
    ]
    for method in ("exact", "traversal"):
        for sh in shapes:
            for plant, soft in ((0.0, False), (0.7, False), (1.0, True)):
                for eos in (None, "planted"):
                    for T in ((1.0,) if method == "exact" else (1.0, 0.8)):
                        c = dict(sh, method=method, seed=seed, sigma=3.0, plant=plant, soft=soft,
                                 eos=eos, temperature=T, philox_seed=5 + seed, philox_offset=seed % 3,
                                 request=seed % 4)
                        cases.append(c)
                        seed += 1
    # full-vocabulary rows, the benchmark's tree shape
    for method in ("exact", "traversal"):
        for plant, soft in ((0.7, False), (1.0, True)):
            cases.append(dict(width=8, depth=8, vocab=128256, method=method, seed=seed, sigma=3.0,
                              plant=plant, soft=soft, eos=None, temperature=1.0, philox_seed=5,
                              philox_offset=0, request=seed % 16))
            seed += 1
    # near-ties between distinct logits after bf16 rounding of the probabilities
    for method in ("exact", "traversal"):
        for sigma in (0.02, 0.3):
            cases.append(dict(width=4, depth=3, vocab=4096, method=method, seed=seed, sigma=sigma,
                              plant=0.0, soft=False, eos=None, temperature=1.0, philox_seed=7,
                              philox_offset=1, request=1))
            seed += 1
    # constant rows: every probability equal, argmax is index 0
    for method in ("exact", "traversal"):
        cases.append(dict(width=4, depth=3, vocab=1024, method=method, seed=seed, sigma=3.0, plant=0.0,
                          soft=False, eos=None, temperature=1.0, philox_seed=9, philox_offset=0,
                          request=0, const_rows=5))
        seed += 1
    return cases


def accept_f32_cases():
    cases = []
    seed = 5000
    shapes = [
        dict(width=2, depth=4, vocab=1024, full=True),     # the 15-node binary tree of the small fp32 model
        dict(width=4, depth=4, vocab=1024),
        dict(width=8, depth=8, vocab=1024),
        dict(width=1, depth=6, vocab=4096),
    ]
    for method in ("exact", "traversal"):
        for sh in shapes:
            for plant, soft in ((0.0, False), (1.0, True)):
                for T in ((1.0,) if method == "exact" else (1.0, 0.8)):
                    cases.append(dict(sh, method=method, seed=seed, sigma=3.0, plant=plant, soft=soft, eos=None,
                                      temperature=T, philox_seed=11 + seed, philox_offset=seed % 3,
                                      request=seed % 4, dtype="f32"))
                    seed += 1
    cases.append(dict(width=4, depth=3, vocab=1024, method="exact", seed=seed, sigma=3.0, plant=0.0, soft=False,
                      eos=None, temperature=1.0, philox_seed=3, philox_offset=0, request=0, const_rows=3,
                      dtype="f32"))
    return cases


def reorder_cases(cache_manager):
    out = []
    rng = np.random.default_rng(7)
    for (L, H, D, pl, max_pages, prompt, n_tree, dtype) in [
        (2, 2, 8, 16, 12, 37, 15, torch.bfloat16),
        (1, 4, 16, 16, 16, 64, 65, torch.bfloat16),
        (3, 1, 4, 16, 8, 7, 9, torch.float32),
        (2, 2, 8, 8, 12, 16, 5, torch.bfloat16),
    ]:
        for trial in range(3):
            pool = cache_manager.KvCachePool(max_pages, L, H, D, pl, dtype, torch.device("cpu"))
            vals = rng.standard_normal(pool.cache_data.shape).astype(np.float32)
            pool.cache_data.copy_(torch.from_numpy(vals).to(dtype))
            before = pool.cache_data.clone()
            req = cache_manager.RequestKvCache(pool, pl, prompt)
            req.increment(n_tree)
            # an accepted path: root plus increasing tree indices, sometimes with the
            # last index repeated (the traversal form of hidden_indices)
            k = int(rng.integers(1, min(n_tree, 6) + 1))
            path = [0] + sorted(rng.choice(np.arange(1, n_tree), size=k - 1, replace=False).tolist()) if n_tree > 1 else [0]
            if trial == 2:
                path = path[1:] + [path[-1]] if len(path) > 1 else path
            offset = prompt + 1
            pages_before = list(req.kv_page_indices)
            req.reorder_cache_with_offset(torch.tensor(path, dtype=torch.long), offset=offset)
            bits_dtype = np.uint16 if dtype == torch.bfloat16 else np.uint32
            view_dtype = torch.int16 if dtype == torch.bfloat16 else torch.int32
            out.append(dict(
                shape=[L, max_pages, 2, pl, H, D], dtype=str(dtype).replace("torch.", ""), prompt=prompt,
                n_tree=n_tree, path=path, offset=offset, pages_before=pages_before,
                kv_len=req.kv_len, last_page_len=req.kv_last_page_len, pages_after=list(req.kv_page_indices),
                free_mask=[bool(v) for v in pool.free_page_mask.tolist()],
                sha1_before=sha1(before.view(view_dtype).numpy().view(bits_dtype)),
                sha1_after=sha1(pool.cache_data.view(view_dtype).numpy().view(bits_dtype)),
                seed_state=None))
            np.save(os.path.join(HERE, f"reorder_{len(out) - 1}_before.npy"),
                    before.view(view_dtype).numpy().view(bits_dtype))
    return out


def mask_cases(Tree):
    out = []
    for seed, (w, d, full, prefix) in enumerate([(2, 3, True, 5), (8, 8, False, 0), (4, 4, False, 17),
                                                 (1, 5, False, 3), (0, 0, False, 4)]):
        rng = np.random.default_rng(1000 + seed)
        t = wl.make_tree(rng, w, d, 512, full=full)
        tree = ref_tree(Tree, t)
        m = tree.create_attention_mask(prefix_length=prefix)
        out.append(dict(seed=1000 + seed, width=w, depth=d, full=full, prefix=prefix,
                        shape=list(m.shape), packed=np.packbits(m.numpy().reshape(-1)).tolist(),
                        parents=t.parents.tolist()))
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("PTS_REFERENCE_SRC"),
                    help="directory holding the reference's parallel_tree_spec package "
                         "(default: $PTS_REFERENCE_SRC)")
    ap.add_argument("--f32-only", action="store_true")
    args = ap.parse_args()
    if not args.ref:
        ap.error("give --ref or set PTS_REFERENCE_SRC")
    sys.path.insert(0, args.ref)
    from parallel_tree_spec.tree import Tree
    from parallel_tree_spec import verification
    from parallel_tree_spec.flashinfer import cache_manager

    torch.set_num_threads(max(1, os.cpu_count() or 1))
    acc32 = [run_accept_case((Tree, verification), c) for c in accept_f32_cases()]
    with open(os.path.join(HERE, "accept_f32.json"), "w") as f:
        json.dump(acc32, f)
    print(f"{len(acc32)} fp32 acceptance cases written")
    if args.f32_only:
        return
    acc = [run_accept_case((Tree, verification), c) for c in accept_cases()]
    with open(os.path.join(HERE, "accept.json"), "w") as f:
        json.dump(acc, f)
    with open(os.path.join(HERE, "reorder.json"), "w") as f:
        json.dump(reorder_cases(cache_manager), f)
    with open(os.path.join(HERE, "mask.json"), "w") as f:
        json.dump(mask_cases(Tree), f)
    print(f"{len(acc)} acceptance cases written")


if __name__ == "__main__":
    main()
