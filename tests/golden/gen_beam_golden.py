"""Golden vectors of the reference's draft beam search with copy-on-write
pages (``beam_search.py:315-616``), run on the CPU.

    python tests/golden/gen_beam_golden.py --ref <checkout>/src
    PTS_REFERENCE_SRC=<checkout>/src python tests/golden/gen_beam_golden.py

The draft model is ``tests/beam_fixture.FakeModel`` (logits and appended K/V
rows from seeded NumPy draws of each beam's token and position), the
attention wrapper a no-op, and the prompt's KV comes in through
``prefilled_logits`` with a pool of seeded random contents.  The fixture
(``beam.json``) stores, per case, the parameters and:

* every batch position the model was given (beam tokens, positions, page
  table, last-page lengths), i.e. the copy-on-write page management;
* the tree (parents, tokens, probabilities, depths);
* the pool's free pages afterwards and a SHA-1 digest of the pool's bytes.

A case whose selection has a tie in score among the first K + 1 candidates is
rejected (torch's top-k order for ties is not specified) and the seed moved.
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

from tests import beam_fixture as bf  # noqa: E402

CASES = [
    # prompt tokens, page length, beams K, depth, temperature, vocab, sigma, pages in the pool
    dict(prompt=13, page_len=4, K=4, depth=6, temperature=1.0, vocab=512, sigma=2.0, max_pages=64),
    dict(prompt=16, page_len=4, K=6, depth=7, temperature=1.0, vocab=700, sigma=3.0, max_pages=96),
    dict(prompt=10, page_len=8, K=3, depth=9, temperature=0.8, vocab=400, sigma=1.5, max_pages=64),
    dict(prompt=5, page_len=16, K=8, depth=5, temperature=1.0, vocab=1000, sigma=2.5, max_pages=64),
    dict(prompt=33, page_len=16, K=6, depth=10, temperature=1.0, vocab=640, sigma=4.0, max_pages=96),
    dict(prompt=7, page_len=4, K=2, depth=12, temperature=1.3, vocab=300, sigma=1.0, max_pages=64),
]
LAYERS, HEADS, DIM = 2, 2, 8


def pool_digest(pool: torch.Tensor) -> str:
    return hashlib.sha1(pool.contiguous().view(torch.int16).cpu().numpy().tobytes()).hexdigest()


def has_ties(model_records, case, prefill_bits) -> bool:
    """Ties among the first K + 1 scores of the initial selection or any step
    (recomputed with torch on the CPU exactly as the reference does)."""
    K, T = case["K"], case["temperature"]
    p0 = torch.softmax(bf.bits_to_bf16(prefill_bits)[0].float().to(torch.bfloat16) / T, dim=-1)
    v = torch.sort(p0.float(), descending=True).values[: K + 1]
    if len(set(v.tolist())) < len(v):
        return True
    return False


def run_case(bs, cm, case, seed):
    torch.Tensor.pin_memory = lambda self, *a, **k: self          # no accelerator here
    P, K = case["page_len"], case["K"]
    pool = cm.KvCachePool(case["max_pages"], LAYERS, HEADS, DIM, P, torch.bfloat16, torch.device("cpu"))
    pool.cache_data.copy_(bf.bits_to_bf16(bf.initial_pool_bits(seed, tuple(pool.cache_data.shape))))
    req = cm.RequestKvCache(pool, P, case["prompt"])
    prompt_tok = seed % case["vocab"]
    pre_bits = bf.step_logits_bits([prompt_tok], [case["prompt"] - 1], case["vocab"], case["sigma"])
    prefilled = bf.bits_to_bf16(pre_bits).unsqueeze(0)                # [1, 1, V]
    model = bf.FakeModel(case["vocab"], case["sigma"], P)
    input_ids = torch.tensor([[prompt_tok]], dtype=torch.long)
    cfg = bs.BeamSearchConfig(topk_len=K, max_depth=case["depth"], temperature=case["temperature"])
    tree, _, _ = bs.beam_search(model, req, input_ids, cfg, bf.FakeWrapper(), prefilled_logits=prefilled)
    parents, tokens, probs, depths = [], [], [], []
    for nd in tree.nodes:
        parents.append(-1 if nd.parent is None else int(nd.parent))
        tokens.append(int(nd.token_id))
        probs.append(float(nd.cumulative_probability))
        depths.append(int(nd.depth))
    free = pool.free_page_mask.nonzero().squeeze(1).tolist()
    return dict(case=case, seed=seed, prompt_token=prompt_tok, prompt_pages=list(req.kv_page_indices),
                steps=model.records, parents=parents, tokens=tokens, probs=probs, depths=depths,
                free_pages=free, pool_sha1=pool_digest(pool.cache_data)), pre_bits, model.records


def step_ties(rec, case, records) -> bool:
    """Recompute every decode step's flat scores as the reference does and
    look for ties among the first K + 1."""
    from oracle import beam as ob
    return ob.reference_has_ties(rec, case, records)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("PTS_REFERENCE_SRC"),
                    help="directory holding the reference's parallel_tree_spec package "
                         "(default: $PTS_REFERENCE_SRC)")
    args = ap.parse_args()
    if not args.ref:
        ap.error("give --ref or set PTS_REFERENCE_SRC")
    sys.path.insert(0, args.ref)
    from parallel_tree_spec import beam_search as bs
    from parallel_tree_spec.flashinfer import cache_manager as cm

    torch.set_num_threads(1)
    out = []
    for ci, case in enumerate(CASES):
        seed = 1000 + 17 * ci
        for _ in range(50):
            rec, pre_bits, records = run_case(bs, cm, case, seed)
            if not has_ties(records, case, pre_bits) and not step_ties(rec, case, records):
                break
            seed += 1
        else:
            raise RuntimeError(f"case {ci}: no tie-free seed")
        out.append(rec)
        print(f"case {ci}: seed {seed}, {len(rec['parents'])} nodes, {len(rec['steps'])} decode steps")
    with open(os.path.join(HERE, "beam.json"), "w") as f:
        json.dump(out, f)
    print(f"{len(out)} beam-search cases written")


if __name__ == "__main__":
    main()
