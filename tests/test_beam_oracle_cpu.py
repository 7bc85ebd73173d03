"""CPU: the beam-search oracle (``oracle/beam.py``) against the golden vectors
of the reference's own ``beam_search`` (``tests/golden/beam.json``, written by
``tests/golden/gen_beam_golden.py``): every decode step's page table, the
tree, the free pages and the pool's bytes after the copy-on-write copies."""
import json
import os

import numpy as np
import pytest

from oracle import beam as ob
from tests import beam_fixture as bf

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "beam.json")
LAYERS, HEADS, DIM = 2, 2, 8


def cases():
    with open(GOLDEN) as f:
        return json.load(f)


def oracle_run(rec):
    c = rec["case"]
    shape = (LAYERS, c["max_pages"], 2, c["page_len"], HEADS, DIM)
    pre = bf.step_logits_bits([rec["prompt_token"]], [c["prompt"] - 1], c["vocab"], c["sigma"])
    return ob.run_beam_search(
        bf.initial_pool_bits(rec["seed"], shape), c["page_len"], c["prompt"], rec["prompt_token"], pre, c["K"],
        c["depth"], c["temperature"],
        lambda toks, pos: bf.step_logits_bits(toks, pos, c["vocab"], c["sigma"]),
        lambda tok, pos: bf.kv_row_bits(tok, pos, LAYERS, HEADS, DIM))


@pytest.mark.parametrize("idx", range(6))
def test_oracle_matches_reference_beam_search(idx):
    rec = cases()[idx]
    got = oracle_run(rec)
    assert got["prompt_pages"] == rec["prompt_pages"]
    assert len(got["steps"]) == len(rec["steps"])
    for s_got, s_ref in zip(got["steps"], rec["steps"]):
        assert s_got == s_ref
    assert got["parents"] == rec["parents"]
    assert got["tokens"] == rec["tokens"]
    assert got["depths"] == rec["depths"]
    assert np.array_equal(np.float32(got["probs"]), np.float32(rec["probs"]))
    assert got["free_pages"] == rec["free_pages"]
    assert got["pool_sha1"] == rec["pool_sha1"]


def test_golden_covers_copy_on_write_and_fresh_pages():
    """The cases include steps that start a new page (offset 0) and steps that
    copy a shared partial page."""
    fresh = cow = 0
    for rec in cases():
        P = rec["case"]["page_len"]
        for s in rec["steps"]:
            if s["positions"][0] % P == 0:
                fresh += 1
            else:
                cow += 1
    assert fresh >= 3 and cow >= 10
