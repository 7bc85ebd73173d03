"""Pin the oracle against the reference's own outputs (golden vectors)."""
import os

import numpy as np
import pytest

from oracle import accept as acc
from oracle import attention as att
from oracle import kv
from oracle.philox import UniformStream, philox4x32_10
from parallel_tree_spec_b200 import workload as wl
from tests.conftest import GOLDEN
from tests.golden_inputs import checked_inputs, sha1


def test_philox_known_answers():
    # Random123 known-answer vectors for Philox4x32-10
    assert [hex(v) for v in philox4x32_10([0, 0, 0, 0], [0, 0])] == \
        ["0x6627e8d5", "0xe169c58d", "0xbc57ac4c", "0x9b00dbd8"]
    assert [hex(v) for v in philox4x32_10([0xFFFFFFFF] * 4, [0xFFFFFFFF] * 2)] == \
        ["0x408f276d", "0x41c83b0e", "0xa20bc7c6", "0x6d5451fd"]
    assert [hex(v) for v in philox4x32_10([0x243F6A88, 0x85A308D3, 0x13198A2E, 0x03707344],
                                          [0xA4093822, 0x299F31D0])] == \
        ["0xd16cfe09", "0x94fdcceb", "0x5001e420", "0x24126ea1"]


def test_oracle_matches_reference_acceptance(accept_golden):
    """Accepted tokens, hidden indices and counts are bit-exact; the per-row
    argmax matches the reference's on every row; the per-node target
    probabilities agree to within one bf16 ulp (summation order)."""
    n_mb = n_mb_diff = 0
    for rec in accept_golden:
        c = rec["case"]
        t, x = checked_inputs(rec)
        T = c.get("temperature", 1.0) if c["method"] == "traversal" else 1.0
        am, p = acc.row_stats(x, T)
        assert am.tolist() == rec["ref_argmax"], c
        if c["method"] == "exact":
            s, h, tl, al = acc.greedy_walk(t.parents, t.tokens, am, rec["case"].get("eos_value"))
        else:
            mb = acc.mb_from_probs(t.parents, t.tokens, p)
            ref_mb = np.asarray(rec["ref_mb_f32"], np.float32)
            d = np.abs(mb - ref_mb)
            ulp = np.abs(ref_mb) * 2.0 ** -7 + 1e-38
            assert np.all(d <= ulp), c
            n_mb += len(mb)
            n_mb_diff += int(np.count_nonzero(d))
            us = UniformStream(c["philox_seed"], c.get("philox_offset", 0), c.get("request", 0))
            s, h, tl, al, nd = acc.traversal_walk(t.parents, t.tokens, t.draft_probs, mb, am, us,
                                                  rec["case"].get("eos_value"))
            assert nd == rec["draws"], c
        assert s == rec["tokens"], c
        assert h == rec["hidden"], c
        assert (tl, al) == (rec["total_len"], rec["accept_len"]), c
    assert n_mb_diff <= max(2, n_mb // 1000)


def test_golden_cases_cover_edges(accept_golden):
    kinds = {(r["case"]["method"], r["case"]["width"], r["case"]["depth"]) for r in accept_golden}
    assert ("exact", 0, 0) in kinds and ("traversal", 0, 0) in kinds      # root only
    assert any(r["case"]["vocab"] == 128256 for r in accept_golden)       # full vocabulary
    assert any(r["accept_len"] >= 4 for r in accept_golden)               # long accepted paths
    assert any(r["case"].get("eos_value") is not None and r["tokens"][-1] == r["case"]["eos_value"]
               for r in accept_golden)                                    # EOS stops the walk


def test_oracle_matches_reference_reorder(reorder_golden):
    for i, rec in enumerate(reorder_golden):
        before = np.load(os.path.join(GOLDEN, f"reorder_{i}_before.npy"))
        assert sha1(before) == rec["sha1_before"]
        cache = before.copy()
        pages = list(rec["pages_before"])
        new_len, last, kept, freed = kv.request_reorder(cache, pages, rec["prompt"] + rec["n_tree"],
                                                        rec["path"], rec["offset"])
        assert sha1(cache) == rec["sha1_after"], i
        assert (new_len, last, kept) == (rec["kv_len"], rec["last_page_len"], rec["pages_after"])
        # the pool-level (flat physical slot) form gives the same bytes for a fresh pool
        flat = before.copy()
        kv.pool_reorder_flat(flat, rec["path"], rec["offset"] - 1)
        assert sha1(flat) == rec["sha1_after"], i


def test_oracle_matches_reference_mask(mask_golden):
    for rec in mask_golden:
        m = att.tree_mask(rec["parents"], rec["prefix"])
        assert [1, 1, *m.shape] == rec["shape"]
        bits = np.unpackbits(np.asarray(rec["packed"], np.uint8))[: m.size].astype(bool)
        assert np.array_equal(bits.reshape(m.shape), m)


def test_attention_oracle_small():
    """The masked paged attention restatement equals a dense masked softmax."""
    rng = np.random.default_rng(3)
    t = wl.make_tree(rng, 3, 3, 100)
    n, P, Hq, Hkv, D, pl = t.size, 21, 4, 2, 8, 16
    kvl = P + n
    pages = rng.permutation(8)[: (kvl + pl - 1) // pl]
    layer = rng.standard_normal((8, 2, pl, Hkv, D)).astype(np.float32)
    q = rng.standard_normal((n, Hq, D)).astype(np.float32)
    mask = att.tree_mask(t.parents, P)
    out = att.tree_attention(q, layer, [pages], [kvl], [0, n], [mask], D ** -0.5)
    k, v = att.gather_kv(layer, pages, kvl)
    for h in range(Hq):
        s = q[:, h] @ k[:, h // 2].T * D ** -0.5
        s[~mask] = -1e30
        p = np.exp(s - s.max(1, keepdims=True))
        p /= p.sum(1, keepdims=True)
        np.testing.assert_allclose(out[:, h], p @ v[:, h // 2], rtol=1e-5, atol=1e-5)


def test_batch_positions():
    bi, pos = kv.batch_positions([10, 70], [3, 2])
    assert bi.tolist() == [0, 0, 0, 1, 1] and pos.tolist() == [7, 8, 9, 68, 69]


@pytest.mark.parametrize("T", [1.0, 0.8])
def test_row_probs_sum_to_one(T):
    rng = np.random.default_rng(0)
    x = wl._bf16_bits(rng.standard_normal((4, 5000)).astype(np.float32) * 3)
    p = acc.row_probs(x, T)
    assert np.allclose(p.sum(-1), 1.0, atol=2e-2)


def test_oracle_matches_reference_acceptance_f32():
    """fp32 logits: accepted paths and argmax exact against the reference run
    on fp32 logits (accept_f32.json); per-node probabilities within 5e-6
    relative (fp32 exp and summation order, and the reference divides by the
    temperature on the CPU where the device multiplies by its reciprocal)."""
    import json
    with open(os.path.join(GOLDEN, "accept_f32.json")) as f:
        recs = json.load(f)
    for rec in recs:
        c = rec["case"]
        t, x = checked_inputs(rec)
        T = c.get("temperature", 1.0) if c["method"] == "traversal" else 1.0
        am, p = acc.row_stats_f32(x, T)
        assert am.tolist() == rec["ref_argmax"], c
        if c["method"] == "exact":
            s, h, tl, al = acc.greedy_walk(t.parents, t.tokens, am, c.get("eos_value"))
        else:
            mb = acc.mb_from_probs(t.parents, t.tokens, p)
            np.testing.assert_allclose(mb, np.asarray(rec["ref_mb_f32"], np.float32), rtol=5e-6, atol=1e-12)
            s, h, tl, al, _ = acc.traversal_walk(t.parents, t.tokens, t.draft_probs, mb, am,
                                                 UniformStream(c["philox_seed"], c.get("philox_offset", 0),
                                                               c.get("request", 0)))
        assert (list(s), list(h), tl, al) == (rec["tokens"], rec["hidden"], rec["total_len"], rec["accept_len"]), c


def test_rope_oracle_matches_transformers():
    """oracle.kv.rope_bf16 = transformers' apply_rotary_pos_emb (the function
    the reference's attention calls before the append) on bf16 CPU tensors,
    bit for bit, for q and k of a Llama-shaped layer."""
    torch = pytest.importorskip("torch")
    mod = pytest.importorskip("transformers.models.llama.modeling_llama")
    from oracle import kv as okv
    g = torch.Generator().manual_seed(3)
    T, Hq, Hkv, D = 37, 8, 2, 128
    q = torch.randn(1, Hq, T, D, generator=g).to(torch.bfloat16)
    k = torch.randn(1, Hkv, T, D, generator=g).to(torch.bfloat16)
    pos = torch.arange(4090, 4090 + T).float()
    inv = 1.0 / (500000.0 ** (torch.arange(0, D, 2).float() / D))
    emb = torch.cat([pos[:, None] * inv[None]] * 2, dim=-1)[None]
    cos, sin = emb.cos().to(torch.bfloat16), emb.sin().to(torch.bfloat16)
    q_ref, k_ref = mod.apply_rotary_pos_emb(q, k, cos, sin)
    bits = lambda t: t.contiguous().view(torch.int16).numpy().view(np.uint16)
    for x, ref in ((q, q_ref), (k, k_ref)):
        got = okv.rope_bf16(bits(x[0].transpose(0, 1)), bits(cos[0]), bits(sin[0]))
        assert np.array_equal(got, bits(ref[0].transpose(0, 1)))
