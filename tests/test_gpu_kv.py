"""GPU parity: paged-KV append, batch positions, compaction and mask packing."""
import os

import numpy as np
import pytest
import torch

from oracle import attention as att
from oracle import kv as okv
from parallel_tree_spec_b200 import kernels as K
from parallel_tree_spec_b200 import workload as wl
from tests.conftest import GOLDEN
from tests.golden_inputs import sha1

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def to_dev_bits(a: np.ndarray) -> torch.Tensor:
    if a.dtype == np.uint16:
        return torch.from_numpy(a.view(np.int16).copy()).to(DEV)
    return torch.from_numpy(a.view(np.int32).copy()).to(DEV)


def from_dev_bits(t: torch.Tensor, dtype) -> np.ndarray:
    return t.cpu().numpy().view(dtype)


@pytest.mark.parametrize("flat", [False, True])
def test_compaction_matches_reference_reorder(reorder_golden, flat):
    for i, rec in enumerate(reorder_golden):
        before = np.load(os.path.join(GOLDEN, f"reorder_{i}_before.npy"))
        pool = to_dev_bits(before)
        L, P, _, pl, H, D = before.shape
        if flat:      # pool-level form: flat physical slots (identity page table)
            pages = list(range(P))
        else:         # request-level form: the request's page table
            pages = rec["pages_before"]
        path = rec["path"]
        K.kv_compact(pool, torch.tensor([0, len(pages)], dtype=torch.int32, device=DEV),
                     torch.tensor(pages, dtype=torch.int32, device=DEV),
                     torch.tensor([path], dtype=torch.int32, device=DEV),
                     torch.tensor([len(path)], dtype=torch.int32, device=DEV),
                     torch.tensor([rec["offset"] - 1], dtype=torch.int32, device=DEV))
        assert sha1(from_dev_bits(pool, before.dtype)) == rec["sha1_after"], i


def test_compaction_batched_page_tables_vs_oracle():
    rng = np.random.default_rng(4)
    L, P, pl, H, D = 3, 64, 16, 8, 128
    pool = rng.integers(0, 2 ** 16, size=(L, P, 2, pl, H, D), dtype=np.uint16)
    perm = rng.permutation(P).tolist()
    tables, paths, offs, lens = [], [], [], []
    cur = 0
    for b in range(5):
        kvl = int(rng.integers(40, 120))
        npg = (kvl + pl - 1) // pl
        tables.append(perm[cur:cur + npg])
        cur += npg
        n_tree = 20
        off = kvl - n_tree
        path = [0] + sorted(rng.choice(np.arange(1, n_tree), size=int(rng.integers(0, 6)), replace=False).tolist())
        if b % 2:
            path = path + [path[-1]]
        paths.append(path)
        offs.append(off)
        lens.append(kvl)
    exp = pool.copy()
    for tb, pth, off, kvl in zip(tables, paths, offs, lens):
        okv.request_reorder(exp, tb, kvl, pth, off + 1)
    dpool = to_dev_bits(pool)
    pind = np.cumsum([0] + [len(t) for t in tables]).astype(np.int32)
    S = max(len(p) for p in paths) + 3
    acc = np.full((5, S), -7, np.int32)          # padding past each count is never read
    for b, pth in enumerate(paths):
        acc[b, :len(pth)] = pth
    counts = np.zeros((5, 4), np.int32)
    counts[:, 0] = [len(p) for p in paths]
    nkv = torch.empty(5, dtype=torch.int32, device=DEV)
    nlast = torch.empty(5, dtype=torch.int32, device=DEV)
    K.kv_compact(dpool, torch.from_numpy(pind).to(DEV), torch.tensor(sum(tables, []), dtype=torch.int32, device=DEV),
                 torch.from_numpy(acc).to(DEV), torch.from_numpy(counts).to(DEV),
                 torch.tensor(offs, dtype=torch.int32, device=DEV), nkv, nlast)
    assert np.array_equal(from_dev_bits(dpool, np.uint16), exp)
    assert nkv.cpu().tolist() == [o + len(p) for o, p in zip(offs, paths)]
    assert nlast.cpu().tolist() == [(o + len(p) - 1) % pl + 1 for o, p in zip(offs, paths)]


def test_append_and_positions_vs_oracle():
    rng = np.random.default_rng(8)
    P, pl, H, D = 40, 16, 8, 128
    layer = rng.integers(0, 2 ** 16, size=(P, 2, pl, H, D), dtype=np.uint16)
    perm = rng.permutation(P).tolist()
    kv_lens, n_app, tables = [], [], []
    cur = 0
    for b in range(4):
        n = int(rng.integers(1, 30))
        kvl = int(rng.integers(n, 100))
        npg = (kvl + pl - 1) // pl
        tables.append(perm[cur:cur + npg])
        cur += npg
        kv_lens.append(kvl)
        n_app.append(n)
    T = sum(n_app)
    k = rng.integers(0, 2 ** 16, size=(T, H, D), dtype=np.uint16)
    v = rng.integers(0, 2 ** 16, size=(T, H, D), dtype=np.uint16)
    bi, pos = okv.batch_positions(kv_lens, n_app)
    exp = layer.copy()
    okv.append(exp, k, v, tables, bi, pos)
    app_ind = torch.tensor(np.cumsum([0] + n_app), dtype=torch.int32, device=DEV)
    dbi, dpos = K.batch_positions(app_ind, torch.tensor(kv_lens, dtype=torch.int32, device=DEV), T)
    assert dbi.cpu().numpy().tolist() == bi.tolist() and dpos.cpu().numpy().tolist() == pos.tolist()
    dl = to_dev_bits(layer).view(torch.bfloat16)
    K.kv_append(to_dev_bits(k).view(torch.bfloat16), to_dev_bits(v).view(torch.bfloat16), dl, dbi, dpos,
                torch.tensor(np.cumsum([0] + [len(t) for t in tables]), dtype=torch.int32, device=DEV),
                torch.tensor(sum(tables, []), dtype=torch.int32, device=DEV))
    assert np.array_equal(from_dev_bits(dl.view(torch.int16), np.uint16), exp)


def test_tree_masks_vs_oracle():
    rng = np.random.default_rng(1)
    trees = [wl.make_tree(rng, w, d, 500) for (w, d) in [(8, 8), (3, 2), (0, 0), (16, 8), (1, 70)]]
    indptr, par, tok, dp = wl.stack_trees(trees)
    words = K.mask_words_for(max(t.size for t in trees))
    bits = K.tree_mask_from_parents(torch.from_numpy(par).to(DEV), torch.from_numpy(indptr).to(DEV), words)
    bits = bits.cpu().numpy().view(np.uint64)
    prefixes = [5, 0, 3, 17, 1]
    flat, mind, kvl = [], [0], []
    for b, t in enumerate(trees):
        a = att.ancestor_mask(t.parents)
        rows = bits[indptr[b]:indptr[b + 1]]
        got = np.array([[(rows[i, j // 64] >> np.uint64(j % 64)) & np.uint64(1) for j in range(t.size)]
                        for i in range(t.size)], dtype=bool)
        assert np.array_equal(got, a), b
        m = att.tree_mask(t.parents, prefixes[b])
        flat.append(m.reshape(-1))
        mind.append(mind[-1] + m.size)
        kvl.append(m.shape[1])
    bits2 = K.tree_mask_from_bool(torch.from_numpy(np.concatenate(flat)).to(DEV), torch.from_numpy(indptr).to(DEV),
                                  torch.tensor(mind, dtype=torch.int32, device=DEV),
                                  torch.tensor(kvl, dtype=torch.int32, device=DEV), words)
    assert np.array_equal(bits2.cpu().numpy().view(np.uint64), bits)
    bad = np.concatenate(flat).copy()
    bad[0] = False
    with pytest.raises(ValueError):
        K.tree_mask_from_bool(torch.from_numpy(bad).to(DEV), torch.from_numpy(indptr).to(DEV),
                              torch.tensor(mind, dtype=torch.int32, device=DEV),
                              torch.tensor(kvl, dtype=torch.int32, device=DEV), words)


def test_tree_prepare_matches_masks_and_positions():
    """pts_tree_prepare (one launch) = pts_tree_mask_from_parents + pts_batch_positions,
    including a 1024-node chain (words = 16) and a root-only tree."""
    rng = np.random.default_rng(12)
    trees = [wl.make_tree(rng, w, d, 500) for (w, d) in [(8, 8), (0, 0), (16, 8), (1, 1023), (3, 5)]]
    indptr, par, tok, dp = wl.stack_trees(trees)
    T = int(indptr[-1])
    words = K.mask_words_for(max(t.size for t in trees))
    dpar, dind = torch.from_numpy(par).to(DEV), torch.from_numpy(indptr).to(DEV)
    seq = torch.tensor([t.size + int(rng.integers(0, 300)) for t in trees], dtype=torch.int32, device=DEV)
    bits, bi, pos = K.tree_prepare(dpar, dind, words, seq)
    ref_bits = K.tree_mask_from_parents(dpar, dind, words)
    rbi, rpos = K.batch_positions(dind, seq, T)
    assert torch.equal(bits, ref_bits)
    assert torch.equal(bi, rbi) and torch.equal(pos, rpos)
    bits2, none_bi, none_pos = K.tree_prepare(dpar, dind, words)
    assert torch.equal(bits2, ref_bits) and none_bi is None and none_pos is None


@pytest.mark.parametrize("shapes", [[(8, 8), (0, 0), (16, 8), (1, 40), (3, 5)], [(0, 0), (2, 1), (1, 3)] * 367])
def test_tree_prepare_append_matches_separate_launches(shapes):
    """pts_tree_prepare_append (one launch) = pts_tree_prepare + pts_kv_append:
    the same masks and positions and every byte of the layer, for a ragged
    batch and for 1101 requests (the append CTAs then search qo_indptr in
    global memory)."""
    rng = np.random.default_rng(len(shapes))
    trees = [wl.make_tree(rng, w, d, 500) for (w, d) in shapes]
    indptr, par, tok, dp = wl.stack_trees(trees)
    T, B = int(indptr[-1]), len(trees)
    Hkv, D, pl = 2, 64, 16
    prefix = rng.integers(0, 70, size=B)
    seq = prefix + np.array([t.size for t in trees])
    npages = (seq + pl - 1) // pl
    P = int(npages.sum()) + 3
    perm = rng.permutation(P)[:int(npages.sum())].astype(np.int32)
    pind = np.concatenate([[0], np.cumsum(npages)]).astype(np.int32)
    layer = torch.randn(P, 2, pl, Hkv, D, generator=torch.Generator().manual_seed(3)).to(torch.bfloat16).to(DEV)
    k = torch.randn(T, Hkv, D, generator=torch.Generator().manual_seed(4)).to(torch.bfloat16).to(DEV)
    v = torch.randn(T, Hkv, D, generator=torch.Generator().manual_seed(5)).to(torch.bfloat16).to(DEV)
    words = K.mask_words_for(max(t.size for t in trees))
    dpar, dind = torch.from_numpy(par).to(DEV), torch.from_numpy(indptr).to(DEV)
    dseq = torch.from_numpy(seq.astype(np.int32)).to(DEV)
    dpind, dperm = torch.from_numpy(pind).to(DEV), torch.from_numpy(perm).to(DEV)
    fused = layer.clone()
    bits, bi, pos = K.tree_prepare_append(dpar, dind, words, dseq, k, v, fused, dpind, dperm)
    sep = layer.clone()
    rbits, rbi, rpos = K.tree_prepare(dpar, dind, words, dseq)
    K.kv_append(k, v, sep, rbi, rpos, dpind, dperm)
    torch.cuda.synchronize()
    assert torch.equal(bits, rbits) and torch.equal(bi, rbi) and torch.equal(pos, rpos)
    assert torch.equal(fused.view(torch.int16), sep.view(torch.int16))
    assert not torch.equal(fused.view(torch.int16), layer.view(torch.int16))


def _rotate_half(x):
    h = x.shape[-1] // 2
    return torch.cat((-x[..., h:], x[..., :h]), dim=-1)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_tree_prepare_append_rope_matches_torch(dtype):
    """pts_tree_prepare_append_rope = apply_rotary_pos_emb in torch (q * cos +
    rotate_half(q) * sin, eager ops in the same dtype) followed by
    pts_tree_prepare_append: bit-exact q, masks, positions and cache bytes."""
    rng = np.random.default_rng(21)
    trees = [wl.make_tree(rng, w, d, 500) for (w, d) in [(8, 8), (0, 0), (4, 3), (2, 5)]]
    indptr, par, tok, dp = wl.stack_trees(trees)
    T, B = int(indptr[-1]), len(trees)
    Hq, Hkv, D, pl = 8, 2, 128, 16
    prefix = rng.integers(0, 70, size=B)
    seq = prefix + np.array([t.size for t in trees])
    npages = (seq + pl - 1) // pl
    P = int(npages.sum()) + 2
    perm = rng.permutation(P)[:int(npages.sum())].astype(np.int32)
    pind = torch.from_numpy(np.concatenate([[0], np.cumsum(npages)]).astype(np.int32)).to(DEV)
    pidx = torch.from_numpy(perm).to(DEV)
    g = torch.Generator().manual_seed(7)
    q = torch.randn(T, Hq, D, generator=g).to(dtype).to(DEV)
    k = torch.randn(T, Hkv, D, generator=g).to(dtype).to(DEV)
    v = torch.randn(T, Hkv, D, generator=g).to(dtype).to(DEV)
    # Llama-style embeddings: positions of the tree tokens, theta 500000, fp32 then the model dtype
    posn = torch.from_numpy(np.concatenate([np.arange(s - t.size, s) for s, t in zip(seq, trees)])).float()
    inv = 1.0 / (500000.0 ** (torch.arange(0, D, 2).float() / D))
    emb = torch.cat([posn[:, None] * inv[None], posn[:, None] * inv[None]], dim=-1)
    cos, sin = emb.cos().to(dtype).to(DEV), emb.sin().to(dtype).to(DEV)
    layer = torch.randn(P, 2, pl, Hkv, D, generator=g).to(dtype).to(DEV)
    words = K.mask_words_for(max(t.size for t in trees))
    dpar, dind = torch.from_numpy(par).to(DEV), torch.from_numpy(indptr).to(DEV)
    dseq = torch.from_numpy(seq.astype(np.int32)).to(DEV)
    fused = layer.clone()
    bits, bi, pos, q_rot = K.tree_prepare_append_rope(dpar, dind, words, dseq, q, k, v, cos, sin, fused, pind, pidx)
    q_ref = q * cos[:, None] + _rotate_half(q) * sin[:, None]
    k_ref = k * cos[:, None] + _rotate_half(k) * sin[:, None]
    sep = layer.clone()
    rbits, rbi, rpos = K.tree_prepare_append(dpar, dind, words, dseq, k_ref, v, sep, pind, pidx)
    torch.cuda.synchronize()
    iv = torch.int16 if dtype == torch.bfloat16 else torch.int32
    assert torch.equal(q_rot.view(iv), q_ref.view(iv))
    assert torch.equal(bits, rbits) and torch.equal(bi, rbi) and torch.equal(pos, rpos)
    assert torch.equal(fused.view(iv), sep.view(iv))


def test_kv_append_rope_matches_torch():
    """pts_kv_append_rope = torch's apply_rotary_pos_emb arithmetic, then
    pts_kv_append: bit-exact rotated q and cache bytes (bf16)."""
    g = torch.Generator().manual_seed(8)
    T, Hq, Hkv, D, pl, P = 40, 4, 2, 128, 16, 8
    bi = torch.tensor([t // 20 for t in range(T)], dtype=torch.int32, device=DEV)
    pos = torch.tensor([5 + t % 20 for t in range(T)], dtype=torch.int32, device=DEV)
    pind = torch.tensor([0, 3, 6], dtype=torch.int32, device=DEV)
    pidx = torch.tensor([4, 0, 7, 2, 5, 1], dtype=torch.int32, device=DEV)
    q = torch.randn(T, Hq, D, generator=g).to(torch.bfloat16).to(DEV)
    k = torch.randn(T, Hkv, D, generator=g).to(torch.bfloat16).to(DEV)
    v = torch.randn(T, Hkv, D, generator=g).to(torch.bfloat16).to(DEV)
    emb = torch.randn(T, D // 2, generator=g) * 30
    emb = torch.cat([emb, emb], dim=-1)
    cos, sin = emb.cos().to(torch.bfloat16).to(DEV), emb.sin().to(torch.bfloat16).to(DEV)
    layer = torch.randn(P, 2, pl, Hkv, D, generator=g).to(torch.bfloat16).to(DEV)
    fused = layer.clone()
    qr = K.kv_append_rope(q, k, v, cos, sin, fused, bi, pos, pind, pidx)
    q_ref = q * cos[:, None] + _rotate_half(q) * sin[:, None]
    k_ref = k * cos[:, None] + _rotate_half(k) * sin[:, None]
    sep = layer.clone()
    K.kv_append(k_ref, v, sep, bi, pos, pind, pidx)
    torch.cuda.synchronize()
    assert torch.equal(qr.view(torch.int16), q_ref.view(torch.int16))
    assert torch.equal(fused.view(torch.int16), sep.view(torch.int16))
