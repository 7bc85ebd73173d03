"""Deterministic stand-ins for the draft model around the beam search (test
infrastructure: the golden generator runs the reference's ``beam_search``
with them on the CPU, the GPU tests run this package's with them).

``FakeModel`` takes the reference's patched forward signature
(``flashinfer/modeling_llama.py:23-104``).  Its logits for a beam depend only
on the beam's input token and position (seeded NumPy normals, rounded to
bf16), and it appends a K/V row per beam into the pool page the batch
position names for that position, as the attention's KV append would
(``flashinfer/attention_wrapper.py:201-212``), so that the copy-on-write page
copies of the beam search move real data.  Every batch position it is given
is recorded.
"""
from __future__ import annotations

import numpy as np
import torch

from oracle.accept import f32_to_bf16_bits


def bits_to_bf16(bits: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(bits, dtype=np.uint16).view(np.int16)).view(torch.bfloat16)


def step_logits_bits(tokens, positions, vocab: int, sigma: float) -> np.ndarray:
    """uint16 [len(tokens), vocab]: bf16 logits of each (token, position)."""
    out = np.empty((len(tokens), vocab), np.uint16)
    for i, (t, p) in enumerate(zip(tokens, positions)):
        rng = np.random.default_rng(int(t) * 100003 + int(p) * 7 + 11)
        out[i] = f32_to_bf16_bits((rng.standard_normal(vocab) * sigma).astype(np.float32))
    return out


def kv_row_bits(token: int, pos: int, num_layers: int, num_heads: int, head_dim: int) -> np.ndarray:
    """uint16 [L, 2, H, D]: the K/V row the model appends for (token, position)."""
    rng = np.random.default_rng(int(token) * 7919 + int(pos) * 31 + 5)
    return f32_to_bf16_bits(rng.standard_normal((num_layers, 2, num_heads, head_dim)).astype(np.float32))


def initial_pool_bits(seed: int, shape) -> np.ndarray:
    rng = np.random.default_rng(seed)
    return f32_to_bf16_bits(rng.standard_normal(shape).astype(np.float32))


class _Out:
    def __init__(self, logits):
        self.logits = logits


class FakeWrapper:
    """prepareAttention is a no-op: the fake model reads no attention."""

    def __init__(self):
        self.plans = []

    def prepareAttention(self, mode, batch_position, page_len, pos_encoding_mode, dtype, attention_mask=None):
        self.plans.append(mode)


class FakeModel(torch.nn.Module):
    def __init__(self, vocab: int, sigma: float, page_len: int):
        super().__init__()
        self.vocab, self.sigma, self.page_len = vocab, sigma, page_len
        self.lm_head = torch.nn.Linear(1, vocab, bias=False).to(torch.bfloat16)
        self.records = []                      # per call: (tokens, positions, indptr, indices, last_page_len)

    def forward(self, input_ids, position_ids=None, past_key_values=None, use_cache=False, kvCachePool=None,
                batch_position=None, mode="decode", flashinferWrapper=None, **kw):
        toks = input_ids[:, -1].cpu().tolist()
        pos = position_ids[:, -1].cpu().tolist()
        bp = batch_position
        indptr = bp.kv_page_indptr.cpu().tolist()
        indices = bp.kv_page_indices.cpu().tolist()
        last = bp.kv_last_page_len.cpu().tolist()
        self.records.append(dict(tokens=toks, positions=pos, indptr=indptr, indices=indices, last_page_len=last))
        pool = kvCachePool.cache_data                       # [L, P, 2, page, H, D]
        L, _, _, _, H, D = pool.shape
        for k, (t, p) in enumerate(zip(toks, pos)):
            page = indices[indptr[k] + p // self.page_len]
            row = bits_to_bf16(kv_row_bits(t, p, L, H, D)).to(pool.device)
            pool[:, page, :, p % self.page_len] = row
        logits = bits_to_bf16(step_logits_bits(toks, pos, self.vocab, self.sigma)).to(input_ids.device)
        return _Out(logits.unsqueeze(1))
