"""Philox4x32-10 counter-based RNG and the traversal uniform stream (oracle).

Philox4x32-10 is restated from its publication (Salmon, Moraes, Dror, Shaw,
"Parallel random numbers: as easy as 1, 2, 3", SC'11): ten rounds of two
32x32->64 multiplies, with the key bumped by the Weyl constants between
rounds.

The stream that stands in for ``torch.rand(1)`` in the reference's traversal
loop (``verification.py:396``: exactly one uniform per loop iteration) is:

    key     = (seed & 0xffffffff, seed >> 32)
    counter = (k >> 2, request, offset & 0xffffffff, offset >> 32)
    u(k)    = (philox(key, counter)[k & 3] >> 8) * 2**-24        (float32)

for draw ``k = 0, 1, 2, ...`` of request ``request``.  The CUDA kernel
computes the same function; tests monkeypatch ``torch.rand`` inside the
reference call to yield these values.
"""
from __future__ import annotations

import numpy as np

PHILOX_M0 = np.uint64(0xD2511F53)
PHILOX_M1 = np.uint64(0xCD9E8D57)
PHILOX_W0 = np.uint32(0x9E3779B9)
PHILOX_W1 = np.uint32(0xBB67AE85)
_MASK32 = np.uint64(0xFFFFFFFF)


def philox4x32_10(counter, key):
    """Vectorised Philox4x32-10.

    counter: uint32 array [..., 4]; key: uint32 array [..., 2] (broadcast).
    Returns uint32 array [..., 4].
    """
    c = np.array(counter, dtype=np.uint32)
    k = np.array(key, dtype=np.uint32)
    c0, c1, c2, c3 = (c[..., i].astype(np.uint64) for i in range(4))
    k0 = np.broadcast_to(k[..., 0], c0.shape).astype(np.uint64)
    k1 = np.broadcast_to(k[..., 1], c0.shape).astype(np.uint64)
    for r in range(10):
        if r > 0:
            k0 = (k0 + np.uint64(PHILOX_W0)) & _MASK32
            k1 = (k1 + np.uint64(PHILOX_W1)) & _MASK32
        p0 = PHILOX_M0 * c0
        p1 = PHILOX_M1 * c2
        hi0, lo0 = p0 >> np.uint64(32), p0 & _MASK32
        hi1, lo1 = p1 >> np.uint64(32), p1 & _MASK32
        n0 = hi1 ^ c1 ^ k0
        n2 = hi0 ^ c3 ^ k1
        c0, c1, c2, c3 = n0, lo1, n2, lo0
    return np.stack([c0, c1, c2, c3], axis=-1).astype(np.uint32)


def traversal_uniforms(seed: int, offset: int, request: int, count: int) -> np.ndarray:
    """First ``count`` uniforms (float32) of request ``request``'s stream."""
    k = np.arange(count, dtype=np.uint64)
    ctr = np.zeros((count, 4), dtype=np.uint32)
    ctr[:, 0] = (k >> np.uint64(2)).astype(np.uint32)
    ctr[:, 1] = np.uint32(request & 0xFFFFFFFF)
    ctr[:, 2] = np.uint32(offset & 0xFFFFFFFF)
    ctr[:, 3] = np.uint32((offset >> 32) & 0xFFFFFFFF)
    key = np.array([seed & 0xFFFFFFFF, (seed >> 32) & 0xFFFFFFFF], dtype=np.uint32)
    out = philox4x32_10(ctr, key)
    lane = out[np.arange(count), (k & np.uint64(3)).astype(np.int64)]
    return ((lane >> np.uint32(8)).astype(np.float32) * np.float32(2.0 ** -24)).astype(np.float32)


class UniformStream:
    """Iterator over one request's uniforms, as ``torch.rand(1)`` would yield."""

    def __init__(self, seed: int, offset: int, request: int, chunk: int = 256):
        self.seed, self.offset, self.request = seed, offset, request
        self._buf = traversal_uniforms(seed, offset, request, chunk)
        self.k = 0

    def next(self) -> np.float32:
        if self.k >= len(self._buf):
            self._buf = traversal_uniforms(self.seed, self.offset, self.request, 2 * len(self._buf))
        u = self._buf[self.k]
        self.k += 1
        return np.float32(u)
