"""Philox4x32-10 counter-based generator, CPU twin of the device generator.

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the
CPU-baseline leg of bench.py.  The product path generates its uniforms on the
device (ecahlang_b200/csrc/common.cuh, ``philox4x32_10``).

Algorithm: Salmon, Moraes, Dror, Shaw, "Parallel Random Numbers: As Easy as
1, 2, 3", SC'11, section 4 (Philox-4x32 with 10 rounds).  Each round maps the
counter (c0, c1, c2, c3) with key (k0, k1) to

    hi0:lo0 = M0 * c0,  hi1:lo1 = M1 * c2
    (c0, c1, c2, c3) <- (hi1 ^ c1 ^ k0, lo1, hi0 ^ c3 ^ k1, lo0)

and bumps the key by the Weyl constants (W0, W1) between rounds.

The sampler's per-row uniform (this file and the device twin agree bit for
bit) is

    counter = (row_lo32, row_hi32, offset_lo32, offset_hi32)
    key     = (seed_lo32, seed_hi32)
    u       = (philox(counter, key)[0] >> 8) * 2**-24      in [0, 1)

which plays the role of the reference's per-row Philox stream
(FlashInfer ``curand_init(seed, row, offset)`` at the call sites
ecahlang/main.py:377-379, :489-491), with the uniform handed to the draw
instead of to a rejection loop.
"""
from __future__ import annotations

import numpy as np

M0 = np.uint64(0xD2511F53)
M1 = np.uint64(0xCD9E8D57)
W0 = np.uint32(0x9E3779B9)
W1 = np.uint32(0xBB67AE85)
_MASK32 = np.uint64(0xFFFFFFFF)


def philox4x32_10(ctr, key):
    """Vectorised Philox4x32-10.

    ctr: uint32 array of shape (..., 4); key: uint32 array of shape (..., 2)
    (broadcastable).  Returns uint32 array of shape (..., 4).
    """
    ctr = np.asarray(ctr, dtype=np.uint32)
    key = np.asarray(key, dtype=np.uint32)
    c0, c1, c2, c3 = (ctr[..., i].astype(np.uint64) for i in range(4))
    k0 = key[..., 0].astype(np.uint32)
    k1 = key[..., 1].astype(np.uint32)
    with np.errstate(over="ignore"):
        for r in range(10):
            if r:
                k0 = (k0 + W0).astype(np.uint32)
                k1 = (k1 + W1).astype(np.uint32)
            p0 = M0 * c0
            p1 = M1 * c2
            hi0, lo0 = p0 >> np.uint64(32), p0 & _MASK32
            hi1, lo1 = p1 >> np.uint64(32), p1 & _MASK32
            c0 = hi1 ^ c1 ^ k0.astype(np.uint64)
            c1 = lo1
            c2 = hi0 ^ c3 ^ k1.astype(np.uint64)
            c3 = lo0
    return np.stack([c0, c1, c2, c3], axis=-1).astype(np.uint32)


def row_uniforms(seed: int, offset: int, batch: int) -> np.ndarray:
    """Per-row uniforms u[r] in [0,1) for one sampler launch (float32)."""
    rows = np.arange(batch, dtype=np.uint64)
    ctr = np.zeros((batch, 4), dtype=np.uint32)
    ctr[:, 0] = (rows & _MASK32).astype(np.uint32)
    ctr[:, 1] = (rows >> np.uint64(32)).astype(np.uint32)
    ctr[:, 2] = np.uint32(offset & 0xFFFFFFFF)
    ctr[:, 3] = np.uint32((offset >> 32) & 0xFFFFFFFF)
    key = np.array([seed & 0xFFFFFFFF, (seed >> 32) & 0xFFFFFFFF], dtype=np.uint32)
    out = philox4x32_10(ctr, key)
    return ((out[:, 0] >> np.uint32(8)).astype(np.float32) * np.float32(2.0 ** -24)).astype(np.float32)
