"""Philox4x32-10 draw stream of the CUDA backend, in numpy — TEST INFRASTRUCTURE ONLY.

Only tests and the smoke check import this.  It restates the production
uniform stream of ``luma_b200`` so the GPU path can be compared bit for bit
with the oracle (``oracle/luma_ref.py``) in Philox mode as well as under
injected draws.

Generator: Philox4x32 with 10 rounds (Salmon, Moraes, Dror and Shaw,
"Parallel Random Numbers: As Easy as 1, 2, 3", SC'11): per round
``(c0, c1, c2, c3) <- (hi(M1*c2) ^ c1 ^ k0, lo(M1*c2), hi(M0*c0) ^ c3 ^ k1,
lo(M0*c0))`` and the key is bumped by the Weyl constants between rounds.

Stream definition (the backend's, not the reference's — the reference's two
backends already use two different generators, optimizer.py:62-68):
* key = the 64-bit seed ``((step << 32) | 2*param_id) ^ base_seed``
  (functional.py:99-106), low word k0, high word k1;
* element ``e`` of a tensor uses the block at counter
  ``((rng_offset + e) >> 1, high word, 0, 0)``; the even element of a pair
  takes words 0 and 1 as (u_m, u_w), the odd element words 2 and 3;
* a word becomes a float32 uniform in [0, 1) as ``(x >> 8) * 2**-24``.
"""

from __future__ import annotations

import numpy as np

M0 = np.uint64(0xD2511F53)
M1 = np.uint64(0xCD9E8D57)
W0 = 0x9E3779B9
W1 = 0xBB67AE85
MASK32 = np.uint64(0xFFFFFFFF)


def philox4x32_10(c0, c1, c2, c3, k0: int, k1: int):
    """Vectorised Philox4x32-10.  Counter words are uint32 arrays."""
    c0 = np.asarray(c0, dtype=np.uint64)
    c1 = np.asarray(c1, dtype=np.uint64)
    c2 = np.asarray(c2, dtype=np.uint64)
    c3 = np.asarray(c3, dtype=np.uint64)
    k0 &= 0xFFFFFFFF
    k1 &= 0xFFFFFFFF
    for _ in range(10):
        p0 = M0 * c0
        p1 = M1 * c2
        hi0, lo0 = p0 >> np.uint64(32), p0 & MASK32
        hi1, lo1 = p1 >> np.uint64(32), p1 & MASK32
        c0, c1, c2, c3 = (hi1 ^ c1 ^ np.uint64(k0)), lo1, (hi0 ^ c3 ^ np.uint64(k1)), lo0
        k0 = (k0 + W0) & 0xFFFFFFFF
        k1 = (k1 + W1) & 0xFFFFFFFF
    return (c0.astype(np.uint32), c1.astype(np.uint32), c2.astype(np.uint32), c3.astype(np.uint32))


def step_seed(base_seed: int, step: int, param_id: int) -> int:
    """64-bit key as an unsigned integer."""
    return (((step << 32) | (param_id * 2)) ^ base_seed) & 0xFFFFFFFFFFFFFFFF


def uniforms(seed: int, numel: int, rng_offset: int = 0):
    """(u_m, u_w) float32 arrays of length numel for one tensor / segment."""
    e = np.arange(numel, dtype=np.uint64) + np.uint64(rng_offset)
    pair = e >> np.uint64(1)
    odd = (e & np.uint64(1)).astype(bool)
    x0, x1, x2, x3 = philox4x32_10(pair & MASK32, pair >> np.uint64(32),
                                   np.zeros_like(pair), np.zeros_like(pair),
                                   seed & 0xFFFFFFFF, seed >> 32)
    wm = np.where(odd, x2, x0)
    ww = np.where(odd, x3, x1)
    scale = np.float32(2.0 ** -24)
    u_m = (wm >> np.uint32(8)).astype(np.float32) * scale
    u_w = (ww >> np.uint32(8)).astype(np.float32) * scale
    return u_m, u_w
