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


# ---------------------------------------------------------------------------
# The same stream with torch int64 tensors (CPU or CUDA), for tests that need
# draws for hundreds of millions of elements.  A uint32 x uint32 product fits
# in 64 bits; torch's int64 multiply keeps its low 64 bits (two's-complement
# wrap-around), so (p >> 32) & MASK and p & MASK are the product's high and
# low words.  Pinned against the numpy restatement above by tests/.
# ---------------------------------------------------------------------------

def _philox_torch(c0, c1, k0, k1):
    import torch
    mask = 0xFFFFFFFF
    c2 = torch.zeros_like(c0)
    c3 = torch.zeros_like(c0)
    for _ in range(10):
        p0 = c0 * int(M0)
        p1 = c2 * int(M1)
        c0, c1, c2, c3 = (((p1 >> 32) & mask) ^ c1 ^ k0, p1 & mask,
                          ((p0 >> 32) & mask) ^ c3 ^ k1, p0 & mask)
        k0 = (k0 + W0) & mask
        k1 = (k1 + W1) & mask
    return c0, c1, c2, c3


def uniforms_torch(seed, numel: int, rng_offset: int = 0, device="cpu", chunk: int = 1 << 26):
    """``uniforms`` as float32 torch tensors on `device`.  `seed` is one key
    (int) or an int64 tensor of per-element keys (one tensor's key repeated,
    for batching many tensors of one step into a single call)."""
    import torch
    u_m = torch.empty(numel, dtype=torch.float32, device=device)
    u_w = torch.empty(numel, dtype=torch.float32, device=device)
    scale = 2.0 ** -24
    for lo in range(0, numel, chunk):
        hi = min(numel, lo + chunk)
        e = torch.arange(lo, hi, dtype=torch.int64, device=device) + rng_offset
        pair = e >> 1
        if isinstance(seed, int):
            s = seed & 0xFFFFFFFFFFFFFFFF
            k0, k1 = s & 0xFFFFFFFF, s >> 32
        else:
            s = seed[lo:hi]
            k0, k1 = s & 0xFFFFFFFF, (s >> 32) & 0xFFFFFFFF
        x0, x1, x2, x3 = _philox_torch(pair & 0xFFFFFFFF, pair >> 32, k0, k1)
        odd = (e & 1).bool()
        wm = torch.where(odd, x2, x0)
        ww = torch.where(odd, x3, x1)
        u_m[lo:hi] = (wm >> 8).to(torch.float32) * scale
        u_w[lo:hi] = (ww >> 8).to(torch.float32) * scale
    return u_m, u_w


def step_draws_torch(base_seed: int, items, device, chunk: int = 1 << 26):
    """Draws of one step for many tensors at once: ``items`` is a list of
    (key, step, param_id, numel, rng_offset); returns {key: (u_m, u_w)}
    (1-D float32 views into two shared buffers).  Elements of one chunk may
    belong to several tensors: keys and counters are per element."""
    import torch
    total = sum(it[3] for it in items)
    u_m = torch.empty(total, dtype=torch.float32, device=device)
    u_w = torch.empty(total, dtype=torch.float32, device=device)
    seeds = torch.empty(total, dtype=torch.int64, device=device)
    ctr = torch.empty(total, dtype=torch.int64, device=device)
    pos = 0
    spans = []
    for key, step, pid, n, off in items:
        s = step_seed(base_seed, step, pid)
        seeds[pos:pos + n] = s - (1 << 64) if s >= (1 << 63) else s
        ctr[pos:pos + n] = torch.arange(off, off + n, dtype=torch.int64, device=device)
        spans.append((key, pos, n))
        pos += n
    scale = 2.0 ** -24
    for lo in range(0, total, chunk):
        hi = min(total, lo + chunk)
        e = ctr[lo:hi]
        pair = e >> 1
        s = seeds[lo:hi]
        x0, x1, x2, x3 = _philox_torch(pair & 0xFFFFFFFF, pair >> 32, s & 0xFFFFFFFF,
                                       (s >> 32) & 0xFFFFFFFF)
        odd = (e & 1).bool()
        u_m[lo:hi] = (torch.where(odd, x2, x0) >> 8).to(torch.float32) * scale
        u_w[lo:hi] = (torch.where(odd, x3, x1) >> 8).to(torch.float32) * scale
    return {key: (u_m[p:p + n], u_w[p:p + n]) for key, p, n in spans}
