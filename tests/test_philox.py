"""Philox4x32-10 draw stream (oracle/philox.py) — CPU.

Known-answer vectors: the Random123 distribution's kat_vectors for
philox4x32 with 10 rounds (counter, key -> output), the published check
values of the generator the CUDA kernels implement."""

import numpy as np
import pytest

from oracle import philox

KAT = [
    ((0x00000000, 0x00000000, 0x00000000, 0x00000000), (0x00000000, 0x00000000),
     (0x6627E8D5, 0xE169C58D, 0xBC57AC4C, 0x9B00DBD8)),
    ((0xFFFFFFFF, 0xFFFFFFFF, 0xFFFFFFFF, 0xFFFFFFFF), (0xFFFFFFFF, 0xFFFFFFFF),
     (0x408F276D, 0x41C83B0E, 0xA20BC7C6, 0x6D5451FD)),
    ((0x243F6A88, 0x85A308D3, 0x13198A2E, 0x03707344), (0xA4093822, 0x299F31D0),
     (0xD16CFE09, 0x94FDCCEB, 0x5001E420, 0x24126EA1)),
]


@pytest.mark.parametrize("ctr,key,want", KAT)
def test_known_answers(ctr, key, want):
    out = philox.philox4x32_10(*[np.array([c], dtype=np.uint32) for c in ctr], *key)
    assert tuple(int(o[0]) for o in out) == want


def test_uniform_stream_layout():
    seed = philox.step_seed(-1234567890123, 7, 3)
    um, uw = philox.uniforms(seed, 9)
    # element 2k and 2k+1 share block k: words (0,1) and (2,3)
    x = philox.philox4x32_10(np.arange(5, dtype=np.uint32), np.zeros(5, np.uint32),
                             np.zeros(5, np.uint32), np.zeros(5, np.uint32),
                             seed & 0xFFFFFFFF, seed >> 32)
    s = np.float32(2.0 ** -24)
    for e in range(9):
        k, odd = divmod(e, 2)
        assert um[e] == np.float32(x[2 * odd][k] >> 8) * s
        assert uw[e] == np.float32(x[2 * odd + 1][k] >> 8) * s
    # offsets continue the same stream
    um2, uw2 = philox.uniforms(seed, 5, rng_offset=4)
    assert np.array_equal(um2, um[4:]) and np.array_equal(uw2, uw[4:])


def test_uniforms_in_unit_interval_and_24bit():
    um, uw = philox.uniforms(philox.step_seed(42, 1, 0), 100_000)
    for u in (um, uw):
        assert u.dtype == np.float32 and u.min() >= 0.0 and u.max() < 1.0
        assert np.all((u * np.float32(2 ** 24)) == np.floor(u * np.float32(2 ** 24)))
        assert abs(float(u.mean()) - 0.5) < 0.01


def test_seed_mix_matches_reference_formula():
    # functional.py:99-106: ((step << 32) | (param_id * 2)) ^ base_seed, as uint64 bits
    for base in (0, 1, -1, 2 ** 63 - 1, -(2 ** 63), 987654321987):
        for step, pid in ((1, 0), (2, 5), (100000, 123456)):
            ref = ((step << 32) | (pid * 2)) ^ base
            assert philox.step_seed(base, step, pid) == ref & 0xFFFFFFFFFFFFFFFF


@pytest.mark.parametrize("seed,n,off", [(0, 17, 0), (-1234567890123, 1000, 8),
                                        (2 ** 63 - 5, 333, 1 << 33), (-(2 ** 63), 64, 6)])
def test_torch_stream_equals_numpy_stream(seed, n, off):
    import torch
    s = philox.step_seed(seed, 5, 9)
    um, uw = philox.uniforms(s, n, off)
    tm, tw = philox.uniforms_torch(s, n, off, chunk=100)
    assert np.array_equal(tm.numpy(), um) and np.array_equal(tw.numpy(), uw)


def test_batched_step_draws_equal_per_tensor_draws():
    base = -987654321987
    items = [("a", 3, 0, 37, 0), ("b", 3, 5, 1, 16), ("c", 3, 7, 200, 1 << 32)]
    out = philox.step_draws_torch(base, items, "cpu", chunk=50)
    for key, step, pid, n, off in items:
        um, uw = philox.uniforms(philox.step_seed(base, step, pid), n, off)
        assert np.array_equal(out[key][0].numpy(), um) and np.array_equal(out[key][1].numpy(), uw)
