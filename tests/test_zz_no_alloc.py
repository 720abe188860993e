"""luma_step_noalloc through the C ABI (GPU).

Some callers of this library cannot allocate device memory themselves: a
framework whose arena or caching allocator already holds the free HBM, an
FFI host with a fixed memory budget, or a step thread that must not call
cudaMalloc because it synchronises the device.  luma_step_noalloc serves
them: it takes the same tensors, descriptor/row tables and LumaSlot state as
luma_step, but keeps pass 1's per-tensor accumulators in a scratch array
built into the library instead of in the caller's slots.

This test steps identical tensors through luma_step and through
luma_step_noalloc, two calls in a row (the first step, then a quantized
step), and requires identical params, codes and scales — the bit-exact bar of
the other parity tests.  It sits in its own file so that it is collected
last, and builds everything it needs itself, so it also runs alone in a fresh
process.
"""

import ctypes

import numpy as np
import pytest
import torch

from luma_b200 import _lib
from luma_b200.engine import Segment, build_desc_table
from luma_b200.hostmath import rows_array, step_row

pytestmark = pytest.mark.gpu

SLOT_BYTES = _lib.SLOT_DTYPE.itemsize
GRID_BYTES = 2 * _lib.GRID_DTYPE.itemsize

# one tensor long enough for the shared decode table (>= 131072 elements in
# one CTA's segment), an unaligned-length one, a tiny one, mixed dtypes
SHAPES = [(5000,), (333, 77), (3,), (24_000_017,)]
PDTYPES = [torch.float32, torch.bfloat16, torch.float32, torch.bfloat16]
HP = dict(lr=1e-3, beta1=0.9, beta2=0.999, eps=1e-8, weight_decay=0.01)
BASE_SEED = -8_070_450_532_247_928_832


class _CallerState:
    """Everything a C caller owns: params, codes, slots (zero-filled)."""

    def __init__(self, params):
        self.params = [p.clone() for p in params]
        self.q_m = [torch.empty_like(p, dtype=torch.int16) for p in self.params]
        self.q_w = [torch.empty_like(p, dtype=torch.int16) for p in self.params]
        self.slots = torch.zeros(len(params) * SLOT_BYTES, dtype=torch.uint8, device="cuda")

    def step(self, entry, grads, t):
        segs = [Segment(p.view(-1), g.view(-1), m.view(-1), w.view(-1), param_id=i, row=0, slot=i)
                for i, (p, g, m, w) in enumerate(zip(self.params, grads, self.q_m, self.q_w))]
        table, total = build_desc_table(segs)
        descs = torch.from_numpy(table.view(np.uint8).copy()).cuda()
        rows = rows_array([step_row(t, HP["lr"], HP["beta1"], HP["beta2"], HP["eps"],
                                    HP["weight_decay"])])
        rows_dev = torch.from_numpy(rows.view(np.uint8).copy()).cuda()
        a = _lib.LumaStepArgs()
        a.descs = descs.data_ptr()
        a.slots = self.slots.data_ptr()
        a.rows = rows_dev.data_ptr()
        a.n_desc = len(segs)
        a.n_rows = 1
        a.total_octets = total
        a.base_seed = BASE_SEED
        stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
        status = entry(ctypes.byref(a), stream)
        assert status == _lib.LUMA_OK, _lib.lib().luma_last_error()
        torch.cuda.synchronize()  # descs/rows_dev stay alive until the kernels finish


def test_noalloc_matches_luma_step_two_calls():
    h = _lib.lib()
    gen = torch.Generator().manual_seed(11)
    params = [(torch.randn(s, generator=gen) * 0.02).to(dt).cuda() for s, dt in zip(SHAPES, PDTYPES)]
    ref = _CallerState(params)
    noalloc = _CallerState(params)
    for t in (1, 2):
        grads = [(torch.randn(s, generator=gen) * 1e-3).to(torch.bfloat16).cuda() for s in SHAPES]
        ref.step(h.luma_step, grads, t)
        noalloc.step(h.luma_step_noalloc, grads, t)
        for i in range(len(SHAPES)):
            assert torch.equal(ref.params[i], noalloc.params[i]), f"call {t}: param {i} differs"
            assert torch.equal(ref.q_m[i], noalloc.q_m[i]), f"call {t}: Q_m {i} differs"
            assert torch.equal(ref.q_w[i], noalloc.q_w[i]), f"call {t}: Q_w {i} differs"
        a = ref.slots.view(len(SHAPES), SLOT_BYTES)
        b = noalloc.slots.view(len(SHAPES), SLOT_BYTES)
        assert torch.equal(a[:, :GRID_BYTES], b[:, :GRID_BYTES]), f"call {t}: scales differ"
        # the caller's accumulator fields are left alone by the no-alloc entry point
        assert int(b[:, GRID_BYTES:].abs().sum()) == 0


def test_noalloc_rejects_tables_beyond_its_scratch():
    h = _lib.lib()
    a = _lib.LumaStepArgs()
    a.n_desc = _lib.NOALLOC_MAX_DESCS + 1
    a.n_rows = 1
    a.total_octets = a.n_desc
    status = h.luma_step_noalloc(ctypes.byref(a), None)
    assert status == _lib.LUMA_ERR_INVALID
    assert str(_lib.NOALLOC_MAX_DESCS).encode() in h.luma_last_error()


def _compare(ref, noalloc, n, tag):
    for i in range(n):
        assert torch.equal(ref.params[i], noalloc.params[i]), f"{tag}: param {i} differs"
        assert torch.equal(ref.q_m[i], noalloc.q_m[i]), f"{tag}: Q_m {i} differs"
        assert torch.equal(ref.q_w[i], noalloc.q_w[i]), f"{tag}: Q_w {i} differs"
    a = ref.slots.view(n, SLOT_BYTES)
    b = noalloc.slots.view(n, SLOT_BYTES)
    assert torch.equal(a[:, :GRID_BYTES], b[:, :GRID_BYTES]), f"{tag}: scales differ"


def test_noalloc_accepts_exactly_its_maximum_table():
    """LUMA_NOALLOC_MAX_DESCS tiny tensors in one call: accepted, and equal to
    luma_step over two calls."""
    h = _lib.lib()
    n = _lib.NOALLOC_MAX_DESCS
    rng = np.random.default_rng(3)
    sizes = [int(k) for k in rng.integers(1, 100, n)]
    gen = torch.Generator().manual_seed(4)
    params = [(torch.randn(s, generator=gen) * 0.02).cuda() for s in sizes]
    ref, noalloc = _CallerState(params), _CallerState(params)
    for t in (1, 2):
        grads = [(torch.randn(s, generator=gen) * 1e-3).cuda() for s in sizes]
        ref.step(h.luma_step, grads, t)
        noalloc.step(h.luma_step_noalloc, grads, t)
        _compare(ref, noalloc, n, f"{n} tensors, call {t}")


def test_noalloc_large_then_small_then_large_table():
    """The scratch array is shared by every call: a large table, then a smaller
    one, then the large one again must each match luma_step."""
    h = _lib.lib()
    gen = torch.Generator().manual_seed(5)
    big_sizes = [int(s) for s in np.random.default_rng(6).integers(1, 3000, 900)] + [2_000_003]
    small_sizes = [7, 4099, 1_000_001]
    states = {}
    for name, sizes in (("big", big_sizes), ("small", small_sizes)):
        params = [(torch.randn(s, generator=gen) * 0.02).cuda() for s in sizes]
        states[name] = (sizes, _CallerState(params), _CallerState(params))
    for k, name in enumerate(("big", "small", "big", "small", "big")):
        sizes, ref, noalloc = states[name]
        t = 1 + sum(1 for x in ("big", "small", "big", "small", "big")[:k] if x == name)
        grads = [(torch.randn(s, generator=gen) * 1e-3).cuda() for s in sizes]
        ref.step(h.luma_step, grads, t)
        noalloc.step(h.luma_step_noalloc, grads, t)
        _compare(ref, noalloc, len(sizes), f"call {k} ({name} table, step {t})")
