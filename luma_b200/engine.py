"""Device-side bookkeeping of the CUDA backend: descriptor table, state slots,
per-step scalar rows, and the call into ``luma_step``.

One ``DeviceEngine`` per CUDA device.  It owns three device buffers (all
allocated through torch's caching allocator, never inside the step kernels):

* ``descs``  — the LumaTensorDesc table.  Rebuilt only when a pointer, size,
  row or slot of a segment changes (new grads, grads that went to None, a
  checkpoint load), otherwise reused step after step;
* ``slots``  — one LumaSlot per tensor (or shard segment): the two grids and
  the pass-1 accumulators.  Zero-filled when created;
* ``rows``   — the LumaStepRow table of this step, uploaded every step from
  a small ring of pinned host buffers (an event guards each ring entry, so a
  buffer is rewritten only after its copy has executed).

Capturable mode (CUDA-graph replay) replaces the per-step rows by a fixed
device table the caller builds once (one block of rows per param group, one
row per step) and adds ``counters``: one int64 step count per slot on the
device, advanced by the library after each step, so a replayed launch finds
its step, row and seed without host work.
"""

from __future__ import annotations

import ctypes
import itertools
from dataclasses import dataclass

import numpy as np
import torch

from . import _lib
from ._lib import DESC_DTYPE, GRID_DTYPE, ROW_DTYPE, SLOT_DTYPE

_DTYPE_CODE = {torch.float32: _lib.F32, torch.bfloat16: _lib.BF16, torch.float16: _lib.F16}

_RING = 4
_TABLE_CACHE = 4


def dtype_code(dt: torch.dtype) -> int:
    return _DTYPE_CODE[dt]


@dataclass
class Segment:
    """One descriptor: a whole tensor or one shard segment of it.  The four
    tensors are contiguous and of equal numel; their shapes do not matter."""
    param: torch.Tensor
    grad: torch.Tensor
    q_m: torch.Tensor
    q_w: torch.Tensor
    param_id: int
    row: int
    slot: int
    rng_offset: int = 0
    u_m: torch.Tensor | None = None
    u_w: torch.Tensor | None = None
    param_mc: int = 0  # multicast (NVLS) address the updated param goes to, 0 for none
    mc_local: bool = False  # with param_mc: also store to `param` (param_mc maps another buffer)

    def key(self) -> tuple:
        return (self.param.data_ptr(), self.grad.data_ptr(), self.q_m.data_ptr(),
                self.q_w.data_ptr(), self.param.numel(), self.param_id, self.row, self.slot,
                self.rng_offset, self.param.dtype, self.grad.dtype,
                0 if self.u_m is None else self.u_m.data_ptr(),
                0 if self.u_w is None else self.u_w.data_ptr(), self.param_mc, self.mc_local)


def build_desc_table(segs: list[Segment]) -> tuple[np.ndarray, int]:
    """numpy LumaTensorDesc table and the total octet count."""
    n = len(segs)
    d = np.zeros(n, dtype=DESC_DTYPE)
    if n == 0:
        return d, 0
    d["param"] = [s.param.data_ptr() for s in segs]
    d["grad"] = [s.grad.data_ptr() for s in segs]
    d["q_m"] = [s.q_m.data_ptr() for s in segs]
    d["q_w"] = [s.q_w.data_ptr() for s in segs]
    d["u_m"] = [0 if s.u_m is None else s.u_m.data_ptr() for s in segs]
    d["u_w"] = [0 if s.u_w is None else s.u_w.data_ptr() for s in segs]
    numel = np.array([s.param.numel() for s in segs], dtype=np.int64)
    octs = (numel + 7) // 8
    d["numel"] = numel
    d["oct_begin"] = np.concatenate([np.zeros(1, np.int64), np.cumsum(octs)[:-1]])
    d["rng_offset"] = [s.rng_offset for s in segs]
    d["param_id"] = [s.param_id for s in segs]
    d["row"] = [s.row for s in segs]
    d["slot"] = [s.slot for s in segs]
    d["param_dtype"] = [dtype_code(s.param.dtype) for s in segs]
    d["grad_dtype"] = [dtype_code(s.grad.dtype) for s in segs]
    ptrs = np.stack([d["param"], d["grad"], d["q_m"], d["q_w"], d["u_m"], d["u_w"]])
    d["vec_ok"] = np.all(ptrs % 16 == 0, axis=0).astype(np.uint8)
    mc = np.array([s.param_mc for s in segs], dtype=np.uint64)
    if mc.any():
        bad = (mc != 0) & (((mc % 8) != 0) | ((d["param"] % 8) != 0))
        if bad.any():
            raise ValueError("a segment with a multicast param address needs param and "
                             "param_mc 8-byte aligned")
    d["param_mc"] = mc
    d["mc_local"] = [1 if (s.param_mc and s.mc_local) else 0 for s in segs]
    return d, int(octs.sum())


class Columns:
    """The descriptor table of a plain step as columns (no multicast, no
    injected draws, counters from 0): the optimizer's per-step fast path.

    ``statics[i]`` is a tuple ``(param_ptr, q_m_ptr, q_w_ptr, numel, param_id,
    slot, param_dtype_code)`` that the caller keeps per parameter and reuses
    step after step (so comparing two signatures mostly compares identical
    objects); ``grad_ptrs``, ``grad_codes`` and ``rows`` change per step."""

    __slots__ = ("statics", "grad_ptrs", "grad_codes", "rows")

    def __init__(self):
        self.statics: list[tuple] = []
        self.grad_ptrs: list[int] = []
        self.grad_codes: list[int] = []
        self.rows: list[int] = []

    def __len__(self) -> int:
        return len(self.statics)

    def signature(self) -> tuple:
        return (tuple(self.statics), tuple(self.grad_ptrs), tuple(self.grad_codes),
                tuple(self.rows))


def build_desc_table_columns(cols: Columns) -> tuple[np.ndarray, int]:
    """numpy LumaTensorDesc table and total octet count of a ``Columns`` (the
    same table ``build_desc_table`` makes for the equivalent segments)."""
    n = len(cols)
    d = np.zeros(n, dtype=DESC_DTYPE)
    if n == 0:
        return d, 0
    st = np.fromiter(itertools.chain.from_iterable(cols.statics), dtype=np.int64,
                     count=7 * n).reshape(n, 7)
    grad = np.array(cols.grad_ptrs, dtype=np.uint64)
    d["param"] = st[:, 0]
    d["grad"] = grad
    d["q_m"] = st[:, 1]
    d["q_w"] = st[:, 2]
    numel = st[:, 3]
    octs = (numel + 7) // 8
    d["numel"] = numel
    d["oct_begin"] = np.concatenate([np.zeros(1, np.int64), np.cumsum(octs)[:-1]])
    d["param_id"] = st[:, 4]
    d["row"] = np.array(cols.rows, dtype=np.int32)
    d["slot"] = st[:, 5]
    d["param_dtype"] = st[:, 6]
    d["grad_dtype"] = np.array(cols.grad_codes, dtype=np.uint8)
    d["vec_ok"] = ((st[:, 0] % 16 == 0) & (st[:, 1] % 16 == 0) & (st[:, 2] % 16 == 0)
                   & (grad % 16 == 0)).astype(np.uint8)
    return d, int(octs.sum())


class DeviceEngine:
    def __init__(self, device: torch.device):
        self.device = device
        self.n_slots = 0
        self.slots = torch.zeros(0, dtype=torch.uint8, device=device)
        self.counters = torch.zeros(0, dtype=torch.int64, device=device)
        self.rows_dev = torch.zeros(ROW_DTYPE.itemsize * 4, dtype=torch.uint8, device=device)
        self._ring = []
        self._ring_i = 0
        self._sig = None
        self._descs_dev = None
        self._n_desc = 0
        self._total_oct = 0
        self._tables: dict[tuple, tuple[torch.Tensor, int, int]] = {}  # sig -> (descs, n, octets)
        self._pinned_tables: list[tuple[torch.Tensor, torch.cuda.Event]] = []  # copies in flight
        self._args = _lib.LumaStepArgs()

    # -- slots ---------------------------------------------------------------
    def ensure_slots(self, n: int) -> None:
        if n <= self.n_slots:
            return
        cap = max(n, 2 * self.n_slots, 16)
        new = torch.zeros(cap * SLOT_DTYPE.itemsize, dtype=torch.uint8, device=self.device)
        cnt = torch.zeros(cap, dtype=torch.int64, device=self.device)
        if self.n_slots:
            new[: self.slots.numel()].copy_(self.slots)
            cnt[: self.counters.numel()].copy_(self.counters)
        self.slots = new
        self.counters = cnt
        self.n_slots = cap
        self._sig = None  # slot base pointer changed
        self._tables.clear()

    def write_grid(self, slot: int, parity: int, rec: np.ndarray) -> None:
        """Store one LumaGrid into grid[parity] of `slot` (stream-ordered)."""
        off = slot * SLOT_DTYPE.itemsize + parity * GRID_DTYPE.itemsize
        src = torch.from_numpy(np.frombuffer(rec.tobytes(), dtype=np.uint8).copy())
        self.slots[off: off + GRID_DTYPE.itemsize].copy_(src)

    def reset_slot(self, slot: int) -> None:
        off = slot * SLOT_DTYPE.itemsize
        self.slots[off: off + SLOT_DTYPE.itemsize].zero_()

    def read_slots(self) -> np.ndarray:
        """All slots as a numpy LumaSlot array (synchronises the device)."""
        host = self.slots.cpu().numpy()
        return host.view(SLOT_DTYPE)

    # -- per step ------------------------------------------------------------
    def _upload_rows(self, rows: np.ndarray, stream: torch.cuda.Stream) -> None:
        nbytes = rows.nbytes
        if self.rows_dev.numel() < nbytes:
            self.rows_dev = torch.zeros(max(nbytes, 2 * self.rows_dev.numel()), dtype=torch.uint8,
                                        device=self.device)
        if not self._ring or self._ring[0][0].numel() < nbytes:
            cap = max(nbytes, 64 * ROW_DTYPE.itemsize)
            self._ring = [(torch.empty(cap, dtype=torch.uint8, pin_memory=True),
                           torch.cuda.Event()) for _ in range(_RING)]
            self._ring_i = 0
        buf, ev = self._ring[self._ring_i]
        self._ring_i = (self._ring_i + 1) % _RING
        ev.synchronize()  # the copy that last read this buffer has executed
        buf.numpy()[:nbytes] = np.frombuffer(rows.tobytes(), dtype=np.uint8)
        with torch.cuda.stream(stream):
            self.rows_dev[:nbytes].copy_(buf[:nbytes], non_blocking=True)
            ev.record(stream)

    def _upload_table(self, table: np.ndarray, stream: torch.cuda.Stream) -> torch.Tensor:
        """Device copy of a descriptor table, stream-ordered from pinned host
        memory (a pageable copy would wait for the kernels still running)."""
        host = torch.from_numpy(table.view(np.uint8)).pin_memory()
        dev = torch.empty(host.numel(), dtype=torch.uint8, device=self.device)
        with torch.cuda.stream(stream):
            dev.copy_(host, non_blocking=True)
        # the pinned buffer is kept until the copy recorded on `stream` has run
        ev = torch.cuda.Event()
        ev.record(stream)
        self._pinned_tables.append((host, ev))
        while self._pinned_tables and self._pinned_tables[0][1].query():
            self._pinned_tables.pop(0)
        return dev

    def step(self, segs: "list[Segment] | Columns", rows: np.ndarray | None, base_seed: int,
             stream: torch.cuda.Stream | None = None, events=None, max_ctas: int = 0,
             row_table: torch.Tensor | None = None,
             grad_scale: torch.Tensor | None = None,
             found_inf: torch.Tensor | None = None) -> None:
        """Launch one step.  `rows`: this step's LumaStepRow records (uploaded);
        or, in capturable mode, `row_table`: a fixed device table (rows=None),
        with the step counts taken from and advanced in ``self.counters``.
        `grad_scale`: optional float32 device scalar every grad is multiplied
        by (in the grad's dtype) inside the kernels.  `found_inf`: optional
        float32 device flag pass 1 raises on an inf/NaN grad; when set, pass 2
        leaves every param, code and step count unchanged."""
        if not len(segs):
            return
        if stream is None:
            stream = torch.cuda.current_stream(self.device)
        if isinstance(segs, Columns):
            sig = segs.signature()
            build = build_desc_table_columns
        else:
            sig = tuple(s.key() for s in segs)
            build = build_desc_table
        if sig != self._sig:
            # A few recent tables are kept, so callers that alternate grad
            # buffers (double buffering) do not rebuild one every step.
            hit = self._tables.get(sig)
            if hit is None:
                if torch.cuda.is_current_stream_capturing():
                    raise RuntimeError("LUMA: the set of parameters with gradients changed while "
                                       "a CUDA graph was being captured")
                table, total = build(segs)
                hit = (self._upload_table(table, stream), len(segs), total)
                if len(self._tables) >= _TABLE_CACHE:
                    self._tables.pop(next(iter(self._tables)))
                self._tables[sig] = hit
            self._descs_dev, self._n_desc, self._total_oct = hit
            self._sig = sig
        a = self._args
        if row_table is None:
            self._upload_rows(rows, stream)
            a.rows = self.rows_dev.data_ptr()
            a.n_rows = len(rows)
            a.step_counters = None
        else:
            a.rows = row_table.data_ptr()
            a.n_rows = row_table.numel() // ROW_DTYPE.itemsize
            a.step_counters = self.counters.data_ptr()
        a.descs = self._descs_dev.data_ptr()
        a.slots = self.slots.data_ptr()
        a.n_desc = self._n_desc
        a.total_octets = self._total_oct
        a.base_seed = ctypes.c_int64(int(base_seed)).value
        for i in range(3):
            a.events[i] = None if events is None else events[i]
        a.max_ctas = max_ctas
        a.grad_scale = None if grad_scale is None else grad_scale.data_ptr()
        a.found_inf = None if found_inf is None else found_inf.data_ptr()
        _lib.check(_lib.lib().luma_step(ctypes.byref(a), ctypes.c_void_p(stream.cuda_stream)),
                   "luma_step")
