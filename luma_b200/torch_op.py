"""``torch.ops.luma_b200.step`` — the multi-tensor step as a PyTorch custom op.

The reference makes its Triton step functions traceable by ``torch.compile``
with ``fullgraph=True`` (IgorYashch/LUMA tests/test_compile.py:84-290).  This
op is the B200 equivalent: one call steps a list of tensors with
``luma_step`` in capturable mode (step counts and per-step scalars on the
device, so the op has no host-side per-step inputs), declares every tensor it
writes (params, codes, slots, step counters) so the compiler orders it
correctly, and has a fake implementation, so Dynamo records it as one node
without graph breaks.  The kernels address exactly the tensors passed in
(the descriptor table is built from their pointers, cached per pointer set),
so the op is also correct when the compiler hands it copies.

``LUMA(..., capturable=True).step_op_args()`` returns the arguments that step
the optimizer's parameters.
"""

from __future__ import annotations

import ctypes

import numpy as np
import torch

from . import _lib
from .engine import Segment, build_desc_table

__all__ = ["step"]

_TABLES: dict[tuple, tuple[torch.Tensor, int]] = {}
_MAX_TABLES = 64


def _desc_table(segs: list[Segment], device: torch.device) -> tuple[torch.Tensor, int]:
    key = tuple(s.key() for s in segs)
    hit = _TABLES.get(key)
    if hit is None:
        if torch.cuda.is_current_stream_capturing():
            raise RuntimeError("luma_b200::step: new tensors while a CUDA graph is being "
                               "captured; call the op once outside capture first")
        table, total = build_desc_table(segs)
        if len(_TABLES) >= _MAX_TABLES:
            _TABLES.clear()
        hit = (torch.from_numpy(table.view(np.uint8).copy()).to(device), total)
        _TABLES[key] = hit
    return hit


@torch.library.custom_op("luma_b200::step",
                         mutates_args=("params", "q_m", "q_w", "slots", "counters"))
def step(params: list[torch.Tensor], grads: list[torch.Tensor], q_m: list[torch.Tensor],
         q_w: list[torch.Tensor], slots: torch.Tensor, counters: torch.Tensor,
         row_table: torch.Tensor, param_ids: list[int], slot_ids: list[int],
         row_bases: list[int], base_seed: int,
         grad_scale: torch.Tensor | None = None) -> None:
    """One LUMA step of every tensor in `params` (contiguous CUDA tensors on one
    device): tensor i uses state slot slot_ids[i], its step count
    counters[slot_ids[i]] (advanced by one) and the rows of its group starting
    at row_table[row_bases[i]]; param_ids[i] keys its Philox stream.
    `grad_scale` (optional float32 scalar) is fused as in ``LUMA.step``."""
    if not params:
        return
    segs = [Segment(p, g, m, w, pid, rb, sl)
            for p, g, m, w, pid, sl, rb in zip(params, grads, q_m, q_w, param_ids, slot_ids,
                                               row_bases)]
    descs, total = _desc_table(segs, params[0].device)
    a = _lib.LumaStepArgs()
    a.descs = descs.data_ptr()
    a.slots = slots.data_ptr()
    a.rows = row_table.data_ptr()
    a.n_desc = len(segs)
    a.n_rows = row_table.numel() // _lib.ROW_DTYPE.itemsize
    a.total_octets = total
    a.base_seed = ctypes.c_int64(int(base_seed)).value
    a.max_ctas = 0
    a.step_counters = counters.data_ptr()
    if grad_scale is not None:
        grad_scale = grad_scale.reshape(1).to(dtype=torch.float32)  # exact for bf16 / fp16
    a.grad_scale = None if grad_scale is None else grad_scale.data_ptr()
    stream = torch.cuda.current_stream(params[0].device)
    _lib.check(_lib.lib().luma_step(ctypes.byref(a), ctypes.c_void_p(stream.cuda_stream)),
               "luma_step")


@step.register_fake
def _step_fake(params, grads, q_m, q_w, slots, counters, row_table, param_ids, slot_ids,
               row_bases, base_seed, grad_scale=None) -> None:
    return None
