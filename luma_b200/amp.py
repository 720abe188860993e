"""``GradScaler.unscale_`` and the inf/NaN skip fused into the LUMA step.

Mixed-precision training with ``torch.amp.GradScaler`` runs, per iteration,
``scaler.step(opt)``: ``unscale_`` (one pass that reads and rewrites every
grad: ``g <- g * (1/scale)`` and a found-inf flag per device,
``torch._amp_foreach_non_finite_check_and_unscale_``), then a host read of the
flag, then ``opt.step()`` unless a grad was inf or NaN (reference usage:
IgorYashch/LUMA tests/test_mixed_precision.py:119-184).

``scaler_step(scaler, opt)`` gives the same results without the extra pass:
the LUMA step reads each grad as ``round_to_grad_dtype(fl32(g) * inv_scale)``
(what ``unscale_`` would have stored), its first pass raises the device flag
on any inf/NaN grad, and its second pass changes nothing when the flag is set.
The flag is recorded in the scaler's per-optimizer state, so
``scaler.update()`` backs off or grows the scale exactly as after
``scaler.step(opt)``.  It relies on ``GradScaler``'s per-optimizer bookkeeping
(``_per_optimizer_states``, ``OptState``), which torch has kept since 1.6.
"""

from __future__ import annotations

import torch
from torch.amp.grad_scaler import OptState

__all__ = ["scaler_step"]


def scaler_step(scaler: torch.amp.GradScaler, optimizer, *args, **kwargs):
    """Drop-in for ``scaler.step(optimizer)`` with a ``luma_b200.LUMA`` optimizer.

    Falls back to ``scaler.step`` when the fused path does not apply: the
    scaler is disabled, the caller already ran ``scaler.unscale_(optimizer)``
    (e.g. to clip), or the stepped params span several devices (a skip must
    cover all of them, which one device's flag cannot order).
    """
    if not scaler.is_enabled():
        return optimizer.step(*args, **kwargs)
    if "closure" in kwargs:
        raise RuntimeError("Closure use is not currently supported if GradScaler is enabled.")
    state = scaler._per_optimizer_states[id(optimizer)]
    if state["stage"] is OptState.STEPPED:
        raise RuntimeError("step() has already been called since the last update().")
    if state["stage"] is OptState.UNSCALED:
        return scaler.step(optimizer, *args, **kwargs)
    grads = [p.grad for g in optimizer.param_groups for p in g["params"] if p.grad is not None]
    if any(gr.dtype == torch.float16 for gr in grads):
        # GradScaler.unscale_ refuses fp16 grads (fp16 params): same error
        raise ValueError("Attempting to unscale FP16 gradients.")
    devices = {gr.device for gr in grads}
    if len(devices) > 1:
        return scaler.step(optimizer, *args, **kwargs)
    scaler._check_scale_growth_tracker("step")
    # The reciprocal in float64, then float32: GradScaler.unscale_'s inv_scale.
    dev = next(iter(devices)) if devices else scaler._scale.device
    inv_scale = scaler._scale.double().reciprocal().float().to(dev)
    found_inf = torch.full((), 0.0, dtype=torch.float32, device=dev)
    retval = optimizer.step(*args, grad_scale=inv_scale, found_inf=found_inf, **kwargs)
    state["found_inf_per_device"] = {found_inf.device: found_inf}
    state["stage"] = OptState.STEPPED
    return retval
