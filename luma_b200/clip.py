"""Gradient-norm clipping fused into the step.

The reference clips before every step (IgorYashch/LUMA
benchmarks/bench_nanogpt.py:218-225: ``clip_grad_norm_(params, 1.0)`` then
``opt.step()``).  ``clip_grad_norm_`` reads every grad for the norm and then
reads and writes every grad again to rescale it.  ``clip_grad_coef`` computes
the same norm and coefficient with PyTorch's own functions and leaves the
grads alone; ``LUMA.step(grad_scale=coef)`` applies the rescaling inside the
step's kernels, element by element as ``torch._foreach_mul_`` would store it,
so the result is bit-identical to clipping first and the extra pass over the
grads disappears.
"""

from __future__ import annotations

import torch

__all__ = ["clip_grad_coef"]


def clip_grad_coef(parameters, max_norm: float, norm_type: float = 2.0,
                   error_if_nonfinite: bool = False,
                   foreach: bool | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """(total_norm, coef): the norm ``clip_grad_norm_`` would return and the
    float32 coefficient it would multiply the grads by,
    ``clamp(max_norm / (total_norm + 1e-6), max=1)``; grads are not modified."""
    if isinstance(parameters, torch.Tensor):
        parameters = [parameters]
    grads = [p.grad for p in parameters if p.grad is not None]
    if not grads:
        return torch.tensor(0.0), torch.tensor(1.0)
    total_norm = torch.nn.utils.get_total_norm(grads, norm_type, error_if_nonfinite, foreach)
    clip_coef = float(max_norm) / (total_norm + 1e-6)
    return total_norm, torch.clamp(clip_coef, max=1.0)
