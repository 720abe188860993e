"""Oracle for the LUMA step — TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
leg may import this module, and only as the checker or the timed CPU
baseline.  The product (``luma_b200``) never calls it.

What it is
----------
A restatement of the reference PyTorch backend of IgorYashch/LUMA
(``src/luma_optimizer/functional.py`` and the per-parameter loop of
``optimizer.py:413-524``), written as the same sequence of torch tensor ops.
The sequence is kept op for op on purpose: every torch op rounds to float32 on
its own, and the device's own ATen kernels decide details such as "tensor /
Python scalar" (a true division on CPU, a multiply by the float32 reciprocal
on CUDA).  Running this oracle on CUDA tensors therefore reproduces, bit for
bit, what the reference backend computes on the same GPU, and running it on
CPU tensors reproduces the reference on CPU (pinned by ``tests/golden``).

Differences from the reference, all test hooks:
* the stochastic-rounding uniforms are passed in explicitly (``rand_m``,
  ``rand_w``) instead of being drawn from a ``torch.Generator``;
* bf16 params (rejected by the reference, optimizer.py:443-448) are stepped by
  up-casting to float32, running the float32 step and rounding once to bf16
  (round to nearest even), which is the bf16 contract of the CUDA backend.
"""

from __future__ import annotations

import math
from typing import Callable

import torch
from torch import Tensor

K_M = (1 << 15) - 1   # config.py:23
K_W = (1 << 16) - 1   # config.py:24
SCALE_FLOOR_M = 1e-9  # config.py:25


# ---------------------------------------------------------------------------
# codec pieces (functional.py:24-176)
# ---------------------------------------------------------------------------

def encode_uint16(values: Tensor) -> Tensor:
    """0..65535 held in int32 -> int16 bits (functional.py:24-26)."""
    return values.to(torch.int16)


def decode_uint16(q: Tensor) -> Tensor:
    """int16 bits -> float 0..65535 (functional.py:29-31)."""
    return (q.to(torch.int32) & 0xFFFF).float()


def log_sr(y: Tensor, delta: float, z_denom: float, rand: Tensor, k_max: int) -> Tensor:
    """Log-to-linear corrected stochastic rounding (functional.py:38-67)."""
    if delta <= 0.0:
        return torch.zeros_like(y)
    lower = y.floor()
    frac = y - lower
    p_up = torch.expm1(frac * delta) / z_denom
    return (lower + (rand < p_up).to(y.dtype)).clamp(0, k_max)


def precompute(S_m: float, S_v: float, eps: float) -> tuple[float, float, float, float, float]:
    """(w_min, delta_m, z_m, delta_w, z_w) in float64 (functional.py:74-92)."""
    w_min = 1.0 / (math.sqrt(S_v) + eps)
    delta_m = math.log1p(S_m) / K_M
    z_m = math.expm1(delta_m)
    ratio = 1.0 / (eps * w_min)
    delta_w = math.log(ratio) / K_W if ratio > 1.0 else 0.0
    z_w = math.expm1(delta_w) if delta_w > 0.0 else 1.0
    return w_min, delta_m, z_m, delta_w, z_w


def make_step_seed(base_seed: int, step: int, param_id: int) -> int:
    """((step << 32) | 2*param_id) ^ base_seed (functional.py:99-106)."""
    return ((step << 32) | (param_id * 2)) ^ base_seed


def decode_momentum(Q_m: Tensor, delta_m: float) -> Tensor:
    """m = sgn(q) * expm1(|q| * delta_m) (functional.py:113-116)."""
    q = Q_m.float()
    return q.sign() * torch.expm1(q.abs() * delta_m)


def decode_preconditioner(Q_w: Tensor, w_min: float, delta_w: float) -> Tensor:
    """w = w_min * exp(q * delta_w) (functional.py:119-126)."""
    return w_min * torch.exp(decode_uint16(Q_w) * delta_w)


def quantize_momentum(m: Tensor, S_m: float, delta_m: float, z_m: float, rand: Tensor) -> Tensor:
    """Signed 15-bit LogSR code of m (functional.py:133-150)."""
    m_clip = m.clamp(-S_m, S_m)
    y = torch.log1p(m_clip.abs()) / delta_m
    mag = log_sr(y, delta_m, z_m, rand, K_M)
    return (m_clip.sign() * mag).to(torch.int16)


def quantize_preconditioner(v: Tensor, eps: float, w_min: float, delta_w: float, z_w: float,
                            rand: Tensor) -> Tensor:
    """Unsigned 16-bit LogSR code of w = 1/(sqrt(v)+eps) (functional.py:153-176)."""
    w = 1.0 / (v.clamp_min(0).sqrt() + eps)
    w_clip = w.clamp(w_min, 1.0 / eps)
    if delta_w > 0.0:
        y = torch.log(w_clip / w_min) / delta_w
    else:
        y = torch.zeros_like(w_clip)
    return encode_uint16(log_sr(y, delta_w, z_w, rand, K_W).to(torch.int32))


# ---------------------------------------------------------------------------
# step functions (functional.py:183-298)
# ---------------------------------------------------------------------------

def init_step(param: Tensor, grad: Tensor, beta1: float, beta2: float, eps: float, lr: float,
              weight_decay: float, rand_m: Tensor, rand_w: Tensor):
    """First step (functional.py:183-228).  Returns (Q_m, Q_w, S_m, S_v)."""
    g = grad.float()
    m = (1.0 - beta1) * g
    v = (1.0 - beta2) * g.square()
    bc1 = 1.0 - beta1
    bc2 = 1.0 - beta2
    param.mul_(1.0 - lr * weight_decay)
    param.addcdiv_(m, (v / bc2).sqrt().add_(eps), value=-(lr / bc1))
    S_m_t, S_v_t = torch.stack([m.abs().max(), v.max()]).tolist()
    S_m = max(S_m_t, SCALE_FLOOR_M)
    S_v = max(S_v_t, 0.0)
    w_min, delta_m, z_m, delta_w, z_w = precompute(S_m, S_v, eps)
    Q_m = quantize_momentum(m, S_m, delta_m, z_m, rand_m)
    Q_w = quantize_preconditioner(v, eps, w_min, delta_w, z_w, rand_w)
    return Q_m, Q_w, S_m, S_v


def update_step(param: Tensor, grad: Tensor, Q_m: Tensor, Q_w: Tensor, S_m: float, S_v: float,
                step: int, beta1: float, beta2: float, eps: float, lr: float,
                weight_decay: float, rand_m: Tensor, rand_w: Tensor):
    """Steps >= 2, two-pass matched scaling (functional.py:231-298).

    Updates param, Q_m, Q_w in place; returns (S_m_next, S_v_next).
    """
    g = grad.float()
    bc1 = 1.0 - beta1 ** step
    bc2 = 1.0 - beta2 ** step
    w_min, delta_m, _, delta_w, _ = precompute(S_m, S_v, eps)
    m = decode_momentum(Q_m, delta_m)
    w = decode_preconditioner(Q_w, w_min, delta_w)
    v = (1.0 / w - eps).clamp_min(0).square()
    m_new = beta1 * m + (1.0 - beta1) * g
    v_new = beta2 * v + (1.0 - beta2) * g.square()
    param.mul_(1.0 - weight_decay * lr)
    param.addcdiv_(m_new, (v_new / bc2).sqrt().add_(eps), value=-(lr / bc1))
    S_m_t, S_v_t = torch.stack([m_new.abs().max(), v_new.max()]).tolist()
    S_m_next = max(S_m_t, SCALE_FLOOR_M)
    S_v_next = max(S_v_t, 0.0)
    w_min_n, delta_m_n, z_m_n, delta_w_n, z_w_n = precompute(S_m_next, S_v_next, eps)
    Q_m.copy_(quantize_momentum(m_new, S_m_next, delta_m_n, z_m_n, rand_m))
    Q_w.copy_(quantize_preconditioner(v_new, eps, w_min_n, delta_w_n, z_w_n, rand_w))
    return S_m_next, S_v_next


def export_moments(Q_m: Tensor, Q_w: Tensor, S_m: float, S_v: float, eps: float):
    """(exp_avg, exp_avg_sq) decoded as optimizer.py:231-235 does."""
    w_min, delta_m, _, delta_w, _ = precompute(S_m, S_v, eps)
    exp_avg = decode_momentum(Q_m, delta_m)
    w = decode_preconditioner(Q_w, w_min, delta_w)
    return exp_avg, (1.0 / w - eps).clamp(min=0).square()


# ---------------------------------------------------------------------------
# optimizer loop (optimizer.py:413-524), draws supplied by a callback
# ---------------------------------------------------------------------------

DrawFn = Callable[[int, int, Tensor], "tuple[Tensor, Tensor]"]
"""draws(param_id, step, like) -> (rand_m, rand_w), float32 tensors shaped like `like`."""


class OracleLUMA:
    """The reference per-parameter loop over the restated step.

    ``params`` is a list of param groups (dicts with "params" and the four
    hyper-parameters) or a list of tensors.  State per tensor follows the
    reference layout: step, param_id, Q_m, Q_w, S_m, S_v.
    """

    def __init__(self, params, lr=1e-3, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.01,
                 draws: DrawFn | None = None):
        params = list(params)
        if params and isinstance(params[0], dict):
            groups = params
        else:
            groups = [{"params": params}]
        defaults = dict(lr=lr, betas=betas, eps=eps, weight_decay=weight_decay)
        self.param_groups = []
        for g in groups:
            full = dict(defaults)
            full.update(g)
            full["params"] = list(g["params"])
            self.param_groups.append(full)
        self.state: dict[int, dict] = {}
        self.draws = draws

    @torch.no_grad()
    def step(self):
        param_idx = 0
        for group in self.param_groups:
            beta1, beta2 = group["betas"]
            eps, lr, wd = group["eps"], group["lr"], group["weight_decay"]
            for p in group["params"]:
                param_idx += 1
                if p.grad is None:
                    continue
                if p.numel() == 0:
                    continue
                st = self.state.setdefault(id(p), {})
                if not st:
                    st["step"] = 0
                    st["param_id"] = param_idx - 1
                st["step"] += 1
                t = st["step"]
                work = p.data.float() if p.dtype == torch.bfloat16 else p.data
                rand_m, rand_w = self.draws(st["param_id"], t, work)
                if t == 1:
                    st["Q_m"], st["Q_w"], st["S_m"], st["S_v"] = init_step(
                        work, p.grad, beta1, beta2, eps, lr, wd, rand_m, rand_w)
                else:
                    st["S_m"], st["S_v"] = update_step(
                        work, p.grad, st["Q_m"], st["Q_w"], st["S_m"], st["S_v"], t,
                        beta1, beta2, eps, lr, wd, rand_m, rand_w)
                if work is not p.data:
                    p.data.copy_(work)

    def state_of(self, p: Tensor) -> dict:
        return self.state[id(p)]
