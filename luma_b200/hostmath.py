"""Host-side scalar math of the LUMA step.

Everything here runs once per tensor or per (param group, step) class, never
per element.  It reproduces the reference's float64 Python arithmetic and the
float32 roundings its tensor ops apply to Python scalars:

* ``precompute`` is the grid precompute of functional.py:74-92 (Python
  ``math``, float64);
* ``grid_record`` turns it into the float32 values the kernels consume — a
  Python scalar multiplying a float32 tensor is rounded to float32, and on
  CUDA ``tensor / scalar`` is ``tensor * fl32(1.0 / scalar)`` (the reciprocal
  taken in float64, then rounded once to float32);
* ``step_row`` holds the per-step scalars of functional.py:262-264 and
  optimizer.py:423-426.
"""

from __future__ import annotations

import math

import numpy as np

from ._lib import GRID_DTYPE, ROW_DTYPE

K_M = (1 << 15) - 1         # reference config.py:23
K_W = (1 << 16) - 1         # reference config.py:24
SCALE_FLOOR_M = 1e-9        # reference config.py:25

_f32 = np.float32


def precompute(S_m: float, S_v: float, eps: float) -> tuple[float, float, float, float, float]:
    """(w_min, delta_m, z_m, delta_w, z_w) for scales (S_m, S_v) — functional.py:74-92."""
    w_min = 1.0 / (math.sqrt(S_v) + eps)
    delta_m = math.log1p(S_m) / K_M
    z_m = math.expm1(delta_m)
    ratio = 1.0 / (eps * w_min)
    delta_w = math.log(ratio) / K_W if ratio > 1.0 else 0.0
    z_w = math.expm1(delta_w) if delta_w > 0.0 else 1.0
    return w_min, delta_m, z_m, delta_w, z_w


def _inv32(x: float) -> np.float32:
    """fl32(1.0 / x), reciprocal in float64: the factor a CUDA float32 tensor is
    multiplied by when it is divided by the Python scalar x."""
    with np.errstate(over="ignore"):
        return _f32(1.0 / x)


def grid_record(S_m: float, S_v: float, eps: float) -> np.ndarray:
    """One LumaGrid (numpy record) for scales (S_m, S_v) and eps."""
    w_min, delta_m, z_m, delta_w, z_w = precompute(S_m, S_v, eps)
    g = np.zeros((), dtype=GRID_DTYPE)
    g["S_m"] = S_m
    g["S_v"] = S_v
    g["eps"] = eps
    g["dm"] = _f32(delta_m)
    g["inv_dm"] = _inv32(delta_m)
    g["inv_zm"] = _inv32(z_m)
    g["s_m32"] = _f32(S_m)
    g["w_min"] = _f32(w_min)
    g["inv_wmin"] = _inv32(w_min)
    g["dw"] = _f32(delta_w)
    g["inv_dw"] = _inv32(delta_w) if delta_w > 0.0 else _f32(0.0)
    g["inv_zw"] = _inv32(z_w)
    g["dw_pos"] = 1 if delta_w > 0.0 else 0
    return g


def step_row(step: int, lr: float, beta1: float, beta2: float, eps: float,
             weight_decay: float) -> tuple:
    """Scalars of one (group, step) class as a LumaStepRow tuple.

    Mirrors functional.py:262-264 (bc1, bc2, eta_t in float64), :278-279
    (decay and addcdiv value), :274-275 (EMA coefficients), :270 (eps) and
    :164 (w_max = 1 / eps).
    """
    bc1 = 1.0 - beta1 ** step
    bc2 = 1.0 - beta2 ** step
    eta = lr / bc1
    with np.errstate(over="ignore"):
        return (step, eps, _f32(beta1), _f32(1.0 - beta1), _f32(beta2), _f32(1.0 - beta2),
                _f32(1.0 - weight_decay * lr), _f32(-eta), _inv32(bc2), _f32(eps),
                _f32(1.0 / eps), _f32(0.0))


def step_rows(steps: np.ndarray, lr: float, beta1: float, beta2: float, eps: float,
              weight_decay: float) -> np.ndarray:
    """``step_row`` for many steps at once (numpy float64 ``power`` calls the
    same libm ``pow`` as Python's ``**``; the other operations are IEEE)."""
    t = np.asarray(steps, dtype=np.int64)
    tf = t.astype(np.float64)
    bc1 = 1.0 - np.power(beta1, tf)
    bc2 = 1.0 - np.power(beta2, tf)
    out = np.zeros(t.shape, dtype=ROW_DTYPE)
    with np.errstate(over="ignore", divide="ignore", invalid="ignore"):
        eta = lr / bc1
        out["step"] = t
        out["eps"] = eps
        out["beta1"] = _f32(beta1)
        out["omb1"] = _f32(1.0 - beta1)
        out["beta2"] = _f32(beta2)
        out["omb2"] = _f32(1.0 - beta2)
        out["decay"] = _f32(1.0 - weight_decay * lr)
        out["neg_eta"] = (-eta).astype(np.float32)
        out["inv_bc2"] = (1.0 / bc2).astype(np.float32)
        out["eps32"] = _f32(eps)
        out["w_max"] = _f32(1.0 / eps)
    return out


def rows_array(rows: list[tuple]) -> np.ndarray:
    return np.array(rows, dtype=ROW_DTYPE)
