"""Known-answer and statistical checks of the oracle's building blocks — CPU.

Mirrors the reference's own unit tests (tests/test_correctness.py:26-168):
uint16 round trip, LogSR unbiasedness, decode known answers."""

import math

import pytest
import torch

from oracle.luma_ref import (K_M, K_W, decode_momentum, decode_preconditioner, decode_uint16,
                             encode_uint16, log_sr, precompute, quantize_preconditioner)


@pytest.mark.parametrize("val", [0, 1, 32767, 32768, 65535])
def test_uint16_roundtrip(val):
    t = torch.tensor([val], dtype=torch.int32)
    assert decode_uint16(encode_uint16(t)).item() == float(val)


def test_uint16_batch_roundtrip():
    vals = torch.arange(0, K_W + 1, step=1000, dtype=torch.int32)
    assert torch.equal(decode_uint16(encode_uint16(vals)), vals.float())


def _unbiased(true_val, delta, z, k_max, to_y, from_q, tol, n=200_000):
    y = torch.full((n,), to_y(true_val))
    q = log_sr(y, delta, z, torch.rand(n), k_max)
    mean = from_q(q).mean().item()
    assert abs(mean - true_val) / abs(true_val) < tol, (true_val, mean)


@pytest.mark.parametrize("val", [0.001, 0.01, 0.1, 0.5, 0.99])
def test_logsr_momentum_unbiased(val):
    dm = math.log1p(1.0) / K_M
    _unbiased(val, dm, math.expm1(dm), K_M, lambda v: math.log1p(v) / dm,
              lambda q: torch.expm1(q * dm), 2e-3)


@pytest.mark.parametrize("frac", [0.01, 0.25, 0.5, 0.75, 0.99])
def test_logsr_preconditioner_unbiased(frac):
    eps = 1e-8
    w_min = 1.0 / (1.0 + eps)
    w_max = 1.0 / eps
    dw = math.log(w_max / w_min) / K_W
    w = w_min + frac * (w_max - w_min)
    _unbiased(w, dw, math.expm1(dw), K_W, lambda v: math.log(v / w_min) / dw,
              lambda q: w_min * torch.exp(q * dw), 1e-3)


def test_decode_momentum_known_answers():
    assert decode_momentum(torch.tensor([0], dtype=torch.int16), 1e-4).item() == 0.0
    assert (decode_momentum(torch.tensor([1, 100, K_M], dtype=torch.int16), 1e-4) > 0).all()
    assert (decode_momentum(torch.tensor([-1, -100], dtype=torch.int16), 1e-4) < 0).all()
    S_m = 2.5
    dm = math.log1p(S_m) / K_M
    assert decode_momentum(torch.tensor([K_M], dtype=torch.int16), dm).item() == pytest.approx(S_m, rel=1e-5)


def test_decode_preconditioner_range_and_zero_variance():
    eps = 1e-8
    w_min, _, _, dw, _ = precompute(1.0, 1.0, eps)
    lo = encode_uint16(torch.tensor([0], dtype=torch.int32))
    hi = encode_uint16(torch.tensor([K_W], dtype=torch.int32))
    assert decode_preconditioner(lo, w_min, dw).item() == pytest.approx(w_min, rel=1e-5)
    assert decode_preconditioner(hi, w_min, dw).item() == pytest.approx(1 / eps, rel=1e-3)
    w_min, _, _, dw, z_w = precompute(1.0, 0.0, eps)
    q = quantize_preconditioner(torch.zeros(16), eps, w_min, dw, z_w, torch.rand(16))
    assert dw == 0.0
    assert torch.allclose(decode_preconditioner(q, w_min, dw), torch.full((16,), 1 / eps))
