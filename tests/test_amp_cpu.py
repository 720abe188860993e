"""Dispatch logic of ``luma_b200.amp.scaler_step`` on CPU (no kernels run).

The fused path passes ``grad_scale = fl32(1/scale)`` (the reciprocal taken in
float64, as ``GradScaler.unscale_`` computes it) and a zeroed ``found_inf``
flag to the optimizer's step, and records the flag in the scaler's
per-optimizer state so that ``scaler.update()`` works as after
``scaler.step``; the other cases fall back to ``scaler.step`` or to a plain
step exactly as ``GradScaler.step`` would behave.
"""

import pytest
import torch
from torch.amp.grad_scaler import OptState

from luma_b200.amp import scaler_step


class FakeLUMA(torch.optim.Optimizer):
    """Records the keyword arguments of every step; never touches params."""

    def __init__(self, params):
        super().__init__(params, {})
        self.calls = []

    def step(self, closure=None, *, grad_scale=None, found_inf=None):
        self.calls.append((grad_scale, found_inf))


def _setup(grad_dtype=torch.float32):
    p = torch.nn.Parameter(torch.zeros(4))
    p.grad_dtype = None  # grads of another dtype than the param are allowed
    p.grad = torch.ones(4, dtype=grad_dtype)
    return p, FakeLUMA([p])


def _scaler(**kw):
    s = torch.amp.GradScaler("cpu", **kw)
    s.scale(torch.ones(()))  # as scaler.scale(loss) does before backward
    return s


def test_fused_path_passes_inverse_scale_and_flag():
    p, opt = _setup()
    scaler = _scaler(init_scale=3.0)
    scaler_step(scaler, opt)
    (gs, fi), = opt.calls
    assert gs.dtype == torch.float32 and gs.item() == torch.tensor(1.0 / 3.0, dtype=torch.float64).float().item()
    assert fi.dtype == torch.float32 and fi.item() == 0.0
    st = scaler._per_optimizer_states[id(opt)]
    assert st["stage"] is OptState.STEPPED and list(st["found_inf_per_device"].values()) == [fi]
    scaler.update()  # no growth on the first step, no error
    assert scaler.get_scale() == 3.0


def test_found_flag_backs_off_the_scale():
    p, opt = _setup()

    class Flagging(FakeLUMA):
        def step(self, closure=None, *, grad_scale=None, found_inf=None):
            found_inf.fill_(1.0)  # the kernels saw an inf grad

    opt = Flagging([p])
    scaler = _scaler(init_scale=8.0, backoff_factor=0.5)
    scaler_step(scaler, opt)
    scaler.update()
    assert scaler.get_scale() == 4.0


def test_disabled_scaler_plain_step_and_fp16_grads_refused():
    p, opt = _setup()
    scaler_step(_scaler(enabled=False), opt)
    assert opt.calls == [(None, None)]
    p16, opt16 = _setup(torch.float16)
    with pytest.raises(ValueError, match="FP16"):
        scaler_step(_scaler(), opt16)


def test_second_step_before_update_is_an_error():
    p, opt = _setup()
    scaler = _scaler()
    scaler_step(scaler, opt)
    with pytest.raises(RuntimeError, match="already been called"):
        scaler_step(scaler, opt)
