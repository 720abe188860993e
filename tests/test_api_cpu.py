"""LUMA front end without a GPU: validation (reference tests/test_basic.py:16-52)
and loud failure instead of any CPU fallback."""

import pytest
import torch
import torch.nn as nn

from luma_b200 import LUMA


def test_default_and_custom_params():
    m = nn.Linear(8, 4)
    assert LUMA(m.parameters()) is not None
    opt = LUMA(m.parameters(), lr=5e-4, betas=(0.95, 0.98), eps=1e-6, weight_decay=0.1)
    assert opt.defaults["lr"] == 5e-4


def test_invalid_backend():
    with pytest.raises(ValueError, match="Invalid backend"):
        LUMA(nn.Linear(8, 4).parameters(), backend="tritonn")
    with pytest.raises(ValueError, match="Invalid backend"):
        LUMA(nn.Linear(8, 4).parameters(), backend="pytorch")


@pytest.mark.parametrize("kwargs", [{"lr": -1}, {"eps": -1}, {"eps": 0}, {"betas": (1.0, 0.999)},
                                    {"betas": (0.9, -0.1)}, {"weight_decay": -0.01}])
def test_invalid_hyperparams(kwargs):
    with pytest.raises(ValueError):
        LUMA(nn.Linear(4, 2).parameters(), **kwargs)


def test_base_seed_from_global_rng():
    torch.manual_seed(7)
    a = LUMA(nn.Linear(2, 2).parameters())._base_seed
    torch.manual_seed(7)
    b = LUMA(nn.Linear(2, 2).parameters())._base_seed
    assert a == b and -(2 ** 63) <= a < 2 ** 63


def test_no_grad_step_is_noop():
    opt = LUMA(nn.Linear(8, 4).parameters())
    opt.step()
    assert opt.state_dict()["state"] == {}


def test_cpu_params_fail_loudly():
    m = nn.Linear(8, 4)
    opt = LUMA(m.parameters())
    m(torch.randn(2, 8)).sum().backward()
    with pytest.raises(RuntimeError, match="CUDA"):
        opt.step()
    assert len(opt.state) == 0  # validation happens before any state change


def test_dtype_and_sparse_validation():
    p = torch.zeros(4, dtype=torch.float64, requires_grad=True)
    p.grad = torch.zeros(4, dtype=torch.float64)
    with pytest.raises(ValueError, match="float32 or bfloat16"):
        LUMA([p]).step()
    emb = nn.Embedding(10, 4, sparse=True)
    opt = LUMA(emb.parameters())
    emb(torch.tensor([1, 2])).sum().backward()
    with pytest.raises(RuntimeError, match="sparse"):
        opt.step()


def test_closure_runs_before_validation():
    m = nn.Linear(4, 2)
    opt = LUMA(m.parameters())
    calls = []

    def closure():
        calls.append(1)
        return torch.tensor(0.0)

    loss = opt.step(closure)  # no grads: nothing to step
    assert calls == [1] and torch.is_tensor(loss)
