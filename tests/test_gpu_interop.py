"""A checkpoint written by the unmodified reference continues on this backend (GPU).

``tests/golden/ref_checkpoint.pt`` holds the ``state_dict()`` of the
reference's ``LUMA(backend="pytorch")`` after three CPU training steps (two
param groups, written by ``tests/golden/make_ref_checkpoint.py``), the params at
that point and the grads of three more steps.  The reference pins the same
kind of cross-backend load for its own two backends
(tests/test_state_dict.py:653-699).

Loaded into ``luma_b200.LUMA`` on CUDA, the state must read back unchanged,
and the next three steps must equal, bit for bit, the reference's algorithm
(the oracle, on CUDA) continuing from the same state with the same uniforms.
"""

import os

import pytest
import torch

from oracle import philox
from oracle.luma_ref import OracleLUMA

pytestmark = pytest.mark.gpu

DEV = "cuda"
FIXTURE = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "ref_checkpoint.pt")


def _setup():
    from luma_b200 import LUMA
    d = torch.load(FIXTURE)
    params = [p.clone().to(DEV) for p in d["params"]]
    oparams = [p.clone().to(DEV) for p in d["params"]]

    def groups(ps):
        return [dict(params=[p for p, gi in zip(ps, d["group_of"]) if gi == k], **hp)
                for k, hp in enumerate(d["groups"])]
    opt = LUMA(groups(params))
    opt.load_state_dict(d["state_dict"])
    return d, opt, params, oparams, groups


def test_reference_checkpoint_reads_back_unchanged():
    d, opt, params, _, _ = _setup()
    ref = d["state_dict"]
    got = opt.state_dict()
    assert got["_base_seed"] == ref["_base_seed"]
    assert [{k: v for k, v in g.items()} for g in got["param_groups"]] == ref["param_groups"]
    assert set(got["state"]) == set(ref["state"])
    for k, st in ref["state"].items():
        g = got["state"][k]
        assert set(g) == set(st)
        assert g["step"] == st["step"] and g["param_id"] == st["param_id"]
        assert (g["S_m"], g["S_v"]) == (st["S_m"], st["S_v"])
        assert torch.equal(g["Q_m"].cpu(), st["Q_m"]) and torch.equal(g["Q_w"].cpu(), st["Q_w"])


def test_reference_checkpoint_continues_bit_exact_vs_oracle():
    d, opt, params, oparams, groups = _setup()
    ref = d["state_dict"]
    ogroups = groups(oparams)
    orc = OracleLUMA(ogroups, draws=lambda pid, t, like: tuple(
        u.view(like.shape) for u in philox.uniforms_torch(
            philox.step_seed(opt._base_seed, t, pid), like.numel(), device=DEV)))
    # the oracle starts from the same reference state
    order = [p for g in ogroups for p in g["params"]]
    for k, p in enumerate(order):
        st = ref["state"][k]
        orc.state[id(p)] = {"step": st["step"], "param_id": st["param_id"],
                            "Q_m": st["Q_m"].to(DEV), "Q_w": st["Q_w"].to(DEV),
                            "S_m": st["S_m"], "S_v": st["S_v"]}
    korder = [p for g in opt.param_groups for p in g["params"]]
    for s, grads in enumerate(d["grads"], start=4):
        for p, q, g in zip(params, oparams, grads):
            p.grad = g.to(DEV)
            q.grad = g.to(DEV)
        opt.step()
        orc.step()
        sd = opt.state_dict()["state"]
        for k, (kp, op) in enumerate(zip(korder, order)):
            assert torch.equal(kp, op), f"step {s} param {k}"
            ost = orc.state[id(op)]
            assert torch.equal(opt.state[kp]["Q_m"], ost["Q_m"]), f"step {s} Q_m {k}"
            assert torch.equal(opt.state[kp]["Q_w"], ost["Q_w"]), f"step {s} Q_w {k}"
            assert (sd[k]["S_m"], sd[k]["S_v"]) == (ost["S_m"], ost["S_v"]), f"step {s} scales {k}"
            assert sd[k]["step"] == ost["step"] == s
