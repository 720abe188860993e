"""Pin the oracle to the reference: replaying every golden fixture through
``oracle.luma_ref.OracleLUMA`` on CPU must reproduce the reference's params,
codes and scales bit for bit (same torch CPU ops, same injected uniforms)."""

import pytest
import torch

from golden_cases import GoldenCase, case_names
from oracle.luma_ref import OracleLUMA


@pytest.mark.parametrize("name", case_names())
def test_oracle_matches_reference_goldens(name):
    case = GoldenCase(name)
    params = case.make_params("cpu")
    cur = {}

    def draws(param_id, step, like):
        return cur[param_id]

    opt = OracleLUMA(case.groups(params), draws=draws)
    for s in range(1, case.steps + 1):
        case.set_grads(params, s)
        cur.clear()
        cur.update(case.draws(s, "cpu"))
        opt.step()
        for i, p in enumerate(params):
            exp = case.expected(s, i)
            assert torch.equal(p.detach(), exp["p"]), f"{name} step {s} param {i}"
            if "qm" in exp:
                st = opt.state_of(p)
                assert torch.equal(st["Q_m"].reshape(-1), exp["qm"].reshape(-1)), (name, s, i)
                assert torch.equal(st["Q_w"].reshape(-1), exp["qw"].reshape(-1)), (name, s, i)
                assert (st["S_m"], st["S_v"]) == exp["S"], (name, s, i)
                assert st["step"] == exp["t"]


def test_golden_fixtures_present():
    names = case_names()
    assert len(names) >= 8
    assert {"basic_f32", "param_bf16", "zero_and_outliers", "ragged"} <= set(names)
