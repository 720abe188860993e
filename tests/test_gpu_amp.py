"""``GradScaler.unscale_`` and the inf/NaN skip fused into the step (GPU).

Reference usage: an fp16 autocast loop with ``torch.amp.GradScaler`` around
``LUMA`` (tests/test_mixed_precision.py:119-184): ``scaler.scale(loss)
.backward(); scaler.step(opt); scaler.update()``, where ``scaler.step``
unscales every grad in a separate pass and skips ``opt.step()`` after an
inf/NaN grad.  ``luma_b200.amp.scaler_step`` does the unscale and the check
inside the step's own passes; params, codes, scales, step counts and the
scaler's scale must stay bit-identical to the unfused loop, through steps
that overflow (the first step included) and steps that do not.
"""

import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _model(seed):
    torch.manual_seed(seed)
    m = torch.nn.Sequential(torch.nn.Linear(64, 512), torch.nn.GELU(), torch.nn.Linear(512, 64),
                            torch.nn.GELU(), torch.nn.Linear(64, 2000)).to(DEV)
    big = torch.nn.Parameter(torch.randn(3_000_000, device=DEV) * 0.02)  # steady-loop sized
    return m, big


def _loss(m, big, x, y):
    with torch.autocast("cuda", dtype=torch.float16):
        out = m(x)
        return torch.nn.functional.mse_loss(out.float(), y) + (big[:2000] * out.float()).mean()


@pytest.mark.parametrize("capturable", [False])
def test_scaler_step_fused_bit_exact_with_skips(capturable):
    from luma_b200 import LUMA
    from luma_b200.amp import scaler_step
    ma, ba = _model(0)
    mb, bb = _model(0)
    pa = list(ma.parameters()) + [ba]
    pb = list(mb.parameters()) + [bb]
    torch.manual_seed(9)
    oa = LUMA(pa, lr=1e-3)
    torch.manual_seed(9)
    ob = LUMA(pb, lr=1e-3)
    sa = torch.amp.GradScaler("cuda", init_scale=2.0 ** 32, backoff_factor=0.25,
                              growth_interval=2)
    sb = torch.amp.GradScaler("cuda", init_scale=2.0 ** 32, backoff_factor=0.25,
                              growth_interval=2)
    gen = torch.Generator(device=DEV).manual_seed(1)
    skipped = stepped = 0
    for it in range(18):
        x = torch.randn(256, 64, device=DEV, generator=gen)
        y = torch.randn(256, 2000, device=DEV, generator=gen)
        for m, big, opt, sc in ((ma, ba, oa, sa), (mb, bb, ob, sb)):
            opt.zero_grad(set_to_none=True)
            sc.scale(_loss(m, big, x, y)).backward()
        before = sa.get_scale()
        sa.step(oa)
        scaler_step(sb, ob)
        sa.update()
        sb.update()
        skipped += sa.get_scale() < before
        stepped += sa.get_scale() >= before
        assert sa.get_scale() == sb.get_scale(), f"iteration {it}: scales of the scalers differ"
        for k, (a, b) in enumerate(zip(pa, pb)):
            assert torch.equal(a, b), f"iteration {it} param {k}"
            st_a, st_b = oa.state.get(a, {}), ob.state.get(b, {})
            assert ("step" in st_a) == ("step" in st_b), f"iteration {it} param {k}: state"
            if "step" in st_a:
                assert st_a["step"] == st_b["step"]
                assert torch.equal(st_a["Q_m"], st_b["Q_m"]) and torch.equal(st_a["Q_w"], st_b["Q_w"])
        da, db = oa.state_dict()["state"], ob.state_dict()["state"]
        assert da.keys() == db.keys()
        for k in da:
            assert (da[k]["S_m"], da[k]["S_v"]) == (db[k]["S_m"], db[k]["S_v"])
    assert skipped >= 2 and stepped >= 4, (skipped, stepped)


def test_preset_found_inf_changes_nothing():
    """A flag already set by the caller (another check) skips the step."""
    from luma_b200 import LUMA
    p = torch.randn(1_000_003, device=DEV) * 0.02
    opt = LUMA([p], lr=1e-3)
    p.grad = torch.randn_like(p) * 1e-3
    opt.step()
    p.grad = torch.randn_like(p) * 1e-3
    opt.step()
    snap = (p.clone(), opt.state[p]["Q_m"].clone(), opt.state[p]["Q_w"].clone(),
            opt.state_dict()["state"][0])
    flag = torch.ones((), device=DEV)
    opt.step(found_inf=flag)
    assert torch.equal(p, snap[0])
    assert torch.equal(opt.state[p]["Q_m"], snap[1]) and torch.equal(opt.state[p]["Q_w"], snap[2])
    sd = opt.state_dict()["state"][0]
    assert sd["step"] == 2 and (sd["S_m"], sd["S_v"]) == (snap[3]["S_m"], snap[3]["S_v"])
    # and a clean flag lets the step run
    flag.zero_()
    opt.step(found_inf=flag)
    assert flag.item() == 0.0 and opt.state[p]["step"] == 3 and not torch.equal(p, snap[0])


def test_nonfinite_grad_raises_flag_and_skips():
    from luma_b200 import LUMA
    ps = [torch.randn(n, device=DEV) * 0.02 for n in (5000, 2_000_001)]
    opt = LUMA(ps, lr=1e-3)
    for p in ps:
        p.grad = torch.randn_like(p) * 1e-3
    opt.step()
    snap = [p.clone() for p in ps]
    for bad in (float("inf"), float("-inf"), float("nan")):
        for p in ps:
            p.grad = torch.randn_like(p) * 1e-3
        ps[1].grad[1_234_567] = bad
        flag = torch.zeros((), device=DEV)
        opt.step(found_inf=flag)
        assert flag.item() == 1.0
        assert all(torch.equal(p, s) for p, s in zip(ps, snap))
        assert all(opt.state[p]["step"] == 1 for p in ps)
