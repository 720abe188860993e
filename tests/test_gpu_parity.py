"""Parity of the CUDA backend with the reference algorithm (GPU).

Bit-exact bar: the oracle (``oracle/luma_ref.py``, the reference's op
sequence) run on CUDA tensors of the same B200 is what the reference's
PyTorch backend computes there.  Fed the same uniforms, the CUDA backend must
produce identical params, Q_m, Q_w and S_m/S_v at every step — with the
golden fixtures' injected uniforms, and with the backend's own Philox stream
(``oracle/philox.py`` restates it on the host).

Tolerance bar (cross-device): against the CPU reference goldens the GPU's
libm and CUDA's "tensor / scalar = tensor * fl32(1/scalar)" rule differ in the
last bit, so codes may move by one grid bin and params by a few ulp.
"""

import math

import numpy as np
import pytest
import torch

from golden_cases import GoldenCase, case_names
from oracle import philox
from oracle.luma_ref import OracleLUMA, decode_momentum, decode_preconditioner, precompute

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _luma():
    from luma_b200 import LUMA
    return LUMA


def _index_map(groups):
    return {id(p): k for k, p in enumerate(p for g in groups for p in g["params"])}


def _same_scale(a, b) -> bool:
    """Equal floats, or both NaN (a NaN grad makes the reference's scale NaN)."""
    return a == b or (math.isnan(a) and math.isnan(b))


def _assert_same_state(tag, opt, oracle, params, oparams, groups):
    """Kernel state of params[i] == oracle state of oparams[i] (codes, scales, step)."""
    sd = opt.state_dict()["state"]
    idx = _index_map(groups)
    for i, (p, op) in enumerate(zip(params, oparams)):
        st = opt.state.get(p)
        ost = oracle.state.get(id(op))
        assert (not st) == (not ost), f"{tag} param {i}: state presence differs"
        if not st:
            continue
        assert torch.equal(st["Q_m"], ost["Q_m"]), f"{tag} param {i}: Q_m differs ({(st['Q_m'] != ost['Q_m']).sum().item()} elems)"
        assert torch.equal(st["Q_w"], ost["Q_w"]), f"{tag} param {i}: Q_w differs ({(st['Q_w'] != ost['Q_w']).sum().item()} elems)"
        s = sd[idx[id(p)]]
        assert _same_scale(s["S_m"], ost["S_m"]) and _same_scale(s["S_v"], ost["S_v"]), \
            f"{tag} param {i}: scales differ ({s['S_m']}, {s['S_v']}) vs ({ost['S_m']}, {ost['S_v']})"
        assert s["step"] == ost["step"]


@pytest.mark.parametrize("name", case_names())
def test_golden_injected_bit_exact_vs_oracle_cuda(name):
    """Golden inputs and uniforms: CUDA kernels == reference op sequence on CUDA."""
    LUMA = _luma()
    case = GoldenCase(name)
    pk = case.make_params(DEV)
    po = case.make_params(DEV)
    gk, go = case.groups(pk), case.groups(po)
    opt = LUMA(gk)
    cur = {}
    opt._set_draw_hook(lambda pid, t, like: cur[pid])
    orc = OracleLUMA(go, draws=lambda pid, t, like: cur[pid])
    for s in range(1, case.steps + 1):
        case.set_grads(pk, s)
        case.set_grads(po, s)
        cur.clear()
        cur.update(case.draws(s, DEV))
        opt.step()
        orc.step()
        for i, (a, b) in enumerate(zip(pk, po)):
            assert torch.equal(a.detach(), b.detach()), (
                f"{name} step {s} param {i}: {(a != b).sum().item()} elements differ")
        _assert_same_state(f"{name} step {s}", opt, orc, pk, po, gk)


def _golden_state_dict(case, step, base_seed):
    """The CPU reference's optimizer state after `step` as a state dict in the
    optimizer's parameter order (group order)."""
    state = {}
    for k, i in enumerate(case.order):
        if f"qm_{step}_{i}" not in case.arr:
            continue
        exp = case.expected(step, i)
        shape = tuple(case.specs[i]["shape"])
        state[k] = {"step": exp["t"], "param_id": k, "Q_m": exp["qm"].reshape(shape),
                    "Q_w": exp["qw"].reshape(shape), "S_m": exp["S"][0], "S_v": exp["S"][1]}
    groups, pos = [], 0
    for gi, g in enumerate(case.meta["groups"]):
        n = sum(1 for i in case.order if case.specs[i]["group"] == gi)
        groups.append(dict(lr=g["lr"], betas=tuple(g["betas"]), eps=g["eps"],
                           weight_decay=g["weight_decay"], params=list(range(pos, pos + n))))
        pos += n
    return {"state": state, "param_groups": groups, "_base_seed": base_seed}


@pytest.mark.parametrize("name", case_names())
def test_golden_cross_device_one_bin(name):
    """CUDA backend vs the CPU reference goldens, one step at a time: every
    step starts from the CPU reference's own params and state of the step
    before (so differences cannot accumulate), takes the same grads and
    uniforms, and must land within one grid bin of the reference's codes and
    within 1e-6 of max|p| of its params (bf16 params: one bf16 rounding).
    The bits may differ because the CPU's libm and its true-division rule for
    "tensor / scalar" differ from CUDA's in the last place."""
    LUMA = _luma()
    case = GoldenCase(name)
    for s in range(1, case.steps + 1):
        if s == 1:
            pk = case.make_params(DEV)
        else:
            pk = []
            for i, spec in enumerate(case.specs):
                t = case.expected(s - 1, i)["p"].to(DEV)
                t.requires_grad_(True)
                t.grad_dtype = None
                pk.append(t)
        opt = LUMA(case.groups(pk))
        if s > 1:
            opt.load_state_dict(_golden_state_dict(case, s - 1, case.base_seed))
        cur = case.draws(s, DEV)
        opt._set_draw_hook(lambda pid, t, like: cur[pid])
        case.set_grads(pk, s)
        opt.step()
        for i, p in enumerate(pk):
            exp = case.expected(s, i)
            got = p.detach().float().cpu()
            want = exp["p"].float()
            tol = 1e-6 * want.abs().max().item() + 1e-12
            if p.dtype == torch.bfloat16:
                tol = max(tol, 2 ** -7 * want.abs().max().item())
            assert (got - want).abs().max().item() <= tol, (name, s, i)
            if "qm" in exp:
                st = opt.state[p]
                assert st["step"] == exp["t"]
                dq_m = (st["Q_m"].cpu().int().reshape(-1) - exp["qm"].int().reshape(-1)).abs()
                qw_k = st["Q_w"].cpu().int().reshape(-1) & 0xFFFF
                qw_r = exp["qw"].int().reshape(-1) & 0xFFFF
                dq_w = (qw_k - qw_r).abs()
                assert dq_m.max().item() <= 1, (name, s, i, dq_m.max().item())
                assert dq_w.max().item() <= 1, (name, s, i, dq_w.max().item())


def _philox_draws(opt):
    def draws(pid, t, like):
        seed = philox.step_seed(opt._base_seed, t, pid)
        um, uw = philox.uniforms(seed, like.numel())
        return (torch.from_numpy(um).reshape(like.shape).to(like.device),
                torch.from_numpy(uw).reshape(like.shape).to(like.device))
    return draws


def _run_pair(shapes, pdt, gdts, steps, seed=0, gscale=1e-2, lr=1e-3, offsets=None):
    """Step the CUDA backend (Philox) and the oracle (host Philox draws) side by side."""
    LUMA = _luma()
    g = torch.Generator(device="cpu").manual_seed(seed)
    pk, po = [], []
    for k, shp in enumerate(shapes):
        base = torch.randn(shp, generator=g) * 0.02
        off = 0 if offsets is None else offsets[k]
        if off:
            # a view at an element offset: exercises the unaligned (scalar) path
            buf = torch.zeros(base.numel() + off, dtype=pdt, device=DEV)
            t = buf[off:].view(shp)
            t.copy_(base.to(pdt))
        else:
            t = base.to(pdt).to(DEV)
        pk.append(t)
        po.append(base.to(pdt).to(DEV))
    for t in pk + po:
        t.grad_dtype = None  # grads may differ in dtype from the param
    opt = LUMA(pk, lr=lr)
    orc = OracleLUMA(po, lr=lr, draws=_philox_draws(opt))
    for s in range(steps):
        for k, shp in enumerate(shapes):
            gd = gdts[k % len(gdts)]
            gr = (torch.randn(shp, generator=g) * gscale).to(gd).to(DEV)
            pk[k].grad = gr.clone()
            po[k].grad = gr.clone()
        opt.step()
        orc.step()
        for k, (a, b) in enumerate(zip(pk, po)):
            assert torch.equal(a.detach(), b.detach()), (
                f"step {s + 1} tensor {k} {tuple(shapes[k])}: {(a != b).sum().item()} differ")
        _assert_same_state(f"step {s + 1}", opt, orc, pk, po, [{"params": pk}])
    return opt, pk


@pytest.mark.parametrize("numel", [1, 7, 8, 9, 1023, 1025, 2048 * 3 + 5, (1 << 20) + 3])
def test_philox_bit_exact_sizes(numel):
    _run_pair([(numel,)], torch.float32, [torch.float32], steps=3)


@pytest.mark.parametrize("pdt", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("gdt", [torch.float32, torch.bfloat16, torch.float16])
def test_philox_bit_exact_dtypes(pdt, gdt):
    _run_pair([(257, 129), (4096,)], pdt, [gdt], steps=3, gscale=1e-3)


def test_unaligned_views_bit_exact():
    shapes = [(1000,), (77, 13), (4096,)]
    _run_pair(shapes, torch.float32, [torch.float32, torch.bfloat16], steps=3, offsets=[1, 3, 0])


def test_ragged_many_tensors_bit_exact():
    rng = np.random.default_rng(0)
    sizes = [int(round(2 ** rng.uniform(0, 14))) for _ in range(300)]
    _run_pair([(n,) for n in sizes], torch.float32, [torch.float32, torch.bfloat16], steps=2)


def test_large_tensor_across_many_ctas_bit_exact():
    """One tensor split over every CTA of the persistent grid plus small ones."""
    _run_pair([(5_000_003,), (3,), (70_001,)], torch.bfloat16, [torch.bfloat16], steps=2, gscale=1e-3)


@pytest.mark.parametrize("pdt", [torch.float32, torch.bfloat16])
def test_long_segments_decode_table_bit_exact(pdt):
    """Segments long enough for the decode table on every CTA (the steady-state
    pass-2 loop), one tensor per grad dtype, ragged lengths."""
    _run_pair([(12_000_011,), (11_999_993,), (12_000_000,)], pdt,
              [torch.float32, torch.float16, torch.bfloat16], steps=3, gscale=1e-3)


def test_branch_free_arithmetic_matches_ieee():
    """The steady loop's reciprocal, square root and quotient equal CUDA's
    IEEE intrinsics on 2^28 random operands each over their ranges of use."""
    from luma_b200 import _lib
    assert _lib.arith_selfcheck(1 << 28, seed=7) == (0, 0, 0)


def test_long_segments_rare_elements_bit_exact():
    """A long tensor (steady-state loop on every CTA) whose grads hold zeros,
    subnormals and tiny values in scattered elements: their m' / v' fall below
    the range of the branch-free arithmetic, so their pairs take the exact
    recomputation; the other pairs stay on the steady loop."""
    LUMA = _luma()
    n = 20_000_003
    gen = torch.Generator().manual_seed(11)
    pk = [(torch.randn(n, generator=gen) * 0.02).to(DEV)]
    po = [pk[0].clone()]
    opt = LUMA(pk, lr=1e-3)
    orc = OracleLUMA(po, lr=1e-3, draws=_philox_draws(opt))
    for step in range(1, 4):
        g = torch.randn(n, generator=gen) * 1e-3
        idx = torch.randint(0, n, (n // 50,), generator=gen)
        kind = torch.randint(0, 3, idx.shape, generator=gen)
        g[idx[kind == 0]] = 0.0
        g[idx[kind == 1]] = 1e-41
        g[idx[kind == 2]] = -3e-30
        pk[0].grad = g.to(DEV)
        po[0].grad = g.to(DEV)
        opt.step()
        orc.step()
        assert torch.equal(pk[0], po[0]), f"step {step}: {(pk[0] != po[0]).sum().item()} params differ"
        _assert_same_state(f"step {step}", opt, orc, pk, po, [{"params": pk}])


@pytest.mark.parametrize("pdt", [torch.float32, torch.bfloat16])
def test_nan_and_huge_grads_bit_exact(pdt):
    """A NaN grad poisons its tensor's scales exactly as the reference's ops
    do; a huge finite grad (v' ~ 1e33) moves its segment off the steady loop's
    verified range; the other tensors are unaffected.  (An infinite grad makes
    the reference's _precompute raise ZeroDivisionError, functional.py:74-92;
    the device step cannot raise and stores the non-finite grid instead.)"""
    LUMA = _luma()
    gen = torch.Generator().manual_seed(12)
    shapes = [(3000,), (20_000_001,), (777,)]
    base = [(torch.randn(s, generator=gen) * 0.02).to(pdt) for s in shapes]
    pk = [b.clone().to(DEV) for b in base]
    po = [b.clone().to(DEV) for b in base]
    for t in pk + po:
        t.grad_dtype = None
    opt = LUMA(pk, lr=1e-3)
    orc = OracleLUMA(po, lr=1e-3, draws=_philox_draws(opt))
    for step in range(1, 4):
        for k, shp in enumerate(shapes):
            g = torch.randn(shp, generator=gen) * 1e-3
            if k == 0 and step >= 2:
                g[5] = float("nan")
            if k == 1 and step >= 2:
                g[123_456] = 1e18
            pk[k].grad = g.to(DEV)
            po[k].grad = g.to(DEV)
        opt.step()
        orc.step()
        for k in range(len(shapes)):
            a, b = pk[k].view(torch.int16 if pdt == torch.bfloat16 else torch.int32), \
                po[k].view(torch.int16 if pdt == torch.bfloat16 else torch.int32)
            assert torch.equal(a, b), f"step {step} tensor {k}: {(a != b).sum().item()} param bit patterns differ"
        _assert_same_state(f"step {step}", opt, orc, pk, po, [{"params": pk}])


def test_export_decode_bit_exact():
    opt, pk = _run_pair([(3000,), (64, 64)], torch.float32, [torch.float32], steps=3)
    exp = opt.export_adamw_state()
    sd = opt.state_dict()
    for k, p in enumerate(pk):
        st = sd["state"][k]
        w_min, delta_m, _, delta_w, _ = precompute(st["S_m"], st["S_v"], 1e-8)
        m = decode_momentum(st["Q_m"], delta_m)
        w = decode_preconditioner(st["Q_w"], w_min, delta_w)
        v = (1.0 / w - 1e-8).clamp(min=0).square()
        assert torch.equal(exp["state"][k]["exp_avg"], m)
        assert torch.equal(exp["state"][k]["exp_avg_sq"], v)


def _crafted_grads(step, n, kind, gen):
    """Gradients that stress the pass-1 maximum search (ties, near-ties,
    zeros, subnormals, isolated spikes, sign flips)."""
    base = torch.randn(n, generator=gen) * 1e-2
    if kind == "const":
        return torch.full((n,), 3e-3)
    if kind == "ulp_ties":
        c = torch.full((n,), 2.5e-3)
        bits = c.view(torch.int32) + torch.arange(n, dtype=torch.int32) % 5
        return bits.view(torch.float32)
    if kind == "zeros":
        return torch.zeros(n)
    if kind == "subnormal":
        return torch.randn(n, generator=gen) * 1e-41
    if kind == "spike_last":
        base[-1] = 7.0
        return base
    if kind == "spike_first":
        base[0] = -7.0
        return base
    if kind == "flip":
        return torch.full((n,), 1e-2 * (-1.0) ** step) + base * 1e-4
    if kind == "quad_spikes":
        # maxima at every offset within a 4-element quad, both signs; at step
        # 4 the largest v' (an earlier spike's, decaying slowly) and the
        # largest |m'| (a new, smaller spike) sit in different elements
        a = 4 * (n // 12) + 2                       # offset 2
        if step == 1:
            base[4 * (n // 20)] = 1.5               # offset 0
        if step == 2:
            base[a] = 3.0
        if step >= 3:
            base[a] = 0.0
            base[a + 4 * 1009 + 1] = -0.37 * step   # offset 3
        if step == 4:
            base[a + 4 * 1009 - 1] = -2.6           # offset 1
        return base
    raise ValueError(kind)


@pytest.mark.parametrize("beta1", [0.9, 0.0])
def test_scale_max_adversarial_bit_exact(beta1):
    LUMA = _luma()
    kinds = ["const", "ulp_ties", "zeros", "subnormal", "spike_last", "spike_first", "flip"]
    sizes = [4099, 70_003, 1_000_001]
    gen = torch.Generator().manual_seed(3)
    shapes = [(n,) for n in sizes for _ in kinds]
    pk = [(torch.randn(s, generator=gen) * 0.02).to(DEV) for s in shapes]
    po = [t.clone() for t in pk]
    opt = LUMA(pk, lr=1e-3, betas=(beta1, 0.999))
    orc = OracleLUMA(po, lr=1e-3, betas=(beta1, 0.999), draws=_philox_draws(opt))
    for step in range(1, 5):
        k = 0
        for n in sizes:
            for kind in kinds:
                g = _crafted_grads(step, n, kind, gen).to(DEV)
                pk[k].grad = g.clone()
                po[k].grad = g.clone()
                k += 1
        opt.step()
        orc.step()
        for i, (a, b) in enumerate(zip(pk, po)):
            assert torch.equal(a, b), f"step {step} tensor {i} ({kinds[i % len(kinds)]})"
        _assert_same_state(f"step {step}", opt, orc, pk, po, [{"params": pk}])


@pytest.mark.parametrize("gdt", [torch.bfloat16, torch.float32])
def test_scale_max_adversarial_long_segments_bit_exact(gdt):
    """The crafted grads on tensors long enough for the decode and bucket
    tables on every CTA, where pass 1 bounds |m'| and v' once per quad of 4
    elements and skips quads that cannot raise the maxima: ties (bound equal
    to the running maximum), all-zero and subnormal grads, spikes at every
    offset within a quad, a maximum of v' apart from the maximum of |m'|."""
    LUMA = _luma()
    kinds = ["ulp_ties", "zeros", "subnormal", "quad_spikes"]
    n = 20_000_011
    gen = torch.Generator().manual_seed(5)
    pk = [(torch.randn(n, generator=gen) * 0.02).to(DEV) for _ in kinds]
    po = [t.clone() for t in pk]
    for t in pk + po:
        t.grad_dtype = None
    opt = LUMA(pk, lr=1e-3)
    orc = OracleLUMA(po, lr=1e-3, draws=_philox_draws(opt))
    for step in range(1, 5):
        for k, kind in enumerate(kinds):
            g = _crafted_grads(step, n, kind, gen).to(gdt).to(DEV)
            pk[k].grad = g.clone()
            po[k].grad = g.clone()
        opt.step()
        orc.step()
        for i, (a, b) in enumerate(zip(pk, po)):
            assert torch.equal(a, b), f"step {step} tensor {i} ({kinds[i]})"
        _assert_same_state(f"step {step}", opt, orc, pk, po, [{"params": pk}])


@pytest.mark.parametrize("pdt,gdt", [(torch.float32, torch.float32), (torch.float32, torch.bfloat16),
                                     (torch.float32, torch.float16), (torch.bfloat16, torch.bfloat16)])
@pytest.mark.parametrize("max_norm", [1e-3, 1e9])
def test_fused_clip_bit_exact(pdt, gdt, max_norm):
    """clip_grad_norm_ then step == step(grad_scale=clip_grad_coef(...)) bit
    for bit (the reference clips before every step, bench_nanogpt.py:218-225),
    with clipping active (max_norm 1e-3) and inactive (coefficient 1); one
    tensor long enough for the steady loops."""
    from luma_b200 import LUMA, clip_grad_coef
    shapes = [(20_000_003,), (4096, 3), (1000,), (7,)]
    gen = torch.Generator().manual_seed(21)
    base = [(torch.randn(s, generator=gen) * 0.02).to(pdt) for s in shapes]
    pa = [b.clone().to(DEV) for b in base]
    pb = [b.clone().to(DEV) for b in base]
    for t in pa + pb:
        t.grad_dtype = None
    torch.manual_seed(5)
    oa = LUMA(pa, lr=1e-3)
    torch.manual_seed(5)
    ob = LUMA(pb, lr=1e-3)
    for step in range(1, 4):
        for k, s in enumerate(shapes):
            g = (torch.randn(s, generator=gen) * 1e-2).to(gdt).to(DEV)
            pa[k].grad = g.clone()
            pb[k].grad = g.clone()
        torch.nn.utils.clip_grad_norm_(pa, max_norm)
        oa.step()
        gb = [p.grad.clone() for p in pb]
        _, coef = clip_grad_coef(pb, max_norm)
        ob.step(grad_scale=coef)
        for k in range(len(shapes)):
            assert torch.equal(pb[k].grad, gb[k]), "grads must not be modified"
            assert torch.equal(pa[k], pb[k]), f"step {step} param {k}: {(pa[k] != pb[k]).sum().item()} differ"
            sa, sb = oa.state[pa[k]], ob.state[pb[k]]
            assert torch.equal(sa["Q_m"], sb["Q_m"]) and torch.equal(sa["Q_w"], sb["Q_w"])
        da, db = oa.state_dict()["state"], ob.state_dict()["state"]
        for k in da:
            assert (da[k]["S_m"], da[k]["S_v"]) == (db[k]["S_m"], db[k]["S_v"])
