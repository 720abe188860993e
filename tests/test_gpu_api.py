"""The reference's API-level test suites, run against the CUDA backend (GPU).

Mirrors IgorYashch/LUMA tests/test_basic.py, test_state_dict.py,
test_determinism.py, test_convergence.py and test_correctness.py
(tracking and LogSR unbiasedness), with bars at least as strict as the
reference's: checkpoint resume and determinism are bitwise (torch.equal),
which the reference's Triton backend only met to 1e-5.
"""

import math
import random

import pytest
import torch
import torch.nn as nn

from oracle import philox
from oracle.luma_ref import (K_M, K_W, precompute, quantize_momentum,
                             quantize_preconditioner)

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")


def LUMA(*a, **k):
    from luma_b200 import LUMA as _L
    return _L(*a, **k)


def seed_all(s=42):
    random.seed(s)
    torch.manual_seed(s)
    torch.cuda.manual_seed_all(s)


def quadratic(d):
    a = torch.rand(d, device=DEV) + 0.5
    b = torch.randn(d, device=DEV)
    return lambda x: 0.5 * (a * (x - b).square()).sum()


def train(opt, x, loss_fn, n):
    loss = None
    for _ in range(n):
        opt.zero_grad()
        loss = loss_fn(x)
        loss.backward()
        opt.step()
    return loss.item()


def fixed_grad_steps(opt, x, g, n):
    for _ in range(n):
        opt.zero_grad()
        x.grad = g.clone()
        opt.step()


# ---- test_basic.py -----------------------------------------------------------

class TestStepping:
    def test_single_and_multiple_steps(self):
        m = nn.Linear(8, 4).to(DEV)
        opt = LUMA(m.parameters())
        for _ in range(10):
            m(torch.randn(2, 8, device=DEV)).sum().backward()
            opt.step()
            opt.zero_grad()
        assert all(p.isfinite().all() for p in m.parameters())

    def test_no_grad_param_skipped(self):
        m = nn.Linear(8, 4).to(DEV)
        opt = LUMA(m.parameters())
        opt.step()
        assert len(opt.state) == 0

    def test_sparse_grad_rejected(self):
        emb = nn.Embedding(10, 4, sparse=True).to(DEV)
        opt = LUMA(emb.parameters())
        emb(torch.tensor([1, 2], device=DEV)).sum().backward()
        with pytest.raises(RuntimeError, match="sparse"):
            opt.step()

    def test_closure(self):
        m = nn.Linear(4, 2).to(DEV)
        opt = LUMA(m.parameters())
        x = torch.randn(2, 4, device=DEV)

        def closure():
            opt.zero_grad()
            loss = m(x).sum()
            loss.backward()
            return loss

        assert torch.is_tensor(opt.step(closure))

    def test_lr_zero_no_update(self):
        m = nn.Linear(8, 4).to(DEV)
        opt = LUMA(m.parameters(), lr=0.0, weight_decay=0.0)
        before = [p.data.clone() for p in m.parameters()]
        m(torch.randn(2, 8, device=DEV)).sum().backward()
        opt.step()
        for p, b in zip(m.parameters(), before):
            assert torch.equal(p.data, b)

    def test_scalar_parameter(self):
        x = torch.tensor(5.0, device=DEV, requires_grad=True)
        opt = LUMA([x], lr=1e-2)
        for _ in range(5):
            opt.zero_grad()
            (x ** 2).backward()
            opt.step()
        assert x.item() < 5.0

    def test_gradient_accumulation_and_zero_grad_modes(self):
        m = nn.Linear(8, 4).to(DEV)
        opt = LUMA(m.parameters(), lr=1e-3)
        before = [p.data.clone() for p in m.parameters()]
        for _ in range(3):
            m(torch.randn(2, 8, device=DEV)).sum().backward()
        opt.step()
        assert all(not torch.equal(p.data, b) for p, b in zip(m.parameters(), before))
        opt.zero_grad(set_to_none=False)
        assert all(p.grad is not None and (p.grad == 0).all() for p in m.parameters())
        m(torch.randn(2, 8, device=DEV)).sum().backward()
        opt.step()
        opt.zero_grad(set_to_none=True)
        assert all(p.grad is None for p in m.parameters())
        m(torch.randn(2, 8, device=DEV)).sum().backward()
        opt.step()
        assert all(p.isfinite().all() for p in m.parameters())

    def test_state_dtypes_shapes_device_and_4_bytes_per_param(self):
        m = nn.Linear(256, 256, bias=False).to(DEV)
        opt = LUMA(m.parameters())
        m(torch.randn(1, 256, device=DEV)).sum().backward()
        opt.step()
        for p in m.parameters():
            s = opt.state[p]
            for k in ("Q_m", "Q_w"):
                assert s[k].dtype == torch.int16 and s[k].shape == p.shape and s[k].is_cuda
            assert s["Q_m"].numel() * 2 + s["Q_w"].numel() * 2 == 4 * p.numel()

    def test_noncontiguous_grad_rejected(self):
        x = torch.randn(8, 8, device=DEV, requires_grad=True)
        opt = LUMA([x])
        x.grad = torch.randn(8, 8, device=DEV).t()
        with pytest.raises(ValueError, match="contiguous gradients"):
            opt.step()

    def test_param_storage_or_layout_changed_between_steps(self):
        """The step keeps per-param checks while a param keeps its storage,
        size and dtype; a param whose data is replaced (new storage), made
        non-contiguous, or whose grads switch dtype between steps is handled
        as on the first step: same results as an optimizer that never saw
        the old tensors, or the same error."""
        seed_all(7)
        a = nn.Parameter(torch.randn(3000, device=DEV) * 0.02)
        b = nn.Parameter(a.detach().clone())
        opt_a, opt_b = LUMA([a], lr=1e-3), LUMA([b], lr=1e-3)
        opt_b._base_seed = opt_a._base_seed
        a.grad_dtype = None  # the last step's grads are bf16
        b.grad_dtype = None
        grads = [torch.randn(3000, device=DEV) * 1e-3 for _ in range(4)]
        for k, g in enumerate(grads):
            if k == 2:
                a.data = a.data.clone()  # new storage under the same Parameter
            a.grad = g.clone() if k != 3 else g.to(torch.bfloat16)
            b.grad = g.clone() if k != 3 else g.to(torch.bfloat16)
            opt_a.step()
            opt_b.step()
            assert torch.equal(a, b), f"step {k + 1}"
        assert torch.equal(opt_a.state[a]["Q_m"], opt_b.state[b]["Q_m"])
        a.data = a.data.view(60, 50).t()  # same storage and size, not contiguous
        a.grad = torch.zeros(50, 60, device=DEV)
        with pytest.raises(ValueError, match="contiguous parameters"):
            opt_a.step()

    def test_bf16_params_and_autocast_grads(self):
        m = nn.Linear(32, 16).to(DEV).to(torch.bfloat16)
        opt = LUMA(m.parameters(), lr=1e-2)
        for _ in range(5):
            opt.zero_grad()
            m(torch.randn(4, 32, device=DEV, dtype=torch.bfloat16)).float().pow(2).mean().backward()
            opt.step()
        assert all(p.dtype == torch.bfloat16 and p.isfinite().all() for p in m.parameters())
        m32 = nn.Linear(32, 1).to(DEV)
        opt32 = LUMA(m32.parameters(), lr=1e-2)
        with torch.autocast("cuda", dtype=torch.float16):
            m32(torch.randn(8, 32, device=DEV)).float().pow(2).mean().backward()
        opt32.step()
        assert all(p.isfinite().all() for p in m32.parameters())


# ---- test_state_dict.py ------------------------------------------------------

class TestStateDict:
    def test_round_trip_is_bitwise(self):
        loss_fn = quadratic(32)
        kw = dict(lr=1e-2, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.01)
        seed_all(0)
        x_ref = torch.randn(32, device=DEV, requires_grad=True)
        opt_ref = LUMA([x_ref], **kw)
        train(opt_ref, x_ref, loss_fn, 10)
        seed_all(0)
        x_a = torch.randn(32, device=DEV, requires_grad=True)
        opt_a = LUMA([x_a], **kw)
        train(opt_a, x_a, loss_fn, 5)
        sd = opt_a.state_dict()
        x_b = x_a.data.clone().requires_grad_(True)
        opt_b = LUMA([x_b], **kw)
        opt_b.load_state_dict(sd)
        train(opt_b, x_b, loss_fn, 5)
        assert torch.equal(x_b.data, x_ref.data)

    def test_keys_no_private_and_before_step(self):
        m = nn.Linear(8, 4).to(DEV)
        opt = LUMA(m.parameters())
        sd0 = opt.state_dict()
        assert sd0["state"] == {} and len(sd0["param_groups"]) == 1
        m(torch.randn(2, 8, device=DEV)).sum().backward()
        opt.step()
        sd = opt.state_dict()
        assert "_base_seed" in sd
        for s in sd["state"].values():
            assert {"step", "param_id", "Q_m", "Q_w", "S_m", "S_v"} <= set(s)
            assert not any(k.startswith("_") for k in s)
            assert isinstance(s["S_m"], float) and s["S_m"] >= 1e-9 and s["S_v"] >= 0.0

    def test_param_id_preserved_double_save_load_multi_group(self):
        m = nn.Sequential(nn.Linear(8, 16), nn.ReLU(), nn.Linear(16, 4)).to(DEV)
        groups = [{"params": m[0].parameters(), "lr": 1e-2},
                  {"params": m[2].parameters(), "lr": 1e-3, "weight_decay": 0.1}]
        opt = LUMA(groups)
        x = torch.randn(4, 8, device=DEV)
        for _ in range(3):
            opt.zero_grad()
            m(x).sum().backward()
            opt.step()
        sd1 = opt.state_dict()
        m2 = nn.Sequential(nn.Linear(8, 16), nn.ReLU(), nn.Linear(16, 4)).to(DEV)
        m2.load_state_dict(m.state_dict())
        opt2 = LUMA([{"params": m2[0].parameters(), "lr": 1e-2},
                     {"params": m2[2].parameters(), "lr": 1e-3, "weight_decay": 0.1}])
        opt2.load_state_dict(sd1)
        sd2 = opt2.state_dict()
        for k, s in sd1["state"].items():
            t = sd2["state"][k]
            assert s["param_id"] == t["param_id"] and s["step"] == t["step"]
            assert (s["S_m"], s["S_v"]) == (t["S_m"], t["S_v"])
            assert torch.equal(s["Q_m"], t["Q_m"]) and torch.equal(s["Q_w"], t["Q_w"])
        for _ in range(3):
            for o, mm in ((opt, m), (opt2, m2)):
                o.zero_grad()
                mm(x).sum().backward()
                o.step()
        for a, b in zip(m.parameters(), m2.parameters()):
            assert torch.equal(a, b)

    def test_export_structure_and_loads_into_adamw(self):
        m = nn.Linear(8, 4).to(DEV)
        opt = LUMA(m.parameters())
        for _ in range(3):
            opt.zero_grad()
            m(torch.randn(2, 8, device=DEV)).pow(2).sum().backward()
            opt.step()
        exp = opt.export_adamw_state()
        assert set(exp) == {"state", "param_groups"}
        for i, p in enumerate(m.parameters()):
            st = exp["state"][i]
            assert st["exp_avg"].shape == p.shape and st["exp_avg_sq"].shape == p.shape
            assert st["step"].item() == 3.0 and (st["exp_avg_sq"] >= 0).all()
        adamw = torch.optim.AdamW(m.parameters(), lr=1e-3)
        adamw.load_state_dict(exp)
        adamw.step()

    def test_import_roundtrip_and_continue(self):
        seed_all(0)
        x = torch.randn(64, device=DEV, requires_grad=True)
        loss_fn = quadratic(64)
        adamw = torch.optim.AdamW([x], lr=1e-2)
        train(adamw, x, loss_fn, 20)
        ad_sd = adamw.state_dict()
        opt = LUMA([x], lr=1e-2)
        opt.import_adamw_state(ad_sd)
        assert opt.state[x]["step"] == 20 and opt.state[x]["param_id"] == 0
        back = opt.export_adamw_state()["state"][0]
        m0, v0 = ad_sd["state"][0]["exp_avg"], ad_sd["state"][0]["exp_avg_sq"]
        # reference bar (test_state_dict.py:522-561): max error / scale < 0.2%
        assert (back["exp_avg"] - m0).abs().max().item() / m0.abs().max().item() < 2e-3
        assert (back["exp_avg_sq"] - v0).abs().max().item() / v0.max().item() < 2e-3
        l0 = loss_fn(x).item()
        train(opt, x, loss_fn, 30)
        assert loss_fn(x).item() < l0

    def test_import_bit_exact_vs_oracle(self):
        seed_all(1)
        x = torch.randn(3001, device=DEV, requires_grad=True)
        adamw = torch.optim.AdamW([x], lr=1e-2)
        for _ in range(4):
            adamw.zero_grad()
            x.grad = torch.randn(3001, device=DEV) * 1e-2
            adamw.step()
        ad_sd = adamw.state_dict()
        opt = LUMA([x], lr=1e-2)
        opt.import_adamw_state(ad_sd)
        m = ad_sd["state"][0]["exp_avg"].float()
        v = ad_sd["state"][0]["exp_avg_sq"].float().clamp(min=0.0)
        S_m = max(m.abs().max().item(), 1e-9)
        S_v = max(v.max().item(), 0.0)
        w_min, dm, zm, dw, zw = precompute(S_m, S_v, 1e-8)
        um, uw = philox.uniforms(philox.step_seed(opt._base_seed, 0, 0), m.numel())
        um = torch.from_numpy(um).to(DEV)
        uw = torch.from_numpy(uw).to(DEV)
        assert torch.equal(opt.state[x]["Q_m"], quantize_momentum(m, S_m, dm, zm, um))
        assert torch.equal(opt.state[x]["Q_w"], quantize_preconditioner(v, 1e-8, w_min, dw, zw, uw))
        s = opt.state_dict()["state"][0]
        assert (s["S_m"], s["S_v"]) == (S_m, S_v)


# ---- test_determinism.py -----------------------------------------------------

class TestDeterminism:
    def test_same_seed_bitwise_and_global_rng_isolation(self):
        seed_all(0)
        x0 = torch.randn(64, device=DEV)
        g = torch.randn(64, device=DEV)

        def run(pollute):
            seed_all(42)
            x = x0.clone().requires_grad_(True)
            opt = LUMA([x], lr=1e-2, weight_decay=0.01)
            for _ in range(30):
                opt.zero_grad()
                x.grad = g.clone()
                if pollute:
                    torch.rand(5000, device=DEV)
                    random.random()
                opt.step()
            s = opt.state[x]
            return x.data.clone(), s["Q_m"].clone(), s["Q_w"].clone()

        a, b = run(False), run(True)
        assert all(torch.equal(u, v) for u, v in zip(a, b))

    def test_different_seed_differs(self):
        seed_all(0)
        g = torch.randn(64, device=DEV)
        x0 = torch.randn(64, device=DEV)
        qs = []
        for s in (100, 200):
            torch.manual_seed(s)
            x = x0.clone().requires_grad_(True)
            opt = LUMA([x], lr=1e-2)
            fixed_grad_steps(opt, x, g, 2)
            qs.append(opt.state[x]["Q_m"].clone())
        assert not torch.equal(qs[0], qs[1])

    def test_checkpoint_resume_bitwise(self):
        seed_all(0)
        x0 = torch.randn(64, device=DEV)
        g = torch.randn(64, device=DEV)
        seed_all(42)
        x_ref = x0.clone().requires_grad_(True)
        opt_ref = LUMA([x_ref], lr=1e-2)
        fixed_grad_steps(opt_ref, x_ref, g, 30)
        seed_all(42)
        x_a = x0.clone().requires_grad_(True)
        opt_a = LUMA([x_a], lr=1e-2)
        fixed_grad_steps(opt_a, x_a, g, 10)
        sd = opt_a.state_dict()
        x_b = x_a.clone().detach().requires_grad_(True)
        opt_b = LUMA([x_b], lr=1e-2)
        opt_b.load_state_dict(sd)
        fixed_grad_steps(opt_b, x_b, g, 20)
        assert torch.equal(x_ref.data, x_b.data)

    def test_multi_param_model_determinism(self):
        def run():
            seed_all(42)
            model = nn.Sequential(nn.Linear(32, 64), nn.ReLU(), nn.Linear(64, 16)).to(DEV)
            opt = LUMA(model.parameters(), lr=1e-3, weight_decay=0.01)
            x = torch.randn(4, 32, device=DEV)
            for _ in range(30):
                opt.zero_grad()
                model(x).sum().backward()
                opt.step()
            return [p.data.clone() for p in model.parameters()]

        for a, b in zip(run(), run()):
            assert torch.equal(a, b)


# ---- test_convergence.py / test_correctness.py -------------------------------

class TestConvergence:
    def test_rosenbrock(self):
        xy = torch.tensor([-1.0, 1.0], device=DEV, requires_grad=True)
        opt = LUMA([xy], lr=1e-3, weight_decay=0.0)
        f = lambda v: (1 - v[0]) ** 2 + 100 * (v[1] - v[0] ** 2) ** 2
        train(opt, xy, f, 3000)
        assert abs(xy[0].item() - 1.0) < 0.5 and abs(xy[1].item() - 1.0) < 0.5

    def test_mlp_classification(self):
        seed_all(0)
        X = torch.randn(200, 20, device=DEV)
        y = (X @ torch.randn(20, device=DEV) > 0).float()
        model = nn.Sequential(nn.Linear(20, 32), nn.ReLU(), nn.Linear(32, 1)).to(DEV)
        opt = LUMA(model.parameters(), lr=1e-3, weight_decay=0.01)
        crit = nn.BCEWithLogitsLoss()
        init = None
        for _ in range(200):
            opt.zero_grad()
            loss = crit(model(X).squeeze(), y)
            init = loss.item() if init is None else init
            loss.backward()
            opt.step()
        assert loss.item() < init * 0.5

    def test_tracks_adamw_on_quadratic(self):
        d = 32
        loss_fn = quadratic(d)
        x_a = torch.randn(d, device=DEV, requires_grad=True)
        x_l = x_a.data.clone().requires_grad_(True)
        oa = torch.optim.AdamW([x_a], lr=1e-2, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.0)
        ol = LUMA([x_l], lr=1e-2, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.0)
        init = loss_fn(x_a).item()
        la, ll = [], []
        for _ in range(300):
            for o, x, L in ((oa, x_a, la), (ol, x_l, ll)):
                o.zero_grad()
                loss = loss_fn(x)
                L.append(loss.item())
                loss.backward()
                o.step()
        assert ll[-1] < init * 0.035
        assert ll[-1] < la[-1] * 1.015 + 1e-7
        for s in (49, 149, 299):
            assert abs(ll[s] - la[s]) / max(la[s], 1e-8) < 0.015
        assert (x_l - x_a).norm().item() < 0.01 * x_a.norm().item() + 1e-6


class TestLogSRUnbiasedThroughKernel:
    """LogSR with the kernel's Philox uniforms is unbiased (reference bars:
    test_correctness.py:40-103, 200k samples, 2e-3 for m, 1e-3 for w)."""

    N = 200_000

    @pytest.mark.parametrize("val", [0.001, 0.01, 0.1, 0.5, 0.99])
    def test_momentum(self, val):
        m = torch.full((self.N,), val, device=DEV)
        m[0] = 1.0  # S_m = 1
        v = torch.full((self.N,), 1e-6, device=DEV)
        x = torch.zeros(self.N, device=DEV, requires_grad=True)
        opt = LUMA([x])
        opt.import_adamw_state({"state": {0: {"step": 5, "exp_avg": m, "exp_avg_sq": v}},
                                "param_groups": []})
        dec = opt.export_adamw_state()["state"][0]["exp_avg"][1:]
        assert abs(dec.double().mean().item() - val) / val < 2e-3

    @pytest.mark.parametrize("frac", [0.01, 0.25, 0.5, 0.75, 0.99])
    def test_preconditioner(self, frac):
        eps = 1e-8
        S_v = 1.0
        w_min = 1.0 / (math.sqrt(S_v) + eps)
        w = w_min + frac * (1.0 / eps - w_min)
        v_val = (1.0 / w - eps) ** 2
        v = torch.full((self.N,), v_val, device=DEV)
        v[0] = S_v
        m = torch.full((self.N,), 1e-3, device=DEV)
        x = torch.zeros(self.N, device=DEV, requires_grad=True)
        opt = LUMA([x], eps=eps)
        opt.import_adamw_state({"state": {0: {"step": 5, "exp_avg": m, "exp_avg_sq": v}},
                                "param_groups": []})
        q = opt.state[x]["Q_w"][1:].to(torch.int32) & 0xFFFF
        _, _, _, dw, _ = precompute(1e-3, S_v, eps)
        w_dec = w_min * torch.exp(q.double() * dw)
        assert abs(w_dec.mean().item() - w) / w < 1e-3


# ---- remaining reference cases (test_convergence.py, test_state_dict.py,
# ---- test_mixed_precision.py) ------------------------------------------------

class TestReferenceCasesMore:
    def test_mlp_regression(self):
        """test_convergence.py:57-78: loss below 10% of its start in 300 steps."""
        seed_all(0)
        X = torch.randn(200, 10, device=DEV)
        y = X @ torch.randn(10, 1, device=DEV) + 0.1 * torch.randn(200, 1, device=DEV)
        model = nn.Sequential(nn.Linear(10, 32), nn.ReLU(), nn.Linear(32, 1)).to(DEV)
        opt = LUMA(model.parameters(), lr=1e-3, weight_decay=0.01)
        init = None
        for _ in range(300):
            opt.zero_grad()
            loss = nn.functional.mse_loss(model(X), y)
            init = loss.item() if init is None else init
            loss.backward()
            opt.step()
        assert loss.item() < init * 0.1

    def test_multi_param_groups_converge(self):
        """test_convergence.py:80-103: two groups with their own lr."""
        seed_all(0)
        model = nn.Sequential(nn.Linear(10, 32), nn.ReLU(), nn.Linear(32, 1)).to(DEV)
        opt = LUMA([{"params": model[0].parameters(), "lr": 2e-3},
                    {"params": model[2].parameters(), "lr": 5e-4}], weight_decay=0.01)
        X, y = torch.randn(100, 10, device=DEV), torch.randn(100, 1, device=DEV)
        init = None
        for _ in range(200):
            opt.zero_grad()
            loss = nn.functional.mse_loss(model(X), y)
            init = loss.item() if init is None else init
            loss.backward()
            opt.step()
        assert loss.item() < init * 0.5

    def test_export_after_one_step_and_multi_group(self):
        """test_state_dict.py:354-416: export at step 1; per-group hyper-
        parameters kept, and the export loads into torch AdamW and trains."""
        m1 = nn.Linear(8, 4).to(DEV)
        o1 = LUMA(m1.parameters())
        m1(torch.randn(1, 8, device=DEV)).sum().backward()
        o1.step()
        assert len(o1.export_adamw_state()["state"]) == 2
        model = nn.Sequential(nn.Linear(10, 16), nn.ReLU(), nn.Linear(16, 1)).to(DEV)
        opt = LUMA([{"params": model[0].parameters(), "lr": 2e-3},
                    {"params": model[2].parameters(), "lr": 5e-4}], weight_decay=0.01)
        for _ in range(3):
            opt.zero_grad()
            model(torch.randn(5, 10, device=DEV)).sum().backward()
            opt.step()
        sd = opt.export_adamw_state()
        assert [g["lr"] for g in sd["param_groups"]] == [2e-3, 5e-4] and len(sd["state"]) == 4
        model2 = nn.Sequential(nn.Linear(10, 16), nn.ReLU(), nn.Linear(16, 1)).to(DEV)
        model2.load_state_dict(model.state_dict())
        adamw = torch.optim.AdamW([{"params": model2[0].parameters(), "lr": 2e-3},
                                   {"params": model2[2].parameters(), "lr": 5e-4}],
                                  weight_decay=0.01)
        adamw.load_state_dict(sd)
        adamw.zero_grad()
        model2(torch.randn(5, 10, device=DEV)).sum().backward()
        adamw.step()
        assert all(p.isfinite().all() for p in model2.parameters())

    def test_import_multi_group_preserves_step_then_trains(self):
        """test_state_dict.py:443-458, 563-608."""
        seed_all(0)
        model = nn.Sequential(nn.Linear(10, 16), nn.ReLU(), nn.Linear(16, 1)).to(DEV)
        groups = lambda: [{"params": model[0].parameters(), "lr": 2e-3},  # noqa: E731
                          {"params": model[2].parameters(), "lr": 5e-4}]
        adamw = torch.optim.AdamW(groups(), weight_decay=0.01)
        X = torch.randn(10, 10, device=DEV)
        for _ in range(5):
            adamw.zero_grad()
            model(X).sum().backward()
            adamw.step()
        luma = LUMA(groups(), weight_decay=0.01)
        luma.import_adamw_state(adamw.state_dict())
        sd = luma.state_dict()
        assert len(sd["state"]) == 4 and all(s["step"] == 5 for s in sd["state"].values())
        for _ in range(5):
            luma.zero_grad()
            model(X).sum().backward()
            luma.step()
        assert all(p.isfinite().all() for p in model.parameters())
        assert all(s["step"] == 10 for s in luma.state_dict()["state"].values())

    def test_import_then_save_load_continues(self):
        """test_state_dict.py:610-646: AdamW -> import -> train -> save -> load
        into a fresh optimizer -> training still lowers the loss."""
        seed_all(0)
        loss_fn = quadratic(32)
        kw = dict(lr=1e-2, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.01)
        x = torch.randn(32, device=DEV, requires_grad=True)
        adamw = torch.optim.AdamW([x], **kw)
        train(adamw, x, loss_fn, 10)
        luma = LUMA([x], **kw)
        luma.import_adamw_state(adamw.state_dict())
        train(luma, x, loss_fn, 5)
        sd = luma.state_dict()
        xr = x.data.clone().requires_grad_(True)
        luma2 = LUMA([xr], **kw)
        luma2.load_state_dict(sd)
        before = loss_fn(xr).item()
        train(luma2, xr, loss_fn, 10)
        assert loss_fn(xr).item() < before

    @pytest.mark.parametrize("adt", [torch.float16, torch.bfloat16])
    def test_autocast_twenty_steps_stable_and_converges(self, adt):
        """test_mixed_precision.py:45-117: autocast forward/backward, fp32
        params; 20 steps finite, and the loss falls."""
        seed_all(0)
        model = nn.Sequential(nn.Linear(32, 64), nn.ReLU(), nn.Linear(64, 1)).to(DEV)
        opt = LUMA(model.parameters(), lr=1e-3)
        X, y = torch.randn(128, 32, device=DEV), torch.randn(128, 1, device=DEV)
        losses = []
        for _ in range(100):
            opt.zero_grad()
            with torch.autocast("cuda", dtype=adt):
                loss = nn.functional.mse_loss(model(X).float(), y)
            loss.backward()
            opt.step()
            losses.append(loss.item())
            if len(losses) == 20:
                assert all(math.isfinite(v) for v in losses)
                assert all(p.isfinite().all() for p in model.parameters())
        assert losses[-1] < losses[0]

    def test_gradscaler_fused_converges(self):
        """test_mixed_precision.py:119-184 with the fused unscale (amp.scaler_step)."""
        from luma_b200.amp import scaler_step
        seed_all(0)
        model = nn.Sequential(nn.Linear(32, 64), nn.ReLU(), nn.Linear(64, 1)).to(DEV)
        opt = LUMA(model.parameters(), lr=1e-3)
        scaler = torch.amp.GradScaler("cuda")
        X, y = torch.randn(128, 32, device=DEV), torch.randn(128, 1, device=DEV)
        losses = []
        for _ in range(100):
            opt.zero_grad()
            with torch.autocast("cuda", dtype=torch.float16):
                loss = nn.functional.mse_loss(model(X).float(), y)
            scaler.scale(loss).backward()
            scaler_step(scaler, opt)
            scaler.update()
            losses.append(loss.item())
        assert all(math.isfinite(v) for v in losses) and losses[-1] < losses[0]
