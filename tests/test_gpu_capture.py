"""CUDA-graph capture and torch.compile of the step (GPU).

Mirrors the reference's claims and tests: the Triton backend is "compatible
with external torch.cuda.CUDAGraph capture" with a device step counter
(optimizer.py:18-19, 382-387), and its step functions compile with
``fullgraph=True`` and no graph breaks, alone and inside a compiled train
step (tests/test_compile.py:84-290).  Here: ``LUMA(capturable=True)``
captured once and replayed must give, bit for bit, what eager steps give;
``torch.ops.luma_b200.step`` compiles without graph breaks and matches.
"""

import pytest
import torch
import torch.nn as nn

pytestmark = pytest.mark.gpu

DEV = "cuda"
SHAPES = [(257, 129), (4096,), (3,), (1000,)]


@pytest.fixture(autouse=True)
def _dynamo_reset():
    torch._dynamo.reset()
    yield
    torch._dynamo.reset()


def _params(pdt, seed=0):
    g = torch.Generator().manual_seed(seed)
    out = [(torch.randn(s, generator=g) * 0.02).to(pdt).to(DEV) for s in SHAPES]
    for t in out:
        t.grad_dtype = None  # grads may differ in dtype from the param
    return out


def _grads(step, pdt_grad=torch.bfloat16):
    g = torch.Generator().manual_seed(1000 + step)
    return [(torch.randn(s, generator=g) * 1e-3).to(pdt_grad).to(DEV) for s in SHAPES]


def _same(opt_a, pa, opt_b, pb, tag):
    for i, (x, y) in enumerate(zip(pa, pb)):
        assert torch.equal(x, y), f"{tag}: param {i} differs"
        sa, sb = opt_a.state[x], opt_b.state[y]
        assert torch.equal(sa["Q_m"], sb["Q_m"]) and torch.equal(sa["Q_w"], sb["Q_w"]), \
            f"{tag}: codes of param {i} differ"
    da, db = opt_a.state_dict()["state"], opt_b.state_dict()["state"]
    for k in da:
        for key in ("step", "S_m", "S_v"):
            assert da[k][key] == db[k][key], f"{tag}: {key} of param {k} differs"


def _pair(pdt, **kw):
    torch.manual_seed(7)
    pe = _params(pdt)
    oe = luma_cls()(pe, lr=1e-3, weight_decay=0.01)
    torch.manual_seed(7)
    pc = _params(pdt)
    oc = luma_cls()(pc, lr=1e-3, weight_decay=0.01, capturable=True, **kw)
    assert oe._base_seed == oc._base_seed
    return pe, oe, pc, oc


def luma_cls():
    from luma_b200 import LUMA
    return LUMA


@pytest.mark.parametrize("pdt", [torch.float32, torch.bfloat16])
def test_graph_replay_bit_exact_vs_eager(pdt):
    pe, oe, pc, oc = _pair(pdt)
    static = [torch.zeros_like(p, dtype=torch.bfloat16) for p in pc]
    for p, g in zip(pc, static):
        p.grad = g
    # two eager steps (first step + one quantized step), then capture
    for t in (1, 2):
        for p, g in zip(pe, _grads(t)):
            p.grad = g
        oe.step()
        for g, src in zip(static, _grads(t)):
            g.copy_(src)
        oc.step()
    torch.cuda.synchronize()
    _same(oe, pe, oc, pc, "eager steps")
    graph = torch.cuda.CUDAGraph()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        with torch.cuda.graph(graph):
            oc.step()  # captured: not executed now
    torch.cuda.current_stream().wait_stream(side)
    for t in range(3, 8):
        for p, g in zip(pe, _grads(t)):
            p.grad = g
        oe.step()
        for g, src in zip(static, _grads(t)):
            g.copy_(src)
        graph.replay()
    torch.cuda.synchronize()
    _same(oe, pe, oc, pc, "after 5 replays")
    assert oc.kernel_error_flags() == 0
    del graph


def test_graph_replay_sees_refreshed_lr():
    pe, oe, pc, oc = _pair(torch.float32)
    static = [torch.zeros_like(p) for p in pc]
    for p, g in zip(pc, static):
        p.grad = g
    for t in (1, 2):
        for p, g in zip(pe, _grads(t, torch.float32)):
            p.grad = g
        oe.step()
        for g, src in zip(static, _grads(t, torch.float32)):
            g.copy_(src)
        oc.step()
    graph = torch.cuda.CUDAGraph()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        with torch.cuda.graph(graph):
            oc.step()
    torch.cuda.current_stream().wait_stream(side)
    for t, lr in zip(range(3, 7), (1e-3, 5e-4, 2e-4, 2e-4)):
        for o in (oe, oc):
            for gr in o.param_groups:
                gr["lr"] = lr
        oc.refresh_capturable_rows()
        for p, g in zip(pe, _grads(t, torch.float32)):
            p.grad = g
        oe.step()
        for g, src in zip(static, _grads(t, torch.float32)):
            g.copy_(src)
        graph.replay()
    torch.cuda.synchronize()
    _same(oe, pe, oc, pc, "lr schedule under replay")
    del graph


def test_capture_steps_exhausted_skips_and_flags():
    from luma_b200 import LUMA
    p = [torch.randn(1000, device=DEV) * 0.02]
    opt = LUMA(p, lr=1e-3, capturable=True, capture_steps=2)
    opt.kernel_error_flags(clear=True)
    for t in (1, 2):
        p[0].grad = torch.randn(1000, device=DEV) * 1e-3
        opt.step()
    assert opt.kernel_error_flags() == 0
    before = p[0].clone()
    p[0].grad = torch.randn(1000, device=DEV) * 1e-3
    opt.step()  # step 3 has no row: skipped on the device
    torch.cuda.synchronize()
    assert torch.equal(p[0], before)
    assert opt.kernel_error_flags(clear=True) == 1  # LUMA_KERR_ROW_RANGE
    assert opt.kernel_error_flags() == 0


def test_custom_op_fullgraph_matches_eager():
    pe, oe, pc, oc = _pair(torch.float32)
    for t in (1, 2):
        for p, g in zip(pe, _grads(t, torch.float32)):
            p.grad = g
        oe.step()
        for p, g in zip(pc, _grads(t, torch.float32)):
            p.grad = g
        oc.step()
    static = [p.grad for p in pc]
    op = torch.compile(lambda kw: torch.ops.luma_b200.step(**kw), fullgraph=True)
    for t in range(3, 6):
        for p, g in zip(pe, _grads(t, torch.float32)):
            p.grad = g
        oe.step()
        for g, src in zip(static, _grads(t, torch.float32)):
            g.copy_(src)
        op(oc.step_op_args())
    torch.cuda.synchronize()
    _same(oe, pe, oc, pc, "compiled op")


def test_custom_op_zero_graph_breaks():
    from luma_b200 import LUMA
    p = [torch.randn(4096, device=DEV) * 0.02]
    opt = LUMA(p, lr=1e-3, capturable=True)
    p[0].grad = torch.randn(4096, device=DEV) * 1e-3
    opt.step()
    explanation = torch._dynamo.explain(lambda kw: torch.ops.luma_b200.step(**kw))(
        opt.step_op_args())
    assert explanation.graph_break_count == 0, explanation.break_reasons


@pytest.mark.parametrize("autocast", [False, True])
def test_compiled_train_step(autocast):
    from luma_b200 import LUMA
    model = nn.Sequential(nn.Linear(32, 64), nn.ReLU(), nn.Linear(64, 1)).to(DEV)
    opt = LUMA(model.parameters(), lr=1e-3)
    x = torch.randn(8, 32, device=DEV)
    y = torch.randn(8, 1, device=DEV)

    @torch.compile()
    def train_step(x, y):
        opt.zero_grad()
        if autocast:
            with torch.amp.autocast("cuda", dtype=torch.float16):
                pred = model(x)
            loss = (pred.float() - y).square().mean()
        else:
            loss = (model(x) - y).square().mean()
        loss.backward()
        opt.step()
        return loss

    losses = [train_step(x, y).item() for _ in range(10)]
    assert all(torch.isfinite(torch.tensor(losses)))
    for p in model.parameters():
        assert p.isfinite().all()
        assert opt.state[p]["step"] == 10
