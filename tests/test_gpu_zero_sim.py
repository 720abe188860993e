"""ZeRO-1 sharded step on ONE GPU, every rank simulated in turn (GPU).

The per-rank math of the sharded step needs no communication: rank r steps
the (tensor, piece) segments of its pieces with per-segment scales,
``param_id`` = the tensor's global index and Philox counter = the segment's
offset inside the tensor (the reference's per-local-shard semantics,
optimizer.py:399-407, tests/test_fsdp.py:139-184).  So each rank of a
world of 2, 4 or 8 is run here as its own ``ZeroLUMA`` over its own replica
with ``step_local`` (no process group), and every segment must equal the
oracle (the reference's op sequence on CUDA) run on that segment alone with
the same draws — bit for bit, after every step.  The gather itself is covered
by the 2-GPU tests and the CPU gloo tests.

Also: a ZeroLUMA checkpoint (``state_dict``) restored into a fresh instance
continues bit-exactly like an uninterrupted run.
"""

import pytest
import torch

from oracle import philox
from oracle.luma_ref import init_step, update_step

pytestmark = pytest.mark.gpu

DEV = "cuda"
SHAPES = [(4096, 64), (1000,), (3,), (256, 257), (70_001,), (64, 64), (5,), (300_007,)]
HP = dict(lr=1e-3, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.01)
SEED = -5_432_109_876_543


def _numel(s):
    return int(torch.tensor(s).prod()) if s else 1


class _SegmentOracle:
    """The reference step on one shard segment as its own tensor."""

    def __init__(self, param, tensor, offset):
        self.p = param.clone()
        self.tensor, self.offset = tensor, offset
        self.st = {}

    def step(self, grad, t):
        b1, b2 = HP["betas"]
        work = self.p.float() if self.p.dtype == torch.bfloat16 else self.p
        um, uw = philox.uniforms_torch(philox.step_seed(SEED, t, self.tensor), self.p.numel(),
                                       self.offset, device=DEV)
        if t == 1:
            self.st["Q_m"], self.st["Q_w"], self.st["S_m"], self.st["S_v"] = init_step(
                work, grad, b1, b2, HP["eps"], HP["lr"], HP["weight_decay"], um, uw)
        else:
            self.st["S_m"], self.st["S_v"] = update_step(
                work, grad, self.st["Q_m"], self.st["Q_w"], self.st["S_m"], self.st["S_v"], t,
                b1, b2, HP["eps"], HP["lr"], HP["weight_decay"], um, uw)
        if work is not self.p:
            self.p.copy_(work)


def _init_flat(lay, pdt, gen):
    from luma_b200.zero import flat_views
    flat = torch.zeros(lay.total, dtype=pdt, device=DEV)
    for v, s in zip(flat_views(flat, lay, SHAPES), SHAPES):
        v.copy_((torch.randn(s, generator=gen) * 0.02).to(pdt))
    return flat


@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("buckets", [1, 3])
@pytest.mark.parametrize("pdt", [torch.bfloat16, torch.float32])
def test_every_simulated_rank_bit_exact_per_segment(world, buckets, pdt):
    from luma_b200.zero import ZeroLUMA, plan_layout, shard_segments
    lay = plan_layout([_numel(s) for s in SHAPES], world, buckets)
    gen = torch.Generator().manual_seed(17)
    flat0 = _init_flat(lay, pdt, gen)
    grads = [(torch.randn(lay.total, generator=gen) * 1e-3).to(torch.bfloat16).to(DEV)
             for _ in range(3)]
    covered = 0
    for rank in range(world):
        flat = flat0.clone()
        opt = ZeroLUMA(flat, lay, rank, base_seed=SEED, gather="nccl", **HP)
        segs = shard_segments(lay, rank)
        oracles = [_SegmentOracle(flat0[sg.flat:sg.flat + sg.length], sg.tensor, sg.offset)
                   for sg in segs]
        for t in range(1, 4):
            g = grads[t - 1]
            gshard = torch.cat([g[slice(*lay.owned(rank, b))] for b in range(lay.buckets)])
            opt.step_local(gshard)
            for sg, o in zip(segs, oracles):
                o.step(g[sg.flat:sg.flat + sg.length], t)
            torch.cuda.synchronize()
            scales = opt.scales()
            for k, (sg, o) in enumerate(zip(segs, oracles)):
                tag = f"world {world} rank {rank} t={t} seg {k} (tensor {sg.tensor}+{sg.offset})"
                assert torch.equal(flat[sg.flat:sg.flat + sg.length], o.p), f"{tag}: params"
                lo = sg.local
                assert torch.equal(opt.q_m[lo:lo + sg.length], o.st["Q_m"]), f"{tag}: Q_m"
                assert torch.equal(opt.q_w[lo:lo + sg.length], o.st["Q_w"]), f"{tag}: Q_w"
                assert scales[k][2:] == (o.st["S_m"], o.st["S_v"]), f"{tag}: scales"
        covered += sum(sg.length for sg in segs)
    assert covered == sum(_numel(s) for s in SHAPES)


@pytest.mark.parametrize("buckets", [1, 3])
def test_zero_checkpoint_resumes_bit_exact(buckets):
    from luma_b200.zero import ZeroLUMA, plan_layout
    world, rank = 4, 1
    lay = plan_layout([_numel(s) for s in SHAPES], world, buckets)
    gen = torch.Generator().manual_seed(23)
    flat0 = _init_flat(lay, torch.bfloat16, gen)
    grads = [(torch.randn(lay.shard, generator=gen) * 1e-3).to(torch.bfloat16).to(DEV)
             for _ in range(5)]
    # uninterrupted
    fa = flat0.clone()
    a = ZeroLUMA(fa, lay, rank, base_seed=SEED, gather="nccl", **HP)
    for g in grads:
        a.step_local(g)
    # interrupted after 2 steps: save, rebuild, load, continue
    fb = flat0.clone()
    b = ZeroLUMA(fb, lay, rank, base_seed=SEED, gather="nccl", **HP)
    for g in grads[:2]:
        b.step_local(g)
    sd = b.state_dict()
    saved_params = fb.cpu()
    del b
    fc = saved_params.to(DEV)
    c = ZeroLUMA(fc, lay, rank, base_seed=7, gather="nccl", lr=0.5)  # overwritten by the load
    c.load_state_dict(sd)
    assert c.t == 2 and c.base_seed == SEED and c.hp["lr"] == HP["lr"]
    for g in grads[2:]:
        c.step_local(g)
    assert torch.equal(fa, fc)
    assert torch.equal(a.q_m, c.q_m) and torch.equal(a.q_w, c.q_w)
    assert a.scales() == c.scales()
    # a checkpoint of another rank or layout is refused
    with pytest.raises(ValueError, match="rank"):
        ZeroLUMA(fc.clone(), lay, 2, gather="nccl").load_state_dict(sd)
    other = plan_layout([_numel(s) for s in SHAPES], 2, buckets)
    with pytest.raises(ValueError, match="layout"):
        ZeroLUMA(torch.zeros(other.total, dtype=torch.bfloat16, device=DEV), other, 1,
                 gather="nccl").load_state_dict(sd)
