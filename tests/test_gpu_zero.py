"""ZeRO-1 sharded step on 2 GPUs: bit-exact per segment, gathered replicas equal.

Each rank steps its flat shard; every (tensor, shard) segment must equal the
oracle (the reference's op sequence on CUDA) run on that segment alone with
the backend's Philox stream (param_id = tensor index, counter offset = the
segment's offset in the tensor).  After the all-gather (NCCL, or copy-engine
pushes over CUDA IPC, or the step's own multicast stores through NVSwitch; for
the sharded-params mode into staging buffers) both ranks must hold the same
full parameter buffer,
and its pieces must be each owner's result.
Skipped with fewer than 2 GPUs.
"""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")]

SHAPES = [(4096, 64), (1000,), (3,), (256, 257), (70_001,), (64, 64), (5,)]
# "+large": one more tensor long enough that every CTA runs the steady pass-2
# loop on its shard, whose multicast stores then carry the gather
LARGE = [(48_000_003,)]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, pdt_name, buckets, gather, out_q):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [root, os.path.join(root, "tests")]
    from luma_b200.zero import ZeroLUMA, alloc_flat, flat_views, plan_layout, shard_segments
    from oracle import philox
    from oracle.luma_ref import OracleLUMA

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
    msgs = []
    try:
        pdt = getattr(torch, pdt_name)
        shapes = SHAPES + (LARGE if gather.endswith("+large") else [])
        gather = gather.removesuffix("+large")
        numels = [int(torch.tensor(s).prod()) if s else 1 for s in shapes]
        lay = plan_layout(numels, world, buckets)
        gen = torch.Generator().manual_seed(5)
        flat = alloc_flat(lay.total, pdt, dev, gather if gather in ("nccl", "copy", "nvls")
                          else "nccl")
        flat.zero_()
        for v, s in zip(flat_views(flat, lay, shapes), shapes):
            v.copy_((torch.randn(s, generator=gen) * 0.02).to(pdt))
        segs = shard_segments(lay, rank)
        sharded = gather.startswith("sharded")
        if sharded:
            # params held as this rank's pieces only; buckets gathered into staging
            full = flat
            flat = torch.cat([full[slice(*lay.owned(rank, b))] for b in range(lay.buckets)])
            gathered = torch.zeros_like(full)

            def consumer(b, view):
                gathered[b * lay.span:(b + 1) * lay.span].copy_(view)

            mode = {"sharded-nvls": "nvls", "sharded-copy": "copy"}.get(gather, "nccl")
            opt = ZeroLUMA(flat, lay, rank, lr=1e-3, base_seed=1234567890123, replica=False,
                           consumer=consumer, gather=mode)
            if opt.gather_mode != mode:
                msgs.append(f"{mode} unavailable: fell back to {opt.gather_mode}")
        else:
            opt = ZeroLUMA(flat, lay, rank, lr=1e-3, base_seed=1234567890123, max_ctas=100,
                           gather=gather)
            if gather == "nvls" and opt.gather_mode != "nvls":
                msgs.append(f"nvls unavailable: fell back to {opt.gather_mode}")

        def pos(sg):
            return sg.local if sharded else sg.flat
        # oracle: every local segment as its own tensor
        oparams = [flat[pos(sg):pos(sg) + sg.length].clone() for sg in segs]
        for p in oparams:
            p.grad_dtype = None

        def draws(k, t, like):
            sg = segs[k]
            um, uw = philox.uniforms(philox.step_seed(opt.base_seed, t, sg.tensor), sg.length,
                                     rng_offset=sg.offset)
            return torch.from_numpy(um).to(dev), torch.from_numpy(uw).to(dev)

        orc = OracleLUMA(oparams, lr=1e-3, draws=draws)
        for t in range(1, 4):
            gfull = (torch.randn(lay.total, generator=gen) * 1e-3).to(torch.bfloat16).to(dev)
            gshard = torch.cat([gfull[slice(*lay.owned(rank, b))] for b in range(lay.buckets)])
            for k, sg in enumerate(segs):
                oparams[k].grad = gfull[sg.flat:sg.flat + sg.length].clone()
            opt.step(gshard)
            orc.step()
            torch.cuda.synchronize()
            for k, sg in enumerate(segs):
                lo = sg.local
                if not torch.equal(flat[pos(sg):pos(sg) + sg.length], oparams[k]):
                    msgs.append(f"t={t} seg {k}: params differ")
                ost = orc.state[id(oparams[k])]
                if not torch.equal(opt.q_m[lo:lo + sg.length], ost["Q_m"]):
                    msgs.append(f"t={t} seg {k}: Q_m differs")
                if not torch.equal(opt.q_w[lo:lo + sg.length], ost["Q_w"]):
                    msgs.append(f"t={t} seg {k}: Q_w differs")
            for k, (ti, off, S_m, S_v) in enumerate(opt.scales()):
                ost = orc.state[id(oparams[k])]
                if (S_m, S_v) != (ost["S_m"], ost["S_v"]):
                    msgs.append(f"t={t} seg {k}: scales differ")
            # replicas identical after the gather
            rep = gathered if sharded else flat
            other = torch.empty_like(rep)
            dist.broadcast(other.copy_(rep), src=0)
            if not torch.equal(other, rep):
                msgs.append(f"t={t}: gathered replicas differ")
            if sharded:
                # every element of this rank's tensors is in the gathered
                # buckets (positions outside every tensor are not data)
                for k, sg in enumerate(segs):
                    if not torch.equal(gathered[sg.flat:sg.flat + sg.length],
                                       flat[sg.local:sg.local + sg.length]):
                        msgs.append(f"t={t}: gathered bucket {sg.bucket} lacks segment {k}")
        opt.close()
        out_q.put((rank, msgs))
    except Exception as exc:  # noqa: BLE001
        out_q.put((rank, [f"exception: {exc!r}"]))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("pdt_name,buckets,gather", [
    ("bfloat16", 1, "nccl"), ("float32", 1, "nccl"), ("bfloat16", 3, "nccl"),
    ("bfloat16", 3, "copy"), ("float32", 1, "copy"), ("bfloat16", 3, "sharded"),
    ("bfloat16", 3, "nvls"), ("float32", 1, "nvls"), ("bfloat16", 3, "sharded-nvls"),
    ("float32", 2, "sharded-nvls"), ("bfloat16", 1, "nvls+large"),
    ("bfloat16", 1, "sharded-nvls+large"), ("bfloat16", 3, "sharded-copy"),
    ("float32", 2, "sharded-copy")])
def test_zero_sharded_step_two_gpus(pdt_name, buckets, gather):
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, pdt_name, buckets, gather, q))
             for r in range(world)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=600) for _ in range(world))
    for p in procs:
        p.join(timeout=120)
    for r in range(world):
        assert results[r] == [], results[r]
    assert all(p.exitcode == 0 for p in procs)
