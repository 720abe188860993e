"""Benchmark of the LUMA optimizer step on B200 (driver contract).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl luma|reference]
                    [--config llama8b|llama70b|llama_layer|gpt2|ragged|cpu21m|nanogpt]
                    [--gather auto|nvls|copy|nccl]

A "step" is one ``LUMA.step()`` over every parameter tensor of the workload
(two kernel launches).  Default workload: Llama-3-8B parameter shapes (291
tensors, 8,030,261,248 params), bf16 params, bf16 grads N(0, 1e-3) drawn once
before timing (as the reference's bench_compile.py times ``opt.step()`` with
grads pre-made).  Params, grads and codes are resident in HBM (64 GB), far
larger than L2, so no L2 flush is needed between steps.

Printed (rank 0, one JSON line): step throughput in Gparams/s (``value``),
achieved HBM bandwidth against the algorithmic bytes per param, the roofline
of the dominant kernel (pass 2) from per-pass CUDA events, ``e2e`` through the
public API with grads copied from pinned host memory every step, the
reference's own PyTorch backend (the unmodified package installed in
``baseline/_ref``) timed on this host's cores, the reference's own GPU kernels
(its Triton backend) beside this backend on the same shapes, and the SM
clocks sampled during timing.

``--impl reference`` times the reference's PyTorch backend on the host CPU
cores (``luma_optimizer.LUMA(backend="pytorch")`` from ``baseline/_ref``,
drawing its own uniforms every step; the oracle restatement only when that
install is absent) on a bounded sample of the same workload.

``--config nanogpt`` runs the end-to-end training configuration instead: GPT-2
small on uniform-random token ids, batch 12 x 1024, LUMA and AdamW trained on
the same batches from the same init.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

import torch  # noqa: E402

METRIC = "LUMA step Gparams/s & HBM GB/s (% of peak), Llama-3-8B shapes, 1/2/4/8 GPU"
NOMINAL_HBM_GBS = 8000.0
FALLBACK_HBM_GBS = 6650.0


# ---------------------------------------------------------------------------
# workloads (synthetic configs with the reference benchmarks' shapes)
# ---------------------------------------------------------------------------

def llama3_8b_shapes():
    d, kv, ffn, vocab, layers = 4096, 1024, 14336, 128256, 32
    shapes = [(vocab, d)]
    for _ in range(layers):
        shapes += [(d, d), (kv, d), (kv, d), (d, d), (ffn, d), (ffn, d), (d, ffn), (d,), (d,)]
    shapes += [(d,), (vocab, d)]
    return shapes


def gpt2_small_shapes():
    d, vocab, ctx = 768, 50257, 1024
    shapes = [(vocab, d), (ctx, d)]
    for _ in range(12):
        shapes += [(d,), (d,), (d, 3 * d), (3 * d,), (d, d), (d,), (d,), (d,),
                   (d, 4 * d), (4 * d,), (4 * d, d), (d,)]
    shapes += [(d,), (d,)]
    return shapes


def ragged_shapes(n=10_000, seed=0):
    import numpy as np
    rng = np.random.default_rng(seed)
    return [(max(1, int(round(2 ** rng.uniform(0, 20)))),) for _ in range(n)]


def llama3_70b_shapes():
    d, kv, ffn, vocab, layers = 8192, 1024, 28672, 128256, 80
    shapes = [(vocab, d)]
    for _ in range(layers):
        shapes += [(d, d), (kv, d), (kv, d), (d, d), (ffn, d), (ffn, d), (d, ffn), (d,), (d,)]
    shapes += [(d,), (vocab, d)]
    return shapes


def llama_layer_shapes():
    d, kv, ffn = 4096, 1024, 14336
    return [(d, d), (kv, d), (kv, d), (d, d), (ffn, d), (ffn, d), (d, ffn), (d,), (d,)]


def cpu21m_shapes():
    return [(1024, 1024)] * 4 + [(4096, 1024)] * 2 + [(1024, 4096)] * 2


CONFIGS = {
    # grads: "normal" N(0, gscale); "sigma" per-tensor sigma log-uniform in
    # [1e-4, 1e-1]; "stress" N(0, gscale) with ~10% all-zero tensors and, in
    # the others, 1% of elements at +-1e4 or +-1e-40 (BASELINE configs 1 and 3)
    "llama8b": dict(shapes=llama3_8b_shapes, pdt=torch.bfloat16, gdt=torch.bfloat16,
                    gscale=1e-3, name="Llama-3-8B shapes (291 tensors), bf16 params, bf16 grads"),
    "llama70b": dict(shapes=llama3_70b_shapes, pdt=torch.bfloat16, gdt=torch.bfloat16,
                     gscale=1e-3, name="Llama-3-70B shapes (723 tensors), bf16 params, bf16 grads "
                     "(N>1: params sharded, buckets gathered into staging buffers)"),
    "llama_layer": dict(shapes=llama_layer_shapes, pdt=torch.bfloat16, gdt=torch.bfloat16,
                        gscale=1e-3, name="one Llama-3-8B decoder layer (9 tensors, 218,112,000 "
                        "params), bf16 params, bf16 grads (profiling case)"),
    "gpt2": dict(shapes=gpt2_small_shapes, pdt=torch.float32, gdt=torch.bfloat16,
                 gscale=1e-3, name="GPT-2 small shapes (148 tensors), fp32 params, bf16 grads"),
    "ragged": dict(shapes=ragged_shapes, pdt=torch.float32, gdt=torch.float32, grads="stress",
                   gscale=1e-2, name="ragged: 10,000 fp32 tensors, numel log-uniform in [1, 2^20], "
                   "grads N(0,1e-2) with ~10% all-zero tensors and 1% elements at +-1e4 / +-1e-40"),
    "cpu21m": dict(shapes=cpu21m_shapes, pdt=torch.float32, gdt=torch.float32, grads="sigma",
                   gscale=1e-2, name="8 fp32 tensors, 20,971,520 params (reference CPU config), "
                   "grads N(0, sigma_t), sigma_t log-uniform in [1e-4, 1e-1]"),
}


def numel(shape):
    return math.prod(shape) if shape else 1


def bytes_per_param(pdt, gdt):
    """Algorithmic HBM bytes per param per step: pass 1 reads g, Q_m, Q_w;
    pass 2 reads g, Q_m, Q_w, p and writes p, Q_m, Q_w."""
    g, p = torch.tensor([], dtype=gdt).element_size(), torch.tensor([], dtype=pdt).element_size()
    pass1 = g + 4
    pass2 = g + 4 + 2 * p + 4
    return pass1, pass2


def measured_peak():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:  # noqa: BLE001
        return FALLBACK_HBM_GBS, "fallback"


def committed_traffic(config):
    """ncu-measured DRAM bytes per param of pass 2, from the committed profile summary."""
    path = os.path.join(ROOT, "profiles", f"luma_pass2_{config}.json")
    try:
        with open(path) as f:
            return float(json.load(f)["dram_bytes_per_param"])
    except Exception:  # noqa: BLE001
        return None


# ---------------------------------------------------------------------------
# clocks sampling
# ---------------------------------------------------------------------------

class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        self.path = None

    def start(self):
        try:
            import tempfile
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200", "-i", str(self.gpu)],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:  # noqa: BLE001
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:  # noqa: BLE001
            self.proc.kill()
        rows = []
        with open(self.path) as f:
            for line in f:
                parts = [x.strip() for x in line.split(",")]
                if len(parts) >= 8:
                    rows.append(parts)
        os.unlink(self.path)
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        smax = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[k] for r in rows for k in range(4) if r[4 + k] == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(smax) if smax else None,
                "reasons": reasons, "samples": len(rows)}


# ---------------------------------------------------------------------------
# CPU baseline: the reference algorithm (oracle restatement) on host cores
# ---------------------------------------------------------------------------

def cpu_sample_shapes(config):
    if config == "llama8b":
        d, kv = 4096, 1024
        return [(d, d), (kv, d), (kv, d), (d, d)], "one Llama-3-8B attention block: q,k,v,o (33,554,432 params)"
    if config == "cpu21m":
        return cpu21m_shapes(), "the full 8-tensor config (20,971,520 params)"
    if config == "gpt2":
        d = 768
        return [(d, 3 * d), (3 * d,), (d, d), (d, 4 * d), (4 * d, d)], "one GPT-2 block's matrices"
    return ragged_shapes(200, seed=1), "200 ragged tensors"


def reference_package():
    """The unmodified reference package installed in baseline/_ref, or None."""
    ref_dir = os.path.join(ROOT, "baseline", "_ref")
    if not os.path.isdir(os.path.join(ref_dir, "luma_optimizer")):
        return None
    if ref_dir not in sys.path:
        sys.path.insert(0, ref_dir)
    import luma_optimizer
    return luma_optimizer


def cpu_baseline(config, steps, warmup, budget_s=20.0):
    """Gparams/s of the reference's PyTorch backend on the host CPU cores (all
    threads): ``luma_optimizer.LUMA(backend="pytorch")`` from baseline/_ref,
    unmodified, drawing its own uniforms every step.  Only if that install is
    missing, the oracle restatement of the same op sequence (fresh uniforms
    every step too).  The reference takes float32 params only
    (optimizer.py:443-448), so bf16-param configs run with float32 params."""
    cores = len(os.sched_getaffinity(0))
    torch.set_num_threads(cores)
    cfg = CONFIGS[config]
    shapes, sample = cpu_sample_shapes(config)
    g = torch.Generator().manual_seed(0)
    params = [torch.nn.Parameter(torch.randn(s, generator=g) * 0.02) for s in shapes]
    grads = [(torch.randn(s, generator=g) * cfg["gscale"]).to(cfg["gdt"]) for s in shapes]
    for p, gr in zip(params, grads):
        p.grad_dtype = None
        p.grad = gr
    ref = reference_package()
    if ref is not None:
        opt = ref.LUMA(params, lr=1e-3, backend="pytorch")
        kind, how = "reference", "luma_optimizer.LUMA(backend='pytorch') from baseline/_ref (unmodified)"
    else:
        from oracle.luma_ref import OracleLUMA  # test infrastructure: CPU baseline leg only

        def draws(pid, t, like):
            return torch.rand(like.shape, generator=g), torch.rand(like.shape, generator=g)

        opt = OracleLUMA(params, lr=1e-3, draws=draws)
        kind, how = "port", "oracle/luma_ref.py (reference op sequence; the reference install is absent)"
    n = sum(numel(s) for s in shapes)
    with torch.no_grad():
        for _ in range(max(warmup, 2)):
            opt.step()
        times = []
        t_end = time.perf_counter() + budget_s
        while len(times) < steps and (not times or time.perf_counter() < t_end):
            t0 = time.perf_counter()
            opt.step()
            times.append(time.perf_counter() - t0)
    t = statistics.median(times)
    return {"value": round(n / t / 1e9, 6), "unit": "Gparams/s", "cores": cores,
            "kind": kind, "steps_timed": len(times),
            "sample": f"{sample}; fp32 params, {str(cfg['gdt']).replace('torch.', '')} grads; "
                      f"median of {len(times)} steps after {max(warmup, 2)} warm-up; {how}"}


# ---------------------------------------------------------------------------
# the CUDA step
# ---------------------------------------------------------------------------

def fill_grads(cfg, grads, gen, seed=0):
    """Draw the config's grads in place (BASELINE.json value distributions)."""
    import numpy as np
    kind = cfg.get("grads", "normal")
    rng = np.random.default_rng(seed)
    sigmas = np.exp(rng.uniform(math.log(1e-4), math.log(1e-1), len(grads)))
    zero = rng.random(len(grads)) < 0.10
    for k, gr in enumerate(grads):
        gr.normal_(0.0, float(sigmas[k]) if kind == "sigma" else cfg["gscale"], generator=gen)
        if kind == "stress":
            if zero[k]:
                gr.zero_()
                continue
            u = torch.rand(gr.shape, device=gr.device, generator=gen)
            sgn = torch.where(torch.rand(gr.shape, device=gr.device, generator=gen) < 0.5, -1.0, 1.0)
            gr[u < 0.005] = 1e4
            gr[(u >= 0.005) & (u < 0.01)] = 1e-40
            gr.mul_(sgn.to(gr.dtype))


def make_workload(config, device, seed=0, pdt=None):
    cfg = CONFIGS[config]
    shapes = cfg["shapes"]()
    gen = torch.Generator(device=device).manual_seed(seed)
    params, grads = [], []
    for s in shapes:
        p = torch.empty(s, dtype=pdt or cfg["pdt"], device=device)
        p.normal_(0.0, 0.02, generator=gen)
        gr = torch.empty(s, dtype=cfg["gdt"], device=device)
        p.grad_dtype = None
        p.grad = gr
        params.append(p)
        grads.append(gr)
    fill_grads(cfg, grads, gen, seed)
    return shapes, params, grads


def run_luma(args, rank, world, local_rank):
    from luma_b200 import LUMA

    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    cfg = CONFIGS[args.config]
    shapes, params, grads = make_workload(args.config, device)
    n_params = sum(numel(s) for s in shapes)
    opt = LUMA(params, lr=1e-3, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.01)
    warmup = max(args.warmup, 1)
    for _ in range(warmup):
        opt.step()
    torch.cuda.synchronize()

    K = args.steps
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(K)]
    stream = torch.cuda.current_stream()
    for trio in evs:
        for e in trio:
            e.record(stream)
    torch.cuda.synchronize()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    sampler = ClockSampler(local_rank)
    sampler.start()
    time.sleep(0.3)
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    start.record(stream)
    for k in range(K):
        opt._step_events = tuple(e.cuda_event for e in evs[k])
        opt.step()
    stop.record(stream)
    torch.cuda.synchronize()
    opt._step_events = None
    clocks = sampler.stop()
    if world > 1:
        torch.distributed.barrier()
    total_ms = start.elapsed_time(stop)
    p1 = [evs[k][0].elapsed_time(evs[k][1]) for k in range(K)]
    p2 = [evs[k][1].elapsed_time(evs[k][2]) for k in range(K)]
    if world > 1:
        t = torch.tensor([total_ms], device=device)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        total_ms = float(t.item())
    ms_per_step = total_ms / K

    # e2e: every step's grads copied from pinned host memory, the step through
    # the public API (LUMA.step), the new per-tensor scales read back to pinned
    # host memory.  Two grad buffers: the upload of step k+1's grads (copy
    # engine, side stream) overlaps step k's kernels.
    e2e = None
    if not args.no_e2e:
        try:
            host = [torch.empty(g.shape, dtype=g.dtype, pin_memory=True) for g in grads]
            for h, g in zip(host, grads):
                h.copy_(g)
            h2d = sum(h.numel() * h.element_size() for h in host)
            eng = next(iter(opt._engines.values()))
            d2h = eng.slots.numel()
            bufs = [grads, [torch.empty_like(g) for g in grads]]
            out = [torch.empty(d2h, dtype=torch.uint8, pin_memory=True) for _ in range(2)]
            up = torch.cuda.Stream()
            main = torch.cuda.current_stream()
            copied = [torch.cuda.Event(), torch.cuda.Event()]
            stepped = [torch.cuda.Event(), torch.cuda.Event()]
            E = max(2, min(K, 5))
            torch.cuda.synchronize()
            t0 = time.perf_counter()

            def upload(k):
                b = k % 2
                with torch.cuda.stream(up):
                    if k >= 2:
                        up.wait_event(stepped[b])  # step k-2 is done with this buffer
                    for h, g in zip(host, bufs[b]):
                        g.copy_(h, non_blocking=True)
                    copied[b].record(up)

            upload(0)
            for k in range(E):
                if k + 1 < E:
                    upload(k + 1)
                b = k % 2
                main.wait_event(copied[b])
                for p, g in zip(params, bufs[b]):
                    p.grad = g
                opt.step()
                out[b].copy_(eng.slots, non_blocking=True)  # this step's S_m / S_v to host
                stepped[b].record(main)
            torch.cuda.synchronize()
            el = time.perf_counter() - t0
            e2e = {"value": round(n_params * E / el / 1e9, 3), "unit": "Gparams/s",
                   "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "steps": E,
                   "pipelining": "double-buffered grads: step k+1's upload overlaps step k"}
            for p, g in zip(params, grads):
                p.grad = g
            del host, bufs, out
        except Exception as exc:  # noqa: BLE001
            e2e = {"value": None, "unit": "Gparams/s", "error": str(exc)[:200]}

    p1b, p2b = bytes_per_param(cfg["pdt"], cfg["gdt"])
    peak, peak_kind = measured_peak()
    p2_ms = statistics.mean(p2)
    achieved = n_params * p2b / (p2_ms * 1e-3) / 1e9
    traffic_pp = committed_traffic(args.config)
    return {
        "n_params": n_params, "ms_per_step": ms_per_step, "pass1_ms": statistics.mean(p1),
        "pass2_ms": p2_ms, "bytes_per_param": p1b + p2b, "pass2_bytes_per_param": p2b,
        "roofline": {"bound": "hbm", "kernel": "luma_pass_kernel<pass2>",
                     "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "peak_source": peak_kind,
                     "traffic": (None if traffic_pp is None else int(traffic_pp * n_params)),
                     "traffic_source": (None if traffic_pp is None else
                                        f"not measured in this run: ncu dram__bytes_read.sum + "
                                        f"dram__bytes_write.sum of pass 2 per param "
                                        f"({traffic_pp} B) from profiles/luma_pass2_{args.config}"
                                        f".json (one Llama-3-8B layer), times this workload's "
                                        f"params")},
        "clocks": clocks, "e2e": e2e, "gpu_launches": 2 * K,
    }


def run_zero(args, rank, world, local_rank):
    """ZeRO-1: this rank steps its pieces of the whole model; the bf16 params
    are all-gathered in place over NCCL, bucket by bucket, each gather
    overlapping the next bucket's kernels (strong scaling)."""
    import torch.distributed as dist

    from luma_b200.zero import ZeroLUMA, alloc_flat, auto_gather, plan_layout

    device = torch.device("cuda", local_rank)
    cfg = CONFIGS[args.config]
    shapes = cfg["shapes"]()
    numels = [numel(s) for s in shapes]
    n_params = sum(numels)
    # A full bf16 replica plus the shard state must fit in HBM; otherwise the
    # params stay sharded and every bucket is gathered into a staging buffer.
    replica = args.config != "llama70b"
    buckets = args.buckets if replica else max(args.buckets, 32)
    lay = plan_layout(numels, world, buckets)
    gen = torch.Generator(device=device).manual_seed(0)
    if args.gather == "auto":
        gather = auto_gather(world) if replica else "nccl"  # as ZeroLUMA resolves it
    else:
        gather = args.gather
    flat = alloc_flat(lay.total if replica else lay.shard, cfg["pdt"], device,
                      gather if replica else "nccl")
    flat.normal_(0.0, 0.02, generator=gen)
    gshard = torch.empty(lay.shard, dtype=cfg["gdt"], device=device)
    gshard.normal_(0.0, cfg["gscale"], generator=gen)
    sms = torch.cuda.get_device_properties(device).multi_processor_count
    max_ctas = max(1, sms - args.reserve_sms) if args.reserve_sms > 0 else 0
    opt = ZeroLUMA(flat, lay, rank, lr=1e-3, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.01,
                   base_seed=1234, max_ctas=max_ctas, gather=gather,
                   copy_streams=args.copy_streams, replica=replica,
                   copy_lockstep=args.copy_lockstep)
    for _ in range(max(args.warmup, 1)):
        opt.step(gshard)
    torch.cuda.synchronize()
    K = args.steps
    stream = torch.cuda.current_stream()

    def timed(fn, sample_clocks=False):
        start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        sampler = ClockSampler(local_rank)
        if sample_clocks and rank == 0:
            sampler.start()
        time.sleep(0.3 if sample_clocks else 0.0)  # every rank: nobody enters late
        dist.barrier()
        torch.cuda.synchronize()
        start.record(stream)
        for _ in range(K):
            fn()
        stop.record(stream)
        torch.cuda.synchronize()
        clocks = sampler.stop() if (sample_clocks and rank == 0) else None
        dist.barrier()
        t = torch.tensor([start.elapsed_time(stop) / K], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item()), clocks

    ms_step, clocks = timed(lambda: opt.step(gshard), sample_clocks=True)

    # breakdown: the local kernels alone and the gathers alone
    ms_local, _ = timed(lambda: opt.step_local(gshard))
    ms_gather, _ = timed(opt.gather)
    e2e = None
    if not args.no_e2e:
        # as at N=1: double-buffered grad uploads, scales read back every step
        host = torch.empty(gshard.shape, dtype=gshard.dtype, pin_memory=True)
        host.copy_(gshard)
        bufs = [gshard, torch.empty_like(gshard)]
        d2h = sum(e.slots.numel() for e in opt.engines)
        out = [[torch.empty(e.slots.numel(), dtype=torch.uint8, pin_memory=True)
                for e in opt.engines] for _ in range(2)]
        up = torch.cuda.Stream()
        main = torch.cuda.current_stream()
        copied = [torch.cuda.Event(), torch.cuda.Event()]
        stepped = [torch.cuda.Event(), torch.cuda.Event()]
        E = max(2, min(K, 5))

        def upload(k):
            b = k % 2
            with torch.cuda.stream(up):
                if k >= 2:
                    up.wait_event(stepped[b])
                bufs[b].copy_(host, non_blocking=True)
                copied[b].record(up)

        dist.barrier()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        upload(0)
        for k in range(E):
            if k + 1 < E:
                upload(k + 1)
            b = k % 2
            main.wait_event(copied[b])
            opt.step(bufs[b])
            for o, e in zip(out[b], opt.engines):
                o.copy_(e.slots, non_blocking=True)
            stepped[b].record(main)
        torch.cuda.synchronize()
        el = torch.tensor([time.perf_counter() - t0], device=device)
        dist.all_reduce(el, op=dist.ReduceOp.MAX)
        e2e = {"value": round(n_params * E / float(el.item()) / 1e9, 3), "unit": "Gparams/s",
               "h2d_bytes_per_step": host.numel() * host.element_size(),
               "d2h_bytes_per_step": d2h, "steps": E,
               "pipelining": "double-buffered grad shards: step k+1's upload overlaps step k"}
        del bufs, out, host

    # consistency: after a full step every rank must hold the same replica
    check = None
    if replica:
        opt.step(gshard)
        torch.cuda.synchronize()
        bits = flat.view(torch.int16 if flat.element_size() == 2 else torch.int32)
        sig = torch.zeros(2, dtype=torch.int64, device=device)
        chunk = 1 << 28  # widened to int64 a chunk at a time
        for lo in range(0, bits.numel(), chunk):
            words = bits[lo:lo + chunk].to(torch.int64)
            pos = torch.arange(lo, lo + words.numel(), device=device, dtype=torch.int64) % 65521 + 1
            sig += torch.stack([words.sum(), (words * pos).sum()])
        del words, pos
        sigs = [torch.empty_like(sig) for _ in range(world)]
        dist.all_gather(sigs, sig)
        check = {"replicas_equal": all(torch.equal(sigs[0], x) for x in sigs),
                 "how": "after one more step: sum and position-weighted sum of every rank's "
                        "replica bits, all-gathered and compared"}
    opt.close()
    p1b, p2b = bytes_per_param(cfg["pdt"], cfg["gdt"])
    peak, peak_kind = measured_peak()
    # pass-2 share of the local step, from the single-GPU split (pass 2 ~ 83%):
    # the roofline here is the local step's algorithmic bytes over its time
    achieved = lay.shard * (p1b + p2b) / (ms_local * 1e-3) / 1e9
    gather_bytes = (world - 1) * lay.shard * flat.element_size()
    return {
        "n_params": n_params, "ms_per_step": ms_step, "pass1_ms": None,
        "pass2_ms": None, "local_step_ms": ms_local, "allgather_ms": ms_gather,
        "allgather_gbs_per_rank": round(gather_bytes / (ms_gather * 1e-3) / 1e9, 1),
        "overlap_saving_ms": round(ms_local + ms_gather - ms_step, 3),
        "step_only_gparams": round(n_params / (ms_local * 1e-3) / 1e9, 3),
        "shard_params": lay.shard, "buckets": lay.buckets, "max_ctas": max_ctas,
        "gather": opt.gather_mode, "replica": replica, "check": check,
        # fused (nvls) gather: bytes each rank receives over the whole step time,
        # a lower bound of the rate its links sustained while the step ran
        "gather_in_step_gbs_per_rank": (round(gather_bytes / (ms_step * 1e-3) / 1e9, 1)
                                        if opt.gather_mode == "nvls" else None),
        "bytes_per_param": p1b + p2b, "pass2_bytes_per_param": p2b,
        "roofline": {"bound": "hbm", "kernel": "luma_pass_kernel<false>+<true> (local step)",
                     "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "peak_source": peak_kind,
                     "traffic": None},
        "clocks": clocks, "e2e": e2e, "gpu_launches": 2 * lay.buckets * K,
    }


def result_line(args, res, world, scaling, dtype, config_out):
    """The driver's JSON line from a run's measurements (rank 0)."""
    n = res["n_params"]
    ms = res["ms_per_step"]
    value = n / (ms * 1e-3) / 1e9
    if res.get("local_step_ms") is not None:
        kernel_ms = res["local_step_ms"]
    else:
        kernel_ms = res["pass1_ms"] + res["pass2_ms"]
    hbm = n / world * res["bytes_per_param"] / (kernel_ms * 1e-3) / 1e9
    peak, _ = measured_peak()
    line = {"metric": METRIC, "value": round(value, 3), "unit": "Gparams/s",
            "n_gpus": world, "steps": args.steps, "warmup": max(args.warmup, 1),
            "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": scaling,
            "vs_baseline": None, "dtype": dtype, "data": "synthetic", "config": config_out,
            "hbm_gbs_per_gpu": round(hbm, 1),
            "hbm_frac_of_measured_peak": round(hbm / peak, 4),
            "hbm_frac_of_nominal_8tbs": round(hbm / NOMINAL_HBM_GBS, 4),
            "pass1_ms": None if res.get("pass1_ms") is None else round(res["pass1_ms"], 4),
            "pass2_ms": None if res.get("pass2_ms") is None else round(res["pass2_ms"], 4),
            "roofline": res["roofline"], "clocks": res["clocks"], "e2e": res["e2e"],
            "gpu_launches": res["gpu_launches"]}
    for key in ("local_step_ms", "allgather_ms", "allgather_gbs_per_rank", "overlap_saving_ms",
                "step_only_gparams", "shard_params", "buckets", "max_ctas", "gather", "replica",
                "check", "gather_in_step_gbs_per_rank"):
        if key in res:
            line[key] = res[key]
    return line


def reference_gpu(args, warmup: int = 2, steps: int = 3) -> dict:
    """This backend and the reference's own GPU kernels (its Triton backend,
    installed unmodified into baseline/_ref) stepping the same params and grads
    of the config's shapes, one after the other on this GPU; CUDA events over
    the timed steps.  The reference takes fp32 params only
    (optimizer.py:443-448), so both run fp32 params with the config's grad
    dtype.  Its kernels receive param_id as a plain int that Triton
    specialises to a constant for 0 and 1 (then `param_id.to(tl.int64)` fails
    to compile, at the first step of a fresh model), so two gradless tensors
    come first and the stepped tensors have ids >= 2; the reference's code
    path itself is unchanged."""
    ref = reference_package()
    if ref is None:
        return {"impl": "reference-triton", "unavailable": "reference not installed in baseline/_ref"}
    from luma_b200 import LUMA
    cfg = CONFIGS[args.config]
    n = sum(numel(s) for s in cfg["shapes"]())

    def timeit(make_opt):
        torch.cuda.empty_cache()
        _, params, _ = make_workload(args.config, torch.device("cuda"), pdt=torch.float32)
        opt = make_opt(params)
        for _ in range(warmup):
            opt.step()
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(steps):
            opt.step()
        e.record()
        torch.cuda.synchronize()
        del opt, params
        return s.elapsed_time(e) / steps

    try:
        ours = timeit(lambda ps: LUMA(ps, lr=1e-3))
        dummies = [torch.zeros(8, device="cuda") for _ in range(2)]
        theirs = timeit(lambda ps: ref.LUMA(dummies + ps, lr=1e-3, backend="triton"))
    except Exception as exc:  # noqa: BLE001
        return {"impl": "reference-triton", "unavailable": f"{type(exc).__name__}: {str(exc)[:160]}"}
    finally:
        torch.cuda.empty_cache()
    gdt = str(cfg["gdt"]).replace("torch.", "")
    return {"impl": "reference Triton backend (baseline/_ref, unmodified) vs luma_b200, same GPU",
            "workload": f"{args.config} shapes, fp32 params (the reference requires fp32), "
                        f"{gdt} grads", "params": n, "warmup": warmup, "steps": steps,
            "luma_b200_ms": round(ours, 3), "reference_triton_ms": round(theirs, 3),
            "luma_b200_gparams": round(n / ours / 1e6, 3),
            "reference_triton_gparams": round(n / theirs / 1e6, 3),
            "speedup": round(theirs / ours, 2)}


# ---------------------------------------------------------------------------
# end-to-end training: GPT-2 small on uniform-random tokens
# ---------------------------------------------------------------------------

class _Block(torch.nn.Module):
    def __init__(self, d, heads, layers):
        super().__init__()
        nn = torch.nn
        self.heads = heads
        self.ln_1, self.ln_2 = nn.LayerNorm(d), nn.LayerNorm(d)
        self.c_attn, self.attn_proj = nn.Linear(d, 3 * d), nn.Linear(d, d)
        self.c_fc, self.mlp_proj = nn.Linear(d, 4 * d), nn.Linear(4 * d, d)
        for lin in (self.attn_proj, self.mlp_proj):  # GPT-2's residual-projection init
            torch.nn.init.normal_(lin.weight, 0.0, 0.02 / math.sqrt(2 * layers))

    def forward(self, x):
        B, T, C = x.shape
        q, k, v = self.c_attn(self.ln_1(x)).split(C, dim=2)
        q, k, v = (t.view(B, T, self.heads, C // self.heads).transpose(1, 2) for t in (q, k, v))
        y = torch.nn.functional.scaled_dot_product_attention(q, k, v, is_causal=True)
        x = x + self.attn_proj(y.transpose(1, 2).reshape(B, T, C))
        return x + self.mlp_proj(torch.nn.functional.gelu(self.c_fc(self.ln_2(x)),
                                                          approximate="tanh"))


class GPT2Small(torch.nn.Module):
    """GPT-2 small (12 layers, d=768, 12 heads, vocab 50257, ctx 1024, lm_head
    tied to the token embedding): 148 parameter tensors, 124,439,808 params."""

    def __init__(self, vocab=50257, ctx=1024, d=768, layers=12, heads=12):
        super().__init__()
        nn = torch.nn
        self.wte, self.wpe = nn.Embedding(vocab, d), nn.Embedding(ctx, d)
        for emb in (self.wte, self.wpe):
            torch.nn.init.normal_(emb.weight, 0.0, 0.02)
        self.blocks = nn.ModuleList(_Block(d, heads, layers) for _ in range(layers))
        self.ln_f = nn.LayerNorm(d)
        self.lm_head = nn.Linear(d, vocab, bias=False)
        self.lm_head.weight = self.wte.weight
        for mod in self.modules():
            if isinstance(mod, nn.Linear) and mod.bias is not None:
                torch.nn.init.zeros_(mod.bias)

    def forward(self, idx, targets):
        pos = torch.arange(idx.shape[1], device=idx.device)
        x = self.wte(idx) + self.wpe(pos)
        for blk in self.blocks:
            x = blk(x)
        logits = self.lm_head(self.ln_f(x))
        return torch.nn.functional.cross_entropy(logits.float().view(-1, logits.shape[-1]),
                                                 targets.view(-1))


def run_nanogpt(args) -> dict:
    """LUMA (this backend) and torch's fused AdamW train GPT-2 small side by
    side from the same init on the same uniform-random token batches (12 x
    1024), bf16 autocast, grad-norm clipping at 1.0 before every step (the
    reference's nanoGPT loop, benchmarks/bench_nanogpt.py:211-226; for LUMA
    the clip is fused into the step with clip_grad_coef).  Reports training
    throughput (tokens/s), optimizer-step time and the two loss trajectories."""
    from luma_b200 import LUMA, clip_grad_coef
    dev = torch.device("cuda")
    B, T, V = 12, 1024, 50257
    hp = dict(lr=6e-4, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1)
    torch.manual_seed(1337)
    m_adamw = GPT2Small().to(dev)
    m_luma = GPT2Small().to(dev)
    m_luma.load_state_dict(m_adamw.state_dict())
    n_params = sum(p.numel() for p in m_luma.parameters())
    o_adamw = torch.optim.AdamW(m_adamw.parameters(), fused=True, **hp)
    o_luma = LUMA(m_luma.parameters(), **hp)
    gen = torch.Generator(device=dev).manual_seed(42)
    stream = torch.cuda.current_stream()

    def train_step(model, opt, x, y, luma):
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
        ev[0].record(stream)
        with torch.autocast("cuda", dtype=torch.bfloat16):
            loss = model(x, y)
        opt.zero_grad(set_to_none=True)
        loss.backward()
        ev[1].record(stream)
        if luma:
            _, coef = clip_grad_coef(model.parameters(), 1.0)
            opt.step(grad_scale=coef)
        else:
            torch.nn.utils.clip_grad_norm_(model.parameters(), 1.0)
            opt.step()
        ev[2].record(stream)
        return loss.detach(), ev

    total = max(args.warmup, 3) + args.steps
    losses = {"luma": [], "adamw": []}
    times = {"luma": [], "adamw": []}
    for it in range(total):
        x = torch.randint(0, V, (B, T), device=dev, generator=gen)
        y = torch.randint(0, V, (B, T), device=dev, generator=gen)
        la, ea = train_step(m_adamw, o_adamw, x, y, False)
        ll, el = train_step(m_luma, o_luma, x, y, True)
        torch.cuda.synchronize()
        losses["adamw"].append(float(la))
        losses["luma"].append(float(ll))
        if it >= total - args.steps:
            times["adamw"].append((ea[0].elapsed_time(ea[2]), ea[1].elapsed_time(ea[2])))
            times["luma"].append((el[0].elapsed_time(el[2]), el[1].elapsed_time(el[2])))
    out = {}
    for k in ("luma", "adamw"):
        step_ms = statistics.median(t[0] for t in times[k])
        opt_ms = statistics.median(t[1] for t in times[k])
        out[k] = {"train_step_ms": round(step_ms, 3), "optimizer_step_ms": round(opt_ms, 4),
                  "tokens_per_s": round(B * T / (step_ms * 1e-3), 1)}
    gap = max(abs(a - b) / b for a, b in zip(losses["luma"], losses["adamw"]))
    marks = sorted({0, total // 4, total // 2, total - 1})
    return {"metric": "GPT-2 small training throughput (nanoGPT-style, uniform-random tokens, "
                      "batch 12x1024), LUMA step on this backend",
            "value": out["luma"]["tokens_per_s"], "unit": "tokens/s", "n_gpus": 1,
            "steps": args.steps, "warmup": max(args.warmup, 3), "higher_is_better": True,
            "data": "synthetic (uniform-random token ids)", "dtype": "bf16 autocast, fp32 params",
            "config": {"workload": "GPT-2 small (124,439,808 params, 148 tensors), batch 12x1024, "
                                   "lr 6e-4, betas (0.9, 0.95), wd 0.1, clip 1.0",
                       "n_params": n_params},
            "luma": out["luma"], "adamw_fused": out["adamw"],
            "loss": {f"step{k + 1}": {"luma": round(losses["luma"][k], 4),
                                      "adamw": round(losses["adamw"][k], 4)} for k in marks},
            "max_rel_loss_gap": round(gap, 5), "gpu_launches": None}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="luma", choices=["luma", "reference"])
    ap.add_argument("--config", default="llama8b", choices=sorted(CONFIGS) + ["nanogpt"])
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--buckets", type=int, default=8,
                    help="N>1: gather buckets (each bucket's gather overlaps the next's kernels)")
    ap.add_argument("--reserve-sms", type=int, default=0,
                    help="N>1, NCCL gather (and copy gather in lockstep): SMs the step kernels "
                         "leave free for NCCL kernels while a gather is in flight")
    ap.add_argument("--copy-streams", type=int, default=1,
                    help="N>1, copy gather: streams the peer pushes are spread over (0: one per peer)")
    ap.add_argument("--copy-lockstep", action="store_true",
                    help="N>2, copy gather on one stream: a barrier between a bucket's pushes, so "
                         "every GPU receives from one peer at a time")
    ap.add_argument("--gather", default="auto", choices=["auto", "nccl", "copy", "nvls"],
                    help="N>1: post-step all-gather by NCCL, by copy-engine pushes over CUDA IPC, "
                         "or fused into pass 2 as NVLink multicast stores (nvls)")
    ap.add_argument("--no-reference-gpu", action="store_true",
                    help="one GPU: skip timing the reference's Triton backend beside this one")
    ap.add_argument("--vs-triton", action="store_true",
                    help="one GPU: also time the reference's Triton backend (baseline/_ref) on the "
                         "config's shapes in fp32 and print a comparison line")
    args = ap.parse_args()
    if args.vs_triton:
        print(json.dumps(reference_gpu(args, warmup=max(args.warmup, 2), steps=args.steps)))
        return

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.config == "nanogpt":
        if rank == 0 and args.impl == "luma":
            print(json.dumps(run_nanogpt(args)))
        return
    cfg = CONFIGS[args.config]
    p1b, p2b = bytes_per_param(cfg["pdt"], cfg["gdt"])
    dtype = "f32 math; params " + str(cfg["pdt"]).replace("torch.", "") + ", grads " + \
        str(cfg["gdt"]).replace("torch.", "") + ", codes int16"
    config_out = {"workload": cfg["name"], "bytes_per_param": p1b + p2b,
                  "l2": "inputs larger than L2 (resident params+grads+codes >> 126 MB)"
                  if args.config in ("llama8b", "llama70b", "ragged", "llama_layer") else "working set may fit L2",
                  "parallelism": (f"zero1-dp{world} (flat shards, per-shard scales, post-step "
                                  f"bf16 param all-gather)" if world > 1 else "single")}

    if args.impl == "reference":
        if rank != 0:
            return
        cb = cpu_baseline(args.config, args.steps, args.warmup, budget_s=60.0)
        # the same config as this backend's line; the reference's own param
        # dtype (it rejects bf16 params) is stated beside it
        line = {"impl": "reference", "metric": METRIC, "value": cb["value"], "unit": "Gparams/s",
                "n_gpus": args.gpus, "steps": cb["steps_timed"], "warmup": max(args.warmup, 2),
                "higher_is_better": True, "scaling": "strong" if world > 1 else "weak",
                "vs_baseline": None, "dtype": dtype, "data": "synthetic", "config": config_out,
                "reference_params": "float32 (the reference rejects bf16 params)",
                "cpu_baseline": cb,
                "e2e": {"value": cb["value"], "unit": "Gparams/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}}
        print(json.dumps(line))
        return

    if world > 1:
        import datetime
        torch.cuda.set_device(local_rank)
        torch.distributed.init_process_group("nccl", device_id=torch.device("cuda", local_rank),
                                             timeout=datetime.timedelta(seconds=300))
        res = run_zero(args, rank, world, local_rank)
        scaling = "strong"
    else:
        if args.config == "llama70b":
            raise SystemExit("llama70b: 141 GB of bf16 params do not fit one GPU with their "
                             "state; run it on 8 GPUs (params sharded)")
        res = run_luma(args, rank, world, local_rank)
        scaling = "weak"
    if rank == 0:
        line = result_line(args, res, world, scaling, dtype, config_out)
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline(args.config, 10, 2)
        if world == 1 and not args.no_reference_gpu:
            line["reference_gpu"] = reference_gpu(args)
        print(json.dumps(line))
    if world > 1:
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
