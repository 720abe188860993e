"""Generate the golden LUMA step vectors from the reference implementation.

Run in a container where the reference (IgorYashch/LUMA) is checked out:

    python tests/golden/make_golden.py --reference /path/to/LUMA/src

It imports ``luma_optimizer`` from that tree, replaces the ``torch.rand``
calls of its functional backend (functional.py:144, 170) with uniforms drawn
from a seeded numpy stream, steps ``LUMA(backend="pytorch")`` on CPU tensors
and records every input and output per step into ``tests/golden/<case>.npz``.
bf16-param cases run the reference on a float32 copy and round the param to
bf16 (nearest even) after every step, the bf16 contract of the CUDA backend.

The fixtures are small (a few thousand elements per case) so the CPU test
suite replays them in seconds.
"""

from __future__ import annotations

import argparse
import json
import os
import sys
import types

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))

DT = {"f32": torch.float32, "bf16": torch.bfloat16, "f16": torch.float16}


def _uniforms(rng: np.random.Generator, shape) -> torch.Tensor:
    n = int(np.prod(shape)) if len(shape) else 1
    u = (rng.integers(0, 1 << 24, size=n, dtype=np.int64).astype(np.float32)
         * np.float32(2.0 ** -24))
    return torch.from_numpy(u.reshape(shape))


def _grad(rng: np.random.Generator, shape, kind: str, scale: float) -> np.ndarray:
    n = int(np.prod(shape)) if len(shape) else 1
    g = rng.standard_normal(n).astype(np.float32) * np.float32(scale)
    if kind == "zero":
        g[:] = 0
    elif kind == "outlier":
        k = max(1, n // 20)
        idx = rng.choice(n, size=k, replace=False)
        g[idx[: k // 2]] = np.float32(1e4) * np.sign(rng.standard_normal(k // 2)).astype(np.float32)
        g[idx[k // 2:]] = np.float32(1e-40) * np.sign(rng.standard_normal(k - k // 2)).astype(np.float32)
    elif kind == "const":
        g[:] = np.float32(scale)
    return g.reshape(shape)


# Each case: list of param specs, groups, steps.  Param spec: (shape, param
# dtype, grad dtype, grad kind, grad scale, group index, steps without grad).
CASES = {
    "basic_f32": dict(
        params=[((37,), "f32", "f32", "normal", 1e-2, 0, []),
                ((8, 9), "f32", "f32", "normal", 1e-1, 0, []),
                ((), "f32", "f32", "normal", 1.0, 0, [])],
        groups=[dict(lr=1e-3, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.01)],
        steps=6),
    "grad_bf16_f16": dict(
        params=[((64, 33), "f32", "bf16", "normal", 1e-3, 0, []),
                ((100,), "f32", "f16", "normal", 1e-2, 0, [])],
        groups=[dict(lr=3e-4, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1)],
        steps=4),
    "param_bf16": dict(
        params=[((50, 20), "bf16", "bf16", "normal", 1e-3, 0, []),
                ((17,), "bf16", "f32", "normal", 1e-2, 0, [])],
        groups=[dict(lr=1e-3, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.01)],
        steps=4),
    "zero_and_outliers": dict(
        params=[((129,), "f32", "f32", "zero", 0.0, 0, []),
                ((300,), "f32", "f32", "outlier", 1e-2, 0, []),
                ((65,), "f32", "f32", "const", 3e-3, 0, [])],
        groups=[dict(lr=1e-3, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.01)],
        steps=4),
    "groups_and_skips": dict(
        params=[((40,), "f32", "f32", "normal", 1e-2, 0, [2]),
                ((33, 3), "f32", "bf16", "normal", 1e-3, 1, []),
                ((9,), "f32", "f32", "normal", 1e-1, 1, [1, 4])],
        groups=[dict(lr=1e-2, betas=(0.8, 0.99), eps=1e-6, weight_decay=0.0),
                dict(lr=5e-4, betas=(0.95, 0.9999), eps=1e-10, weight_decay=0.05)],
        steps=5),
    "lr_zero_and_big_eps": dict(
        params=[((31,), "f32", "f32", "normal", 1e-2, 0, []),
                ((24,), "f32", "f32", "normal", 1e-20, 1, [])],
        groups=[dict(lr=0.0, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.0),
                dict(lr=1e-3, betas=(0.9, 0.999), eps=1.0, weight_decay=0.01)],
        steps=3),
    "ragged": dict(
        params=[((n,), "f32", "f32", "normal", s, 0, [])
                for n, s in [(1, 1e-2), (7, 1e-3), (8, 1e-2), (9, 1e-1), (15, 1e-2),
                             (16, 1e-4), (127, 1e-2), (255, 1e-3), (1025, 1e-2), (513, 1.0)]],
        groups=[dict(lr=1e-3, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.01)],
        steps=3),
    "long_run": dict(
        params=[((2000,), "f32", "f32", "normal", 1e-2, 0, [])],
        groups=[dict(lr=1e-2, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.01)],
        steps=20),
}


class _RandFeeder:
    """Stand-in for the ``torch`` module inside the reference's functional.py:
    forwards everything to torch except ``rand``, which returns queued draws."""

    def __init__(self):
        self.queue: list[torch.Tensor] = []

    def make_module(self):
        feeder = self
        mod = types.ModuleType("torch_with_fed_rand")

        def rand(*size, dtype=None, device=None, generator=None, **kw):
            shape = tuple(size[0]) if len(size) == 1 and isinstance(size[0], (tuple, list, torch.Size)) else tuple(size)
            u = feeder.queue.pop(0)
            assert tuple(u.shape) == shape, (u.shape, shape)
            return u.to(dtype=dtype or torch.float32, device=device or "cpu")

        mod.__dict__.update({k: getattr(torch, k) for k in dir(torch) if not k.startswith("__")})
        mod.rand = rand
        return mod


def run_case(name: str, spec: dict, LUMA, F, seed: int) -> dict:
    rng = np.random.default_rng(seed)
    feeder = _RandFeeder()
    saved_torch = F.torch
    F.torch = feeder.make_module()
    out: dict[str, np.ndarray] = {}
    meta = {"name": name, "steps": spec["steps"], "groups": spec["groups"], "params": []}
    try:
        ref_params = []      # float32 tensors stepped by the reference
        for i, (shape, pdt, gdt, kind, scale, gi, skips) in enumerate(spec["params"]):
            n = int(np.prod(shape)) if len(shape) else 1
            p0 = (rng.standard_normal(n).astype(np.float32) * np.float32(0.02)).reshape(shape)
            p = torch.from_numpy(p0.copy())
            if pdt == "bf16":
                p = p.bfloat16().float()
            out[f"p0_{i}"] = p.bfloat16().view(torch.int16).numpy() if pdt == "bf16" else p.numpy().copy()
            param = torch.nn.Parameter(p)
            param.grad_dtype = None  # grads may be bf16/fp16 (autocast-style)
            ref_params.append(param)
            meta["params"].append(dict(shape=list(shape), param_dtype=pdt, grad_dtype=gdt,
                                       group=gi, skips=skips))
        groups = []
        for gi, g in enumerate(spec["groups"]):
            ps = [ref_params[i] for i, s in enumerate(spec["params"]) if s[5] == gi]
            groups.append(dict(params=ps, lr=g["lr"], betas=tuple(g["betas"]), eps=g["eps"],
                               weight_decay=g["weight_decay"]))
        torch.manual_seed(seed)
        opt = LUMA(groups, backend="pytorch")
        meta["base_seed"] = opt._base_seed
        order = [p for g in groups for p in g["params"]]
        index_of = {id(p): i for i, p in enumerate(ref_params)}
        for s in range(1, spec["steps"] + 1):
            for p in ref_params:
                p.grad = None
            for p in order:
                i = index_of[id(p)]
                shape, pdt, gdt, kind, scale, gi, skips = spec["params"][i]
                if s in skips:
                    continue
                g = torch.from_numpy(_grad(rng, tuple(shape), kind, scale)).to(DT[gdt])
                p.grad = g
                key = f"g_{s}_{i}"
                out[key] = g.view(torch.int16).numpy().copy() if gdt != "f32" else g.numpy().copy()
                um = _uniforms(rng, tuple(shape))
                uw = _uniforms(rng, tuple(shape))
                out[f"um_{s}_{i}"] = um.numpy().copy()
                out[f"uw_{s}_{i}"] = uw.numpy().copy()
                feeder.queue += [um, uw]
            opt.step()
            assert not feeder.queue, "unconsumed draws"
            for i, p in enumerate(ref_params):
                if spec["params"][i][1] == "bf16":
                    p.data.copy_(p.data.bfloat16().float())
                    out[f"p_{s}_{i}"] = p.data.bfloat16().view(torch.int16).numpy().copy()
                else:
                    out[f"p_{s}_{i}"] = p.data.numpy().copy()
                st = opt.state[p]
                if st:
                    out[f"qm_{s}_{i}"] = st["Q_m"].numpy().copy()
                    out[f"qw_{s}_{i}"] = st["Q_w"].numpy().copy()
                    out[f"S_{s}_{i}"] = np.array([st["S_m"], st["S_v"]], dtype=np.float64)
                    out[f"t_{s}_{i}"] = np.array([st["step"]], dtype=np.int64)
    finally:
        F.torch = saved_torch
    out["meta"] = np.frombuffer(json.dumps(meta).encode(), dtype=np.uint8)
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="path to the reference's src/ directory")
    ap.add_argument("--out", default=HERE)
    args = ap.parse_args()
    sys.path.insert(0, args.reference)
    from luma_optimizer import LUMA  # noqa: E402
    from luma_optimizer import functional as F  # noqa: E402

    torch.set_num_threads(1)
    for k, (name, spec) in enumerate(sorted(CASES.items())):
        arrays = run_case(name, spec, LUMA, F, seed=1000 + k)
        path = os.path.join(args.out, f"{name}.npz")
        np.savez_compressed(path, **arrays)
        print(f"{name}: {len(arrays)} arrays -> {os.path.relpath(path)} "
              f"({os.path.getsize(path) // 1024} KB)")


if __name__ == "__main__":
    main()
