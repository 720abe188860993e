"""Loader and replay helpers for the golden fixtures in tests/golden/.

Each ``<case>.npz`` holds one run of the reference LUMA (backend "pytorch",
CPU) with injected uniforms: initial params ``p0_i``, per step ``s`` the
grads ``g_s_i``, uniforms ``um_s_i``/``uw_s_i`` and the outputs ``p_s_i``,
``qm_s_i``, ``qw_s_i``, ``S_s_i`` (S_m, S_v) and ``t_s_i`` (state step).
bf16/fp16 arrays are stored as their int16 bit patterns.
"""

from __future__ import annotations

import glob
import json
import os

import numpy as np
import torch

GOLDEN_DIR = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
DT = {"f32": torch.float32, "bf16": torch.bfloat16, "f16": torch.float16}


def case_names() -> list[str]:
    return sorted(os.path.basename(p)[:-4] for p in glob.glob(os.path.join(GOLDEN_DIR, "*.npz")))


class GoldenCase:
    def __init__(self, name: str):
        self.name = name
        z = np.load(os.path.join(GOLDEN_DIR, f"{name}.npz"))
        self.arr = {k: z[k] for k in z.files}
        self.meta = json.loads(bytes(self.arr.pop("meta")).decode())
        self.steps = self.meta["steps"]
        self.specs = self.meta["params"]
        self.base_seed = self.meta["base_seed"]
        # param_id = position in group order (the reference's enumeration)
        order = []
        for gi in range(len(self.meta["groups"])):
            order += [i for i, s in enumerate(self.specs) if s["group"] == gi]
        self.order = order
        self.param_id_of = {i: k for k, i in enumerate(order)}

    def _tensor(self, key: str, dt: str, shape) -> torch.Tensor:
        a = self.arr[key]
        t = torch.from_numpy(a.copy())
        if dt != "f32":
            t = t.view(DT[dt])
        return t.reshape(shape)

    def make_params(self, device) -> list[torch.Tensor]:
        ps = []
        for i, s in enumerate(self.specs):
            t = self._tensor(f"p0_{i}", s["param_dtype"], tuple(s["shape"])).to(device)
            t.requires_grad_(True)
            t.grad_dtype = None
            ps.append(t)
        return ps

    def groups(self, params) -> list[dict]:
        out = []
        for gi, g in enumerate(self.meta["groups"]):
            out.append(dict(params=[params[i] for i in self.order if self.specs[i]["group"] == gi],
                            lr=g["lr"], betas=tuple(g["betas"]), eps=g["eps"],
                            weight_decay=g["weight_decay"]))
        return out

    def set_grads(self, params, step: int) -> None:
        for i, (p, s) in enumerate(zip(params, self.specs)):
            key = f"g_{step}_{i}"
            if key in self.arr:
                p.grad = self._tensor(key, s["grad_dtype"], tuple(s["shape"])).to(p.device)
            else:
                p.grad = None

    def draws(self, step: int, device) -> dict[int, tuple[torch.Tensor, torch.Tensor]]:
        """param_id -> (u_m, u_w) for this step."""
        out = {}
        for i, s in enumerate(self.specs):
            key = f"um_{step}_{i}"
            if key in self.arr:
                shape = tuple(s["shape"])
                out[self.param_id_of[i]] = (
                    torch.from_numpy(self.arr[key].copy()).reshape(shape).to(device),
                    torch.from_numpy(self.arr[f"uw_{step}_{i}"].copy()).reshape(shape).to(device))
        return out

    def expected(self, step: int, i: int) -> dict:
        s = self.specs[i]
        out = {"p": self._tensor(f"p_{step}_{i}", s["param_dtype"], tuple(s["shape"]))}
        if f"qm_{step}_{i}" in self.arr:
            out["qm"] = torch.from_numpy(self.arr[f"qm_{step}_{i}"].copy())
            out["qw"] = torch.from_numpy(self.arr[f"qw_{step}_{i}"].copy())
            out["S"] = tuple(float(x) for x in self.arr[f"S_{step}_{i}"])
            out["t"] = int(self.arr[f"t_{step}_{i}"][0])
        return out
