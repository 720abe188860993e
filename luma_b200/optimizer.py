"""LUMA optimizer — ``torch.optim.Optimizer`` front end of the B200 backend.

Drop-in for ``luma_optimizer.LUMA`` (IgorYashch/LUMA
src/luma_optimizer/optimizer.py:39-524): same constructor, same per-parameter
state (``step``, ``param_id``, ``Q_m``, ``Q_w`` int16, and ``S_m``/``S_v`` in
``state_dict()``), same ``_base_seed`` seeding, same ``export_adamw_state`` /
``import_adamw_state``.  The step itself runs as two sm_100a launches over
every parameter at once (``libluma_b200.so``, reached through ctypes); there
is no per-tensor Python work beyond validation and bookkeeping, no host
synchronisation and no CPU fallback.

Backends: ``"cuda"`` (this package) — ``"auto"`` and ``"triton"`` select it
too, since it replaces the reference's Triton backend.  The reference's
``"pytorch"`` backend is not part of this package.
"""

from __future__ import annotations

import ctypes
import math

import numpy as np
import torch
from torch.optim import Optimizer

from . import _lib
from .engine import Columns, DeviceEngine, Segment
from .hostmath import SCALE_FLOOR_M, grid_record, precompute, rows_array, step_row, step_rows

_BACKENDS = {"auto", "cuda", "triton"}
_PLAIN_TENSOR_TYPES = (torch.Tensor, torch.nn.Parameter)
_GRAD_CODE = {torch.float32: _lib.F32, torch.bfloat16: _lib.BF16, torch.float16: _lib.F16}
_PARAM_CODE = {torch.float32: _lib.F32, torch.bfloat16: _lib.BF16}


def _ParamEntry(p, param: torch.Tensor) -> list:
    """What holds for a parameter while its storage, size and dtype stay (one
    address is never on two devices): [p, param, data_ptr, numel, dtype,
    device index, shape, dtype code, state dict (set by the first step that
    uses the entry), descriptor tuple or None].  Raises for a param the step
    cannot take."""
    numel = param.numel()
    if numel:
        if param.dtype not in _PARAM_CODE:
            raise ValueError(
                f"LUMA requires float32 or bfloat16 parameters (got {param.dtype}).")
        if not param.is_cuda:
            raise RuntimeError(
                f"LUMA backend 'cuda' requires CUDA tensors (param on {param.device}).")
    return [p, param, param.data_ptr(), numel, param.dtype, param.get_device(), param.shape,
            _PARAM_CODE.get(param.dtype, -1), None, None]


class LUMA(Optimizer):
    r"""LUMA: Log-space Unbiased Momentum AdamW, B200 backend.

    Parameters
    ----------
    params : iterable of parameters or parameter-group dicts.
    lr : float, learning rate (default 1e-3).
    betas : (float, float), EMA coefficients (default (0.9, 0.999)).
    eps : float, denominator term (default 1e-8).
    weight_decay : float, decoupled weight decay (default 0.01).
    backend : "auto" | "cuda" | "triton" — all run the CUDA kernels.
    capturable : bool (default False).  True makes ``step()`` safe to capture
        in a CUDA graph and replay (like the reference's Triton backend,
        optimizer.py:18-19, 382-387): the step count of every parameter lives
        on the device and advances inside the launch, and the per-step scalars
        come from a device table with one row per (param group, step) for
        steps 1..capture_steps, built from the group hyper-parameters.  After
        changing a hyper-parameter (an LR schedule), call
        ``refresh_capturable_rows()`` outside the graph; replays read the
        refreshed table.  Take at least one eager step before capturing.
    capture_steps : int (default 2**17), rows per group in capturable mode; a
        step past it is skipped and reported by ``kernel_error_flags()``.

    Params may be float32 or bfloat16 (bf16 params are updated in float32
    arithmetic and rounded once to bf16, nearest even); grads float32,
    bfloat16 or float16.  All tensors must be contiguous CUDA tensors.

    Stochastic rounding draws come from Philox4x32-10 keyed by
    ``((step << 32) | 2*param_id) ^ _base_seed`` with the element index as
    counter, so every rank with the same ``_base_seed`` produces the same
    codes (DDP) and a checkpoint round trip resumes bit for bit.
    """

    def __init__(self, params, lr: float = 1e-3, betas: tuple[float, float] = (0.9, 0.999),
                 eps: float = 1e-8, weight_decay: float = 0.01, backend: str = "auto",
                 capturable: bool = False, capture_steps: int = 1 << 17):
        # Validation order and messages follow optimizer.py:80-89.
        if lr < 0.0:
            raise ValueError(f"Invalid learning rate: {lr}")
        if eps <= 0.0:
            raise ValueError(f"Invalid epsilon: {eps}")
        if not 0.0 <= betas[0] < 1.0:
            raise ValueError(f"Invalid beta1: {betas[0]}")
        if not 0.0 <= betas[1] < 1.0:
            raise ValueError(f"Invalid beta2: {betas[1]}")
        if weight_decay < 0.0:
            raise ValueError(f"Invalid weight_decay: {weight_decay}")
        defaults = dict(lr=lr, betas=betas, eps=eps, weight_decay=weight_decay)
        super().__init__(params, defaults)
        # Same draw from the global torch RNG as optimizer.py:94-96, so ranks
        # seeded identically share the quantization noise.
        self._base_seed: int = int(
            torch.randint(-(2 ** 63), 2 ** 63 - 1, (1,), dtype=torch.int64).item())
        if backend not in _BACKENDS:
            raise ValueError(f"Invalid backend: {backend}. Expected one of "
                             f"{{'auto', 'cuda', 'triton'}} (this package runs the CUDA "
                             f"backend; the reference's 'pytorch' backend is not included).")
        self.backend = "cuda"
        self._engines: dict[torch.device, DeviceEngine] = {}
        self._slot_count: dict[torch.device, int] = {}
        self._draw_hook = None
        self._step_events = None  # optional (ev0, ev1, ev2) cudaEvent_t handles, timing hook
        if capture_steps < 1:
            raise ValueError(f"Invalid capture_steps: {capture_steps}")
        self.capturable = bool(capturable)
        self.capture_steps = int(capture_steps)
        self._row_tables: dict[torch.device, tuple[tuple, torch.Tensor]] = {}
        self._scale_refs: dict[torch.device, torch.Tensor] = {}
        self._pcache: list = []  # per param position: _ParamEntry, while valid
        self._state_ref = self.state
        self._state_len = 0

    # ------------------------------------------------------------------
    # helpers
    # ------------------------------------------------------------------
    @staticmethod
    def _unwrap_tensor(t):
        """DTensor (FSDP2) -> local shard (optimizer.py:399-407)."""
        if t is None:
            return None
        if hasattr(t, "_local_tensor"):
            return t._local_tensor
        return t

    def _engine(self, device: torch.device) -> DeviceEngine:
        eng = self._engines.get(device)
        if eng is None:
            _lib.lib()  # fail loudly here if the library is missing
            eng = DeviceEngine(device)
            self._engines[device] = eng
            self._slot_count[device] = 0
        return eng

    def _new_slot(self, device: torch.device) -> int:
        eng = self._engine(device)
        k = self._slot_count[device]
        self._slot_count[device] = k + 1
        eng.ensure_slots(k + 1)
        return k

    def _set_draw_hook(self, fn) -> None:
        """Test hook: ``fn(param_id, step, param) -> (u_m, u_w)`` float32 CUDA
        tensors with param's numel replace the Philox uniforms (the kernels'
        injected-draw path).  ``None`` restores Philox."""
        self._draw_hook = fn

    # -- capturable mode -----------------------------------------------------
    def _hyper_key(self) -> tuple:
        return tuple((g["lr"], g["betas"][0], g["betas"][1], g["eps"], g["weight_decay"])
                     for g in self.param_groups)

    def _row_table(self, device: torch.device) -> torch.Tensor:
        """Device LumaStepRow table, capture_steps rows per group (built on
        first use and whenever a hyper-parameter changed)."""
        key = self._hyper_key()
        cached = self._row_tables.get(device)
        if cached is not None and cached[0] == key:
            return cached[1]
        if torch.cuda.is_current_stream_capturing():
            raise RuntimeError("LUMA(capturable=True): hyper-parameters changed (or no eager "
                               "step was taken) before CUDA graph capture; call "
                               "refresh_capturable_rows() outside the graph")
        steps = np.arange(1, self.capture_steps + 1, dtype=np.int64)
        table = np.concatenate([step_rows(steps, *k) for k in key])
        host = torch.from_numpy(table.view(np.uint8).copy())
        if cached is not None and cached[1].numel() == host.numel():
            dev_tab = cached[1]  # same size: refresh in place (graphs hold this address)
            dev_tab.copy_(host.to(device))
        else:
            dev_tab = host.to(device)
        self._row_tables[device] = (key, dev_tab)
        return dev_tab

    @torch.no_grad()
    def refresh_capturable_rows(self) -> None:
        """Rebuild the capturable-mode row tables from the current group
        hyper-parameters (in place, so captured graphs see the new values)."""
        for dev in list(self._row_tables):
            self._row_table(dev)

    def _sync_steps(self) -> None:
        """Capturable mode: state["step"] from the device step counters."""
        if not self.capturable:
            return
        counts = {dev: eng.counters.cpu() for dev, eng in self._engines.items()}
        for group in self.param_groups:
            for p in group["params"]:
                st = self.state.get(p)
                if not st or "_slot" not in st or "step" not in st:
                    continue
                st["step"] = int(counts[self._unwrap_tensor(p).device][st["_slot"]])

    def _set_step_count(self, device: torch.device, slot: int, step: int) -> None:
        if self.capturable:
            self._engine(device).counters[slot] = step

    def step_op_args(self) -> dict:
        """Capturable mode: keyword arguments of ``torch.ops.luma_b200.step``
        that step this optimizer's parameters exactly as ``step()`` does (the
        parameters with gradients and their state as of the last eager
        ``step()``; one device)."""
        if not self.capturable:
            raise RuntimeError("step_op_args() needs LUMA(..., capturable=True)")
        if len(self._engines) != 1:
            raise RuntimeError("step_op_args() needs exactly one device with stepped params")
        (dev, eng), = self._engines.items()
        out = dict(params=[], grads=[], q_m=[], q_w=[], param_ids=[], slot_ids=[], row_bases=[])
        for gi, group in enumerate(self.param_groups):
            for p in group["params"]:
                st = self.state.get(p)
                if p.grad is None or not st or "_slot" not in st or "Q_m" not in st:
                    continue
                out["params"].append(self._unwrap_tensor(p))
                out["grads"].append(self._unwrap_tensor(p.grad))
                out["q_m"].append(st["Q_m"])
                out["q_w"].append(st["Q_w"])
                out["param_ids"].append(st["param_id"])
                out["slot_ids"].append(st["_slot"])
                out["row_bases"].append(gi * self.capture_steps)
        out.update(slots=eng.slots, counters=eng.counters, row_table=self._row_table(dev),
                   base_seed=self._base_seed)
        return out

    def kernel_error_flags(self, clear: bool = False) -> int:
        """LUMA_KERR_* flags raised by the step kernels on the current device."""
        return _lib.kernel_error_flags(clear)

    def _grid_scales(self) -> dict[int, tuple[float, float]]:
        """(S_m, S_v) per state-holding param, read from the device slots."""
        self._sync_steps()
        out = {}
        host = {dev: eng.read_slots() for dev, eng in self._engines.items()}
        for group in self.param_groups:
            for p in group["params"]:
                st = self.state.get(p)
                if not st or "_slot" not in st or "step" not in st:
                    continue
                param = self._unwrap_tensor(p)
                g = host[param.device][st["_slot"]]["grid"][st["step"] & 1]
                out[id(p)] = (float(g["S_m"]), float(g["S_v"]))
        return out

    # ------------------------------------------------------------------
    # checkpointing (optimizer.py:119-183)
    # ------------------------------------------------------------------
    def state_dict(self) -> dict:
        """Portable state dict: per param ``step, param_id, Q_m, Q_w, S_m, S_v``
        plus top-level ``_base_seed``; no private (``_``) keys."""
        scales = self._grid_scales()
        raw = super().state_dict()
        by_index = {}
        idx = 0
        for group in self.param_groups:
            for p in group["params"]:
                by_index[idx] = p
                idx += 1
        clean = {}
        for k, s in raw["state"].items():
            cs = {key: v for key, v in s.items() if not key.startswith("_")}
            if not cs:
                continue  # a param with a slot but no step taken yet
            p = by_index.get(k)
            if p is not None and id(p) in scales:
                cs["S_m"], cs["S_v"] = scales[id(p)]
            clean[k] = cs
        raw["state"] = clean
        raw["_base_seed"] = self._base_seed
        return raw

    def load_state_dict(self, state_dict: dict) -> None:
        """Load a state dict written by this backend or by the reference.

        Q_m/Q_w are kept as int16 codes (torch's loader would cast them to the
        param dtype); S_m/S_v move into the device slot of each param.
        """
        self._base_seed = state_dict.get("_base_seed", self._base_seed)
        sd = dict(state_dict)
        sd["state"] = {k: dict(v) for k, v in state_dict["state"].items()}
        codes = {}
        for k, s in sd["state"].items():
            codes[k] = {key: s.pop(key) for key in ("Q_m", "Q_w") if key in s}
        saved_ids = [i for g in sd["param_groups"] for i in g["params"]]
        super().load_state_dict(sd)
        params = [p for g in self.param_groups for p in g["params"]]
        pmap = dict(zip(saved_ids, params))
        eps_of = {id(p): g["eps"] for g in self.param_groups for p in g["params"]}
        for k, cd in codes.items():
            p = pmap.get(int(k) if isinstance(k, str) else k)
            if p is None:
                continue
            st = self.state[p]
            param = self._unwrap_tensor(p)
            for key, v in cd.items():
                # always a copy: a state dict taken from a live optimizer holds
                # that optimizer's own code tensors
                st[key] = v.to(device=param.device, dtype=torch.int16, copy=True)
        for p in params:
            st = self.state.get(p)
            if not st or "S_m" not in st:
                continue
            param = self._unwrap_tensor(p)
            if not param.is_cuda:
                continue
            slot = st.get("_slot")
            if slot is None:
                slot = self._new_slot(param.device)
                st["_slot"] = slot
            eng = self._engine(param.device)
            eng.reset_slot(slot)
            eng.write_grid(slot, st["step"] & 1, grid_record(st["S_m"], st["S_v"], eps_of[id(p)]))
            self._set_step_count(param.device, slot, st["step"])
            st.pop("S_m")
            st.pop("S_v")

    # ------------------------------------------------------------------
    # AdamW interop (optimizer.py:189-335)
    # ------------------------------------------------------------------
    def export_adamw_state(self) -> dict:
        """Decoded float32 ``exp_avg`` / ``exp_avg_sq`` in torch.optim.AdamW layout."""
        scales = self._grid_scales()
        param_to_idx = {}
        idx = 0
        for group in self.param_groups:
            for p in group["params"]:
                param_to_idx[id(p)] = idx
                idx += 1
        adamw_state = {}
        for group in self.param_groups:
            eps = group["eps"]
            for p in group["params"]:
                st = self.state.get(p)
                if not st or "Q_m" not in st:
                    continue
                S_m, S_v = scales[id(p)] if id(p) in scales else (st["S_m"], st["S_v"])
                w_min, delta_m, _, delta_w, _ = precompute(S_m, S_v, eps)
                q_m, q_w = st["Q_m"], st["Q_w"]
                exp_avg = torch.empty(q_m.shape, dtype=torch.float32, device=q_m.device)
                exp_avg_sq = torch.empty(q_m.shape, dtype=torch.float32, device=q_m.device)
                if q_m.numel():
                    stream = torch.cuda.current_stream(q_m.device)
                    _lib.check(_lib.lib().luma_decode(
                        q_m.data_ptr(), q_w.data_ptr(), q_m.numel(),
                        float(np.float32(delta_m)), float(np.float32(w_min)),
                        float(np.float32(delta_w)), float(np.float32(eps)),
                        exp_avg.data_ptr(), exp_avg_sq.data_ptr(),
                        ctypes.c_void_p(stream.cuda_stream)), "luma_decode")
                adamw_state[param_to_idx[id(p)]] = {
                    "step": torch.tensor(float(st["step"])),
                    "exp_avg": exp_avg,
                    "exp_avg_sq": exp_avg_sq,
                }
        param_groups = []
        for group in self.param_groups:
            pg = {k: v for k, v in group.items() if k != "params"}
            pg["params"] = [param_to_idx[id(p)] for p in group["params"]]
            param_groups.append(pg)
        return {"state": adamw_state, "param_groups": param_groups}

    def import_adamw_state(self, adamw_sd: dict) -> None:
        """Quantize a ``torch.optim.AdamW`` state dict into LUMA codes.

        Follows optimizer.py:256-335: per entry, step is kept, ``exp_avg`` and
        ``exp_avg_sq`` (clamped at 0) become float32 on the param's device,
        ``S_m = max(max|m|, 1e-9)``, ``S_v = max(max v, 0)``, and the codes are
        written with LogSR on that grid, the uniforms keyed by the seed
        ``(_base_seed, step 0, param index)`` (here the Philox stream).
        Hyper-parameters are not imported.
        """
        all_params = []
        group_of = {}
        for group in self.param_groups:
            for p in group["params"]:
                group_of[len(all_params)] = group
                all_params.append(p)
        for idx_key, st_in in adamw_sd["state"].items():
            idx = int(idx_key) if isinstance(idx_key, str) else idx_key
            if idx >= len(all_params):
                raise ValueError(f"AdamW state has index {idx} but LUMA only has "
                                 f"{len(all_params)} parameters")
            p = all_params[idx]
            eps = group_of[idx]["eps"]
            step_val = st_in["step"]
            step = int(step_val.item() if isinstance(step_val, torch.Tensor) else step_val)
            param = self._unwrap_tensor(p)
            device = param.device if param is not None else p.device
            if device.type != "cuda":
                raise RuntimeError(f"LUMA backend 'cuda' requires CUDA tensors (param on {device}).")
            m = st_in["exp_avg"].to(device).float().contiguous()
            v = st_in["exp_avg_sq"].to(device).float().clamp(min=0.0).contiguous()
            S_m = max(m.abs().max().item(), SCALE_FLOOR_M)
            S_v = max(v.max().item(), 0.0)
            grid = np.zeros(1, dtype=_lib.GRID_DTYPE)
            grid[0] = grid_record(S_m, S_v, eps)
            q_m = torch.empty(m.shape, dtype=torch.int16, device=device)
            q_w = torch.empty(m.shape, dtype=torch.int16, device=device)
            seed = ((0 << 32) | (idx * 2)) ^ self._base_seed  # functional.py:99-106, step 0
            seed = ctypes.c_int64(seed & 0xFFFFFFFFFFFFFFFF).value
            um = uw = None
            if self._draw_hook is not None:
                um, uw = (t.reshape(-1).contiguous() for t in self._draw_hook(idx, 0, m))
            stream = torch.cuda.current_stream(device)
            with torch.cuda.device(device):
                _lib.check(_lib.lib().luma_quantize(
                    m.data_ptr(), v.data_ptr(), m.numel(), grid.ctypes.data,
                    float(np.float32(eps)), float(np.float32(1.0 / eps)), seed, 0,
                    None if um is None else um.data_ptr(), None if uw is None else uw.data_ptr(),
                    q_m.data_ptr(), q_w.data_ptr(), ctypes.c_void_p(stream.cuda_stream)),
                    "luma_quantize")
            state = self.state[p]
            state["step"] = step
            state["param_id"] = idx
            state["Q_m"] = q_m
            state["Q_w"] = q_w
            slot = state.get("_slot")
            if slot is None:
                slot = self._new_slot(device)
                state["_slot"] = slot
            eng = self._engine(device)
            eng.reset_slot(slot)
            eng.write_grid(slot, step & 1, grid[0])
            self._set_step_count(device, slot, step)
            state.pop("S_m", None)
            state.pop("S_v", None)
            if um is not None:
                torch.cuda.current_stream(device).synchronize()  # injected draws outlive the kernel

    # ------------------------------------------------------------------
    # step (optimizer.py:413-524)
    # ------------------------------------------------------------------
    @torch.compiler.disable
    @torch.no_grad()
    def step(self, closure=None, *, grad_scale: torch.Tensor | None = None,
             found_inf: torch.Tensor | None = None):
        """One optimisation step for every parameter with a gradient.

        ``grad_scale``: optional one-element float32 / bfloat16 / float16
        tensor c (the clip coefficient carries the grads' dtype); every grad
        element g is then used as ``round_to_grad_dtype(fl32(g) * fl32(c))`` —
        what ``torch._foreach_mul_(grads, c)`` would have stored — without
        touching the grads.  With ``c`` from ``luma_b200.clip_grad_coef`` this fuses
        ``clip_grad_norm_``'s rescaling pass into the step (bit-identical to
        clipping first; the reference's training loop clips before every step,
        benchmarks/bench_nanogpt.py:218-225).

        Under ``torch.compile`` this method runs eagerly (one graph break at
        the call): its host side is table bookkeeping for a single library
        call.  ``torch.ops.luma_b200.step`` is the traceable form.

        ``found_inf``: optional one-element float32 tensor on the params'
        (single) device, the per-device flag of ``torch.amp.GradScaler``.  Pass
        1 sets it to 1.0 if any grad element is inf or NaN (checked before
        ``grad_scale`` is applied, as ``GradScaler.unscale_`` checks), and a set
        flag makes the step change nothing, like the ``optimizer.step()`` that
        ``GradScaler.step`` skips.  With ``grad_scale = 1/scale`` this fuses
        ``scaler.unscale_(opt); scaler.step(opt)`` into the step's own passes
        over the grads (``luma_b200.amp.scaler_step``).  Outside capturable
        mode the flag is read back once after the launch (one host sync, as
        ``GradScaler.step`` does) to keep the per-parameter ``step`` counts."""
        if grad_scale is not None:
            if not isinstance(grad_scale, torch.Tensor) or grad_scale.numel() != 1 \
                    or grad_scale.dtype not in (torch.float32, torch.bfloat16, torch.float16):
                raise ValueError("grad_scale must be a one-element float32, bfloat16 or "
                                 "float16 tensor")
        if found_inf is not None:
            if not isinstance(found_inf, torch.Tensor) or found_inf.numel() != 1 \
                    or found_inf.dtype != torch.float32 or not found_inf.is_cuda \
                    or not found_inf.is_contiguous():
                raise ValueError("found_inf must be a one-element contiguous float32 CUDA tensor")
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()

        # Pass A: validate everything before touching any state.  This loop
        # and the next run once per tensor every step (with 10,000 tensors
        # every microsecond per tensor is 10 ms per step), so what stays valid
        # while a param keeps its storage, size and dtype (its device, shape,
        # dtype checks and its state dict) is kept per param position in
        # self._pcache, and tensors are not used as dict keys (their hash is a
        # Python call).
        if self.state is not self._state_ref or len(self.state) != self._state_len:
            self._pcache = []  # state replaced, cleared or grown from outside step()
            self._state_ref = self.state
        pcache = self._pcache
        work = []
        idx = -1
        plain = _PLAIN_TENSOR_TYPES
        for gi, group in enumerate(self.param_groups):
            for p in group["params"]:
                idx += 1
                grad = p.grad
                if grad is None:
                    continue
                param = p if type(p) in plain else self._unwrap_tensor(p)
                if type(grad) not in plain:
                    grad = self._unwrap_tensor(grad)
                if idx >= len(pcache):
                    pcache.extend([None] * (idx + 1 - len(pcache)))
                if grad.is_sparse and param.numel():
                    raise RuntimeError("LUMA does not support sparse gradients")
                e = pcache[idx]
                if e is None or e[0] is not p or e[1] is not param or e[2] != param.data_ptr() \
                        or e[3] != param.numel() or e[4] is not param.dtype:
                    e = pcache[idx] = _ParamEntry(p, param)
                if e[3] == 0:
                    continue  # empty FSDP shard on this rank
                if not param.is_contiguous():
                    raise ValueError("LUMA CUDA kernel requires contiguous parameters")
                gcode = _GRAD_CODE.get(grad.dtype)
                if gcode is None:
                    raise ValueError(f"LUMA requires float32/bfloat16/float16 gradients "
                                     f"(got {grad.dtype}).")
                if grad.get_device() != e[5]:
                    raise ValueError("LUMA requires the gradient on the parameter's device")
                if grad.shape != e[6]:
                    raise ValueError("LUMA requires the gradient to have the parameter's shape")
                if not grad.is_contiguous():
                    raise ValueError("LUMA CUDA kernel requires contiguous gradients")
                work.append((e, grad, gi, idx, gcode))

        # Pass B: state bookkeeping and the per-device descriptor columns (or
        # segments, when the draw hook supplies per-tensor uniforms).
        hook = self._draw_hook
        if hook is not None and self.capturable:
            raise RuntimeError("the draw hook is not available in capturable mode")
        per_idx: dict[int, tuple] = {}
        last_dev, cols, rowmap = None, None, None
        last_gt, last_row = None, 0
        for e, grad, gi, pidx, gcode in work:
            param, state = e[1], e[8]
            if state is None:
                state = e[8] = self.state[e[0]]
            t = state.get("step", 0) + 1
            if t == 1:
                state["param_id"] = pidx
                state["Q_m"] = torch.empty_like(param, dtype=torch.int16)
                state["Q_w"] = torch.empty_like(param, dtype=torch.int16)
            state["step"] = t
            slot = state.get("_slot")
            if slot is None:
                slot = state["_slot"] = self._new_slot(param.device)
            if e[5] != last_dev:
                last_dev, last_gt = e[5], None
                entry = per_idx.get(last_dev)
                if entry is None:
                    entry = per_idx[last_dev] = ([] if hook is not None else Columns(), {})
                cols, rowmap = entry
            if self.capturable:
                row = gi * self.capture_steps  # the group's block of the row table
            elif last_gt is not None and last_gt[0] == gi and last_gt[1] == t:
                row = last_row
            else:
                last_gt = (gi, t)
                row = rowmap.get(last_gt)
                if row is None:
                    row = rowmap[last_gt] = len(rowmap)
                last_row = row
            q_m = state["Q_m"]
            if hook is not None:
                seg = Segment(param, grad, q_m, state["Q_w"], state["param_id"], row, slot)
                um, uw = hook(state["param_id"], t, param)
                seg.u_m = um.reshape(-1)
                seg.u_w = uw.reshape(-1)
                cols.append(seg)
                continue
            # (param address, codes, param_id, slot) change rarely: one tuple
            # per param, rebuilt when one of them did
            sk = e[9]
            if sk is None or sk[0] is not q_m or sk[1] != state["param_id"] or sk[2] != slot:
                sk = e[9] = (q_m, state["param_id"], slot,
                             (e[2], q_m.data_ptr(), state["Q_w"].data_ptr(), e[3],
                              state["param_id"], slot, e[7]))
            cols.statics.append(sk[3])
            cols.grad_ptrs.append(grad.data_ptr())
            cols.grad_codes.append(gcode)
            cols.rows.append(row)
        self._state_len = len(self.state)

        per_dev = {torch.device("cuda", k): v for k, v in per_idx.items()}
        if found_inf is not None:
            if len(per_dev) > 1:
                raise RuntimeError("found_inf: the fused inf check needs every stepped param on "
                                   "one device (a skip must apply to all of them)")
            if per_dev and found_inf.device != next(iter(per_dev)):
                raise ValueError("found_inf must be on the params' device")
        for dev, (segs, rowmap) in per_dev.items():
            gs = None
            if grad_scale is not None:
                gs = grad_scale.reshape(1).to(device=dev, dtype=torch.float32, non_blocking=True)
                gs = self._keep_scale(dev, gs)
            if self.capturable:
                self._engine(dev).step(segs, None, self._base_seed, events=self._step_events,
                                       row_table=self._row_table(dev), grad_scale=gs,
                                       found_inf=found_inf)
                continue
            rows = [None] * len(rowmap)
            for (gi, t), r in rowmap.items():
                g = self.param_groups[gi]
                rows[r] = step_row(t, g["lr"], g["betas"][0], g["betas"][1], g["eps"],
                                   g["weight_decay"])
            self._engine(dev).step(segs, rows_array(rows), self._base_seed,
                                   events=self._step_events, grad_scale=gs, found_inf=found_inf)
        if found_inf is not None and work and not self.capturable and bool(found_inf.item()):
            self._undo_steps(work)
        return loss

    def _undo_steps(self, work) -> None:
        """A step the kernels skipped (inf/NaN grads): restore the per-param
        step counts; a param whose first step was skipped gets no state, as if
        ``step()`` had not been called (its slot is kept for the next try)."""
        for e, *_ in work:
            state = e[8]
            state["step"] -= 1
            if state["step"] == 0:
                for key in ("step", "param_id", "Q_m", "Q_w"):
                    state.pop(key, None)

    def _keep_scale(self, device: torch.device, gs: torch.Tensor) -> torch.Tensor:
        """Hold a reference to a per-device copy of the scale until the next
        step (the kernels read it asynchronously)."""
        self._scale_refs[device] = gs
        return gs
