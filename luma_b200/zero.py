"""ZeRO-1 sharded LUMA step: per-rank flat shards plus a bf16 param all-gather.

LUMA's scales are per tensor shard by design (the reference's FSDP support
keeps one ``S_m``/``S_v`` per local shard, optimizer.py:399-407,
tests/test_fsdp.py:139-184), so the step partitions without any exchange:

* all params live as views into one flat buffer, each tensor starting at a
  multiple of 8 elements (16-byte aligned for bf16, 32 for fp32);
* the flat space is cut into ``world`` equal contiguous shards (a multiple of
  8 elements each, the last padded); rank r steps the pieces of every tensor
  that fall in shard r — one descriptor per (tensor, shard) segment, with
  its own scales, ``param_id`` = the tensor's global index and Philox
  counter = the segment's offset inside the tensor;
* after the step every rank holds the new values of its shard only; one
  in-place ``all_gather_into_tensor`` over NCCL (sendbuf = recvbuf + rank *
  shard) gives every rank the full updated params.

Grads are read only on the local shard (what a reduce-scatter delivers).
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from .engine import DeviceEngine, Segment
from .hostmath import rows_array, step_row

ALIGN = 8


@dataclass(frozen=True)
class FlatLayout:
    """Placement of tensors in the flat buffer and the shard size."""
    numels: tuple[int, ...]
    starts: tuple[int, ...]     # flat offset of each tensor (multiple of ALIGN)
    world: int
    shard: int                  # elements per rank (multiple of ALIGN)

    @property
    def total(self) -> int:
        return self.world * self.shard


@dataclass(frozen=True)
class ShardSegment:
    tensor: int      # index of the tensor (global param index)
    offset: int      # first element inside the tensor
    length: int      # elements
    flat: int        # flat offset of the first element


def plan_layout(numels, world: int) -> FlatLayout:
    """Tensor starts rounded up to ALIGN; shard = ceil(used / world) rounded to ALIGN."""
    if world < 1:
        raise ValueError("world must be >= 1")
    starts, pos = [], 0
    for n in numels:
        if n < 0:
            raise ValueError("negative numel")
        starts.append(pos)
        pos += -(-n // ALIGN) * ALIGN
    shard = -(-pos // world)
    shard = -(-shard // ALIGN) * ALIGN
    return FlatLayout(tuple(int(n) for n in numels), tuple(starts), world, max(shard, ALIGN))


def shard_segments(layout: FlatLayout, rank: int) -> list[ShardSegment]:
    """Segments of every tensor that fall in rank's shard, in flat order."""
    lo, hi = rank * layout.shard, (rank + 1) * layout.shard
    segs = []
    for i, (n, s) in enumerate(zip(layout.numels, layout.starts)):
        a, b = max(lo, s), min(hi, s + n)
        if a < b:
            segs.append(ShardSegment(i, a - s, b - a, a))
    return segs


def flat_views(flat: torch.Tensor, layout: FlatLayout, shapes) -> list[torch.Tensor]:
    """The tensors as views into the flat buffer."""
    out = []
    for (shape, n, s) in zip(shapes, layout.numels, layout.starts):
        out.append(flat[s:s + n].view(shape))
    return out


class ZeroLUMA:
    """LUMA step over this rank's flat shard, then an NCCL all-gather.

    ``flat_param``: the full flat param buffer (fp32 or bf16), every rank a
    replica, laid out by ``layout`` (see ``plan_layout`` / ``flat_views``).
    ``step(grad_shard)`` takes this rank's grad shard: a flat tensor of
    ``layout.shard`` elements covering ``[rank*shard, (rank+1)*shard)``.
    """

    def __init__(self, flat_param: torch.Tensor, layout: FlatLayout, rank: int,
                 lr: float = 1e-3, betas=(0.9, 0.999), eps: float = 1e-8,
                 weight_decay: float = 0.01, base_seed: int | None = None,
                 process_group=None):
        if flat_param.dim() != 1 or flat_param.numel() != layout.total:
            raise ValueError(f"flat_param must be 1-D with {layout.total} elements")
        if flat_param.dtype not in (torch.float32, torch.bfloat16):
            raise ValueError("flat_param must be float32 or bfloat16")
        if not flat_param.is_cuda:
            raise RuntimeError("ZeroLUMA requires a CUDA flat_param")
        self.flat = flat_param
        self.layout = layout
        self.rank = rank
        self.hp = dict(lr=lr, betas=betas, eps=eps, weight_decay=weight_decay)
        if base_seed is None:
            base_seed = int(torch.randint(-(2 ** 63), 2 ** 63 - 1, (1,), dtype=torch.int64).item())
        self.base_seed = base_seed
        self.pg = process_group
        self.segments = shard_segments(layout, rank)
        dev = flat_param.device
        self.q_m = torch.zeros(layout.shard, dtype=torch.int16, device=dev)
        self.q_w = torch.zeros(layout.shard, dtype=torch.int16, device=dev)
        self.engine = DeviceEngine(dev)
        self.engine.ensure_slots(max(1, len(self.segments)))
        self.t = 0
        self.events = None  # optional (ev0, ev1, ev2) cudaEvent_t handles (timing)

    def local_param_shard(self) -> torch.Tensor:
        s = self.layout.shard
        return self.flat[self.rank * s:(self.rank + 1) * s]

    def _segments(self, grad_shard: torch.Tensor) -> list[Segment]:
        base = self.rank * self.layout.shard
        out = []
        for k, sg in enumerate(self.segments):
            lo = sg.flat - base
            out.append(Segment(self.flat[sg.flat:sg.flat + sg.length],
                               grad_shard[lo:lo + sg.length],
                               self.q_m[lo:lo + sg.length], self.q_w[lo:lo + sg.length],
                               param_id=sg.tensor, row=0, slot=k, rng_offset=sg.offset))
        return out

    @torch.no_grad()
    def step_local(self, grad_shard: torch.Tensor) -> None:
        """Update this rank's shard (two kernel launches, no communication)."""
        if grad_shard.numel() != self.layout.shard or not grad_shard.is_contiguous():
            raise ValueError(f"grad_shard must be contiguous with {self.layout.shard} elements")
        self.t += 1
        b1, b2 = self.hp["betas"]
        row = step_row(self.t, self.hp["lr"], b1, b2, self.hp["eps"], self.hp["weight_decay"])
        self.engine.step(self._segments(grad_shard), rows_array([row]), self.base_seed,
                         events=self.events)

    @torch.no_grad()
    def gather(self) -> None:
        """In-place all-gather of every rank's shard into the flat buffer."""
        import torch.distributed as dist
        if self.layout.world == 1:
            return
        dist.all_gather_into_tensor(self.flat, self.local_param_shard(), group=self.pg)

    def step(self, grad_shard: torch.Tensor) -> None:
        self.step_local(grad_shard)
        self.gather()

    def scales(self) -> list[tuple[int, int, float, float]]:
        """(tensor, offset, S_m, S_v) of every local segment (synchronises)."""
        host = self.engine.read_slots()
        out = []
        for k, sg in enumerate(self.segments):
            g = host[k]["grid"][self.t & 1]
            out.append((sg.tensor, sg.offset, float(g["S_m"]), float(g["S_v"])))
        return out
