"""ZeRO-1 sharded LUMA step: per-rank flat shards plus a bf16 param all-gather.

LUMA's scales are per tensor shard by design (the reference's FSDP support
keeps one ``S_m``/``S_v`` per local shard, optimizer.py:399-407,
tests/test_fsdp.py:139-184), so the step partitions without any exchange:

* all params live as views into one flat buffer, each tensor starting at a
  multiple of 8 elements (16-byte aligned for bf16, 32 for fp32);
* the flat space is cut into ``buckets`` equal spans and every span into
  ``world`` equal pieces (multiples of 8 elements; the tail is padding):
  rank r owns piece r of every bucket.  With one bucket this is the plain
  contiguous 1/world shard;
* rank r steps the pieces of every tensor that fall in its pieces — one
  descriptor per (tensor, piece) segment with its own scales, ``param_id`` =
  the tensor's global index and Philox counter = the segment's offset inside
  the tensor;
* bucket b of every rank is contiguous, so one in-place
  ``all_gather_into_tensor`` per bucket (NCCL, sendbuf = recvbuf + rank *
  piece) gives every rank the full updated params.  ``step`` issues bucket
  b's gather on a side stream while the kernels of bucket b+1 run; the pass
  kernels can be capped below one CTA per SM (``max_ctas``) so NCCL's kernels
  find free SMs.

Grads are read only on the owned pieces (what a reduce-scatter with the same
layout delivers): ``grad_shard`` holds them back to back, bucket by bucket.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from .engine import DeviceEngine, Segment
from .hostmath import rows_array, step_row

ALIGN = 8


@dataclass(frozen=True)
class FlatLayout:
    """Placement of tensors in the flat buffer and the ownership pattern."""
    numels: tuple[int, ...]
    starts: tuple[int, ...]     # flat offset of each tensor (multiple of ALIGN)
    world: int
    piece: int                  # elements a rank owns per bucket (multiple of ALIGN)
    buckets: int = 1

    @property
    def span(self) -> int:
        """Elements per bucket (all ranks)."""
        return self.world * self.piece

    @property
    def shard(self) -> int:
        """Elements owned per rank (all buckets)."""
        return self.buckets * self.piece

    @property
    def total(self) -> int:
        return self.buckets * self.span

    def owned(self, rank: int, bucket: int) -> tuple[int, int]:
        lo = bucket * self.span + rank * self.piece
        return lo, lo + self.piece


@dataclass(frozen=True)
class ShardSegment:
    tensor: int      # index of the tensor (global param index)
    offset: int      # first element inside the tensor
    length: int      # elements
    flat: int        # flat offset of the first element
    local: int       # offset inside the rank's shard (grad_shard, codes)
    bucket: int


def plan_layout(numels, world: int, buckets: int = 1) -> FlatLayout:
    """Tensor starts rounded up to ALIGN; piece = ceil(used / (world*buckets)) rounded to ALIGN."""
    if world < 1 or buckets < 1:
        raise ValueError("world and buckets must be >= 1")
    starts, pos = [], 0
    for n in numels:
        if n < 0:
            raise ValueError("negative numel")
        starts.append(pos)
        pos += -(-n // ALIGN) * ALIGN
    piece = -(-pos // (world * buckets))
    piece = -(-piece // ALIGN) * ALIGN
    return FlatLayout(tuple(int(n) for n in numels), tuple(starts), world, max(piece, ALIGN),
                      buckets)


def shard_segments(layout: FlatLayout, rank: int, bucket: int | None = None) -> list[ShardSegment]:
    """Segments of every tensor inside rank's pieces (of one bucket, or all), in flat order."""
    out = []
    for b in (range(layout.buckets) if bucket is None else [bucket]):
        lo, hi = layout.owned(rank, b)
        for i, (n, s) in enumerate(zip(layout.numels, layout.starts)):
            a, e = max(lo, s), min(hi, s + n)
            if a < e:
                out.append(ShardSegment(i, a - s, e - a, a, b * layout.piece + (a - lo), b))
    return out


def flat_views(flat: torch.Tensor, layout: FlatLayout, shapes) -> list[torch.Tensor]:
    """The tensors as views into the flat buffer."""
    return [flat[s:s + n].view(shape) for shape, n, s in zip(shapes, layout.numels, layout.starts)]


class ZeroLUMA:
    """LUMA step over this rank's pieces, then per-bucket NCCL all-gathers.

    ``flat_param``: the full flat param buffer (fp32 or bf16), every rank a
    replica, laid out by ``layout`` (``plan_layout`` / ``flat_views``).
    ``step(grad_shard)`` takes this rank's grads, ``layout.shard`` elements:
    its piece of bucket 0, then of bucket 1, and so on.
    """

    def __init__(self, flat_param: torch.Tensor, layout: FlatLayout, rank: int,
                 lr: float = 1e-3, betas=(0.9, 0.999), eps: float = 1e-8,
                 weight_decay: float = 0.01, base_seed: int | None = None,
                 process_group=None, max_ctas: int = 0):
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
        self.max_ctas = max_ctas
        self.bucket_segments = [shard_segments(layout, rank, b) for b in range(layout.buckets)]
        dev = flat_param.device
        self.q_m = torch.zeros(layout.shard, dtype=torch.int16, device=dev)
        self.q_w = torch.zeros(layout.shard, dtype=torch.int16, device=dev)
        self.engines = []
        for segs in self.bucket_segments:
            eng = DeviceEngine(dev)
            eng.ensure_slots(max(1, len(segs)))
            self.engines.append(eng)
        self.comm = torch.cuda.Stream(device=dev)
        self.t = 0
        self.events = None  # optional (ev0, ev1, ev2) cudaEvent_t handles for bucket 0 (timing)

    @property
    def segments(self) -> list[ShardSegment]:
        return [sg for segs in self.bucket_segments for sg in segs]

    def _engine_segments(self, b: int, grad_shard: torch.Tensor) -> list[Segment]:
        out = []
        for k, sg in enumerate(self.bucket_segments[b]):
            lo = sg.local
            out.append(Segment(self.flat[sg.flat:sg.flat + sg.length],
                               grad_shard[lo:lo + sg.length],
                               self.q_m[lo:lo + sg.length], self.q_w[lo:lo + sg.length],
                               param_id=sg.tensor, row=0, slot=k, rng_offset=sg.offset))
        return out

    def _check(self, grad_shard: torch.Tensor) -> None:
        if grad_shard.numel() != self.layout.shard or not grad_shard.is_contiguous():
            raise ValueError(f"grad_shard must be contiguous with {self.layout.shard} elements")

    def _row(self):
        b1, b2 = self.hp["betas"]
        return rows_array([step_row(self.t, self.hp["lr"], b1, b2, self.hp["eps"],
                                    self.hp["weight_decay"])])

    def _step_bucket(self, b: int, grad_shard: torch.Tensor, rows, max_ctas: int) -> None:
        segs = self._engine_segments(b, grad_shard)
        self.engines[b].step(segs, rows, self.base_seed,
                             events=self.events if b == 0 else None, max_ctas=max_ctas)

    def _gather_bucket(self, b: int) -> None:
        import torch.distributed as dist
        s = self.layout.span
        lo, hi = self.layout.owned(self.rank, b)
        dist.all_gather_into_tensor(self.flat[b * s:(b + 1) * s], self.flat[lo:hi], group=self.pg)

    @torch.no_grad()
    def step_local(self, grad_shard: torch.Tensor) -> None:
        """Update this rank's pieces (two kernel launches per bucket, no communication)."""
        self._check(grad_shard)
        self.t += 1
        rows = self._row()
        for b in range(self.layout.buckets):
            self._step_bucket(b, grad_shard, rows, 0)

    @torch.no_grad()
    def gather(self) -> None:
        """All-gather every bucket (in place) on the current stream."""
        if self.layout.world == 1:
            return
        for b in range(self.layout.buckets):
            self._gather_bucket(b)

    @torch.no_grad()
    def step(self, grad_shard: torch.Tensor) -> None:
        """Step every bucket; bucket b's gather overlaps bucket b+1's kernels."""
        self._check(grad_shard)
        self.t += 1
        rows = self._row()
        if self.layout.world == 1:
            for b in range(self.layout.buckets):
                self._step_bucket(b, grad_shard, rows, 0)
            return
        main = torch.cuda.current_stream(self.flat.device)
        for b in range(self.layout.buckets):
            # while an earlier bucket's gather may be in flight, leave SMs to NCCL
            self._step_bucket(b, grad_shard, rows, self.max_ctas if b > 0 else 0)
            done = torch.cuda.Event()
            done.record(main)
            self.comm.wait_event(done)
            with torch.cuda.stream(self.comm):
                self._gather_bucket(b)
        main.wait_stream(self.comm)

    def scales(self) -> list[tuple[int, int, float, float]]:
        """(tensor, offset, S_m, S_v) of every local segment, bucket order (synchronises)."""
        out = []
        for segs, eng in zip(self.bucket_segments, self.engines):
            host = eng.read_slots()
            for k, sg in enumerate(segs):
                g = host[k]["grid"][self.t & 1]
                out.append((sg.tensor, sg.offset, float(g["S_m"]), float(g["S_v"])))
        return out
