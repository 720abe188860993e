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
* ``gather="copy"`` replaces NCCL's gather by copy-engine pushes: every rank
  maps the peers' flat buffers (CUDA IPC, ``PeerGather``) and, as soon as
  bucket b's kernels are done, copies its piece of bucket b into every peer
  (one ``cudaMemcpyAsync`` per peer, each peer on its own stream).  No SM is
  taken from the step kernels.  Two stream-ordered barriers (an all-reduce of
  one element) bound the pushes: the one before the first push makes sure
  every peer has finished with its replica of the previous step (nothing still
  reads a piece about to be overwritten), the one after the last push tells
  every rank that all pieces have arrived.

* ``gather="nvls"`` fuses the gather into the step itself: the flat buffer
  lives in symmetric memory (``alloc_flat``, torch's
  ``_symmetric_memory``) bound to an NVLink multicast object, and pass 2
  writes every updated param through the multicast address
  (``LumaTensorDesc.param_mc``, ``multimem.st``): the NVSwitch delivers each
  write to every GPU, so when the step's kernels end, every replica holds
  every rank's pieces.  No copy, no NCCL transfer, no SM taken from the step
  beyond its own stores; a stream-ordered barrier before the step (peers are
  done reading their replicas) and one after it (all pieces have landed)
  bound it.

Grads are read only on the owned pieces (what a reduce-scatter with the same
layout delivers): ``grad_shard`` holds them back to back, bucket by bucket.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from .engine import DeviceEngine, Segment
from .hostmath import grid_record, rows_array, step_row

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

    def to_dict(self) -> dict:
        return {"numels": list(self.numels), "starts": list(self.starts), "world": self.world,
                "piece": self.piece, "buckets": self.buckets}

    @staticmethod
    def from_dict(d: dict) -> "FlatLayout":
        return FlatLayout(tuple(int(n) for n in d["numels"]), tuple(int(s) for s in d["starts"]),
                          int(d["world"]), int(d["piece"]), int(d["buckets"]))


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


def alloc_flat(numel: int, dtype: torch.dtype, device, gather: str) -> torch.Tensor:
    """The flat param buffer for ``ZeroLUMA``: symmetric memory for
    ``gather="nvls"`` (it must be bound to a multicast object), a plain CUDA
    tensor otherwise."""
    if gather == "nvls":
        import torch.distributed._symmetric_memory as symm_mem
        return symm_mem.empty(numel, dtype=dtype, device=device)
    return torch.empty(numel, dtype=dtype, device=device)


class NvlsGather:
    """Multicast (NVLS) address of a symmetric-memory flat buffer and the
    stream-ordered barrier around the fused step.  Collective to construct;
    raises ``PeerMapError`` on every rank if any rank cannot get a multicast
    mapping (outcome agreed by a collective)."""

    def __init__(self, flat: torch.Tensor, rank: int, process_group=None):
        import torch.distributed as dist
        import torch.distributed._symmetric_memory as symm_mem
        err, base = None, 0
        try:
            group = process_group if process_group is not None else dist.group.WORLD
            self.handle = symm_mem.rendezvous(flat, group)
            if not self.handle.multicast_ptr:
                err = "no NVLink multicast support on this device / driver"
            else:
                # the multicast mapping covers the whole symmetric buffer; the
                # tensor sits at the same offset in it on every rank
                local = int(self.handle.buffer_ptrs[self.handle.rank])
                base = int(self.handle.multicast_ptr) + (flat.data_ptr() - local)
        except Exception as exc:  # noqa: BLE001 - any failure means: no multicast
            err = f"{type(exc).__name__}: {exc}"
        errs = [None] * dist.get_world_size(process_group)
        dist.all_gather_object(errs, err, group=process_group)
        failed = [e for e in errs if e is not None]
        if failed:
            self.handle = None
            raise PeerMapError(f"NVLS multicast unavailable: {failed[0]}")
        self.mc_base = base
        self.pg = process_group
        self.token = torch.zeros(1, dtype=torch.float32, device=flat.device)

    def barrier(self) -> None:
        """All ranks reach this point of their streams (an all-reduce of one
        element on the current stream)."""
        import torch.distributed as dist
        dist.all_reduce(self.token, group=self.pg)

    def close(self) -> None:
        torch.cuda.synchronize(self.token.device)
        self.handle = None


def auto_gather(world: int) -> str:
    """Gather measured fastest on B200 (Llama-3-8B, 8 buckets): copy engines up
    to 4 ranks (2 ranks: 207.5 Gparams/s against NVLS 178.1 and NCCL 158.9;
    4 ranks: 354 against NCCL 212), NCCL at 8 (304-312 against copy engines
    291 and NVLS 237), where every rank receives 7/8 of the params and NCCL's
    transfer rate (643 GB/s per rank) beats the copy engines' (580)."""
    return "copy" if world <= 4 else "nccl"


def push_order(rank: int, world: int, copy_streams: int) -> list[tuple[int, int]]:
    """(peer, stream index) in the order this rank pushes to its peers: rank+1,
    rank+2, ... (mod world), so that the ranks start on different peers (with
    every rank pushing to peer 0 first the 4-GPU gather ran at half the rate);
    peers are dealt round-robin over min(copy_streams, world-1) streams
    (copy_streams <= 0: one stream per peer)."""
    peers = [(rank + k) % world for k in range(1, world)]
    if not peers:
        return []
    n_st = max(1, min(copy_streams if copy_streams > 0 else len(peers), len(peers)))
    return [(p, k % n_st) for k, p in enumerate(peers)]


def lockstep_applies(requested: bool, copy_streams: int, world: int) -> bool:
    """Whether the copy gather runs in lockstep: a stream-ordered barrier
    between consecutive pushes of a bucket, so that in phase k every rank
    pushes to rank + k (``push_order``) and every GPU receives from exactly one
    peer at a time.  Only with one copy stream (the pushes are then ordered)
    and more than two ranks (with two there is one push per bucket)."""
    return bool(requested) and copy_streams == 1 and world > 2


def gather_bucket_into(staging: torch.Tensor, shard: torch.Tensor, layout: FlatLayout,
                       bucket: int, group=None) -> torch.Tensor:
    """Sharded-params mode: all-gather bucket `bucket` of every rank's shard
    (``shard`` holds this rank's pieces back to back) into `staging`
    (``layout.span`` elements: rank r's piece at ``r * layout.piece``), which
    then holds flat positions ``[bucket * span, (bucket + 1) * span)``."""
    import torch.distributed as dist
    p = layout.piece
    view = staging[:layout.span]
    dist.all_gather_into_tensor(view, shard[bucket * p:(bucket + 1) * p], group=group)
    return view


class PeerMapError(RuntimeError):
    """Some rank could not export or map the flat buffer over CUDA IPC (raised
    on every rank, after the ranks have agreed on it)."""


class PeerGather:
    """Copy-engine all-gather of the flat buffer's bucket pieces over CUDA IPC.

    Collective to construct (every rank of ``process_group``).  ``begin`` and
    ``finish`` are stream-ordered barriers on ``comm``; ``push(b, event)``
    copies this rank's piece of bucket b into every peer after ``event``.

    The buffer must be plain ``cudaMalloc`` memory (PyTorch's default caching
    allocator); memory from ``PYTORCH_CUDA_ALLOC_CONF=expandable_segments:True``
    is VMM-backed and has no IPC handle.  A failure to export or map on any
    rank raises ``PeerMapError`` on all ranks (the outcome is agreed by a
    collective, so no rank is left waiting in a later one).
    """

    def __init__(self, flat: torch.Tensor, layout: FlatLayout, rank: int, process_group=None,
                 copy_streams: int = 1, lockstep: bool = False):
        import torch.distributed as dist

        from . import _lib
        self._lib = _lib
        self.flat = flat
        self.layout = layout
        self.rank = rank
        self.pg = process_group
        try:
            info, err = _lib.ipc_export(flat.data_ptr()), None
        except (_lib.LumaError, ValueError) as exc:
            info, err = None, str(exc)
        infos = [None] * layout.world
        dist.all_gather_object(infos, (info, err), group=process_group)
        bad = [(r, e) for r, (i, e) in enumerate(infos) if i is None]
        if bad:
            raise PeerMapError(f"rank {bad[0][0]} cannot export its buffer over CUDA IPC: "
                               f"{bad[0][1]}")
        self.bases = {}
        self.peer_ptr = {}
        err = None
        for p, (hi, _) in enumerate(infos):
            if p == rank:
                continue
            try:
                base = _lib.ipc_open(hi[0])
            except (_lib.LumaError, ValueError) as exc:
                err = f"rank {rank} cannot map rank {p}'s buffer: {exc}"
                break
            self.bases[p] = base
            self.peer_ptr[p] = base + hi[1]
        errs = [None] * layout.world
        dist.all_gather_object(errs, err, group=process_group)
        failed = [e for e in errs if e is not None]
        if failed:
            for base in self.bases.values():
                _lib.ipc_close(base)
            raise PeerMapError(failed[0])
        dev = flat.device
        self.comm = torch.cuda.Stream(device=dev)
        order = push_order(rank, layout.world, copy_streams)
        n_st = 1 + max(k for _, k in order)
        self.copy_streams = [torch.cuda.Stream(device=dev) for _ in range(n_st)]
        self.streams = {p: self.copy_streams[k] for p, k in order}
        self.order = [p for p, _ in order]
        self.lockstep = lockstep_applies(lockstep, n_st, layout.world)
        self.token = torch.zeros(1, dtype=torch.float32, device=dev)
        self.phase_token = torch.zeros(1, dtype=torch.float32, device=dev)

    def _barrier(self) -> None:
        import torch.distributed as dist
        with torch.cuda.stream(self.comm):
            dist.all_reduce(self.token, group=self.pg)

    def begin(self, main: torch.cuda.Stream) -> None:
        """Barrier after everything queued on `main` so far (all ranks)."""
        self.comm.wait_stream(main)
        self._barrier()
        for st in self.copy_streams:
            st.wait_stream(self.comm)

    def push(self, bucket: int, ready: torch.cuda.Event) -> None:
        """This rank's piece of bucket `bucket` into the same place of every
        peer's buffer."""
        lo, hi = self.layout.owned(self.rank, bucket)
        es = self.flat.element_size()
        self.push_range(self.flat.data_ptr() + lo * es, lo * es, (hi - lo) * es, ready)

    def push_range(self, src: int, dst_off: int, nbytes: int, ready: torch.cuda.Event,
                   local: bool = False) -> None:
        """`nbytes` at device address `src` to byte offset `dst_off` of every
        peer's buffer (and of this rank's own buffer when `local`), on the
        copy streams after `ready`."""
        for st in self.copy_streams:
            st.wait_event(ready)
        if self.lockstep:
            import torch.distributed as dist
            st = self.copy_streams[0]
            for k, p in enumerate(self.order):
                if k:
                    with torch.cuda.stream(st):
                        dist.all_reduce(self.phase_token, group=self.pg)
                self._lib.copy_async(self.peer_ptr[p] + dst_off, src, nbytes, st)
        else:
            for p, st in self.streams.items():
                self._lib.copy_async(self.peer_ptr[p] + dst_off, src, nbytes, st)
        if local:
            self._lib.copy_async(self.flat.data_ptr() + dst_off, src, nbytes,
                                 self.copy_streams[0])

    def finish(self, main: torch.cuda.Stream) -> None:
        """Barrier after every push; `main` then sees the full replica."""
        for st in self.copy_streams:
            self.comm.wait_stream(st)
        self._barrier()
        main.wait_stream(self.comm)

    def close(self) -> None:
        torch.cuda.synchronize(self.flat.device)
        for base in self.bases.values():
            self._lib.ipc_close(base)
        self.bases.clear()
        self.peer_ptr.clear()


def make_peer_gather(flat: torch.Tensor, layout: FlatLayout, rank: int, process_group=None,
                     copy_streams: int = 1, lockstep: bool = False) -> PeerGather | None:
    """A PeerGather, or None (with a warning, on every rank alike) when the
    buffer cannot be shared over CUDA IPC; the caller then gathers by NCCL."""
    import warnings
    try:
        return PeerGather(flat, layout, rank, process_group, copy_streams, lockstep)
    except PeerMapError as exc:
        warnings.warn(f"ZeroLUMA: copy-engine gather unavailable ({exc}); using NCCL instead",
                      RuntimeWarning, stacklevel=3)
        return None


class ZeroLUMA:
    """LUMA step over this rank's pieces, then per-bucket all-gathers.

    ``flat_param``: the full flat param buffer (fp32 or bf16), every rank a
    replica, laid out by ``layout`` (``plan_layout`` / ``flat_views``).
    ``step(grad_shard)`` takes this rank's grads, ``layout.shard`` elements:
    its piece of bucket 0, then of bucket 1, and so on.

    ``replica=False`` is the mode for models whose full replica does not fit
    next to the shard state (Llama-3-70B on 8 GPUs: 141 GB of bf16 params):
    ``flat_param`` then holds only this rank's pieces (``layout.shard``
    elements, the grads' layout), and each bucket is all-gathered (NCCL, or
    with ``gather="copy"`` by copy-engine pushes into the peers' staging
    buffers over CUDA IPC, or with ``gather="nvls"`` by the step's multicast
    stores) into one of ``staging`` rotating buffers of ``layout.span`` elements;
    ``consumer(bucket, view)``, called with the gather's stream current, gets
    each gathered bucket before its buffer is reused.  Positions of a view
    outside every tensor (alignment gaps, the last bucket's padding) are not
    data: NCCL and copy gathers carry the shards' values there, the nvls
    staging mode leaves them as they were.  ``gather="auto"`` picks NCCL in
    this mode.

    ``copy_lockstep`` (copy gather, one copy stream, more than 2 ranks): a
    barrier between the pushes of a bucket, so that in phase k every rank
    pushes to rank + k and every GPU receives from one peer at a time; the
    step kernels then run on ``max_ctas`` CTAs so the barriers' NCCL kernels
    find free SMs.
    """

    def __init__(self, flat_param: torch.Tensor, layout: FlatLayout, rank: int,
                 lr: float = 1e-3, betas=(0.9, 0.999), eps: float = 1e-8,
                 weight_decay: float = 0.01, base_seed: int | None = None,
                 process_group=None, max_ctas: int = 0, gather: str = "nccl",
                 copy_streams: int = 1, replica: bool = True, staging: int = 2,
                 consumer=None, copy_lockstep: bool = False):
        want = layout.total if replica else layout.shard
        if flat_param.dim() != 1 or flat_param.numel() != want:
            raise ValueError(f"flat_param must be 1-D with {want} elements")
        if staging < 1:
            raise ValueError("staging must be >= 1")
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
        if gather not in ("nccl", "copy", "auto", "nvls"):
            raise ValueError(f"gather must be 'nccl', 'copy', 'nvls' or 'auto', got {gather!r}")
        if gather == "auto":
            # sharded params: NCCL (measured at 4 and 8 ranks); replicas: by world size
            gather = auto_gather(layout.world) if replica else "nccl"
        self.replica = replica
        self.consumer = consumer
        self.staging = []
        self.staging_mc = []
        self.staging_peers = None
        self.peers = None
        self.nvls = None
        self._token = torch.zeros(1, dtype=torch.float32, device=dev)
        if not replica:
            # the gathered buckets go to rotating staging buffers: filled by the
            # step's own multicast stores (nvls), by copy-engine pushes into the
            # peers' staging buffers (copy) or by NCCL
            if layout.world == 1 or gather not in ("nvls", "copy"):
                gather = "nccl"
            if gather == "copy":
                # one allocation for all staging buffers (one IPC mapping per
                # peer); at least two, so a push never overwrites a bucket a
                # peer's consumer may still read
                n_st = max(staging, 2)
                whole = torch.empty(n_st * layout.span, dtype=flat_param.dtype, device=dev)
                self.staging_peers = make_peer_gather(whole, layout, rank, process_group, 1,
                                                      copy_lockstep)
                if self.staging_peers is None:
                    gather = "nccl"
                else:
                    self.staging = [whole[k * layout.span:(k + 1) * layout.span]
                                    for k in range(n_st)]
            if layout.world > 1 and gather == "nvls":
                import warnings
                try:
                    self.staging = [alloc_flat(layout.span, flat_param.dtype, dev, "nvls")
                                    for _ in range(max(staging, 2))]
                    self.staging_mc = [NvlsGather(buf, rank, process_group)
                                       for buf in self.staging]
                except PeerMapError as exc:
                    warnings.warn(f"ZeroLUMA: {exc}; gathering the buckets with NCCL instead",
                                  RuntimeWarning, stacklevel=2)
                    gather, self.staging, self.staging_mc = "nccl", [], []
            if layout.world > 1 and not self.staging:
                self.staging = [torch.empty(layout.span, dtype=flat_param.dtype, device=dev)
                                for _ in range(staging)]
        elif gather == "nvls" and layout.world == 1:
            gather = "copy"
        if gather == "nvls" and replica:
            import warnings
            try:
                self.nvls = NvlsGather(flat_param, rank, process_group)
            except PeerMapError as exc:
                warnings.warn(f"ZeroLUMA: {exc}; using the copy-engine gather instead",
                              RuntimeWarning, stacklevel=2)
                gather = "copy"
        if gather == "copy" and replica and layout.world > 1:
            self.peers = make_peer_gather(flat_param, layout, rank, process_group, copy_streams,
                                          copy_lockstep)
            if self.peers is None:
                gather = "nccl"
        self.gather_mode = gather
        self.t = 0
        self.events = None  # optional (ev0, ev1, ev2) cudaEvent_t handles for bucket 0 (timing)

    @property
    def segments(self) -> list[ShardSegment]:
        return [sg for segs in self.bucket_segments for sg in segs]

    def _engine_segments(self, b: int, grad_shard: torch.Tensor,
                         multicast: bool = False) -> list[Segment]:
        out = []
        es = self.flat.element_size()
        own_lo = self.layout.owned(self.rank, b)[0]
        for k, sg in enumerate(self.bucket_segments[b]):
            lo = sg.local
            pos = sg.flat if self.replica else sg.local
            mc, mc_local = 0, False
            if multicast and self.replica:
                mc = self.nvls.mc_base + pos * es  # the replica itself
            elif multicast:
                # this rank's piece of the bucket's staging buffer; the shard
                # copy is stored too
                sm = self.staging_mc[b % len(self.staging_mc)]
                mc = sm.mc_base + (self.rank * self.layout.piece + sg.flat - own_lo) * es
                mc_local = True
            out.append(Segment(self.flat[pos:pos + sg.length],
                               grad_shard[lo:lo + sg.length],
                               self.q_m[lo:lo + sg.length], self.q_w[lo:lo + sg.length],
                               param_id=sg.tensor, row=0, slot=k, rng_offset=sg.offset,
                               param_mc=mc, mc_local=mc_local))
        return out

    def _check(self, grad_shard: torch.Tensor) -> None:
        if grad_shard.numel() != self.layout.shard or not grad_shard.is_contiguous():
            raise ValueError(f"grad_shard must be contiguous with {self.layout.shard} elements")

    def _row(self):
        b1, b2 = self.hp["betas"]
        return rows_array([step_row(self.t, self.hp["lr"], b1, b2, self.hp["eps"],
                                    self.hp["weight_decay"])])

    def _step_bucket(self, b: int, grad_shard: torch.Tensor, rows, max_ctas: int,
                     grad_scale: torch.Tensor | None = None, multicast: bool = False) -> None:
        segs = self._engine_segments(b, grad_shard, multicast)
        self.engines[b].step(segs, rows, self.base_seed,
                             events=self.events if b == 0 else None, max_ctas=max_ctas,
                             grad_scale=grad_scale)

    def _gather_bucket(self, b: int) -> None:
        import torch.distributed as dist
        if not self.replica and self.staging_mc:
            # the multicast copy of this rank's piece, then every piece has landed
            from . import _lib
            es = self.flat.element_size()
            sm = self.staging_mc[b % len(self.staging_mc)]
            p = self.layout.piece
            _lib.mc_copy(sm.mc_base + self.rank * p * es, self.flat.data_ptr() + b * p * es, p * es,
                         torch.cuda.current_stream(self.flat.device))
            sm.barrier()
            if self.consumer is not None:
                self.consumer(b, self.staging[b % len(self.staging)][:self.layout.span])
            return
        if not self.replica:
            view = gather_bucket_into(self.staging[b % len(self.staging)], self.flat, self.layout,
                                      b, self.pg)
            if self.consumer is not None:
                self.consumer(b, view)
            return
        s = self.layout.span
        lo, hi = self.layout.owned(self.rank, b)
        dist.all_gather_into_tensor(self.flat[b * s:(b + 1) * s], self.flat[lo:hi], group=self.pg)

    def _staged_pushes(self, main: torch.cuda.Stream, ready_of) -> None:
        """Sharded-params mode with copy engines: for every bucket b, after the
        event ``ready_of(b)`` (which may launch b's kernels), push this rank's
        piece into every GPU's staging buffer b % S, this one's included; an
        all-reduce of one element on the gather stream then says that every
        piece of b has landed, and ``consumer(b, view)`` runs on that stream.
        Bucket b's pushes wait for bucket b-1's barrier, which every rank
        reaches only after its consumer(b-2): with S >= 2 buffers no push
        overwrites a bucket a consumer may still read.  A barrier first says
        that every rank is done with the last call's buckets."""
        import torch.distributed as dist
        sp, comm = self.staging_peers, self.comm
        es = self.flat.element_size()
        p, span, n_st = self.layout.piece, self.layout.span, len(self.staging)
        copy = sp.copy_streams[0]
        comm.wait_stream(main)
        with torch.cuda.stream(comm):
            dist.all_reduce(self._token, group=self.pg)
        gate = torch.cuda.Event()
        gate.record(comm)
        for b in range(self.layout.buckets):
            ready = ready_of(b)
            copy.wait_event(gate)
            sp.push_range(self.flat.data_ptr() + b * p * es,
                          ((b % n_st) * span + self.rank * p) * es, p * es, ready, local=True)
            pushed = torch.cuda.Event()
            pushed.record(copy)
            comm.wait_event(pushed)
            with torch.cuda.stream(comm):
                dist.all_reduce(self._token, group=self.pg)
                gate = torch.cuda.Event()
                gate.record(comm)
                if self.consumer is not None:
                    self.consumer(b, self.staging[b % n_st])
        main.wait_stream(comm)

    @torch.no_grad()
    def step_local(self, grad_shard: torch.Tensor,
                   grad_scale: torch.Tensor | None = None) -> None:
        """Update this rank's pieces (two kernel launches per bucket, no communication)."""
        self._check(grad_shard)
        if grad_scale is not None:
            grad_scale = grad_scale.reshape(1).to(device=self.flat.device, dtype=torch.float32)
        self.t += 1
        rows = self._row()
        for b in range(self.layout.buckets):
            self._step_bucket(b, grad_shard, rows, 0, grad_scale)

    @torch.no_grad()
    def gather(self) -> None:
        """All-gather every bucket (in place), ordered after the current stream."""
        if self.layout.world == 1:
            return
        main = torch.cuda.current_stream(self.flat.device)
        if self.nvls is not None:
            from . import _lib
            es = self.flat.element_size()
            self.nvls.barrier()
            for b in range(self.layout.buckets):
                lo, hi = self.layout.owned(self.rank, b)
                _lib.mc_copy(self.nvls.mc_base + lo * es, self.flat.data_ptr() + lo * es,
                             (hi - lo) * es, main)
            self.nvls.barrier()
            return
        if self.peers is not None:
            self.peers.begin(main)
            done = torch.cuda.Event()
            done.record(main)
            for b in range(self.layout.buckets):
                self.peers.push(b, done)
            self.peers.finish(main)
            return
        if self.staging_peers is not None:
            ready = torch.cuda.Event()
            ready.record(main)
            self._staged_pushes(main, lambda b: ready)
            return
        if self.staging_mc:
            self.staging_mc[0].barrier()  # every rank is done with the last call's buckets
        for b in range(self.layout.buckets):
            self._gather_bucket(b)

    @torch.no_grad()
    def step(self, grad_shard: torch.Tensor, grad_scale: torch.Tensor | None = None) -> None:
        """Step every bucket; bucket b's gather overlaps bucket b+1's kernels.
        `grad_scale`: optional one-element device tensor fused into the step as
        in ``LUMA.step`` (e.g. the global clip coefficient)."""
        self._check(grad_shard)
        if grad_scale is not None:
            grad_scale = grad_scale.reshape(1).to(device=self.flat.device, dtype=torch.float32)
        self.t += 1
        rows = self._row()
        if self.layout.world == 1:
            for b in range(self.layout.buckets):
                self._step_bucket(b, grad_shard, rows, 0, grad_scale)
            return
        main = torch.cuda.current_stream(self.flat.device)
        if self.staging_peers is not None:
            cap = self.max_ctas if self.staging_peers.lockstep else 0

            def kernels(b):
                self._step_bucket(b, grad_shard, rows, cap, grad_scale)
                done = torch.cuda.Event()
                done.record(main)
                return done
            self._staged_pushes(main, kernels)
            return
        if self.staging_mc:
            # bucket b's kernels write its pieces into every rank's staging
            # buffer b % S; the barrier after them says all pieces have landed
            # and that every rank has run consumer(b - 1), so bucket b + 1 may
            # overwrite the buffer bucket b - 1 used (two buffers suffice); the
            # barrier first says every rank is done with the last call's buckets
            self.staging_mc[0].barrier()
            for b in range(self.layout.buckets):
                self._step_bucket(b, grad_shard, rows, 0, grad_scale, multicast=True)
                self.staging_mc[b % len(self.staging_mc)].barrier()
                if self.consumer is not None:
                    self.consumer(b, self.staging[b % len(self.staging)][:self.layout.span])
            return
        if self.nvls is not None:
            # the gather is the kernels' own multicast stores
            self.nvls.barrier()
            for b in range(self.layout.buckets):
                self._step_bucket(b, grad_shard, rows, 0, grad_scale, multicast=True)
            self.nvls.barrier()
            return
        if self.peers is not None:
            # copy engines: bucket b's pushes overlap bucket b+1's kernels; in
            # lockstep the barriers between pushes are NCCL kernels, which
            # need SMs the step kernels leave free (max_ctas)
            self.peers.begin(main)
            cap = self.max_ctas if self.peers.lockstep else 0
            for b in range(self.layout.buckets):
                self._step_bucket(b, grad_shard, rows, cap, grad_scale)
                done = torch.cuda.Event()
                done.record(main)
                self.peers.push(b, done)
            self.peers.finish(main)
            return
        for b in range(self.layout.buckets):
            # while an earlier bucket's gather may be in flight, leave SMs to NCCL
            self._step_bucket(b, grad_shard, rows, self.max_ctas if b > 0 else 0, grad_scale)
            done = torch.cuda.Event()
            done.record(main)
            self.comm.wait_event(done)
            with torch.cuda.stream(self.comm):
                self._gather_bucket(b)
        main.wait_stream(self.comm)

    def close(self) -> None:
        """Unmap the peers' buffers (copy gather) or drop the multicast handle
        (nvls); call before destroying the process group."""
        if self.peers is not None:
            self.peers.close()
            self.peers = None
        if self.staging_peers is not None:
            self.staging_peers.close()
            self.staging_peers = None
        if self.nvls is not None:
            self.nvls.close()
            self.nvls = None
        for sm in self.staging_mc:
            sm.close()
        self.staging_mc = []

    # -- checkpointing ------------------------------------------------------
    def state_dict(self) -> dict:
        """This rank's optimizer state (synchronises): step count, seed,
        hyper-parameters, layout and rank, the rank's codes (``q_m``, ``q_w``,
        ``layout.shard`` elements each, on CPU) and one ``(tensor, offset,
        length, S_m, S_v)`` entry per local segment — the reference's
        per-local-shard state (optimizer.py:119-144 per param: step, Q_m, Q_w,
        S_m, S_v; one entry per shard segment here).  The params are the
        model's state and are saved by the caller."""
        segs = self.segments
        scales = self.scales() if self.t > 0 else [(sg.tensor, sg.offset, 0.0, 0.0)
                                                    for sg in segs]
        return {"t": self.t, "base_seed": self.base_seed, "rank": self.rank,
                "replica": self.replica, "hp": {**self.hp, "betas": tuple(self.hp["betas"])},
                "layout": self.layout.to_dict(),
                "q_m": self.q_m.cpu(), "q_w": self.q_w.cpu(),
                "segments": [(sg.tensor, sg.offset, sg.length, S_m, S_v)
                             for sg, (_, _, S_m, S_v) in zip(segs, scales)]}

    def load_state_dict(self, sd: dict) -> None:
        """Restore a ``state_dict()`` of the same rank and layout: the next
        ``step`` continues bit for bit (same codes, grids, step count, seed)."""
        if FlatLayout.from_dict(sd["layout"]) != self.layout:
            raise ValueError("ZeroLUMA.load_state_dict: the checkpoint's layout differs "
                             "(tensor sizes, world, buckets or piece)")
        if int(sd["rank"]) != self.rank:
            raise ValueError(f"ZeroLUMA.load_state_dict: checkpoint of rank {sd['rank']}, "
                             f"this is rank {self.rank}")
        segs = self.segments
        entries = sd["segments"]
        if len(entries) != len(segs) or any(
                (e[0], e[1], e[2]) != (sg.tensor, sg.offset, sg.length)
                for e, sg in zip(entries, segs)):
            raise ValueError("ZeroLUMA.load_state_dict: segment list differs")
        self.t = int(sd["t"])
        self.base_seed = int(sd["base_seed"])
        hp = dict(sd["hp"])
        hp["betas"] = tuple(hp["betas"])
        self.hp = hp
        self.q_m.copy_(sd["q_m"].to(self.q_m.device, torch.int16))
        self.q_w.copy_(sd["q_w"].to(self.q_w.device, torch.int16))
        k = 0
        for segs_b, eng in zip(self.bucket_segments, self.engines):
            for j in range(len(segs_b)):
                eng.reset_slot(j)
                if self.t > 0:
                    _, _, _, S_m, S_v = entries[k]
                    eng.write_grid(j, self.t & 1, grid_record(float(S_m), float(S_v),
                                                              self.hp["eps"]))
                k += 1

    def scales(self) -> list[tuple[int, int, float, float]]:
        """(tensor, offset, S_m, S_v) of every local segment, bucket order (synchronises)."""
        out = []
        for segs, eng in zip(self.bucket_segments, self.engines):
            host = eng.read_slots()
            for k, sg in enumerate(segs):
                g = host[k]["grid"][self.t & 1]
                out.append((sg.tensor, sg.offset, float(g["S_m"]), float(g["S_v"])))
        return out
