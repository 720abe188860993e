"""ZeRO-1 shard planning and the post-step gather, on CPU.

The planner must cut the flat parameter space into equal shards whose
per-tensor segments cover every element exactly once, start 8-aligned inside
their tensor (Philox counter and 128-bit loads) and keep the global tensor
index; the gather is checked with two gloo ranks on CPU: each rank writes its
shard, the in-place all_gather_into_tensor must rebuild the full buffer."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from luma_b200.zero import ALIGN, flat_views, plan_layout, shard_segments


def llama_like_numels():
    d, kv, ffn = 512, 128, 1792
    out = [5000 * d]
    for _ in range(3):
        out += [d * d, kv * d, kv * d, d * d, ffn * d, ffn * d, d * ffn, d, d]
    return out + [d, 5000 * d]


@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
@pytest.mark.parametrize("buckets", [1, 3, 8])
@pytest.mark.parametrize("numels", [llama_like_numels(), [1, 7, 8, 9, 1025, 3, 0, 17],
                                    list(np.random.default_rng(0).integers(1, 5000, 300))])
def test_segments_partition_every_tensor(world, buckets, numels):
    lay = plan_layout(numels, world, buckets)
    assert lay.piece % ALIGN == 0 and lay.total >= sum(-(-n // ALIGN) * ALIGN for n in numels)
    assert lay.shard == buckets * lay.piece and lay.total == world * lay.shard
    assert all(s % ALIGN == 0 for s in lay.starts)
    covered = [np.zeros(n, dtype=np.int32) for n in numels]
    for r in range(world):
        local = np.zeros(lay.shard, dtype=np.int32)
        for sg in shard_segments(lay, r):
            lo, hi = lay.owned(r, sg.bucket)
            assert lo <= sg.flat and sg.flat + sg.length <= hi
            assert sg.local == sg.bucket * lay.piece + (sg.flat - lo)
            assert sg.offset % ALIGN == 0 and sg.flat % ALIGN == 0 and sg.local % ALIGN == 0
            assert sg.flat == lay.starts[sg.tensor] + sg.offset
            covered[sg.tensor][sg.offset:sg.offset + sg.length] += 1
            local[sg.local:sg.local + sg.length] += 1
        assert local.max() <= 1
    for c in covered:
        assert np.all(c == 1)


def test_flat_views_share_storage():
    shapes = [(3, 5), (7,), (2, 2, 2)]
    lay = plan_layout([15, 7, 8], 2)
    flat = torch.zeros(lay.total)
    views = flat_views(flat, lay, shapes)
    for k, v in enumerate(views):
        v.fill_(k + 1)
    for k, (v, s) in enumerate(zip(views, lay.starts)):
        assert v.data_ptr() == flat.data_ptr() + 4 * s
        assert torch.all(flat[s:s + v.numel()] == k + 1)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _gather_worker(rank, world, port, numels, buckets, out_q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        lay = plan_layout(numels, world, buckets)
        flat = torch.full((lay.total,), -1.0)
        # "step": this rank writes a known value into every element it owns
        for sg in shard_segments(lay, rank):
            flat[sg.flat:sg.flat + sg.length] = torch.arange(sg.length, dtype=torch.float32) + \
                1000.0 * sg.tensor + sg.offset
        out = flat.clone()
        for b in range(buckets):  # per-bucket in-place gather, as ZeroLUMA.gather does
            lo, hi = lay.owned(rank, b)
            dist.all_gather_into_tensor(out[b * lay.span:(b + 1) * lay.span], out[lo:hi].clone())
        ok = True
        for t, (n, s) in enumerate(zip(lay.numels, lay.starts)):
            want = torch.arange(n, dtype=torch.float32) + 1000.0 * t
            ok &= bool(torch.equal(out[s:s + n], want))
        out_q.put((rank, ok))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,buckets", [(2, 1), (2, 3)])
def test_gather_rebuilds_params_gloo(world, buckets):
    numels = [37, 1024, 5, 999, 64]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gather_worker, args=(r, world, port, numels, buckets, q))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    results = dict(q.get(timeout=10) for _ in range(world))
    assert all(results.values()), results


def test_auto_gather_policy():
    from luma_b200.zero import auto_gather
    assert [auto_gather(w) for w in (1, 2, 4, 8)] == ["copy", "copy", "copy", "nccl"]


def _staged_worker(rank, world, port, numels, buckets, out_q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from luma_b200.zero import gather_bucket_into
        lay = plan_layout(numels, world, buckets)
        # sharded params: this rank's pieces back to back (the grads' layout)
        shard = torch.full((lay.shard,), -1.0)
        for sg in shard_segments(lay, rank):
            shard[sg.local:sg.local + sg.length] = torch.arange(sg.length, dtype=torch.float32) + \
                1000.0 * sg.tensor + sg.offset
        staging = [torch.empty(lay.span) for _ in range(2)]
        full = torch.full((lay.total,), -1.0)
        for b in range(buckets):  # rotating staging buffers, consumed bucket by bucket
            view = gather_bucket_into(staging[b % 2], shard, lay, b)
            full[b * lay.span:(b + 1) * lay.span] = view
        ok = True
        for t, (n, s) in enumerate(zip(lay.numels, lay.starts)):
            want = torch.arange(n, dtype=torch.float32) + 1000.0 * t
            ok &= bool(torch.equal(full[s:s + n], want))
        out_q.put((rank, ok))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,buckets", [(2, 1), (2, 4), (3, 3)])
def test_staged_gather_rebuilds_buckets_gloo(world, buckets):
    """Sharded-params mode: each bucket gathered into a rotating staging buffer
    holds the flat positions of that bucket."""
    numels = [37, 1024, 5, 999, 64]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_staged_worker, args=(r, world, port, numels, buckets, q))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    results = dict(q.get(timeout=10) for _ in range(world))
    assert all(results.values()), results


def test_zero_luma_validates_buffers_on_cpu():
    from luma_b200.zero import ZeroLUMA
    lay = plan_layout([100, 37], 2, 2)
    with pytest.raises(ValueError, match="elements"):
        ZeroLUMA(torch.zeros(lay.total + 1, dtype=torch.bfloat16), lay, 0)
    with pytest.raises(ValueError, match="elements"):  # sharded mode holds lay.shard elements
        ZeroLUMA(torch.zeros(lay.total, dtype=torch.bfloat16), lay, 0, replica=False)
    with pytest.raises(ValueError, match="staging"):
        ZeroLUMA(torch.zeros(lay.shard, dtype=torch.bfloat16), lay, 0, replica=False, staging=0)
    with pytest.raises(ValueError, match="float32 or bfloat16"):
        ZeroLUMA(torch.zeros(lay.total, dtype=torch.float16), lay, 0)
    with pytest.raises(RuntimeError, match="CUDA"):
        ZeroLUMA(torch.zeros(lay.total, dtype=torch.bfloat16), lay, 0)


@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("streams", [1, 2, 0])
def test_push_order_rotates_and_covers_peers(world, streams):
    from luma_b200.zero import push_order
    firsts = []
    for r in range(world):
        order = push_order(r, world, streams)
        peers = [p for p, _ in order]
        assert sorted(peers) == [p for p in range(world) if p != r]
        assert peers[0] == (r + 1) % world
        n_st = len({k for _, k in order})
        assert n_st == (world - 1 if streams <= 0 else min(streams, world - 1))
        firsts.append(peers[0])
    # at every position of the order, the ranks target distinct peers (a permutation)
    for pos in range(world - 1):
        assert len({push_order(r, world, streams)[pos][0] for r in range(world)}) == world


def test_lockstep_applies_only_to_one_ordered_stream_beyond_two_ranks():
    from luma_b200.zero import lockstep_applies, push_order
    assert lockstep_applies(True, 1, 8) and lockstep_applies(True, 1, 3)
    assert not lockstep_applies(False, 1, 8)
    assert not lockstep_applies(True, 2, 8)   # pushes on two streams are not ordered
    assert not lockstep_applies(True, 1, 2)   # one push per bucket: nothing to separate
    # in lockstep, phase k of every rank targets a distinct peer (a permutation)
    for world in (3, 4, 8):
        for k in range(world - 1):
            assert len({push_order(r, world, 1)[k][0] for r in range(world)}) == world


def _peer_fallback_worker(rank, world, port, out_q):
    import warnings
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from luma_b200.zero import make_peer_gather
        lay = plan_layout([100, 37], world)
        # host memory has no CUDA IPC handle: the export fails on every rank,
        # like VMM-backed (expandable_segments) device memory does
        with warnings.catch_warnings(record=True) as w:
            warnings.simplefilter("always")
            pg = make_peer_gather(torch.zeros(lay.total), lay, rank)
        dist.barrier()  # no rank is left inside a collective
        out_q.put((rank, (pg is None, any("using NCCL" in str(x.message) for x in w))))
    finally:
        dist.destroy_process_group()


def test_copy_gather_falls_back_to_nccl_on_every_rank_gloo():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_peer_fallback_worker, args=(r, world, port, q))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    results = dict(q.get(timeout=10) for _ in range(world))
    assert all(v == (True, True) for v in results.values()), results


def test_layout_dict_round_trip():
    from luma_b200.zero import FlatLayout
    lay = plan_layout([100, 37, 1, 4096], 4, 3)
    assert FlatLayout.from_dict(lay.to_dict()) == lay
    other = plan_layout([100, 37, 1, 4096], 2, 3)
    assert FlatLayout.from_dict(other.to_dict()) != lay
