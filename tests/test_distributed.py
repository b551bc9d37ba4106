"""Data-parallel layer on CPU ranks (gloo, world size 2): sharding and the gradient all-reduce,
plus rank failure handled on the host."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from dynaworld_b200.distributed import GradientAllReduce, allreduce_gradients, shard_views, shared_span


def test_shard_views_cover_and_balance():
    for n, world in [(16, 1), (16, 8), (5, 2), (3, 4), (32, 8)]:
        shards = [shard_views(n, world, r) for r in range(world)]
        assert shards[0].start == 0 and shards[-1].stop == n
        assert all(a.stop == b.start for a, b in zip(shards, shards[1:]))
        assert max(s.count for s in shards) - min(s.count for s in shards) <= 1


def test_shard_views_whole_sets():
    shards = [shard_views(64 * 8, 8, r, views_per_set=8, shared_set=False) for r in range(8)]
    assert all(s.start % 8 == 0 and s.count == 64 for s in shards)
    with pytest.raises(ValueError):
        shard_views(10, 2, 0, views_per_set=4, shared_set=False)
    with pytest.raises(ValueError):
        shard_views(10, 2, 2)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, mode, results):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=10))
    try:
        if mode == "sum":
            g1 = torch.full((3, 4), float(rank + 1))
            g2 = torch.arange(5, dtype=torch.float32) * (rank + 1)
            allreduce_gradients([g1, None, g2])
            results[rank] = (g1.sum().item(), g2.tolist())
        elif mode == "span":
            # views of one flat buffer, as the render backward returns them: reduced in place
            flat = torch.arange(12, dtype=torch.float32) * (rank + 1)
            views = [flat[0:3].view(3, 1), flat[3:7], flat[7:12].view(5)]
            assert shared_span(views) is not None
            allreduce_gradients(views)
            red = GradientAllReduce(buckets=2)
            assert red.active()
            extra = torch.ones(4) * (rank + 1)
            red.reduce([extra[:2], extra[2:]])
            red.finish()
            results[rank] = (flat.tolist(), extra.tolist())
        elif mode == "rank_dies":
            if rank == 1:
                raise SystemExit(3)  # leaves between steps, nothing in flight
            try:
                allreduce_gradients([torch.ones(4)])
                results[rank] = "no error"
            except Exception as exc:  # the collective ends with an error instead of hanging
                results[rank] = type(exc).__name__
    finally:
        if dist.is_initialized():
            try:
                dist.destroy_process_group()
            except Exception:
                pass


def test_allreduce_sums_across_two_ranks():
    port = _free_port()
    with mp.get_context("spawn").Manager() as m:
        results = m.dict()
        mp.spawn(_worker, args=(2, port, "sum", results), nprocs=2, join=True)
        assert results[0] == results[1]
        assert results[0][0] == pytest.approx(12 * 3.0)
        assert results[0][1] == pytest.approx([0.0, 3.0, 6.0, 9.0, 12.0])


def test_shared_span_detects_one_flat_buffer():
    flat = torch.zeros(10)
    assert shared_span([flat[4:10], flat[0:4]]) is not None
    assert shared_span([flat[0:4], flat[5:10]]) is None  # a gap
    assert shared_span([flat[0:4], torch.zeros(6)]) is None  # another storage
    assert shared_span([flat.view(2, 5)[:, :2]]) is None  # not contiguous
    span = shared_span([flat[2:5], flat[5:9]])
    assert span.numel() == 7 and span.data_ptr() == flat[2:].data_ptr()


def test_allreduce_in_place_on_views_and_reducer():
    port = _free_port()
    with mp.get_context("spawn").Manager() as m:
        results = m.dict()
        mp.spawn(_worker, args=(2, port, "span", results), nprocs=2, join=True)
        assert results[0] == results[1]
        assert results[0][0] == pytest.approx([3.0 * i for i in range(12)])
        assert results[0][1] == pytest.approx([3.0] * 4)


def test_dead_rank_surfaces_as_error_not_hang():
    port = _free_port()
    ctx = mp.get_context("spawn")
    with ctx.Manager() as m:
        results = m.dict()
        procs = [ctx.Process(target=_worker, args=(r, 2, port, "rank_dies", results)) for r in range(2)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(timeout=60)
        alive = [p for p in procs if p.is_alive()]
        for p in alive:
            p.kill()
        assert not alive, "a rank hung after its peer died"
        assert procs[1].exitcode == 3
        assert results.get(0) not in (None, "no error")
