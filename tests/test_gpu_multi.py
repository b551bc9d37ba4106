"""Data parallelism on 2 GPUs (NCCL): two ranks render disjoint halves of the frames of one scene
and all-reduce the Gaussian gradients; the result must equal one GPU rendering every frame.
Skipped unless two CUDA devices are visible."""
import datetime
import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu

FRAMES = 8


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _grads(wl, device):
    from gpu_helpers import render_raw

    out = render_raw(wl, device=device)
    return {k: v for k, v in out.items() if k.startswith("grad_")}, out["loss"]


def _rank(rank, world, port, queue, mode="explicit"):
    import sys

    sys.path.insert(0, os.path.dirname(__file__))
    sys.path.insert(0, os.path.dirname(os.path.dirname(__file__)))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import torch.distributed as dist

    from dynaworld_b200 import synthetic
    from dynaworld_b200.distributed import allreduce_gradients, shard_views

    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    try:
        full = synthetic.dynamic128(scale=0.125, image_scale=0.5, frames=FRAMES)
        sh = shard_views(FRAMES, world, rank)
        part = full.views(sh.start, sh.stop)
        if mode == "reducer":  # summed inside the backward, overlapped with the chain rule
            from dynaworld_b200.distributed import GradientAllReduce
            from dynaworld_b200.render import set_gradient_reducer

            set_gradient_reducer(GradientAllReduce(buckets=3))
            grads, _ = _grads(part, dev)
            set_gradient_reducer(None)
            tensors = [grads[k].to(dev) for k in sorted(grads)]
        else:
            grads, _ = _grads(part, dev)
            tensors = [grads[k].to(dev) for k in sorted(grads)]
            allreduce_gradients(tensors)
        if rank == 0:
            single, _ = _grads(full, dev)
            worst = 0.0
            for k, t in zip(sorted(grads), tensors):
                ref = single[k]
                worst = max(worst, (t.cpu() - ref).abs().max().item() / max(ref.abs().max().item(), 1e-30))
            queue.put(worst)
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("mode", ["explicit", "reducer"])
def test_two_gpu_allreduce_matches_single_gpu(mode):
    ctx = torch.multiprocessing.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, queue, mode)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    worst = queue.get(timeout=10)
    assert worst <= 1e-5, worst
