"""Head-sharded (batch-sharded) multi-GPU bench path, host side on CPU.

Each batch index has its own seed, so the shards of any GPU count concatenate
to the same global tensors; gloo ranks agree on the max-over-ranks time.
"""
import os
import socket

import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import bench


def test_shards_concatenate_to_the_same_global_tensors():
    B, S, H, D = 8, 16, 2, 16
    full = bench.gen_shard(0, B, S, H, D, 1.0, torch.device("cpu"))
    for world in (2, 4, 8):
        parts = [bench.gen_shard(r * B // world, (r + 1) * B // world, S, H, D, 1.0,
                                 torch.device("cpu")) for r in range(world)]
        for i in range(4):
            assert torch.equal(torch.cat([p[i] for p in parts]), full[i])


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    t = torch.tensor([float(10 + rank)], dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    q.put((rank, float(t.item())))
    dist.destroy_process_group()


def test_max_over_ranks_timing():
    s = socket.socket(); s.bind(("127.0.0.1", 0)); port = s.getsockname()[1]; s.close()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    [p.start() for p in ps]
    res = [q.get(timeout=60) for _ in range(2)]
    [p.join(timeout=30) for p in ps]
    assert all(v == 11.0 for _, v in res)


def test_near_gpu_restores_affinity_and_tolerates_unknown_gpu():
    # Without a GPU (or NVML) the GPU-local CPU set is unknown: the context
    # runs the body unchanged and leaves the process affinity as it was.
    before = os.sched_getaffinity(0)
    with bench.near_gpu(0) as known:
        if not known:
            assert os.sched_getaffinity(0) == before
    assert os.sched_getaffinity(0) == before
