"""The multi-rank host logic of bench.py on CPU: two gloo ranks on 127.0.0.1 take the max of
their timings and compute the weak-scaling job rate the way `bench.py --gpus N` does under
torchrun (no GPU, no collective on the data path)."""
import os
import socket
import sys

import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, out):
    sys.path.insert(0, ROOT)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import bench
        elapsed_ms = 10.0 + 5.0 * rank       # rank 1 is the slow one
        t = bench.rank_max(dist, elapsed_ms, "cpu")
        rate = bench.job_rate(4096 * 20, world, t)
        out[rank].copy_(torch.tensor([t, rate], dtype=torch.float64))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_max_time_and_weak_scaling_rate():
    world = 2
    port = _free_port()
    out = [torch.zeros(2, dtype=torch.float64).share_memory_() for _ in range(world)]
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_rank, args=(r, world, port, out)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    for r in range(world):
        t, rate = out[r].tolist()
        assert t == 15.0                           # every rank sees the slowest rank's time
        assert abs(rate - 4096 * 20 * 2 / 0.015) < 1e-6 * rate


def test_single_process_identity():
    sys.path.insert(0, ROOT)
    import bench
    assert bench.rank_max(None, 3.5, "cpu") == 3.5
    assert bench.job_rate(100, 1, 1000.0) == 100.0
