"""CPU tests of the multi-process (one process per GPU) host logic with the gloo
backend, world size 2: batch slices are disjoint and cover the global batch, the
throughput aggregation takes the slowest rank's time and sums every rank's
images, and a failing rank surfaces as an error on the other rank's collective
instead of a hang (short process-group timeout)."""
import os
import sys
from datetime import timedelta
from pathlib import Path

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parent.parent


def _init(rank, world, port):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=20))


def _aggregate_worker(rank, world, port, q):
    sys.path.insert(0, str(ROOT))
    import bench
    _init(rank, world, port)
    try:
        ms, images = bench.job_throughput(10.0 + 5.0 * rank, 4 * (rank + 1), world)
        q.put((rank, ms, images, bench.rank_images(rank, 2)))
    finally:
        dist.destroy_process_group()


def _failing_worker(rank, world, port, q):
    _init(rank, world, port)
    if rank == 1:
        # this rank dies between steps, with nothing of its own in flight
        dist.destroy_process_group()
        q.put((rank, "left"))
        return
    try:
        t = torch.ones(1)
        dist.all_reduce(t)
        q.put((rank, "no error"))
    except Exception as e:  # gloo reports the missing peer
        q.put((rank, f"error: {type(e).__name__}"))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def _run(target, world, port):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=target, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=120)
    return sorted(out, key=lambda x: x[0])


def test_throughput_aggregation_two_ranks():
    res = _run(_aggregate_worker, 2, 29731)
    for rank, ms, images, imgs in res:
        assert ms == 15.0           # slowest rank
        assert images == 4 + 8      # every rank's images
    assert res[0][3] == [0, 1] and res[1][3] == [2, 3]  # disjoint, contiguous slices


def test_rank_failure_is_reported_not_hung():
    res = _run(_failing_worker, 2, 29733)
    assert res[1][1] == "left"
    assert res[0][1].startswith("error")
