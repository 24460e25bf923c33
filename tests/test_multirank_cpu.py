"""Multi-rank host logic on CPU with the gloo backend (world size 2).

The data path has no collective: each rank derives its own cameras from the same plan, and
ranks only meet at the benchmark's barrier and max-over-ranks timing. These tests run those
pieces as real processes, and check that a rank which never arrives ends the others' wait with
an error instead of a hang (the short process-group timeout the benchmark also uses).
"""

from __future__ import annotations

import datetime
import os
import socket

import pytest
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank: int, world: int, port: int, seconds: float) -> None:
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=seconds))


def _shard_worker(rank: int, world: int, port: int, q) -> None:
    from shipinfer_b200.shard import shard_of

    import sys
    sys.path.insert(0, os.path.join(os.path.dirname(__file__)))
    from _data import camera_mix

    _init(rank, world, port, 30)
    fps, _ = camera_mix()
    load = {f"cam{c:02d}": f for c, f in fps.items()}
    mine = shard_of(load, list(range(world)), rank)
    gathered = [None] * world
    dist.all_gather_object(gathered, list(mine))
    # max over ranks of a per-rank "elapsed", as bench.py reports it
    import torch

    t = torch.tensor([float(rank + 1) * 1.5], dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    dist.barrier()
    dist.destroy_process_group()
    if rank == 0:
        q.put((gathered, float(t.item()), sorted(load)))


def test_two_ranks_partition_the_cameras_and_agree_on_the_max():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    mp.start_processes(_shard_worker, args=(2, port, q), nprocs=2, join=True, start_method="spawn")
    gathered, tmax, cameras = q.get(timeout=30)
    flat = [c for shard in gathered for c in shard]
    assert sorted(flat) == cameras and len(set(flat)) == len(flat), "every camera on exactly one rank"
    assert tmax == 3.0
    loads = [sum(160.0 if c == "cam00" else 20.0 for c in shard) for shard in gathered]
    assert abs(loads[0] - loads[1]) <= 20.0, "LPT balance by offered fps"


def _absent_worker(rank: int, world: int, port: int, q) -> None:
    _init(rank, world, port, 3)
    if rank == 1:
        dist.destroy_process_group()  # leaves between steps and never reaches the barrier
        return
    try:
        dist.barrier()
        q.put("returned")
    except Exception as exc:  # the short timeout turns the missing rank into an error
        q.put(f"error: {type(exc).__name__}")


@pytest.mark.timeout(60)
def test_a_rank_that_never_arrives_is_an_error_not_a_hang():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = mp.start_processes(_absent_worker, args=(2, port, q), nprocs=2, join=False, start_method="spawn")
    outcome = q.get(timeout=45)
    for p in procs.processes:
        p.join(timeout=15)
        if p.is_alive():
            p.kill()
    assert outcome.startswith("error"), outcome


def _bench_dist_worker(rank: int, world: int, port: int, q) -> None:
    """bench.py's own Dist (gloo on CPU tensors), driven by the env torchrun sets."""
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, root)
    os.environ.update({"RANK": str(rank), "WORLD_SIZE": str(world), "LOCAL_RANK": str(rank),
                       "MASTER_ADDR": "127.0.0.1", "MASTER_PORT": str(port)})
    import bench

    d = bench.Dist()
    d.init()
    d.barrier()
    per_rank = d.gather(10.0 + rank)
    top = d.max(10.0 + rank)
    summary = bench.per_rank_summary(per_rank, steps=2)
    backend = dist.get_backend()
    d.close()
    if rank == 0:
        q.put((per_rank, top, summary, backend))


def test_bench_plumbing_gathers_per_rank_times_on_gloo():
    """The benchmark's barrier, max over ranks and per-rank gather run on gloo (NCCL is never
    initialised); per_rank_ms reports each rank's per-step time and their min / median / max."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    mp.start_processes(_bench_dist_worker, args=(2, port, q), nprocs=2, join=True, start_method="spawn")
    per_rank, top, summary, backend = q.get(timeout=30)
    assert backend == "gloo"
    assert per_rank == [10.0, 11.0] and top == 11.0
    assert summary == {"min": 5.0, "median": 5.25, "max": 5.5, "ranks": [5.0, 5.5]}
