"""Data-parallel bench plumbing on CPU: world size 2 over gloo (127.0.0.1).

bench.py --gpus N runs N independent replicas; the only cross-rank steps are
the barrier and the max-over-ranks of the measured times (the job finishes
with its slowest replica), and each rank serves its own synthetic requests.
"""
from __future__ import annotations

import os
import socket

import torch.multiprocessing as mp


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank: int, world: int, port: int, errors) -> None:
    import torch
    import torch.distributed as dist
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world)
        import bench
        t = bench.max_over_ranks(torch, dist, 10.0 + 5.0 * rank, "cpu")
        assert t == 10.0 + 5.0 * (world - 1), t
        seeds = [None] * world
        dist.all_gather_object(seeds, bench.rank_seed(rank))
        assert len(set(seeds)) == world  # every replica its own requests
        dist.barrier()
        dist.destroy_process_group()
    except BaseException as e:
        import traceback
        errors.put(f"rank {rank}: {e!r}\n{traceback.format_exc()}")


def test_dp_max_over_ranks_world2():
    world = 2
    ctx = mp.get_context("spawn")
    errors = ctx.SimpleQueue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, errors)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    msgs = []
    while not errors.empty():
        msgs.append(errors.get())
    assert not alive and not msgs, "\n".join(msgs)


def test_single_rank_is_identity():
    import torch
    import bench
    assert bench.max_over_ranks(torch, None, 3.5, "cpu") == 3.5
