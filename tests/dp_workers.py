"""Picklable worker functions for the data-parallel launcher tests (CPU only)."""

import os
import time


def square(rank, world, episode):
    return {"rank": rank, "world": world, "value": episode * episode, "pid": os.getpid()}


def fail_on_rank1(rank, world, episode):
    # Fails only where rank 1 meets episode 2 (the first attempt's sharding); a
    # retry reshards the leftover episodes so the same episode lands on rank 0.
    if rank == 1 and episode == 2:
        raise RuntimeError("injected failure on rank 1")
    return episode * episode


def exit_on_rank0(rank, world, episode):
    if rank == 0:
        os._exit(3)
    return episode


def hang_on_rank1(rank, world, episode):
    if rank == 1:
        time.sleep(3600)
    return episode


def gloo_rank(rank, world, port, out):
    import torch
    import torch.distributed as dist

    from umic_b200.dp import episode_shard, max_over_ranks

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        eps = episode_shard(8, world, rank)
        local = float(sum(eps)) + rank  # a per-rank "time"
        dist.barrier()
        m = max_over_ranks(local)
        gathered = [None] * world
        dist.all_gather_object(gathered, eps)
        out.put((rank, m, gathered))
    finally:
        dist.destroy_process_group()


def bench_ranks(rank, world, port, out):
    """bench.py's host coordination on gloo: its cfg4 / cfg5 episode shards, barrier
    and max over ranks, as each torchrun rank runs them."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world), LOCAL_RANK=str(rank))
    import bench

    ranks = bench.Ranks(world)
    try:
        lm = bench._share(bench.TOTAL_EPISODES, rank, world)
        flow = bench._share(bench.FLOW_EPISODES, rank, world)
        ranks.barrier()
        m = ranks.max(float(flow[1] * 10 + rank))
        out.put((rank, lm, flow, m, os.environ.get("GLOO_SOCKET_IFNAME")))
    finally:
        ranks.close()


def progress_stall(path):
    """bench.py's Progress on a rank of a 2-rank job whose phase outlasts the watchdog:
    stderr (fd 2) goes to `path`."""
    import time

    fd = os.open(path, os.O_WRONLY | os.O_CREAT | os.O_TRUNC, 0o644)
    os.dup2(fd, 2)
    import bench

    progress = bench.Progress(rank=1, world=2, stall_s=0.5)
    progress("a phase that stalls")
    time.sleep(1.3)
    progress("the next phase")
    progress.close()
    time.sleep(0.8)  # cancelled: no further dump
