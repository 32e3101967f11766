"""Episode data parallelism: one process per GPU, static shards, no collective.

Inference episodes are independent, so they are split into contiguous blocks,
one per rank, and each rank runs its block on its own GPU. Nothing is
exchanged on the data path (no NCCL); the only cross-rank operations are the
start barrier and the max-over-ranks of the timing, which bench.py takes from
a torch.distributed gloo group (`max_over_ranks` below; CPU tensors, no NCCL).

`run_workers` is the host-side launcher for jobs that do not come from
torchrun: it spawns one process per rank (CUDA_VISIBLE_DEVICES pinned when GPUs
are used), gathers each episode's result over a pipe, and watches every rank
for a non-zero exit, an exception or a time limit. Results are deterministic
per episode seed, so the episodes of a failed rank can be re-run (`retries`).
"""

from __future__ import annotations

import dataclasses
import multiprocessing as mp
import os
import queue
import time
import traceback
from typing import Any, Callable


def episode_shard(total: int, world: int, rank: int) -> list[int]:
    """Contiguous block of episode ids for `rank` (sizes differ by at most one)."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} / world {world}")
    base, extra = divmod(total, world)
    start = rank * base + min(rank, extra)
    return list(range(start, start + base + (1 if rank < extra else 0)))


def max_over_ranks(value: float, device=None) -> float:
    """Max of a per-rank scalar over the default process group (any backend)."""
    import torch
    import torch.distributed as dist

    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return value
    t = torch.tensor([value], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


@dataclasses.dataclass
class RankFailure:
    rank: int
    episodes: list[int]
    reason: str


@dataclasses.dataclass
class DPResult:
    results: dict[int, Any]
    failures: list[RankFailure]  # failures whose episodes are still missing
    history: list[RankFailure]  # every failure seen, including recovered ones
    wall_s: float

    @property
    def ok(self) -> bool:
        return not self.failures


def _worker_main(worker, rank, world, episodes, q, env):
    os.environ.update(env)
    try:
        for ep in episodes:
            q.put(("result", rank, ep, worker(rank, world, ep)))
        q.put(("done", rank, None, None))
    except BaseException:  # noqa: BLE001 - reported to the parent, then exit non-zero
        q.put(("error", rank, None, traceback.format_exc(limit=5)))
        raise


def run_workers(worker: Callable[[int, int, int], Any], total_episodes: int, nprocs: int,
                timeout_s: float = 600.0, use_gpus: bool = False, retries: int = 0,
                poll_s: float = 0.05) -> DPResult:
    """Runs worker(rank, world, episode) for every episode over `nprocs` processes.

    The worker must be a picklable top-level function. A rank that raises, exits
    non-zero or exceeds `timeout_s` is recorded in `failures` with the episodes it
    did not deliver; its process is terminated. With retries > 0 those episodes
    are run again on fresh processes.
    """
    ctx = mp.get_context("spawn")
    t0 = time.time()
    results: dict[int, Any] = {}
    todo = list(range(total_episodes))
    failures: list[RankFailure] = []
    for attempt in range(retries + 1):
        if not todo:
            break
        world = min(nprocs, len(todo))
        q = ctx.Queue()
        procs, owned = {}, {}
        for r in range(world):
            eps = [todo[i] for i in episode_shard(len(todo), world, r)]
            env = {"CUDA_VISIBLE_DEVICES": str(r)} if use_gpus else {}
            p = ctx.Process(target=_worker_main, args=(worker, r, world, eps, q, env),
                            daemon=True)
            p.start()
            procs[r], owned[r] = p, eps
        pending = {r: set(owned[r]) for r in procs}
        done, errors = set(), {}
        deadline = time.time() + timeout_s
        while len(done) + len(errors) < world:
            try:
                kind, r, ep, payload = q.get(timeout=poll_s)
                if kind == "result":
                    results[ep] = payload
                    pending[r].discard(ep)
                elif kind == "done":
                    done.add(r)
                else:
                    errors[r] = f"exception: {payload.strip().splitlines()[-1]}"
            except queue.Empty:
                pass
            for r, p in procs.items():
                if r in done or r in errors:
                    continue
                if not p.is_alive() and p.exitcode not in (0, None):
                    errors[r] = f"exit code {p.exitcode}"
            if time.time() > deadline:
                for r in procs:
                    if r not in done and r not in errors:
                        errors[r] = f"timeout after {timeout_s:.1f} s"
                break
        for r, p in procs.items():
            if p.is_alive():
                p.terminate()  # only our own child processes, by handle
            p.join(timeout=5)
        attempt_failures = [RankFailure(r, sorted(pending[r]), errors[r]) for r in sorted(errors)]
        failures.extend(attempt_failures)
        todo = sorted(ep for f in attempt_failures for ep in f.episodes)
    missing = [f for f in failures if any(ep not in results for ep in f.episodes)]
    return DPResult(results=results, failures=missing, history=failures,
                    wall_s=time.time() - t0)
