"""Episode data parallelism on CPU: sharding, the process launcher with injected
failures (an exception, a non-zero exit, a hang), and the world-size-2 gloo path
bench.py uses for its barrier and max-over-ranks timing (with bench.py's own
cfg4 / cfg5 sharding)."""

import multiprocessing as mp
import socket

import pytest

import dp_workers
from umic_b200.dp import episode_shard, run_workers


@pytest.mark.parametrize("total,world", [(8, 1), (8, 2), (8, 3), (8, 8), (32, 8), (5, 8)])
def test_shards_cover_every_episode_once(total, world):
    shards = [episode_shard(total, world, r) for r in range(world)]
    flat = [e for s in shards for e in s]
    assert flat == list(range(total))
    sizes = [len(s) for s in shards]
    assert max(sizes) - min(sizes) <= 1


def test_launcher_gathers_all_results():
    res = run_workers(dp_workers.square, 8, 2, timeout_s=120)
    assert res.ok and sorted(res.results) == list(range(8))
    assert all(res.results[e]["value"] == e * e for e in range(8))
    assert {res.results[e]["rank"] for e in range(8)} == {0, 1}


def test_exception_on_a_rank_is_reported_and_retried():
    res = run_workers(dp_workers.fail_on_rank1, 4, 2, timeout_s=120, retries=0)
    assert not res.ok
    assert res.failures[0].rank == 1 and "injected failure" in res.failures[0].reason
    assert res.failures[0].episodes == [2, 3]
    res = run_workers(dp_workers.fail_on_rank1, 4, 2, timeout_s=120, retries=1)
    assert sorted(res.results) == [0, 1, 2, 3]
    assert len(res.history) == 1


def test_rank_exit_is_detected():
    res = run_workers(dp_workers.exit_on_rank0, 4, 2, timeout_s=60)
    assert [f.rank for f in res.failures] == [0]
    assert "exit code 3" in res.failures[0].reason
    assert sorted(res.results) == [2, 3]


def test_hung_rank_times_out():
    res = run_workers(dp_workers.hang_on_rank1, 4, 2, timeout_s=8)
    assert [f.rank for f in res.failures] == [1]
    assert "timeout" in res.failures[0].reason
    assert res.wall_s < 60


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_gloo_world_size_2_barrier_and_max():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=dp_workers.gloo_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = sorted(q.get(timeout=120) for _ in range(2))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    # rank 0: episodes 0..3 (sum 6); rank 1: 4..7 (sum 22) + 1 -> max 23 on both
    assert out[0][1] == out[1][1] == 23.0
    assert out[0][2] == [[0, 1, 2, 3], [4, 5, 6, 7]]


@pytest.mark.parametrize("world", [2, 3, 8])
def test_bench_gloo_ranks_shard_cfg4_and_cfg5(world):
    """bench.py's Ranks on a gloo group: every cfg4 (8) and cfg5 (32) episode lands on
    exactly one rank in contiguous blocks, and the max over ranks reaches every rank.
    With a loopback master address the group runs over the loopback device."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=dp_workers.bench_ranks, args=(r, world, port, q))
             for r in range(world)]
    for p in procs:
        p.start()
    out = sorted(q.get(timeout=180) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for total, col in ((8, 1), (32, 2)):
        covered = []
        for row in out:
            first, count = row[col]
            covered.extend(range(first, first + count))
        assert covered == list(range(total))
    flow_counts = [row[2][1] for row in out]
    expect = max(c * 10 + r for r, c in enumerate(flow_counts))
    assert all(row[3] == expect for row in out)
    assert all(row[4] == "lo" for row in out)


def test_bench_progress_watchdog(tmp_path):
    """bench.py's phase markers and stall watchdog: a phase that outlasts the watchdog's
    limit gets the rank's Python stack on stderr; after close() nothing more is dumped."""
    path = tmp_path / "stderr.txt"
    p = mp.get_context("spawn").Process(target=dp_workers.progress_stall, args=(str(path),))
    p.start()
    p.join(timeout=120)
    assert p.exitcode == 0
    text = path.read_text()
    assert "[bench rank 1 +" in text and "] a phase that stalls" in text
    assert "] the next phase" in text
    dumps = text.count("progress_stall")
    assert 1 <= dumps <= 3  # one or two dumps during the 1.3 s stall, none after close()
    assert text.index("a phase that stalls") < text.index("progress_stall") < text.index(
        "the next phase")
