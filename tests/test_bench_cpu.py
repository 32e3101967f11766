"""bench.py's host-side pieces on CPU: the clock-record parser (it decides which
throttle reasons a run reports), the roofline peaks and the episode shares."""

import bench


class _DoneProc:
    """Stands in for the finished nvidia-smi process."""

    def terminate(self):
        pass

    def wait(self, timeout=None):
        return 0


def _sampler(lines):
    s = bench.ClockSampler(0)
    s.proc = _DoneProc()
    s.lines = list(lines)
    return s


def test_clock_record_median_and_reasons():
    # clocks.sm, clocks.max.sm, power.draw, hw_slowdown, hw_thermal, sw_thermal, sw_power_cap
    lines = ["1395, 1965, 998.1, Not Active, Not Active, Not Active, Active",
             "1410, 1965, 1001.3, Not Active, Not Active, Not Active, Active",
             "1380, 1965, 995.0, Not Active, Not Active, Not Active, Not Active",
             "garbage", ""]
    r = _sampler(lines).stop()
    assert r["sm_mhz"] == 1395 and r["sm_max_mhz"] == 1965 and r["samples"] == 3
    assert r["reasons"] == ["sw_power_cap"]


def test_clock_record_flags_thermal_and_hw_slowdown():
    lines = ["1200, 1965, 700.0, Active, Not Active, Active, Not Active"]
    r = _sampler(lines).stop()
    assert r["reasons"] == ["hw_slowdown", "sw_thermal_slowdown"]


def test_clock_record_without_nvidia_smi():
    r = bench.ClockSampler(0).stop()
    assert r["sm_mhz"] is None and r["reasons"] == ["nvidia-smi unavailable"]


def test_peaks_measured_file_or_fallback(tmp_path, monkeypatch):
    monkeypatch.setattr(bench, "ROOT", tmp_path)
    p = bench._peaks()  # no measured file: the pool's earlier measurement
    assert p["source"] == "fallback" and p["hbm_gbs"] == 6650.0
    (tmp_path / "MEASURED_PEAKS.json").write_text(
        '{"hbm_gbs": 6546.9, "bf16_tflops": 1639.8, "bf16_tflops_sustained": 1396.8}')
    p = bench._peaks()
    assert p["source"] == "measured"
    assert (p["hbm_gbs"], p["bf16_tflops"], p["bf16_tflops_sustained"]) == (6546.9, 1639.8,
                                                                             1396.8)


def test_episode_shares_cover_the_workloads_at_every_n():
    for world in (1, 2, 4, 8):
        for total in (bench.TOTAL_EPISODES, bench.FLOW_EPISODES):
            blocks = [bench._share(total, r, world) for r in range(world)]
            covered = [e for first, count in blocks for e in range(first, first + count)]
            assert covered == list(range(total))
            assert max(c for _, c in blocks) - min(c for _, c in blocks) <= 1
