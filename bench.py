"""LM prefill benchmark (BASELINE cfg4) for the B200 fused-inference hot path.

Workload: the 36-layer Qwen3-VL-shaped LM (hidden 4096, GQA 32/8 x 128,
SwiGLU 12288, vocab 151936), random-init weights ~N(0, 0.02), patched with
umic_b200.apply(); 8 independent episodes of 3100 uniform-random token ids,
sharded over the ranks (8 episodes in total) and run as one batched prefill per
rank. A step = one prefill of this rank's episodes into an in-place KV cache,
ending with the greedy next token. The metric is prefill tokens/s for the whole
job; `e2e` is the same through the public API with the token ids copied from
pinned host memory and the next tokens read back inside the timed region.

Also on the line, at every N: `decode` (the 64 greedy cfg4 steps, CUDA-graph
replay) and `flow` (cfg5: 32 flow-matching episodes sharded 32/N per rank, 10
Euler steps each over a 3100-token prefix, episodes/s of the whole job). At one
GPU also `kernels` (cfg1 block and cfg2 norm / RoPE kernels vs unfused eager),
`vision` (cfg3) and the eager comparisons, from a subprocess. Ranks share no
data: a gloo group carries only the start / stop barriers and the max over
ranks of each device-timed region (no NCCL anywhere).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl umic|reference]

--impl reference times the reference's eager CPU path (the unpatched HF model the
reference patches: full 36-layer prefill of one 3100-token episode per step) on
the host cores and prints the same JSON line with impl=reference.
"""

from __future__ import annotations

import argparse
import datetime
import faulthandler
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
for _p in (ROOT, ROOT / "umic-alpamayo_b200"):
    if str(_p) not in sys.path:
        sys.path.insert(0, str(_p))

METRIC = "prefill tokens/s (LM cfg4, 3100-token episodes)"
UNIT = "tokens/s"
TOTAL_EPISODES = 8
TOKENS = 3100
LAYERS = 36
HIDDEN, INTER = 4096, 12288
FLOW_EPISODES = 32
# DRAM bytes (read + write) of one dual-GEMM launch at the 8-episode shape (M = 24800),
# measured by ncu (2.111 GB read + 0.608 GB written) on the CTA-pair kernel.
DUAL_GEMM_TRAFFIC_M24800 = 2.72e9


def _peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained", d["bf16_tflops"]),
                "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0,
            "source": "fallback"}


def _config(world: int, episodes: int) -> dict:
    return {"workload": "cfg4 LM prefill", "model": "36L-4096H-GQA32/8-SwiGLU12288",
            "global_batch": TOTAL_EPISODES, "seq_len": TOKENS, "episodes_per_rank": episodes,
            "parallelism": f"episode-dp{world}",
            "l2": "inputs larger than L2 (15.4 GB of weights streamed per step)"}


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during the timed region."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.lines: list[str] = []
        self.t: threading.Thread | None = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100", "-i", str(self.index)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self.t = threading.Thread(target=self._read, daemon=True)
        self.t.start()

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        if self.t:
            self.t.join(timeout=2)
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 7:
                continue
            try:
                sm.append(float(parts[0]))
                smax = float(parts[1])
            except ValueError:
                continue
            for n, v in zip(names, parts[3:7]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax,
                "reasons": sorted(reasons), "samples": len(sm)}


def _dist():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def _share(total: int, rank: int, world: int) -> tuple[int, int]:
    """(first unit, units) of `rank`'s contiguous block of `total` episodes."""
    from umic_b200.dp import episode_shard

    block = episode_shard(total, world, rank)
    return (block[0] if block else 0), len(block)


# ----------------------------------------------------------------- reference arm

def run_reference(args) -> None:
    """The reference's eager CPU path on the host cores, rank 0 only: every step is a
    full 36-layer prefill of one 3100-token episode (a bounded sample of the 8-episode
    workload; tokens/s does not depend on how many episodes run one after another)."""
    world, rank, _ = _dist()
    if rank != 0:
        return
    from oracle.cpu_baseline import CpuLM, time_lm_prefill

    lm = CpuLM(LAYERS)
    r = time_lm_prefill(tokens=TOKENS, layers=LAYERS, warmup=args.warmup, repeats=args.steps,
                        model=lm)
    total = sum(r["seconds"])
    value = args.steps * TOKENS / total
    cpu = {"value": value, "unit": UNIT, "cores": r["torch_threads"], "kind": "port",
           "sample": r["sample"], "cpu": r["cpu"], "physical_cores": r["physical_cores"],
           "logical_cores": r["logical_cores"], "seconds_per_step": r["seconds"]}
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": total / args.steps * 1e3,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (random-init weights, uniform token ids)", "impl": "reference",
        "config": _config(args.gpus, _share(TOTAL_EPISODES, 0, args.gpus)[1]),
        "cpu_baseline": cpu,
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# -------------------------------------------------------------------- GPU arm

class Progress:
    """Multi-rank runs only: a line on stderr as each rank begins a phase, and a
    watchdog that dumps every thread's Python stack to stderr when no new phase has
    begun for `stall_s` seconds, so that a rank which stops shows where."""

    def __init__(self, rank: int, world: int, stall_s: float = 240.0):
        self.on = world > 1
        self.rank = rank
        self.stall_s = stall_s
        self.t0 = time.monotonic()

    def __call__(self, phase: str) -> None:
        if not self.on:
            return
        print(f"[bench rank {self.rank} +{time.monotonic() - self.t0:.1f}s] {phase}",
              file=sys.stderr, flush=True)
        faulthandler.dump_traceback_later(self.stall_s, repeat=True, file=sys.__stderr__)

    def close(self) -> None:
        if self.on:
            faulthandler.cancel_dump_traceback_later()


class Ranks:
    """Host-side coordination of the ranks: barriers and max-over-ranks through a gloo
    group (CPU tensors). Nothing on the data path is exchanged."""

    # A rank that waits this long for the others ends with an error instead of waiting on.
    TIMEOUT_S = 300

    def __init__(self, world: int):
        self.world = world
        if world > 1:
            import torch.distributed as dist

            # All ranks share one host. Without an interface named, gloo binds to the
            # address the host name resolves to, which on an isolated box need not be
            # reachable even from the same host; the loopback device always is.
            if os.environ.get("MASTER_ADDR", "127.0.0.1") in ("127.0.0.1", "localhost"):
                os.environ.setdefault("GLOO_SOCKET_IFNAME", "lo")
            dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=self.TIMEOUT_S))
            self.dist = dist

    def barrier(self) -> None:
        if self.world > 1:
            self.dist.barrier()

    def max(self, x: float) -> float:
        from umic_b200.dp import max_over_ranks

        return max_over_ranks(x) if self.world > 1 else x

    def close(self) -> None:
        if self.world > 1:
            self.dist.barrier()
            self.dist.destroy_process_group()


def _timed(ranks: Ranks, fn, steps: int) -> float:
    """Device time (ms) of `steps` calls, barrier + synchronize on both sides, max over
    ranks."""
    import torch

    ranks.barrier()
    torch.cuda.synchronize()
    s = torch.cuda.Event(enable_timing=True)
    e = torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(steps):
        fn()
    e.record()
    torch.cuda.synchronize()
    ranks.barrier()
    return ranks.max(s.elapsed_time(e))


def _flow_dp(ranks: Ranks, dev, rank: int, world: int, runs: int = 3) -> dict:
    """cfg5 sharded: this rank's block of the 32 episodes (64 action tokens, 10 Euler
    steps over a 3100-token prefix) through the patched expert with the step graph;
    episodes/s of the whole job from the max over ranks."""
    import torch

    from umic_b200 import UmicConfig, apply
    from umic_b200.extras import _prefix_cache
    from umic_b200.workloads import (CFG5_EXPERT, FLOW_STEPS, FLOW_TOKENS, AlpamayoStandIn,
                                     build_text_model, flow_sample)

    first, count = _share(FLOW_EPISODES, rank, world)
    cfg = CFG5_EXPERT
    expert = build_text_model(cfg, device=dev, seed=5)
    g = torch.Generator().manual_seed(31)
    x_all = torch.randn(FLOW_EPISODES, FLOW_TOKENS, cfg["hidden_size"], generator=g)
    x0 = x_all[first:first + count].to(dev, torch.bfloat16)
    cache = _prefix_cache(cfg["num_hidden_layers"], count, cfg["num_key_value_heads"], TOKENS,
                          cfg["head_dim"], dev, seed=30 + rank)
    apply(AlpamayoStandIn(torch.nn.Module(), expert=expert),
          UmicConfig(decode_graph=False, decode_cache=False))
    for _ in range(2):  # eager warm-up steps, graph capture, first replays
        flow_sample(expert, cache, TOKENS, x0, graph=True)
    ms = _timed(ranks, lambda: flow_sample(expert, cache, TOKENS, x0, graph=True), runs) / runs
    return {"episodes": FLOW_EPISODES, "episodes_per_rank": count, "action_tokens": FLOW_TOKENS,
            "prefix_tokens": TOKENS, "euler_steps": FLOW_STEPS, "dp_ms": ms,
            "episodes_per_s": FLOW_EPISODES / (ms / 1e3), "scaling": "strong"}


def run_umic(args) -> None:
    import torch

    world, rank, local = _dist()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    progress = Progress(rank, world)
    progress("joining the group")
    ranks = Ranks(world)
    progress("building the model")

    from umic_b200 import UmicConfig, apply
    from umic_b200.kernels import _common as kc
    from umic_b200.workloads import AlpamayoStandIn, build_vlm, kv_cache_for, prefill, prefill_ids

    first, episodes = _share(TOTAL_EPISODES, rank, world)
    n_decode = args.decode_steps
    vlm = build_vlm(device=dev, seed=4)
    all_ids = prefill_ids(TOTAL_EPISODES, TOKENS, seed=4)
    ids_host = all_ids[first:first + episodes].contiguous().pin_memory()
    ids = ids_host.to(dev)
    cache = kv_cache_for(vlm, episodes, TOKENS + n_decode + 8, dev)

    def step():
        cache.crop(0)
        return prefill(vlm, ids, cache)

    # ---- unfused torch-eager GPU path on the same weights (reported, not the metric):
    # the unpatched HF model with its own DynamicCache, as the reference starts from.
    eager = {}
    if not args.skip_eager:
        def eager_step():
            with torch.no_grad():
                out = vlm(input_ids=ids, use_cache=True, logits_to_keep=1)
            return out.logits[:, -1].argmax(-1)

        progress("unfused eager steps")
        ref_next = eager_step().clone()
        eager_step()
        n_e = max(2, args.steps // 2)
        ms = _timed(ranks, eager_step, n_e) / n_e
        eager = {"value": TOTAL_EPISODES * TOKENS / (ms / 1e3), "ms_per_step": ms,
                 "what": "unpatched HF modules + DynamicCache, bf16, SDPA, same weights/inputs"}
    progress("apply and warm-up")
    model = AlpamayoStandIn(vlm)
    report = apply(model, UmicConfig(max_new_tokens=n_decode + 8))

    # ---- warm-up, then the timed prefill steps (inputs resident in HBM)
    for _ in range(args.warmup):
        nxt = step()
    torch.cuda.synchronize()
    parity = {}
    if eager:
        parity["first_token_match"] = f"{int((nxt == ref_next).sum())}/{episodes}"
    before = sum(v for k, v in kc.stats.items() if k.startswith("umic_"))
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    progress("timed prefill steps")
    clocks = ClockSampler(vis.split(",")[local] if vis else local)
    clocks.start()
    kc.start_probe("umic_gemm_gate_silu_mul")
    torch.cuda.nvtx.range_push("umic_timed")  # lets ncu --nvtx-include select this region
    ms_total = _timed(ranks, step, args.steps)
    torch.cuda.nvtx.range_pop()
    dur = kc.stop_probe("umic_gemm_gate_silu_mul")
    clk = clocks.stop()
    launches = sum(v for k, v in kc.stats.items() if k.startswith("umic_")) - before
    ms_step = ms_total / args.steps
    value = TOTAL_EPISODES * TOKENS / (ms_step / 1e3)

    # ---- e2e through the public API: H2D ids, prefill, D2H next tokens per step
    nxt_host = torch.empty(episodes, dtype=torch.long).pin_memory()

    def e2e_step():
        ids.copy_(ids_host, non_blocking=True)
        n = step()
        nxt_host.copy_(n, non_blocking=True)

    progress("end-to-end steps")
    e2e_ms = _timed(ranks, e2e_step, args.steps) / args.steps
    e2e_value = TOTAL_EPISODES * TOKENS / (e2e_ms / 1e3)

    # ---- cfg4 decode: 64 greedy steps, CUDA-graph replay (third pass)
    decode = {}
    if n_decode > 0:
        def decode_run():
            cache.crop(0)
            t = prefill(vlm, ids, cache)
            torch.cuda.synchronize()
            s = torch.cuda.Event(enable_timing=True)
            e = torch.cuda.Event(enable_timing=True)
            s.record()
            with torch.no_grad():
                for _ in range(n_decode):
                    out = vlm(input_ids=t[:, None], past_key_values=cache, use_cache=True,
                              logits_to_keep=1)
                    t = out.logits[:, -1].argmax(-1)
            e.record()
            torch.cuda.synchronize()
            model._umic_decode_runner.finish()
            return s.elapsed_time(e)

        # pass 1: eager warm-up steps + capture of the other lengths; pass 2 captures the
        # warm-up lengths; pass 3 replays every step
        progress("decode: capture passes")
        decode_run()
        decode_run()
        progress("decode: replay pass")
        ranks.barrier()
        dms = ranks.max(decode_run())
        decode = {"steps": n_decode, "ms_per_step": dms / n_decode,
                  "tokens_per_s": TOTAL_EPISODES * n_decode / (dms / 1e3),
                  "graphs": len(model._umic_decode_runner.graphs)}
    model._umic_decode_runner.release()

    peaks = _peaks()
    flops = 2.0 * 2 * episodes * TOKENS * INTER * HIDDEN  # gate + up per launch
    avg_ms = statistics.mean(dur) if dur else float("nan")
    achieved = flops / (avg_ms / 1e3) / 1e12 if dur else None
    roofline = {"bound": "tensor", "kernel": "umic_gemm_gate_silu_mul",
                "achieved": achieved, "peak": peaks["bf16_tflops_sustained"], "unit": "TFLOP/s",
                "frac": achieved / peaks["bf16_tflops_sustained"] if achieved else None,
                "peak_source": f"{peaks['source']} (sustained: timed inside the step)",
                "flops_per_launch": flops, "launches": len(dur), "avg_ms": avg_ms,
                "traffic": args.traffic if args.traffic is not None else
                DUAL_GEMM_TRAFFIC_M24800 * episodes * TOKENS / 24800,
                "traffic_note": "ncu dram read+write bytes per launch at M=24800, scaled by "
                                "rows when a rank has fewer episodes"}

    # ---- cfg5 flow, sharded over the ranks
    del cache
    torch.cuda.empty_cache()
    progress("flow")
    flow = _flow_dp(ranks, dev, rank, world) if not args.skip_flow else {}
    progress("report")

    cpu_base = None
    if rank == 0 and world == 1 and not args.skip_cpu:
        cpu_base = _cpu_baselines()

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (random-init weights, uniform token ids)",
            "config": _config(world, episodes),
            "e2e": {"value": e2e_value, "unit": UNIT,
                    "h2d_bytes_per_step": ids_host.numel() * 8,
                    "d2h_bytes_per_step": nxt_host.numel() * 8},
            "roofline": roofline, "cpu_baseline": cpu_base, "clocks": clk,
            "gpu_launches": launches, "decode": decode, "flow": flow, "eager_gpu": eager,
            "parity": parity, "apply_report": report,
        }
        if eager and eager.get("ms_per_step"):
            line["speedup_vs_eager_gpu"] = eager["ms_per_step"] / ms_step
        if world == 1 and not args.skip_extras:
            extras = _extras()
            line["flow"] = {**extras.pop("flow", {}), **flow}
            line.update(extras)
        print(json.dumps(line), flush=True)
    progress.close()
    ranks.close()


def _cpu_baselines() -> dict:
    """The reference's eager CPU path on the host cores: the full cfg4 prefill (one
    3100-token episode, warm-up + median of 3), plus cfg1 and cfg2 as separate entries."""
    from oracle.cpu_baseline import time_cfg1_block, time_cfg2_kernels, time_lm_prefill

    r = time_lm_prefill(tokens=TOKENS, layers=LAYERS, warmup=1, repeats=3)
    return {"value": r["tokens_per_s"], "unit": UNIT, "cores": r["torch_threads"],
            "kind": "port", "sample": r["sample"], "cpu": r["cpu"],
            "physical_cores": r["physical_cores"], "logical_cores": r["logical_cores"],
            "configs": {"cfg1": time_cfg1_block(), "cfg2": time_cfg2_kernels()}}


def _extras() -> dict:
    """cfg1/cfg2 kernels, cfg3 (ViT) and cfg5 (flow expert) against eager, from
    `python -m umic_b200.extras` in a subprocess so its apply() patches stay out of
    this process."""
    try:
        res = subprocess.run([sys.executable, "-m", "umic_b200.extras"],
                             cwd=str(ROOT / "umic-alpamayo_b200"), capture_output=True,
                             text=True, timeout=1200)
        lines = [ln for ln in res.stdout.splitlines() if ln.startswith("{")]
        if res.returncode == 0 and lines:
            return json.loads(lines[-1])
        return {"extras_error": (res.stderr.strip().splitlines() or ["no output"])[-1][:300]}
    except Exception as exc:  # noqa: BLE001 - a failed side measurement must not lose the line
        return {"extras_error": str(exc)[:300]}


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["umic", "reference"], default="umic")
    ap.add_argument("--decode-steps", type=int, default=64)
    ap.add_argument("--skip-eager", action="store_true")
    ap.add_argument("--skip-cpu", action="store_true")
    ap.add_argument("--skip-flow", action="store_true")
    ap.add_argument("--skip-extras", action="store_true",
                    help="skip the cfg1/cfg2 kernel, cfg3 ViT and eager flow timings")
    ap.add_argument("--traffic", type=float, default=None,
                    help="ncu dram bytes per launch of the dominant kernel, if measured")
    args = ap.parse_args()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_umic(args)


if __name__ == "__main__":
    main()
