"""LM prefill benchmark (BASELINE cfg4) for the B200 fused-inference hot path.

Workload: the 36-layer Qwen3-VL-shaped LM (hidden 4096, GQA 32/8 x 128,
SwiGLU 12288, vocab 151936), random-init weights ~N(0, 0.02), patched with
umic_b200.apply(); 8 independent episodes of 3100 uniform-random token ids,
sharded over the ranks (strong scaling: 8 episodes in total) and run as one
batched prefill per rank. A step = one prefill of this rank's episodes into an
in-place KV cache, ending with the greedy next token. The metric is prefill
tokens/s for the whole job; `e2e` is the same through the public API with
the token ids copied from pinned host memory and the next tokens read back
inside the timed region. The 64 greedy decode steps of cfg4 are measured after
the timed prefill and reported under `decode` (CUDA-graph replay).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl umic|reference]

--impl reference times the reference's eager CPU path on the host cores (the
reference's GPU path is Triton JIT code for Jetson Thor; its CPU path is the
HF eager model it patches) and prints the same JSON line with impl=reference.
"""

from __future__ import annotations

import argparse
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
# DRAM bytes (read + write) of one dual-GEMM launch at the 8-episode shape
# (M = 24800): 2.111 GB read + 0.608 GB written, from `ncu --set full` of the
# CTA-pair kernel with the TMA-store epilogue (profiles/gemm_gate_silu_mul_cfg4_prefill.md).
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


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during the timed region."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
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


def _episodes_for(rank: int, world: int) -> int:
    base, extra = divmod(TOTAL_EPISODES, world)
    return base + (1 if rank < extra else 0)


def run_reference(args) -> None:
    """The reference's eager CPU path on the host cores (rank 0 only)."""
    world, rank, _ = _dist()
    if rank != 0:
        return
    from oracle.cpu_baseline import time_layer_prefill

    res = None
    vals = []
    for _ in range(max(1, args.steps)):
        res = time_layer_prefill(tokens=TOKENS, layers_total=LAYERS, repeats=1)
        vals.append(res["tokens_per_s"])
    v = statistics.median(vals)
    line = {
        "metric": METRIC, "value": v, "unit": UNIT, "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": TOKENS / v * 1e3, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "impl": "reference",
        "config": {"workload": "cfg4 LM prefill, 3100-token episode, eager HF decoder on CPU",
                   "layers": LAYERS, "tokens": TOKENS},
        "cpu_baseline": {"value": v, "unit": UNIT, "cores": res["cores"], "kind": "port",
                         "sample": res["sample"], "cpu": res["cpu"]},
        "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_umic(args) -> None:
    import torch
    import torch.distributed as dist

    world, rank, local = _dist()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                device_id=dev)

    from umic_b200 import UmicConfig, apply, integrate
    from umic_b200.kernels import _common as kc
    from umic_b200.workloads import AlpamayoStandIn, build_vlm, kv_cache_for, prefill, prefill_ids

    episodes = _episodes_for(rank, world)
    n_decode = args.decode_steps
    vlm = build_vlm(device=dev, seed=4)
    all_ids = prefill_ids(TOTAL_EPISODES, TOKENS, seed=4)
    start = sum(_episodes_for(r, world) for r in range(rank))
    ids_host = all_ids[start:start + episodes].contiguous().pin_memory()
    ids = ids_host.to(dev)
    cache = kv_cache_for(vlm, episodes, TOKENS + n_decode + 8, dev)

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def timed(fn, steps):
        barrier()
        torch.cuda.synchronize()
        s = torch.cuda.Event(enable_timing=True)
        e = torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(steps):
            fn()
        e.record()
        torch.cuda.synchronize()
        barrier()
        return max_over_ranks(s.elapsed_time(e))

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

        ref_next = eager_step().clone()
        eager_step()
        n_e = max(2, args.steps // 2)
        ms = timed(eager_step, n_e) / n_e
        eager = {"value": TOTAL_EPISODES * TOKENS / (ms / 1e3), "ms_per_step": ms,
                 "what": "unpatched HF modules + DynamicCache, bf16, SDPA, same weights/inputs"}
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
    clocks = ClockSampler(vis.split(",")[local] if vis else local)
    clocks.start()
    kc.start_probe("umic_gemm_gate_silu_mul")
    torch.cuda.nvtx.range_push("umic_timed")  # lets ncu --nvtx-include select this region
    ms_total = timed(step, args.steps)
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

    e2e_ms = timed(e2e_step, args.steps) / args.steps
    e2e_value = TOTAL_EPISODES * TOKENS / (e2e_ms / 1e3)

    # ---- cfg4 decode: 64 greedy steps, CUDA-graph replay (second pass)
    decode = {}
    if n_decode > 0:
        def decode_run():
            cache.crop(0)
            t = prefill(vlm, ids, cache)
            torch.cuda.synchronize()
            s = torch.cuda.Event(enable_timing=True)
            e = torch.cuda.Event(enable_timing=True)
            s.record()
            toks = [t]
            with torch.no_grad():
                for _ in range(n_decode):
                    out = vlm(input_ids=t[:, None], past_key_values=cache, use_cache=True,
                              logits_to_keep=1)
                    t = out.logits[:, -1].argmax(-1)
                    toks.append(t)
            e.record()
            torch.cuda.synchronize()
            model._umic_decode_runner.finish()
            return s.elapsed_time(e), torch.stack(toks, 1)

        # The first pass runs the runner's eager warm-up steps and captures the graphs of
        # the remaining KV lengths; the second captures the warm-up lengths; the third
        # replays every step.
        decode_run()
        decode_run()
        dms, toks = decode_run()
        dms = max_over_ranks(dms)
        decode = {"steps": n_decode, "ms_per_step": dms / n_decode,
                  "tokens_per_s": TOTAL_EPISODES * n_decode
                  / (dms / 1e3), "graphs": len(model._umic_decode_runner.graphs)}

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

    cpu_base = None
    if rank == 0 and world == 1 and not args.skip_cpu:
        from oracle.cpu_baseline import time_layer_prefill

        r = time_layer_prefill(tokens=TOKENS, layers_total=LAYERS, repeats=2)
        cpu_base = {"value": r["tokens_per_s"], "unit": UNIT, "cores": r["cores"],
                    "kind": "port", "sample": r["sample"], "cpu": r["cpu"]}

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (random-init weights, uniform token ids)",
            "config": {"workload": "cfg4 LM prefill", "model": "36L-4096H-GQA32/8-SwiGLU12288",
                       "global_batch": TOTAL_EPISODES, "seq_len": TOKENS,
                       "episodes_per_rank": episodes, "parallelism": f"episode-dp{world}",
                       "l2": "inputs larger than L2 (15.4 GB of weights streamed per step)"},
            "e2e": {"value": e2e_value, "unit": UNIT,
                    "h2d_bytes_per_step": ids_host.numel() * 8,
                    "d2h_bytes_per_step": nxt_host.numel() * 8},
            "roofline": roofline, "cpu_baseline": cpu_base, "clocks": clk,
            "gpu_launches": launches, "decode": decode, "eager_gpu": eager, "parity": parity,
            "apply_report": report,
        }
        if eager and eager.get("ms_per_step"):
            line["speedup_vs_eager_gpu"] = eager["ms_per_step"] / ms_step
        if world == 1 and not args.skip_extras:
            line.update(_extras())
        print(json.dumps(line), flush=True)
    model._umic_decode_runner.release()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def _extras() -> dict:
    """cfg3 (ViT) and cfg5 (flow expert) timings from `python -m umic_b200.extras`, run
    in a subprocess so their apply() patches stay out of this process."""
    import subprocess

    try:
        res = subprocess.run([sys.executable, "-m", "umic_b200.extras"],
                             cwd=str(ROOT / "umic-alpamayo_b200"), capture_output=True,
                             text=True, timeout=900)
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
    ap.add_argument("--skip-extras", action="store_true",
                    help="skip the cfg3 ViT and cfg5 flow timings (umic_b200.extras)")
    ap.add_argument("--traffic", type=float, default=None,
                    help="ncu dram bytes per launch of the dominant kernel, if measured")
    args = ap.parse_args()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_umic(args)


if __name__ == "__main__":
    main()
