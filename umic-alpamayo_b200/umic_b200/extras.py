"""Timings of the two secondary configurations, in a process of their own.

    python -m umic_b200.extras            # prints one JSON object

* vision (cfg3): the 27-block ViT over 16 images of 448 x 448 (16 384 patches),
  unpatched transformers eager vs after `apply()` (fused pipeline: patch-embed GEMM,
  add+LayerNorm, in-place vision RoPE, packed varlen attention, fc1 + tanh-GELU GEMM).
* flow (cfg5): the 18-layer action expert, 32 episodes x 64 action tokens over a
  3100-token prefix KV, 10 Euler steps; unpatched eager vs after `apply()`, with the
  Euler step run eagerly and as a replayed CUDA graph.

Weights are random (seeded), inputs synthetic; each timing is the median of three
runs after warm-up, with CUDA events on the current stream. bench.py runs this in a
subprocess so the global patches `apply()` installs (RoPE functions, attention
registrations) cannot leak into the other measurement.
"""

from __future__ import annotations

import json
import statistics

import torch

from . import integrate
from .optimize import UmicConfig, apply
from .workloads import (CFG5_EXPERT, FLOW_STEPS, AlpamayoStandIn, build_text_model,
                        build_vision_model, flow_sample, vit_inputs)


def _timed(fn, runs: int = 3, warmup: int = 2) -> float:
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    out = []
    for _ in range(runs):
        s = torch.cuda.Event(enable_timing=True)
        e = torch.cuda.Event(enable_timing=True)
        s.record()
        fn()
        e.record()
        torch.cuda.synchronize()
        out.append(s.elapsed_time(e))
    return statistics.median(out)


def _rel(a: torch.Tensor, b: torch.Tensor) -> float:
    a, b = a.float(), b.float()
    return float((a - b).norm() / b.norm().clamp_min(1e-30))


def measure_vision(dev: torch.device, images: int = 16) -> dict:
    vis = build_vision_model(device=dev)
    pix, grid = vit_inputs(images=images, device=dev)

    def run():
        with torch.no_grad():
            return vis(pix, grid_thw=grid)

    eager_ms = _timed(run)
    ref = run().last_hidden_state
    holder = torch.nn.Module()
    holder.vlm = torch.nn.Module()
    holder.vlm.visual = vis
    report = apply(holder, UmicConfig(decode_graph=False, decode_cache=False, decode_gemv=False))
    try:
        ours_ms = _timed(run)
        got = run().last_hidden_state
    finally:
        integrate.unfuse_mlps(holder)
        integrate.unfuse_rope()
    return {"images": images, "patches": int(pix.shape[0]), "eager_ms": eager_ms,
            "ms": ours_ms, "speedup": eager_ms / ours_ms,
            "rel_err_vs_eager": _rel(got, ref),
            "fused": {k: v for k, v in report.items() if k.startswith("ve_")}}


def _prefix_cache(layers: int, episodes: int, heads: int, tokens: int, dim: int, dev,
                  seed: int = 30):
    from transformers.cache_utils import DynamicCache

    g = torch.Generator(device=dev).manual_seed(seed)
    c = DynamicCache()
    for i in range(layers):
        k = torch.randn(episodes, heads, tokens, dim, generator=g, device=dev).bfloat16()
        v = torch.randn(episodes, heads, tokens, dim, generator=g, device=dev).bfloat16()
        c.update(k, v, i)
    return c


def measure_flow(dev: torch.device, episodes: int = 32, tokens: int = 64,
                 prefix: int = 3100) -> dict:
    cfg = CFG5_EXPERT
    expert = build_text_model(cfg, device=dev, seed=5)
    heads_kv = cfg["num_key_value_heads"]
    head_dim = cfg["head_dim"]
    g = torch.Generator(device=dev).manual_seed(31)
    x0 = torch.randn(episodes, tokens, cfg["hidden_size"], generator=g, device=dev).bfloat16()
    cache = _prefix_cache(cfg["num_hidden_layers"], episodes, heads_kv, prefix, head_dim, dev)
    eager_ms = _timed(lambda: flow_sample(expert, cache, prefix, x0), warmup=1)
    ref = flow_sample(expert, cache, prefix, x0)
    holder = AlpamayoStandIn(torch.nn.Module(), expert=expert)
    apply(holder, UmicConfig(decode_graph=False, decode_cache=False))
    try:
        ours_ms = _timed(lambda: flow_sample(expert, cache, prefix, x0))
        graph_ms = _timed(lambda: flow_sample(expert, cache, prefix, x0, graph=True))
        got = flow_sample(expert, cache, prefix, x0, graph=True)
    finally:
        integrate.unfuse_mlps(holder)
        integrate.unfuse_rope()
    return {"episodes": episodes, "action_tokens": tokens, "prefix_tokens": prefix,
            "euler_steps": FLOW_STEPS, "eager_ms": eager_ms, "ms": ours_ms,
            "graph_ms": graph_ms, "speedup": eager_ms / min(ours_ms, graph_ms),
            "rel_err_vs_eager": _rel(got, ref)}


def main() -> None:
    dev = torch.device("cuda", torch.cuda.current_device())
    out = {"vision": measure_vision(dev)}
    torch.cuda.empty_cache()
    out["flow"] = measure_flow(dev)
    print(json.dumps(out), flush=True)


if __name__ == "__main__":
    main()
