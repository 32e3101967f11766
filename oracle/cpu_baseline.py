"""The reference's eager CPU path, timed on the host cores (test / baseline infrastructure).

Used only by bench.py's CPU-baseline leg and its `--impl reference` arm. It runs
the unpatched HF Qwen3-VL text decoder layer -- the eager module the reference
patches (transformers qwen3_vl Qwen3VLTextDecoderLayer, which
src/umic/integrate.py:180-209 replaces) -- with the LM config of the benchmark
(hidden 4096, GQA 32/8 x 128, SwiGLU 12288, RoPE theta 1e6) in bf16 with SDPA,
on one 3100-token episode, using every host thread. A full prefill is 36 such
layers, so the bounded sample (one layer) is scaled by the layer count; the
embedding lookup, final norm and one-row lm_head are below 0.1 % of the work
and are not timed.
"""

from __future__ import annotations

import os
import time


def _cpu_info() -> str:
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def time_layer_prefill(tokens: int = 3100, layers_total: int = 36, repeats: int = 3,
                       threads: int | None = None, seed: int = 0) -> dict:
    """Median seconds for one eager decoder layer over `tokens` tokens on the CPU and
    the implied whole-model prefill throughput (tokens/s)."""
    import torch
    from transformers import Qwen3VLTextConfig
    from transformers.models.qwen3_vl.modeling_qwen3_vl import (Qwen3VLTextDecoderLayer,
                                                                Qwen3VLTextRotaryEmbedding)

    threads = threads or os.cpu_count() or 1
    prev_threads = torch.get_num_threads()
    torch.set_num_threads(threads)
    try:
        cfg = Qwen3VLTextConfig(vocab_size=151936, hidden_size=4096, intermediate_size=12288,
                                num_hidden_layers=layers_total, num_attention_heads=32,
                                num_key_value_heads=8, head_dim=128, rms_norm_eps=1e-6,
                                rope_parameters={"rope_type": "default", "rope_theta": 1e6,
                                                 "mrope_section": [24, 20, 20]})
        cfg._attn_implementation = "sdpa"
        torch.manual_seed(seed)
        prev = torch.get_default_dtype()
        torch.set_default_dtype(torch.bfloat16)
        try:
            layer = Qwen3VLTextDecoderLayer(cfg, 0).eval()
            rot = Qwen3VLTextRotaryEmbedding(cfg)
        finally:
            torch.set_default_dtype(prev)
        with torch.no_grad():
            for p in layer.parameters():
                p.normal_(0.0, 0.02) if p.dim() > 1 else p.fill_(1.0)
            x = torch.randn(1, tokens, 4096, dtype=torch.bfloat16)
            pos = torch.arange(tokens)[None]
            pe = rot(x, pos)

            def run():
                return layer(x, position_embeddings=pe, attention_mask=None, position_ids=pos)

            run()  # warm-up (allocator, oneDNN kernels)
            ts = []
            for _ in range(repeats):
                t0 = time.perf_counter()
                run()
                ts.append(time.perf_counter() - t0)
        ts.sort()
        t_layer = ts[len(ts) // 2]
        return {
            "seconds_per_layer": t_layer,
            "tokens_per_s": tokens / (t_layer * layers_total),
            "cores": threads,
            "cpu": _cpu_info(),
            "sample": f"1 of {layers_total} eager HF decoder layers over one {tokens}-token "
                      f"episode (bf16, SDPA, median of {repeats}), scaled x{layers_total}",
        }
    finally:
        torch.set_num_threads(prev_threads)
