"""The reference's eager CPU path, timed on the host cores (test / baseline infrastructure).

Used only by bench.py's CPU-baseline leg and its `--impl reference` arm. What runs
is the unpatched code the reference patches -- transformers' Qwen3-VL modules and
functions in bf16 with SDPA, the reference's `gate_silu_mul_eager`
(src/umic/kernels/fused_ffn.py:31-43) restated -- on every host thread:

  * cfg4: the full 36-layer text model (embedding, 36 Qwen3VLTextDecoderLayer,
    final RMSNorm) over one 3100-token episode, then the last token's lm_head
    row: a whole prefill per step (src/umic/integrate.py:180-209 patches these
    layers);
  * cfg1: the pre-norm SwiGLU block, add + HF RMSNorm, then silu(n Wg^T) * (n Wu^T)
    and the down projection plus the residual, at [3100, 4096] x 12288;
  * cfg2: the four norm / RoPE calls the reference patches, HF eager (add +
    RMSNorm, add + LayerNorm, apply_rotary_pos_emb, apply_rotary_pos_emb_vision).

Weights are random ~N(0, 0.02): one seeded random block tiled over every matrix
(drawing 8 B values one by one takes minutes on the CPU and the arithmetic does
not depend on the values). Timings: `warmup` untimed runs, then the median (and
all samples) of `repeats` timed runs, wall clock.
"""

from __future__ import annotations

import os
import statistics
import time

LM_CONFIG = dict(vocab_size=151936, hidden_size=4096, intermediate_size=12288,
                 num_hidden_layers=36, num_attention_heads=32, num_key_value_heads=8,
                 head_dim=128, rms_norm_eps=1e-6,
                 rope_parameters={"rope_type": "default", "rope_theta": 1e6,
                                  "mrope_section": [24, 20, 20]})


def cpu_info() -> dict:
    model, phys = "unknown", set()
    try:
        cur = {}
        with open("/proc/cpuinfo") as f:
            for line in f:
                if ":" not in line:
                    if "physical id" in cur and "core id" in cur:
                        phys.add((cur["physical id"], cur["core id"]))
                    cur = {}
                    continue
                k, v = (t.strip() for t in line.split(":", 1))
                cur[k] = v
                if k == "model name":
                    model = v
    except OSError:
        pass
    return {"cpu": model, "logical_cores": os.cpu_count() or 1,
            "physical_cores": len(phys) or None}


def _threads(threads: int | None) -> int:
    return threads or os.cpu_count() or 1


def _fill_random(params, seed: int = 0, std: float = 0.02, block: int = 1 << 24) -> None:
    import torch

    g = torch.Generator().manual_seed(seed)
    src = (torch.randn(block, generator=g) * std).to(torch.bfloat16)
    for p in params:
        flat = p.view(-1)
        if p.dim() == 1:
            flat.fill_(1.0)
            continue
        for off in range(0, flat.numel(), block):
            n = min(block, flat.numel() - off)
            flat[off:off + n].copy_(src[:n])


def _timed(fn, warmup: int, repeats: int) -> list[float]:
    for _ in range(warmup):
        fn()
    out = []
    for _ in range(repeats):
        t0 = time.perf_counter()
        fn()
        out.append(time.perf_counter() - t0)
    return out


class CpuLM:
    """The unpatched transformers text model of the LM config, bf16, on the CPU."""

    def __init__(self, layers: int = 36, seed: int = 0):
        import torch
        from transformers import Qwen3VLTextConfig
        from transformers.models.qwen3_vl.modeling_qwen3_vl import (Qwen3VLTextModel,
                                                                    Qwen3VLTextRotaryEmbedding)

        cfg = Qwen3VLTextConfig(**dict(LM_CONFIG, num_hidden_layers=layers))
        cfg._attn_implementation = "sdpa"
        prev = torch.get_default_dtype()
        torch.set_default_dtype(torch.bfloat16)
        try:
            with torch.device("meta"):
                model = Qwen3VLTextModel(cfg)
        finally:
            torch.set_default_dtype(prev)
        self.model = model.to_empty(device="cpu").eval()
        # the RoPE buffers came from the meta device empty: rebuild them on the CPU
        self.model.rotary_emb = Qwen3VLTextRotaryEmbedding(cfg)
        self.lm_head = torch.empty(cfg.vocab_size, cfg.hidden_size, dtype=torch.bfloat16)
        with torch.no_grad():
            _fill_random([p for p in self.model.parameters()] + [self.lm_head], seed)
        self.layers = layers

    def prefill(self, ids):
        """Hidden states of every token, then the last token's logits (greedy next)."""
        import torch

        with torch.no_grad():
            h = self.model(input_ids=ids, use_cache=False).last_hidden_state
            logits = torch.nn.functional.linear(h[:, -1], self.lm_head)
        return logits.argmax(-1)


def time_lm_prefill(tokens: int = 3100, layers: int = 36, warmup: int = 1, repeats: int = 3,
                    threads: int | None = None, seed: int = 0, model: CpuLM | None = None) -> dict:
    """Wall-clock seconds of full eager prefills of one `tokens`-token episode."""
    import torch

    th = _threads(threads)
    prev = torch.get_num_threads()
    torch.set_num_threads(th)
    try:
        lm = model or CpuLM(layers, seed)
        g = torch.Generator().manual_seed(seed + 1)
        ids = torch.randint(0, LM_CONFIG["vocab_size"], (1, tokens), generator=g)
        ts = _timed(lambda: lm.prefill(ids), warmup, repeats)
    finally:
        torch.set_num_threads(prev)
    med = statistics.median(ts)
    return {"seconds": ts, "seconds_median": med, "tokens_per_s": tokens / med,
            "torch_threads": th, **cpu_info(),
            "sample": f"full {lm.layers}-layer eager HF text model (bf16, SDPA) prefill of one "
                      f"{tokens}-token episode + last-token lm_head; {warmup} warm-up, median "
                      f"of {repeats}"}


def time_cfg1_block(rows: int = 3100, hidden: int = 4096, inter: int = 12288, warmup: int = 1,
                    repeats: int = 3, threads: int | None = None, seed: int = 0) -> dict:
    """cfg1 on the CPU: n = RMSNorm(x + residual) (HF module), out = (x + residual) +
    down(silu(n Wg^T) * (n Wu^T)), the reference's eager formula, bf16."""
    import torch
    from transformers.models.qwen3_vl.modeling_qwen3_vl import Qwen3VLTextRMSNorm

    th = _threads(threads)
    prev = torch.get_num_threads()
    torch.set_num_threads(th)
    try:
        g = torch.Generator().manual_seed(seed)
        x = torch.randn(rows, hidden, generator=g).bfloat16()
        r = torch.randn(rows, hidden, generator=g).bfloat16()
        norm = Qwen3VLTextRMSNorm(hidden, eps=1e-6).to(torch.bfloat16)
        with torch.no_grad():
            norm.weight.copy_(1 + 0.05 * torch.randn(hidden, generator=g))
        wg, wu = (torch.empty(inter, hidden, dtype=torch.bfloat16) for _ in range(2))
        wd = torch.empty(hidden, inter, dtype=torch.bfloat16)
        _fill_random([wg, wu, wd], seed)
        F = torch.nn.functional

        def block():
            with torch.no_grad():
                s = x + r
                n = norm(s)
                h = F.silu(n @ wg.t()) * (n @ wu.t())  # gate_silu_mul_eager (fused_ffn.py:31-43)
                return s + F.linear(h, wd)

        ts = _timed(block, warmup, repeats)
    finally:
        torch.set_num_threads(prev)
    med = statistics.median(ts)
    flops = 2.0 * rows * hidden * inter * 3
    return {"ms": med * 1e3, "seconds": ts, "tflops": flops / med / 1e12, "torch_threads": th,
            "sample": f"cfg1 SwiGLU block [{rows},{hidden}]x{inter} eager bf16; {warmup} "
                      f"warm-up, median of {repeats}"}


def time_cfg2_kernels(warmup: int = 2, repeats: int = 5, threads: int | None = None,
                      seed: int = 1) -> dict:
    """cfg2 a-d through transformers' eager functions on the CPU (bf16 inputs): the four
    calls the reference replaces with its norm / RoPE kernels."""
    import torch
    from transformers import Qwen3VLTextConfig
    from transformers.models.qwen3_vl import modeling_qwen3_vl as hf

    th = _threads(threads)
    prev = torch.get_num_threads()
    torch.set_num_threads(th)
    out = {}
    try:
        g = torch.Generator().manual_seed(seed)

        def rn(*s):
            return torch.randn(*s, generator=g).bfloat16()

        def record(name, fn, nbytes):
            with torch.no_grad():
                ts = _timed(fn, warmup, repeats)
            med = statistics.median(ts)
            out[name] = {"us": med * 1e6, "gbs": nbytes / med / 1e9}

        # (a) add + RMSNorm [3100, 4096]
        x, r = rn(3100, 4096), rn(3100, 4096)
        rms = hf.Qwen3VLTextRMSNorm(4096, eps=1e-6).to(torch.bfloat16)

        def add_rms():
            s = x + r
            return rms(s), s

        record("cfg2a_add_rmsnorm", add_rms, 4 * 3100 * 4096 * 2)
        # (b) add + LayerNorm [16384, 1280]
        xv, rv = rn(16384, 1280), rn(16384, 1280)
        ln = torch.nn.LayerNorm(1280, eps=1e-6).to(torch.bfloat16)

        def add_ln():
            s = xv + rv
            return ln(s), s

        record("cfg2b_add_layernorm", add_ln, 4 * 16384 * 1280 * 2)
        # (c) text RoPE, theta 1e6, head_dim 128, positions 0..3099
        cfg = Qwen3VLTextConfig(**LM_CONFIG)
        rot = hf.Qwen3VLTextRotaryEmbedding(cfg)
        q, k = rn(1, 32, 3100, 128), rn(1, 8, 3100, 128)
        cos, sin = rot(q, torch.arange(3100)[None].expand(3, 1, 3100))
        record("cfg2c_text_rope", lambda: hf.apply_rotary_pos_emb(q, k, cos, sin),
               2 * (32 + 8) * 3100 * 128 * 2 + 2 * 3100 * 128 * 2)
        # (d) vision RoPE, head_dim 80, 16 images x 32 x 32 patches
        qv, kv = rn(16384, 16, 80), rn(16384, 16, 80)
        f = torch.randn(16384, 40, generator=g)
        emb = torch.cat((f, f), -1)
        vc, vs = emb.cos(), emb.sin()
        record("cfg2d_vision_rope", lambda: hf.apply_rotary_pos_emb_vision(qv, kv, vc, vs),
               2 * 2 * 16384 * 16 * 80 * 2 + 2 * 16384 * 80 * 4)
    finally:
        torch.set_num_threads(prev)
    out["torch_threads"] = th
    out["sample"] = f"HF eager functions, bf16; {warmup} warm-up, median of {repeats}"
    return out
