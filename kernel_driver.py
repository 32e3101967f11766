"""Runs one kernel of the library a few times on a BASELINE shape (profiling driver).

    python kernel_driver.py <mode> [rows] [--iters N] [--time]

Used to capture a single kernel under ncu. Modes and shapes:
  dual           gate/up dual-accumulator GEMM, x [rows=24800, 4096], W [12288, 4096] x 2
  qo             linear GEMM, x [rows=24800, 4096], W [4096, 4096]
  qo_cublas      the same shape through torch (cuBLAS), for side-by-side counters
  qk_prep        q/k RMSNorm + RoPE + K/V cache write, [rows=8 episodes, 3100, 32/8, 128]
  add_rmsnorm    [3100, 4096]                  (cfg2a)
  add_layernorm  [16384, 1280]                 (cfg2b)
  rmsnorm_axpy   x + dt * rmsnorm(h) in place, [rows=2048, 2048] (cfg5 Euler update)
  rope_text      q [3100, 32, 128], k [3100, 8, 128], bf16 tables   (cfg2c)
  rope_vision    q, k [16384, 16, 80] views of qkv, fp32 tables     (cfg2d)
  gemv           x [rows=8, 4096], W [12288, 4096]
  vit            the cfg3 encoder after apply(), rows = images (16)
  decode         one graph-replayed cfg4 decode step of rows = 8 episodes
  flow           one cfg5 flow sample (10 graph-replayed Euler steps of the 18-layer
                 expert) for rows = 32 episodes over a 3100-token prefix cache
  kv             K/V [8, 8, 3100, 128] appended into [8, 8, 3172, 128]
  attn           flow-step attention: q [rows=32 episodes, 16, 64, 128] over the
                 3164-key prefix of a [32, 8, 3172, 128] cache, lower-right causal mask
                 (mask packing + umic_attention_rows)
  attn_nomask    the same without a mask
  attn_sdpa      the same shape and mask through torch SDPA (what transformers runs)
Inputs are seeded random tensors created on cuda:0 before the launches. Without --time
the first call runs alone and the next --iters calls run inside the NVTX range "drv"
(`ncu --nvtx --nvtx-include "drv/"` captures just those). --time runs
3 warm-up launches and then times --iters launches back to back with CUDA events
(the inputs of the attention modes exceed L2), printing microseconds per launch.
"""


from __future__ import annotations

import argparse
import sys
from pathlib import Path

_ROOT = Path(__file__).resolve().parent
for _p in (_ROOT, _ROOT / "umic-alpamayo_b200"):
    if str(_p) not in sys.path:
        sys.path.insert(0, str(_p))

import torch


def make(mode: str, rows: int | None):
    from umic_b200.kernels import (add_layernorm, add_rmsnorm, apply_rotary_text_inplace,
                                   apply_rotary_vision, gate_silu_mul_nk, kv_append, linear,
                                   linear_gemv)
    from umic_b200.kernels.attention import qk_norm_rope_kv

    dev = torch.device("cuda", 0)
    bf = torch.bfloat16
    torch.manual_seed(0)
    if mode == "dual":
        x = torch.randn(rows or 24800, 4096, device=dev, dtype=bf)
        wg = torch.randn(12288, 4096, device=dev, dtype=bf) * 0.02
        wu = torch.randn_like(wg)
        return lambda: gate_silu_mul_nk(x, wg, wu)
    if mode == "qo":
        x = torch.randn(rows or 24800, 4096, device=dev, dtype=bf)
        w = torch.randn(4096, 4096, device=dev, dtype=bf) * 0.02
        return lambda: linear(x, w)
    if mode == "qo_cublas":  # the same shape on cuBLAS, for side-by-side counters
        x = torch.randn(rows or 24800, 4096, device=dev, dtype=bf)
        w = torch.randn(4096, 4096, device=dev, dtype=bf) * 0.02
        return lambda: torch.nn.functional.linear(x, w)
    if mode == "qk_prep":
        b, s, hq, hk, d = (rows or 8), 3100, 32, 8, 128
        q = torch.randn(b, s, hq * d, device=dev, dtype=bf).view(b, s, hq, d)
        k = torch.randn(b, s, hk * d, device=dev, dtype=bf).view(b, s, hk, d)
        v = torch.randn_like(k)
        qw = torch.ones(d, device=dev, dtype=bf)
        c = torch.randn(b, s, d, device=dev, dtype=bf)
        sn = torch.randn_like(c)
        kb = torch.zeros(b, hk, s + 72, d, device=dev, dtype=bf)
        vb = torch.zeros_like(kb)
        return lambda: qk_norm_rope_kv(q, k, v, qw, qw, 1e-6, 1e-6, c, sn, kb, vb, 0)
    if mode == "add_rmsnorm":
        x = torch.randn(3100, 4096, device=dev, dtype=bf)
        r = torch.randn_like(x)
        w = torch.randn(4096, device=dev, dtype=bf)
        return lambda: add_rmsnorm(x, r, w, 1e-6)
    if mode == "rmsnorm_axpy":  # the flow Euler update at the cfg5 shape (32 x 64 tokens)
        from umic_b200.kernels import rmsnorm_axpy

        h = torch.randn(rows or 2048, 2048, device=dev, dtype=bf)
        x = torch.randn_like(h)
        w = torch.ones(2048, device=dev, dtype=bf)
        return lambda: rmsnorm_axpy(h, w, 1e-6, x, 0.1, out=x)
    if mode == "add_layernorm":
        x = torch.randn(16384, 1280, device=dev, dtype=bf)
        r = torch.randn_like(x)
        w = torch.ones(1280, device=dev, dtype=bf)
        b = torch.zeros_like(w)
        return lambda: add_layernorm(x, r, w, b, 1e-6)
    if mode == "rope_text":
        q = torch.randn(1, 3100, 32, 128, device=dev, dtype=bf).transpose(1, 2)
        k = torch.randn(1, 3100, 8, 128, device=dev, dtype=bf).transpose(1, 2)
        c = torch.randn(1, 3100, 128, device=dev, dtype=bf)
        s = torch.randn_like(c)
        return lambda: apply_rotary_text_inplace(q, k, c, s)
    if mode == "rope_vision":
        qkv = torch.randn(16384, 3, 16, 80, device=dev, dtype=bf)
        q, k, _ = qkv.unbind(1)
        c = torch.randn(16384, 80, device=dev)
        s = torch.randn_like(c)
        return lambda: apply_rotary_vision(q, k, c, s)
    if mode == "gemv":
        x = torch.randn(rows or 8, 4096, device=dev, dtype=bf)
        w = torch.randn(12288, 4096, device=dev, dtype=bf)
        return lambda: linear_gemv(x, w)
    if mode in ("attn", "attn_nomask", "attn_sdpa"):
        from umic_b200.kernels.attention import attention_rows

        b, hq, hk, t, lk, cap, d = (rows or 32), 16, 8, 64, 3164, 3172, 128
        q = torch.randn(b, t, hq, d, device=dev, dtype=bf).transpose(1, 2)
        kb = torch.randn(b, hk, cap, d, device=dev, dtype=bf)
        vb = torch.randn_like(kb)
        mask = torch.ones(t, lk, dtype=torch.bool, device=dev).tril(diagonal=lk - t)
        mask = mask[None, None].expand(b, 1, t, lk).contiguous()
        k, v = kb[:, :, :lk], vb[:, :, :lk]
        if mode == "attn_nomask":
            return lambda: attention_rows(q, k, v, None, d ** -0.5)
        if mode == "attn_sdpa":
            return lambda: torch.nn.functional.scaled_dot_product_attention(
                q, k, v, attn_mask=mask, scale=d ** -0.5, enable_gqa=True)
        return lambda: attention_rows(q, k, v, mask, d ** -0.5)
    if mode == "kv":
        kb = torch.zeros(8, 8, 3172, 128, device=dev, dtype=bf)
        vb = torch.zeros_like(kb)
        kn = torch.randn(8, 3100, 8, 128, device=dev, dtype=bf).transpose(1, 2)
        vn = torch.randn_like(kn)
        return lambda: kv_append(kb, vb, kn, vn, 0)
    if mode == "vit":  # the whole cfg3 encoder (16 images) after apply(): one forward a call
        from umic_b200 import UmicConfig, apply
        from umic_b200.workloads import build_vision_model, vit_inputs

        vis = build_vision_model(device=dev)
        pix, grid = vit_inputs(images=rows or 16, device=dev)
        holder = torch.nn.Module()
        holder.vlm = torch.nn.Module()
        holder.vlm.visual = vis
        apply(holder, UmicConfig(decode_graph=False, decode_cache=False, decode_gemv=False))

        def vit():
            with torch.no_grad():
                vis(pix, grid_thw=grid)
        return vit
    if mode == "decode":  # one cfg4 decode step of `rows` episodes (graph replay) per call
        from umic_b200 import UmicConfig, apply
        from umic_b200.workloads import AlpamayoStandIn, build_vlm, kv_cache_for, prefill_ids

        b = rows or 8
        vlm = build_vlm(device=dev, seed=4)
        ids = prefill_ids(b, 3100, seed=4, device=dev)
        model = AlpamayoStandIn(vlm)
        apply(model, UmicConfig(max_new_tokens=80))
        cache = kv_cache_for(vlm, b, 3100 + 80, dev)
        runner = model._umic_decode_runner
        with torch.no_grad():
            out = vlm(input_ids=ids, past_key_values=cache, use_cache=True, logits_to_keep=1)
        tok = out.logits[:, -1].argmax(-1)[:, None]
        base = cache.get_seq_length()

        def step():
            # the same KV length each call: after the runner's two warm-up steps every call
            # replays one captured graph
            if runner.in_decode:
                cache.set_pos(base)
            with torch.no_grad():
                vlm(input_ids=tok, past_key_values=cache, use_cache=True, logits_to_keep=1)
        return step
    if mode == "flow":  # one cfg5 flow sample (10 Euler steps, graph replay) per call
        from umic_b200 import UmicConfig, apply
        from umic_b200.extras import _prefix_cache
        from umic_b200.workloads import (CFG5_EXPERT, PREFILL_TOKENS, AlpamayoStandIn,
                                         build_text_model, flow_sample)

        e = rows or 32
        expert = build_text_model(CFG5_EXPERT, device=dev, seed=5)
        apply(AlpamayoStandIn(torch.nn.Module(), expert=expert),
              UmicConfig(decode_graph=False, decode_cache=False))
        x0 = torch.randn(e, 64, CFG5_EXPERT["hidden_size"], device=dev, dtype=bf)
        cache = _prefix_cache(CFG5_EXPERT["num_hidden_layers"], e,
                              CFG5_EXPERT["num_key_value_heads"], PREFILL_TOKENS,
                              CFG5_EXPERT["head_dim"], dev)
        return lambda: flow_sample(expert, cache, PREFILL_TOKENS, x0, graph=True)
    raise SystemExit(f"unknown mode {mode}")


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("mode")
    ap.add_argument("rows", nargs="?", type=int, default=None)
    ap.add_argument("--iters", type=int, default=3)
    ap.add_argument("--time", action="store_true")
    a = ap.parse_args()
    fn = make(a.mode, a.rows)
    if a.time:
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(a.iters):
            fn()
        e.record()
        torch.cuda.synchronize()
        print(f"{a.mode}: {s.elapsed_time(e) * 1e3 / a.iters:.1f} us per launch "
              f"({a.iters} back to back)")
        return
    fn()  # first call outside the range: lazy initialisation, graph capture
    torch.cuda.synchronize()
    torch.cuda.nvtx.range_push("drv")  # ncu --nvtx --nvtx-include "drv/" selects these calls
    for _ in range(a.iters):
        fn()
    torch.cuda.synchronize()
    torch.cuda.nvtx.range_pop()
    print("ok", a.mode)


if __name__ == "__main__":
    main()
