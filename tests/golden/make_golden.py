"""Generates the golden fixtures that pin the CPU oracle to the reference.

Run where the reference project's source tree is available, naming its `src`
directory with --ref-src or the UMIC_REF_SRC environment variable; the fixtures
are committed, so the tests never need the reference at run time:

    python tests/golden/make_golden.py --ref-src <reference>/src

What is recorded (small seeded cases, CPU):
  * outputs of the reference's own Triton kernels run by Triton's CPU
    interpreter (TRITON_INTERPRET=1): _rmsnorm_kernel, _add_rmsnorm_kernel,
    _layernorm_kernel, _add_layernorm_kernel, _rope_kernel (text and vision
    layouts), _gate_silu_mul_kernel and _linear_kernel (plain / bias / GELU).
    The interpreter's bf16 tl.dot is unreliable, so the two GEMM kernels are fed
    the same bf16 values carried in fp32 and their fp32 outputs are stored;
    the same kernels again on edge shapes (4096 / 2048 / 1000 / 80 wide rows, one
    row, inputs of large magnitude, 64-wide rotary heads, a partial last k-block);
  * the reference's eager CPU path: gate_silu_mul_eager in bf16;
  * the HF transformers eager functions the reference patches
    (apply_rotary_pos_emb, apply_rotary_pos_emb_vision, Qwen3VLTextRMSNorm);
  * a scripted sequence on the reference's InplaceKVCache (append, crop,
    graph-mode writes) with every visible length and buffer snapshot;
  * the reference's structural-match counts (dry_run) on tiny random
    Qwen3-VL models.
"""

from __future__ import annotations

import argparse
import json
import os
import sys
from pathlib import Path

os.environ["TRITON_INTERPRET"] = "1"

OUT = Path(__file__).resolve().parent


def _gen(seed):
    import torch

    return torch.Generator().manual_seed(seed)


def kernels(fixtures: dict) -> None:
    import torch
    from umic.kernels import fused_ffn, layernorm, linear, rmsnorm, rope

    bf = torch.bfloat16
    g = _gen(100)
    # RMSNorm family: rows x n
    for tag, (rows, n) in {"a": (6, 256), "b": (5, 128), "c": (3, 1280)}.items():
        x = torch.randn(rows, n, generator=g).to(bf)
        r = torch.randn(rows, n, generator=g).to(bf)
        w = (1 + 0.05 * torch.randn(n, generator=g)).to(bf)
        y = rmsnorm.rmsnorm_triton(x, w, 1e-6)
        yn, ys = rmsnorm.add_rmsnorm_triton(x, r, w, 1e-6)
        fixtures[f"rmsnorm_{tag}"] = dict(x=x, r=r, w=w, eps=1e-6, y=y, normed=yn, summed=ys)
    for tag, (rows, n) in {"a": (4, 1280), "b": (3, 1152)}.items():
        x = torch.randn(rows, n, generator=g).to(bf)
        r = torch.randn(rows, n, generator=g).to(bf)
        w = torch.randn(n, generator=g).to(bf)
        b = torch.randn(n, generator=g).to(bf)
        y = layernorm.layernorm_triton(x, w, b, 1e-6)
        yn, ys = layernorm.add_layernorm_triton(x, r, w, b, 1e-6)
        fixtures[f"layernorm_{tag}"] = dict(x=x, r=r, w=w, b=b, eps=1e-6, y=y, normed=yn,
                                            summed=ys)
    # RoPE, vision layout [S, H, D] with fp32 cos/sin
    s, h, d = 7, 3, 80
    q = torch.randn(s, h, d, generator=g).to(bf)
    k = torch.randn(s, 2, d, generator=g).to(bf)
    f = torch.randn(s, d // 2, generator=g)
    cos, sin = torch.cat((f, f), -1).cos(), torch.cat((f, f), -1).sin()
    qo, ko = rope.apply_rotary_vision_triton(q, k, cos, sin)
    fixtures["rope_vision"] = dict(q=q, k=k, cos=cos, sin=sin, q_out=qo, k_out=ko)
    # RoPE, text layout [H, S, D] walked as (s_dim=1, h_dim=0), bf16 cos/sin
    qt = torch.randn(4, 9, 128, generator=g).to(bf)
    pos = torch.arange(9).float()
    inv = 1.0 / (1e6 ** (torch.arange(0, 128, 2).float() / 128))
    fr = pos[:, None] * inv[None]
    emb = torch.cat((fr, fr), -1)
    ct, st = emb.cos().to(bf), emb.sin().to(bf)
    qto = rope._apply_one(qt, ct, st, 1, 0)
    fixtures["rope_text"] = dict(q=qt, cos=ct, sin=st, q_out=qto)
    # GEMMs: bf16 values carried in fp32 through the interpreter
    x = torch.randn(70, 64, generator=g).to(bf)
    wg = (0.1 * torch.randn(64, 96, generator=g)).to(bf)
    wu = (0.1 * torch.randn(64, 96, generator=g)).to(bf)
    h32 = fused_ffn.gate_silu_mul_triton(x.float(), wg.float(), wu.float(), block_m=32,
                                         block_n=32, block_k=32)
    h_eager = fused_ffn.gate_silu_mul_eager(x, wg, wu)
    fixtures["gate_silu_mul"] = dict(x=x, w_gate=wg, w_up=wu, h_fp32=h32, h_eager_bf16=h_eager)
    w = (0.1 * torch.randn(48, 64, generator=g)).to(bf)
    b = torch.randn(48, generator=g).to(bf)
    fixtures["linear"] = dict(
        x=x, w=w, b=b,
        y_fp32=linear.linear_triton(x.float(), w.float()),
        y_bias_fp32=linear.linear_triton(x.float(), w.float(), b.float()),
        y_gelu_fp32=linear.linear_triton(x.float(), w.float(), b.float(), act="gelu"))


def edge_cases(fixtures: dict) -> None:
    """More shapes through the same reference kernels, on their own seed (the cases above
    stay as they were): the cfg4 and cfg5 row widths, a width that is not a power of two
    (masked tail of the kernel's block), one-row inputs, a larger eps, inputs of large
    magnitude, a 64-wide rotary head, and GEMMs whose K ends in a partial block."""
    import torch
    from umic.kernels import fused_ffn, layernorm, linear, rmsnorm, rope

    bf = torch.bfloat16
    g = _gen(400)
    for tag, (rows, n, eps, scale) in {"w4096": (2, 4096, 1e-6, 1.0),
                                       "w2048": (3, 2048, 1e-6, 1.0),
                                       "w1000": (3, 1000, 1e-6, 1.0),
                                       "row1": (1, 128, 1e-5, 1.0),
                                       "big": (2, 256, 1e-6, 300.0)}.items():
        x = (scale * torch.randn(rows, n, generator=g)).to(bf)
        r = (scale * torch.randn(rows, n, generator=g)).to(bf)
        w = (1 + 0.05 * torch.randn(n, generator=g)).to(bf)
        y = rmsnorm.rmsnorm_triton(x, w, eps)
        yn, ys = rmsnorm.add_rmsnorm_triton(x, r, w, eps)
        fixtures[f"rmsnorm_{tag}"] = dict(x=x, r=r, w=w, eps=eps, y=y, normed=yn, summed=ys)
    for tag, (rows, n, eps) in {"w1000": (2, 1000, 1e-6), "w80": (3, 80, 1e-5),
                                "row1": (1, 1280, 1e-6)}.items():
        x = torch.randn(rows, n, generator=g).to(bf)
        r = torch.randn(rows, n, generator=g).to(bf)
        w = torch.randn(n, generator=g).to(bf)
        b = torch.randn(n, generator=g).to(bf)
        y = layernorm.layernorm_triton(x, w, b, eps)
        yn, ys = layernorm.add_layernorm_triton(x, r, w, b, eps)
        fixtures[f"layernorm_{tag}"] = dict(x=x, r=r, w=w, b=b, eps=eps, y=y, normed=yn,
                                            summed=ys)
    # text layout, 64-wide heads, 2 heads x 5 positions, theta 1e4
    qt = torch.randn(2, 5, 64, generator=g).to(bf)
    pos = torch.arange(5).float() + 17
    inv = 1.0 / (1e4 ** (torch.arange(0, 64, 2).float() / 64))
    fr = pos[:, None] * inv[None]
    emb = torch.cat((fr, fr), -1)
    ct, st = emb.cos().to(bf), emb.sin().to(bf)
    fixtures["rope_text_d64"] = dict(q=qt, cos=ct, sin=st, q_out=rope._apply_one(qt, ct, st, 1, 0))
    # GEMMs with K = 72 (a partial last k-block) and M, N not multiples of the blocks
    x = torch.randn(33, 72, generator=g).to(bf)
    wg = (0.1 * torch.randn(72, 40, generator=g)).to(bf)
    wu = (0.1 * torch.randn(72, 40, generator=g)).to(bf)
    h32 = fused_ffn.gate_silu_mul_triton(x.float(), wg.float(), wu.float(), block_m=32,
                                         block_n=32, block_k=32)
    fixtures["gate_silu_mul_ktail"] = dict(x=x, w_gate=wg, w_up=wu, h_fp32=h32)
    w = (0.1 * torch.randn(40, 72, generator=g)).to(bf)
    b = torch.randn(40, generator=g).to(bf)
    fixtures["linear_ktail"] = dict(
        x=x, w=w, b=b,
        y_bias_fp32=linear.linear_triton(x.float(), w.float(), b.float()),
        y_gelu_fp32=linear.linear_triton(x.float(), w.float(), b.float(), act="gelu"))


def hf_eager(fixtures: dict) -> None:
    import torch
    import transformers.models.qwen3_vl.modeling_qwen3_vl as m

    bf = torch.bfloat16
    g = _gen(200)
    q = torch.randn(1, 4, 9, 128, generator=g).to(bf)
    k = torch.randn(1, 2, 9, 128, generator=g).to(bf)
    pos = torch.arange(9).float()
    inv = 1.0 / (1e6 ** (torch.arange(0, 128, 2).float() / 128))
    fr = pos[:, None] * inv[None]
    emb = torch.cat((fr, fr), -1)[None]
    cos, sin = emb.cos().to(bf), emb.sin().to(bf)
    qo, ko = m.apply_rotary_pos_emb(q, k, cos, sin)
    fixtures["hf_text_rope"] = dict(q=q, k=k, cos=cos, sin=sin, q_out=qo, k_out=ko)
    qv = torch.randn(7, 3, 80, generator=g).to(bf)
    kv = torch.randn(7, 3, 80, generator=g).to(bf)
    f = torch.randn(7, 40, generator=g)
    cv, sv = torch.cat((f, f), -1).cos(), torch.cat((f, f), -1).sin()
    qvo, kvo = m.apply_rotary_pos_emb_vision(qv, kv, cv, sv)
    fixtures["hf_vision_rope"] = dict(q=qv, k=kv, cos=cv, sin=sv, q_out=qvo, k_out=kvo)
    norm = m.Qwen3VLTextRMSNorm(256, eps=1e-6)
    with torch.no_grad():
        norm.weight.copy_(1 + 0.05 * torch.randn(256, generator=g))
    norm = norm.to(bf)
    x = torch.randn(5, 256, generator=g).to(bf)
    with torch.no_grad():
        y = norm(x)
    fixtures["hf_rmsnorm"] = dict(x=x, w=norm.weight.detach().clone(), eps=1e-6, y=y)


def kv_cache_sequence(fixtures: dict) -> None:
    import torch
    from transformers.cache_utils import DynamicCache
    from umic.cache import InplaceKVCache

    g = _gen(300)
    b, h, base, d = 2, 3, 5, 8
    dyn = DynamicCache()
    k0 = torch.randn(b, h, base, d, generator=g)
    v0 = torch.randn(b, h, base, d, generator=g)
    dyn.update(k0, v0, 0)
    cache = InplaceKVCache.from_dynamic(dyn, extra_tokens=4, margin=2)
    steps = []
    for n in (2, 1):
        kn = torch.randn(b, h, n, d, generator=g)
        vn = torch.randn(b, h, n, d, generator=g)
        kk, vv = cache.layers[0].update(kn, vn)
        steps.append(dict(op="update", n=n, k_new=kn, v_new=vn, len=cache.get_seq_length(),
                          keys=kk.clone(), values=vv.clone()))
    cache.crop(-2)
    steps.append(dict(op="crop", arg=-2, len=cache.get_seq_length()))
    cache.crop(6)
    steps.append(dict(op="crop", arg=6, len=cache.get_seq_length()))
    kn = torch.randn(b, h, 3, d, generator=g)
    vn = torch.randn(b, h, 3, d, generator=g)
    kk, vv = cache.layers[0].update(kn, vn)
    steps.append(dict(op="update", n=3, k_new=kn, v_new=vn, len=cache.get_seq_length(),
                      keys=kk.clone(), values=vv.clone()))
    overflow = None
    try:
        cache.layers[0].update(torch.zeros(b, h, 5, d), torch.zeros(b, h, 5, d))
    except RuntimeError as e:  # capacity 11, pos 9
        overflow = str(e)
    steps.append(dict(op="overflow", message=overflow))
    fixtures["kv_cache"] = dict(k0=k0, v0=v0, extra=4, margin=2, steps=steps,
                                capacity=cache.layers[0]._k_buf.shape[2])


def matcher_counts() -> dict:
    import torch
    from transformers import Qwen3VLConfig
    from transformers.models.qwen3_vl.modeling_qwen3_vl import Qwen3VLForConditionalGeneration
    from umic import integrate

    sys.path.insert(0, str(OUT.parent.parent / "umic-alpamayo_b200"))
    from umic_b200.workloads import tiny_qwen3vl_configs

    counts = {}
    for name, (tc, vc) in tiny_qwen3vl_configs().items():
        torch.manual_seed(0)
        model = Qwen3VLForConditionalGeneration(Qwen3VLConfig(text_config=tc, vision_config=vc))
        lm = model.model.language_model
        vis = model.model.visual
        counts[name] = {
            "fuse_mlps": integrate.fuse_mlps(lm, dry_run=True),
            "fuse_linears": integrate.fuse_linears(lm, dry_run=True),
            "fuse_rmsnorms": integrate.fuse_rmsnorms(lm, dry_run=True),
            "fuse_add_rmsnorm": integrate.fuse_add_rmsnorm(lm, dry_run=True),
            "fuse_layernorms": integrate.fuse_layernorms(vis, dry_run=True),
            "fuse_patch_embed_linear": integrate.fuse_patch_embed_linear(vis, dry_run=True),
            "fuse_vision_attention_varlen": integrate.fuse_vision_attention_varlen(vis,
                                                                                   dry_run=True),
            "fuse_vision_encoder_pipeline": integrate.fuse_vision_encoder_pipeline(vis,
                                                                                   dry_run=True),
            "fuse_gelu_mlps": integrate.fuse_gelu_mlps(vis, dry_run=True),
            "fuse_mlps_whole_model": integrate.fuse_mlps(model, dry_run=True),
            "fuse_rmsnorms_whole_model": integrate.fuse_rmsnorms(model, dry_run=True),
        }
    return counts


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref-src", default=os.environ.get("UMIC_REF_SRC"),
                    help="the reference project's src directory (or set UMIC_REF_SRC)")
    args = ap.parse_args()
    if not args.ref_src:
        ap.error("name the reference's src directory with --ref-src or UMIC_REF_SRC")
    sys.path.insert(0, args.ref_src)
    import torch

    fixtures: dict = {}
    kernels(fixtures)
    edge_cases(fixtures)
    hf_eager(fixtures)
    kv_cache_sequence(fixtures)
    torch.save(fixtures, OUT / "reference_vectors.pt")
    (OUT / "matcher_counts.json").write_text(json.dumps(matcher_counts(), indent=1) + "\n")
    print("wrote", OUT / "reference_vectors.pt", OUT / "matcher_counts.json")


if __name__ == "__main__":
    main()
