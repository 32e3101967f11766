"""fp32 restatements of the reference's hot-path arithmetic (test infrastructure).

Every function takes bf16 (or fp32) CPU tensors, computes in float32 (float64
where stated) and returns float32, i.e. the "fp32-accumulated reference" the
parity bar is quoted against. Each cites the reference lines it follows
(paths relative to soonhong99/umic-alpamayo).
"""

from __future__ import annotations

import math

import torch


def _f(t: torch.Tensor) -> torch.Tensor:
    return t.detach().to("cpu", torch.float32)


def rel_err(a: torch.Tensor, b: torch.Tensor) -> float:
    """||a - b||_2 / ||b||_2 in fp64 (scripts/check_env.py:124-125)."""
    a64 = a.detach().cpu().double()
    b64 = b.detach().cpu().double()
    den = b64.norm().item()
    return (a64 - b64).norm().item() / (den if den > 0 else 1.0)


def max_rel_err(a: torch.Tensor, b: torch.Tensor) -> float:
    """Per-tensor max relative error: max|a - b| / max|b| (the north-star parity metric)."""
    a64 = a.detach().cpu().double()
    b64 = b.detach().cpu().double()
    den = b64.abs().max().item()
    return (a64 - b64).abs().max().item() / (den if den > 0 else 1.0)


def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    """y = x * rsqrt(mean(x^2) + eps) * w in fp32 (src/umic/kernels/rmsnorm.py:44-51)."""
    xf = _f(x)
    var = (xf * xf).mean(-1, keepdim=True)
    return xf * torch.rsqrt(var + eps) * _f(w)


def rmsnorm_axpy(x, w, eps, base, alpha):
    """base + alpha * rmsnorm(x) in fp32: the flow sampler's Euler step x + dt * v with
    v the expert's final RMSNorm output (P9 ode_step, docs/260610_01_umic_design_ko.md:72,
    composed with rmsnorm.py:44-51)."""
    return _f(base) + float(alpha) * rmsnorm(x, w, eps)


def add_rmsnorm(x, r, w, eps):
    """(normed, summed): s = x + r in fp32, normed = rmsnorm(s) (rmsnorm.py:91-101)."""
    s = _f(x) + _f(r)
    var = (s * s).mean(-1, keepdim=True)
    return s * torch.rsqrt(var + eps) * _f(w), s


def layernorm(x, w, b, eps):
    """(x - mean) * rsqrt(var + eps) * w + b, biased variance (layernorm.py:43-52)."""
    xf = _f(x)
    mean = xf.mean(-1, keepdim=True)
    d = xf - mean
    var = (d * d).mean(-1, keepdim=True)
    return d * torch.rsqrt(var + eps) * _f(w) + _f(b)


def add_layernorm(x, r, w, b, eps):
    """(normed, summed) with the sum in fp32 (layernorm.py:87-100)."""
    s = _f(x) + _f(r)
    mean = s.mean(-1, keepdim=True)
    d = s - mean
    var = (d * d).mean(-1, keepdim=True)
    return d * torch.rsqrt(var + eps) * _f(w) + _f(b), s


def rope_rotate_half(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """out[d] = x[d]*cos[d] + sign(d)*x[partner(d)]*sin[d], partner = d +/- D/2,
    sign = -1 on the first half (src/umic/kernels/rope.py:45-60; equivalent to HF's
    q*cos + rotate_half(q)*sin). cos/sin broadcast against x's leading dims."""
    xf = _f(x)
    half = xf.shape[-1] // 2
    rot = torch.cat((-xf[..., half:], xf[..., :half]), dim=-1)
    return xf * _f(cos) + rot * _f(sin)


def text_rope_cos_sin(positions: torch.Tensor, head_dim: int, theta: float):
    """1-D text RoPE tables as HF's Qwen3-VL text rotary embedding builds them for
    equal t/h/w position streams: inv_freq = theta^(-2i/D), emb = cat(f, f), fp32
    (transformers qwen3_vl Qwen3VLTextRotaryEmbedding.forward). Returns fp32 [S, D]."""
    inv_freq = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.int64).float()
                                / head_dim))
    freqs = positions.float()[:, None] * inv_freq[None, :]
    emb = torch.cat((freqs, freqs), dim=-1)
    return emb.cos(), emb.sin()


def silu(v: torch.Tensor) -> torch.Tensor:
    return v * torch.sigmoid(v)


def gate_silu_mul(x, w_gate_kn, w_up_kn):
    """silu(x @ Wg) * (x @ Wu) with fp32 accumulation and fp32 epilogue; weights [K, N]
    (src/umic/kernels/fused_ffn.py:31-43 formula, :86-87 fp32 epilogue)."""
    xf = _f(x)
    return silu(xf @ _f(w_gate_kn)) * (xf @ _f(w_up_kn))


def linear(x, w_nk, bias=None, act=None, residual=None):
    """x @ W^T (+bias) (+erf-GELU) in fp32 (src/umic/kernels/linear.py:65-86); act
    "gelu_tanh" is HF's gelu_pytorch_tanh; residual is added last."""
    y = _f(x) @ _f(w_nk).t()
    if bias is not None:
        y = y + _f(bias)
    if act in ("gelu", "gelu_erf"):
        y = 0.5 * y * (1.0 + torch.erf(y / math.sqrt(2.0)))
    elif act == "gelu_tanh":
        y = 0.5 * y * (1.0 + torch.tanh(math.sqrt(2.0 / math.pi) * (y + 0.044715 * y ** 3)))
    if residual is not None:
        y = y + _f(residual)
    return y


def swiglu_block(x, residual, norm_w, eps, w_gate_nk, w_up_nk, w_down_nk):
    """The cfg1 pre-norm SwiGLU block: n = RMSNorm(x + residual);
    out = (x + residual) + down(silu(gate(n)) * up(n)), all fp32
    (src/umic/integrate.py:44-55 + :180-209 composed)."""
    normed, summed = add_rmsnorm(x, residual, norm_w, eps)
    h = silu(normed @ _f(w_gate_nk).t()) * (normed @ _f(w_up_nk).t())
    return summed + h @ _f(w_down_nk).t()


def attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, mask: torch.Tensor | None,
              scale: float) -> torch.Tensor:
    """softmax(scale * q k^T, masked) v in fp32 with grouped-query heads -> [B, T, Hq, D].

    The attention transformers runs for the patched Qwen3 attention (sdpa_attention_forward
    in transformers/integrations/sdpa_attention.py: repeat_kv over the query heads, then
    torch SDPA with the boolean mask, True = attend), which the reference leaves in
    place. q [B, Hq, T, D], k / v [B, Hkv, L, D], mask broadcastable to [B, Hq, T, L].
    Rows that attend to nothing come out as zeros."""
    qf, kf, vf = _f(q), _f(k), _f(v)
    g = qf.shape[1] // kf.shape[1]
    kf = kf.repeat_interleave(g, 1)
    vf = vf.repeat_interleave(g, 1)
    s = (qf @ kf.transpose(-1, -2)) * scale
    if mask is not None:
        s = s.masked_fill(~mask.detach().cpu()[..., : kf.shape[2]], float("-inf"))
    p = torch.nan_to_num(torch.softmax(s, -1), nan=0.0)
    return (p @ vf).transpose(1, 2)
