"""Module-level fusion injection: the reference's drop-in API on B200 kernels.

Mirrors src/umic/integrate.py of soonhong99/umic-alpamayo: the `forward` of
structurally matching submodules (duck-typed, never class-based) is rebound to
a fused implementation at load time; weights are shared as views, never copied
or changed. Every `fuse_*` function keeps the reference's name, arguments,
dry_run semantics and return value (a match count, or a bool for the
module-global patches). What changes is what runs behind the patched forwards:
hand-written sm_100a kernels from libumic_b200.so instead of Triton/cuBLAS,
including the rows < FUSE_MIN_ROWS (decode) regime, which the reference left
on cuBLAS and which here runs the weight-streaming GEMV.

The installed transformers (5.5) differs from the version the reference was
written against (>=4.56): decoder layers no longer take `cache_position`, the
vision encoder returns a BaseModelOutputWithDeepstackFeatures, and the VLM
exposes its language model / vision tower under `.model`. The patched forwards
follow the installed API.
"""

from __future__ import annotations

import logging
import math

import torch
from torch import nn

from .kernels import rope as _rope
from .kernels.fused_ffn import gate_silu_mul_nk
from .kernels.layernorm import add_layernorm, layernorm
from .kernels.linear import linear, linear_gemv, linear_gemv_residual
from .kernels.rmsnorm import add_rmsnorm, rmsnorm

logger = logging.getLogger(__name__)

_SILU_NAMES = ("silu", "swish")

# Below this row count a projection is a GEMV (decode, seq = 1): it runs the
# HBM-bound weight-streaming kernel; at or above it, the tcgen05 GEMM
# (regime-aware dispatch, src/umic/integrate.py:27-30).
FUSE_MIN_ROWS = 64

# Projection sites routed to the tensor-core GEMM at >= FUSE_MIN_ROWS rows
# (src/umic/integrate.py:91). k/v stay on their original Linear in prefill.
INEFFICIENT_LINEAR_NAMES = ("q_proj", "o_proj")

# ViT sites for the same GEMM (src/umic/integrate.py:93-95); not applied by
# apply(), as in the reference.
VIT_LINEAR_NAMES = ("qkv",)


def _eps_of(module: nn.Module, default: float = 1e-6) -> float:
    eps = getattr(module, "variance_epsilon", None)
    if eps is None:
        eps = getattr(module, "eps", default)
    return float(eps)


# --------------------------------------------------------------- SwiGLU MLP

def _is_p5_mlp(module: nn.Module) -> bool:
    """gate_proj/up_proj/down_proj bias-free Linears + a SiLU-family activation
    (src/umic/integrate.py:33-41)."""
    for attr in ("gate_proj", "up_proj", "down_proj"):
        sub = getattr(module, attr, None)
        if not isinstance(sub, nn.Linear) or sub.bias is not None:
            return False
    act = getattr(module, "act_fn", None) or getattr(module, "act", None)
    act_name = type(act).__name__.lower() if act is not None else ""
    return any(s in act_name for s in _SILU_NAMES)


def _project(lin: nn.Linear, x2d: torch.Tensor, residual: torch.Tensor | None = None):
    """A Linear on the B200 kernels: GEMV below FUSE_MIN_ROWS, tcgen05 GEMM above; a
    residual is added in either kernel's epilogue."""
    if x2d.shape[0] < FUSE_MIN_ROWS:
        if residual is None:
            return linear_gemv(x2d, lin.weight, lin.bias, weights_ready=True)
        return linear_gemv_residual(x2d, lin.weight, residual, lin.bias, weights_ready=True)
    return linear(x2d, lin.weight, lin.bias, residual=residual)


def mlp_forward(mlp: nn.Module, x: torch.Tensor,
                residual: torch.Tensor | None = None) -> torch.Tensor:
    """down(silu(gate(x)) * up(x)) [+ residual], x [..., H].

    gate/up run as one fused kernel (dual-accumulator GEMM or gated GEMV); the
    down projection runs on the GEMM, or the GEMV below FUSE_MIN_ROWS, with the
    residual add in its epilogue when `residual` is given.
    """
    shape = x.shape
    x2d = x.reshape(-1, shape[-1])
    h = gate_silu_mul_nk(x2d, mlp.gate_proj.weight, mlp.up_proj.weight, weights_ready=True)
    r2d = residual.reshape(-1, residual.shape[-1]) if residual is not None else None
    out = _project(mlp.down_proj, h, r2d)
    return out.reshape(*shape[:-1], out.shape[-1])


def _fused_mlp_forward(self: nn.Module, x: torch.Tensor) -> torch.Tensor:
    """P5-fused replacement (src/umic/integrate.py:44-55)."""
    return mlp_forward(self, x)


def fuse_mlps(model: nn.Module, dry_run: bool = False) -> int:
    """Swap the forward of every P5-matching MLP (src/umic/integrate.py:58-77)."""
    count = 0
    for name, module in model.named_modules():
        if _is_p5_mlp(module):
            count += 1
            if not dry_run:
                module.forward = _fused_mlp_forward.__get__(module)
                module._umic_p5 = True
                logger.info("P5 fused: %s", name)
    logger.info("fuse_mlps: %d module(s) %s", count,
                "matched (dry run)" if dry_run else "patched")
    return count


# ------------------------------------------------------------- projections

def _patched_linear_forward(self: nn.Linear, x: torch.Tensor) -> torch.Tensor:
    """GEMV below FUSE_MIN_ROWS, tcgen05 GEMM above (src/umic/integrate.py:98-107)."""
    shape = x.shape
    x2d = x.reshape(-1, shape[-1])
    out = _project(self, x2d)
    return out.reshape(*shape[:-1], out.shape[-1])


def fuse_linears(model: nn.Module, names: tuple[str, ...] = INEFFICIENT_LINEAR_NAMES,
                 dry_run: bool = False) -> int:
    """Swap the forward of nn.Linear submodules whose attribute name matches
    (src/umic/integrate.py:110-131)."""
    count = 0
    for name, module in model.named_modules():
        leaf = name.rsplit(".", 1)[-1]
        if leaf in names and isinstance(module, nn.Linear):
            count += 1
            if not dry_run:
                module.forward = _patched_linear_forward.__get__(module)
    logger.info("fuse_linears(%s): %d module(s) %s", names, count,
                "matched (dry run)" if dry_run else "patched")
    return count


def _decode_gemv_forward(self: nn.Linear, x: torch.Tensor) -> torch.Tensor:
    """Decode-only rebind: the GEMV below FUSE_MIN_ROWS, the original Linear above."""
    shape = x.shape
    x2d = x.reshape(-1, shape[-1])
    if x2d.shape[0] >= FUSE_MIN_ROWS or not x2d.is_cuda or x2d.dtype != torch.bfloat16:
        return nn.functional.linear(x, self.weight, self.bias)
    out = linear_gemv(x2d, self.weight, self.bias, weights_ready=True)
    return out.reshape(*shape[:-1], out.shape[-1])


def fuse_decode_linears(model: nn.Module, dry_run: bool = False) -> int:
    """Route every remaining (not yet rebound) nn.Linear of `model` to the GEMV
    when it sees fewer than FUSE_MIN_ROWS rows. Extends the reference, which
    left decode projections on cuBLAS (src/umic/integrate.py:27-30,48-50)."""
    count = 0
    for _, module in model.named_modules():
        if isinstance(module, nn.Linear) and "forward" not in module.__dict__:
            count += 1
            if not dry_run:
                module.forward = _decode_gemv_forward.__get__(module)
    return count


# --------------------------------------------------------------- attention

def _is_qk_norm_attention(module: nn.Module) -> bool:
    """q/k/v/o projections plus per-head q_norm / k_norm (Qwen3 text attention)."""
    for attr in ("q_proj", "k_proj", "v_proj", "o_proj"):
        if not isinstance(getattr(module, attr, None), nn.Linear):
            return False
    for attr in ("q_norm", "k_norm"):
        w = getattr(getattr(module, attr, None), "weight", None)
        if not isinstance(w, torch.Tensor) or w.dim() != 1:
            return False
    return all(hasattr(module, a) for a in ("head_dim", "scaling", "layer_idx", "config"))


def _fused_attention_forward(self, hidden_states, position_embeddings=None, attention_mask=None,
                             past_key_values=None, **kwargs):
    """Text attention with its input path fused: projections (one multi-matrix GEMV
    below FUSE_MIN_ROWS; tcgen05 GEMM for q and the original Linears for k / v above),
    then one kernel for q_norm / k_norm, RoPE and the KV-cache write, then the
    model's attention backend and o_proj. Follows HF's Qwen3VLTextAttention.forward;
    layouts the kernel does not cover run the original forward."""
    from transformers.modeling_utils import ALL_ATTENTION_FUNCTIONS
    from transformers.models.qwen3_vl.modeling_qwen3_vl import eager_attention_forward

    from .cache import InplaceKVCache
    from .kernels.attention import qk_norm_rope_kv
    from .kernels.linear import linear_gemv_multi

    d = self.head_dim
    cos, sin = position_embeddings if position_embeddings is not None else (None, None)
    if (cos is None or hidden_states.dim() != 3 or not hidden_states.is_cuda
            or hidden_states.dtype != torch.bfloat16 or d not in (64, 128, 256)
            or cos.dim() != 3 or cos.shape[-1] != d
            or (torch.is_grad_enabled()
                and (hidden_states.requires_grad or self.q_proj.weight.requires_grad))):
        return type(self).forward(self, hidden_states, position_embeddings, attention_mask,
                                  past_key_values=past_key_values, **kwargs)
    b, s, _ = hidden_states.shape
    x2d = hidden_states.reshape(-1, hidden_states.shape[-1])
    if x2d.shape[0] < FUSE_MIN_ROWS:
        q, k, v = linear_gemv_multi(
            x2d, [self.q_proj.weight, self.k_proj.weight, self.v_proj.weight],
            [self.q_proj.bias, self.k_proj.bias, self.v_proj.bias], weights_ready=True)
    else:
        q = linear(x2d, self.q_proj.weight, self.q_proj.bias)
        k = nn.functional.linear(x2d, self.k_proj.weight, self.k_proj.bias)
        v = nn.functional.linear(x2d, self.v_proj.weight, self.v_proj.bias)
    q4, k4, v4 = q.view(b, s, -1, d), k.view(b, s, -1, d), v.view(b, s, -1, d)
    qn, kn = self.q_norm, self.k_norm
    layer = (past_key_values.layers[self.layer_idx]
             if isinstance(past_key_values, InplaceKVCache) else None)
    if layer is not None:
        kb, vb, pos = layer.reserve(s)
        qk_norm_rope_kv(q4, k4, v4, qn.weight, kn.weight, _eps_of(qn), _eps_of(kn), cos, sin,
                        kb, vb, pos)
        keys, values = layer.keys, layer.values
    else:
        qk_norm_rope_kv(q4, k4, None, qn.weight, kn.weight, _eps_of(qn), _eps_of(kn), cos, sin)
        keys, values = k4.transpose(1, 2), v4.transpose(1, 2)
        if past_key_values is not None:
            keys, values = past_key_values.update(keys, values, self.layer_idx)
    impl = self.config._attn_implementation
    attn = (gqa_sdpa_attention if impl == "sdpa"
            else ALL_ATTENTION_FUNCTIONS.get_interface(impl, eager_attention_forward))
    out, weights = attn(self, q4.transpose(1, 2), keys, values, attention_mask,
                        dropout=0.0 if not self.training else self.attention_dropout,
                        scaling=self.scaling, **kwargs)
    out = out.reshape(b, s, -1).contiguous()
    return self.o_proj(out), weights


def gqa_sdpa_attention(module: nn.Module, query: torch.Tensor, key: torch.Tensor,
                       value: torch.Tensor, attention_mask: torch.Tensor | None,
                       dropout: float = 0.0, scaling: float | None = None,
                       is_causal: bool | None = None, **kwargs):
    """transformers' "sdpa" attention (same mask and causal rules) with SDPA's native
    grouped-query path for every mask. transformers 5.x expands K/V to the query heads
    (repeat_kv) whenever a mask is passed -- e.g. the flow expert's 64 action tokens
    over a 3.1 k-token prefix, two ~0.4 GB copies per layer per step; SDPA with
    enable_gqa takes the boolean mask directly (cuDNN kernel, same result). A boolean
    mask over few query rows per KV head (at most 128, e.g. 64 action tokens x 2
    query heads) goes to the tcgen05 kernel (kernels.attention.attention_rows)."""
    if attention_mask is not None and attention_mask.dim() == 4:
        attention_mask = attention_mask[:, :, :, : key.shape[-2]]
        if (attention_mask.dtype == torch.bool and query.shape[2] > 1 and dropout == 0.0
                and query.is_cuda and query.dtype == torch.bfloat16):
            # Few query rows per KV head over a long prefix (the flow expert's action
            # tokens over the cached prefix): the tcgen05 kernel reads the mask itself.
            from .kernels.attention import attention_rows

            out = attention_rows(query, key, value, attention_mask,
                                 scaling if scaling is not None else query.shape[-1] ** -0.5)
            if out is not None:
                return out, None
    causal = is_causal if is_causal is not None else getattr(module, "is_causal", True)
    causal = bool(query.shape[2] > 1 and attention_mask is None and causal)
    out = nn.functional.scaled_dot_product_attention(
        query, key, value, attn_mask=attention_mask, dropout_p=dropout, scale=scaling,
        is_causal=causal, enable_gqa=query.shape[1] != key.shape[1])
    return out.transpose(1, 2).contiguous(), None


def fuse_attention(model: nn.Module, dry_run: bool = False) -> int:
    """Fuse the attention input path (projections, q/k norm, RoPE, KV write) of every
    Qwen3-style text attention module. No single reference counterpart: it merges the
    reference's q/o-projection, RMSNorm, text-RoPE and in-place-cache patches
    (src/umic/integrate.py:98-167, 661-682; src/umic/cache.py:50-80) into one path."""
    count = 0
    for _, module in model.named_modules():
        if not _is_qk_norm_attention(module):
            continue
        count += 1
        if not dry_run:
            module.forward = _fused_attention_forward.__get__(module)
    logger.info("fuse_attention: %d module(s) %s", count,
                "matched (dry run)" if dry_run else "patched")
    return count


# ---------------------------------------------------------------- RMSNorm

def _patched_rmsnorm_forward(self: nn.Module, x: torch.Tensor) -> torch.Tensor:
    """One kernel for the eager pow/mean/mul/cast chain (src/umic/integrate.py:134-141)."""
    return rmsnorm(x, self.weight, _eps_of(self))


def fuse_rmsnorms(model: nn.Module, dry_run: bool = False) -> int:
    """Class name contains "rmsnorm" and a 1-D weight (src/umic/integrate.py:144-167)."""
    count = 0
    for _, module in model.named_modules():
        if "rmsnorm" not in type(module).__name__.lower():
            continue
        w = getattr(module, "weight", None)
        if not isinstance(w, torch.Tensor) or w.dim() != 1:
            continue
        count += 1
        if not dry_run:
            module.forward = _patched_rmsnorm_forward.__get__(module)
    logger.info("fuse_rmsnorms: %d module(s) %s", count,
                "matched (dry run)" if dry_run else "patched")
    return count


def _is_residual_decoder_layer(module: nn.Module) -> bool:
    """Pre-norm attn + MLP decoder block (src/umic/integrate.py:170-177)."""
    return all(hasattr(module, a) for a in
               ("input_layernorm", "post_attention_layernorm", "self_attn", "mlp"))


def _fused_residual_layer_forward(self, hidden_states, position_embeddings=None,
                                  attention_mask=None, position_ids=None, past_key_values=None,
                                  use_cache=False, **kwargs):
    """Decoder layer with the attention residual folded into post_attention_layernorm
    (src/umic/integrate.py:180-209). When the MLP is P5-fused, its residual add
    also moves into the down-projection epilogue, of the GEMM or (decode rows) the
    GEMV (the reference left that add eager, integrate.py:207-208)."""
    residual = hidden_states
    hidden_states = self.input_layernorm(hidden_states)
    hidden_states, _ = self.self_attn(
        hidden_states=hidden_states, attention_mask=attention_mask, position_ids=position_ids,
        past_key_values=past_key_values, use_cache=use_cache,
        position_embeddings=position_embeddings, **kwargs)
    hidden_states, residual = add_rmsnorm(hidden_states, residual,
                                          self.post_attention_layernorm.weight,
                                          _eps_of(self.post_attention_layernorm))
    mlp = self.mlp
    if getattr(mlp, "_umic_p5", False) and mlp.forward.__func__ is _fused_mlp_forward:
        return mlp_forward(mlp, hidden_states, residual=residual)
    hidden_states = mlp(hidden_states)
    return residual + hidden_states


def fuse_add_rmsnorm(model: nn.Module, dry_run: bool = False) -> int:
    """Patch every pre-norm decoder layer (src/umic/integrate.py:212-231)."""
    count = 0
    for _, module in model.named_modules():
        if not _is_residual_decoder_layer(module):
            continue
        count += 1
        if not dry_run:
            module.forward = _fused_residual_layer_forward.__get__(module)
    logger.info("fuse_add_rmsnorm: %d decoder layer(s) %s", count,
                "matched (dry run)" if dry_run else "patched")
    return count


# -------------------------------------------------------------- LayerNorm

def _patched_layernorm_forward(self: nn.LayerNorm, x: torch.Tensor) -> torch.Tensor:
    return layernorm(x, self.weight, self.bias, self.eps)


def fuse_layernorms(model: nn.Module, dry_run: bool = False) -> int:
    """Last-dim affine nn.LayerNorm with bias (src/umic/integrate.py:234-258)."""
    count = 0
    for _, module in model.named_modules():
        if (isinstance(module, nn.LayerNorm) and len(module.normalized_shape) == 1
                and module.weight is not None and module.bias is not None):
            count += 1
            if not dry_run:
                module.forward = _patched_layernorm_forward.__get__(module)
    logger.info("fuse_layernorms: %d module(s) %s", count,
                "matched (dry run)" if dry_run else "patched")
    return count


# ------------------------------------------------------------ GELU MLP (ViT)

_FC1_NAMES = ("fc1", "linear_fc1", "up_proj")
_FC2_NAMES = ("fc2", "linear_fc2", "down_proj")


def _gelu_kind(act) -> str | None:
    """'gelu_tanh' / 'gelu' (erf) for a GELU-family activation module, else None."""
    if act is None:
        return None
    name = type(act).__name__.lower()
    if "gelu" not in name and getattr(act, "__name__", "") != "gelu":
        return None
    approx = getattr(act, "approximate", None)
    if approx == "tanh" or "tanh" in name:
        return "gelu_tanh"
    return "gelu"


def _is_gelu_mlp(module: nn.Module):
    """fc1 -> GELU -> fc2, dimension-preserving (src/umic/integrate.py:266-289)."""
    fc1 = next((getattr(module, n) for n in _FC1_NAMES
                if isinstance(getattr(module, n, None), nn.Linear)), None)
    fc2 = next((getattr(module, n) for n in _FC2_NAMES
                if isinstance(getattr(module, n, None), nn.Linear)), None)
    if fc1 is None or fc2 is None or hasattr(module, "gate_proj"):
        return None
    if fc1.in_features != fc2.out_features:
        return None
    act = getattr(module, "act_fn", None) or getattr(module, "act", None) \
        or getattr(module, "activation_fn", None)
    if _gelu_kind(act) is None:
        return None
    return fc1, fc2


def _fused_gelu_mlp_forward(self: nn.Module, x: torch.Tensor) -> torch.Tensor:
    """fc1 + GELU in one GEMM epilogue, then fc2 (src/umic/integrate.py:292-303). The
    epilogue uses the module's own GELU form (tanh or erf); the reference always
    used erf (linear.py:83-86) although the ViT uses tanh. fc2 is a plain Linear
    with nothing to fuse, so it stays on cuBLAS (as the reference leaves plain
    Linears): at the ViT shape (N = 1280: 5 column tiles over 74 CTA pairs) cuBLAS's
    tiling wins (27.7 vs 28.3 ms for the 27-block encoder over 16 images)."""
    fc1, fc2 = self._umic_fc
    shape = x.shape
    x2d = x.reshape(-1, shape[-1])
    if x2d.shape[0] < FUSE_MIN_ROWS:
        act = getattr(self, "act_fn", None) or getattr(self, "act")
        return fc2(act(fc1(x)))
    h = linear(x2d, fc1.weight, fc1.bias, act=self._umic_gelu)
    out = nn.functional.linear(h, fc2.weight, fc2.bias)
    return out.reshape(*shape[:-1], out.shape[-1])


def fuse_gelu_mlps(model: nn.Module, dry_run: bool = False) -> int:
    """Fuse fc1+GELU for GELU-MLP modules (src/umic/integrate.py:306-319)."""
    count = 0
    for _, module in model.named_modules():
        pair = _is_gelu_mlp(module)
        if pair is None:
            continue
        count += 1
        if not dry_run:
            act = getattr(module, "act_fn", None) or getattr(module, "act", None) \
                or getattr(module, "activation_fn", None)
            module._umic_fc = pair
            module._umic_gelu = _gelu_kind(act)
            module.forward = _fused_gelu_mlp_forward.__get__(module)
    logger.info("fuse_gelu_mlps: %d module(s) %s", count,
                "matched (dry run)" if dry_run else "patched")
    return count


# ------------------------------------------------------------ patch embed

def _is_full_stride_conv(module: nn.Module) -> bool:
    """ConvNd with stride == kernel, no padding, groups 1 (src/umic/integrate.py:322-340)."""
    if not isinstance(module, (nn.Conv1d, nn.Conv2d, nn.Conv3d)):
        return False
    if module.groups != 1:
        return False
    if any(p != 0 for p in module.padding):
        return False
    return tuple(module.stride) == tuple(module.kernel_size)


def _is_patch_embed_container(module: nn.Module):
    proj = getattr(module, "proj", None)
    if proj is None or not _is_full_stride_conv(proj):
        return None
    return proj


def _patched_patch_embed_forward(self: nn.Module, hidden_states: torch.Tensor) -> torch.Tensor:
    """conv(reshape(x)) == Linear on the flat patch (src/umic/integrate.py:356-360),
    on the tcgen05 GEMM with the bias in the epilogue (K = 1176 has a partial
    last k-block, read as zeros by TMA)."""
    weight2d, bias, in_features = self._umic_patch_linear
    x = hidden_states.reshape(-1, in_features).to(dtype=weight2d.dtype)
    if x.is_cuda and x.dtype == torch.bfloat16:
        return linear(x, weight2d, bias)
    return nn.functional.linear(x, weight2d, bias)


def fuse_patch_embed_linear(model: nn.Module, dry_run: bool = False) -> int:
    """Full-stride ConvNd patch embed -> Linear on a weight view (src/umic/integrate.py:363-389)."""
    count = 0
    for name, module in model.named_modules():
        conv = _is_patch_embed_container(module)
        if conv is None:
            continue
        count += 1
        if not dry_run:
            in_features = conv.in_channels * math.prod(conv.kernel_size)
            weight2d = conv.weight.reshape(conv.out_channels, -1)
            module._umic_patch_linear = (weight2d, conv.bias, in_features)
            module.forward = _patched_patch_embed_forward.__get__(module)
            logger.info("patch-embed conv->linear fused: %s", name)
    return count


# ------------------------------------------------ packed varlen ViT attention

def _is_seqlen_packed_attention(module: nn.Module) -> bool:
    """qkv + proj + num_heads + scaling, forward takes cu_seqlens
    (src/umic/integrate.py:392-407)."""
    if not all(hasattr(module, a) for a in ("qkv", "proj", "num_heads", "scaling")):
        return False
    if not isinstance(getattr(module, "qkv"), nn.Linear):
        return False
    import inspect
    try:
        sig = inspect.signature(type(module).forward)
    except (TypeError, ValueError):
        return False
    return "cu_seqlens" in sig.parameters


def _fused_seqlen_attn_forward(self: nn.Module, hidden_states: torch.Tensor,
                               cu_seqlens: torch.Tensor, rotary_pos_emb=None,
                               position_embeddings=None, **kwargs) -> torch.Tensor:
    """One packed varlen attention call instead of split / per-image / cat
    (src/umic/integrate.py:410-458). Images of one size run on the tcgen05 attention
    kernel; other packings keep torch's varlen flash attention. RoPE runs in place on
    the B200 kernel."""
    import transformers.models.qwen3_vl.modeling_qwen3_vl as _mod

    seq_length = hidden_states.shape[0]
    qkv = self.qkv(hidden_states).reshape(seq_length, 3, self.num_heads, -1)
    query_states, key_states, value_states = qkv.unbind(1)
    cos, sin = position_embeddings
    query_states, key_states = _mod.apply_rotary_pos_emb_vision(query_states, key_states, cos, sin)
    cache: dict = self._umic_attn_cache
    if cache.get("cu_seqlens_ref") is not cu_seqlens:
        cache["cu_seqlens_ref"] = cu_seqlens
        lens = cu_seqlens[1:] - cu_seqlens[:-1]
        lo, hi = (int(v) for v in torch.stack((lens.min(), lens.max())).tolist())
        cache["max_seqlen"] = hi
        cache["uniform_len"] = hi if lo == hi and hi > 0 else 0
    max_seqlen = cache["max_seqlen"]
    n = cache["uniform_len"]
    if n and query_states.is_cuda and query_states.dtype == torch.bfloat16:
        # Images of one size: [images, heads, patches, head_dim] views of the packed
        # qkv, attention on the tcgen05 kernel (128-patch tiles per image and head).
        from .kernels.attention import attention_rows

        imgs, heads, hd = seq_length // n, self.num_heads, query_states.shape[-1]
        q4, k4, v4 = (t.view(imgs, n, heads, hd).transpose(1, 2)
                      for t in (query_states, key_states, value_states))
        out4 = attention_rows(q4, k4, v4, None, self.scaling)
        if out4 is not None:
            return self.proj(out4.reshape(seq_length, -1))
    out = torch.ops.aten._flash_attention_forward(
        query_states, key_states, value_states, cu_seqlens, cu_seqlens, max_seqlen, max_seqlen,
        0.0, False, False, scale=self.scaling)
    attn_output = out[0].reshape(seq_length, -1)
    return self.proj(attn_output)


def fuse_vision_attention_varlen(model: nn.Module, dry_run: bool = False) -> int:
    """(src/umic/integrate.py:461-478)"""
    count = 0
    for _, module in model.named_modules():
        if not _is_seqlen_packed_attention(module):
            continue
        count += 1
        if not dry_run:
            module._umic_attn_cache = {}
            module.forward = _fused_seqlen_attn_forward.__get__(module)
    return count


# -------------------------------------------------- ViT pipeline forward

def _is_deepstack_vision_encoder(module: nn.Module) -> bool:
    """grid_thw-driven ViT with deepstack taps (src/umic/integrate.py:481-506)."""
    blocks = getattr(module, "blocks", None)
    if not blocks or len(blocks) == 0:
        return False
    b0 = blocks[0]
    if not all(hasattr(b0, a) for a in ("norm1", "norm2", "attn", "mlp")):
        return False
    if not (isinstance(getattr(b0, "norm1", None), nn.LayerNorm)
            and isinstance(getattr(b0, "norm2", None), nn.LayerNorm)):
        return False
    merger = getattr(module, "merger", None)
    if merger is None or not all(hasattr(merger, a) for a in
                                 ("norm", "linear_fc1", "act_fn", "linear_fc2",
                                  "use_postshuffle_norm", "hidden_size")):
        return False
    return all(hasattr(module, a) for a in
               ("patch_embed", "deepstack_merger_list", "deepstack_visual_indexes",
                "fast_pos_embed_interpolate", "rot_pos_emb"))


def _fused_vision_encoder_forward(self: nn.Module, hidden_states: torch.Tensor,
                                  grid_thw: torch.Tensor, **kwargs):
    """grid_thw constants cached; 24 of 27 residual adds folded into the next
    LayerNorm, intra- and cross-block, and the last into the merger norm
    (src/umic/integrate.py:509-611). Returns the installed transformers' output
    type (BaseModelOutputWithDeepstackFeatures)."""
    import torch.nn.functional as F
    from transformers.models.qwen3_vl.modeling_qwen3_vl import (
        BaseModelOutputWithDeepstackFeatures)

    cache: dict = self._umic_ve_cache
    key = tuple(grid_thw.reshape(-1).tolist())
    if cache.get("key") != key:
        pos_embeds = self.fast_pos_embed_interpolate(grid_thw)
        rotary_pos_emb = self.rot_pos_emb(grid_thw)
        seq_len = int(sum(t * h * w for t, h, w in grid_thw.tolist()))
        rotary_pos_emb_r = rotary_pos_emb.reshape(seq_len, -1)
        emb = torch.cat((rotary_pos_emb_r, rotary_pos_emb_r), dim=-1)
        cu_seqlens = torch.repeat_interleave(
            grid_thw[:, 1] * grid_thw[:, 2], grid_thw[:, 0]).cumsum(dim=0, dtype=torch.int32)
        cu_seqlens = F.pad(cu_seqlens, (1, 0), value=0)
        cache["key"] = key
        cache["consts"] = (pos_embeds.detach().clone(),
                           (emb.cos().detach().contiguous(), emb.sin().detach().contiguous()),
                           cu_seqlens.detach().clone())
    pos_embeds, position_embeddings, cu_seqlens = cache["consts"]
    hidden_states = self.patch_embed(hidden_states)
    hidden_states = hidden_states + pos_embeds
    seq_len = hidden_states.shape[0]
    hidden_states = hidden_states.reshape(seq_len, -1)

    deepstack_set: set = self._umic_deepstack_set
    merger = self.merger
    deepstack_feature_lists = []
    pending = None
    for layer_num, blk in enumerate(self.blocks):
        norm1, norm2, attn, mlp = blk.norm1, blk.norm2, blk.attn, blk.mlp
        if pending is None:
            normed1 = norm1(hidden_states)
        else:
            normed1, hidden_states = add_layernorm(pending, hidden_states, norm1.weight,
                                                   norm1.bias, norm1.eps)
            pending = None
        attn_out = attn(normed1, cu_seqlens=cu_seqlens, position_embeddings=position_embeddings,
                        **kwargs)
        normed2, hidden_states = add_layernorm(attn_out, hidden_states, norm2.weight, norm2.bias,
                                               norm2.eps)
        mlp_out = mlp(normed2)
        if layer_num in deepstack_set:
            hidden_states = hidden_states + mlp_out
            deepstack_feature_lists.append(self.deepstack_merger_list[
                self.deepstack_visual_indexes.index(layer_num)](hidden_states))
        else:
            pending = mlp_out
    if pending is not None and not merger.use_postshuffle_norm:
        normed, hidden_states = add_layernorm(pending, hidden_states, merger.norm.weight,
                                              merger.norm.bias, merger.norm.eps)
        x = normed.view(-1, merger.hidden_size)
        merged = merger.linear_fc2(merger.act_fn(merger.linear_fc1(x)))
    else:
        if pending is not None:
            hidden_states = hidden_states + pending
        merged = merger(hidden_states)
    return BaseModelOutputWithDeepstackFeatures(
        last_hidden_state=hidden_states, pooler_output=merged,
        deepstack_features=deepstack_feature_lists)


def fuse_vision_encoder_pipeline(model: nn.Module, dry_run: bool = False) -> int:
    """(src/umic/integrate.py:614-638)"""
    count = 0
    for name, module in model.named_modules():
        if not _is_deepstack_vision_encoder(module):
            continue
        count += 1
        if not dry_run:
            module._umic_ve_cache = {}
            module._umic_deepstack_set = set(module.deepstack_visual_indexes)
            module.forward = _fused_vision_encoder_forward.__get__(module)
            logger.info("vision encoder pipeline fused: %s", name)
    return count


# ------------------------------------------------------ module-global RoPE

def fuse_vision_rope() -> bool:
    """HF apply_rotary_pos_emb_vision -> in-place B200 kernel (src/umic/integrate.py:641-658)."""
    try:
        import transformers.models.qwen3_vl.modeling_qwen3_vl as mod
    except ImportError:
        logger.warning("fuse_vision_rope: qwen3_vl module not found")
        return False
    if getattr(mod.apply_rotary_pos_emb_vision, "_umic_fused", False):
        return True
    fused = _rope.make_vision_rope(mod.apply_rotary_pos_emb_vision)
    fused._umic_fused = True
    fused._umic_original = mod.apply_rotary_pos_emb_vision
    mod.apply_rotary_pos_emb_vision = fused
    return True


def fuse_text_rope() -> bool:
    """HF apply_rotary_pos_emb -> in-place B200 kernel; unsupported layouts fall
    back to the original (src/umic/integrate.py:661-682)."""
    try:
        import transformers.models.qwen3_vl.modeling_qwen3_vl as mod
    except ImportError:
        logger.warning("fuse_text_rope: qwen3_vl module not found")
        return False
    if getattr(mod.apply_rotary_pos_emb, "_umic_fused", False):
        return True
    fused = _rope.make_text_rope(mod.apply_rotary_pos_emb)
    fused._umic_fused = True
    fused._umic_original = mod.apply_rotary_pos_emb
    mod.apply_rotary_pos_emb = fused
    return True


def unfuse_rope() -> None:
    """Restore HF's module-global RoPE functions (test / A-B helper)."""
    import transformers.models.qwen3_vl.modeling_qwen3_vl as mod

    for name in ("apply_rotary_pos_emb", "apply_rotary_pos_emb_vision"):
        orig = getattr(getattr(mod, name), "_umic_original", None)
        if orig is not None:
            setattr(mod, name, orig)


def fuse_bf16_residual(visual: nn.Module, dtype: torch.dtype = torch.bfloat16) -> bool:
    """Cast the ViT residual stream back to bf16 at blocks[0] (src/umic/integrate.py:685-712)."""
    blocks = getattr(visual, "blocks", None)
    if not blocks:
        return False

    def _pre(module, args, kwargs):
        hs = args[0] if args else kwargs.get("hidden_states")
        if hs is None or hs.dtype == dtype:
            return None
        if args:
            return (hs.to(dtype),) + args[1:], kwargs
        kwargs["hidden_states"] = hs.to(dtype)
        return args, kwargs

    blocks[0].register_forward_pre_hook(_pre, with_kwargs=True)
    return True


# -------------------------------------------------------------- KV cache hook

def fuse_repeat_cache(repeat_module: nn.Module, extra_tokens_hint: int = 64) -> None:
    """Convert a DynamicCache to InplaceKVCache once per source cache and re-sync
    its write pointer on every call (src/umic/integrate.py:715-756)."""
    from transformers.cache_utils import DynamicCache

    from .cache import InplaceKVCache

    state: dict[str, object] = {"orig_id": None, "converted": None}

    def _pre_hook(module, args, kwargs):
        pkv = kwargs.get("past_key_values")
        if pkv is None or isinstance(pkv, InplaceKVCache):
            return None
        if not isinstance(pkv, DynamicCache) or not getattr(pkv, "layers", None):
            return None
        if any(getattr(lyr, "keys", None) is None for lyr in pkv.layers):
            return None
        n_new = 0
        emb = kwargs.get("inputs_embeds")
        if emb is not None:
            n_new = emb.shape[1]
        if state["orig_id"] != id(pkv):
            state["orig_id"] = id(pkv)
            state["converted"] = InplaceKVCache.from_dynamic(
                pkv, extra_tokens=max(n_new, extra_tokens_hint))
        conv = state["converted"]
        conv.crop(pkv.get_seq_length())
        kwargs["past_key_values"] = conv
        return args, kwargs

    repeat_module.register_forward_pre_hook(_pre_hook, with_kwargs=True)


def unfuse_mlps(model: nn.Module) -> int:
    """Delete every instance-level forward override (src/umic/integrate.py:759-766)."""
    count = 0
    for _, module in model.named_modules():
        if "forward" in module.__dict__:
            del module.__dict__["forward"]
            count += 1
    return count
