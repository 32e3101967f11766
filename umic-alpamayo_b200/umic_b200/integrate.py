"""Drop-in rebinding of matched modules onto the B200 kernels.

Design: a motif registry with one walker. A `Motif` pairs a structural matcher
(attributes, types and shapes only -- never a class identity, so any model that
carries the motif matches) with the forward that replaces the matched module's.
`_rebind(model, motif, dry_run)` is the only place that walks a model: it
collects every site whose matcher returns a binding, installs the motif's
forward on each (unless dry_run), logs one line and returns the count.

A binding (`*Site` records below) is what the fused forward needs, resolved
once at install time and stored on the module as `_umic_site`: the Linears of a
SwiGLU block, the GELU form of a ViT MLP, the weight view of a patch-embed conv,
the segment layout cache of a packed attention. Parameters are referenced,
never copied, and read at call time, so a later `load_state_dict` is seen.

The public `fuse_*` functions are the walker applied to one motif each. They
keep the interface of the reference's src/umic/integrate.py -- names,
arguments, dry_run, the returned count (or bool for the module-global RoPE
swaps) and which modules match -- while everything behind the patched forwards
is this build's: tcgen05 GEMMs and the weight-streaming GEMV below
FUSE_MIN_ROWS (the reference kept cuBLAS there), the fused attention input
(q/k norm + RoPE + KV write in one kernel), residual adds in GEMM/GEMV
epilogues, the tcgen05 prefix attention for the flow expert and the ViT.

The installed transformers (5.5) is newer than the reference's target
(>= 4.56): decoder layers take no `cache_position`, the vision encoder returns
BaseModelOutputWithDeepstackFeatures, and the VLM keeps its language model and
vision tower under `.model`. The forwards here follow the installed API.
"""

from __future__ import annotations

import contextlib
import inspect
import logging
import math
import types
from dataclasses import dataclass, field
from typing import Any, Callable

import torch
from torch import nn

from .kernels import rope as _rope
from .kernels.fused_ffn import gate_silu_mul_nk
from .kernels.layernorm import add_layernorm, layernorm
from .kernels.linear import linear, linear_gemv, linear_gemv_residual
from .kernels.rmsnorm import add_rmsnorm, rmsnorm, rmsnorm_axpy

logger = logging.getLogger(__name__)

# Row-count regime switch (src/umic/integrate.py:27-30): below it a projection is
# HBM-bound (decode, one token per row) and runs the weight-streaming GEMV; at or
# above it, the tcgen05 GEMM.
FUSE_MIN_ROWS = 64

# Projection sites routed to the GEMM at >= FUSE_MIN_ROWS rows (src/umic/integrate.py:91);
# k_proj / v_proj keep their Linear in prefill.
INEFFICIENT_LINEAR_NAMES = ("q_proj", "o_proj")

# ViT projection sites for the same GEMM (src/umic/integrate.py:93-95).
VIT_LINEAR_NAMES = ("qkv",)

_SITE = "_umic_site"


# =========================================================== registry + walker

@dataclass(frozen=True)
class Motif:
    """A structural pattern and the forward that replaces a matching module's."""

    label: str
    match: Callable[[nn.Module], Any]  # -> binding, or None when the module does not match
    forward: Callable[..., Any] | None  # installed as the module's bound forward


def _install(module: nn.Module, forward: Callable[..., Any], site: Any) -> None:
    module.__dict__[_SITE] = site
    module.forward = types.MethodType(forward, module)


def _site(module: nn.Module, kind: type | tuple[type, ...]):
    """The binding this package installed on `module`, if it is of `kind`."""
    if "forward" not in module.__dict__:
        return None
    s = module.__dict__.get(_SITE)
    return s if isinstance(s, kind) else None


def _rebind(model: nn.Module, motif: Motif, dry_run: bool,
            install: Callable[[nn.Module, Any], None] | None = None) -> int:
    found = []
    for name, module in model.named_modules():
        binding = motif.match(module)
        if binding is not None:
            found.append((name, module, binding))
    if not dry_run:
        for name, module, binding in found:
            if install is not None:
                install(module, binding)
            else:
                _install(module, motif.forward, binding)
            logger.debug("%s -> %s", motif.label, name or type(module).__name__)
    logger.info("%s: %d site(s)%s", motif.label, len(found), " matched (dry run)" if dry_run else "")
    return len(found)


def unfuse_mlps(model: nn.Module) -> int:
    """Remove every instance-level forward installed on `model`'s modules (and their
    bindings), restoring the class forwards; returns how many were removed
    (src/umic/integrate.py:759-766)."""
    removed = 0
    for module in model.modules():
        removed += module.__dict__.pop("forward", None) is not None
        module.__dict__.pop(_SITE, None)
    return removed


# ================================================================= helpers

def _eps_of(module: nn.Module, default: float = 1e-6) -> float:
    for attr in ("variance_epsilon", "eps"):
        v = getattr(module, attr, None)
        if v is not None:
            return float(v)
    return default


def _linear_without_bias(module: nn.Module, attr: str) -> nn.Linear | None:
    sub = getattr(module, attr, None)
    return sub if isinstance(sub, nn.Linear) and sub.bias is None else None


def _first_present(module: nn.Module, attrs: tuple[str, ...]):
    """First truthy attribute among `attrs` (a module that defines none gives None)."""
    for a in attrs:
        v = getattr(module, a, None)
        if v:
            return v
    return None


def _rows(x: torch.Tensor) -> torch.Tensor:
    return x.reshape(-1, x.shape[-1])


def _project_rows(lin: nn.Linear, x2d: torch.Tensor, residual: torch.Tensor | None = None,
                  act: str | None = None) -> torch.Tensor:
    """lin(x2d) [+ residual] on the B200 kernels, regime by row count: the GEMV below
    FUSE_MIN_ROWS (residual in its epilogue), the tcgen05 GEMM above (bias, activation
    and residual in its epilogue)."""
    if x2d.shape[0] >= FUSE_MIN_ROWS or act is not None:
        return linear(x2d, lin.weight, lin.bias, act=act, residual=residual)
    if residual is not None:
        return linear_gemv_residual(x2d, lin.weight, residual, lin.bias, weights_ready=True)
    return linear_gemv(x2d, lin.weight, lin.bias, weights_ready=True)


# ============================================================ P5 SwiGLU MLP

@dataclass(frozen=True)
class SwiGLUSite:
    gate: nn.Module
    up: nn.Module
    down: nn.Module


def _match_swiglu(module: nn.Module) -> SwiGLUSite | None:
    """gate_proj / up_proj / down_proj bias-free Linears and an activation (act_fn or
    act) whose class name contains "silu" or "swish" (src/umic/integrate.py:33-41)."""
    linears = [_linear_without_bias(module, a) for a in ("gate_proj", "up_proj", "down_proj")]
    if any(lin is None for lin in linears):
        return None
    act = _first_present(module, ("act_fn", "act"))
    kind = type(act).__name__.lower() if act is not None else ""
    if "silu" not in kind and "swish" not in kind:
        return None
    return SwiGLUSite(*linears)


def swiglu(site: SwiGLUSite, x: torch.Tensor, residual: torch.Tensor | None = None):
    """down(silu(gate(x)) * up(x)) [+ residual] over the last dim of x: one dual-accumulator
    kernel for gate/up (tcgen05 GEMM, or the gated GEMV for decode rows), then the down
    projection with the residual add in its epilogue."""
    x2d = _rows(x)
    h = gate_silu_mul_nk(x2d, site.gate.weight, site.up.weight, weights_ready=True)
    out = _project_rows(site.down, h, None if residual is None else _rows(residual))
    return out.view(*x.shape[:-1], out.shape[-1])


def mlp_forward(mlp: Any, x: torch.Tensor, residual: torch.Tensor | None = None):
    """`swiglu` for any object carrying gate_proj / up_proj / down_proj (weights `[N, K]`)."""
    return swiglu(SwiGLUSite(mlp.gate_proj, mlp.up_proj, mlp.down_proj), x, residual)


def _swiglu_forward(self: nn.Module, x: torch.Tensor) -> torch.Tensor:
    return swiglu(self.__dict__[_SITE], x)


P5_SWIGLU = Motif("P5 gate_silu_mul MLP", _match_swiglu, _swiglu_forward)


def fuse_mlps(model: nn.Module, dry_run: bool = False) -> int:
    """Rebind every SwiGLU MLP (src/umic/integrate.py:58-77). Unlike the reference, rows
    below FUSE_MIN_ROWS do not fall back to cuBLAS: they take the gated GEMV."""
    return _rebind(model, P5_SWIGLU, dry_run)


# ============================================================= projections

def _projection_forward(self: nn.Linear, x: torch.Tensor) -> torch.Tensor:
    out = _project_rows(self, _rows(x))
    return out.view(*x.shape[:-1], out.shape[-1])


def _decode_projection_forward(self: nn.Linear, x: torch.Tensor) -> torch.Tensor:
    """The GEMV for decode rows; every other call keeps the Linear's own math."""
    x2d = _rows(x)
    if x2d.shape[0] >= FUSE_MIN_ROWS or not x2d.is_cuda or x2d.dtype != torch.bfloat16:
        return nn.functional.linear(x, self.weight, self.bias)
    out = linear_gemv(x2d, self.weight, self.bias, weights_ready=True)
    return out.view(*x.shape[:-1], out.shape[-1])


def fuse_linears(model: nn.Module, names: tuple[str, ...] = INEFFICIENT_LINEAR_NAMES,
                 dry_run: bool = False) -> int:
    """Rebind the nn.Linear modules whose attribute name is in `names`
    (src/umic/integrate.py:110-131): the GEMM at >= FUSE_MIN_ROWS rows, the GEMV below."""
    leaf_names = frozenset(names)
    return _rebind_named(model, f"projections {tuple(names)}", _projection_forward,
                         lambda leaf, m: isinstance(m, nn.Linear) and leaf in leaf_names,
                         dry_run)


def _rebind_named(model: nn.Module, label: str, forward: Callable[..., Any],
                  pred: Callable[[str, nn.Module], bool], dry_run: bool) -> int:
    """`_rebind` for a motif decided by the attribute name a module is reached under."""
    leaf = {id(m): name.rpartition(".")[2] for name, m in model.named_modules()}
    return _rebind(model, Motif(label, lambda m: True if pred(leaf[id(m)], m) else None, forward),
                   dry_run)


DECODE_GEMV = Motif("decode GEMV for the remaining Linears",
                    lambda m: True if isinstance(m, nn.Linear) and "forward" not in m.__dict__
                    else None,
                    _decode_projection_forward)


def fuse_decode_linears(model: nn.Module, dry_run: bool = False) -> int:
    """Route every not yet rebound nn.Linear to the GEMV for calls with fewer than
    FUSE_MIN_ROWS rows. Extends the reference, which left decode projections on cuBLAS
    (src/umic/integrate.py:27-30, 48-50)."""
    return _rebind(model, DECODE_GEMV, dry_run)


# =============================================================== RMSNorm

@dataclass(frozen=True)
class NormSite:
    eps: float
    # Euler-update epilogue (see `axpy_epilogue`): (base, alpha) while a flow step runs
    axpy: list = field(default_factory=list, compare=False)


def _match_rmsnorm(module: nn.Module) -> NormSite | None:
    """Class name containing "rmsnorm" with a 1-D weight (src/umic/integrate.py:144-167)."""
    w = getattr(module, "weight", None)
    if "rmsnorm" in type(module).__name__.lower() and isinstance(w, torch.Tensor) and w.dim() == 1:
        return NormSite(_eps_of(module))
    return None


def _rmsnorm_forward(self: nn.Module, x: torch.Tensor) -> torch.Tensor:
    site: NormSite = self.__dict__[_SITE]
    if site.axpy:
        base, alpha = site.axpy[-1]
        return rmsnorm_axpy(x, self.weight, site.eps, base, alpha)
    return rmsnorm(x, self.weight, site.eps)


RMSNORM = Motif("RMSNorm", _match_rmsnorm, _rmsnorm_forward)


def fuse_rmsnorms(model: nn.Module, dry_run: bool = False) -> int:
    """One kernel per RMSNorm-family module instead of the eager pow/mean/mul/cast
    chain (src/umic/integrate.py:134-167)."""
    return _rebind(model, RMSNORM, dry_run)


@contextlib.contextmanager
def axpy_epilogue(norm: nn.Module, base: torch.Tensor, alpha: float):
    """While active, the rebound RMSNorm `norm` returns base + alpha * norm(x) from the
    same single pass (umic_rmsnorm_axpy) instead of norm(x).

    This is the flow sampler's Euler update x <- x + dt * v fused into the kernel that
    produces v, when v is the action expert's final RMSNorm output (P9 ode_step of the
    reference's design, docs/260610_01_umic_design_ko.md:72, never built there). Raises
    if `norm` is not an RMSNorm rebound by `fuse_rmsnorms`."""
    site = _site(norm, NormSite)
    if site is None:
        raise ValueError("axpy_epilogue needs an RMSNorm rebound by fuse_rmsnorms")
    site.axpy.append((base, float(alpha)))
    try:
        yield
    finally:
        site.axpy.pop()


def has_axpy_epilogue(norm: nn.Module | None) -> bool:
    return norm is not None and _site(norm, NormSite) is not None


# ============================================= decoder layer: residual folds

@dataclass(frozen=True)
class LayerSite:
    post_norm: nn.Module


def _match_decoder_layer(module: nn.Module) -> LayerSite | None:
    """Pre-norm attention + MLP decoder layer (src/umic/integrate.py:170-177)."""
    need = ("input_layernorm", "post_attention_layernorm", "self_attn", "mlp")
    return LayerSite(module.post_attention_layernorm) if all(hasattr(module, a) for a in need) \
        else None


def _decoder_layer_forward(self: nn.Module, hidden_states: torch.Tensor,
                           position_embeddings=None, **kwargs) -> torch.Tensor:
    """stream -> norm -> attention; the attention residual add runs inside the
    post-attention RMSNorm (one kernel, two outputs: the MLP input and the new
    stream); the MLP residual add runs in the down projection's epilogue when the MLP
    is a rebound SwiGLU block (the reference kept both adds eager, integrate.py:180-209)."""
    site: LayerSite = self.__dict__[_SITE]
    attn_out = self.self_attn(hidden_states=self.input_layernorm(hidden_states),
                              position_embeddings=position_embeddings, **kwargs)[0]
    mlp_in, stream = add_rmsnorm(attn_out, hidden_states, site.post_norm.weight,
                                 _eps_of(site.post_norm))
    mlp_site = _site(self.mlp, SwiGLUSite)
    if mlp_site is not None:
        return swiglu(mlp_site, mlp_in, residual=stream)
    return stream + self.mlp(mlp_in)


DECODER_LAYER = Motif("decoder layer (add+RMSNorm residual fold)", _match_decoder_layer,
                      _decoder_layer_forward)


def fuse_add_rmsnorm(model: nn.Module, dry_run: bool = False) -> int:
    """Fold the decoder layers' residual adds into kernels that already read the
    operands (src/umic/integrate.py:212-231)."""
    return _rebind(model, DECODER_LAYER, dry_run)


# ============================================ text attention input path (f2)

def _match_qk_norm_attention(module: nn.Module):
    """q/k/v/o Linears, per-head q_norm / k_norm with 1-D weights, and the attributes the
    attention forward reads (Qwen3-style text attention)."""
    if not all(isinstance(getattr(module, a, None), nn.Linear)
               for a in ("q_proj", "k_proj", "v_proj", "o_proj")):
        return None
    for a in ("q_norm", "k_norm"):
        w = getattr(getattr(module, a, None), "weight", None)
        if not isinstance(w, torch.Tensor) or w.dim() != 1:
            return None
    if not all(hasattr(module, a) for a in ("head_dim", "scaling", "layer_idx", "config")):
        return None
    return True


def _kernel_covers(self, hidden_states: torch.Tensor, cos) -> bool:
    if cos is None or hidden_states.dim() != 3 or not hidden_states.is_cuda:
        return False
    if hidden_states.dtype != torch.bfloat16 or self.head_dim not in (64, 128, 256):
        return False
    if cos.dim() != 3 or cos.shape[-1] != self.head_dim:
        return False
    return not (torch.is_grad_enabled()
                and (hidden_states.requires_grad or self.q_proj.weight.requires_grad))


def _qkv_rows(self, x2d: torch.Tensor):
    """q, k, v projections: one three-matrix GEMV for decode rows; above FUSE_MIN_ROWS
    the tcgen05 GEMM for q and the model's own Linears for k and v (as the reference
    keeps them, src/umic/integrate.py:80-91)."""
    if x2d.shape[0] < FUSE_MIN_ROWS:
        from .kernels.linear import linear_gemv_multi

        lins = (self.q_proj, self.k_proj, self.v_proj)
        return linear_gemv_multi(x2d, [m.weight for m in lins], [m.bias for m in lins],
                                 weights_ready=True)
    return (linear(x2d, self.q_proj.weight, self.q_proj.bias),
            nn.functional.linear(x2d, self.k_proj.weight, self.k_proj.bias),
            nn.functional.linear(x2d, self.v_proj.weight, self.v_proj.bias))


def _qk_attention_forward(self, hidden_states, position_embeddings=None, attention_mask=None,
                          past_key_values=None, **kwargs):
    """Text attention whose input path is one kernel: after the projections,
    umic_qk_norm_rope_kv normalises q and k per head, rotates them and writes k and v
    into the in-place cache slots `InplaceLayer.reserve` hands out (no DynamicCache
    concatenation). The model's attention backend and o_proj follow. Layouts outside
    the kernel's coverage run the class forward."""
    cos = position_embeddings[0] if position_embeddings is not None else None
    if not _kernel_covers(self, hidden_states, cos):
        return type(self).forward(self, hidden_states, position_embeddings, attention_mask,
                                  past_key_values=past_key_values, **kwargs)
    out, probs = _qk_attention_core(self, hidden_states, position_embeddings, attention_mask,
                                    past_key_values, kwargs)
    return self.o_proj(out), probs


def _qk_attention_core(self, hidden_states, position_embeddings, attention_mask,
                       past_key_values, kwargs):
    """The fused attention up to o_proj: returns ([b, s, heads * head_dim] attention
    output, probabilities or None). The caller checked `_kernel_covers`."""
    from transformers.modeling_utils import ALL_ATTENTION_FUNCTIONS
    from transformers.models.qwen3_vl.modeling_qwen3_vl import eager_attention_forward

    from .cache import InplaceKVCache
    from .kernels.attention import qk_norm_rope_kv

    cos, sin = position_embeddings
    b, s, _ = hidden_states.shape
    d = self.head_dim
    q, k, v = (t.view(b, s, -1, d) for t in _qkv_rows(self, _rows(hidden_states)))
    norms = (self.q_norm.weight, self.k_norm.weight, _eps_of(self.q_norm), _eps_of(self.k_norm))
    if isinstance(past_key_values, InplaceKVCache):
        layer = past_key_values.layers[self.layer_idx]
        k_buf, v_buf, pos = layer.reserve(s)
        qk_norm_rope_kv(q, k, v, *norms, cos, sin, k_buf, v_buf, pos)
        keys, values = layer.keys, layer.values
    else:
        qk_norm_rope_kv(q, k, None, *norms, cos, sin)  # k normalised and rotated in place
        keys, values = k.transpose(1, 2), v.transpose(1, 2)
        if past_key_values is not None:
            keys, values = past_key_values.update(keys, values, self.layer_idx)
    backend = self.config._attn_implementation
    attend = gqa_sdpa_attention if backend == "sdpa" else \
        ALL_ATTENTION_FUNCTIONS.get_interface(backend, eager_attention_forward)
    out, probs = attend(self, q.transpose(1, 2), keys, values, attention_mask,
                        dropout=self.attention_dropout if self.training else 0.0,
                        scaling=self.scaling, **kwargs)
    return out.reshape(b, s, -1).contiguous(), probs


def gqa_sdpa_attention(module: nn.Module, query: torch.Tensor, key: torch.Tensor,
                       value: torch.Tensor, attention_mask: torch.Tensor | None,
                       dropout: float = 0.0, scaling: float | None = None,
                       is_causal: bool | None = None, **kwargs):
    """transformers' "sdpa" attention (its mask and causal rules) without the K/V head
    expansion transformers 5.x performs whenever a mask is passed (two ~0.4 GB copies per
    layer per flow step at the cfg5 shape): a boolean mask over few query rows per KV
    head (the flow expert's action tokens over the cached prefix) goes to the tcgen05
    kernel (kernels.attention.attention_rows), which reads the mask itself; anything else
    to SDPA with enable_gqa."""
    if attention_mask is not None and attention_mask.dim() == 4:
        attention_mask = attention_mask[..., : key.shape[-2]]
        rows_kernel_ok = (attention_mask.dtype == torch.bool and query.shape[2] > 1
                          and dropout == 0.0 and query.is_cuda and query.dtype == torch.bfloat16)
        if rows_kernel_ok:
            from .kernels.attention import attention_rows

            out = attention_rows(query, key, value, attention_mask,
                                 scaling if scaling is not None else query.shape[-1] ** -0.5)
            if out is not None:
                return out, None
    causal = is_causal if is_causal is not None else getattr(module, "is_causal", True)
    causal = bool(causal and attention_mask is None and query.shape[2] > 1)
    out = nn.functional.scaled_dot_product_attention(
        query, key, value, attn_mask=attention_mask, dropout_p=dropout, scale=scaling,
        is_causal=causal, enable_gqa=query.shape[1] != key.shape[1])
    return out.transpose(1, 2).contiguous(), None


QK_ATTENTION = Motif("attention input (q/k norm + RoPE + KV write)", _match_qk_norm_attention,
                     _qk_attention_forward)


def fuse_attention(model: nn.Module, dry_run: bool = False) -> int:
    """Rebind every Qwen3-style text attention so its input path is one kernel. No single
    reference counterpart: it merges the q/o-projection, RMSNorm, text-RoPE and
    in-place-cache patches (src/umic/integrate.py:98-167, 661-682; src/umic/cache.py:50-80)."""
    return _rebind(model, QK_ATTENTION, dry_run)


# ============================================================== LayerNorm

def _match_layernorm(module: nn.Module):
    """Last-dim affine nn.LayerNorm with a bias (src/umic/integrate.py:241-258)."""
    ok = (isinstance(module, nn.LayerNorm) and len(module.normalized_shape) == 1
          and module.weight is not None and module.bias is not None)
    return True if ok else None


def _layernorm_forward(self: nn.LayerNorm, x: torch.Tensor) -> torch.Tensor:
    return layernorm(x, self.weight, self.bias, self.eps)


LAYERNORM = Motif("LayerNorm", _match_layernorm, _layernorm_forward)


def fuse_layernorms(model: nn.Module, dry_run: bool = False) -> int:
    """One kernel per LayerNorm (src/umic/integrate.py:234-258)."""
    return _rebind(model, LAYERNORM, dry_run)


# ============================================================ ViT GELU MLP

_FC1_NAMES = ("fc1", "linear_fc1", "up_proj")
_FC2_NAMES = ("fc2", "linear_fc2", "down_proj")


@dataclass(frozen=True)
class GeluMLPSite:
    fc1: nn.Linear
    fc2: nn.Linear
    act: nn.Module
    gelu: str  # "gelu_tanh" or "gelu" (erf): the epilogue form
    fc2_on_gemm: bool = False


def _gelu_form(act) -> str | None:
    if act is None:
        return None
    cls = type(act).__name__.lower()
    if "gelu" not in cls and getattr(act, "__name__", "") != "gelu":
        return None
    return "gelu_tanh" if (getattr(act, "approximate", None) == "tanh" or "tanh" in cls) \
        else "gelu"


def _match_gelu_mlp(module: nn.Module) -> GeluMLPSite | None:
    """fc1 -> GELU -> fc2 without a gate, dimension preserving (fc1 in == fc2 out), so a
    ViT patch merger that changes width does not match (src/umic/integrate.py:266-289)."""
    def first_linear(names):
        for n in names:
            if isinstance(getattr(module, n, None), nn.Linear):
                return getattr(module, n)
        return None

    fc1, fc2 = first_linear(_FC1_NAMES), first_linear(_FC2_NAMES)
    if fc1 is None or fc2 is None or hasattr(module, "gate_proj"):
        return None
    if fc1.in_features != fc2.out_features:
        return None
    act = _first_present(module, ("act_fn", "act", "activation_fn"))
    form = _gelu_form(act)
    return None if form is None else GeluMLPSite(fc1, fc2, act, form)


def _gelu_mlp_forward(self: nn.Module, x: torch.Tensor) -> torch.Tensor:
    """fc1 with the module's own GELU (tanh or erf) in the GEMM epilogue -- the reference
    always used erf (linear.py:83-86) although the ViT's is tanh -- then fc2, on the GEMM
    when the site says so, else the Linear's own math. Decode-sized calls run eagerly."""
    site: GeluMLPSite = self.__dict__[_SITE]
    x2d = _rows(x)
    if x2d.shape[0] < FUSE_MIN_ROWS:
        return site.fc2(site.act(site.fc1(x)))
    h = linear(x2d, site.fc1.weight, site.fc1.bias, act=site.gelu)
    out = (linear(h, site.fc2.weight, site.fc2.bias) if site.fc2_on_gemm
           else nn.functional.linear(h, site.fc2.weight, site.fc2.bias))
    return out.view(*x.shape[:-1], out.shape[-1])


GELU_MLP = Motif("GELU MLP (fc1 + GELU epilogue)", _match_gelu_mlp, _gelu_mlp_forward)


def fuse_gelu_mlps(model: nn.Module, dry_run: bool = False, fc2_on_gemm: bool = False) -> int:
    """fc1 + GELU as one GEMM for every GELU MLP (src/umic/integrate.py:306-319);
    `fc2_on_gemm` also moves fc2 onto the tcgen05 GEMM."""
    def install(module, site):
        _install(module, _gelu_mlp_forward,
                 GeluMLPSite(site.fc1, site.fc2, site.act, site.gelu, fc2_on_gemm))

    return _rebind(model, GELU_MLP, dry_run, install)


# ========================================================== P10 patch embed

@dataclass(frozen=True)
class PatchEmbedSite:
    conv: nn.Module
    in_features: int


def _is_patchify_conv(module) -> bool:
    """A ConvNd whose stride equals its kernel, with no padding and one group: it never
    overlaps, so it is a Linear on each flattened patch (src/umic/integrate.py:322-340)."""
    return (isinstance(module, (nn.Conv1d, nn.Conv2d, nn.Conv3d)) and module.groups == 1
            and all(p == 0 for p in module.padding)
            and tuple(module.stride) == tuple(module.kernel_size))


def _match_patch_embed(module: nn.Module) -> PatchEmbedSite | None:
    """A module whose `.proj` is a patchify conv (src/umic/integrate.py:343-353)."""
    conv = getattr(module, "proj", None)
    if conv is None or not _is_patchify_conv(conv):
        return None
    return PatchEmbedSite(conv, conv.in_channels * math.prod(conv.kernel_size))


def _patch_embed_forward(self: nn.Module, hidden_states: torch.Tensor) -> torch.Tensor:
    """The conv as a GEMM on the flat patches, bias in the epilogue; the conv weight is
    viewed as [out, in_features] (K = 1176 at cfg3: the partial last k-block is read as
    zeros by TMA)."""
    site: PatchEmbedSite = self.__dict__[_SITE]
    w2d = site.conv.weight.view(site.conv.out_channels, site.in_features)
    patches = hidden_states.reshape(-1, site.in_features).to(w2d.dtype)
    if patches.is_cuda and patches.dtype == torch.bfloat16:
        return linear(patches, w2d, site.conv.bias)
    return nn.functional.linear(patches, w2d, site.conv.bias)


PATCH_EMBED = Motif("P10 patch embed conv -> GEMM", _match_patch_embed, _patch_embed_forward)


def fuse_patch_embed_linear(model: nn.Module, dry_run: bool = False) -> int:
    """Patchify ConvNd containers -> GEMM on a view of the conv weight
    (src/umic/integrate.py:363-389)."""
    return _rebind(model, PATCH_EMBED, dry_run)


# ================================================ packed ViT attention

@dataclass
class PackedAttentionSite:
    """Segment layout of the last cu_seqlens seen, keyed by its storage and version so
    an in-place update of the same tensor is noticed."""

    key: tuple = ()
    max_len: int = 0
    uniform_len: int = 0  # every segment this long, else 0

    def layout(self, cu_seqlens: torch.Tensor) -> tuple[int, int]:
        key = (cu_seqlens.data_ptr(), cu_seqlens._version, tuple(cu_seqlens.shape),
               cu_seqlens.device)
        if key != self.key:
            lens = (cu_seqlens[1:] - cu_seqlens[:-1]).to(torch.int64)
            lo, hi = (int(v) for v in torch.stack((lens.min(), lens.max())).tolist())
            self.key, self.max_len = key, hi
            self.uniform_len = hi if (lo == hi and hi > 0) else 0
        return self.max_len, self.uniform_len


def _match_packed_attention(module: nn.Module) -> PackedAttentionSite | None:
    """qkv (a Linear) + proj + num_heads + scaling, and a forward taking cu_seqlens
    (src/umic/integrate.py:392-407)."""
    if not all(hasattr(module, a) for a in ("qkv", "proj", "num_heads", "scaling")):
        return None
    if not isinstance(module.qkv, nn.Linear):
        return None
    try:
        params = inspect.signature(type(module).forward).parameters
    except (TypeError, ValueError):
        return None
    return PackedAttentionSite() if "cu_seqlens" in params else None


def _packed_attention_forward(self: nn.Module, hidden_states: torch.Tensor,
                              cu_seqlens: torch.Tensor, rotary_pos_emb=None,
                              position_embeddings=None, **kwargs) -> torch.Tensor:
    """All images in one call: q/k rotated in place (the module-global vision RoPE),
    then, when every image has the same patch count, the tcgen05 attention over
    [images, heads, patches, head_dim] views of the packed qkv; otherwise torch's
    varlen flash attention over cu_seqlens (src/umic/integrate.py:410-458)."""
    import transformers.models.qwen3_vl.modeling_qwen3_vl as hf

    site: PackedAttentionSite = self.__dict__[_SITE]
    n_tok = hidden_states.shape[0]
    q, k, v = self.qkv(hidden_states).view(n_tok, 3, self.num_heads, -1).unbind(1)
    q, k = hf.apply_rotary_pos_emb_vision(q, k, *position_embeddings)
    max_len, per_image = site.layout(cu_seqlens)
    if per_image and q.is_cuda and q.dtype == torch.bfloat16:
        from .kernels.attention import attention_rows

        imgs, hd = n_tok // per_image, q.shape[-1]
        q4, k4, v4 = (t.view(imgs, per_image, self.num_heads, hd).transpose(1, 2)
                      for t in (q, k, v))
        out = attention_rows(q4, k4, v4, None, self.scaling)
        if out is not None:
            return self.proj(out.reshape(n_tok, -1))
    out = torch.ops.aten._flash_attention_forward(q, k, v, cu_seqlens, cu_seqlens, max_len,
                                                  max_len, 0.0, False, False,
                                                  scale=self.scaling)[0]
    return self.proj(out.reshape(n_tok, -1))


PACKED_ATTENTION = Motif("packed varlen ViT attention", _match_packed_attention,
                         _packed_attention_forward)


def fuse_vision_attention_varlen(model: nn.Module, dry_run: bool = False) -> int:
    """One packed attention call per ViT attention module instead of split / per-image /
    cat (src/umic/integrate.py:461-478)."""
    return _rebind(model, PACKED_ATTENTION, dry_run)


# ============================================== ViT encoder pipeline forward

@dataclass
class EncoderSite:
    taps: dict  # block index -> its deepstack merger
    grid_key: tuple = ()
    consts: tuple = ()  # (pos_embeds, (cos, sin), cu_seqlens) for grid_key


def _match_deepstack_encoder(module: nn.Module) -> EncoderSite | None:
    """A grid_thw-driven ViT: LayerNorm pre-norm blocks (norm1 / norm2 / attn / mlp), a
    final merger (norm + fc1 / act / fc2), patch embed and deepstack taps
    (src/umic/integrate.py:481-506)."""
    blocks = getattr(module, "blocks", None)
    if not blocks:
        return None
    first = blocks[0]
    if not all(hasattr(first, a) for a in ("norm1", "norm2", "attn", "mlp")):
        return None
    if not (isinstance(first.norm1, nn.LayerNorm) and isinstance(first.norm2, nn.LayerNorm)):
        return None
    merger = getattr(module, "merger", None)
    merger_attrs = ("norm", "linear_fc1", "act_fn", "linear_fc2", "use_postshuffle_norm",
                    "hidden_size")
    if merger is None or not all(hasattr(merger, a) for a in merger_attrs):
        return None
    enc_attrs = ("patch_embed", "deepstack_merger_list", "deepstack_visual_indexes",
                 "fast_pos_embed_interpolate", "rot_pos_emb")
    if not all(hasattr(module, a) for a in enc_attrs):
        return None
    return EncoderSite({})


def _grid_constants(enc: nn.Module, grid_thw: torch.Tensor, n_tok: int) -> tuple:
    """Position embeddings, RoPE tables and segment offsets of one image grid; they depend
    on grid_thw only, so the pipeline computes them once per distinct grid."""
    pos = enc.fast_pos_embed_interpolate(grid_thw)
    freqs = enc.rot_pos_emb(grid_thw).reshape(n_tok, -1)
    angles = torch.cat((freqs, freqs), dim=-1)
    per_image = (grid_thw[:, 1] * grid_thw[:, 2]).repeat_interleave(grid_thw[:, 0])
    ends = per_image.cumsum(0, dtype=torch.int32)
    cu = torch.cat((ends.new_zeros(1), ends))
    return pos.detach(), (angles.cos().contiguous(), angles.sin().contiguous()), cu


def _layernorm_folding(norm: nn.LayerNorm, stream: torch.Tensor, pending):
    """norm(stream + pending) and the new stream; the add runs inside the LayerNorm
    kernel when a pending branch output exists."""
    if pending is None:
        return norm(stream), stream
    return add_layernorm(pending, stream, norm.weight, norm.bias, norm.eps)


def _encoder_forward(self: nn.Module, hidden_states: torch.Tensor, grid_thw: torch.Tensor,
                     **kwargs):
    """The ViT forward with every residual add that feeds a LayerNorm folded into that
    LayerNorm's kernel: a block's MLP output stays pending and is added by the next
    block's norm1 (or by the merger's norm after the last block); only the deepstack
    taps, whose mergers normalise a 4x wider view, materialise the sum
    (src/umic/integrate.py:509-611, 24 of 27 adds at cfg3). Grid constants are cached
    per grid. Returns transformers 5.5's BaseModelOutputWithDeepstackFeatures."""
    from transformers.models.qwen3_vl.modeling_qwen3_vl import (
        BaseModelOutputWithDeepstackFeatures)

    site: EncoderSite = self.__dict__[_SITE]
    x = self.patch_embed(hidden_states)
    n_tok = x.shape[0]
    key = tuple(grid_thw.flatten().tolist())
    if key != site.grid_key:
        site.grid_key, site.consts = key, _grid_constants(self, grid_thw, n_tok)
    pos, rope_tables, cu_seqlens = site.consts
    stream = (x + pos).reshape(n_tok, -1)
    pending = None
    features = []
    for i, blk in enumerate(self.blocks):
        h, stream = _layernorm_folding(blk.norm1, stream, pending)
        attn_out = blk.attn(h, cu_seqlens=cu_seqlens, position_embeddings=rope_tables, **kwargs)
        h, stream = add_layernorm(attn_out, stream, blk.norm2.weight, blk.norm2.bias,
                                  blk.norm2.eps)
        pending = blk.mlp(h)
        tap = site.taps.get(i)
        if tap is not None:
            stream, pending = stream + pending, None
            features.append(tap(stream))
    merger = self.merger
    if pending is not None and not merger.use_postshuffle_norm:
        h, stream = _layernorm_folding(merger.norm, stream, pending)
        pooled = merger.linear_fc2(merger.act_fn(merger.linear_fc1(h.view(-1,
                                                                          merger.hidden_size))))
    else:
        if pending is not None:
            stream = stream + pending
        pooled = merger(stream)
    return BaseModelOutputWithDeepstackFeatures(last_hidden_state=stream, pooler_output=pooled,
                                                deepstack_features=features)


def _install_encoder(module: nn.Module, site: EncoderSite) -> None:
    taps = {idx: module.deepstack_merger_list[j]
            for j, idx in enumerate(module.deepstack_visual_indexes)}
    _install(module, _encoder_forward, EncoderSite(taps))


VIT_ENCODER = Motif("ViT encoder pipeline", _match_deepstack_encoder, _encoder_forward)


def fuse_vision_encoder_pipeline(model: nn.Module, dry_run: bool = False) -> int:
    """The grid-cached, residual-folding ViT forward (src/umic/integrate.py:614-638). It
    calls patch_embed / attn / mlp as submodules, so it composes with their own patches."""
    return _rebind(model, VIT_ENCODER, dry_run, _install_encoder)


# ============================================= module-global RoPE functions

def _swap_hf_function(attr: str, make: Callable[[Callable], Callable]) -> bool:
    """Replace transformers' qwen3_vl module-level `attr` by make(original), once."""
    try:
        import transformers.models.qwen3_vl.modeling_qwen3_vl as hf
    except ImportError:
        logger.warning("qwen3_vl modeling module not found; %s left as is", attr)
        return False
    current = getattr(hf, attr)
    if getattr(current, "_umic_original", None) is None:
        fused = make(current)
        fused._umic_fused = True
        fused._umic_original = current
        setattr(hf, attr, fused)
        logger.info("%s -> in-place B200 RoPE kernel", attr)
    return True


def fuse_vision_rope() -> bool:
    """HF apply_rotary_pos_emb_vision -> the in-place kernel (src/umic/integrate.py:641-658)."""
    return _swap_hf_function("apply_rotary_pos_emb_vision", _rope.make_vision_rope)


def fuse_text_rope() -> bool:
    """HF apply_rotary_pos_emb -> the in-place kernel; layouts it does not cover call the
    original (src/umic/integrate.py:661-682)."""
    return _swap_hf_function("apply_rotary_pos_emb", _rope.make_text_rope)


def unfuse_rope() -> None:
    """Put transformers' original RoPE functions back."""
    import transformers.models.qwen3_vl.modeling_qwen3_vl as hf

    for attr in ("apply_rotary_pos_emb", "apply_rotary_pos_emb_vision"):
        original = getattr(getattr(hf, attr), "_umic_original", None)
        if original is not None:
            setattr(hf, attr, original)


# =================================================== hooks on the ViT / caches

class _CastStreamHook:
    """Forward pre-hook: hands the block its hidden_states (first positional argument or
    keyword) in `dtype`."""

    def __init__(self, dtype: torch.dtype):
        self.dtype = dtype

    def __call__(self, module, args, kwargs):
        if args:
            hs = args[0]
            if isinstance(hs, torch.Tensor) and hs.dtype != self.dtype:
                return (hs.to(self.dtype), *args[1:]), kwargs
            return None
        hs = kwargs.get("hidden_states")
        if isinstance(hs, torch.Tensor) and hs.dtype != self.dtype:
            return args, {**kwargs, "hidden_states": hs.to(self.dtype)}
        return None


def fuse_bf16_residual(visual: nn.Module, dtype: torch.dtype = torch.bfloat16) -> bool:
    """Keep the ViT residual stream in bf16 from the first block on: fp32 position
    embeddings otherwise promote it (src/umic/integrate.py:685-712)."""
    blocks = getattr(visual, "blocks", None)
    if not blocks:
        return False
    blocks[0].register_forward_pre_hook(_CastStreamHook(dtype), with_kwargs=True)
    return True


class _RepeatCacheAdapter:
    """Forward pre-hook that swaps a caller's DynamicCache for an InplaceKVCache.

    The first call that brings a fully populated DynamicCache allocates the in-place
    copy (prefix + max(new tokens, hint) + margin slots); later calls with the same
    source only move the write pointer back to the source's length, which is the
    caller's own crop, in O(1). The source is tracked by weak reference, so a new cache
    that happens to reuse a collected object's id is never mistaken for the old one."""

    def __init__(self, extra_tokens_hint: int):
        self.hint = extra_tokens_hint
        self.source = None  # weakref to the DynamicCache last converted
        self.inplace = None

    def __call__(self, module, args, kwargs):
        import weakref

        from transformers.cache_utils import DynamicCache

        from .cache import InplaceKVCache

        src = kwargs.get("past_key_values")
        if not isinstance(src, DynamicCache) or isinstance(src, InplaceKVCache):
            return None
        layers = getattr(src, "layers", None)
        if not layers or any(getattr(l, "keys", None) is None for l in layers):
            return None  # generate() makes lazy layers before the prefill fills them
        if self.source is None or self.source() is not src:
            embeds = kwargs.get("inputs_embeds")
            new = 0 if embeds is None else embeds.shape[1]
            self.inplace = InplaceKVCache.from_dynamic(src, extra_tokens=max(new, self.hint))
            self.source = weakref.ref(src)
        self.inplace.crop(src.get_seq_length())
        return args, {**kwargs, "past_key_values": self.inplace}


def fuse_repeat_cache(repeat_module: nn.Module, extra_tokens_hint: int = 64) -> None:
    """Serve `repeat_module`'s append-then-crop loop (the flow expert's steps over a
    shared prefix) from an in-place KV cache (src/umic/integrate.py:715-756)."""
    repeat_module.register_forward_pre_hook(_RepeatCacheAdapter(extra_tokens_hint),
                                            with_kwargs=True)
