"""One-call application: `umic_b200.apply(model, UmicConfig)`.

Mirrors src/umic/optimize.py of soonhong99/umic-alpamayo: same UmicConfig
fields and defaults, same report keys, same order of patches, and the same
rule that a model where nothing matches is left unchanged (no error).
Additions, on by default and reported:
  * attention_fusion: the text attention input path (projections, per-head
    q/k RMSNorm, RoPE, KV-cache write) runs as one kernel after the projections;
  * decode_gemv: every remaining LM / expert Linear runs the GEMV kernel when
    it sees fewer than FUSE_MIN_ROWS rows (the reference left those on cuBLAS);
  * vision_gemm_fusion: the ViT MLPs run fc1 with the tanh-GELU in the GEMM
    epilogue (the reference's epilogue was erf-only, so it kept them on cuBLAS);
  * the expert's MLPs and q/o projections take the same GEMMs as the LM;
  * the LM / expert lookups also accept the transformers 5.x layout, where the
    VLM holds its language model and vision tower under `.model`.
"""

from __future__ import annotations

import dataclasses
import logging

from torch import nn

logger = logging.getLogger(__name__)


@dataclasses.dataclass
class UmicConfig:
    """Which optimizations to apply (defaults: the reference's adopted set,
    src/umic/optimize.py:34-72, plus the additions listed above)."""

    mlp_fusion: bool = True
    linear_fusion: bool = True
    norm_fusion: bool = True
    add_rmsnorm_fusion: bool = True
    text_rope_fusion: bool = True
    vision_fusion: bool = True
    flow_cache: bool = True
    decode_cache: bool = True
    decode_graph: bool = True
    adaptive_flow: bool = False
    max_new_tokens: int = 96
    decode_gemv: bool = True
    attention_fusion: bool = True
    vision_gemm_fusion: bool = True


def _has_layers(m) -> bool:
    return m is not None and hasattr(m, "layers")


def find_lm_module(model: nn.Module) -> nn.Module | None:
    """The LM trunk under model.vlm (src/umic/optimize.py:75-89), also looking one
    level deeper (vlm.model.language_model) for transformers 5.x."""
    vlm = getattr(model, "vlm", None)
    if vlm is None:
        return None
    for attr in ("language_model", "model"):
        cand = getattr(vlm, attr, None)
        if cand is None:
            continue
        if _has_layers(cand):
            return cand
        for sub_attr in ("model", "language_model"):
            sub = getattr(cand, sub_attr, None)
            if _has_layers(sub):
                return cand if sub_attr == "model" else sub
    return None


def find_visual(model: nn.Module) -> nn.Module | None:
    vlm = getattr(model, "vlm", None)
    if vlm is None:
        return None
    vis = getattr(vlm, "visual", None)
    if vis is None:
        vis = getattr(getattr(vlm, "model", None), "visual", None)
    return vis


def apply(model: nn.Module, config: UmicConfig | None = None) -> dict:
    """Patch all configured optimizations into `model`, in place; returns a report
    of match counts / flags (src/umic/optimize.py:92-168)."""
    from . import integrate

    cfg = config or UmicConfig()
    report: dict[str, object] = {}

    lm = find_lm_module(model)
    if lm is None:
        logger.warning("umic_b200.apply: no LM trunk found under model.vlm - LM fusions skipped")
    if lm is not None:
        if cfg.mlp_fusion:
            report["lm_mlp_fused"] = integrate.fuse_mlps(lm)
        if cfg.linear_fusion:
            report["lm_linear_fused"] = integrate.fuse_linears(lm)
        if cfg.norm_fusion:
            report["lm_rmsnorm_fused"] = integrate.fuse_rmsnorms(lm)
        if cfg.add_rmsnorm_fusion:
            report["lm_add_rmsnorm_fused"] = integrate.fuse_add_rmsnorm(lm)
        if cfg.attention_fusion:
            report["lm_attention_fused"] = integrate.fuse_attention(lm)

    if cfg.text_rope_fusion:
        report["text_rope_fused"] = integrate.fuse_text_rope()

    visual = find_visual(model)
    if cfg.vision_fusion and visual is not None:
        report["ve_layernorm_fused"] = integrate.fuse_layernorms(visual)
        report["ve_rope_fused"] = integrate.fuse_vision_rope()
        report["ve_bf16_residual"] = integrate.fuse_bf16_residual(visual)
        report["ve_patch_embed_fused"] = integrate.fuse_patch_embed_linear(visual)
        report["ve_attn_varlen_fused"] = integrate.fuse_vision_attention_varlen(visual)
        report["ve_pipeline_fused"] = integrate.fuse_vision_encoder_pipeline(visual)
        if cfg.vision_gemm_fusion:
            # fc1 + tanh-GELU in one GEMM epilogue (the reference left the ViT MLPs on
            # cuBLAS because its epilogue was erf-GELU, src/umic/integrate.py:93-95)
            report["ve_gelu_mlp_fused"] = integrate.fuse_gelu_mlps(visual)

    expert = getattr(model, "expert", None)
    if expert is not None:
        # The expert's flow step runs 64 action tokens per episode (>= FUSE_MIN_ROWS),
        # so its MLPs and q/o projections take the same GEMMs as the LM (the
        # reference fused only its norms).
        if cfg.mlp_fusion:
            report["expert_mlp_fused"] = integrate.fuse_mlps(expert)
        if cfg.linear_fusion:
            report["expert_linear_fused"] = integrate.fuse_linears(expert)
        if cfg.attention_fusion:
            report["expert_attention_fused"] = integrate.fuse_attention(expert)
    if cfg.flow_cache and expert is not None:
        integrate.fuse_repeat_cache(expert)
        report["flow_cache_hook"] = True
        if cfg.norm_fusion:
            report["expert_rmsnorm_fused"] = integrate.fuse_rmsnorms(expert)
        if cfg.add_rmsnorm_fusion:
            report["expert_add_rmsnorm_fused"] = integrate.fuse_add_rmsnorm(expert)

    vlm = getattr(model, "vlm", None)
    if cfg.decode_gemv:
        n = 0
        if lm is not None:
            n += integrate.fuse_decode_linears(lm)
        head = getattr(vlm, "lm_head", None) if vlm is not None else None
        if isinstance(head, nn.Linear) and "forward" not in head.__dict__:
            n += integrate.fuse_decode_linears(head)
        if expert is not None:
            n += integrate.fuse_decode_linears(expert)
        report["decode_gemv_fused"] = n

    if vlm is not None:
        if cfg.decode_graph:
            from .graph import fuse_decode_graph

            model._umic_decode_runner = fuse_decode_graph(vlm, max_new_tokens=cfg.max_new_tokens)
            report["decode_graph"] = True
        elif cfg.decode_cache:
            integrate.fuse_repeat_cache(vlm, extra_tokens_hint=128)
            report["decode_cache_hook"] = True

    if cfg.adaptive_flow:
        logger.warning("adaptive_flow is an opt-in approximation of the reference's flow "
                       "sampler (src/umic/diffusion.py); it is not part of this build")
        report["adaptive_flow"] = False

    logger.info("umic_b200.apply report: %s", report)
    return report
