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
    epilogue (the reference's epilogue was erf-only, so it kept them on cuBLAS), and
    the ViT attention's qkv projection runs on the same GEMM;
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


# Where the LM trunk may sit under model.vlm, in lookup order: (module to return, module
# that must hold the decoder `layers`), both as attribute paths relative to model.vlm.
# The first three pairs are the reference's lookup (src/umic/optimize.py:75-89); the
# last covers transformers 5.x, whose VLM keeps the text model at .model.language_model.
_LM_CANDIDATES = (
    ("language_model", "language_model"),
    ("language_model", "language_model.model"),
    ("model", "model"),
    ("model", "model.model"),
    ("language_model.language_model", "language_model.language_model"),
    ("model.language_model", "model.language_model"),
)
_VISUAL_PATHS = ("visual", "model.visual")


def _at(root, path: str):
    obj = root
    for attr in path.split("."):
        obj = getattr(obj, attr, None)
        if obj is None:
            return None
    return obj


def find_lm_module(model: nn.Module) -> nn.Module | None:
    """The LM trunk under model.vlm: the first candidate of _LM_CANDIDATES whose holder
    has decoder layers, or None."""
    vlm = getattr(model, "vlm", None)
    if vlm is None:
        return None
    for ret, holder in _LM_CANDIDATES:
        if hasattr(_at(vlm, holder), "layers"):
            return _at(vlm, ret)
    return None


def find_visual(model: nn.Module) -> nn.Module | None:
    """The vision tower under model.vlm (transformers 4.x or 5.x layout), or None."""
    vlm = getattr(model, "vlm", None)
    if vlm is None:
        return None
    return next((v for v in (_at(vlm, p) for p in _VISUAL_PATHS) if v is not None), None)


def _lm_phase(lm: nn.Module, cfg: UmicConfig, report: dict, prefix: str) -> None:
    from . import integrate

    steps = (
        (cfg.mlp_fusion, "mlp", integrate.fuse_mlps),
        (cfg.linear_fusion, "linear", integrate.fuse_linears),
        (cfg.norm_fusion, "rmsnorm", integrate.fuse_rmsnorms),
        (cfg.add_rmsnorm_fusion, "add_rmsnorm", integrate.fuse_add_rmsnorm),
        (cfg.attention_fusion, "attention", integrate.fuse_attention),
    )
    for enabled, what, fuse in steps:
        if enabled:
            report[f"{prefix}_{what}_fused"] = fuse(lm)


def _vision_phase(visual: nn.Module, cfg: UmicConfig, report: dict) -> None:
    from . import integrate

    report["ve_layernorm_fused"] = integrate.fuse_layernorms(visual)
    report["ve_rope_fused"] = integrate.fuse_vision_rope()
    report["ve_bf16_residual"] = integrate.fuse_bf16_residual(visual)
    report["ve_patch_embed_fused"] = integrate.fuse_patch_embed_linear(visual)
    report["ve_attn_varlen_fused"] = integrate.fuse_vision_attention_varlen(visual)
    report["ve_pipeline_fused"] = integrate.fuse_vision_encoder_pipeline(visual)
    if cfg.vision_gemm_fusion:
        # fc1 with the tanh-GELU in the GEMM epilogue (the reference's epilogue was erf
        # only, so it left the ViT MLPs on cuBLAS, src/umic/integrate.py:93-95), and the
        # attention's qkv projection with its bias in the epilogue (the site the reference
        # measured its own kernel winning, 1.23 vs 2.22 ms, but left off by default).
        # fc2 and proj (N = 1280: five column tiles for 74 CTA pairs) stay on cuBLAS,
        # which is faster at that width.
        report["ve_gelu_mlp_fused"] = integrate.fuse_gelu_mlps(visual)
        report["ve_linear_fused"] = integrate.fuse_linears(visual,
                                                           names=integrate.VIT_LINEAR_NAMES)


def _expert_phase(expert: nn.Module, cfg: UmicConfig, report: dict) -> None:
    from . import integrate

    # 64 action tokens per episode and step (>= FUSE_MIN_ROWS): the expert takes the
    # LM's GEMMs too; the reference fused only its norms and its cache.
    if cfg.mlp_fusion:
        report["expert_mlp_fused"] = integrate.fuse_mlps(expert)
    if cfg.linear_fusion:
        report["expert_linear_fused"] = integrate.fuse_linears(expert)
    if cfg.attention_fusion:
        report["expert_attention_fused"] = integrate.fuse_attention(expert)
    if cfg.flow_cache:
        integrate.fuse_repeat_cache(expert)
        report["flow_cache_hook"] = True
        if cfg.norm_fusion:
            report["expert_rmsnorm_fused"] = integrate.fuse_rmsnorms(expert)
        if cfg.add_rmsnorm_fusion:
            report["expert_add_rmsnorm_fused"] = integrate.fuse_add_rmsnorm(expert)


def _decode_phase(model: nn.Module, lm, expert, cfg: UmicConfig, report: dict) -> None:
    from . import integrate

    vlm = getattr(model, "vlm", None)
    if cfg.decode_gemv:
        head = getattr(vlm, "lm_head", None)
        roots = [lm, head if isinstance(head, nn.Linear) else None, expert]
        report["decode_gemv_fused"] = sum(integrate.fuse_decode_linears(r) for r in roots
                                          if r is not None)
    if vlm is None:
        return
    if cfg.decode_graph:
        from .graph import fuse_decode_graph

        model._umic_decode_runner = fuse_decode_graph(vlm, max_new_tokens=cfg.max_new_tokens)
        report["decode_graph"] = True
    elif cfg.decode_cache:
        integrate.fuse_repeat_cache(vlm, extra_tokens_hint=128)
        report["decode_cache_hook"] = True


def apply(model: nn.Module, config: UmicConfig | None = None) -> dict:
    """Rebind every configured motif of `model` in place and return the report of match
    counts and flags (src/umic/optimize.py:92-168). Phases, in the reference's order:
    LM trunk, text RoPE, vision tower, action expert, decode (GEMV + graphs)."""
    from . import integrate

    cfg = config or UmicConfig()
    report: dict[str, object] = {}
    lm = find_lm_module(model)
    if lm is None:
        logger.warning("umic_b200.apply: no LM trunk under model.vlm; LM fusions skipped")
    else:
        _lm_phase(lm, cfg, report, "lm")
    if cfg.text_rope_fusion:
        report["text_rope_fused"] = integrate.fuse_text_rope()
    visual = find_visual(model)
    if cfg.vision_fusion and visual is not None:
        _vision_phase(visual, cfg, report)
    expert = getattr(model, "expert", None)
    if expert is not None:
        _expert_phase(expert, cfg, report)
    _decode_phase(model, lm, expert, cfg, report)
    if cfg.adaptive_flow:
        logger.warning("adaptive_flow is an opt-in approximation of the reference's flow "
                       "sampler (src/umic/diffusion.py); it is not part of this build")
        report["adaptive_flow"] = False
    logger.info("umic_b200.apply report: %s", report)
    return report
