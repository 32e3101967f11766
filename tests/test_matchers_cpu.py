"""Drop-in boundary on CPU: the structural matchers find exactly what the
reference's matchers find (counts recorded from the reference by
tests/golden/make_golden.py), and apply() keeps the reference's config / report
contract. Patching needs no GPU; nothing here runs a kernel."""

import dataclasses
import json
from pathlib import Path

import pytest
import torch
from torch import nn

from umic_b200 import UmicConfig, apply, integrate
from umic_b200.workloads import AlpamayoStandIn, tiny_qwen3vl_configs

COUNTS = json.loads((Path(__file__).resolve().parent / "golden" / "matcher_counts.json")
                    .read_text())

# src/umic/optimize.py:62-72 of the reference
REFERENCE_CONFIG_FIELDS = {
    "mlp_fusion": True, "linear_fusion": True, "norm_fusion": True, "add_rmsnorm_fusion": True,
    "text_rope_fusion": True, "vision_fusion": True, "flow_cache": True, "decode_cache": True,
    "decode_graph": True, "adaptive_flow": False, "max_new_tokens": 96,
}


def _tiny(name):
    from transformers import Qwen3VLConfig
    from transformers.models.qwen3_vl.modeling_qwen3_vl import Qwen3VLForConditionalGeneration

    tc, vc = tiny_qwen3vl_configs()[name]
    torch.manual_seed(0)
    return Qwen3VLForConditionalGeneration(Qwen3VLConfig(text_config=tc, vision_config=vc))


@pytest.mark.parametrize("name", sorted(COUNTS))
def test_dry_run_counts_match_reference(name):
    model = _tiny(name)
    lm, vis = model.model.language_model, model.model.visual
    got = {
        "fuse_mlps": integrate.fuse_mlps(lm, dry_run=True),
        "fuse_linears": integrate.fuse_linears(lm, dry_run=True),
        "fuse_rmsnorms": integrate.fuse_rmsnorms(lm, dry_run=True),
        "fuse_add_rmsnorm": integrate.fuse_add_rmsnorm(lm, dry_run=True),
        "fuse_layernorms": integrate.fuse_layernorms(vis, dry_run=True),
        "fuse_patch_embed_linear": integrate.fuse_patch_embed_linear(vis, dry_run=True),
        "fuse_vision_attention_varlen": integrate.fuse_vision_attention_varlen(vis, dry_run=True),
        "fuse_vision_encoder_pipeline": integrate.fuse_vision_encoder_pipeline(vis, dry_run=True),
        "fuse_gelu_mlps": integrate.fuse_gelu_mlps(vis, dry_run=True),
        "fuse_mlps_whole_model": integrate.fuse_mlps(model, dry_run=True),
        "fuse_rmsnorms_whole_model": integrate.fuse_rmsnorms(model, dry_run=True),
    }
    assert got == COUNTS[name]
    # dry_run patches nothing
    assert not any("forward" in m.__dict__ for m in model.modules())


def test_config_is_a_superset_of_the_reference():
    fields = {f.name: f.default for f in dataclasses.fields(UmicConfig)}
    for k, v in REFERENCE_CONFIG_FIELDS.items():
        assert fields[k] == v


def test_apply_report_and_patching():
    model = AlpamayoStandIn(_tiny("t2_v4"))
    try:
        report = apply(model)
        assert report["lm_mlp_fused"] == 2 and report["lm_linear_fused"] == 4
        assert report["lm_rmsnorm_fused"] == 9 and report["lm_add_rmsnorm_fused"] == 2
        assert report["lm_attention_fused"] == 2
        assert report["text_rope_fused"] is True and report["decode_graph"] is True
        assert report["ve_layernorm_fused"] == 11 and report["ve_pipeline_fused"] == 1
        assert report["ve_patch_embed_fused"] == 1 and report["ve_attn_varlen_fused"] == 4
        lm = model.vlm.model.language_model
        assert lm.layers[0].mlp.forward.__func__ is integrate._swiglu_forward
        assert lm.layers[0].self_attn.q_proj.forward.__func__ is integrate._projection_forward
        assert lm.layers[0].input_layernorm.forward.__func__ is integrate._rmsnorm_forward
        assert isinstance(lm.layers[0].mlp._umic_site, integrate.SwiGLUSite)
        assert lm.layers[0].mlp._umic_site.gate is lm.layers[0].mlp.gate_proj
        import transformers.models.qwen3_vl.modeling_qwen3_vl as mod
        assert getattr(mod.apply_rotary_pos_emb, "_umic_fused", False)
        # weights shared, never copied
        w = lm.layers[0].mlp.gate_proj.weight
        assert w.data_ptr() == lm.layers[0].mlp.gate_proj.weight.data_ptr()
    finally:
        integrate.unfuse_rope()
        integrate.unfuse_mlps(model)
    assert not any("forward" in m.__dict__ or "_umic_site" in m.__dict__
                   for m in model.modules())


def test_nothing_matches_is_a_noop():
    class Plain(nn.Module):
        def __init__(self):
            super().__init__()
            self.fc = nn.Linear(4, 4)

    model = Plain()
    report = apply(model, UmicConfig(text_rope_fusion=False))
    assert report == {"decode_gemv_fused": 0}
    assert "forward" not in model.fc.__dict__


def test_patched_text_rope_falls_back_for_unsupported_layouts():
    """CPU tensors and unsqueeze_dim != 1 go to the original function, called with the
    transformers 5.x keyword signature (the reference passed 6 positional args)."""
    import transformers.models.qwen3_vl.modeling_qwen3_vl as mod

    orig = mod.apply_rotary_pos_emb
    try:
        assert integrate.fuse_text_rope()
        q = torch.randn(1, 2, 5, 16)
        k = torch.randn(1, 1, 5, 16)
        cos, sin = torch.randn(1, 5, 16), torch.randn(1, 5, 16)
        out = mod.apply_rotary_pos_emb(q, k, cos, sin)
        ref = orig(q, k, cos, sin)
        assert torch.equal(out[0], ref[0]) and torch.equal(out[1], ref[1])
    finally:
        integrate.unfuse_rope()
    assert mod.apply_rotary_pos_emb is orig
