"""Pins the CPU oracle to the reference: golden vectors produced by the reference's
own Triton kernels (CPU interpreter), its eager CPU path, the HF eager functions
it patches, and its KV-cache class (tests/golden/make_golden.py)."""

from pathlib import Path

import pytest
import torch

import oracle

GOLDEN = Path(__file__).resolve().parent / "golden" / "reference_vectors.pt"


@pytest.fixture(scope="module")
def gv():
    return torch.load(GOLDEN, weights_only=False)


def _trunc_bf16(t: torch.Tensor) -> torch.Tensor:
    """fp32 -> bf16 by truncation: how Triton's CPU interpreter (which produced the
    reference-kernel vectors) casts; on a GPU the same kernels round to nearest."""
    i = t.float().contiguous().view(torch.int32)
    return (i & ~0xFFFF).view(torch.float32)


def _same_as_interpreted_kernel(oracle_fp32, ref_bf16):
    """Bit-exact: the oracle's fp32 result, cast the interpreter's way, equals the
    reference kernel's output element for element."""
    assert torch.equal(_trunc_bf16(oracle_fp32), ref_bf16.float())


def _same_as_rn(oracle_fp32, ref_bf16):
    """Bit-exact against an output rounded to nearest (HF fp32 eager math)."""
    assert torch.equal(oracle_fp32.to(torch.bfloat16), ref_bf16)


@pytest.mark.parametrize("tag", ["a", "b", "c", "w4096", "w2048", "w1000", "row1", "big"])
def test_rmsnorm_vs_reference_kernel(gv, tag):
    c = gv[f"rmsnorm_{tag}"]
    _same_as_interpreted_kernel(oracle.rmsnorm(c["x"], c["w"], c["eps"]), c["y"])
    normed, summed = oracle.add_rmsnorm(c["x"], c["r"], c["w"], c["eps"])
    _same_as_interpreted_kernel(normed, c["normed"])
    _same_as_interpreted_kernel(summed, c["summed"])


@pytest.mark.parametrize("tag", ["a", "b", "w1000", "w80", "row1"])
def test_layernorm_vs_reference_kernel(gv, tag):
    c = gv[f"layernorm_{tag}"]
    _same_as_interpreted_kernel(oracle.layernorm(c["x"], c["w"], c["b"], c["eps"]), c["y"])
    normed, summed = oracle.add_layernorm(c["x"], c["r"], c["w"], c["b"], c["eps"])
    _same_as_interpreted_kernel(normed, c["normed"])
    _same_as_interpreted_kernel(summed, c["summed"])


def test_rope_vs_reference_kernel(gv):
    c = gv["rope_vision"]
    _same_as_interpreted_kernel(
        oracle.rope_rotate_half(c["q"], c["cos"][:, None], c["sin"][:, None]), c["q_out"])
    _same_as_interpreted_kernel(
        oracle.rope_rotate_half(c["k"], c["cos"][:, None], c["sin"][:, None]), c["k_out"])
    for key in ("rope_text", "rope_text_d64"):  # [H, S, D] with [S, D] tables
        t = gv[key]
        _same_as_interpreted_kernel(
            oracle.rope_rotate_half(t["q"], t["cos"][None], t["sin"][None]), t["q_out"])


def test_gemm_formulas_vs_reference_kernels(gv):
    c = gv["gate_silu_mul"]
    h = oracle.gate_silu_mul(c["x"], c["w_gate"], c["w_up"])
    assert oracle.max_rel_err(h, c["h_fp32"]) < 1e-5
    # the reference's eager CPU path rounds at every op: same result within bf16 noise
    assert oracle.max_rel_err(c["h_eager_bf16"], h) < 1e-2
    lin = gv["linear"]
    assert oracle.max_rel_err(oracle.linear(lin["x"], lin["w"]), lin["y_fp32"]) < 1e-5
    assert oracle.max_rel_err(oracle.linear(lin["x"], lin["w"], lin["b"]),
                              lin["y_bias_fp32"]) < 1e-5
    assert oracle.max_rel_err(oracle.linear(lin["x"], lin["w"], lin["b"], act="gelu"),
                              lin["y_gelu_fp32"]) < 1e-5


def test_gemm_formulas_with_a_partial_k_block(gv):
    """K = 72: the reference kernels' last k-block is masked; M and N end mid-block."""
    c = gv["gate_silu_mul_ktail"]
    assert oracle.max_rel_err(oracle.gate_silu_mul(c["x"], c["w_gate"], c["w_up"]),
                              c["h_fp32"]) < 1e-5
    lin = gv["linear_ktail"]
    assert oracle.max_rel_err(oracle.linear(lin["x"], lin["w"], lin["b"]),
                              lin["y_bias_fp32"]) < 1e-5
    assert oracle.max_rel_err(oracle.linear(lin["x"], lin["w"], lin["b"], act="gelu"),
                              lin["y_gelu_fp32"]) < 1e-5


def test_hf_eager_functions(gv):
    c = gv["hf_text_rope"]
    cos, sin = c["cos"][:, None], c["sin"][:, None]  # HF unsqueeze_dim=1
    assert oracle.max_rel_err(c["q_out"], oracle.rope_rotate_half(c["q"], cos, sin)) < 1e-2
    assert oracle.max_rel_err(c["k_out"], oracle.rope_rotate_half(c["k"], cos, sin)) < 1e-2
    v = gv["hf_vision_rope"]
    _same_as_rn(oracle.rope_rotate_half(v["q"], v["cos"][:, None], v["sin"][:, None]),
                v["q_out"])
    n = gv["hf_rmsnorm"]
    assert oracle.max_rel_err(n["y"], oracle.rmsnorm(n["x"], n["w"], n["eps"])) < 1e-2


def test_text_rope_tables_match_hf():
    from transformers import Qwen3VLTextConfig
    from transformers.models.qwen3_vl.modeling_qwen3_vl import Qwen3VLTextRotaryEmbedding

    cfg = Qwen3VLTextConfig(hidden_size=4096, num_attention_heads=32, head_dim=128,
                            rope_parameters={"rope_type": "default", "rope_theta": 1e6,
                                             "mrope_section": [24, 20, 20]})
    rot = Qwen3VLTextRotaryEmbedding(cfg)
    pos = torch.arange(50)
    cos_hf, sin_hf = rot(torch.zeros(1, dtype=torch.float32), pos[None])
    cos_o, sin_o = oracle.text_rope_cos_sin(pos, 128, 1e6)
    assert torch.allclose(cos_hf[0], cos_o, atol=1e-6)
    assert torch.allclose(sin_hf[0], sin_o, atol=1e-6)


def test_kv_cache_oracle_replays_reference_sequence(gv):
    c = gv["kv_cache"]
    ref = oracle.KVCacheOracle(c["k0"].to(torch.float32), c["v0"].to(torch.float32), c["extra"],
                               margin=c["margin"])
    assert ref.cap == c["capacity"]
    for st in c["steps"]:
        if st["op"] == "update":
            k, v = ref.update(st["k_new"], st["v_new"])
            assert torch.equal(k, st["keys"]) and torch.equal(v, st["values"])
            assert ref.get_seq_length() == st["len"]
        elif st["op"] == "crop":
            ref.crop(st["arg"])
            assert ref.get_seq_length() == st["len"]
        elif st["op"] == "overflow":
            with pytest.raises(RuntimeError) as e:
                z = torch.zeros(c["k0"].shape[0], c["k0"].shape[1], 5, c["k0"].shape[3])
                ref.update(z, z)
            assert str(e.value) == st["message"]


def test_attention_oracle_matches_transformers_sdpa():
    """oracle.attention against the attention transformers runs for the patched Qwen3
    attention (sdpa_attention_forward: repeat_kv + torch SDPA), on CPU in fp32, with the
    flow expert's mask (new tokens over a cached prefix) and without a mask."""
    from transformers.integrations.sdpa_attention import sdpa_attention_forward

    class M(torch.nn.Module):
        num_key_value_groups = 2
        is_causal = True

    g = torch.Generator().manual_seed(17)
    q = torch.randn(2, 16, 24, 128, generator=g)
    k = torch.randn(2, 8, 200, 128, generator=g)
    v = torch.randn(2, 8, 200, 128, generator=g)
    mask = torch.ones(24, 200, dtype=torch.bool).tril(diagonal=200 - 24)[None, None]
    mask = mask.expand(2, 1, 24, 200)
    for m in (mask, None):
        ref, _ = sdpa_attention_forward(M(), q, k, v, m, scaling=128 ** -0.5, is_causal=False)
        got = oracle.attention(q, k, v, m, 128 ** -0.5)
        assert oracle.rel_err(got, ref) < 1e-5
