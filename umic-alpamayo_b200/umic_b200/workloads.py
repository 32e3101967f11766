"""Synthetic stand-ins for the Alpamayo-style stack, built from the BASELINE configs.

The Alpamayo 1.5 weights, its dataset clip and its flow sampler are not
available, so the workloads are random-init HF Qwen3-VL modules of the stated
shapes (weights ~N(0, 0.02) from transformers' own initialiser, norm weights 1)
driven by seeded synthetic inputs:
  cfg3  ViT: 27 blocks, hidden 1280, 16 x 80 heads, MLP 5120 (tanh GELU),
        patch 14 x 14 x 2 x 3 = 1176, 16 images of 448 x 448 -> 16 x 1024 tokens
  cfg4  LM: 36 layers, hidden 4096, GQA 32 q / 8 kv x 128, SwiGLU 12288,
        vocab 151936, RoPE theta 1e6; prefill 3100 tokens + 64 greedy steps
  cfg5  flow expert: 18 layers, hidden 2048, GQA 16 / 8 x 128, SwiGLU 8192;
        64 action tokens, 10 Euler steps over a 3100-token prefix KV
`AlpamayoStandIn` carries them as `.vlm` / `.expert` so `apply()` finds them
where it finds Alpamayo's.
"""

from __future__ import annotations

import contextlib
from dataclasses import dataclass, field

import torch
from torch import nn

CFG4_TEXT = dict(vocab_size=151936, hidden_size=4096, intermediate_size=12288,
                 num_hidden_layers=36, num_attention_heads=32, num_key_value_heads=8,
                 head_dim=128, rms_norm_eps=1e-6, max_position_embeddings=32768,
                 rope_parameters={"rope_type": "default", "rope_theta": 1e6,
                                  "mrope_section": [24, 20, 20]})
CFG5_EXPERT = dict(vocab_size=1024, hidden_size=2048, intermediate_size=8192,
                   num_hidden_layers=18, num_attention_heads=16, num_key_value_heads=8,
                   head_dim=128, rms_norm_eps=1e-6, max_position_embeddings=32768,
                   rope_parameters={"rope_type": "default", "rope_theta": 1e6,
                                    "mrope_section": [24, 20, 20]})
CFG3_VISION = dict(depth=27, hidden_size=1280, intermediate_size=5120, num_heads=16,
                   patch_size=14, temporal_patch_size=2, in_channels=3, spatial_merge_size=2,
                   out_hidden_size=4096, num_position_embeddings=2304,
                   deepstack_visual_indexes=[8, 16, 24], hidden_act="gelu_pytorch_tanh")
TINY_VISION = dict(depth=1, hidden_size=64, intermediate_size=128, num_heads=2, patch_size=14,
                   out_hidden_size=4096, num_position_embeddings=64,
                   deepstack_visual_indexes=[])
PREFILL_TOKENS = 3100
DECODE_STEPS = 64
FLOW_TOKENS = 64
FLOW_STEPS = 10


@contextlib.contextmanager
def _build_ctx(device, dtype=torch.bfloat16):
    prev = torch.get_default_dtype()
    torch.set_default_dtype(dtype)
    try:
        with torch.device(device):
            yield
    finally:
        torch.set_default_dtype(prev)


def _finish(model: nn.Module) -> nn.Module:
    model.eval()
    for p in model.parameters():
        p.requires_grad_(False)
    return model


def text_config(**overrides):
    from transformers import Qwen3VLTextConfig

    kw = dict(CFG4_TEXT)
    kw.update(overrides)
    cfg = Qwen3VLTextConfig(**kw)
    cfg._attn_implementation = "sdpa"
    return cfg


def build_vlm(text: dict | None = None, vision: dict | None = None, device="cuda",
              seed: int = 4) -> nn.Module:
    """Random-init Qwen3VLForConditionalGeneration (bf16, eval, no grad) on `device`."""
    from transformers import Qwen3VLConfig
    from transformers.models.qwen3_vl.modeling_qwen3_vl import Qwen3VLForConditionalGeneration

    cfg = Qwen3VLConfig(text_config=dict(text or CFG4_TEXT),
                        vision_config=dict(vision or TINY_VISION))
    cfg._attn_implementation = "sdpa"
    cfg.text_config._attn_implementation = "sdpa"
    cfg.vision_config._attn_implementation = "sdpa"
    torch.manual_seed(seed)
    with _build_ctx(device):
        model = Qwen3VLForConditionalGeneration(cfg)
    return _finish(model)


def build_text_model(text: dict | None = None, device="cuda", seed: int = 5) -> nn.Module:
    from transformers.models.qwen3_vl.modeling_qwen3_vl import Qwen3VLTextModel

    cfg = text_config(**(text or CFG5_EXPERT))
    torch.manual_seed(seed)
    with _build_ctx(device):
        model = Qwen3VLTextModel(cfg)
    return _finish(model)


def build_vision_model(vision: dict | None = None, device="cuda", seed: int = 3) -> nn.Module:
    from transformers.models.qwen3_vl.configuration_qwen3_vl import Qwen3VLVisionConfig
    from transformers.models.qwen3_vl.modeling_qwen3_vl import Qwen3VLVisionModel

    cfg = Qwen3VLVisionConfig(**(vision or CFG3_VISION))
    cfg._attn_implementation = "sdpa"
    torch.manual_seed(seed)
    with _build_ctx(device):
        model = Qwen3VLVisionModel(cfg)
    return _finish(model)


def tiny_qwen3vl_configs() -> dict:
    """Tiny Qwen3-VL (text, vision) config pairs for structural-match checks."""
    rope = {"rope_type": "default", "rope_theta": 1e6, "mrope_section": [2, 3, 3]}
    t2 = dict(vocab_size=512, hidden_size=64, intermediate_size=128, num_hidden_layers=2,
              num_attention_heads=4, num_key_value_heads=2, head_dim=16, rms_norm_eps=1e-6,
              rope_parameters=rope)
    v4 = dict(depth=4, hidden_size=32, intermediate_size=64, num_heads=2, patch_size=14,
              out_hidden_size=64, num_position_embeddings=64, deepstack_visual_indexes=[1, 2])
    t3 = dict(t2, num_hidden_layers=3)
    v2 = dict(v4, depth=2, deepstack_visual_indexes=[0])
    return {"t2_v4": (t2, v4), "t3_v2": (t3, v2)}


class AlpamayoStandIn(nn.Module):
    """Container with Alpamayo's attribute layout: `.vlm` (+ `.expert`)."""

    def __init__(self, vlm: nn.Module, expert: nn.Module | None = None):
        super().__init__()
        self.vlm = vlm
        if expert is not None:
            self.expert = expert


# ------------------------------------------------------------------ inputs

def prefill_ids(episodes: int, tokens: int = PREFILL_TOKENS, vocab: int = 151936,
                seed: int = 4, device="cpu") -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    return torch.randint(0, vocab, (episodes, tokens), generator=g).to(device)


def vit_inputs(images: int = 16, side: int = 448, patch: int = 14, temporal: int = 2,
               seed: int = 3, device="cpu"):
    """Flattened patches [images * (side/patch)^2, 3 * temporal * patch^2] of
    uniform[-1, 1] pixels and grid_thw [images, 3]."""
    g = torch.Generator().manual_seed(seed)
    grid = side // patch
    n = images * grid * grid
    pix = (torch.rand(n, 3 * temporal * patch * patch, generator=g) * 2 - 1)
    grid_thw = torch.tensor([[1, grid, grid]] * images, dtype=torch.long)
    return pix.to(device=device, dtype=torch.bfloat16), grid_thw.to(device)


# ------------------------------------------------------------------ loops

def kv_cache_for(vlm: nn.Module, batch: int, capacity: int, device):
    from .cache import InplaceKVCache

    tc = vlm.config.text_config
    return InplaceKVCache.allocate(tc.num_hidden_layers, batch, tc.num_key_value_heads,
                                   tc.head_dim, capacity, device)


@torch.no_grad()
def prefill(vlm: nn.Module, input_ids: torch.Tensor, cache) -> torch.Tensor:
    """One prefill pass writing `cache`; returns the greedy next token per row."""
    out = vlm(input_ids=input_ids, past_key_values=cache, use_cache=True, logits_to_keep=1)
    return out.logits[:, -1].argmax(-1)


@torch.no_grad()
def greedy_generate(vlm: nn.Module, input_ids: torch.Tensor, new_tokens: int,
                    cache=None) -> torch.Tensor:
    """Prefill + (new_tokens - 1) greedy decode steps; returns [B, new_tokens] ids.

    Decode calls go through vlm.forward, so a DecodeGraphRunner installed by
    apply() replays its per-length graphs here."""
    b, s = input_ids.shape
    if cache is None:
        cache = kv_cache_for(vlm, b, s + new_tokens + 8, input_ids.device)
    else:
        cache.crop(0)
    nxt = prefill(vlm, input_ids, cache)
    toks = [nxt]
    for _ in range(new_tokens - 1):
        out = vlm(input_ids=nxt[:, None], past_key_values=cache, use_cache=True,
                  logits_to_keep=1)
        nxt = out.logits[:, -1].argmax(-1)
        toks.append(nxt)
    runner = getattr(vlm.forward, "__self__", None)
    if runner is not None and hasattr(runner, "finish"):
        runner.finish()
    return torch.stack(toks, 1)


@dataclass
class FlowState:
    """Per-batch state of the synthetic flow-matching sampler (cfg5)."""

    prefix_cache: object
    base_len: int
    x: torch.Tensor
    extras: dict = field(default_factory=dict)


@torch.no_grad()
def flow_step(expert: nn.Module, cache, base_len: int, x: torch.Tensor) -> torch.Tensor:
    """Velocity of the action tokens x [B, T, H]: one expert pass attending to the
    prefix KV; the T tokens are appended at [base, base + T) and cropped back."""
    cache.crop(base_len)
    b, t, _ = x.shape
    pos = torch.arange(base_len, base_len + t, device=x.device).unsqueeze(0).expand(b, t)
    out = expert(inputs_embeds=x, past_key_values=cache, use_cache=True, position_ids=pos)
    cache.crop(base_len)
    return out.last_hidden_state


@torch.no_grad()
def flow_sample(expert: nn.Module, cache, base_len: int, x0: torch.Tensor,
                steps: int = FLOW_STEPS, graph: bool = False) -> torch.Tensor:
    """Euler integration x <- x + dt * v(x) over `steps` steps.

    When apply() has rebound the expert's final RMSNorm, the update runs inside that
    norm's kernel (integrate.axpy_epilogue): a step is the expert pass and nothing else.

    graph=True runs the steps through FlowStepGraph (the reference's unwired
    graph.py:179-253): after two eager warm-up steps one whole Euler step -- the
    expert pass with its prefix-KV append and crop, and the update x + dt * v --
    is captured once as a CUDA graph and replayed (same shapes and buffer
    addresses every step; only x changes). The runner is kept on the expert per
    (shape, dtype, cache, prefix length, steps), so later calls replay every step."""
    from . import integrate
    from .graph import FlowStepGraph

    dt = 1.0 / steps
    final_norm = getattr(expert, "norm", None)
    fused_update = integrate.has_axpy_epilogue(final_norm)

    def euler(x: torch.Tensor, t: torch.Tensor | None) -> torch.Tensor:
        if fused_update:
            # the velocity is the expert's final RMSNorm output: that kernel writes
            # x + dt * v directly (umic_rmsnorm_axpy), v is never stored
            with integrate.axpy_epilogue(final_norm, x, dt):
                return flow_step(expert, cache, base_len, x)
        return x + dt * flow_step(expert, cache, base_len, x)

    x = x0
    if not graph:
        for _ in range(steps):
            x = euler(x, None)
        return x
    key = (tuple(x0.shape), x0.dtype, id(cache), base_len, steps)
    runners = expert.__dict__.setdefault("_umic_flow_graphs", {})
    runner = runners.get(key)
    if runner is None:
        runner = runners[key] = FlowStepGraph(euler)
    t = torch.zeros(1, device=x0.device)
    for i in range(steps):
        t.fill_(i * dt)  # the flow time; the stand-in expert does not condition on it
        x = runner(x, t)
    return x


def smoke_decoder(device) -> None:
    """A 2-layer Qwen3-VL-shaped model through apply(): prefill + 4 graph decode
    steps; the token stream must equal the unpatched model's on the same weights."""
    from . import integrate
    from .optimize import UmicConfig, apply

    small = dict(CFG4_TEXT, num_hidden_layers=2, hidden_size=512, intermediate_size=1024,
                 num_attention_heads=8, num_key_value_heads=4, vocab_size=4096)
    vlm = build_vlm(text=small, device=device, seed=11)
    ids = prefill_ids(2, 96, vocab=4096, seed=12, device=device)
    ref = greedy_generate(vlm, ids, 5)
    model = AlpamayoStandIn(vlm)
    report = apply(model, UmicConfig(max_new_tokens=16))
    try:
        got = greedy_generate(vlm, ids, 5)
        got2 = greedy_generate(vlm, ids, 5)  # replays the captured graphs
    finally:
        model._umic_decode_runner.release()
        integrate.unfuse_mlps(model)
        integrate.unfuse_rope()
    assert report["lm_mlp_fused"] == 2 and report["lm_add_rmsnorm_fused"] == 2, report
    assert torch.equal(got, got2), "graph replay changed the token stream"
    agree = (got == ref).float().mean().item()
    print(f"smoke decoder: report={report} token agreement with eager={agree:.2f}")
