"""Greedy token-stream parity at the full cfg4 LM configuration.

Model: the 36-layer decoder, hidden 4096, GQA 32 q / 8 kv heads of 128, SwiGLU 12288,
RMSNorm eps 1e-6, RoPE theta 1e6, the full 151936-token vocabulary, random-init weights
~N(0, 0.02) (seed 4, as bench.py). Workload: 8 episodes x 3100 uniform token ids, a
batched prefill, then 64 greedy steps. Our path goes through `apply()` with the in-place
KV cache and the per-KV-length CUDA-graph decode; the references are the same model
unpatched in bf16 (the unfused eager GPU path) and an fp32 copy (TF32 off).

With random weights the top-1 / top-2 logit gap of a step is often inside bf16 rounding
noise, so two bf16 implementations -- ours and eager -- can pick different tokens where
the fp32 model sees a near tie (the reference's 3106/3106 identical tokens,
docs/260611_output_equivalence.md:9-16, were measured with trained weights). The test
therefore checks, at every position where ours and eager pick different tokens with the
same prefix:
  * teacher-forced along the eager stream (all 8 x 64 positions share their prefix),
  * free-running (the first divergence of each episode),
that the fp32 model's top-1 / top-2 gap on that prefix lies inside the bf16 noise
measured on the same prefix: noise = max over the vocabulary of |eager - fp32| logits.
Ours must also be no noisier than eager against fp32, and the teacher-forced agreement
with the fp32 argmax (along the fp32 stream) must match eager's. Graph replay must be
bit-reproducible.
"""

import copy

import pytest
import torch
from transformers.cache_utils import DynamicCache

from umic_b200 import UmicConfig, apply, integrate
from umic_b200.kernels import stats
from umic_b200.workloads import (DECODE_STEPS, PREFILL_TOKENS, AlpamayoStandIn, build_vlm,
                                 kv_cache_for, prefill_ids)

pytestmark = pytest.mark.gpu

EPISODES = 8
# Ours may be at most this much noisier than eager at one position / on average.
NOISE_SLACK_POS, NOISE_SLACK_MEAN = 1.5, 1.1


@pytest.fixture(autouse=True)
def _strict_fp32():
    prev = (torch.backends.cuda.matmul.allow_tf32, torch.backends.cudnn.allow_tf32)
    torch.backends.cuda.matmul.allow_tf32 = torch.backends.cudnn.allow_tf32 = False
    yield
    torch.backends.cuda.matmul.allow_tf32, torch.backends.cudnn.allow_tf32 = prev
    integrate.unfuse_rope()


def _stream(vlm, ids, steps, cache, forced=None):
    """Prefill + decode. Returns (greedy tokens [B, steps], fp32 logits [B, steps, V]).
    With `forced` [B, steps - 1], step t + 1 is fed forced[:, t] instead of the argmax."""
    toks, logits = [], []
    with torch.no_grad():
        out = vlm(input_ids=ids, past_key_values=cache, use_cache=True, logits_to_keep=1)
        for t in range(steps):
            lg = out.logits[:, -1].float()
            nxt = lg.argmax(-1)
            toks.append(nxt)
            logits.append(lg)
            if t + 1 == steps:
                break
            feed = nxt if forced is None else forced[:, t]
            out = vlm(input_ids=feed[:, None], past_key_values=cache, use_cache=True,
                      logits_to_keep=1)
    runner = getattr(vlm.forward, "__self__", None)
    if runner is not None and hasattr(runner, "finish"):
        runner.finish()
    return torch.stack(toks, 1), torch.stack(logits, 1)


def _divergence_report(name, tok_a, l_a, tok_b, l_b, l32):
    """Positions where a and b chose differently on the same prefix: the fp32 top-1 /
    top-2 gap there, against the bf16 noise of b and a (max |logit - fp32|)."""
    noise_a = (l_a - l32).abs().amax(-1)
    noise_b = (l_b - l32).abs().amax(-1)
    top2 = l32.topk(2, dim=-1).values
    gap = top2[..., 0] - top2[..., 1]
    diff = tok_a != tok_b
    rows = []
    for e, p in diff.nonzero().tolist():
        rows.append((e, p, float(gap[e, p]), float(noise_b[e, p]), float(noise_a[e, p])))
    print(f"{name}: {int(diff.sum())} of {diff.numel()} positions differ")
    for e, p, g, nb, na in rows:
        print(f"  episode {e} step {p}: fp32 top-2 gap {g:.4f}, eager noise {nb:.4f}, "
              f"ours noise {na:.4f}")
    return rows, noise_a, noise_b


def test_cfg4_greedy_token_stream(cuda):
    vlm = build_vlm(device=cuda, seed=4)
    ids = prefill_ids(EPISODES, PREFILL_TOKENS, seed=4, device=cuda)
    steps = DECODE_STEPS

    # unpatched bf16 eager: free-running stream
    tok_e, l_e = _stream(vlm, ids, steps, DynamicCache())
    # fp32 copy: its free-running stream, then teacher-forced along the eager stream
    ref32 = copy.deepcopy(vlm).float()
    tok_32, l_32 = _stream(ref32, ids, steps, DynamicCache())
    _, l32_on_e = _stream(ref32, ids, steps, DynamicCache(), forced=tok_e[:, :-1])
    del ref32
    torch.cuda.empty_cache()
    # eager teacher-forced along the fp32 stream
    _, l_e_on32 = _stream(vlm, ids, steps, DynamicCache(), forced=tok_32[:, :-1])

    model = AlpamayoStandIn(vlm)
    report = apply(model, UmicConfig(max_new_tokens=steps + 8))
    try:
        cache = kv_cache_for(vlm, EPISODES, PREFILL_TOKENS + steps + 8, cuda)
        stats.clear()
        tok_o, l_o = _stream(vlm, ids, steps, cache)
        assert stats["umic_gemm_gate_silu_mul"] >= 36 and stats["umic_qk_norm_rope_kv"] >= 36
        cache.crop(0)
        tok_o2, l_o2 = _stream(vlm, ids, steps, cache)  # every step a graph replay
        cache.crop(0)
        _, l_o_on_e = _stream(vlm, ids, steps, cache, forced=tok_e[:, :-1])
        cache.crop(0)
        _, l_o_on32 = _stream(vlm, ids, steps, cache, forced=tok_32[:, :-1])
        graphs = len(model._umic_decode_runner.graphs)
    finally:
        model._umic_decode_runner.release()
        integrate.unfuse_mlps(model)
    assert report["lm_mlp_fused"] == 36 and report["decode_graph"] is True
    assert graphs == steps - 1, graphs  # one graph per KV length after the prefill
    assert torch.equal(tok_o, tok_o2) and torch.equal(l_o, l_o2), "graph replay not reproducible"

    # ---- free-running agreement
    def agree(a, b):
        return float((a == b).float().mean())

    def first_div(a, b):
        d = (a != b).int()
        return [int(r.argmax()) if r.any() else a.shape[1] for r in d]

    print(f"free-running token agreement: ours/eager {agree(tok_o, tok_e):.3f}, "
          f"ours/fp32 {agree(tok_o, tok_32):.3f}, eager/fp32 {agree(tok_e, tok_32):.3f}")
    print(f"first divergence step per episode, ours vs eager: {first_div(tok_o, tok_e)}; "
          f"eager vs fp32: {first_div(tok_e, tok_32)}")

    # ---- teacher-forced along the eager stream: every position shares its prefix
    pick_o = l_o_on_e.argmax(-1)
    rows, noise_o, noise_e = _divergence_report("teacher-forced on the eager stream, ours vs "
                                                "eager", pick_o, l_o_on_e, tok_e, l_e, l32_on_e)
    for e, p, gap, ne, no in rows:
        assert gap <= 2 * NOISE_SLACK_POS * ne, (e, p, gap, ne, no)
    print(f"logit noise vs fp32 on the eager stream: ours mean {float(noise_o.mean()):.4f} "
          f"max {float(noise_o.max()):.4f}; eager mean {float(noise_e.mean()):.4f} "
          f"max {float(noise_e.max()):.4f}")
    assert float(noise_o.mean()) <= NOISE_SLACK_MEAN * float(noise_e.mean())
    assert float(noise_o.max()) <= NOISE_SLACK_POS * float(noise_e.max())

    # ---- free-running: the first divergence of each episode also shares its prefix
    for e, p in enumerate(first_div(tok_o, tok_e)):
        if p == steps:
            continue
        top2 = l32_on_e[e, p].topk(2).values
        gap = float(top2[0] - top2[1])
        ne = float((l_e[e, p] - l32_on_e[e, p]).abs().max())
        print(f"  free-running episode {e}: first divergence at step {p}, fp32 top-2 gap "
              f"{gap:.4f}, eager noise {ne:.4f}")
        assert gap <= 2 * NOISE_SLACK_POS * ne, (e, p, gap, ne)

    # ---- teacher-forced along the fp32 stream: agreement with the fp32 argmax
    a32 = tok_32
    agree_o, agree_e = agree(l_o_on32.argmax(-1), a32), agree(l_e_on32.argmax(-1), a32)
    print(f"teacher-forced on the fp32 stream, top-1 agreement with fp32: ours {agree_o:.4f}, "
          f"eager {agree_e:.4f}")
    assert agree_o >= agree_e - 2.0 / a32.numel()
