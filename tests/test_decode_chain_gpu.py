"""The decode chain kernel (umic_decode_mlp_chain) against the unfused decode kernels.

One decoder layer's decode-step tail -- o_proj, the attention-residual add with the
post-attention RMSNorm, gate/up with SiLU, down_proj with the MLP residual -- runs as the
phases of one persistent kernel. It splits every weight matrix over the CTAs exactly as
the streaming GEMV does and sums split row blocks in the same CTA order, and its
add+RMSNorm uses the norm kernel's thread partition and reduction order, so the output
must equal the unfused sequence (umic_gemv -> umic_add_rmsnorm -> umic_gemv_gate_silu_mul
-> umic_gemv_residual) bit for bit; it is also checked against the fp32 formula.
"""

import pytest
import torch

import oracle
from umic_b200.kernels import add_rmsnorm, stats
from umic_b200.kernels.decode import decode_mlp_chain
from umic_b200.kernels.fused_ffn import gate_silu_mul_nk
from umic_b200.kernels.linear import linear_gemv, linear_gemv_residual

pytestmark = pytest.mark.gpu


def _randn(*shape, seed, dev, scale=1.0):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(*shape, generator=g) * scale).to(torch.bfloat16).to(dev)


def _layer(dev, hidden, inter, k_attn, seed=0):
    w_o = _randn(hidden, k_attn, seed=seed + 1, dev=dev, scale=0.02)
    post = (1 + 0.05 * torch.randn(hidden, generator=torch.Generator().manual_seed(seed + 2)))
    post = post.to(torch.bfloat16).to(dev)
    wg = _randn(inter, hidden, seed=seed + 3, dev=dev, scale=0.02)
    wu = _randn(inter, hidden, seed=seed + 4, dev=dev, scale=0.02)
    wd = _randn(hidden, inter, seed=seed + 5, dev=dev, scale=0.02)
    return w_o, post, wg, wu, wd


def _unfused(attn, resid, w_o, post, wg, wu, wd):
    o = linear_gemv(attn, w_o, weights_ready=True)
    normed, summed = add_rmsnorm(o, resid, post, 1e-6)
    h = gate_silu_mul_nk(normed, wg, wu, weights_ready=True)
    return linear_gemv_residual(h, wd, summed, weights_ready=True)


@pytest.mark.parametrize("m", [8, 1, 4, 16])
def test_decode_chain_matches_unfused_bitwise(cuda, m):
    """cfg4 shapes: hidden 4096, 32 x 128 attention width, SwiGLU 12288."""
    w_o, post, wg, wu, wd = _layer(cuda, 4096, 12288, 4096)
    attn = _randn(m, 4096, seed=10, dev=cuda)
    resid = _randn(m, 4096, seed=11, dev=cuda, scale=4.0)
    stats.clear()
    got = decode_mlp_chain(attn, w_o, resid, post, 1e-6, wg, wu, wd)
    assert got is not None and stats["umic_decode_mlp_chain"] == 1
    ref = _unfused(attn, resid, w_o, post, wg, wu, wd)
    assert torch.equal(got, ref), float((got.float() - ref.float()).abs().max())
    again = decode_mlp_chain(attn, w_o, resid, post, 1e-6, wg, wu, wd)
    assert torch.equal(got, again)  # the workspace came back clean
    if m == 8:
        s = resid.float().cpu() + attn.float().cpu() @ w_o.float().cpu().t()
        n = s * torch.rsqrt((s * s).mean(-1, keepdim=True) + 1e-6) * post.float().cpu()
        h = torch.nn.functional.silu(n @ wg.float().cpu().t()) * (n @ wu.float().cpu().t())
        ref32 = s + h @ wd.float().cpu().t()
        assert oracle.max_rel_err(got, ref32) <= 1e-2


def test_decode_chain_in_a_cuda_graph(cuda):
    """Captured once and replayed with new inputs: the cooperative launch is captured and
    its barrier counters return to zero between replays."""
    w_o, post, wg, wu, wd = _layer(cuda, 4096, 12288, 4096, seed=20)
    attn = _randn(8, 4096, seed=21, dev=cuda)
    resid = _randn(8, 4096, seed=22, dev=cuda)
    decode_mlp_chain(attn, w_o, resid, post, 1e-6, wg, wu, wd)  # workspace before capture
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        out = decode_mlp_chain(attn, w_o, resid, post, 1e-6, wg, wu, wd)
    assert out is not None
    for seed in (23, 24, 25):
        attn.copy_(_randn(8, 4096, seed=seed, dev=cuda))
        g.replay()
        torch.cuda.synchronize()
        assert torch.equal(out, _unfused(attn, resid, w_o, post, wg, wu, wd))


def test_decode_chain_declines_uncovered_shapes(cuda):
    w_o, post, wg, wu, wd = _layer(cuda, 1024, 3072, 1024, seed=30)  # too few units per CTA
    attn = _randn(8, 1024, seed=31, dev=cuda)
    resid = _randn(8, 1024, seed=32, dev=cuda)
    stats.clear()
    assert decode_mlp_chain(attn, w_o, resid, post, 1e-6, wg, wu, wd) is None
    assert stats["decode_mlp_chain_fallback"] == 1
    assert decode_mlp_chain(_randn(17, 1024, seed=33, dev=cuda), w_o,
                            _randn(17, 1024, seed=34, dev=cuda), post, 1e-6, wg, wu, wd) is None
