"""GPU parity of every C-ABI kernel against the CPU oracle (fp32 restatement).

Bar: per-tensor max relative error <= 1e-2 and L2 relative error <= 1e-2 against
the fp32-accumulated oracle (check_env.py used 2e-2).
Shapes: the BASELINE configs (cfg1/cfg2 sizes) plus small, odd and empty shapes
that exercise tails and the non-vectorised paths.
"""

import pytest
import torch

import oracle
from umic_b200 import _lib
from umic_b200.kernels import (add_layernorm, add_rmsnorm, apply_rotary_text_inplace,
                               apply_rotary_vision, gate_silu_mul, gate_silu_mul_nk, kv_append,
                               layernorm, linear, linear_gemv, rmsnorm, rmsnorm_axpy, stats)
from umic_b200.kernels.attention import qk_norm_rope_kv
from umic_b200.kernels.linear import linear_gemv_multi

pytestmark = pytest.mark.gpu

TOL = 1e-2


def _close(out, ref, tol=TOL):
    mre = oracle.max_rel_err(out, ref)
    l2 = oracle.rel_err(out, ref)
    assert mre <= tol and l2 <= tol, f"max_rel_err={mre:.3e} l2={l2:.3e}"


def _randn(*shape, seed, dev, dtype=torch.bfloat16, scale=1.0):
    g = torch.Generator(device="cpu").manual_seed(seed)
    return (torch.randn(*shape, generator=g) * scale).to(dtype).to(dev)


# ------------------------------------------------------------------ norms

NORM_SHAPES = [(3100, 4096), (99, 128), (7, 1280), (5, 2048), (33, 1152), (3, 100), (1, 8),
               (2, 24), (4, 16384 + 8)]


@pytest.mark.parametrize("rows,n", NORM_SHAPES)
@pytest.mark.parametrize("wdt", [torch.bfloat16, torch.float32])
def test_rmsnorm(cuda, rows, n, wdt):
    x = _randn(rows, n, seed=1, dev=cuda)
    w = (1 + 0.05 * _randn(n, seed=2, dev="cpu", dtype=torch.float32)).to(wdt).to(cuda)
    if n > 16384:
        with pytest.raises(RuntimeError):
            rmsnorm(x, w, 1e-6)
        return
    y = rmsnorm(x, w, 1e-6)
    assert y.dtype == torch.bfloat16 and y.shape == x.shape
    _close(y, oracle.rmsnorm(x.cpu(), w.cpu(), 1e-6))


@pytest.mark.parametrize("rows,n", NORM_SHAPES[:-1])
def test_add_rmsnorm(cuda, rows, n):
    x = _randn(rows, n, seed=3, dev=cuda)
    r = _randn(rows, n, seed=4, dev=cuda)
    w = (1 + 0.05 * _randn(n, seed=5, dev=cuda, dtype=torch.float32)).to(torch.bfloat16)
    normed, summed = add_rmsnorm(x, r, w, 1e-6)
    rn, rs = oracle.add_rmsnorm(x.cpu(), r.cpu(), w.cpu(), 1e-6)
    _close(normed, rn)
    _close(summed, rs)


@pytest.mark.parametrize("rows,n", [(32 * 64, 2048), (99, 128), (5, 2048), (3, 100), (1, 8)])
@pytest.mark.parametrize("inplace", [False, True])
def test_rmsnorm_axpy(cuda, rows, n, inplace):
    """The flow sampler's Euler update x + dt * rmsnorm(h) * w in one pass (cfg5 shape:
    32 episodes x 64 action tokens x 2048), against the fp32 formula; in place
    (out = x) and out of place; (3, 100) takes the unaligned scalar path."""
    h = _randn(rows, n, seed=40, dev=cuda)
    x = _randn(rows, n, seed=41, dev=cuda)
    w = (1 + 0.05 * _randn(n, seed=42, dev="cpu", dtype=torch.float32)).to(torch.bfloat16)
    w = w.to(cuda)
    ref = oracle.rmsnorm_axpy(h.cpu(), w.cpu(), 1e-6, x.cpu(), 0.1)
    if inplace:
        y = rmsnorm_axpy(h, w, 1e-6, x, 0.1, out=x)
        assert y is x
    else:
        x0 = x.clone()
        y = rmsnorm_axpy(h, w, 1e-6, x, 0.1)
        assert torch.equal(x, x0)
    _close(y, ref)


def test_rmsnorm_axpy_strided_rows(cuda):
    big = _randn(64, 2048 + 64, seed=43, dev=cuda)
    h = big[:, :2048]  # row stride 2112
    x = _randn(64, 2048, seed=44, dev=cuda)
    w = _randn(2048, seed=45, dev=cuda)
    _close(rmsnorm_axpy(h, w, 1e-6, x, -0.25), oracle.rmsnorm_axpy(h.cpu(), w.cpu(), 1e-6,
                                                                  x.cpu(), -0.25))


def test_rmsnorm_strided_rows(cuda):
    base = _randn(64, 4096 + 64, seed=6, dev=cuda)
    x = base[:, :4096]  # row stride 4160
    w = _randn(4096, seed=7, dev=cuda)
    _close(rmsnorm(x, w, 1e-6), oracle.rmsnorm(x.cpu(), w.cpu(), 1e-6))


def test_rmsnorm_per_head_layout(cuda):
    # q_norm over [B, S, H, 128] (the HF q_proj output viewed per head)
    x = _randn(1, 3100, 32, 128, seed=8, dev=cuda)
    w = _randn(128, seed=9, dev=cuda)
    _close(rmsnorm(x, w, 1e-6), oracle.rmsnorm(x.cpu(), w.cpu(), 1e-6))


@pytest.mark.parametrize("rows,n", [(16384, 1280), (4096, 1152), (7, 1280), (5, 80), (3, 100)])
def test_layernorm(cuda, rows, n):
    x = _randn(rows, n, seed=10, dev=cuda)
    w = _randn(n, seed=11, dev=cuda)
    b = _randn(n, seed=12, dev=cuda)
    _close(layernorm(x, w, b, 1e-6), oracle.layernorm(x.cpu(), w.cpu(), b.cpu(), 1e-6))


@pytest.mark.parametrize("rows,n", [(16384, 1280), (33, 1280), (9, 4096), (3, 100)])
def test_add_layernorm(cuda, rows, n):
    x = _randn(rows, n, seed=13, dev=cuda)
    r = _randn(rows, n, seed=14, dev=cuda)
    w = torch.ones(n, device=cuda, dtype=torch.bfloat16)
    b = _randn(n, seed=15, dev=cuda)
    normed, summed = add_layernorm(x, r, w, b, 1e-6)
    rn, rs = oracle.add_layernorm(x.cpu(), r.cpu(), w.cpu(), b.cpu(), 1e-6)
    _close(normed, rn)
    _close(summed, rs)


def test_norm_empty_rows(cuda):
    x = torch.empty(0, 4096, device=cuda, dtype=torch.bfloat16)
    w = torch.ones(4096, device=cuda, dtype=torch.bfloat16)
    assert rmsnorm(x, w, 1e-6).shape == (0, 4096)


# ------------------------------------------------------------------- RoPE

@pytest.mark.parametrize("batch,seq,hq,hk,d", [(1, 3100, 32, 8, 128), (2, 37, 4, 2, 128),
                                               (1, 5, 3, 1, 20), (1, 1, 32, 8, 128)])
def test_text_rope_inplace(cuda, batch, seq, hq, hk, d):
    q = _randn(batch, seq, hq, d, seed=20, dev=cuda).transpose(1, 2)  # HF [B, H, S, D] view
    k = _randn(batch, seq, hk, d, seed=21, dev=cuda).transpose(1, 2)
    pos = torch.arange(seq).unsqueeze(0) + torch.arange(batch).unsqueeze(1) * 7
    cs = [oracle.text_rope_cos_sin(p, d, 1e6) for p in pos]
    cos = torch.stack([c for c, _ in cs]).to(torch.bfloat16).to(cuda)
    sin = torch.stack([s for _, s in cs]).to(torch.bfloat16).to(cuda)
    q0, k0 = q.cpu(), k.cpu()
    qo, ko = apply_rotary_text_inplace(q, k, cos, sin)
    assert qo.data_ptr() == q.data_ptr() and ko.data_ptr() == k.data_ptr()
    _close(q, oracle.rope_rotate_half(q0, cos.cpu()[:, None], sin.cpu()[:, None]))
    _close(k, oracle.rope_rotate_half(k0, cos.cpu()[:, None], sin.cpu()[:, None]))


@pytest.mark.parametrize("seq,h,d", [(16384, 16, 80), (100, 3, 80), (7, 2, 20)])
def test_vision_rope_inplace(cuda, seq, h, d):
    qkv = _randn(seq, 3, h, d, seed=22, dev=cuda)
    q, k, _ = qkv.unbind(1)  # row stride 3*h*d like the HF qkv view
    f = _randn(seq, d // 2, seed=23, dev=cuda, dtype=torch.float32)
    emb = torch.cat((f, f), -1)
    cos, sin = emb.cos(), emb.sin()
    q0, k0 = q.cpu(), k.cpu()
    apply_rotary_vision(q, k, cos, sin)
    _close(q, oracle.rope_rotate_half(q0, cos.cpu()[:, None], sin.cpu()[:, None]))
    _close(k, oracle.rope_rotate_half(k0, cos.cpu()[:, None], sin.cpu()[:, None]))
    # v untouched
    assert torch.equal(qkv[:, 2].cpu(), _randn(seq, 3, h, d, seed=22, dev="cpu")[:, 2])


# --------------------------------------------------------------------- KV

def test_kv_append_host_and_device_pos(cuda):
    b, h, base, d, extra = 2, 8, 40, 128, 10
    k0 = _randn(b, h, base, d, seed=30, dev="cpu")
    v0 = _randn(b, h, base, d, seed=31, dev="cpu")
    ref = oracle.KVCacheOracle(k0, v0, extra)
    kb = torch.zeros(b, h, ref.cap, d, dtype=torch.bfloat16, device=cuda)
    vb = torch.zeros_like(kb)
    kb[:, :, :base] = k0.to(cuda)
    vb[:, :, :base] = v0.to(cuda)
    pos = base
    for n, seed in ((3, 32), (1, 33)):
        kn = _randn(b, n, h, d, seed=seed, dev=cuda).transpose(1, 2)  # strided [B,H,n,D]
        vn = _randn(b, n, h, d, seed=seed + 100, dev=cuda).transpose(1, 2)
        kv_append(kb, vb, kn, vn, pos)
        ref.update(kn.cpu(), vn.cpu())
        pos += n
    dpos = torch.tensor([pos], dtype=torch.int64, device=cuda)
    kn = _randn(b, h, 1, d, seed=40, dev=cuda)
    vn = _randn(b, h, 1, d, seed=41, dev=cuda)
    kv_append(kb, vb, kn, vn, dpos)
    ref.graph_update(kn.cpu(), vn.cpu(), pos, pos + 1)
    assert torch.equal(kb.cpu(), ref.k) and torch.equal(vb.cpu(), ref.v)
    with pytest.raises(RuntimeError, match="overflow"):
        kv_append(kb, vb, _randn(b, h, 30, d, seed=1, dev=cuda),
                  _randn(b, h, 30, d, seed=2, dev=cuda), pos)
    # device position past capacity: no write, error bit set
    _lib.device_errors(cuda, clear=True)
    snapshot = kb.clone()
    bad = torch.tensor([ref.cap], dtype=torch.int64, device=cuda)
    kv_append(kb, vb, kn, vn, bad)
    assert _lib.device_errors(cuda, clear=True) & _lib.DEVERR_KV_OVERFLOW
    assert torch.equal(kb, snapshot)


# ------------------------------------------------- fused attention input

def _qk_ref(x, w, eps, cos, sin):
    # per-head RMSNorm then rotate-half RoPE, fp32 (oracle formulas); x [B, S, H, D]
    n = oracle.rmsnorm(x, w, eps)
    return oracle.rope_rotate_half(n, cos[:, :, None], sin[:, :, None])


@pytest.mark.parametrize("batch,seq,hq,hk,d,tdt", [
    (2, 300, 32, 8, 128, torch.bfloat16), (1, 1, 16, 8, 128, torch.bfloat16),
    (3, 5, 4, 2, 64, torch.bfloat16), (1, 7, 2, 1, 256, torch.bfloat16),
    (2, 9, 6, 3, 128, torch.float32), (1, 3, 40, 40, 64, torch.float32)])
def test_qk_norm_rope_kv(cuda, batch, seq, hq, hk, d, tdt):
    """tdt: dtype of the cos / sin tables and the per-head norm weights."""
    q = _randn(batch, seq, hq * d, seed=200, dev=cuda).view(batch, seq, hq, d)
    k = _randn(batch, seq, hk * d, seed=201, dev=cuda).view(batch, seq, hk, d)
    v = _randn(batch, seq, hk * d, seed=202, dev=cuda).view(batch, seq, hk, d)
    qw = (1 + 0.1 * _randn(d, seed=203, dev=cuda, dtype=torch.float32)).to(tdt)
    kw = (1 + 0.1 * _randn(d, seed=204, dev=cuda, dtype=torch.float32)).to(tdt)
    pos = torch.arange(seq).unsqueeze(0) + 11 * torch.arange(batch).unsqueeze(1)
    cs = [oracle.text_rope_cos_sin(p, d, 1e6) for p in pos]
    cos = torch.stack([c for c, _ in cs]).to(tdt).to(cuda)
    sin = torch.stack([x for _, x in cs]).to(tdt).to(cuda)
    q_ref = _qk_ref(q.cpu(), qw.cpu(), 1e-6, cos.cpu(), sin.cpu())
    k_ref = _qk_ref(k.cpu(), kw.cpu(), 1e-6, cos.cpu(), sin.cpu())
    cap, start = seq + 9, 4
    kb = torch.zeros(batch, hk, cap, d, device=cuda, dtype=torch.bfloat16)
    vb = torch.zeros_like(kb)
    q1 = q.clone()
    stats.clear()
    qk_norm_rope_kv(q1, k.clone(), v, qw, kw, 1e-6, 1e-6, cos, sin, kb, vb, start)
    assert stats["umic_qk_norm_rope_kv"] == 1
    _close(q1, q_ref)
    _close(kb[:, :, start:start + seq].transpose(1, 2), k_ref)
    assert torch.equal(vb[:, :, start:start + seq].transpose(1, 2).cpu(), v.cpu())
    assert int(kb[:, :, :start].count_nonzero()) == 0  # nothing outside the new slots
    assert int(kb[:, :, start + seq:].count_nonzero()) == 0
    # without a cache: k rotated in place
    q2, k2 = q.clone(), k.clone()
    qk_norm_rope_kv(q2, k2, None, qw, kw, 1e-6, 1e-6, cos, sin)
    _close(q2, q_ref)
    _close(k2, k_ref)
    # device position (graph replay) writes the same bytes
    if seq == 1:
        kb2, vb2 = torch.zeros_like(kb), torch.zeros_like(vb)
        dpos = torch.tensor([start], device=cuda, dtype=torch.int64)
        qk_norm_rope_kv(q.clone(), k.clone(), v, qw, kw, 1e-6, 1e-6, cos, sin, kb2, vb2, dpos)
        assert torch.equal(kb2, kb) and torch.equal(vb2, vb)


def test_qk_norm_rope_kv_overflow(cuda):
    q = _randn(1, 4, 2, 128, seed=210, dev=cuda)
    k = _randn(1, 4, 1, 128, seed=211, dev=cuda)
    cos = torch.ones(1, 4, 128, device=cuda, dtype=torch.bfloat16)
    sin = torch.zeros_like(cos)
    kb = torch.zeros(1, 1, 6, 128, device=cuda, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="overflow"):
        qk_norm_rope_kv(q, k, k, None, None, 1e-6, 1e-6, cos, sin, kb, kb.clone(), 3)


@pytest.mark.parametrize("m", [1, 8, 20])
def test_gemv_multi_qkv(cuda, m):
    x = _randn(m, 4096, seed=220, dev=cuda)
    ws = [_randn(n, 4096, seed=221 + i, dev=cuda, scale=0.02)
          for i, n in enumerate((4096, 1024, 1000))]
    bs = [None, _randn(1024, seed=230, dev=cuda), None]
    stats.clear()
    outs = linear_gemv_multi(x, ws, bs)
    assert stats["umic_gemv_multi"] == 1
    for o, w, b in zip(outs, ws, bs):
        _close(o, oracle.linear(x.cpu(), w.cpu(), None if b is None else b.cpu()))


# ------------------------------------------------------------------ GEMV

@pytest.mark.parametrize("m,n,k", [(1, 4096, 4096), (8, 4096, 4096), (3, 1000, 4096),
                                   (17, 2048, 2048), (63, 256, 12288), (1, 24, 40)])
@pytest.mark.parametrize("with_bias", [False, True])
def test_gemv(cuda, m, n, k, with_bias):
    x = _randn(m, k, seed=50, dev=cuda)
    w = _randn(n, k, seed=51, dev=cuda, scale=0.02)
    bias = _randn(n, seed=52, dev=cuda) if with_bias else None
    stats.clear()
    y = linear_gemv(x, w, bias)
    assert stats["umic_gemv"] == 1
    _close(y, oracle.linear(x.cpu(), w.cpu(), None if bias is None else bias.cpu()))


@pytest.mark.parametrize("m,n,k", [(1, 12288, 4096), (8, 12288, 4096), (5, 8192, 2048),
                                   (40, 512, 1024)])
def test_gemv_gate_silu_mul(cuda, m, n, k):
    x = _randn(m, k, seed=53, dev=cuda)
    wg = _randn(n, k, seed=54, dev=cuda, scale=0.02)
    wu = _randn(n, k, seed=55, dev=cuda, scale=0.02)
    stats.clear()
    h = gate_silu_mul_nk(x, wg, wu)
    assert stats["umic_gemv_gate_silu_mul"] == 1
    _close(h, oracle.gate_silu_mul(x.cpu(), wg.cpu().t(), wu.cpu().t()))


# ------------------------------------------- GEMV engines (streaming vs cluster)

def _gemv_abi(x, w, bias, ws, flags=0):
    """umic_gemv through the C ABI with an explicit workspace (ptr, bytes) or none."""
    m, k = x.shape
    n = w.shape[0]
    y = torch.empty(m, n, device=x.device, dtype=torch.bfloat16)
    _lib.call("umic_gemv", x.device, x.data_ptr(), k, w.data_ptr(), k, _lib.ptr(bias),
              y.data_ptr(), n, m, n, k, ws[0], ws[1], flags)
    return y


@pytest.mark.parametrize("m,n,k", [(8, 4096, 4096), (1, 1000, 4104), (16, 64, 37888),
                                   (9, 3000, 520), (2, 151936, 256)])
def test_gemv_streaming_engine(cuda, m, n, k):
    """With a workspace (streaming engine) and without (cluster engine) the result matches
    the oracle; two streaming calls in a row are bit-identical (the kernel returns the
    workspace counters to zero and reduces split row blocks in a fixed order)."""
    x = _randn(m, k, seed=240, dev=cuda)
    w = _randn(n, k, seed=241, dev=cuda, scale=0.02)
    bias = _randn(n, seed=242, dev=cuda)
    ws = _lib.gemv_workspace(cuda, n)
    assert ws[0] is not None and ws[1] >= _lib.lib().umic_gemv_workspace_bytes(n)
    y1 = _gemv_abi(x, w, bias, ws)
    y2 = _gemv_abi(x, w, bias, ws)
    torch.cuda.synchronize()  # the weights are settled: they may be streamed early
    y3 = _gemv_abi(x, w, bias, ws, flags=_lib.GEMV_WEIGHTS_READY)
    y0 = _gemv_abi(x, w, bias, (None, 0))
    assert torch.equal(y1, y2) and torch.equal(y1, y3)
    ref = oracle.linear(x.cpu(), w.cpu(), bias.cpu())
    _close(y1, ref)
    _close(y0, ref)
    assert _lib.device_errors(cuda, clear=True) == 0


def test_gemv_streaming_workspace_reuse_across_shapes(cuda):
    """One workspace serves calls of growing and shrinking row counts in any order (the
    counters of a larger call must find zeros, whatever earlier calls left in the slots)."""
    ws = _lib.gemv_workspace(cuda, 40000)
    for i, (m, n, k) in enumerate([(1, 256, 4096), (8, 4096, 4096), (2, 12288, 2048),
                                   (1, 40000, 512), (8, 1000, 4096), (4, 12288, 4096)]):
        x = _randn(m, k, seed=260 + i, dev=cuda)
        w = _randn(n, k, seed=270 + i, dev=cuda, scale=0.02)
        _close(_gemv_abi(x, w, None, ws), oracle.linear(x.cpu(), w.cpu()))


def test_gemv_streaming_workspace_checks(cuda):
    x = _randn(8, 512, seed=243, dev=cuda)
    w = _randn(256, 512, seed=244, dev=cuda, scale=0.02)
    ptr, size = _lib.gemv_workspace(cuda, 256)
    with pytest.raises(_lib.UmicError, match="workspace"):
        _gemv_abi(x, w, None, (ptr, 1024))
    with pytest.raises(_lib.UmicError, match="aligned"):
        _gemv_abi(x, w, None, (ptr + 16, size - 16))
    with pytest.raises(_lib.UmicError, match="flags"):
        _gemv_abi(x, w, None, (ptr, size), flags=6)
    # the workspace is untouched by rejected calls: a proper call still matches
    _close(_gemv_abi(x, w, None, (ptr, size)), oracle.linear(x.cpu(), w.cpu()))


def test_gemv_multi_unaligned_segments_use_cluster_engine(cuda):
    """Segment boundaries off the 64-row grid of the streaming engine run the cluster
    engine (boundaries on 16 rows), with the same results."""
    x = _randn(4, 1024, seed=245, dev=cuda)
    ws = [_randn(n, 1024, seed=246 + i, dev=cuda, scale=0.02) for i, n in enumerate((1008, 40))]
    stats.clear()
    outs = linear_gemv_multi(x, ws)
    assert stats["umic_gemv_multi"] == 1
    for o, w in zip(outs, ws):
        _close(o, oracle.linear(x.cpu(), w.cpu()))


def test_gemv_gated_streaming_repeatable(cuda):
    x = _randn(8, 4096, seed=250, dev=cuda)
    wg = _randn(12288, 4096, seed=251, dev=cuda, scale=0.02)
    wu = _randn(12288, 4096, seed=252, dev=cuda, scale=0.02)
    h1 = gate_silu_mul_nk(x, wg, wu)
    h2 = gate_silu_mul_nk(x, wg, wu)
    assert torch.equal(h1, h2)
    _close(h1, oracle.gate_silu_mul(x.cpu(), wg.cpu().t(), wu.cpu().t()))


# ------------------------------------------- GEMV with the residual add in its epilogue

@pytest.mark.parametrize("m", [1, 8, 16])
def test_gemv_residual_epilogue(cuda, m):
    from umic_b200.kernels.linear import linear_gemv_residual

    h = _randn(m, 12288, seed=300, dev=cuda)
    wd = _randn(4096, 12288, seed=301, dev=cuda, scale=0.02)
    bias = _randn(4096, seed=304, dev=cuda)
    res_in = _randn(m, 4096, seed=302, dev=cuda)
    stats.clear()
    out = linear_gemv_residual(h, wd, res_in, bias, weights_ready=True)
    assert stats["umic_gemv_residual"] == 1 and stats["gemv_residual_fallback"] == 0
    _close(out, oracle.linear(h.cpu(), wd.cpu(), bias.cpu()) + res_in.cpu().float())
    # y may be the residual buffer itself
    y = res_in.clone()
    ws, ws_bytes = _lib.gemv_workspace(cuda, 4096)
    _lib.call("umic_gemv_residual", cuda, h.data_ptr(), h.stride(0), wd.data_ptr(),
              wd.stride(0), bias.data_ptr(), y.data_ptr(), y.stride(0), y.data_ptr(),
              y.stride(0), m, 4096, 12288, ws, ws_bytes, 0)
    assert torch.equal(y, out)


def test_gemv_residual_outside_streaming_engine(cuda):
    from umic_b200.kernels.linear import linear_gemv_residual

    h = _randn(20, 12288, seed=303, dev=cuda)
    wd = _randn(4096, 12288, seed=301, dev=cuda, scale=0.02)
    res_in = _randn(20, 4096, seed=305, dev=cuda)
    stats.clear()
    out = linear_gemv_residual(h, wd, res_in)  # 20 rows: GEMV, then the add
    assert stats["gemv_residual_fallback"] == 1 and stats["umic_gemv"] == 1
    _close(out, oracle.linear(h.cpu(), wd.cpu()) + res_in.cpu().float())
    with pytest.raises(ValueError):
        linear_gemv_residual(h, wd, res_in[:8])


# ------------------------------------------------------------------ GEMM

def _gpu_ref_linear(x, w, bias=None, act=None, residual=None):
    torch.backends.cuda.matmul.allow_tf32 = False
    y = x.float() @ w.float().t()
    if bias is not None:
        y = y + bias.float()
    if act == "gelu":
        y = torch.nn.functional.gelu(y)
    elif act == "gelu_tanh":
        y = torch.nn.functional.gelu(y, approximate="tanh")
    if residual is not None:
        y = y + residual.float()
    return y


@pytest.mark.parametrize("m,n,k", [(3100, 4096, 4096), (130, 256, 64), (1, 512, 128),
                                   (257, 520, 200), (16384, 1280, 1176), (64, 2048, 2048)])
def test_gemm(cuda, m, n, k):
    x = _randn(m, k, seed=60, dev=cuda)
    w = _randn(n, k, seed=61, dev=cuda, scale=0.02)
    stats.clear()
    y = linear(x, w)
    assert stats["umic_gemm"] == 1 and stats["linear_fallback"] == 0
    _close(y, _gpu_ref_linear(x, w))
    # the first and last row blocks also against the CPU oracle (fp32 restatement)
    for rows in (slice(0, 64), slice(max(0, m - 64), m)):
        _close(y[rows], oracle.linear(x[rows].cpu(), w.cpu()))


@pytest.mark.parametrize("m,n,k,act,res", [
    (256, 2048, 2048, None, False),       # the flow expert's q/o at 4 episodes: 8 tiles, 8 ranges
    (256, 2048, 8192, None, True),        # its down_proj, residual in the epilogue
    (512, 1024, 4096, "gelu_tanh", False),  # bias + GELU after the split sum
    (100, 2048, 2048, None, False),       # single-CTA tiles
    (300, 520, 1000, None, True),         # ragged rows, columns and k: 4 ranges
    (1024, 2048, 2048, None, False),      # 32 tiles: 2 ranges of 4 chunks each
    (256, 2048, 768, None, False),        # 3 ranges (chunks 2 / 3 / 3)
    (256, 2048, 1280, None, True),        # 5 ranges
    (256, 1024, 1536, None, False),       # 6 ranges
    (512, 1024, 1792, "gelu", False),     # 7 ranges (6 partner blocks per owned chunk)
])
def test_gemm_split_k(cuda, m, n, k, act, res):
    """Under-filled tile grids run split-K (each k range of a tile half owns some of its
    32-column chunks and sums every range's partial of them in range order): against
    fp32, against the unsplit kernel, and deterministic from call to call."""
    x = _randn(m, k, seed=70, dev=cuda)
    w = _randn(n, k, seed=71, dev=cuda, scale=0.02)
    b = _randn(n, seed=72, dev=cuda) if act else None
    r = _randn(m, n, seed=73, dev=cuda) if res else None
    assert _lib.lib().umic_gemm_workspace_bytes(m, n, k) > 0
    stats.clear()
    y = linear(x, w, b, act=act, residual=r)
    assert stats["umic_gemm_split_k"] == 1
    _close(y, _gpu_ref_linear(x, w, b, act, r))
    _close(y[:64], oracle.linear(x[:64].cpu(), w.cpu(), None if b is None else b.cpu(), act,
                                 None if r is None else r[:64].cpu()))
    y1 = linear(x, w, b, act=act, residual=r, split_k=False)
    assert oracle.rel_err(y, y1) <= 2e-3  # the same sums in another order
    assert torch.equal(y, linear(x, w, b, act=act, residual=r))


def test_gemm_small_vs_cpu_oracle(cuda):
    x = _randn(200, 136, seed=62, dev=cuda)
    w = _randn(264, 136, seed=63, dev=cuda, scale=0.05)
    _close(linear(x, w), oracle.linear(x.cpu(), w.cpu()))


@pytest.mark.parametrize("act", [None, "gelu", "gelu_tanh"])
def test_gemm_bias_act_residual(cuda, act):
    m, n, k = 300, 1280, 1176
    x = _randn(m, k, seed=64, dev=cuda)
    w = _randn(n, k, seed=65, dev=cuda, scale=0.02)
    b = _randn(n, seed=66, dev=cuda)
    r = _randn(m, n, seed=67, dev=cuda)
    y = linear(x, w, b, act=act, residual=r)
    _close(y, oracle.linear(x.cpu(), w.cpu(), b.cpu(), act, r.cpu()))


@pytest.mark.parametrize("m,n,k", [(3100, 12288, 4096), (64, 8192, 2048), (100, 128, 64),
                                   (130, 264, 136)])
def test_gemm_gate_silu_mul(cuda, m, n, k):
    x = _randn(m, k, seed=70, dev=cuda)
    wg = _randn(n, k, seed=71, dev=cuda, scale=0.02)
    wu = _randn(n, k, seed=72, dev=cuda, scale=0.02)
    stats.clear()
    h = gate_silu_mul(x, wg.t(), wu.t())  # reference convention: [K, N] .t() views
    assert stats["umic_gemm_gate_silu_mul"] == 1
    torch.backends.cuda.matmul.allow_tf32 = False
    g = x.float() @ wg.float().t()
    u = x.float() @ wu.float().t()
    _close(h, torch.nn.functional.silu(g) * u)


def test_gemm_repeat_deterministic(cuda):
    x = _randn(1000, 1024, seed=80, dev=cuda)
    w = _randn(768, 1024, seed=81, dev=cuda, scale=0.02)
    a = linear(x, w)
    b = linear(x, w)
    assert torch.equal(a, b)


# --------------------------------------------- attention over a cached prefix

def _attn_ref(q, k, v, mask, scale):
    """fp32 softmax(scale q k^T, masked) v with grouped heads -> [B, T, Hq, D]; rows
    that attend to nothing are zeros (the kernel's convention)."""
    g = q.shape[1] // k.shape[1]
    kf = k.float().repeat_interleave(g, 1)
    vf = v.float().repeat_interleave(g, 1)
    s = (q.float() @ kf.transpose(-1, -2)) * scale
    if mask is not None:
        s = s.masked_fill(~mask[..., : k.shape[2]], float("-inf"))
    p = torch.nan_to_num(torch.softmax(s, -1), nan=0.0)
    return (p @ vf).transpose(1, 2)


@pytest.mark.parametrize("b,hq,hkv,t,lk,cap,kind,d", [
    (4, 16, 8, 64, 3164, 3172, "lower_right", 128),  # the flow expert's step (4 episodes)
    (2, 32, 8, 32, 1000, 1000, "lower_right", 128),  # 4 query heads per KV head, 128 rows
    (3, 8, 8, 16, 100, 128, None, 128),              # no mask, keys not a multiple of 64
    (2, 16, 8, 64, 64, 64, "lower_right", 128),      # one block: plain causal
    (2, 16, 8, 64, 700, 704, "random", 128),         # arbitrary mask, some rows see nothing
    (2, 4, 2, 8, 200, 200, "per_head", 128),         # a mask per query head
    (2, 16, 16, 1024, 1024, 1024, None, 80),         # the ViT: 128-patch tiles, head_dim 80
    (1, 4, 4, 200, 300, 304, "random", 128),         # tiles with a ragged last one, masked
    (1, 2, 2, 130, 77, 80, None, 96),                # ragged tiles and keys, head_dim 96
])
def test_attention_rows(cuda, b, hq, hkv, t, lk, cap, kind, d):
    from umic_b200.kernels.attention import attention_rows

    q = _randn(b, t, hq, d, seed=90, dev=cuda).transpose(1, 2)  # HF's [B, Hq, T, D] view
    kbuf = _randn(b, hkv, cap, d, seed=91, dev=cuda)
    vbuf = _randn(b, hkv, cap, d, seed=92, dev=cuda)
    k, v = kbuf[:, :, :lk], vbuf[:, :, :lk]  # prefix views of cache buffers
    mask = None
    if kind == "lower_right":
        mask = torch.ones(t, lk, dtype=torch.bool, device=cuda).tril(diagonal=lk - t)
        mask = mask[None, None].expand(b, 1, t, lk)
    elif kind == "random":
        g = torch.Generator(device="cpu").manual_seed(93)
        mask = (torch.rand(b, 1, t, lk + 5, generator=g) > 0.3).to(cuda)
        mask[0, 0, 3] = False  # a row with no visible key
    elif kind == "per_head":
        g = torch.Generator(device="cpu").manual_seed(94)
        mask = (torch.rand(b, hq, t, lk, generator=g) > 0.5).to(cuda)
        mask[..., 0] = True
    scale = d ** -0.5
    stats.clear()
    out = attention_rows(q, k, v, mask, scale)  # head dims below 128 are zero-padded inside
    assert out is not None and stats["umic_attention_rows"] == 1
    assert out.shape == (b, t, hq, d)
    ref = _attn_ref(q, k, v, mask, scale)
    _close(out, ref)
    if kind != "random":  # torch SDPA (bf16) on the same inputs, for scale
        sdpa = torch.nn.functional.scaled_dot_product_attention(
            q, k, v, attn_mask=mask, scale=scale, enable_gqa=True).transpose(1, 2)
        e_ours, e_sdpa = oracle.rel_err(out, ref), oracle.rel_err(sdpa, ref)
        print(f"attention_rows {kind}: l2 vs fp32 ours {e_ours:.2e}, torch sdpa {e_sdpa:.2e}")
        assert e_ours <= max(2e-3, 1.5 * e_sdpa)
    assert torch.equal(out, attention_rows(q, k, v, mask, scale))  # deterministic
    if kind == "random":
        assert float(out[0, 3].float().abs().max()) == 0.0


@pytest.mark.parametrize("b,h,t,lk", [(2, 1, 64, 3164), (1, 3, 5, 32), (3, 2, 7, 33), (1, 1, 1, 1)])
def test_mask_pack_bits(cuda, b, h, t, lk):
    g = torch.Generator(device="cpu").manual_seed(99)
    mask = (torch.rand(b, h, t, lk + 3, generator=g) > 0.5).to(cuda)
    words = (lk + 31) // 32
    bits = torch.full((b, h, t, words), -1, device=cuda, dtype=torch.int32)
    _lib.call("umic_mask_pack_bits", cuda, mask.data_ptr(), mask.stride(0), mask.stride(1),
              mask.stride(2), b, h, t, lk, bits.data_ptr(), bits.stride(0), bits.stride(1),
              bits.stride(2))
    m = torch.zeros(b, h, t, words * 32, dtype=torch.int64)
    m[..., :lk] = mask[..., :lk].cpu().long()
    ref = (m.view(b, h, t, words, 32) << torch.arange(32)).sum(-1)
    got = bits.cpu().long() & 0xFFFFFFFF
    assert torch.equal(got, ref)


def test_attention_rows_declines_uncovered_shapes(cuda):
    from umic_b200.kernels.attention import attention_rows

    q = _randn(1, 16, 100, 128, seed=95, dev=cuda)  # 2 heads x 100 rows per KV head
    k = _randn(1, 8, 300, 128, seed=96, dev=cuda)
    stats.clear()
    assert attention_rows(q, k, k, None, 0.1) is None
    q48 = _randn(1, 4, 8, 48, seed=97, dev=cuda)  # head_dim 48
    k48 = _randn(1, 2, 64, 48, seed=98, dev=cuda)
    assert attention_rows(q48, k48, k48, None, 0.1) is None
    assert stats["attention_rows_fallback"] == 2 and stats["umic_attention_rows"] == 0


def test_no_device_error_after_suite(cuda):
    assert _lib.device_errors(cuda, clear=True) == 0
