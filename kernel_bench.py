"""Single-kernel micro-benchmark of the library against cuBLAS / eager torch.

    python kernel_bench.py [--out results.json]
    python kernel_bench.py --reference [--out results.json]   (the reference's own Triton
        kernels, from its offline install in baseline/_ref, beside this build's)

Each case is timed with CUDA events around one launch after 3 warm-up launches,
with a 256 MB buffer read between launches to flush L2 (a read leaves no dirty
lines whose write-back would land in the timed launch); the median of 20 is
reported as (ms, GB/s or TFLOP/s). GEMM cases also report the relative error
against cuBLAS on the same inputs. The decode GEMV shapes are also timed back to
back over enough weight copies to exceed L2 (the regime of a decode step), for
the streaming engine (with a workspace) and the cluster engine (without).
"""

import json
import sys
from pathlib import Path

_ROOT = Path(__file__).resolve().parent
for _p in (_ROOT, _ROOT / "umic-alpamayo_b200"):
    if str(_p) not in sys.path:
        sys.path.insert(0, str(_p))

import torch

from umic_b200.kernels import (add_layernorm, add_rmsnorm, apply_rotary_text_inplace,
                               apply_rotary_vision, gate_silu_mul_nk, linear, linear_gemv)


def main() -> None:
    dev = torch.device("cuda", 0)
    torch.manual_seed(0)
    flush = torch.ones(64 * 1024 * 1024, dtype=torch.int32, device=dev)

    def t(fn, iters=20, flushl2=True):
        for _ in range(3): fn()
        torch.cuda.synchronize()
        ts = []
        for _ in range(iters):
            if flushl2: flush.sum()
            s = torch.cuda.Event(enable_timing=True); e = torch.cuda.Event(enable_timing=True)
            s.record(); fn(); e.record(); torch.cuda.synchronize()
            ts.append(s.elapsed_time(e))
        ts.sort(); return ts[len(ts)//2]

    res = {}
    bf = torch.bfloat16
    x = torch.randn(3100, 4096, device=dev, dtype=bf); r = torch.randn_like(x); w = torch.randn(4096, device=dev, dtype=bf)
    ms = t(lambda: add_rmsnorm(x, r, w, 1e-6)); res["add_rmsnorm_3100x4096"] = (ms, 101.6e6 / (ms * 1e-3) / 1e9)
    xv = torch.randn(16384, 1280, device=dev, dtype=bf); rv = torch.randn_like(xv); wv = torch.ones(1280, device=dev, dtype=bf); bv = torch.zeros(1280, device=dev, dtype=bf)
    ms = t(lambda: add_layernorm(xv, rv, wv, bv, 1e-6)); res["add_layernorm_16384x1280"] = (ms, 16384*1280*2*4 / (ms*1e-3) / 1e9)
    q = torch.randn(1, 3100, 32, 128, device=dev, dtype=bf).transpose(1, 2); k = torch.randn(1, 3100, 8, 128, device=dev, dtype=bf).transpose(1, 2)
    cos = torch.randn(1, 3100, 128, device=dev, dtype=bf); sin = torch.randn_like(cos)
    ms = t(lambda: apply_rotary_text_inplace(q, k, cos, sin)); res["text_rope"] = (ms, 65.1e6/(ms*1e-3)/1e9)
    qkv = torch.randn(16384, 3, 16, 80, device=dev, dtype=bf); qq, kk, _ = qkv.unbind(1)
    cv = torch.randn(16384, 80, device=dev); sv = torch.randn_like(cv)
    ms = t(lambda: apply_rotary_vision(qq, kk, cv, sv)); res["vision_rope_qk"] = (ms, 2*94.4e6/(ms*1e-3)/1e9)
    for (m, n, kd) in [(3100, 4096, 4096), (24800, 4096, 4096), (8192, 8192, 8192)]:
        a = torch.randn(m, kd, device=dev, dtype=bf); b = torch.randn(n, kd, device=dev, dtype=bf) * 0.02
        fl = 2.0 * m * n * kd
        ms = t(lambda: linear(a, b)); res[f"gemm_{m}x{n}x{kd}"] = (ms, fl / (ms*1e-3) / 1e12)
        ms = t(lambda: torch.nn.functional.linear(a, b)); res[f"cublas_{m}x{n}x{kd}"] = (ms, fl / (ms*1e-3) / 1e12)
        err = ((linear(a, b).float() - torch.nn.functional.linear(a, b).float()).norm() / torch.nn.functional.linear(a, b).float().norm()).item()
        res[f"gemm_{m}x{n}x{kd}_relerr"] = err
    for m in [3100, 24800]:
        a = torch.randn(m, 4096, device=dev, dtype=bf); wg = torch.randn(12288, 4096, device=dev, dtype=bf)*0.02; wu = torch.randn_like(wg)
        fl = 2.0 * 2 * m * 12288 * 4096
        ms = t(lambda: gate_silu_mul_nk(a, wg, wu)); res[f"dual_{m}"] = (ms, fl/(ms*1e-3)/1e12)
        ms = t(lambda: torch.nn.functional.silu(torch.nn.functional.linear(a, wg)) * torch.nn.functional.linear(a, wu)); res[f"eager_dual_{m}"] = (ms, fl/(ms*1e-3)/1e12)
    for (m, n, kd) in [(8, 1024, 4096), (8, 4096, 4096), (8, 4096, 12288), (1, 1024, 4096)]:
        xs = torch.randn(m, kd, device=dev, dtype=bf); W = torch.randn(n, kd, device=dev, dtype=bf)
        ms = t(lambda: linear_gemv(xs, W)); res[f"gemv_m{m}_{n}x{kd}"] = (ms, W.numel()*2/(ms*1e-3)/1e9)
        ms = t(lambda: torch.nn.functional.linear(xs, W)); res[f"cublas_gemv_m{m}_{n}x{kd}"] = (ms, W.numel()*2/(ms*1e-3)/1e9)
    for m in [1, 8]:
        xs = torch.randn(m, 4096, device=dev, dtype=bf); W = torch.randn(12288, 4096, device=dev, dtype=bf)
        ms = t(lambda: linear_gemv(xs, W)); res[f"gemv_m{m}_12288x4096"] = (ms, W.numel()*2/(ms*1e-3)/1e9)
        ms = t(lambda: torch.nn.functional.linear(xs, W)); res[f"cublas_gemv_m{m}"] = (ms, W.numel()*2/(ms*1e-3)/1e9)
        W2 = torch.randn(151936, 4096, device=dev, dtype=bf)
        ms = t(lambda: linear_gemv(xs, W2)); res[f"gemv_m{m}_lmhead"] = (ms, W2.numel()*2/(ms*1e-3)/1e9)
        del W2
    # decode GEMV engines, back to back over rotating weight copies (> 600 MB in total)
    from umic_b200 import _lib

    def gemv_call(xs, W, ws):
        m_, k_ = xs.shape
        n_ = W.shape[0]
        y = torch.empty(m_, n_, device=dev, dtype=bf)
        _lib.call("umic_gemv", dev, xs.data_ptr(), k_, W.data_ptr(), k_, None, y.data_ptr(), n_,
                  m_, n_, k_, ws[0], ws[1], _lib.GEMV_WEIGHTS_READY if ws[0] else 0)

    for (n, kd) in [(4096, 4096), (6144, 4096), (12288, 4096), (4096, 12288), (151936, 4096)]:
        copies = max(2, -(-600_000_000 // (n * kd * 2)))
        Ws = [torch.randn(n, kd, device=dev, dtype=bf) for _ in range(copies)]
        xs = torch.randn(8, kd, device=dev, dtype=bf)
        for name, ws in (("stream", _lib.gemv_workspace(dev, n)), ("cluster", (None, 0))):
            for i in range(3):
                gemv_call(xs, Ws[i % copies], ws)
            torch.cuda.synchronize()
            reps = copies * 4
            s0 = torch.cuda.Event(enable_timing=True); e0 = torch.cuda.Event(enable_timing=True)
            s0.record()
            for i in range(reps):
                gemv_call(xs, Ws[i % copies], ws)
            e0.record(); torch.cuda.synchronize()
            ms = s0.elapsed_time(e0) / reps
            res[f"gemv_b2b_{name}_m8_{n}x{kd}"] = (ms, n * kd * 2 / (ms * 1e-3) / 1e9)
        del Ws
    # The decode step's GEMV sequence as the decode graph runs it: 36 layers x (q/k/v in
    # one launch, o_proj, gate+up gated, down_proj) + lm_head, x of 8 rows, captured in a
    # CUDA graph and replayed; weights (15.1 GB) stream from HBM every replay.
    from umic_b200.kernels.linear import linear_gemv_multi
    layers = 36
    mats = []
    for _ in range(layers):
        mats.append(dict(q=torch.randn(4096, 4096, device=dev, dtype=bf) * 0.02,
                         k=torch.randn(1024, 4096, device=dev, dtype=bf) * 0.02,
                         v=torch.randn(1024, 4096, device=dev, dtype=bf) * 0.02,
                         o=torch.randn(4096, 4096, device=dev, dtype=bf) * 0.02,
                         g=torch.randn(12288, 4096, device=dev, dtype=bf) * 0.02,
                         u=torch.randn(12288, 4096, device=dev, dtype=bf) * 0.02,
                         d=torch.randn(4096, 12288, device=dev, dtype=bf) * 0.02))
    head = torch.randn(151936, 4096, device=dev, dtype=bf) * 0.02
    chain_bytes = sum(sum(t.numel() for t in m_.values()) for m_ in mats) * 2 + head.numel() * 2
    xs = torch.randn(8, 4096, device=dev, dtype=bf)

    def step():
        h = xs
        for m_ in mats:
            q, _, _ = linear_gemv_multi(h, [m_["q"], m_["k"], m_["v"]], weights_ready=True)
            a = linear_gemv(q, m_["o"], weights_ready=True)
            gu = gate_silu_mul_nk(a, m_["g"], m_["u"], weights_ready=True)
            h = linear_gemv(gu, m_["d"], weights_ready=True)
        return linear_gemv(h, head, weights_ready=True)

    for _ in range(2):
        step()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step()
    graph.replay()
    torch.cuda.synchronize()
    ms = t(graph.replay, iters=10, flushl2=False)
    res["decode_gemv_chain_m8"] = (ms, chain_bytes / (ms * 1e-3) / 1e9)
    del mats, head, graph
    for kk_, v in res.items():
        print(kk_, v)
    if "--out" in sys.argv:
        json.dump(res, open(sys.argv[sys.argv.index("--out") + 1], "w"), indent=1)


def reference_side_by_side() -> dict:
    """The reference's own Triton kernels (its `umic` package, installed offline into
    baseline/_ref) beside this build's kernels, on the BASELINE cfg1 / cfg2 shapes and the
    q/o projection, timed the same way (one launch between L2 flushes, median of 20).
    Also reports the relative L2 difference between the two outputs."""
    ref_dir = _ROOT / "baseline" / "_ref"
    if not (ref_dir / "umic").is_dir():
        return {"unavailable": "the reference is not installed in baseline/_ref"}
    sys.path.insert(0, str(ref_dir))
    from umic.kernels import fused_ffn as rf_ffn, layernorm as rf_ln, linear as rf_lin, \
        rmsnorm as rf_rms, rope as rf_rope

    if not rf_ffn.HAS_TRITON:
        return {"unavailable": "Triton did not import in the reference package"}
    dev = torch.device("cuda", 0)
    bf = torch.bfloat16
    flush = torch.ones(64 * 1024 * 1024, dtype=torch.int32, device=dev)

    def t(fn, iters=20):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        ts = []
        for _ in range(iters):
            flush.sum()
            s0 = torch.cuda.Event(enable_timing=True)
            e0 = torch.cuda.Event(enable_timing=True)
            s0.record()
            fn()
            e0.record()
            torch.cuda.synchronize()
            ts.append(s0.elapsed_time(e0))
        ts.sort()
        return ts[len(ts) // 2]

    def rel(a, b):
        return float((a.float() - b.float()).norm() / b.float().norm())

    g = torch.Generator(device=dev).manual_seed(0)
    res = {}

    def row(name, ours, theirs, units, work, pick=lambda o: o):
        ms_o, ms_t = t(ours), t(theirs)
        res[name] = {"ours_ms": ms_o, "reference_triton_ms": ms_t, "speedup": ms_t / ms_o,
                     units: [work / (ms_o * 1e-3), work / (ms_t * 1e-3)],
                     "rel_l2_diff": rel(pick(ours()), pick(theirs()))}

    # cfg1 gate/up (fused SiLU-mul) and the q/o projection at one episode
    x = torch.randn(3100, 4096, device=dev, dtype=bf, generator=g)
    wg = torch.randn(12288, 4096, device=dev, dtype=bf, generator=g) * 0.02
    wu = torch.randn(12288, 4096, device=dev, dtype=bf, generator=g) * 0.02
    row("gate_silu_mul_3100x12288x4096", lambda: gate_silu_mul_nk(x, wg, wu),
        lambda: rf_ffn.gate_silu_mul(x, wg.t(), wu.t()), "tflops", 4.0 * 3100 * 12288 * 4096 / 1e12)
    wq = torch.randn(4096, 4096, device=dev, dtype=bf, generator=g) * 0.02
    row("linear_3100x4096x4096", lambda: linear(x, wq), lambda: rf_lin.linear_triton(x, wq),
        "tflops", 2.0 * 3100 * 4096 * 4096 / 1e12)
    wd = torch.randn(4096, 12288, device=dev, dtype=bf, generator=g) * 0.02
    h = torch.randn(3100, 12288, device=dev, dtype=bf, generator=g)
    row("linear_3100x4096x12288", lambda: linear(h, wd), lambda: rf_lin.linear_triton(h, wd),
        "tflops", 2.0 * 3100 * 4096 * 12288 / 1e12)
    # cfg2 (a) add+RMSNorm, (b) add+LayerNorm, (c) text RoPE, (d) vision RoPE
    r = torch.randn_like(x)
    w = (1 + 0.05 * torch.randn(4096, device=dev, generator=g)).to(bf)
    row("add_rmsnorm_3100x4096", lambda: add_rmsnorm(x, r, w, 1e-6),
        lambda: rf_rms.add_rmsnorm_triton(x, r, w, 1e-6), "gbs", 101.6e6 / 1e9,
        pick=lambda o: o[0])
    xv = torch.randn(16384, 1280, device=dev, dtype=bf, generator=g)
    rv = torch.randn_like(xv)
    wv = torch.ones(1280, device=dev, dtype=bf)
    bv = torch.zeros(1280, device=dev, dtype=bf)
    row("add_layernorm_16384x1280", lambda: add_layernorm(xv, rv, wv, bv, 1e-6),
        lambda: rf_ln.add_layernorm_triton(xv, rv, wv, bv, 1e-6), "gbs", 167.8e6 / 1e9,
        pick=lambda o: o[0])
    q = torch.randn(1, 3100, 32, 128, device=dev, dtype=bf, generator=g).transpose(1, 2)
    k = torch.randn(1, 3100, 8, 128, device=dev, dtype=bf, generator=g).transpose(1, 2)
    cos = torch.randn(1, 3100, 128, device=dev, dtype=bf, generator=g)
    sin = torch.randn_like(cos)
    text_rope = rf_rope.make_text_rope(None)
    q2, k2 = q.clone(), k.clone()
    ms_o = t(lambda: apply_rotary_text_inplace(q2, k2, cos, sin))
    ms_t = t(lambda: text_rope(q, k, cos, sin))
    q3, k3 = q.clone(), k.clone()
    apply_rotary_text_inplace(q3, k3, cos, sin)
    qr, kr = text_rope(q, k, cos, sin)
    res["text_rope_3100"] = {"ours_ms": ms_o, "reference_triton_ms": ms_t, "speedup": ms_t / ms_o,
                             "gbs": [65.1e6 / (ms_o * 1e-3) / 1e9, 65.1e6 / (ms_t * 1e-3) / 1e9],
                             "rel_l2_diff": max(rel(q3, qr), rel(k3, kr))}
    qkv = torch.randn(16384, 3, 16, 80, device=dev, dtype=bf, generator=g)
    qq, kk, _ = qkv.unbind(1)
    cv = torch.randn(16384, 80, device=dev, generator=g)
    sv = torch.randn_like(cv)
    ms_o = t(lambda: apply_rotary_vision(qq, kk, cv, sv))
    ms_t = t(lambda: rf_rope.apply_rotary_vision_triton(qq, kk, cv, sv))
    q4, k4 = qq.clone(), kk.clone()
    apply_rotary_vision(q4, k4, cv, sv)
    qr, kr = rf_rope.apply_rotary_vision_triton(qq, kk, cv, sv)
    res["vision_rope_16384"] = {"ours_ms": ms_o, "reference_triton_ms": ms_t,
                                "speedup": ms_t / ms_o,
                                "gbs": [2 * 94.4e6 / (ms_o * 1e-3) / 1e9,
                                        2 * 94.4e6 / (ms_t * 1e-3) / 1e9],
                                "rel_l2_diff": max(rel(q4, qr), rel(k4, kr))}
    return res


if __name__ == "__main__":
    if "--reference" in sys.argv:
        out = reference_side_by_side()
        print(json.dumps(out, indent=1))
        if "--out" in sys.argv:
            json.dump(out, open(sys.argv[sys.argv.index("--out") + 1], "w"), indent=1)
    else:
        main()
