"""gate_silu_mul on the B200 kernels: silu(x @ Wg) * (x @ Wu) in one pass.

`gate_silu_mul(x, w_gate, w_up)` keeps the reference's convention
(src/umic/kernels/fused_ffn.py:121-126): weights given as [K, N] — in practice
the free `.t()` views of nn.Linear weights (integrate.py:51-53). Those views
are handed to the kernels as the underlying [N, K] storage, so nothing is
copied. Rows >= FUSE_MIN_ROWS run the dual-accumulator tcgen05 GEMM
(umic_gemm_gate_silu_mul); fewer rows run the weight-streaming gated GEMV
(umic_gemv_gate_silu_mul). There is no CPU path: CPU tensors raise.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

from .. import _lib
from ._common import probe_begin, probe_end, require_bf16, require_cuda, row_stride, stats

FUSE_MIN_ROWS = 64


def _nk_from_kn(w: torch.Tensor) -> torch.Tensor:
    """[K, N] argument -> [N, K] K-major tensor (a view when w is a .t() view)."""
    wt = w.t()
    return wt if wt.stride(-1) == 1 else wt.contiguous()


def gate_silu_mul_nk(x2d: torch.Tensor, w_gate: torch.Tensor, w_up: torch.Tensor, *,
                     weights_ready: bool = False) -> torch.Tensor:
    """h = silu(x2d @ w_gate.T) * (x2d @ w_up.T) with nn.Linear-layout weights [N, K].

    weights_ready (GEMV regime only): the weights are not written by the kernel
    enqueued just before this call, so they may be streamed while it finishes."""
    dev = require_cuda("gate_silu_mul", x2d, w_gate, w_up)
    require_bf16("gate_silu_mul", x2d, w_gate, w_up)
    m, k = x2d.shape
    n = w_gate.shape[0]
    if w_gate.shape != (n, k) or w_up.shape != (n, k):
        raise ValueError(f"gate_silu_mul: weights {tuple(w_gate.shape)}/{tuple(w_up.shape)} "
                         f"vs x K={k}")
    if x2d.stride(-1) != 1:
        x2d = x2d.contiguous()
    if w_gate.stride(-1) != 1:
        w_gate = w_gate.contiguous()
    if w_up.stride(-1) != 1:
        w_up = w_up.contiguous()
    h = torch.empty((m, n), device=x2d.device, dtype=x2d.dtype)
    if m < FUSE_MIN_ROWS:
        if w_gate.stride(0) != w_up.stride(0):
            w_up = w_up.contiguous()
            w_gate = w_gate.contiguous()
        ws, ws_bytes = _lib.gemv_workspace(dev, n)
        rc = _lib.try_call("umic_gemv_gate_silu_mul", dev, x2d.data_ptr(), row_stride(x2d),
                           w_gate.data_ptr(), w_up.data_ptr(), row_stride(w_gate),
                           h.data_ptr(), n, m, n, k, ws, ws_bytes,
                           _lib.GEMV_WEIGHTS_READY if weights_ready else 0)
        name = "umic_gemv_gate_silu_mul"
    else:
        tok = probe_begin("umic_gemm_gate_silu_mul")
        rc = _lib.try_call("umic_gemm_gate_silu_mul", dev, x2d.data_ptr(), row_stride(x2d),
                           w_gate.data_ptr(), row_stride(w_gate), w_up.data_ptr(),
                           row_stride(w_up), h.data_ptr(), n, m, n, k)
        probe_end(tok)
        name = "umic_gemm_gate_silu_mul"
    if rc:
        stats["gate_silu_mul_fallback"] += 1
        return F.silu(F.linear(x2d, w_gate)) * F.linear(x2d, w_up)
    stats[name] += 1
    return h


def gate_silu_mul(x: torch.Tensor, w_gate: torch.Tensor, w_up: torch.Tensor) -> torch.Tensor:
    """silu(x @ w_gate) * (x @ w_up); x [M, K], w_gate / w_up [K, N]."""
    if x.dim() != 2 or w_gate.dim() != 2 or w_up.dim() != 2:
        raise ValueError("gate_silu_mul: expects 2-D x [M, K] and weights [K, N]")
    if w_gate.shape[0] != x.shape[1] or w_up.shape != w_gate.shape:
        raise ValueError(f"gate_silu_mul: shapes x{tuple(x.shape)} wg{tuple(w_gate.shape)} "
                         f"wu{tuple(w_up.shape)}")
    return gate_silu_mul_nk(x, _nk_from_kn(w_gate), _nk_from_kn(w_up))


# Name of the reference's fused path (src/umic/kernels/fused_ffn.py:93).
gate_silu_mul_triton = gate_silu_mul
