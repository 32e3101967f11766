"""Projections on the B200 kernels: tcgen05 GEMM (umic_gemm) and the decode GEMV (umic_gemv).

`linear(x, weight, bias, act, residual)` mirrors the reference's linear_triton
(src/umic/kernels/linear.py:118-145): x [M, K] times an nn.Linear weight
[N, K] without copying it, optional bias, optional GELU epilogue ("gelu" is
the erf form the reference used; "gelu_tanh" is HF's gelu_pytorch_tanh), plus
an optional fused residual add. `linear_gemv` is the HBM-bound path for fewer
than FUSE_MIN_ROWS rows (the reference left those on cuBLAS,
src/umic/integrate.py:104-105).
Shapes the kernels reject (N or K not a multiple of 8, misaligned views) go to
torch's own GPU linear, as the reference leaves unmatched sites on cuBLAS;
the `stats` counter records every such call.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

from .. import _lib
from ._common import require_bf16, require_cuda, row_stride, stats

_ACTS = {None: _lib.EPI_NONE, "gelu": _lib.EPI_GELU_ERF, "gelu_erf": _lib.EPI_GELU_ERF,
         "gelu_tanh": _lib.EPI_GELU_TANH}

GEMV_MAX_ROWS = 64


def _torch_linear(x2d, weight, bias, act, residual):
    y = F.linear(x2d, weight, bias)
    if act in ("gelu", "gelu_erf"):
        y = F.gelu(y)
    elif act == "gelu_tanh":
        y = F.gelu(y, approximate="tanh")
    if residual is not None:
        y = y + residual
    return y


def _k_major(t: torch.Tensor) -> torch.Tensor:
    return t if t.stride(-1) == 1 else t.contiguous()


def linear(x2d: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None = None,
           act: str | None = None, residual: torch.Tensor | None = None,
           split_k: bool = True) -> torch.Tensor:
    """y = act(x2d @ weight.T + bias) + residual on the tcgen05 GEMM. Shapes whose output
    tiles would leave most of the GPU idle run split-K through a per-device workspace
    (umic_gemm_ws) unless split_k is False."""
    if act not in _ACTS:
        raise ValueError(f"linear: unsupported act {act!r}")
    dev = require_cuda("linear", x2d, weight, bias, residual)
    require_bf16("linear", x2d, weight, bias, residual)
    m, k = x2d.shape
    n = weight.shape[0]
    if weight.shape[1] != k:
        raise ValueError(f"linear: x has K={k}, weight is {tuple(weight.shape)}")
    x2d = _k_major(x2d)
    weight = _k_major(weight)
    y = torch.empty((m, n), device=x2d.device, dtype=x2d.dtype)
    if residual is not None and residual.stride(-1) != 1:
        residual = residual.contiguous()
    ws, ws_bytes = _lib.gemm_workspace(dev, m, n, k) if split_k else (None, 0)
    args = (x2d.data_ptr(), row_stride(x2d), weight.data_ptr(), row_stride(weight),
            _lib.ptr(bias), _lib.ptr(residual),
            row_stride(residual) if residual is not None else 0, y.data_ptr(), n, m, n, k,
            _ACTS[act])
    if ws is not None:
        rc = _lib.try_call("umic_gemm_ws", dev, *args, ws, ws_bytes)
        stats["umic_gemm_split_k"] += 0 if rc else 1
    else:
        rc = _lib.try_call("umic_gemm", dev, *args)
    if rc:
        stats["linear_fallback"] += 1
        return _torch_linear(x2d, weight, bias, act, residual)
    stats["umic_gemm"] += 1
    return y


def linear_gemv(x2d: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None = None, *,
                weights_ready: bool = False) -> torch.Tensor:
    """y = x2d @ weight.T + bias for x2d with fewer than 64 rows (weight-streaming).

    weights_ready: the weight is not written by the kernel enqueued just before this
    call (true for module parameters inside a forward pass), so its stream may begin
    while that kernel is finishing."""
    dev = require_cuda("linear_gemv", x2d, weight, bias)
    require_bf16("linear_gemv", x2d, weight, bias)
    m, k = x2d.shape
    n = weight.shape[0]
    if m > GEMV_MAX_ROWS:
        raise ValueError(f"linear_gemv: {m} rows > {GEMV_MAX_ROWS}")
    x2d = _k_major(x2d)
    weight = _k_major(weight)
    y = torch.empty((m, n), device=x2d.device, dtype=x2d.dtype)
    ws, ws_bytes = _lib.gemv_workspace(dev, n)
    rc = _lib.try_call("umic_gemv", dev, x2d.data_ptr(), row_stride(x2d), weight.data_ptr(),
                       row_stride(weight), _lib.ptr(bias), y.data_ptr(), n, m, n, k, ws,
                       ws_bytes, _lib.GEMV_WEIGHTS_READY if weights_ready else 0)
    if rc:
        stats["gemv_fallback"] += 1
        return F.linear(x2d, weight, bias)
    stats["umic_gemv"] += 1
    return y


def linear_gemv_multi(x2d: torch.Tensor, weights: list[torch.Tensor],
                      biases: list[torch.Tensor | None] | None = None, *,
                      weights_ready: bool = False) -> list[torch.Tensor]:
    """[x2d @ w.T + b for each w] in one launch (x2d with fewer than 64 rows); used for
    the q/k/v projections of a decode step."""
    import ctypes

    dev = require_cuda("linear_gemv_multi", x2d, *weights)
    require_bf16("linear_gemv_multi", x2d, *weights)
    m, k = x2d.shape
    cnt = len(weights)
    biases = biases or [None] * cnt
    if m > GEMV_MAX_ROWS or not 1 <= cnt <= 3 or any(w.shape[1] != k for w in weights):
        raise ValueError("linear_gemv_multi: bad shapes")
    x2d = _k_major(x2d)
    weights = [_k_major(w) for w in weights]
    outs = [torch.empty((m, w.shape[0]), device=x2d.device, dtype=x2d.dtype) for w in weights]
    P = ctypes.c_void_p * cnt
    I = ctypes.c_int64 * cnt
    ws, ws_bytes = _lib.gemv_workspace(dev, sum(w.shape[0] for w in weights))
    rc = _lib.try_call("umic_gemv_multi", dev, x2d.data_ptr(), row_stride(x2d), cnt,
                       P(*[w.data_ptr() for w in weights]), I(*[row_stride(w) for w in weights]),
                       I(*[w.shape[0] for w in weights]), P(*[_lib.ptr(b) for b in biases]),
                       P(*[o.data_ptr() for o in outs]), I(*[o.shape[1] for o in outs]), m, k,
                       ws, ws_bytes, _lib.GEMV_WEIGHTS_READY if weights_ready else 0)
    if rc:
        stats["gemv_fallback"] += 1
        return [F.linear(x2d, w, b) for w, b in zip(weights, biases)]
    stats["umic_gemv_multi"] += 1
    return outs


# Name of the reference interface (src/umic/kernels/linear.py:118).
linear_triton = linear



def linear_gemv_residual(x2d: torch.Tensor, weight: torch.Tensor, residual: torch.Tensor,
                         bias: torch.Tensor | None = None, *,
                         weights_ready: bool = False) -> torch.Tensor:
    """y = x2d @ weight.T + bias + residual in one streaming-GEMV launch, the residual
    add in the epilogue (C ABI: umic_gemv_residual); x2d has at most 16 rows. Shapes
    outside the streaming engine run the GEMV and the add as two ops."""
    dev = require_cuda("linear_gemv_residual", x2d, weight, residual, bias)
    require_bf16("linear_gemv_residual", x2d, weight, residual, bias)
    m, k = x2d.shape
    n = weight.shape[0]
    if residual.shape != (m, n):
        raise ValueError(f"linear_gemv_residual: residual {tuple(residual.shape)} != {(m, n)}")
    x2d = _k_major(x2d)
    weight = _k_major(weight)
    residual = _k_major(residual)
    y = torch.empty((m, n), device=x2d.device, dtype=x2d.dtype)
    ws, ws_bytes = _lib.gemv_workspace(dev, n)
    rc = _lib.ERR_UNSUPPORTED
    if m <= 16 and ws is not None:
        rc = _lib.try_call("umic_gemv_residual", dev, x2d.data_ptr(), row_stride(x2d),
                           weight.data_ptr(), row_stride(weight), _lib.ptr(bias),
                           residual.data_ptr(), row_stride(residual), y.data_ptr(), n, m, n, k,
                           ws, ws_bytes, _lib.GEMV_WEIGHTS_READY if weights_ready else 0)
    if rc:
        stats["gemv_residual_fallback"] += 1
        return linear_gemv(x2d, weight, bias, weights_ready=weights_ready) + residual
    stats["umic_gemv_residual"] += 1
    return y
