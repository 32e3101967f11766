"""LayerNorm and add+LayerNorm on the B200 kernels (umic_layernorm, umic_add_layernorm).

Same contract as the reference's layernorm.py (src/umic/kernels/layernorm.py:54-124):
mean / variance in fp32, one bf16 rounding, outputs in x's dtype and shape.
"""

from __future__ import annotations

import torch

from .. import _lib
from ._common import require_bf16, require_cuda, row_stride, rows_view, stats
from .rmsnorm import _w_dtype


def _affine(weight: torch.Tensor, bias: torch.Tensor | None, n: int):
    w = weight.contiguous()
    b = bias.contiguous() if bias is not None else torch.zeros_like(w)
    if b.dtype != w.dtype:
        b = b.to(w.dtype)
    if w.numel() != n or b.numel() != n:
        raise ValueError(f"layernorm: affine params must have {n} elements")
    return w, b


def layernorm(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None,
              eps: float) -> torch.Tensor:
    """y = bf16((x - mean) * rsqrt(var + eps) * weight + bias) over the last dim."""
    dev = require_cuda("layernorm", x, weight, bias)
    require_bf16("layernorm", x)
    shape = x.shape
    x2d, n = rows_view(x)
    w, b = _affine(weight, bias, n)
    out = torch.empty((x2d.shape[0], n), device=x.device, dtype=x.dtype)
    _lib.call("umic_layernorm", dev, x2d.data_ptr(), row_stride(x2d), w.data_ptr(),
              b.data_ptr(), _w_dtype(w), out.data_ptr(), n, x2d.shape[0], n, float(eps))
    stats["umic_layernorm"] += 1
    return out.reshape(shape)


def add_layernorm(x: torch.Tensor, residual: torch.Tensor, weight: torch.Tensor,
                  bias: torch.Tensor | None, eps: float) -> tuple[torch.Tensor, torch.Tensor]:
    """Return (layernorm(x + residual), x + residual), sum in fp32."""
    dev = require_cuda("add_layernorm", x, residual, weight, bias)
    require_bf16("add_layernorm", x, residual)
    if residual.shape != x.shape:
        raise ValueError("add_layernorm: x and residual shapes differ")
    shape = x.shape
    x2d, n = rows_view(x)
    r2d, _ = rows_view(residual)
    w, b = _affine(weight, bias, n)
    rows = x2d.shape[0]
    normed = torch.empty((rows, n), device=x.device, dtype=x.dtype)
    summed = torch.empty((rows, n), device=x.device, dtype=x.dtype)
    _lib.call("umic_add_layernorm", dev, x2d.data_ptr(), row_stride(x2d), r2d.data_ptr(),
              row_stride(r2d), w.data_ptr(), b.data_ptr(), _w_dtype(w), normed.data_ptr(), n,
              summed.data_ptr(), n, rows, n, float(eps))
    stats["umic_add_layernorm"] += 1
    return normed.reshape(shape), summed.reshape(shape)


# Names of the reference interface (src/umic/kernels/layernorm.py:54,102).
layernorm_triton = layernorm
add_layernorm_triton = add_layernorm
