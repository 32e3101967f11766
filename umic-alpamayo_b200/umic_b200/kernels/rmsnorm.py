"""RMSNorm and add+RMSNorm on the B200 kernels (C ABI: umic_rmsnorm, umic_add_rmsnorm).

Same contract as the reference's rmsnorm.py (src/umic/kernels/rmsnorm.py:53-134):
fp32 statistics, one bf16 rounding, outputs freshly allocated in x's dtype
and shape. The add variant returns (normed, summed) with the sum taken in fp32
before its bf16 store.
"""

from __future__ import annotations

import torch

from .. import _lib
from ._common import require_bf16, require_cuda, row_stride, rows_view, stats


def _w_dtype(w: torch.Tensor) -> int:
    if w.dtype == torch.float32:
        return _lib.DTYPE_FP32
    if w.dtype == torch.bfloat16:
        return _lib.DTYPE_BF16
    raise TypeError(f"norm weight dtype {w.dtype} not supported (bf16 or fp32)")


def rmsnorm(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    """y = bf16(x * rsqrt(mean(x^2) + eps) * weight) over the last dim."""
    dev = require_cuda("rmsnorm", x, weight)
    require_bf16("rmsnorm", x)
    shape = x.shape
    x2d, n = rows_view(x)
    w = weight.contiguous()
    if w.numel() != n:
        raise ValueError(f"rmsnorm: weight has {w.numel()} elements, rows have {n}")
    out = torch.empty((x2d.shape[0], n), device=x.device, dtype=x.dtype)
    _lib.call("umic_rmsnorm", dev, x2d.data_ptr(), row_stride(x2d), w.data_ptr(), _w_dtype(w),
              out.data_ptr(), n, x2d.shape[0], n, float(eps))
    stats["umic_rmsnorm"] += 1
    return out.reshape(shape)


def add_rmsnorm(x: torch.Tensor, residual: torch.Tensor, weight: torch.Tensor,
                eps: float) -> tuple[torch.Tensor, torch.Tensor]:
    """Return (rmsnorm(x + residual) * weight, x + residual), sum in fp32."""
    dev = require_cuda("add_rmsnorm", x, residual, weight)
    require_bf16("add_rmsnorm", x, residual)
    if residual.shape != x.shape:
        raise ValueError(f"add_rmsnorm: shapes differ {tuple(x.shape)} vs {tuple(residual.shape)}")
    shape = x.shape
    x2d, n = rows_view(x)
    r2d, _ = rows_view(residual)
    w = weight.contiguous()
    if w.numel() != n:
        raise ValueError(f"add_rmsnorm: weight has {w.numel()} elements, rows have {n}")
    rows = x2d.shape[0]
    normed = torch.empty((rows, n), device=x.device, dtype=x.dtype)
    summed = torch.empty((rows, n), device=x.device, dtype=x.dtype)
    _lib.call("umic_add_rmsnorm", dev, x2d.data_ptr(), row_stride(x2d), r2d.data_ptr(),
              row_stride(r2d), w.data_ptr(), _w_dtype(w), normed.data_ptr(), n,
              summed.data_ptr(), n, rows, n, float(eps))
    stats["umic_add_rmsnorm"] += 1
    return normed.reshape(shape), summed.reshape(shape)


def rmsnorm_axpy(x: torch.Tensor, weight: torch.Tensor, eps: float, base: torch.Tensor,
                 alpha: float, out: torch.Tensor | None = None) -> torch.Tensor:
    """base + alpha * rmsnorm(x) * weight in one pass (fp32 inside, one bf16 rounding).

    The Euler update x + dt * v of the flow sampler when the velocity v is an RMSNorm
    output. `out` may be `base` itself for an in-place update; by default a new tensor
    of base's shape is returned."""
    dev = require_cuda("rmsnorm_axpy", x, weight, base, out)
    require_bf16("rmsnorm_axpy", x, base, out)
    if base.shape != x.shape:
        raise ValueError(f"rmsnorm_axpy: shapes differ {tuple(x.shape)} vs {tuple(base.shape)}")
    x2d, n = rows_view(x)
    b2d, _ = rows_view(base)
    w = weight.contiguous()
    if w.numel() != n:
        raise ValueError(f"rmsnorm_axpy: weight has {w.numel()} elements, rows have {n}")
    rows = x2d.shape[0]
    if out is None:
        y = torch.empty((rows, n), device=x.device, dtype=x.dtype)
    else:
        if out.shape != x.shape:
            raise ValueError("rmsnorm_axpy: out must have x's shape")
        y, _ = rows_view(out)
        if out.numel() and y.data_ptr() != out.data_ptr():
            raise ValueError("rmsnorm_axpy: out must be row-addressable in place")
    _lib.call("umic_rmsnorm_axpy", dev, x2d.data_ptr(), row_stride(x2d), w.data_ptr(),
              _w_dtype(w), b2d.data_ptr(), row_stride(b2d), float(alpha), y.data_ptr(),
              row_stride(y), rows, n, float(eps))
    stats["umic_rmsnorm_axpy"] += 1
    return out if out is not None else y.reshape(x.shape)


# Names of the reference interface (src/umic/kernels/rmsnorm.py:53,103).
rmsnorm_triton = rmsnorm
add_rmsnorm_triton = add_rmsnorm
