"""In-place KV append on the B200 kernel (C ABI: umic_kv_append).

Writes new K/V tokens into preallocated [B, H, capacity, D] buffers at a token
position given either as a Python int (checked on the host: overflow raises
RuntimeError like InplaceLayer.update, src/umic/cache.py:65-68) or as a device
int64 tensor read at execution time (capture-safe; replaces the graph-mode
index_copy_ of cache.py:59-60). A device position out of range skips the write
and raises the library's device error bit (read with umic_b200.device_errors()).
"""

from __future__ import annotations

import torch

from .. import _lib
from ._common import require_bf16, require_cuda, stats


def kv_append(k_buf: torch.Tensor, v_buf: torch.Tensor, k_new: torch.Tensor,
              v_new: torch.Tensor, pos: int | torch.Tensor) -> None:
    dev = require_cuda("kv_append", k_buf, v_buf, k_new, v_new)
    require_bf16("kv_append", k_buf, v_buf, k_new, v_new)
    if k_buf.shape != v_buf.shape or k_buf.stride() != v_buf.stride():
        raise ValueError("kv_append: K and V buffers must share shape and strides")
    b, h, cap, d = k_buf.shape
    if k_new.shape != v_new.shape or k_new.dim() != 4 or k_new.shape[0] != b or \
            k_new.shape[1] != h or k_new.shape[3] != d:
        raise ValueError(f"kv_append: new tokens {tuple(k_new.shape)} do not match buffer "
                         f"{tuple(k_buf.shape)}")
    if k_buf.stride(-1) != 1 or k_new.stride(-1) != 1 or v_new.stride(-1) != 1:
        raise ValueError("kv_append: head_dim must be contiguous")
    n = k_new.shape[2]
    if isinstance(pos, torch.Tensor):
        if pos.dtype != torch.int64 or pos.device != k_buf.device or pos.numel() < 1:
            raise ValueError("kv_append: device position must be an int64 tensor on the "
                             "buffer's device")
        host_pos, dpos = 0, pos.data_ptr()
    else:
        host_pos, dpos = int(pos), None
    try:
        _lib.call("umic_kv_append", dev, k_buf.data_ptr(), v_buf.data_ptr(), k_buf.stride(0),
                  k_buf.stride(1), k_buf.stride(2), cap, k_new.data_ptr(), k_new.stride(0),
                  k_new.stride(1), k_new.stride(2), v_new.data_ptr(), v_new.stride(0),
                  v_new.stride(1), v_new.stride(2), b, h, n, d, host_pos, dpos)
    except _lib.UmicError as e:
        if e.code == _lib.ERR_OVERFLOW:
            raise RuntimeError(str(e).split(": ", 1)[-1]) from None
        raise
    stats["umic_kv_append"] += 1
