"""The decode step's MLP half of a decoder layer in one launch (C ABI: umic_decode_mlp_chain).

For one token per episode (m <= 16 rows) the layer's tail after attention is four
dependent HBM-bound operations: o_proj, the attention-residual add with the
post-attention RMSNorm, the gated gate/up projection, and down_proj with the MLP
residual. As separate launches each pays a fixed cost of several microseconds against
5-40 us of weight streaming; umic_decode_mlp_chain runs them as the phases of one
persistent kernel whose weight stream continues across the phase boundaries. The result
equals the unfused decode kernels' bit for bit.
"""

from __future__ import annotations

import torch

from .. import _lib
from ._common import require_bf16, require_cuda, row_stride, stats


def _align256(n: int) -> int:
    return (n + 255) // 256 * 256


def decode_mlp_chain(attn: torch.Tensor, w_o: torch.Tensor, residual: torch.Tensor,
                     post_w: torch.Tensor, post_eps: float, w_gate: torch.Tensor,
                     w_up: torch.Tensor, w_down: torch.Tensor) -> torch.Tensor | None:
    """out = residual' + down(silu(gate(n)) * up(n)), n = RMSNorm(residual' ) * post_w,
    residual' = residual + attn @ w_o.T, all rows at once (attn [m, k], residual [m, h]).

    Returns None when the kernel does not cover the call (more than 16 rows, widths not a
    multiple of 64, non-contiguous rows, no workspace while a capture runs); the caller
    then keeps its unfused path."""
    dev = require_cuda("decode_mlp_chain", attn, w_o, residual, post_w, w_gate, w_up, w_down)
    require_bf16("decode_mlp_chain", attn, w_o, residual, w_gate, w_up, w_down)
    m, k = attn.shape
    hidden, inter = residual.shape[1], w_gate.shape[0]
    if (m > 16 or residual.shape[0] != m or w_o.shape != (hidden, k)
            or w_up.shape != w_gate.shape or w_gate.shape[1] != hidden
            or w_down.shape != (hidden, inter) or post_w.numel() != hidden
            or post_w.dtype not in (torch.bfloat16, torch.float32)):
        return None
    tensors = (attn, w_o, residual, w_gate, w_up, w_down)
    if any(t.stride(-1) != 1 for t in tensors) or residual.stride(0) != hidden \
            or w_gate.stride(0) != w_up.stride(0):
        return None
    ws, ws_bytes = _lib.chain_workspace(dev)
    if ws is None:
        return None
    post = post_w.contiguous()
    out = torch.empty((m, hidden), device=dev, dtype=attn.dtype)
    row_h = _align256(m * hidden * 2)
    scratch = torch.empty(3 * row_h + _align256(m * inter * 2), device=dev, dtype=torch.uint8)
    rc = _lib.try_call("umic_decode_mlp_chain", dev, attn.data_ptr(), row_stride(attn),
                       w_o.data_ptr(), row_stride(w_o), residual.data_ptr(), hidden,
                       post.data_ptr(),
                       _lib.DTYPE_FP32 if post.dtype == torch.float32 else _lib.DTYPE_BF16,
                       float(post_eps), w_gate.data_ptr(), w_up.data_ptr(), row_stride(w_gate),
                       w_down.data_ptr(), row_stride(w_down), out.data_ptr(), hidden,
                       scratch.data_ptr(), scratch.numel(), m, hidden, k, inter, ws, ws_bytes)
    if rc:
        stats["decode_mlp_chain_fallback"] += 1
        return None
    stats["umic_decode_mlp_chain"] += 1
    return out
