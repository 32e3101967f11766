"""In-place rotary embedding on the B200 kernel (C ABI: umic_rope_inplace).

Drop-ins for the reference's RoPE entry points (src/umic/kernels/rope.py):
  * apply_rotary_vision(q, k, cos, sin)   <- apply_rotary_vision_triton (rope.py:78-84)
  * make_text_rope(fallback)              <- make_text_rope (rope.py:86-107)
Both rotate q and k in one launch and IN PLACE (the reference allocated
q_out/k_out); they return the same tensors. Math in fp32, one bf16 rounding.
Layouts the kernel does not cover (partial rotary dim, unsqueeze_dim != 1,
non-bf16 q/k, CPU tensors) go to the original function, as in the reference
(rope.py:97-99); the original is called with keywords so the transformers 5.x
signature (q, k, cos, sin, unsqueeze_dim=1) is honoured.
"""

from __future__ import annotations

import torch

from .. import _lib
from ._common import require_bf16, require_cuda, stats


def _cos_dtype(c: torch.Tensor) -> int:
    if c.dtype == torch.float32:
        return _lib.DTYPE_FP32
    if c.dtype == torch.bfloat16:
        return _lib.DTYPE_BF16
    raise TypeError(f"rope: cos/sin dtype {c.dtype} not supported")


def rope_inplace_bshd(q: torch.Tensor, k: torch.Tensor | None, cos: torch.Tensor,
                      sin: torch.Tensor, q_strides: tuple[int, int, int],
                      k_strides: tuple[int, int, int] | None, batch: int, seq: int, hq: int,
                      hk: int, c_strides: tuple[int, int]) -> None:
    """Low-level call: q/k addressed as [batch, seq, head, dim] through strides."""
    dev = require_cuda("rope_inplace", q, k, cos, sin)
    require_bf16("rope_inplace", q, k)
    d = q.shape[-1]
    if cos.stride(-1) != 1 or sin.stride(-1) != 1 or q.stride(-1) != 1 or (
            k is not None and k.stride(-1) != 1):
        raise ValueError("rope_inplace: head_dim must be contiguous")
    if cos.stride() != sin.stride() or cos.dtype != sin.dtype:
        raise ValueError("rope_inplace: cos and sin must share layout and dtype")
    ks = k_strides or (0, 0, 0)
    _lib.call("umic_rope_inplace", dev, q.data_ptr(), q_strides[0], q_strides[1], q_strides[2],
              hq, k.data_ptr() if k is not None else None, ks[0], ks[1], ks[2], hk,
              cos.data_ptr(), sin.data_ptr(), c_strides[0], c_strides[1], _cos_dtype(cos),
              batch, seq, d)
    stats["umic_rope_inplace"] += 1


def apply_rotary_text_inplace(q: torch.Tensor, k: torch.Tensor, cos: torch.Tensor,
                              sin: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """HF text layout: q [B, Hq, S, D], k [B, Hk, S, D], cos/sin [B or 1, S, D]."""
    b, hq, s, d = q.shape
    hk = k.shape[1]
    c_sb = cos.stride(0) if cos.shape[0] > 1 else 0
    rope_inplace_bshd(q, k, cos, sin, (q.stride(0), q.stride(2), q.stride(1)),
                      (k.stride(0), k.stride(2), k.stride(1)), b, s, hq, hk,
                      (c_sb, cos.stride(1)))
    return q, k


def apply_rotary_vision(q: torch.Tensor, k: torch.Tensor, cos: torch.Tensor,
                        sin: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Drop-in for HF apply_rotary_pos_emb_vision: q/k [S, H, D], cos/sin [S, D]."""
    s, hq, d = q.shape
    hk = k.shape[1]
    rope_inplace_bshd(q, k, cos, sin, (0, q.stride(0), q.stride(1)),
                      (0, k.stride(0), k.stride(1)), 1, s, hq, hk, (0, cos.stride(0)))
    return q, k


def _text_supported(q, k, cos, sin, unsqueeze_dim) -> bool:
    return (unsqueeze_dim == 1 and q.is_cuda and q.dim() == 4 and k.dim() == 4
            and cos.dim() == 3 and sin.shape == cos.shape
            and q.dtype == torch.bfloat16 and k.dtype == torch.bfloat16
            and cos.dtype in (torch.bfloat16, torch.float32)
            and cos.shape[-1] == q.shape[-1] == k.shape[-1]
            and cos.shape[0] in (1, q.shape[0]) and cos.shape[1] == q.shape[2]
            and q.shape[0] == k.shape[0] and q.shape[2] == k.shape[2]
            and q.stride(-1) == 1 and k.stride(-1) == 1
            and cos.stride(-1) == 1 and sin.stride() == cos.stride()
            and not (q.requires_grad or k.requires_grad))


def make_text_rope(fallback):
    """Build a drop-in for HF apply_rotary_pos_emb (q/k: [B, H, S, D]), in place."""

    def apply_rotary_text(q, k, cos, sin, position_ids=None, unsqueeze_dim=1):
        if not _text_supported(q, k, cos, sin, unsqueeze_dim):
            stats["rope_text_fallback"] += 1
            return fallback(q, k, cos, sin, unsqueeze_dim=unsqueeze_dim)
        return apply_rotary_text_inplace(q, k, cos, sin)

    return apply_rotary_text


def vision_supported(q, k, cos, sin) -> bool:
    return (q.is_cuda and q.dim() == 3 and k.dim() == 3 and cos.dim() == 2
            and q.dtype == torch.bfloat16 and k.dtype == torch.bfloat16
            and cos.dtype in (torch.bfloat16, torch.float32) and sin.shape == cos.shape
            and cos.shape[-1] == q.shape[-1] == k.shape[-1] and cos.shape[0] == q.shape[0]
            and q.shape[0] == k.shape[0] and q.stride(-1) == 1 and k.stride(-1) == 1
            and cos.stride(-1) == 1 and sin.stride() == cos.stride()
            and not (q.requires_grad or k.requires_grad))


def make_vision_rope(fallback):
    """Build a drop-in for HF apply_rotary_pos_emb_vision, in place."""

    def apply_rotary_vision_fused(q, k, cos, sin):
        if not vision_supported(q, k, cos, sin):
            stats["rope_vision_fallback"] += 1
            return fallback(q, k, cos, sin)
        return apply_rotary_vision(q, k, cos, sin)

    return apply_rotary_vision_fused


# Name of the reference interface (src/umic/kernels/rope.py:78).
apply_rotary_vision_triton = apply_rotary_vision
