"""Attention on the B200 kernels (C ABI: umic_qk_norm_rope_kv, umic_attention_rows).

qk_norm_rope_kv: one launch does what the HF attention forward (transformers
qwen3_vl Qwen3VLTextAttention.forward) runs as four steps after the projections:
q_norm / k_norm per head, apply_rotary_pos_emb, and the KV-cache write
(past_key_values.update -> InplaceLayer.update, src/umic/cache.py:50-80).

attention_rows: the attention itself for few query rows per KV head over a long
cached prefix under a boolean mask -- the flow expert's action tokens over the
prefix KV, which torch's SDPA sends to an sm80-generation cuDNN kernel -- and for
one query head per KV head in 128-token tiles (the ViT's per-image attention).
"""

from __future__ import annotations

import torch

from .. import _lib
from ._common import require_bf16, require_cuda, stats
from .rmsnorm import _w_dtype
from .rope import _cos_dtype


def qk_norm_rope_kv(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor | None,
                    q_weight: torch.Tensor | None, k_weight: torch.Tensor | None, q_eps: float,
                    k_eps: float, cos: torch.Tensor, sin: torch.Tensor, k_buf=None, v_buf=None,
                    pos: int | torch.Tensor = 0) -> None:
    """q [B, S, Hq, D] and k / v [B, S, Hk, D] (any strides, D contiguous).

    q is normalised and rotated in place. With k_buf / v_buf ([B, Hk, cap, D]) the
    normalised, rotated k and v are written at token `pos` (int, or a device int64
    tensor for graph replay); without them k is rotated in place.
    """
    dev = require_cuda("qk_norm_rope_kv", q, k, v, cos, sin, k_buf, v_buf)
    require_bf16("qk_norm_rope_kv", q, k, v, k_buf, v_buf)
    b, s, hq, d = q.shape
    hk = k.shape[2]
    if k.shape[:2] != (b, s) or k.shape[3] != d:
        raise ValueError("qk_norm_rope_kv: q / k shapes differ")
    if cos.shape[-1] != d or cos.stride(-1) != 1 or sin.stride() != cos.stride():
        raise ValueError("qk_norm_rope_kv: cos/sin must be [B or 1, S, D] with D contiguous")
    c_sb = cos.stride(0) if cos.shape[0] > 1 else 0
    if q_weight is not None and k_weight is not None and q_weight.dtype != k_weight.dtype:
        k_weight = k_weight.to(q_weight.dtype)
    qw = q_weight.contiguous() if q_weight is not None else None
    kw = k_weight.contiguous() if k_weight is not None else None
    wref = qw if qw is not None else kw
    wdt = _w_dtype(wref) if wref is not None else _lib.DTYPE_BF16
    if k_buf is not None:
        if v is None or v_buf is None or v.shape != k.shape:
            raise ValueError("qk_norm_rope_kv: a cache write needs v and v_buf")
        cap = k_buf.shape[2]
        bs = (k_buf.stride(0), k_buf.stride(1), k_buf.stride(2))
        if isinstance(pos, torch.Tensor):
            host_pos, dpos = 0, pos.data_ptr()
        else:
            host_pos, dpos = int(pos), None
    else:
        cap, bs, host_pos, dpos = 0, (0, 0, 0), 0, None
    vs = (v.stride(0), v.stride(1), v.stride(2)) if v is not None else (0, 0, 0)
    try:
        _lib.call("umic_qk_norm_rope_kv", dev, q.data_ptr(), q.stride(0), q.stride(1),
                  q.stride(2), hq, k.data_ptr(), k.stride(0), k.stride(1), k.stride(2),
                  _lib.ptr(v), vs[0], vs[1], vs[2], hk, _lib.ptr(qw), _lib.ptr(kw), wdt,
                  float(q_eps), float(k_eps), cos.data_ptr(), sin.data_ptr(), c_sb,
                  cos.stride(1), _cos_dtype(cos), _lib.ptr(k_buf), _lib.ptr(v_buf), bs[0],
                  bs[1], bs[2], cap, host_pos, dpos, b, s, d)
    except _lib.UmicError as e:
        if e.code == _lib.ERR_OVERFLOW:
            raise RuntimeError(str(e).split(": ", 1)[-1]) from None
        raise
    stats["umic_qk_norm_rope_kv"] += 1


# The packed form of the last mask seen. Every layer of a model's forward receives the
# same boolean mask (transformers builds it once per forward), so it is packed once and
# reused by the other layers. The key holds the mask's base tensor by weak reference
# (alive tensors cannot share memory, so a reused address never matches a dead mask),
# the view's geometry and the version counter (an in-place write invalidates it).
_mask_cache: dict = {"base": None, "key": None, "bits": None}


def _packed_mask(mask: torch.Tensor, lk: int, dev: torch.device) -> torch.Tensor:
    import weakref

    base = mask if mask._base is None else mask._base
    key = (mask.data_ptr(), tuple(mask.shape), tuple(mask.stride()), mask._version, lk,
           torch.cuda.is_current_stream_capturing())
    ref = _mask_cache["base"]
    if ref is not None and ref() is base and _mask_cache["key"] == key:
        stats["mask_bits_reused"] += 1
        return _mask_cache["bits"]
    src = mask if mask.stride(-1) == 1 else mask.contiguous()
    hm, words = src.shape[1], (lk + 31) // 32
    bits = torch.empty(src.shape[0], hm, src.shape[2], words, device=dev, dtype=torch.int32)
    _lib.call("umic_mask_pack_bits", dev, src.data_ptr(), src.stride(0), src.stride(1),
              src.stride(2), src.shape[0], hm, src.shape[2], lk, bits.data_ptr(),
              bits.stride(0), bits.stride(1), bits.stride(2))
    stats["umic_mask_pack_bits"] += 1
    _mask_cache.update(base=weakref.ref(base), key=key, bits=bits)
    return bits


def attention_rows(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                   mask: torch.Tensor | None, scale: float) -> torch.Tensor | None:
    """softmax(scale * q k^T, masked) v with grouped-query heads, on the tcgen05 kernel.

    q [B, Hq, T, D], k / v [B, Hkv, Lk, D] (any strides, D contiguous), mask a bool
    tensor broadcastable to [B, Hq, T, >= Lk] (True = attend) or None; the mask is
    packed to bits first (umic_mask_pack_bits, one launch). Returns
    [B, T, Hq, D] (the layout transformers' attention functions return), or None
    when the kernel does not cover the shape (head_dim 64..128, a multiple of 8; either
    Hq / Hkv * T <= 128 query rows per KV head with T a multiple of 8, or Hq == Hkv
    with any T, cut into 128-token tiles) so the caller keeps its own path.
    """
    dev = require_cuda("attention_rows", q, k, v, mask)
    require_bf16("attention_rows", q, k, v)
    bsz, hq, t, d = q.shape
    hkv, lk = k.shape[1], k.shape[2]
    if k.shape != v.shape or k.shape[0] != bsz or k.shape[3] != d:
        raise ValueError(f"attention_rows: q {tuple(q.shape)} / k {tuple(k.shape)} / "
                         f"v {tuple(v.shape)}")
    if q.stride(-1) != 1 or k.stride(-1) != 1 or v.stride(-1) != 1:
        return None
    bits, ws = None, (0, 0, 0)
    if mask is not None:
        if mask.dtype != torch.bool or mask.dim() != 4 or mask.shape[-1] < lk:
            return None
        if mask.shape[1] not in (1, hq) or mask.shape[0] not in (1, bsz) or \
                mask.shape[2] not in (1, t):
            return None
        bits = _packed_mask(mask, lk, dev)
        hm = bits.shape[1]
        ws = (bits.stride(0) if bits.shape[0] > 1 else 0, bits.stride(1) if hm > 1 else 0,
              bits.stride(2) if bits.shape[2] > 1 else 0)
    out = torch.empty(bsz, t, hq, d, device=dev, dtype=q.dtype)
    rc = _lib.try_call("umic_attention_rows", dev, q.data_ptr(), q.stride(0), q.stride(1),
                       q.stride(2), k.data_ptr(), k.stride(0), k.stride(1), k.stride(2),
                       v.data_ptr(), v.stride(0), v.stride(1), v.stride(2), _lib.ptr(bits),
                       ws[0], ws[1], ws[2], out.data_ptr(), out.stride(0), out.stride(2),
                       out.stride(1), bsz, hq, hkv, t, lk, d, float(scale))
    if rc:
        stats["attention_rows_fallback"] += 1
        return None
    stats["umic_attention_rows"] += 1
    return out
