"""B200 kernel wrappers, one module per reference kernel file (src/umic/kernels/*.py)."""

from ._common import reset_stats, stats
from .fused_ffn import FUSE_MIN_ROWS, gate_silu_mul, gate_silu_mul_nk
from .kv import kv_append
from .layernorm import add_layernorm, layernorm
from .linear import linear, linear_gemv
from .rmsnorm import add_rmsnorm, rmsnorm, rmsnorm_axpy
from .rope import apply_rotary_text_inplace, apply_rotary_vision, make_text_rope

__all__ = [
    "FUSE_MIN_ROWS", "add_layernorm", "add_rmsnorm", "apply_rotary_text_inplace",
    "apply_rotary_vision", "gate_silu_mul", "gate_silu_mul_nk", "kv_append", "layernorm",
    "linear", "linear_gemv", "make_text_rope", "reset_stats", "rmsnorm", "rmsnorm_axpy",
    "stats",
]
