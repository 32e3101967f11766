"""CPU oracle for the UMIC fused-inference hot path -- TEST INFRASTRUCTURE ONLY.

This package restates, on the CPU and in fp32/fp64 torch arithmetic, what the
reference project (soonhong99/umic-alpamayo) computes on its hot path. It is
the checker the GPU kernels are compared against. Only tests/,
__graft_entry__.smoke() and bench.py's CPU-baseline / reference legs may import
it; the product (umic_b200) never does and has no CPU path of its own.

Pinning: the restatement is checked against golden vectors produced by the
reference's own code run in this container (its Triton kernels under
TRITON_INTERPRET=1, its eager functions and its KV-cache class) and by the HF
transformers eager modules it patches; see tests/golden/make_golden.py and
tests/test_oracle_golden.py.
"""

from .formulas import (  # noqa: F401
    add_layernorm,
    add_rmsnorm,
    attention,
    gate_silu_mul,
    layernorm,
    linear,
    rel_err,
    max_rel_err,
    rmsnorm,
    rmsnorm_axpy,
    rope_rotate_half,
    swiglu_block,
    text_rope_cos_sin,
)
from .kvcache import KVCacheOracle  # noqa: F401
