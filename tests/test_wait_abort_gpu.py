"""The bounded-wait abort path, exercised on the GPU without a fault or a hang.

Every mbarrier wait in the TMA-fed kernels gives up after a cycle limit: the CTA sets
UMIC_DEVERR_WAIT_TIMEOUT, lets its copies in flight land, drains its MMAs, frees its
tensor memory and exits. `umic_debug_stall` arms one launch in which CTA 0 announces the
bytes of a shared-memory stage that it never loads -- a barrier that nothing completes --
with a short limit, so the wait runs out in milliseconds. Each test checks that the call
returns, that the host reads the error bit, and that the next calls on the same context
are correct (tensor memory was freed, barriers re-initialise, the GEMV workspace is
usable again once zeroed).
"""

import pytest
import torch

from umic_b200 import _lib
from umic_b200.kernels import gate_silu_mul_nk, linear, linear_gemv

pytestmark = pytest.mark.gpu

LIMIT = 20_000_000  # SM cycles, about 10 ms


def _randn(*shape, seed, dev, scale=1.0):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(*shape, generator=g) * scale).to(torch.bfloat16).to(dev)


def _stalled(cuda, kernel, fn):
    assert _lib.device_errors(cuda, clear=True) == 0
    _lib.arm_stall(kernel, LIMIT)
    fn()
    flags = _lib.device_errors(cuda, clear=True)  # synchronises: the launch came back
    assert flags & _lib.DEVERR_WAIT_TIMEOUT, flags


@pytest.mark.parametrize("m", [512, 100])  # CTA pairs, and single CTAs (m <= 128)
@pytest.mark.parametrize("split_k", [True, False])
def test_gemm_wait_timeout_unwinds(cuda, m, split_k):
    """Both shapes run split-K when allowed (6 / 3 output tiles): the stalled unit never
    counts in, its partners give up on the count, and the workspace keeps their stale
    counts until it is zeroed; the next calls -- with new inputs, so no leftover partial
    can pass for a fresh one -- are correct."""
    x = _randn(m, 1024, seed=1, dev=cuda)
    w = _randn(768, 1024, seed=2, dev=cuda, scale=0.05)
    assert (_lib.lib().umic_gemm_workspace_bytes(m, 768, 1024) > 0)
    _stalled(cuda, 1, lambda: linear(x, w, split_k=split_k))
    _lib.zero_gemv_workspaces()  # counters of a split launch that unwound
    for seed in (10, 11, 12):
        x2 = _randn(m, 1024, seed=seed, dev=cuda)
        ref = torch.nn.functional.linear(x2.float(), w.float())
        y = linear(x2, w, split_k=split_k)
        assert (y.float() - ref).norm() / ref.norm() < 1e-2
        assert torch.equal(y, linear(x2, w, split_k=split_k))
    assert _lib.device_errors(cuda, clear=True) == 0


def test_dual_gemm_wait_timeout_unwinds(cuda):
    x = _randn(640, 512, seed=3, dev=cuda)
    wg = _randn(1024, 512, seed=4, dev=cuda, scale=0.05)
    wu = _randn(1024, 512, seed=5, dev=cuda, scale=0.05)
    ref = gate_silu_mul_nk(x, wg, wu).clone()
    _stalled(cuda, 1, lambda: gate_silu_mul_nk(x, wg, wu))
    assert torch.equal(gate_silu_mul_nk(x, wg, wu), ref)
    assert _lib.device_errors(cuda, clear=True) == 0


def test_streaming_gemv_wait_timeout_unwinds(cuda):
    x = _randn(8, 4096, seed=6, dev=cuda)
    w = _randn(12288, 4096, seed=7, dev=cuda, scale=0.02)
    ref = linear_gemv(x, w).clone()
    _stalled(cuda, 2, lambda: linear_gemv(x, w))
    _lib.zero_gemv_workspaces()  # the unwound launch may have left row-block counters
    for _ in range(3):
        assert torch.equal(linear_gemv(x, w), ref)
    assert _lib.device_errors(cuda, clear=True) == 0


@pytest.mark.parametrize("m,n", [(8, 12288), (4, 4096), (1, 151936)])
def test_streaming_gemv_fast_merge_equals_general_merge(cuda, m, n):
    """A row block split between two CTAs is merged either through the shortcut (the
    second CTA finds its partner's partial already posted and sums it at once) or the
    general path (count, then the last arrival sums every partial in CTA order); which
    one runs depends on timing. Forcing the general path must give the same bits."""
    x = _randn(m, 4096, seed=8, dev=cuda)
    w = _randn(n, 4096, seed=9, dev=cuda, scale=0.02)
    runs = [linear_gemv(x, w).clone() for _ in range(3)]
    _lib.arm_stall(3, 1)
    general = linear_gemv(x, w)
    for r in runs:
        assert torch.equal(r, general)
    assert _lib.device_errors(cuda, clear=True) == 0
