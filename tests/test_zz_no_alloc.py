"""The allocation-free GEMV entry point (umic_gemv_noalloc) against the workspace
entry point (umic_gemv) it mirrors.

umic_gemv_noalloc is for hosts that cannot allocate device memory when they call
in -- an embedded control loop that reserved its memory at start-up and may not
call cudaMalloc (it can synchronise the device and has no latency bound), or an FFI
runtime that owns its device pool -- so its scratch is a static device array that
lives in the library image.

This file is collected last, so the scratch array is exercised both in a fresh
process (run the file alone) and after every other GPU test has used the device.
The two entry points run the same streaming kernel over the same unit partition,
so their results must agree bit for bit, on two calls in a row (the second call
also checks that the first left the counters usable).
"""

import pytest
import torch

import oracle
from umic_b200 import _lib

pytestmark = pytest.mark.gpu


def _randn(*shape, seed, dev, scale=1.0):
    g = torch.Generator(device="cpu").manual_seed(seed)
    return (torch.randn(*shape, generator=g) * scale).to(torch.bfloat16).to(dev)


def _noalloc(x, w, bias):
    m, k = x.shape
    n = w.shape[0]
    y = torch.empty(m, n, device=x.device, dtype=torch.bfloat16)
    _lib.call("umic_gemv_noalloc", x.device, x.data_ptr(), k, w.data_ptr(), k, _lib.ptr(bias),
              y.data_ptr(), n, m, n, k)
    return y


def _with_workspace(x, w, bias):
    m, k = x.shape
    n = w.shape[0]
    y = torch.empty(m, n, device=x.device, dtype=torch.bfloat16)
    ws, ws_bytes = _lib.gemv_workspace(x.device, n)
    _lib.call("umic_gemv", x.device, x.data_ptr(), k, w.data_ptr(), k, _lib.ptr(bias),
              y.data_ptr(), n, m, n, k, ws, ws_bytes, 0)
    return y


@pytest.mark.parametrize("m,n,k,with_bias", [(8, 4096, 4096, False), (1, 12288, 4096, True),
                                             (16, 1000, 4104, True), (3, 64, 37888, False)])
def test_noalloc_matches_workspace_entry(cuda, m, n, k, with_bias):
    x = _randn(m, k, seed=300, dev=cuda)
    w = _randn(n, k, seed=301, dev=cuda, scale=0.02)
    bias = _randn(n, seed=302, dev=cuda) if with_bias else None
    a1 = _noalloc(x, w, bias)
    b1 = _with_workspace(x, w, bias)
    a2 = _noalloc(x, w, bias)
    b2 = _with_workspace(x, w, bias)
    assert torch.equal(a1, b1) and torch.equal(a2, b2) and torch.equal(a1, a2)
    ref = oracle.linear(x.cpu(), w.cpu(), None if bias is None else bias.cpu())
    err = oracle.rel_err(a1, ref)
    assert err <= 1e-2, err
    assert _lib.device_errors(cuda, clear=True) == 0


def test_noalloc_allocates_nothing(cuda):
    x = _randn(8, 2048, seed=310, dev=cuda)
    w = _randn(6144, 2048, seed=311, dev=cuda, scale=0.02)
    y = torch.empty(8, 6144, device=cuda, dtype=torch.bfloat16)
    before = torch.cuda.memory_allocated(cuda)
    for _ in range(2):
        _lib.call("umic_gemv_noalloc", cuda, x.data_ptr(), 2048, w.data_ptr(), 2048, None,
                  y.data_ptr(), 6144, 8, 6144, 2048)
    torch.cuda.synchronize(cuda)
    assert torch.cuda.memory_allocated(cuda) == before


def test_noalloc_rejects_sizes_beyond_its_scratch(cuda):
    x = _randn(17, 64, seed=320, dev=cuda)
    w = _randn(64, 64, seed=321, dev=cuda)
    y = torch.empty(17, 64, device=cuda, dtype=torch.bfloat16)
    with pytest.raises(_lib.UmicError, match="1..16"):
        _lib.call("umic_gemv_noalloc", cuda, x.data_ptr(), 64, w.data_ptr(), 64, None,
                  y.data_ptr(), 64, 17, 64, 64)
    # a matrix taller than the static scratch covers is refused before any launch
    # (the weight pointer is never dereferenced: the size check comes first)
    big = (1 << 20) + 64
    with pytest.raises(_lib.UmicError, match="static scratch maximum"):
        _lib.call("umic_gemv_noalloc", cuda, x.data_ptr(), 64, w.data_ptr(), 64, None,
                  y.data_ptr(), big, 1, big, 64)
