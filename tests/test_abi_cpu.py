"""CPU checks of the C ABI: the library loads, exports every symbol the header
declares, and rejects bad arguments on the host before touching a GPU."""

import ctypes
import re
from pathlib import Path

import pytest

from umic_b200 import _lib

ROOT = Path(__file__).resolve().parent.parent
HEADER = ROOT / "include" / "umic_b200.h"


def _declared() -> list[str]:
    return re.findall(r"UMIC_API\s+(?:int|size_t|const char\*)\s+(umic_\w+)\(", HEADER.read_text())


def test_library_exports_every_declared_symbol():
    L = _lib.lib()
    declared = _declared()
    assert len(declared) >= 14
    for name in declared:
        assert hasattr(L, name), f"{name} declared in the header but not exported"
    assert set(declared) == set(_lib.exported_symbols())


def test_abi_version():
    assert _lib.lib().umic_abi_version() == 2


def test_null_pointer_rejected_on_host():
    L = _lib.lib()
    rc = L.umic_rmsnorm(None, 8, None, 0, None, 8, 4, 8, ctypes.c_float(1e-6), None)
    assert rc == 1
    assert "null" in _lib.last_message()


def test_bad_sizes_rejected_on_host():
    L = _lib.lib()
    fake = ctypes.c_void_p(16)  # never dereferenced: the size check fails first
    assert L.umic_gemm(fake, 8, fake, 8, None, None, 0, fake, 8, 4, 4, 0, 0, None) == 1
    assert L.umic_gemm(fake, 12, fake, 12, None, None, 0, fake, 16, 4, 16, 12, 0, None) == 3
    assert "multiple of 8" in _lib.last_message()
    assert L.umic_gemv(fake, 8, fake, 8, None, fake, 8, 65, 8, 8, None, 0, 0, None) == 2
    assert L.umic_rope_inplace(fake, 0, 0, 0, 1, None, 0, 0, 0, 0, fake, fake, 0, 0, 0, 1, 1, 7,
                               None) == 1
    assert L.umic_kv_append(fake, fake, 0, 0, 0, 10, fake, 0, 0, 0, fake, 0, 0, 0, 1, 1, 4, 8,
                            8, None, None) == 5
    assert "overflow" in _lib.last_message()


def test_gemv_workspace_contract_on_host():
    """The workspace size grows with the rows of a call; a workspace that is too small
    or misaligned is rejected before any launch (only checked once the streaming
    engine is chosen, which needs the SM count of a device)."""
    L = _lib.lib()
    fake = ctypes.c_void_p(16)
    # m > 64 is rejected whatever the workspace
    assert L.umic_gemv(fake, 8, fake, 8, None, fake, 8, 65, 8, 8, fake, 1 << 20, 0, None) == 2


def test_empty_work_is_a_noop():
    L = _lib.lib()
    fake = ctypes.c_void_p(16)
    assert L.umic_rmsnorm(fake, 8, fake, 0, fake, 8, 0, 8, ctypes.c_float(1e-6), None) == 0
    assert L.umic_gemm(fake, 8, fake, 8, None, None, 0, fake, 8, 0, 8, 8, 0, None) == 0


def test_kernel_wrappers_refuse_cpu_tensors():
    import torch

    from umic_b200.kernels import linear, rmsnorm

    x = torch.zeros(4, 8, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="no CPU path"):
        rmsnorm(x, torch.ones(8, dtype=torch.bfloat16), 1e-6)
    with pytest.raises(RuntimeError, match="no CPU path"):
        linear(x, torch.zeros(8, 8, dtype=torch.bfloat16))


def test_attention_rows_rejects_uncovered_shapes_on_host():
    L = _lib.lib()
    fake = ctypes.c_void_p(16)  # never dereferenced: the shape check fails first
    # head_dim 48, and 2 x 72 = 144 query rows per KV head, are declined before any launch
    assert L.umic_attention_rows(fake, 0, 0, 0, fake, 0, 0, 0, fake, 0, 0, 0, None, 0, 0, 0,
                                 fake, 0, 0, 0, 1, 4, 2, 8, 64, 48, ctypes.c_float(0.1),
                                 None) == 2
    assert "64..128" in _lib.last_message()
    assert L.umic_attention_rows(fake, 0, 0, 0, fake, 0, 0, 0, fake, 0, 0, 0, None, 0, 0, 0,
                                 fake, 0, 0, 0, 1, 16, 8, 72, 64, 128, ctypes.c_float(0.1),
                                 None) == 2
    assert "144 query rows" in _lib.last_message()
    # empty work returns at once
    assert L.umic_attention_rows(None, 0, 0, 0, None, 0, 0, 0, None, 0, 0, 0, None, 0, 0, 0,
                                 None, 0, 0, 0, 0, 16, 8, 64, 64, 128, ctypes.c_float(0.1),
                                 None) == 0


def test_binding_arity_matches_header():
    """Every ctypes signature has as many arguments as the header's declaration (a
    missing trailing stream would reach the runtime as a truncated integer)."""
    text = HEADER.read_text()
    for name, args in _lib._SIGNATURES.items():
        m = re.search(r"UMIC_API\s+(?:int|size_t|const char\*)\s+" + name + r"\(([^;]*)\);",
                      text, re.S)
        assert m, name
        params = [p for p in m.group(1).split(",") if p.strip() and p.strip() != "void"]
        assert len(params) == len(args), f"{name}: header {len(params)} vs binding {len(args)}"


@pytest.mark.parametrize("o_st", [0, -2048, 12])
def test_attention_rows_rejects_bad_output_strides_on_host(o_st):
    """Output strides must be positive multiples of 8 like the input strides: a zero or
    negative stride would make rows overwrite one another or write before the buffer."""
    L = _lib.lib()
    fake = ctypes.c_void_p(256)  # never dereferenced: the stride check fails first
    rc = L.umic_attention_rows(fake, 8 * 16 * 64 * 128, 64 * 128, 128,
                               fake, 8 * 64 * 128, 64 * 128, 128,
                               fake, 8 * 64 * 128, 64 * 128, 128, None, 0, 0, 0,
                               fake, 64 * 16 * 128, 128, o_st, 1, 16, 8, 64, 64, 128,
                               ctypes.c_float(0.1), None)
    assert rc == 3
    assert "strides" in _lib.last_message()


def test_debug_stall_rejects_bad_arguments():
    L = _lib.lib()
    assert L.umic_debug_stall(0, 1000) == 1
    assert L.umic_debug_stall(1, 0) == 1
    assert "umic_debug_stall" in _lib.last_message()


def test_gemm_split_plan_on_host():
    """Split-K only for shapes whose tiles fill at most half the CTA pairs: the flow
    expert's projections at 4 episodes get a workspace, the LM prefill shapes none."""
    L = _lib.lib()
    assert L.umic_gemm_workspace_bytes(256, 2048, 2048) > 0
    # 8 tiles x 2 halves x 8 ranges (the cap: one 32-column chunk per range) x 128 KB
    # of fp32 partials behind a 4 KB counter area, on a 148-SM B200
    assert L.umic_gemm_workspace_bytes(256, 2048, 2048) == 4096 + 8 * 2 * 8 * 128 * 1024
    assert L.umic_gemm_workspace_bytes(256, 2048, 8192) > 0
    assert L.umic_gemm_workspace_bytes(24800, 4096, 4096) == 0
    assert L.umic_gemm_workspace_bytes(3100, 4096, 4096) == 0
    assert L.umic_gemm_workspace_bytes(256, 2048, 256) == 0  # too few k-blocks to split


def _split_plan_bytes(m, n, k, sms=148):
    """The split-K planner's rule, restated: 256-row pair tiles (128-row single-CTA tiles
    for m <= 128) by 256 columns; split only when the tiles fill at most half the units
    (CTA pairs, or CTAs) and there are at least 8 k-blocks of 64; ranges = min(units per
    tile, k-blocks / 4, 8); workspace = 4 KB of counters + 2 halves x ranges x 128 x 256
    fp32 per tile."""
    pair = m > 128
    tiles = -(-m // (256 if pair else 128)) * -(-n // 256)
    kblocks = -(-k // 64)
    units = sms // 2 if pair else sms
    if tiles * 2 > units or kblocks < 8:
        return 0
    s = min(units // tiles, kblocks // 4, 8)
    return 0 if s < 2 else 4096 + tiles * 2 * s * 128 * 256 * 4


def test_gemm_split_plan_matches_its_rule():
    L = _lib.lib()
    for m in (1, 64, 128, 129, 256, 512, 1000, 2048):
        for n in (256, 1024, 2048, 4096, 6144):
            for k in (256, 512, 1024, 2048, 8192):
                assert L.umic_gemm_workspace_bytes(m, n, k) == _split_plan_bytes(m, n, k), \
                    (m, n, k)
