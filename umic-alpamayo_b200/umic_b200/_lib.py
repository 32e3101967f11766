"""ctypes binding of libumic_b200.so (the C ABI declared in include/umic_b200.h).

This is the only place Python touches the native library. Every call goes
through `call()`, which passes the current torch CUDA stream, keeps the
library's CUDA runtime on the tensor's device and turns a non-zero status into
a RuntimeError carrying the library's one-line reason. There is no fallback:
if the library is missing or fails to load, the first kernel call raises.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / "libumic_b200.so"

_c_i64 = ctypes.c_int64
_c_i32 = ctypes.c_int32
_c_int = ctypes.c_int
_c_f32 = ctypes.c_float
_c_p = ctypes.c_void_p
_c_size = ctypes.c_size_t
_c_u32 = ctypes.c_uint32

# name -> argument types (all return int status unless listed in _RESTYPES)
_SIGNATURES: dict[str, list] = {
    "umic_abi_version": [],
    "umic_last_error_message": [],
    "umic_set_device": [_c_int],
    "umic_device_errors": [ctypes.POINTER(ctypes.c_uint32), _c_int],
    "umic_debug_stall": [_c_int, _c_i64],
    "umic_rmsnorm": [_c_p, _c_i64, _c_p, _c_int, _c_p, _c_i64, _c_i64, _c_i64, _c_f32, _c_p],
    "umic_rmsnorm_axpy": [_c_p, _c_i64, _c_p, _c_int, _c_p, _c_i64, _c_f32, _c_p, _c_i64,
                          _c_i64, _c_i64, _c_f32, _c_p],
    "umic_add_rmsnorm": [_c_p, _c_i64, _c_p, _c_i64, _c_p, _c_int, _c_p, _c_i64, _c_p, _c_i64,
                         _c_i64, _c_i64, _c_f32, _c_p],
    "umic_layernorm": [_c_p, _c_i64, _c_p, _c_p, _c_int, _c_p, _c_i64, _c_i64, _c_i64, _c_f32,
                       _c_p],
    "umic_add_layernorm": [_c_p, _c_i64, _c_p, _c_i64, _c_p, _c_p, _c_int, _c_p, _c_i64, _c_p,
                           _c_i64, _c_i64, _c_i64, _c_f32, _c_p],
    "umic_rope_inplace": [_c_p, _c_i64, _c_i64, _c_i64, _c_i32, _c_p, _c_i64, _c_i64, _c_i64,
                          _c_i32, _c_p, _c_p, _c_i64, _c_i64, _c_int, _c_i64, _c_i64, _c_i32,
                          _c_p],
    "umic_kv_append": [_c_p, _c_p, _c_i64, _c_i64, _c_i64, _c_i64, _c_p, _c_i64, _c_i64, _c_i64,
                       _c_p, _c_i64, _c_i64, _c_i64, _c_i64, _c_i32, _c_i64, _c_i32, _c_i64,
                       _c_p, _c_p],
    "umic_gemv": [_c_p, _c_i64, _c_p, _c_i64, _c_p, _c_p, _c_i64, _c_i64, _c_i64, _c_i64, _c_p,
                  _c_size, _c_u32, _c_p],
    "umic_gemv_gate_silu_mul": [_c_p, _c_i64, _c_p, _c_p, _c_i64, _c_p, _c_i64, _c_i64, _c_i64,
                                _c_i64, _c_p, _c_size, _c_u32, _c_p],
    "umic_gemv_multi": [_c_p, _c_i64, _c_i32, ctypes.POINTER(_c_p), ctypes.POINTER(_c_i64),
                        ctypes.POINTER(_c_i64), ctypes.POINTER(_c_p), ctypes.POINTER(_c_p),
                        ctypes.POINTER(_c_i64), _c_i64, _c_i64, _c_p, _c_size, _c_u32, _c_p],
    "umic_gemv_workspace_bytes": [_c_i64],
    "umic_gemv_residual": [_c_p, _c_i64, _c_p, _c_i64, _c_p, _c_p, _c_i64, _c_p, _c_i64, _c_i64,
                           _c_i64, _c_i64, _c_p, _c_size, _c_u32, _c_p],
    "umic_gemv_noalloc": [_c_p, _c_i64, _c_p, _c_i64, _c_p, _c_p, _c_i64, _c_i64, _c_i64,
                          _c_i64, _c_p],
    "umic_qk_norm_rope_kv": [_c_p, _c_i64, _c_i64, _c_i64, _c_i32, _c_p, _c_i64, _c_i64, _c_i64,
                             _c_p, _c_i64, _c_i64, _c_i64, _c_i32, _c_p, _c_p, _c_int, _c_f32,
                             _c_f32, _c_p, _c_p, _c_i64, _c_i64, _c_int, _c_p, _c_p, _c_i64,
                             _c_i64, _c_i64, _c_i64, _c_i64, _c_p, _c_i64, _c_i64, _c_i32, _c_p],
    "umic_attention_rows": [_c_p, _c_i64, _c_i64, _c_i64, _c_p, _c_i64, _c_i64, _c_i64, _c_p,
                            _c_i64, _c_i64, _c_i64, _c_p, _c_i64, _c_i64, _c_i64, _c_p, _c_i64,
                            _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64,
                            _c_f32, _c_p],
    "umic_mask_pack_bits": [_c_p, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _c_p,
                            _c_i64, _c_i64, _c_i64, _c_p],
    "umic_gemm": [_c_p, _c_i64, _c_p, _c_i64, _c_p, _c_p, _c_i64, _c_p, _c_i64, _c_i64, _c_i64,
                  _c_i64, _c_int, _c_p],
    "umic_gemm_ws": [_c_p, _c_i64, _c_p, _c_i64, _c_p, _c_p, _c_i64, _c_p, _c_i64, _c_i64,
                     _c_i64, _c_i64, _c_int, _c_p, _c_size, _c_p],
    "umic_gemm_workspace_bytes": [_c_i64, _c_i64, _c_i64],
    "umic_gemm_gate_silu_mul": [_c_p, _c_i64, _c_p, _c_i64, _c_p, _c_i64, _c_p, _c_i64, _c_i64,
                                _c_i64, _c_i64, _c_p],
}
_RESTYPES = {"umic_last_error_message": ctypes.c_char_p, "umic_gemv_workspace_bytes": _c_size,
             "umic_gemm_workspace_bytes": _c_size}

ERR_NAMES = {1: "INVALID_ARG", 2: "UNSUPPORTED", 3: "ALIGNMENT", 4: "LAUNCH", 5: "OVERFLOW",
             6: "DEVICE"}
ERR_UNSUPPORTED = 2
ERR_ALIGNMENT = 3
ERR_OVERFLOW = 5

DTYPE_BF16 = 0
DTYPE_FP32 = 1
EPI_NONE, EPI_GELU_ERF, EPI_GELU_TANH = 0, 1, 2
GEMV_WEIGHTS_READY = 1
DEVERR_KV_OVERFLOW = 1
DEVERR_WAIT_TIMEOUT = 2

_lib = None
_lock = threading.Lock()
_tls = threading.local()


class UmicError(RuntimeError):
    """A C-ABI call returned a non-zero status."""

    def __init__(self, name: str, code: int, msg: str):
        super().__init__(f"{name} failed ({ERR_NAMES.get(code, code)}): {msg}")
        self.code = code


def lib() -> ctypes.CDLL:
    """Loads the library once; raises if it is not built."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not LIB_PATH.exists():
                    raise RuntimeError(
                        f"{LIB_PATH.name} is not built; run __graft_entry__.build() or "
                        "python umic-alpamayo_b200/umic_b200/_build.py")
                L = ctypes.CDLL(str(LIB_PATH))
                for name, args in _SIGNATURES.items():
                    fn = getattr(L, name)
                    fn.argtypes = args
                    fn.restype = _RESTYPES.get(name, ctypes.c_int)
                _lib = L
    return _lib


def exported_symbols() -> list[str]:
    return list(_SIGNATURES)


def _ensure_device(device: torch.device) -> None:
    idx = device.index if device.index is not None else torch.cuda.current_device()
    if getattr(_tls, "device", None) != idx:
        rc = lib().umic_set_device(idx)
        if rc:
            raise UmicError("umic_set_device", rc, last_message())
        _tls.device = idx


def last_message() -> str:
    m = lib().umic_last_error_message()
    return m.decode() if m else ""


def stream_ptr(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def call(name: str, device: torch.device, *args) -> None:
    """Calls `name` with args + the current stream of `device`; raises on error."""
    _ensure_device(device)
    fn = getattr(lib(), name)
    rc = fn(*args, stream_ptr(device))
    if rc:
        raise UmicError(name, rc, last_message())


def try_call(name: str, device: torch.device, *args) -> int:
    """Like call() but returns UNSUPPORTED / ALIGNMENT codes instead of raising."""
    _ensure_device(device)
    rc = getattr(lib(), name)(*args, stream_ptr(device))
    if rc and rc not in (ERR_UNSUPPORTED, ERR_ALIGNMENT):
        raise UmicError(name, rc, last_message())
    return rc


def device_errors(device: torch.device | None = None, clear: bool = True) -> int:
    """Reads (and by default clears) the device-side error bits; synchronises."""
    _ensure_device(device or torch.device("cuda", torch.cuda.current_device()))
    v = ctypes.c_uint32(0)
    rc = lib().umic_device_errors(ctypes.byref(v), 1 if clear else 0)
    if rc:
        raise UmicError("umic_device_errors", rc, last_message())
    return int(v.value)


def arm_stall(kernel: int, wait_limit_cycles: int) -> None:
    """Test hook: the next launch of `kernel` (1 = GEMM, 2 = streaming GEMV) stalls one CTA
    and unwinds after `wait_limit_cycles`; 3 makes the next streaming GEMV merge split row
    blocks only through its general path (see umic_debug_stall in the header)."""
    rc = lib().umic_debug_stall(kernel, wait_limit_cycles)
    if rc:
        raise UmicError("umic_debug_stall", rc, last_message())


def zero_gemv_workspaces() -> None:
    """Zeroes every streaming-GEMV and split-K GEMM workspace of this process (needed after
    a launch that unwound on a wait timeout: its counters may be left non-zero)."""
    for buf in list(_workspaces.values()) + list(_gemm_workspaces.values()):
        buf.zero_()
    for dev_idx in set(_workspaces) | set(_gemm_workspaces):
        torch.cuda.synchronize(dev_idx)


_gemm_workspaces: dict[int, torch.Tensor] = {}


def gemm_workspace(device: torch.device, m: int, n: int, k: int) -> tuple[int | None, int]:
    """(pointer, bytes) of the split-K GEMM workspace of `device` for this shape, or
    (None, 0) when the shape needs no split. One zero-filled buffer per device for the
    process (captured graphs hold its address; an outgrown buffer is retired, never freed);
    the kernel returns its counters to zero after every call. While a capture runs and the
    buffer is too small, (None, 0): the call then runs without splitting."""
    _ensure_device(device)
    need = int(lib().umic_gemm_workspace_bytes(m, n, k))
    if need == 0:
        return None, 0
    idx = device.index if device.index is not None else torch.cuda.current_device()
    buf = _gemm_workspaces.get(idx)
    if buf is None or buf.numel() < need:
        if torch.cuda.is_current_stream_capturing():
            return None, 0
        if buf is not None:
            _retired.append(buf)
        buf = torch.zeros(need, dtype=torch.uint8, device=device)
        torch.cuda.current_stream(device).synchronize()
        _gemm_workspaces[idx] = buf
    return buf.data_ptr(), buf.numel()


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


_MIN_WORKSPACE = 8 << 20
_workspaces: dict[int, torch.Tensor] = {}
_retired: list[torch.Tensor] = []


def gemv_workspace(device: torch.device, rows: int) -> tuple[int | None, int]:
    """(pointer, bytes) of the streaming GEMV's scratch on `device` for `rows` weight rows.

    One zero-filled buffer per device, kept for the life of the process: captured CUDA
    graphs hold its address, so a buffer outgrown by a larger call is retired, never
    freed. The kernel returns its counters to zero after every call. Calls that share
    the buffer must be ordered on one stream (overlapping calls would race on it).
    No buffer is created while a CUDA graph is being captured; such a call gets
    (None, 0) and runs the workspace-free engine."""
    _ensure_device(device)
    need = int(lib().umic_gemv_workspace_bytes(rows))
    idx = device.index if device.index is not None else torch.cuda.current_device()
    buf = _workspaces.get(idx)
    if buf is None or buf.numel() < need:
        if torch.cuda.is_current_stream_capturing():
            return None, 0
        if buf is not None:
            _retired.append(buf)
        buf = torch.zeros(max(need, _MIN_WORKSPACE), dtype=torch.uint8, device=device)
        torch.cuda.current_stream(device).synchronize()  # zeroed before any stream uses it
        _workspaces[idx] = buf
    return buf.data_ptr(), buf.numel()

