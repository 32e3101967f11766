"""Argument checks and call accounting shared by the kernel wrappers."""

from __future__ import annotations

import collections

import torch

# Calls that ran on the native library vs calls that took a documented
# GPU fallback (unsupported layout -> the original torch function, as the
# reference does for layouts its kernels do not cover, rope.py:97-99).
stats: collections.Counter = collections.Counter()


def reset_stats() -> None:
    stats.clear()


def require_cuda(name: str, *tensors: torch.Tensor | None) -> torch.device:
    dev = None
    for t in tensors:
        if t is None:
            continue
        if not t.is_cuda:
            raise RuntimeError(f"{name}: tensors must be on a CUDA device (got {t.device}); "
                               "umic_b200 has no CPU path")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise RuntimeError(f"{name}: tensors on different devices ({dev} vs {t.device})")
    assert dev is not None
    return dev


def require_bf16(name: str, *tensors: torch.Tensor | None) -> None:
    for t in tensors:
        if t is not None and t.dtype != torch.bfloat16:
            raise TypeError(f"{name}: expected bfloat16, got {t.dtype}")


def rows_view(x: torch.Tensor) -> tuple[torch.Tensor, int]:
    """[..., n] -> 2-D [rows, n] view with unit last stride (copies only if needed)."""
    n = x.shape[-1]
    x2d = x.reshape(-1, n)
    if x2d.stride(-1) != 1 or (x2d.shape[0] > 1 and x2d.stride(0) < n):
        x2d = x2d.contiguous()
    return x2d, n


def row_stride(t: torch.Tensor) -> int:
    return t.stride(0) if t.shape[0] > 1 else t.shape[1]


# ------------------------------------------------------------ launch probes
# A benchmark can ask for CUDA events around every launch of a named kernel
# (recorded on the launching stream) to time that kernel inside a longer step.
_probes: dict[str, list] = {}


def start_probe(name: str) -> None:
    _probes[name] = []


def stop_probe(name: str) -> list[float]:
    """Stops recording; returns per-launch durations in ms (synchronises)."""
    evs = _probes.pop(name, [])
    if evs:
        evs[-1][1].synchronize()
    return [s.elapsed_time(e) for s, e in evs]


def probe_begin(name: str):
    lst = _probes.get(name)
    if lst is None:
        return None
    s = torch.cuda.Event(enable_timing=True)
    s.record()
    return lst, s


def probe_end(token) -> None:
    if token is None:
        return
    lst, s = token
    e = torch.cuda.Event(enable_timing=True)
    e.record()
    lst.append((s, e))
