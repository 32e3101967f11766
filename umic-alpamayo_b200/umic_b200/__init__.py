"""umic_b200: B200-native (sm_100a) fused-inference hot path with UMIC's drop-in API.

The reference (soonhong99/umic-alpamayo) rebinds the forwards of matching
modules of a loaded model to fused kernels (src/umic/integrate.py) through one
call, `umic.apply(model, UmicConfig)` (src/umic/optimize.py). This package keeps
that API; behind it every fused op is a hand-written CUDA kernel for sm_100a
in libumic_b200.so (C ABI: include/umic_b200.h), called through ctypes.
"""

from . import _lib
from ._lib import UmicError, device_errors
from .optimize import UmicConfig, apply

__version__ = "0.1.0"

__all__ = ["UmicConfig", "UmicError", "apply", "device_errors", "__version__"]
