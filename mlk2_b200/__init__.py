"""mlk2_b200: B200 (sm_100a) execution path for MLK+ Kernel IR modules.

The product is the C-ABI shared library ``libmlkb200.so`` built in this
directory from ``csrc/`` (see ``include/mlkb200.h``). This package only loads
it and exposes thin ctypes wrappers; there is no Python or CPU fallback for
any kernel: when the library is missing, every entry point raises.
"""
from __future__ import annotations

import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libmlkb200.so")

# Status codes (include/mlkb200.h).
OK = 0
ERR_NEG_STORE = 1
ERR_CUDA_MEM = 2
ERR_LAUNCH = 3
ERR_NO_DEVICE = 4
ERR_NCCL = 5
ERR_TIMEOUT = 6
ERR_UNSUPPORTED = 7
ERR_INVALID = 8
ERR_NOT_BOUND = 9

F16, F32, F64 = 1, 2, 3
KIND_MAP, KIND_SOFTMAX, KIND_MATMUL, KIND_REDUCESUM, KIND_QK_SOFTMAX = 1, 2, 3, 4, 5


class MLKBError(RuntimeError):
    """A libmlkb200 entry point returned a nonzero status."""

    def __init__(self, status: int, message: str):
        super().__init__(f"mlkb status {status}: {message}")
        self.status = status


_lib = None


def lib() -> ctypes.CDLL:
    """The loaded libmlkb200.so (raises if it has not been built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise MLKBError(ERR_NO_DEVICE, f"{LIB_PATH} is missing: run __graft_entry__.build()")
        _lib = ctypes.CDLL(LIB_PATH, mode=ctypes.RTLD_GLOBAL)
        from . import _sigs

        _sigs.declare(_lib)
    return _lib


def check(status: int) -> None:
    """Raise MLKBError for a nonzero status, with the library's message."""
    if status != OK:
        msg = lib().mlkb_last_error().decode(errors="replace")
        raise MLKBError(status, msg)


def version() -> str:
    return lib().mlkb_version().decode()
