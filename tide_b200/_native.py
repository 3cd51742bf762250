"""Loading of the native parts.  There is no fallback: if the CUDA library or
the operator extension is missing, the first call raises and says how to
build it (python -c "import __graft_entry__ as g; g.build()" or
python tide_b200/build.py)."""
from __future__ import annotations

import ctypes
import threading
from pathlib import Path

import torch

PKG = Path(__file__).resolve().parent
LIB_PATH = PKG / "libtide_b200.so"
EXT_PATH = PKG / "_C.so"

_lock = threading.Lock()
_lib = None
_ops_loaded = False


class NativeMissing(RuntimeError):
    pass


def lib() -> ctypes.CDLL:
    """The C ABI library (include/tide_b200.h), loaded once."""
    global _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise NativeMissing(f"{LIB_PATH} is missing: build it with `python tide_b200/build.py`")
            _lib = ctypes.CDLL(str(LIB_PATH))
            from tide_b200 import capi
            capi.declare(_lib)
    return _lib


def ops():
    """torch.ops.tide with the CUDA operators registered, loaded once."""
    global _ops_loaded
    with _lock:
        if not _ops_loaded:
            if not EXT_PATH.exists():
                raise NativeMissing(f"{EXT_PATH} is missing: build it with `python tide_b200/build.py`")
            torch.ops.load_library(str(EXT_PATH))
            _ops_loaded = True
    return torch.ops.tide


def require_cuda(t: torch.Tensor, what: str) -> None:
    if not t.is_cuda:
        raise RuntimeError(f"{what} must live on a CUDA device: tide_b200 runs its early-exit path "
                           f"only as sm_100a kernels (no CPU path)")
