"""gfxinfer-b200: a B200-native decode engine for the gfxinfer token loop.

The product is libgfxb200.so (hand-written sm_100a CUDA kernels and the C++
runtime behind the C ABI in include/gfxb/gfxb.h). This package only loads it
and offers thin ctypes/torch conveniences. There is no CPU fallback: every
entry point raises if the library or a CUDA device is missing.
"""
from __future__ import annotations

import ctypes
import os

PACKAGE = os.path.dirname(os.path.abspath(__file__))
LIBRARY = os.path.join(PACKAGE, "libgfxb200.so")

W2, W3, W4 = 1, 2, 3
BITS_TO_FORMAT = {2: W2, 3: W3, 4: W4}

STATUS_NAMES = {0: "ok", 1: "invalid_argument", 2: "io_error", 3: "corrupt_artifact",
                4: "unsupported", 5: "cuda_error", 6: "out_of_memory", 7: "internal"}


class GfxbError(RuntimeError):
    def __init__(self, status: int, message: str) -> None:
        super().__init__(f"{STATUS_NAMES.get(status, status)}: {message}")
        self.status = status


_lib = None


def lib() -> ctypes.CDLL:
    """Load libgfxb200.so (built by gfxinfer_b200.build); raise if absent."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIBRARY):
            raise RuntimeError(f"{LIBRARY} is missing: run `python -m gfxinfer_b200.build` first")
        from . import abi

        _lib = ctypes.CDLL(LIBRARY)
        abi.declare(_lib)
    return _lib


def check(status: int) -> None:
    if status != 0:
        message = lib().gfxb_last_error_message().decode()
        raise GfxbError(status, message)
