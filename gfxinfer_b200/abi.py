"""ctypes declarations for every entry point in include/gfxb/gfxb.h."""
from __future__ import annotations

import ctypes
from ctypes import POINTER, c_char, c_char_p, c_int, c_size_t, c_uint, c_uint32, c_uint64, c_void_p


class DeviceInfo(ctypes.Structure):
    _fields_ = [("index", c_int), ("compute_major", c_int), ("compute_minor", c_int),
                ("multiprocessors", c_int), ("global_memory_bytes", c_uint64), ("name", c_char * 128)]


class GemvMatrix(ctypes.Structure):
    _fields_ = [("codes", c_void_p), ("scales", c_void_p), ("output", c_void_p),
                ("rows", c_size_t), ("output_f16", c_int)]


P = c_void_p

# name -> (restype, argtypes); kept in declaration order of include/gfxb/gfxb.h.
SIGNATURES: dict[str, tuple] = {
    "gfxb_last_error_message": (c_char_p, []),
    "gfxb_abi_version": (c_int, []),
    "gfxb_require_sm100_device": (c_int, [c_int, POINTER(DeviceInfo)]),
    "gfxb_repack_rowmajor_to_b200": (c_int, [c_int, P, P, c_size_t, c_size_t, P]),
    "gfxb_repack_gfx12_to_b200": (c_int, [c_int, P, P, c_size_t, c_size_t, P]),
    "gfxb_tile_scales": (c_int, [P, P, c_size_t, c_size_t, P]),
    "gfxb_pack_activation": (c_int, [c_int, P, P, P, P, P, c_size_t, c_uint, P]),
    "gfxb_lowbit_gemv": (c_int, [c_int, POINTER(GemvMatrix), c_uint, P, P, P, c_size_t, c_uint, P]),
    "gfxb_quantize_activation_i4": (c_int, [P, P, P, c_size_t, c_uint, P]),
    "gfxb_quantize_activation_i8": (c_int, [P, P, P, c_size_t, c_uint, P]),
    "gfxb_gfx12_i4_gemm": (c_int, [c_int, P, P, P, P, P, c_size_t, c_size_t, c_uint, c_int, P]),
    "gfxb_gfx12_i8_gemm": (c_int, [c_int, P, P, P, P, P, c_size_t, c_size_t, c_uint, P]),
}


def declare(lib: ctypes.CDLL) -> None:
    for name, (restype, argtypes) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = restype
        fn.argtypes = argtypes
