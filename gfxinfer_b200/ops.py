"""Torch-tensor conveniences over the C ABI (device memory and streams only).

Every function launches the library's CUDA kernels on the current torch
stream; torch supplies allocation, nothing else.
"""
from __future__ import annotations

import torch

from . import abi, check, lib


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _p(t: torch.Tensor | None) -> int:
    return 0 if t is None else t.data_ptr()


def require_sm100(index: int = 0) -> abi.DeviceInfo:
    info = abi.DeviceInfo()
    check(lib().gfxb_require_sm100_device(index, info))
    return info


def repack_rowmajor(fmt: int, codes: torch.Tensor, rows: int, cols: int) -> torch.Tensor:
    out = torch.empty_like(codes)
    check(lib().gfxb_repack_rowmajor_to_b200(fmt, _p(codes), _p(out), rows, cols, _stream()))
    return out


def repack_gfx12(fmt: int, codes: torch.Tensor, rows: int, cols: int) -> torch.Tensor:
    out = torch.empty_like(codes)
    check(lib().gfxb_repack_gfx12_to_b200(fmt, _p(codes), _p(out), rows, cols, _stream()))
    return out


def tile_scales(scales_f16: torch.Tensor, rows: int, cols: int) -> torch.Tensor:
    out = torch.empty_like(scales_f16)
    check(lib().gfxb_tile_scales(_p(scales_f16), _p(out), rows, cols, _stream()))
    return out


def pack_activation(x_f16: torch.Tensor, bits: int = 4, want_packed_a4: bool = False):
    batch, cols = x_f16.shape
    dev = x_f16.device
    codes = torch.empty((batch, cols), dtype=torch.int8, device=dev)
    scales = torch.empty((batch, cols // 128), dtype=torch.float16, device=dev)
    sums = torch.empty((batch, cols // 128), dtype=torch.int32, device=dev)
    packed = torch.empty((batch, cols // 2), dtype=torch.uint8, device=dev) if want_packed_a4 else None
    check(lib().gfxb_pack_activation(bits, _p(x_f16), _p(codes), _p(scales), _p(sums), _p(packed), cols,
                                     batch, _stream()))
    return codes, scales, sums, packed


def lowbit_gemv(fmt: int, matrices, act_codes, act_scales, act_sums, cols: int, batch: int) -> None:
    """matrices: list of (codes, tiled_scales, output, rows, output_f16)."""
    arr = (abi.GemvMatrix * len(matrices))()
    for i, (codes, scales, output, rows, f16) in enumerate(matrices):
        arr[i] = abi.GemvMatrix(_p(codes), _p(scales), _p(output), rows, int(f16))
    check(lib().gfxb_lowbit_gemv(fmt, arr, len(matrices), _p(act_codes), _p(act_scales), _p(act_sums),
                                 cols, batch, _stream()))


def quantize_a4(x_f16: torch.Tensor):
    batch, cols = x_f16.shape
    packed = torch.empty((batch, cols // 2), dtype=torch.uint8, device=x_f16.device)
    scales = torch.empty((batch, cols // 128), dtype=torch.float16, device=x_f16.device)
    check(lib().gfxb_quantize_activation_i4(_p(x_f16), _p(packed), _p(scales), cols, batch, _stream()))
    return packed, scales


def quantize_a8(x_f16: torch.Tensor):
    batch, cols = x_f16.shape
    q = torch.empty((batch, cols), dtype=torch.int8, device=x_f16.device)
    scales = torch.empty((batch, cols // 128), dtype=torch.float16, device=x_f16.device)
    check(lib().gfxb_quantize_activation_i8(_p(x_f16), _p(q), _p(scales), cols, batch, _stream()))
    return q, scales


def gfx12_i4_gemm(fmt, tiled, tiled_scales, packed_a4, a_scales, rows, cols, batch):
    out = torch.empty((batch, rows), dtype=torch.float32, device=tiled.device)
    check(lib().gfxb_gfx12_i4_gemm(fmt, _p(tiled), _p(tiled_scales), _p(packed_a4), _p(a_scales), _p(out),
                                   rows, cols, batch, 1, _stream()))
    return out


def gfx12_i8_gemm(fmt, tiled, tiled_scales, a8, a_scales, rows, cols, batch):
    out = torch.empty((batch, rows), dtype=torch.float32, device=tiled.device)
    check(lib().gfxb_gfx12_i8_gemm(fmt, _p(tiled), _p(tiled_scales), _p(a8), _p(a_scales), _p(out),
                                   rows, cols, batch, _stream()))
    return out


def lowbit_gemv_f16(fmt: int, matrices, x_f16: torch.Tensor) -> None:
    """fp16-activation GEMV; matrices: list of (codes, tiled_scales, output, rows, output_f16)."""
    batch, cols = x_f16.shape
    arr = (abi.GemvMatrix * len(matrices))()
    for i, (codes, scales, output, rows, f16) in enumerate(matrices):
        arr[i] = abi.GemvMatrix(_p(codes), _p(scales), _p(output), rows, int(f16))
    check(lib().gfxb_lowbit_gemv_f16(fmt, arr, len(matrices), _p(x_f16), cols, batch, _stream()))


def gfx12_f16_gemm(fmt, tiled, tiled_scales, x_f16, rows, cols, batch):
    out = torch.empty((batch, rows), dtype=torch.float32, device=tiled.device)
    check(lib().gfxb_gfx12_f16_gemm(fmt, _p(tiled), _p(tiled_scales), _p(x_f16), _p(out), rows, cols, batch,
                                    _stream()))
    return out


# ---- weight packing (the reference's src/quantization.cpp on the device) ------

DTYPE_F32, DTYPE_BF16 = 5, 4
LAYOUT_B200, LAYOUT_GFX12, LAYOUT_ROWMAJOR = 0, 1, 2


def _dtype_code(weights: torch.Tensor) -> int:
    if weights.dtype == torch.float32:
        return DTYPE_F32
    if weights.dtype == torch.bfloat16:
        return DTYPE_BF16
    raise TypeError("weights must be float32 or bfloat16")


def packed_row_bytes(fmt: int, cols: int) -> int:
    return int(lib().gfxb_packed_row_bytes(fmt, cols))


def quantize_group128(fmt: int, weights: torch.Tensor):
    """quantize_group128 (quantization.cpp:163-220): [N][K] fp32/bf16 -> (row-major codes, fp32 scales)."""
    rows, cols = weights.shape
    weights = weights.contiguous()
    codes = torch.empty(rows * packed_row_bytes(fmt, cols), dtype=torch.uint8, device=weights.device)
    scales = torch.empty((rows, cols // 128), dtype=torch.float32, device=weights.device)
    check(lib().gfxb_quantize_group128(fmt, _dtype_code(weights), _p(weights), rows, cols, _p(codes), _p(scales),
                                       _stream()))
    return codes, scales


def tile_group128_for_gfx12(fmt: int, codes: torch.Tensor, scales: torch.Tensor, rows: int, cols: int):
    """tile_group128_for_gfx12 (quantization.cpp:253-318) on the device."""
    tiled = torch.empty_like(codes)
    tiled_scales = torch.empty_like(scales)
    check(lib().gfxb_tile_group128_for_gfx12(fmt, _p(codes), _p(scales), rows, cols, _p(tiled), _p(tiled_scales),
                                             _stream()))
    return tiled, tiled_scales


def dequantize_group128(fmt: int, codes: torch.Tensor, scales: torch.Tensor, rows: int, cols: int) -> torch.Tensor:
    out = torch.empty((rows, cols), dtype=torch.float32, device=codes.device)
    check(lib().gfxb_dequantize_group128(fmt, _p(codes), _p(scales), rows, cols, _p(out), _stream()))
    return out


def convert_group128(fmt: int, weights: torch.Tensor, layout: int = LAYOUT_B200):
    """write_quantized (converter.cpp:345-393) for one weight: codes in `layout` and fp16 scales."""
    rows, cols = weights.shape
    weights = weights.contiguous()
    dev = weights.device
    codes = torch.empty(rows * packed_row_bytes(fmt, cols), dtype=torch.uint8, device=dev)
    scales = torch.empty(rows * (cols // 128), dtype=torch.float16, device=dev)
    scratch = torch.empty(int(lib().gfxb_convert_scratch_bytes(fmt, rows, cols)), dtype=torch.uint8, device=dev)
    check(lib().gfxb_convert_group128(fmt, _dtype_code(weights), _p(weights), rows, cols, layout, _p(codes),
                                      _p(scales), _p(scratch), scratch.numel(), _stream()))
    return codes, scales
