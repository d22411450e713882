"""`.gfxi` artifact files (include/gfxb/artifact.h) from Python.

Mirrors the reference's ArtifactView / ArtifactWriter (include/gfxinfer/artifact.h:
open, identity, tensors, find, data, auxiliary; write) over the C ABI. Tensor
payloads are exposed as read-only numpy views of the memory-mapped file.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass, field

import numpy as np

from . import abi, check, lib

DTYPE_U8, DTYPE_I32, DTYPE_F16, DTYPE_BF16, DTYPE_F32 = 1, 2, 3, 4, 5
QUANT_NONE, QUANT_W2G128, QUANT_W3G128, QUANT_W4G128, QUANT_W8G128, QUANT_FP8_ROW = 0, 1, 2, 3, 4, 5


def crc64(data, state: int = 0) -> int:
    """CRC64-ECMA (artifact.cpp:192-214) of a bytes-like object, continued from `state`."""
    buf = np.frombuffer(memoryview(data).cast("B"), np.uint8)
    out = ctypes.c_uint64()
    check(lib().gfxb_crc64_ecma(state, buf.ctypes.data if buf.size else None, buf.size, ctypes.byref(out)))
    return out.value


@dataclass
class Tensor:
    name: str
    dtype: int
    quantization: int
    dimensions: tuple
    data: np.ndarray
    aux: np.ndarray | None
    alignment: int
    data_offset: int
    aux_offset: int
    data_crc64: int


def _bytes_at(address: int, size: int) -> np.ndarray:
    if size == 0:
        return np.zeros(0, np.uint8)
    array = np.ctypeslib.as_array((ctypes.c_uint8 * size).from_address(address))
    array.flags.writeable = False
    return array


class Artifact:
    """A mapped, validated artifact (ArtifactView::open, artifact.cpp:274-407)."""

    def __init__(self, path: str, verify_checksums: bool = True) -> None:
        handle = ctypes.c_void_p()
        check(lib().gfxb_artifact_open(str(path).encode(), int(verify_checksums), ctypes.byref(handle)))
        self._handle = handle

    def close(self) -> None:
        if self._handle:
            lib().gfxb_artifact_close(self._handle)
            self._handle = ctypes.c_void_p()

    def __enter__(self):
        return self

    def __exit__(self, *exc) -> None:
        self.close()

    def __del__(self) -> None:
        try:
            self.close()
        except Exception:
            pass

    def identity(self) -> dict:
        ident = abi.ArtifactIdentity()
        check(lib().gfxb_artifact_identity_of(self._handle, ctypes.byref(ident)))
        return {k: getattr(ident, k).decode() for k in ("target_arch", "model_id", "weights_id", "recipe_id")}

    def file_bytes(self) -> int:
        out = ctypes.c_uint64()
        check(lib().gfxb_artifact_file_bytes(self._handle, ctypes.byref(out)))
        return out.value

    def _wrap(self, view: abi.TensorView) -> Tensor:
        dims = tuple(view.dimensions[i] for i in range(view.rank))
        return Tensor(view.name.decode(), view.dtype, view.quantization, dims, _bytes_at(view.data, view.data_bytes),
                      _bytes_at(view.aux, view.aux_bytes) if view.aux_bytes else None, view.alignment,
                      view.data_offset, view.aux_offset, view.data_crc64)

    def tensors(self) -> list[Tensor]:
        count = ctypes.c_size_t()
        check(lib().gfxb_artifact_tensor_count(self._handle, ctypes.byref(count)))
        out = []
        for i in range(count.value):
            view = abi.TensorView()
            check(lib().gfxb_artifact_tensor_at(self._handle, i, ctypes.byref(view)))
            out.append(self._wrap(view))
        return out

    def find(self, name: str) -> Tensor | None:
        view = abi.TensorView()
        found = ctypes.c_int()
        check(lib().gfxb_artifact_find(self._handle, name.encode(), ctypes.byref(view), ctypes.byref(found)))
        return self._wrap(view) if found.value else None


@dataclass
class TensorWrite:
    name: str
    dtype: int
    quantization: int
    dimensions: tuple
    data: bytes | np.ndarray
    aux: bytes | np.ndarray | None = None
    alignment: int = 256
    _keep: list = field(default_factory=list, repr=False)


def _buffer(value) -> np.ndarray:
    return np.ascontiguousarray(np.frombuffer(memoryview(value).cast("B"), np.uint8))


def write(path: str, identity: dict, tensors: list[TensorWrite]) -> None:
    """ArtifactWriter::write (artifact.cpp:426-562): atomic write of a whole artifact."""
    ident = abi.ArtifactIdentity(*(identity[k].encode() for k in ("target_arch", "model_id", "weights_id", "recipe_id")))
    items = (abi.TensorWrite * max(1, len(tensors)))()
    keep = []
    for i, t in enumerate(tensors):
        data = _buffer(t.data)
        aux = _buffer(t.aux) if t.aux is not None else np.zeros(0, np.uint8)
        name = t.name.encode()
        keep += [data, aux, name]
        dims = (ctypes.c_uint64 * 4)(*(list(t.dimensions) + [0] * (4 - len(t.dimensions))))
        items[i] = abi.TensorWrite(name, t.dtype, t.quantization, len(t.dimensions), dims,
                                   data.ctypes.data if data.size else None, data.size,
                                   aux.ctypes.data if aux.size else None, aux.size, t.alignment)
    check(lib().gfxb_artifact_write(str(path).encode(), ctypes.byref(ident), items, len(tensors)))


LAYOUT_B200, LAYOUT_GFX12 = 0, 1


def convert(path: str, identity: dict, tensors: dict, layout: int = LAYOUT_B200, mlp_bits: int = 3,
            w3_start_layer: int = 0, w4_tail_layers: int = 0, head_bits: int = 4, layers: int | None = None,
            chunk_rows: int = 1024, device: int = 0) -> None:
    """convert_qwen38 (converter.cpp) for in-memory weights: `tensors` maps reference tensor names to
    float32 or bfloat16 arrays (numpy float32, or uint16 arrays holding bf16 bits). 2-D tensors are
    quantized on `device` by choose_quantization's rules, the rest stored as bf16."""
    ident = abi.ArtifactIdentity(*(identity[k].encode() for k in ("target_arch", "model_id", "weights_id", "recipe_id")))
    if layers is None:
        prefix = "model.language_model.layers."
        ids = [int(n[len(prefix):].split(".")[0]) for n in tensors if n.startswith(prefix)]
        layers = max(ids) + 1 if ids else 0
    items = (abi.ConvertSource * len(tensors))()
    keep = []
    for i, (name, array) in enumerate(tensors.items()):
        array = np.ascontiguousarray(array)
        if array.dtype == np.float32:
            dtype = DTYPE_F32
        elif array.dtype == np.uint16:
            dtype = DTYPE_BF16
        else:
            raise TypeError(f"{name}: weights must be float32 or bf16 bits (uint16)")
        encoded = name.encode()
        keep += [array, encoded]
        dims = (ctypes.c_uint64 * 4)(*(list(array.shape) + [0] * (4 - array.ndim)))
        items[i] = abi.ConvertSource(encoded, dtype, array.ndim, dims, array.ctypes.data, array.nbytes)
    options = abi.ConvertOptions(layout, mlp_bits, w3_start_layer, w4_tail_layers, head_bits, layers, chunk_rows)
    check(lib().gfxb_convert_to_artifact(str(path).encode(), ctypes.byref(ident), items, len(tensors),
                                         ctypes.byref(options), device))
