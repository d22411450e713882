"""ctypes bindings to the CPU oracle (oracle/_build/liboracle.so).

Test infrastructure: only tests/, __graft_entry__.smoke() and bench.py's
CPU-baseline leg use this module, always as the checker.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from ctypes import POINTER, c_double, c_float, c_int, c_size_t, c_uint, c_uint16, c_uint32, c_uint64, c_void_p

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
ORACLE_SO = os.path.join(ROOT, "oracle", "_build", "liboracle.so")
REF_SO = os.path.join(ROOT, "oracle", "_ref", "libgfxref.so")

W2, W3, W4 = 1, 2, 3
BITS_TO_FORMAT = {2: W2, 3: W3, 4: W4}


def _ptr(array: np.ndarray) -> c_void_p:
    return c_void_p(array.ctypes.data) if array is not None else c_void_p(0)


def build_oracle() -> None:
    if not os.path.exists(ORACLE_SO):
        subprocess.run(["make", "-C", os.path.join(ROOT, "oracle"), "oracle"], check=True,
                       stdout=subprocess.DEVNULL)


class ModelConfig(ctypes.Structure):
    _fields_ = [
        ("hidden", c_uint32), ("intermediate", c_uint32), ("layers", c_uint32),
        ("attention_interval", c_uint32), ("gdn_key_heads", c_uint32),
        ("gdn_value_heads", c_uint32), ("q_heads", c_uint32), ("kv_heads", c_uint32),
        ("vocab", c_uint32), ("draft_vocab", c_uint32), ("mlp_bits", c_uint32),
        ("proj_bits", c_uint32), ("head_bits", c_uint32), ("emb_bits", c_uint32),
        ("activation_bits", c_uint32), ("max_context", c_uint32), ("seed", c_uint64),
    ]


def model_config(**kw) -> ModelConfig:
    """Full-size defaults are BASELINE config 2 (64 layers, vocab 151936, W3 MLP, W4 rest, A4)."""
    defaults = dict(hidden=5120, intermediate=17408, layers=64, attention_interval=4,
                    gdn_key_heads=16, gdn_value_heads=48, q_heads=24, kv_heads=4,
                    vocab=151936, draft_vocab=98304, mlp_bits=3, proj_bits=4, head_bits=4,
                    emb_bits=4, activation_bits=4, max_context=512, seed=0x5EED)
    defaults.update(kw)
    return ModelConfig(**defaults)


SMALL_MODEL = dict(hidden=1024, intermediate=2048, layers=8, gdn_key_heads=4, gdn_value_heads=16,
                   q_heads=8, kv_heads=2, vocab=4096, draft_vocab=3072, max_context=320)
"""Every dimension of BASELINE config 2 scaled down, same structure (3 GDN : 1 attention layers)."""


class Oracle:
    def __init__(self) -> None:
        build_oracle()
        lib = ctypes.CDLL(ORACLE_SO)
        self.lib = lib
        sig = {
            "or_f32_to_f16": (c_uint16, [c_float]),
            "or_f16_to_f32": (c_float, [c_uint16]),
            "or_f32_to_bf16": (c_uint16, [c_float]),
            "or_expf": (c_float, [c_float]),
            "or_log1pf": (c_float, [c_float]),
            "or_packed_row_bytes": (c_size_t, [c_int, c_size_t]),
            "or_quantize_group128": (c_int, [c_void_p, c_size_t, c_size_t, c_int, c_void_p, c_void_p]),
            "or_tile_gfx12": (c_int, [c_void_p, c_void_p, c_size_t, c_size_t, c_int, c_void_p, c_void_p]),
            "or_unpack_logical": (None, [c_void_p, c_size_t, c_size_t, c_int, c_void_p]),
            "or_quantize_activation_i4": (None, [c_void_p, c_size_t, c_uint, c_void_p, c_void_p]),
            "or_quantize_activation_i8": (None, [c_void_p, c_size_t, c_uint, c_void_p, c_void_p]),
            "or_unpack_a4": (None, [c_void_p, c_size_t, c_void_p]),
            "or_gemv_int": (None, [c_void_p, c_void_p, c_size_t, c_size_t, c_void_p, c_void_p, c_uint, c_void_p]),
            "or_gemv_f16": (None, [c_void_p, c_void_p, c_size_t, c_size_t, c_void_p, c_uint, c_void_p]),
            "or_rms_norm": (None, [c_void_p, c_void_p, c_size_t, c_float, c_int, c_void_p]),
            "or_residual_add_rms_norm": (None, [c_void_p, c_void_p, c_void_p, c_size_t, c_float, c_int, c_void_p, c_void_p]),
            "or_silu_multiply_f16": (None, [c_void_p, c_void_p, c_size_t, c_void_p]),
            "or_gdn_conv_update": (None, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_size_t, c_uint]),
            "or_gdn_recurrent": (None, [c_void_p] * 12 + [c_uint, c_uint, c_uint]),
            "or_gdn_restore": (None, [c_void_p] * 6 + [c_size_t, c_uint, c_uint, c_uint]),
            "or_rope_table": (None, [c_size_t, c_uint, c_float, c_void_p, c_void_p]),
            "or_qk_norm_rope": (None, [c_void_p, c_size_t, c_void_p, c_uint, c_size_t, c_void_p, c_void_p, c_uint, c_void_p]),
            "or_gated_attention": (None, [c_void_p, c_void_p, c_void_p, c_void_p, c_size_t, c_uint, c_uint, c_void_p]),
            "or_argmax": (c_uint32, [c_void_p, c_size_t]),
            "or_model_create": (c_void_p, [POINTER(ModelConfig), c_int]),
            "or_model_create_cycled": (c_void_p, [POINTER(ModelConfig), c_uint]),
            "or_model_block_step": (c_int, [c_void_p, c_void_p, c_uint, c_void_p]),
            "or_model_prefill": (c_int, [c_void_p, c_void_p, c_size_t]),
            "or_model_destroy": (None, [c_void_p]),
            "or_model_greedy_step": (c_int, [c_void_p, c_uint32, POINTER(c_uint32)]),
            "or_model_mtp_draft": (c_int, [c_void_p, c_uint32, c_int, POINTER(c_uint32)]),
            "or_model_position": (c_size_t, [c_void_p]),
            "or_model_timing": (None, [c_void_p, POINTER(c_double), POINTER(c_double), POINTER(c_size_t)]),
            "or_set_threads": (c_int, [c_int]),
            "or_model_last_hidden": (c_void_p, [c_void_p]),
            "or_model_logits": (c_void_p, [c_void_p]),
            "or_prompt_token": (c_uint32, [c_uint64, c_uint32, c_uint32]),
            "or_gen_codes_rowmajor": (None, [c_uint64, c_uint32, c_size_t, c_size_t, c_int, c_void_p]),
            "or_gen_scales": (None, [c_uint64, c_uint32, c_size_t, c_int, c_void_p]),
            "or_gen_bf16": (None, [c_uint64, c_uint32, c_size_t, c_float, c_float, c_void_p]),
        }
        for name, (restype, argtypes) in sig.items():
            fn = getattr(lib, name)
            fn.restype = restype
            fn.argtypes = argtypes

    # -- packing --------------------------------------------------------------
    def quantize(self, weights: np.ndarray, fmt: int):
        weights = np.ascontiguousarray(weights, dtype=np.float32)
        rows, cols = weights.shape
        codes = np.zeros(rows * self.lib.or_packed_row_bytes(fmt, cols), np.uint8)
        scales = np.zeros(rows * (cols // 128) if cols % 128 == 0 else 1, np.float32)
        status = self.lib.or_quantize_group128(_ptr(weights), rows, cols, fmt, _ptr(codes), _ptr(scales))
        return status, codes, scales

    def tile(self, codes, scales, rows, cols, fmt):
        tiled = np.zeros_like(codes)
        tiled_scales = np.zeros_like(scales)
        status = self.lib.or_tile_gfx12(_ptr(codes), _ptr(scales), rows, cols, fmt, _ptr(tiled), _ptr(tiled_scales))
        return status, tiled, tiled_scales

    def logical(self, codes, rows, cols, fmt) -> np.ndarray:
        out = np.zeros((rows, cols), np.int8)
        self.lib.or_unpack_logical(_ptr(codes), rows, cols, fmt, _ptr(out))
        return out

    # -- activations ------------------------------------------------------------
    def quantize_a4(self, x_f16: np.ndarray):
        x = np.ascontiguousarray(x_f16, dtype=np.float16)
        batch, cols = x.shape
        packed = np.zeros((batch, cols // 2), np.uint8)
        scales = np.zeros((batch, cols // 128), np.float16)
        self.lib.or_quantize_activation_i4(_ptr(x), cols, batch, _ptr(packed), _ptr(scales))
        values = np.zeros((batch, cols), np.int8)
        self.lib.or_unpack_a4(_ptr(packed), batch * cols, _ptr(values))
        return packed, scales, values

    def quantize_a8(self, x_f16: np.ndarray):
        x = np.ascontiguousarray(x_f16, dtype=np.float16)
        batch, cols = x.shape
        q = np.zeros((batch, cols), np.int8)
        scales = np.zeros((batch, cols // 128), np.float16)
        self.lib.or_quantize_activation_i8(_ptr(x), cols, batch, _ptr(q), _ptr(scales))
        return q, scales

    def gemv(self, w_logical: np.ndarray, w_scales_f16: np.ndarray, a: np.ndarray, a_scales_f16: np.ndarray) -> np.ndarray:
        rows, cols = w_logical.shape
        batch = a.shape[0]
        out = np.zeros((batch, rows), np.float32)
        self.lib.or_gemv_int(_ptr(np.ascontiguousarray(w_logical)), _ptr(np.ascontiguousarray(w_scales_f16)), rows, cols,
                             _ptr(np.ascontiguousarray(a)), _ptr(np.ascontiguousarray(a_scales_f16)), batch, _ptr(out))
        return out

    def gemv_f16(self, w_logical, w_scales_f16, x_f16) -> np.ndarray:
        rows, cols = w_logical.shape
        batch = x_f16.shape[0]
        out = np.zeros((batch, rows), np.float64)
        self.lib.or_gemv_f16(_ptr(np.ascontiguousarray(w_logical)), _ptr(np.ascontiguousarray(w_scales_f16)), rows, cols,
                             _ptr(np.ascontiguousarray(x_f16, dtype=np.float16)), batch, _ptr(out))
        return out


class Reference:
    """The reference's own src/quantization.cpp and src/artifact.cpp, built by oracle/Makefile into oracle/_ref."""

    def __init__(self) -> None:
        lib = ctypes.CDLL(REF_SO)
        self.lib = lib
        lib.ref_quantize_group128.restype = c_int
        lib.ref_quantize_group128.argtypes = [c_void_p, c_size_t, c_size_t, c_int, c_void_p, c_void_p]
        lib.ref_tile_gfx12.restype = c_int
        lib.ref_tile_gfx12.argtypes = [c_void_p, c_void_p, c_size_t, c_size_t, c_int, c_void_p, c_void_p]
        lib.ref_packed_row_bytes.restype = c_size_t
        lib.ref_packed_row_bytes.argtypes = [c_int, c_size_t]
        lib.ref_test_matrix.restype = None
        lib.ref_test_matrix.argtypes = [c_uint, c_float, c_size_t, c_void_p]
        lib.ref_dequantized_weight.restype = c_float
        lib.ref_dequantized_weight.argtypes = [c_void_p, c_void_p, c_size_t, c_size_t, c_int, c_size_t, c_size_t]

        lib.ref_artifact_write.restype = c_int
        lib.ref_artifact_write.argtypes = [ctypes.c_char_p] * 5 + [c_size_t] + [c_void_p] * 10
        lib.ref_artifact_open.restype = c_int
        lib.ref_artifact_open.argtypes = [ctypes.c_char_p, c_int, c_void_p, c_void_p]
        lib.ref_artifact_tensor.restype = c_int
        lib.ref_artifact_tensor.argtypes = [ctypes.c_char_p, c_size_t, c_void_p, c_void_p, c_void_p, c_void_p]

    @staticmethod
    def available() -> bool:
        return os.path.exists(REF_SO)

    # -- .gfxi container (src/artifact.cpp) ---------------------------------------
    def artifact_write(self, path: str, identity: dict, tensors: list) -> int:
        """tensors: list of (name, dtype, quantization, dims, data_bytes_obj, aux_bytes_obj_or_None, alignment)."""
        n = len(tensors)
        keep = []
        names = (ctypes.c_char_p * n)(*[t[0].encode() for t in tensors])
        dtypes = np.array([t[1] for t in tensors], np.uint16)
        quants = np.array([t[2] for t in tensors], np.uint16)
        ranks = np.array([len(t[3]) for t in tensors], np.uint16)
        dims = np.zeros((n, 4), np.uint64)
        data_ptrs, aux_ptrs = (c_void_p * n)(), (c_void_p * n)()
        data_bytes, aux_bytes = np.zeros(n, np.uint64), np.zeros(n, np.uint64)
        alignments = np.array([t[6] if len(t) > 6 else 256 for t in tensors], np.uint32)
        for i, (_, _, _, shape, data, aux, *_) in enumerate(tensors):
            dims[i, :len(shape)] = shape
            d = np.frombuffer(memoryview(data).cast("B"), np.uint8)
            keep.append(d)
            data_ptrs[i], data_bytes[i] = d.ctypes.data, d.size
            if aux is not None:
                a = np.frombuffer(memoryview(aux).cast("B"), np.uint8)
                keep.append(a)
                aux_ptrs[i], aux_bytes[i] = a.ctypes.data, a.size
        ident = [identity[k].encode() for k in ("target_arch", "model_id", "weights_id", "recipe_id")]
        return self.lib.ref_artifact_write(str(path).encode(), *ident, n, names, _ptr(dtypes), _ptr(quants),
                                           _ptr(ranks), _ptr(dims), data_ptrs, _ptr(data_bytes), aux_ptrs,
                                           _ptr(aux_bytes), _ptr(alignments))

    def artifact_open(self, path: str, verify: bool = True):
        count, size = np.zeros(1, np.uint64), np.zeros(1, np.uint64)
        status = self.lib.ref_artifact_open(str(path).encode(), int(verify), _ptr(count), _ptr(size))
        return status, int(count[0]), int(size[0])

    def artifact_tensor(self, path: str, index: int) -> dict:
        name = ctypes.create_string_buffer(256)
        dims, meta, spans = np.zeros(4, np.uint64), np.zeros(3, np.uint16), np.zeros(5, np.uint64)
        status = self.lib.ref_artifact_tensor(str(path).encode(), index, name, _ptr(dims), _ptr(meta), _ptr(spans))
        assert status == 0, status
        rank = int(meta[2])
        return {"name": name.value.decode(), "dtype": int(meta[0]), "quantization": int(meta[1]),
                "dimensions": tuple(int(d) for d in dims[:rank]), "data_offset": int(spans[0]),
                "data_bytes": int(spans[1]), "aux_offset": int(spans[2]), "aux_bytes": int(spans[3]),
                "data_crc64": int(spans[4])}

    def test_matrix(self, seed: int, stddev: float, rows: int, cols: int) -> np.ndarray:
        out = np.zeros(rows * cols, np.float32)
        self.lib.ref_test_matrix(seed, stddev, out.size, _ptr(out))
        return out.reshape(rows, cols)

    def quantize(self, weights: np.ndarray, fmt: int):
        weights = np.ascontiguousarray(weights, dtype=np.float32)
        rows, cols = weights.shape
        codes = np.zeros(rows * self.lib.ref_packed_row_bytes(fmt, cols), np.uint8)
        scales = np.zeros(max(1, rows * (cols // 128)), np.float32)
        status = self.lib.ref_quantize_group128(_ptr(weights), rows, cols, fmt, _ptr(codes), _ptr(scales))
        return status, codes, scales

    def tile(self, codes, scales, rows, cols, fmt):
        tiled = np.zeros_like(codes)
        tiled_scales = np.zeros_like(scales)
        status = self.lib.ref_tile_gfx12(_ptr(codes), _ptr(scales), rows, cols, fmt, _ptr(tiled), _ptr(tiled_scales))
        return status, tiled, tiled_scales


class OracleModel:
    """Scalar forward of the synthetic model (oracle.c or_model_*)."""

    def __init__(self, oracle: Oracle, config: ModelConfig, include_mtp: bool = True,
                 resident_layers: int = 0) -> None:
        """resident_layers > 0: every layer runs but only that many hold their own weights (timing only)."""
        self.oracle = oracle
        self.config = config
        if resident_layers:
            handle = oracle.lib.or_model_create_cycled(ctypes.byref(config), resident_layers)
        else:
            handle = oracle.lib.or_model_create(ctypes.byref(config), int(include_mtp))
        self.handle = c_void_p(handle)

    def greedy_step(self, token: int) -> int:
        out = c_uint32()
        assert self.oracle.lib.or_model_greedy_step(self.handle, token, ctypes.byref(out)) == 0
        return out.value

    def block_step(self, tokens) -> list[int]:
        """Up to 64 tokens, layer-major; one argmax per token (same bits as stepping them one by one)."""
        ids = np.ascontiguousarray(tokens, dtype=np.uint32)
        out = np.zeros(len(ids), np.uint32)
        assert self.oracle.lib.or_model_block_step(self.handle, _ptr(ids), len(ids), _ptr(out)) == 0
        return [int(x) for x in out]

    def prefill(self, tokens) -> None:
        """A prompt of any length without the LM head."""
        ids = np.ascontiguousarray(tokens, dtype=np.uint32)
        assert self.oracle.lib.or_model_prefill(self.handle, _ptr(ids), len(ids)) == 0

    def position(self) -> int:
        return int(self.oracle.lib.or_model_position(self.handle))

    def mtp_draft(self, token: int, use_mtp_hidden: bool = False) -> int:
        out = c_uint32()
        assert self.oracle.lib.or_model_mtp_draft(self.handle, token, int(use_mtp_hidden), ctypes.byref(out)) == 0
        return out.value

    def timing(self):
        layer, head, tokens = c_double(), c_double(), c_size_t()
        self.oracle.lib.or_model_timing(self.handle, ctypes.byref(layer), ctypes.byref(head), ctypes.byref(tokens))
        return layer.value, head.value, tokens.value

    def last_hidden(self) -> np.ndarray:
        ptr = self.oracle.lib.or_model_last_hidden(self.handle)
        return np.ctypeslib.as_array(ctypes.cast(ptr, POINTER(ctypes.c_uint16)), (self.config.hidden,)).copy()

    def logits(self) -> np.ndarray:
        ptr = self.oracle.lib.or_model_logits(self.handle)
        return np.ctypeslib.as_array(ctypes.cast(ptr, POINTER(ctypes.c_float)), (self.config.vocab,)).copy()

    def close(self) -> None:
        if self.handle:
            self.oracle.lib.or_model_destroy(self.handle)
            self.handle = c_void_p()

    def __del__(self) -> None:
        try:
            self.close()
        except Exception:
            pass


def prompt_tokens(oracle: Oracle, seed: int, vocab: int, count: int) -> list[int]:
    return [oracle.lib.or_prompt_token(seed, vocab, i) for i in range(count)]
