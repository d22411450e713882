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

class ModelConfig(ctypes.Structure):
    _fields_ = [(name, c_uint32) for name in (
        "hidden", "intermediate", "layers", "attention_interval", "gdn_key_heads", "gdn_value_heads",
        "q_heads", "kv_heads", "vocab", "draft_vocab", "mlp_bits", "proj_bits", "head_bits", "emb_bits",
        "activation_bits", "max_context")] + [("seed", c_uint64)]


class SessionConfig(ctypes.Structure):
    _fields_ = [("maximum_context_tokens", c_uint32), ("graph_verifier_batch", c_uint32), ("use_graphs", c_uint32),
                ("step_kernel", c_uint32)]


STEP_AUTO, STEP_LAUNCHES, STEP_PERSISTENT = 0, 1, 2


class TpShardInfo(ctypes.Structure):
    _fields_ = [(name, c_uint32) for name in (
        "gdn_key_heads", "gdn_key_head0", "gdn_value_heads", "gdn_value_head0", "q_heads", "q_head0",
        "kv_heads", "kv_head0", "intermediate", "intermediate0", "vocab", "vocab0", "fc_columns", "fc_column0",
        "gdn_channels")]


class ArtifactIdentity(ctypes.Structure):
    _fields_ = [("target_arch", c_char * 16), ("model_id", c_char * 32), ("weights_id", c_char * 32),
                ("recipe_id", c_char * 64)]


class TensorView(ctypes.Structure):
    _fields_ = [("name", c_char_p), ("dtype", ctypes.c_uint16), ("quantization", ctypes.c_uint16),
                ("rank", ctypes.c_uint16), ("flags", ctypes.c_uint16), ("alignment", c_uint32),
                ("dimensions", c_uint64 * 4), ("data", c_void_p), ("data_bytes", c_uint64), ("aux", c_void_p),
                ("aux_bytes", c_uint64), ("data_offset", c_uint64), ("aux_offset", c_uint64),
                ("data_crc64", c_uint64)]


class TensorWrite(ctypes.Structure):
    _fields_ = [("name", c_char_p), ("dtype", ctypes.c_uint16), ("quantization", ctypes.c_uint16),
                ("rank", ctypes.c_uint16), ("dimensions", c_uint64 * 4), ("data", c_void_p), ("data_bytes", c_uint64),
                ("aux", c_void_p), ("aux_bytes", c_uint64), ("alignment", c_uint32)]


class ConvertSource(ctypes.Structure):
    _fields_ = [("name", c_char_p), ("dtype", ctypes.c_uint16), ("rank", ctypes.c_uint16),
                ("dimensions", c_uint64 * 4), ("data", c_void_p), ("data_bytes", c_uint64)]


class ConvertOptions(ctypes.Structure):
    _fields_ = [(name, c_uint32) for name in (
        "layout", "mlp_bits", "w3_start_layer", "w4_tail_layers", "head_bits", "layers", "chunk_rows")]


class ArtifactLoadOptions(ctypes.Structure):
    _fields_ = [(name, c_uint32) for name in (
        "activation_bits", "max_context", "draft_vocab", "include_mtp", "verify_checksums")]


# name -> (restype, argtypes); kept in declaration order of include/gfxb/gfxb.h, then artifact.h.
SIGNATURES: dict[str, tuple] = {
    "gfxb_last_error_message": (c_char_p, []),
    "gfxb_abi_version": (c_int, []),
    "gfxb_require_sm100_device": (c_int, [c_int, POINTER(DeviceInfo)]),
    "gfxb_repack_rowmajor_to_b200": (c_int, [c_int, P, P, c_size_t, c_size_t, P]),
    "gfxb_repack_gfx12_to_b200": (c_int, [c_int, P, P, c_size_t, c_size_t, P]),
    "gfxb_tile_scales": (c_int, [P, P, c_size_t, c_size_t, P]),
    "gfxb_packed_row_bytes": (c_size_t, [c_int, c_size_t]),
    "gfxb_quantize_group128": (c_int, [c_int, c_int, P, c_size_t, c_size_t, P, P, P]),
    "gfxb_tile_group128_for_gfx12": (c_int, [c_int, P, P, c_size_t, c_size_t, P, P, P]),
    "gfxb_dequantize_group128": (c_int, [c_int, P, P, c_size_t, c_size_t, P, P]),
    "gfxb_dequantized_weight": (ctypes.c_float, [c_int, P, P, c_size_t, c_size_t, c_size_t, c_size_t]),
    "gfxb_convert_scratch_bytes": (c_size_t, [c_int, c_size_t, c_size_t]),
    "gfxb_convert_group128": (c_int, [c_int, c_int, P, c_size_t, c_size_t, c_int, P, P, P, c_size_t, P]),
    "gfxb_pack_activation": (c_int, [c_int, P, P, P, P, P, c_size_t, c_uint, P]),
    "gfxb_lowbit_gemv": (c_int, [c_int, POINTER(GemvMatrix), c_uint, P, P, P, c_size_t, c_uint, P]),
    "gfxb_quantize_activation_i4": (c_int, [P, P, P, c_size_t, c_uint, P]),
    "gfxb_quantize_activation_i8": (c_int, [P, P, P, c_size_t, c_uint, P]),
    "gfxb_gfx12_i4_gemm": (c_int, [c_int, P, P, P, P, P, c_size_t, c_size_t, c_uint, c_int, P]),
    "gfxb_gfx12_i8_gemm": (c_int, [c_int, P, P, P, P, P, c_size_t, c_size_t, c_uint, P]),
    "gfxb_lowbit_gemv_f16": (c_int, [c_int, POINTER(GemvMatrix), c_uint, P, c_size_t, c_uint, P]),
    "gfxb_gfx12_f16_gemm": (c_int, [c_int, P, P, P, P, c_size_t, c_size_t, c_uint, P]),
    "gfxb_residual_rms_norm_pack": (c_int, [P, P, P, P, P, c_size_t, c_uint, ctypes.c_float, c_int, c_int, P, P, P, P, P]),
    "gfxb_silu_multiply_pack": (c_int, [P, P, c_size_t, c_uint, P, c_int, P, P, P, P, P]),
    "gfxb_gdn_conv_update": (c_int, [P, P, P, P, P, P, c_size_t, c_uint, P]),
    "gfxb_gdn_recurrent": (c_int, [P] * 13 + [c_uint, c_uint, c_uint, P]),
    "gfxb_gdn_restore_prefix_all": (c_int, [P] * 6 + [c_size_t, c_uint, c_uint, c_uint, c_uint, c_uint, P]),
    "gfxb_rope_table": (c_int, [c_size_t, c_uint, ctypes.c_float, P, P]),
    "gfxb_qk_rms_norm_rope": (c_int, [P, P, P, c_uint, c_size_t, P, P, P, c_uint, c_size_t, c_uint, P, P, c_size_t,
                                      c_uint64, P, c_uint, P, P, P, c_size_t, P]),
    "gfxb_gated_attention_scratch_bytes": (c_size_t, [c_uint, c_size_t, c_uint]),
    "gfxb_decode_attention_scratch_bytes": (c_size_t, [c_uint, c_size_t]),
    "gfxb_decode_attention": (c_int, [P, P, c_size_t, P, P, c_size_t, P, c_uint, P, P, c_size_t, P, P, c_size_t,
                                      c_uint64, P, c_uint, c_uint, P, P, c_size_t, P]),
    "gfxb_gated_attention": (c_int, [P, P, P, P, P, c_size_t, P, c_size_t, c_uint, c_uint, c_uint, P, c_size_t, P]),
    "gfxb_gated_attention_static_scratch": (c_int, [P, P, P, P, P, c_size_t, P, c_size_t, c_uint, c_uint, c_uint, P]),
    "gfxb_argmax_scratch_bytes": (c_size_t, [c_uint]),
    "gfxb_argmax": (c_int, [P, P, P, c_size_t, c_size_t, c_uint, P, c_size_t, P]),
    "gfxb_read_device_errors": (c_int, [POINTER(c_uint32)]),
    "gfxb_nccl_unique_id": (c_int, [P]),
    "gfxb_tp_shard": (c_int, [POINTER(ModelConfig), c_int, c_int, POINTER(TpShardInfo)]),
    "gfxb_engine_create_synthetic": (c_int, [POINTER(ModelConfig), c_int, c_int, c_int, P, c_int, POINTER(c_void_p)]),
    "gfxb_engine_destroy": (c_int, [P]),
    "gfxb_engine_abort": (c_int, [P]),
    "gfxb_engine_weight_bytes": (c_int, [P, POINTER(c_uint64)]),
    "gfxb_session_create": (c_int, [P, POINTER(SessionConfig), POINTER(c_void_p)]),
    "gfxb_session_destroy": (c_int, [P]),
    "gfxb_session_greedy_step": (c_int, [P, c_uint32, POINTER(c_uint32)]),
    "gfxb_session_block_step": (c_int, [P, POINTER(c_uint32), c_uint, POINTER(c_uint32)]),
    "gfxb_session_mtp_draft": (c_int, [P, c_uint32, POINTER(c_uint32)]),
    "gfxb_session_speculative_step": (c_int, [P, c_uint32, c_uint, POINTER(c_uint32), POINTER(c_uint), POINTER(c_uint)]),
    "gfxb_session_speculative_step_with_drafts": (c_int, [P, c_uint32, POINTER(c_uint32), c_uint, POINTER(c_uint32),
                                                          POINTER(c_uint), POINTER(c_uint)]),
    "gfxb_session_prefill": (c_int, [P, POINTER(c_uint32), c_size_t, POINTER(c_uint32)]),
    "gfxb_session_position": (c_int, [P, POINTER(c_uint64)]),
    "gfxb_session_enqueue_greedy": (c_int, [P, c_uint32, c_uint]),
    "gfxb_session_sync": (c_int, [P]),
    "gfxb_session_last_token": (c_int, [P, POINTER(c_uint32)]),
    "gfxb_session_stream": (c_void_p, [P]),
    "gfxb_session_enqueue_gemv": (c_int, [P, c_int, c_uint, POINTER(c_uint64)]),
    "gfxb_session_enqueue_operation": (c_int, [P, c_int, c_uint, POINTER(c_uint64)]),
    "gfxb_session_time_operation": (c_int, [P, c_int, c_uint, c_int, POINTER(ctypes.c_float), POINTER(c_uint64)]),
    "gfxb_session_read_state": (c_int, [P, P, P, c_size_t]),
    "gfxb_session_trace_step": (c_int, [P, c_uint32, POINTER(c_uint32), P, c_size_t, POINTER(c_uint), POINTER(c_uint),
                                        P]),
    "gfxb_crc64_ecma": (c_int, [c_uint64, P, c_size_t, POINTER(c_uint64)]),
    "gfxb_artifact_open": (c_int, [c_char_p, c_int, POINTER(c_void_p)]),
    "gfxb_artifact_close": (c_int, [P]),
    "gfxb_artifact_identity_of": (c_int, [P, POINTER(ArtifactIdentity)]),
    "gfxb_artifact_file_bytes": (c_int, [P, POINTER(c_uint64)]),
    "gfxb_artifact_tensor_count": (c_int, [P, POINTER(c_size_t)]),
    "gfxb_artifact_tensor_at": (c_int, [P, c_size_t, POINTER(TensorView)]),
    "gfxb_artifact_find": (c_int, [P, c_char_p, POINTER(TensorView), POINTER(c_int)]),
    "gfxb_artifact_write": (c_int, [c_char_p, POINTER(ArtifactIdentity), POINTER(TensorWrite), c_size_t]),
    "gfxb_convert_to_artifact": (c_int, [c_char_p, POINTER(ArtifactIdentity), POINTER(ConvertSource), c_size_t,
                                         POINTER(ConvertOptions), c_int]),
    "gfxb_engine_create_from_artifact": (c_int, [c_char_p, POINTER(ArtifactLoadOptions), c_int, c_int, c_int, P,
                                                 POINTER(c_void_p)]),
    "gfxb_engine_config": (c_int, [P, POINTER(ModelConfig)]),
    "gfxb_engine_export_artifact": (c_int, [P, c_char_p, c_char_p]),
}


def declare(lib: ctypes.CDLL) -> None:
    for name, (restype, argtypes) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = restype
        fn.argtypes = argtypes
