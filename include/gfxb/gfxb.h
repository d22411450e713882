/*
 * gfxinfer-b200 C ABI.
 *
 * A thin, allocation-free launch layer over hand-written sm_100a kernels. It
 * replaces the reference engine's HIP launchers (include/gfxinfer/lowbit_gemv.h,
 * include/gfxinfer/qwen_ops.h) and device layer (src/device.cpp). Conventions:
 *
 *  - Every entry point returns a gfxb_status whose values mirror the
 *    reference's ErrorCode (include/gfxinfer/status.h:11-20); the message of
 *    the last failure on the calling thread is gfxb_last_error_message().
 *  - Pointers are device pointers owned by the caller unless stated otherwise;
 *    fp16 buffers are IEEE binary16 bit patterns (uint16_t), bf16 likewise.
 *  - `stream` is a cudaStream_t passed as void*. Launchers never synchronise.
 *  - Validation happens on the host before any launch and reports
 *    GFXB_INVALID_ARGUMENT / GFXB_UNSUPPORTED, as the reference launchers do.
 */
#ifndef GFXB_GFXB_H
#define GFXB_GFXB_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Mirrors gfxinfer::ErrorCode (status.h:11-20); hip_error becomes cuda_error. */
typedef enum {
  GFXB_OK = 0,
  GFXB_INVALID_ARGUMENT = 1,
  GFXB_IO_ERROR = 2,
  GFXB_CORRUPT_ARTIFACT = 3,
  GFXB_UNSUPPORTED = 4,
  GFXB_CUDA_ERROR = 5,
  GFXB_OUT_OF_MEMORY = 6,
  GFXB_INTERNAL = 7
} gfxb_status;

/* Weight formats: the reference Quantization values (artifact.h:22-29). */
enum { GFXB_W2 = 1, GFXB_W3 = 2, GFXB_W4 = 3 };

const char* gfxb_last_error_message(void);
int gfxb_abi_version(void);

/* ---- device layer (replaces src/device.cpp:37-90) ------------------------- */
typedef struct {
  int index;
  int compute_major;
  int compute_minor;
  int multiprocessors;
  uint64_t global_memory_bytes;
  char name[128];
} gfxb_device_info;

/* Fails with GFXB_UNSUPPORTED unless the device is sm_100 (B200). Replaces
 * require_gfx1200_device (device.cpp:65-90). */
int gfxb_require_sm100_device(int device_index, gfxb_device_info* info);

/* ---- weight layout ---------------------------------------------------------
 * B200 tiled layout ("b200"): codes [N/16][K/128][block], one block per
 * 16-row x 128-column tile-group, BITS*256 bytes, lane-major so each of a
 * warp's 32 lanes reads its tensor-core fragment with one or two 16-byte
 * loads. Scales [N/16][K/128][16] fp16, the gfx12 tiled scale order
 * (quantization.cpp:311-314). Same byte count as the reference layouts. */

/* Reference row-major packed codes (quantization.cpp:94-124) -> b200 codes. */
int gfxb_repack_rowmajor_to_b200(int format, const uint8_t* rowmajor_codes, uint8_t* b200_codes,
                                 size_t rows, size_t columns, void* stream);
/* Reference gfx12 tiled codes (quantization.cpp:253-318) -> b200 codes. */
int gfxb_repack_gfx12_to_b200(int format, const uint8_t* gfx12_codes, uint8_t* b200_codes,
                              size_t rows, size_t columns, void* stream);
/* Row-major fp16 scales [N][K/128] -> tiled [N/16][K/128][16]. */
int gfxb_tile_scales(const uint16_t* rowmajor_scales, uint16_t* tiled_scales, size_t rows,
                     size_t columns, void* stream);

/* ---- weight packing (the reference's src/quantization.cpp on the device) ----
 * Row-major packed codes ("PackedMatrix", quantization.h): W2 four codes per
 * byte, W3 three 16-byte bit planes per 128-group, W4 two nibbles per byte;
 * fp32 group scales [N][K/128]. Bit-identical to the reference's host code. */

/* packed_row_bytes (quantization.cpp:154-161); 0 for an unknown format. Host. */
size_t gfxb_packed_row_bytes(int format, size_t columns);
/* quantize_group128 (quantization.cpp:163-220): fp32 or bf16 weights
 * (input_dtype GFXB_DTYPE_F32 / GFXB_DTYPE_BF16 of artifact.h) [N][K] ->
 * row-major codes (16-byte aligned) and fp32 scales, per 128-group the
 * reference's choose_scale (amax / {3,4,8}, four least-squares refits with
 * double sums in column order). Waits for the stream and returns
 * GFXB_INVALID_ARGUMENT when a weight is not finite, as the reference does;
 * allocates a 4-byte flag with cudaMallocAsync on the stream. */
int gfxb_quantize_group128(int format, int input_dtype, const void* weights, size_t rows, size_t columns,
                           uint8_t* codes, float* scales, void* stream);
/* tile_group128_for_gfx12 (quantization.cpp:253-318): row-major codes and fp32
 * scales -> the reference's gfx12 tiled codes (W3 as sequential 3-bit codes)
 * and scales [N/16][K/128][16]. N % 16 == 0. */
int gfxb_tile_group128_for_gfx12(int format, const uint8_t* codes, const float* scales, size_t rows, size_t columns,
                                 uint8_t* tiled_codes, float* tiled_scales, void* stream);
/* dequantize_group128 (quantization.cpp:237-251): fp32 [N][K] = level * scale. */
int gfxb_dequantize_group128(int format, const uint8_t* codes, const float* scales, size_t rows, size_t columns,
                             float* output, void* stream);
/* dequantized_weight (quantization.cpp:222-235) over HOST buffers: NaN for an
 * index outside the matrix or an invalid shape. */
float gfxb_dequantized_weight(int format, const uint8_t* codes, const float* scales, size_t rows, size_t columns,
                              size_t row, size_t column);

/* Conversion of one weight for the engines (the converter's write_quantized,
 * converter.cpp:345-393): fp32 or bf16 [N][K] -> quantize_group128 -> codes in
 * `layout` and fp16 scales rounded to nearest even (__float2half):
 *   GFXB_LAYOUT_B200:     b200 codes, scales [N/16][K/128][16] (recipe b200-v1)
 *   GFXB_LAYOUT_GFX12:    gfx12 tiled codes, W3 sequential, scales [N/16][K/128][16]
 *                         (the reference's tiled recipes)
 *   GFXB_LAYOUT_ROWMAJOR: row-major codes, scales [N][K/128] (embeddings)
 * scratch: gfxb_convert_scratch_bytes() bytes, 16-byte aligned. Waits for the
 * stream (non-finite weights give GFXB_INVALID_ARGUMENT). */
enum { GFXB_LAYOUT_B200 = 0, GFXB_LAYOUT_GFX12 = 1, GFXB_LAYOUT_ROWMAJOR = 2 };
size_t gfxb_convert_scratch_bytes(int format, size_t rows, size_t columns);
int gfxb_convert_group128(int format, int input_dtype, const void* weights, size_t rows, size_t columns, int layout,
                          uint8_t* codes, uint16_t* scales, void* scratch, size_t scratch_bytes, void* stream);

/* ---- activation packs --------------------------------------------------------
 * The B200 GEMVs read activations as a pack: int8 codes in mma-fragment order
 * [B][K] (within each 128-group the 32 bytes a lane feeds to the tensor core
 * are contiguous), fp16 group scales [B][K/128] and int32 group code sums
 * [B][K/128]. Quantization is the reference's A4/A8 rule
 * (lowbit_gemv.hip:373-436): scale = fp16(amax/7 or amax/127), code =
 * clamp(rint(x/scale)). `packed_a4` (optional, A4 only) additionally receives
 * the reference's packed-nibble layout [B][K/2]. */
int gfxb_pack_activation(int activation_bits, const uint16_t* input, int8_t* codes,
                         uint16_t* scales, int32_t* sums, uint8_t* packed_a4, size_t columns,
                         unsigned batch, void* stream);

/* ---- GEMV -------------------------------------------------------------------
 * y[b][n] = sum over groups g (ascending) of fp32 fma( int32 dot_g,
 * ws[n][g] * as[b][g] ) (lowbit_gemv.hip:490-537): bit-identical to the
 * reference arithmetic. Output batch-major [B][N], fp32 or fp16. */
typedef struct {
  const uint8_t* codes;    /* b200 layout */
  const uint16_t* scales;  /* tiled fp16 */
  void* output;            /* [B][rows], fp32 or fp16 */
  size_t rows;             /* multiple of 16 */
  int output_f16;          /* 0: fp32, 1: fp16 (launch_gfx12_i4_gemm_half) */
} gfxb_gemv_matrix;

/* One launch for 1..4 matrices that share K, format and input (replaces
 * launch_gfx12_i4_gemm / _half / _fused and launch_gfx12_i8_gemm when the
 * weights are in the b200 layout). batch in [1, 32]. */
int gfxb_lowbit_gemv(int format, const gfxb_gemv_matrix* matrices, unsigned matrix_count,
                     const int8_t* act_codes, const uint16_t* act_scales,
                     const int32_t* act_sums, size_t columns, unsigned batch, void* stream);

/* FP16-activation GEMV over the b200 layout: y[b][n] = sum_k fp16(q * ws) *
 * x[b][k], fp32 accumulation on the f16 tensor cores (the reference's
 * gfx12_f16_gemm arithmetic, lowbit_gemv.hip:757-834; its summation order is
 * the tensor cores', so results match an exact sum within ~1e-5 relative).
 * activations [B][K] fp16 (8-byte aligned), 1..4 matrices sharing K and
 * format, batch in [1, 32]. W2, W3 and W4. */
int gfxb_lowbit_gemv_f16(int format, const gfxb_gemv_matrix* matrices, unsigned matrix_count,
                         const uint16_t* activations, size_t columns, unsigned batch, void* stream);

/* ---- reference-layout drop-ins (lowbit_gemv.h:79-170) ------------------------ */
int gfxb_quantize_activation_i4(const uint16_t* input, uint8_t* packed_output, uint16_t* scales,
                                size_t columns, unsigned batch, void* stream);
int gfxb_quantize_activation_i8(const uint16_t* input, int8_t* quantized_output,
                                uint16_t* scales, size_t columns, unsigned batch, void* stream);
/* Replaces launch_gfx12_i4_gemm (lowbit_gemv.h:100-111): gfx12 tiled weights
 * (W3 in the sequential 3-bit fragment order), packed A4 activations. */
int gfxb_gfx12_i4_gemm(int format, const uint8_t* tiled_weights,
                       const uint16_t* tiled_weight_scales, const uint8_t* packed_activations,
                       const uint16_t* activation_scales, float* output, size_t rows,
                       size_t columns, unsigned batch, int sequential_w3, void* stream);
/* Replaces launch_gfx12_i8_gemm (lowbit_gemv.h:147-157); also accepts W3. */
int gfxb_gfx12_i8_gemm(int format, const uint8_t* tiled_weights,
                       const uint16_t* tiled_weight_scales, const int8_t* quantized_activations,
                       const uint16_t* activation_scales, float* output, size_t rows,
                       size_t columns, unsigned batch, void* stream);

/* Replaces launch_gfx12_f16_gemm (lowbit_gemv.h:161-170): gfx12 tiled weights
 * (quantization.cpp:253-318; W3 in the sequential 3-bit fragment order, which
 * the reference does not support here), fp16 activations [B][K], fp32 output
 * [B][N]. Same argument checks and error codes as the reference launcher. */
int gfxb_gfx12_f16_gemm(int format, const uint8_t* tiled_weights, const uint16_t* tiled_weight_scales,
                        const uint16_t* activations, float* output, size_t rows, size_t columns,
                        unsigned batch, void* stream);

/* ---- decode-path operators (qwen_ops.h) -------------------------------------
 * Fused forms of the reference launchers; each optional output may be NULL. */

/* residual add + RMSNorm (+ activation pack). Replaces launch_rms_norm(_batch),
 * launch_residual_add_rms_norm_batch and the A4/A8 quantizer that follows
 * them (qwen_ops.h, lowbit_gemv.h:79-95). update == NULL: plain RMSNorm of
 * `input`. act_bits 0 (no pack), 4 or 8. */
int gfxb_residual_rms_norm_pack(const uint16_t* input, const float* update, uint16_t* residual_out,
                                const uint16_t* bf16_weight, uint16_t* normalized_out, size_t elements,
                                unsigned batch, float epsilon, int add_unit_offset, int act_bits,
                                int8_t* act_codes, uint16_t* act_scales, int32_t* act_sums,
                                uint8_t* packed_a4, void* stream);
/* fp16(silu(gate) * up) (+ pack). Replaces launch_silu_multiply and
 * launch_silu_multiply_quantize_i4. */
int gfxb_silu_multiply_pack(const float* gate, const float* up, size_t elements_per_row, unsigned batch,
                            uint16_t* product_out, int act_bits, int8_t* act_codes, uint16_t* act_scales,
                            int32_t* act_sums, uint8_t* packed_a4, void* stream);
/* Replaces launch_gdn_conv_update(_block) (qwen_ops.h). */
int gfxb_gdn_conv_update(const float* projected, const uint16_t* bf16_weight, const uint16_t* initial_state,
                         uint16_t* final_state, uint16_t* output, uint16_t* appended_log, size_t channels,
                         unsigned batch, void* stream);
/* Replaces launch_gdn_recurrent_decode(_block). States [Hv][128][128] fp32. */
int gfxb_gdn_recurrent(const uint16_t* qkv, const float* z, const float* a, const float* b,
                       const uint16_t* a_log, const uint16_t* dt_bias, const uint16_t* norm_weight,
                       const float* initial_state, float* final_state, uint16_t* output, float* key_log,
                       float* delta_log, float* decay_log, unsigned key_heads, unsigned value_heads,
                       unsigned batch, void* stream);
/* Replaces launch_gdn_restore_prefix_all. */
int gfxb_gdn_restore_prefix_all(uint16_t* conv_states, float* recurrent_states, const uint16_t* conv_logs,
                                const float* key_logs, const float* delta_logs, const float* decay_logs,
                                size_t channels, unsigned key_heads, unsigned value_heads, unsigned layers,
                                unsigned maximum_logged_tokens, unsigned accepted_tokens, void* stream);
/* Host helper: RoPE cos/sin table [positions][rotary/2] (theta^(-2f/rotary)). */
int gfxb_rope_table(size_t positions, unsigned rotary, float theta, float* cos_table, float* sin_table);
/* Replaces launch_qk_rms_norm_rope_block(_indirect_position) and, when
 * key_cache != NULL, launch_kv_append_block(_indirect_position). */
int gfxb_qk_rms_norm_rope(const float* q_input, const uint16_t* q_weight, uint16_t* q_output,
                          unsigned q_heads, size_t q_stride, const float* k_input, const uint16_t* k_weight,
                          uint16_t* k_output, unsigned k_heads, size_t k_stride, unsigned rotary,
                          const float* cos_table, const float* sin_table, size_t table_positions,
                          uint64_t base_position, const uint64_t* device_base_position, unsigned batch,
                          const float* v_input, uint16_t* key_cache, uint16_t* value_cache, size_t capacity,
                          void* stream);
/* Scratch (bytes) needed by gfxb_gated_attention for `batch` tokens. */
size_t gfxb_gated_attention_scratch_bytes(unsigned q_heads, size_t capacity, unsigned batch);
/* Replaces launch_gated_attention_decode(_block)(_indirect_position). */
int gfxb_gated_attention(const uint16_t* query, const float* gate_projection, const uint16_t* key_cache,
                         const uint16_t* value_cache, uint16_t* output, size_t base_token_count,
                         const uint64_t* device_base_position, size_t capacity, unsigned q_heads,
                         unsigned kv_heads, unsigned batch, void* scratch, size_t scratch_bytes, void* stream);
/* Allocation-free variant of gfxb_gated_attention, with no counterpart in the
 * reference. For callers that cannot allocate device memory (a host framework
 * that owns the memory budget, loops that cannot afford an allocation's
 * implicit synchronisation, fixed memory maps): the chunk partials live in a
 * 4 MiB array compiled into the library, held by every GPU that loads it
 * until exit. Limit: batch x q_heads x ceil(capacity / 128) x 258 x 4 bytes
 * <= 4 MiB, else GFXB_INVALID_ARGUMENT. The first call on a device looks up
 * the array's device address (cudaGetSymbolAddress, device current); make
 * that first call before any stream capture. All calls share the array:
 * calls that overlap on the GPU (other streams, other threads) race. Nothing
 * needs clearing between calls; each call writes every partial it reads. */
int gfxb_gated_attention_static_scratch(const uint16_t* query, const float* gate_projection,
                                        const uint16_t* key_cache, const uint16_t* value_cache, uint16_t* output,
                                        size_t base_token_count, const uint64_t* device_base_position,
                                        size_t capacity, unsigned q_heads, unsigned kv_heads, unsigned batch,
                                        void* stream);
/* Scratch (bytes) needed by gfxb_decode_attention: the chunk partials and one
 * merge counter per query head. */
size_t gfxb_decode_attention_scratch_bytes(unsigned q_heads, size_t capacity);
/* Single-token decode attention in one launch: the Q/K RMSNorm(1+w) + NeoX
 * RoPE of gfxb_qk_rms_norm_rope (batch 1, with the KV append) followed by
 * gfxb_gated_attention over positions 0..position. Replaces the reference's
 * launch_qk_norm_rope + launch_gated_attention_decode pair of one decode
 * step (qwen_ops.hip:599-766); outputs and cache rows are bit-identical to
 * that pair's. The position is `position`, or *device_position when that is
 * non-null. Zero-fill the scratch once before the first call: every call
 * leaves its counters at zero again. */
int gfxb_decode_attention(const float* q_input, const uint16_t* q_weight, size_t q_stride, const float* k_input,
                          const uint16_t* k_weight, size_t k_stride, const float* v_input, unsigned rotary,
                          const float* cos_table, const float* sin_table, size_t table_positions,
                          uint16_t* key_cache, uint16_t* value_cache, size_t capacity, uint64_t position,
                          const uint64_t* device_position, unsigned q_heads, unsigned kv_heads,
                          uint16_t* output, void* scratch, size_t scratch_bytes, void* stream);
size_t gfxb_argmax_scratch_bytes(unsigned batch);
/* Replaces launch_argmax(_batch)(_mapped). */
int gfxb_argmax(const float* logits, const uint32_t* token_ids, uint32_t* tokens, size_t vocabulary_size,
                size_t row_stride, unsigned batch, void* scratch, size_t scratch_bytes, void* stream);
/* Reads (and clears) the device-side error flags set by bounded waits and
 * range checks (1: wait timeout, 2: RoPE position beyond table, 4: KV append
 * beyond capacity, 8: attention beyond capacity). Synchronous. */
int gfxb_read_device_errors(uint32_t* flags);

/* ---- engine and decode session (engine.h, qwen_runtime.h) ------------------- */

/* Model shape and synthetic-weight recipe. Field order is shared with the CPU
 * oracle's or_model_config. */
typedef struct {
  uint32_t hidden, intermediate, layers, attention_interval;
  uint32_t gdn_key_heads, gdn_value_heads, q_heads, kv_heads;
  uint32_t vocab, draft_vocab;
  uint32_t mlp_bits, proj_bits, head_bits, emb_bits;
  uint32_t activation_bits; /* 4 (A4) or 8 (A8) */
  uint32_t max_context;
  uint64_t seed;
} gfxb_model_config;

typedef struct gfxb_engine gfxb_engine;
typedef struct gfxb_session gfxb_session;

/* NCCL unique id for tensor parallelism (128 bytes), created on rank 0 and
 * shared with the other ranks by the caller. */
int gfxb_nccl_unique_id(void* id128);

/* This rank's slice of every sharded dimension (heads, rows, columns): first
 * index and count. Column-parallel: GDN key/value heads (qkv, z), attention
 * query heads (q) and the KV heads they read, MLP rows, LM-head vocabulary
 * rows. Row-parallel: GDN out, attention o, MLP down (K = the slices above),
 * MTP fc (K slice of the 2*hidden input). Host-only; validates the config. */
typedef struct {
  uint32_t gdn_key_heads, gdn_key_head0, gdn_value_heads, gdn_value_head0;
  uint32_t q_heads, q_head0, kv_heads, kv_head0;
  uint32_t intermediate, intermediate0, vocab, vocab0, fc_columns, fc_column0;
  uint32_t gdn_channels;
} gfxb_tp_shard_info;
int gfxb_tp_shard(const gfxb_model_config* config, int tp_rank, int tp_size, gfxb_tp_shard_info* shard);

/* Engine::create for a seeded random-init model (replaces engine.cpp:62-216 for
 * synthetic weights). tp_size 1 needs no NCCL id. Weights are generated on the
 * device, shard by shard, into one arena. */
int gfxb_engine_create_synthetic(const gfxb_model_config* config, int device, int tp_rank, int tp_size,
                                 const void* nccl_id128, int include_mtp, gfxb_engine** engine);
int gfxb_engine_destroy(gfxb_engine* engine);
/* Aborts the engine's NCCL communicator (callable from another thread while a
 * step is blocked on a peer that failed): pending collectives end with an
 * error instead of waiting for the lost rank. The engine can only be
 * destroyed afterwards. */
int gfxb_engine_abort(gfxb_engine* engine);
int gfxb_engine_weight_bytes(const gfxb_engine* engine, uint64_t* bytes);

typedef struct {
  uint32_t maximum_context_tokens;
  uint32_t graph_verifier_batch; /* 0: no speculative graph; else drafts + 1 */
  uint32_t use_graphs;           /* capture the greedy step in a CUDA graph */
  uint32_t step_kernel;          /* GFXB_STEP_*: how a batch-1 greedy step runs */
} gfxb_session_config;

/* Batch-1 greedy step execution. LAUNCHES runs the per-operation kernels
 * (captured in a CUDA graph when use_graphs is set). PERSISTENT runs the
 * persistent token kernel (one launch per token: every layer, the LM head and
 * the argmax, with the weight stream running ahead across layers) and fails
 * session creation with GFXB_UNSUPPORTED where it cannot run (tensor
 * parallelism, hidden size not 256 x {4, 8, 16, 20}). AUTO picks the faster
 * path measured on B200, currently the per-operation launches. Both paths
 * produce identical bits. */
enum { GFXB_STEP_AUTO = 0, GFXB_STEP_LAUNCHES = 1, GFXB_STEP_PERSISTENT = 2 };

int gfxb_session_create(gfxb_engine* engine, const gfxb_session_config* config, gfxb_session** session);
int gfxb_session_destroy(gfxb_session* session);
/* QwenDecodeSession::greedy_step (qwen_runtime.cpp:1264-1318). */
int gfxb_session_greedy_step(gfxb_session* session, uint32_t input_token, uint32_t* output_token);
/* QwenDecodeSession::block_step (qwen_runtime.cpp:1320-1392), 1..32 tokens. */
int gfxb_session_block_step(gfxb_session* session, const uint32_t* input_tokens, unsigned count,
                            uint32_t* output_tokens);
/* QwenDecodeSession::mtp_draft (qwen_runtime.cpp:1394-1419). */
int gfxb_session_mtp_draft(gfxb_session* session, uint32_t next_token, uint32_t* draft_token);
/* QwenDecodeSession::speculative_step (qwen_runtime.cpp:1421-1544): tokens
 * receives accepted drafts + the correction (at most draft_count + 1). When
 * the session was created with graph_verifier_batch == draft_count + 1, the
 * round's device work (MTP draft chain, verifier block with rollback logs,
 * token downloads) replays one CUDA graph captured at session creation
 * (prepare_speculative_graphs, :642-713); other draft counts run the same
 * work eagerly. Acceptance, rollback replay and the MTP cache advance follow
 * on the host as in the reference. */
int gfxb_session_speculative_step(gfxb_session* session, uint32_t seed_token, unsigned draft_count,
                                  uint32_t* tokens, unsigned* token_count, unsigned* accepted_drafts);
/* speculative_step verifying the caller's drafts instead of the MTP chain's
 * proposals (no counterpart in the reference, whose drafts always come from
 * its MTP layer): for callers with a drafter of their own (prompt lookup,
 * n-gram tables, a separate draft model) and for tests that need rounds
 * with full or partial acceptance. The MTP chain still runs, so the MTP
 * cache stays aligned with the target as after a regular round. The round
 * runs eagerly (never from the captured speculative graph). drafts: 1..31
 * token ids. Acceptance, rollback and commit are those of
 * gfxb_session_speculative_step. */
int gfxb_session_speculative_step_with_drafts(gfxb_session* session, uint32_t seed_token, const uint32_t* drafts,
                                              unsigned draft_count, uint32_t* tokens, unsigned* token_count,
                                              unsigned* accepted_drafts);
/* Chunked prefill, replacing the reference CLI's token-by-token prompt loop
 * (src/cli/main.cpp:1056-1070): the prompt runs as causal blocks of up to 32
 * tokens (the block_step forward, qwen_runtime.cpp:1320-1392) and the LM head
 * runs only for its last token, whose argmax is written to next_token. The
 * session state afterwards equals that after greedy_step over every prompt
 * token. */
int gfxb_session_prefill(gfxb_session* session, const uint32_t* tokens, size_t count, uint32_t* next_token);
int gfxb_session_position(const gfxb_session* session, uint64_t* position);
/* Device-resident decode: enqueue `steps` greedy steps on the session stream,
 * each step's argmax feeding the next, no host synchronisation. The host
 * position is advanced; call gfxb_session_sync before reading results. */
int gfxb_session_enqueue_greedy(gfxb_session* session, uint32_t first_token, unsigned steps);
int gfxb_session_sync(gfxb_session* session);
int gfxb_session_last_token(gfxb_session* session, uint32_t* token);
void* gfxb_session_stream(gfxb_session* session);
/* Enqueues `launches` GEMV launches of one projection kind (0: MLP gate+up
 * fused, 1: MLP down, 2: GDN qkv/z/a/b fused), cycling over the layers so
 * each launch reads its weights from HBM; `bytes` receives the algorithmic
 * bytes of one launch (codes, fp16 scales, A4 activation, fp32 outputs).
 * Used to time the dominant kernel in isolation. */
int gfxb_session_enqueue_gemv(gfxb_session* session, int kind, unsigned launches, uint64_t* bytes);
/* Enqueues `launches` launches of one decode operation at batch 1, cycling
 * over the layers that carry it (each launch reads its own weights or states
 * from HBM), for timing kernels in isolation; `bytes` receives the
 * algorithmic bytes one launch moves (weights, scales, states, activations,
 * outputs). The operations write the session's buffers, and GDN_STEP and
 * ATTENTION also its recurrent states and KV caches (ATTENTION at the
 * session's position): time them on a session made for timing. */
enum {
  GFXB_OP_MLP_GATE_UP = 0, GFXB_OP_MLP_DOWN = 1, GFXB_OP_GDN_IN = 2, GFXB_OP_GDN_OUT = 3, GFXB_OP_ATTN_QKV = 4,
  GFXB_OP_ATTN_O = 5, GFXB_OP_LM_HEAD = 6, GFXB_OP_GDN_STEP = 7, GFXB_OP_ATTENTION = 8, GFXB_OP_NORM_PACK = 9,
  GFXB_OP_SILU_PACK = 10
};
int gfxb_session_enqueue_operation(gfxb_session* session, int kind, unsigned launches, uint64_t* bytes);
/* Times gfxb_session_enqueue_operation: `launches` launches (after 8 warm-up
 * launches) captured in a CUDA graph and replayed (use_graph != 0) or
 * enqueued directly, between CUDA events on the session stream; writes the
 * mean microseconds per launch. Synchronous. */
int gfxb_session_time_operation(gfxb_session* session, int kind, unsigned launches, int use_graph,
                                float* microseconds, uint64_t* bytes);
/* One greedy step on the persistent token kernel with its timeline recorded
 * (GFXB_UNSUPPORTED when the session runs per-operation launches). timeline
 * receives [op_count + 1][2][ctas] globaltimer nanoseconds: entry (i, 0, c)
 * is when CTA c finished operation i - 1 and reached the grid barrier before
 * operation i, (i, 1, c) when that barrier released it; i = 0 is the kernel
 * start and i = op_count its end. op_kinds (optional, op_count entries): 1
 * GEMV (| activation source << 4 | weight bits << 8), 2 GDN, 3 attention,
 * 4 argmax. For profiling; the step's result is that of greedy_step. */
int gfxb_session_trace_step(gfxb_session* session, uint32_t input_token, uint32_t* output_token,
                            uint64_t* timeline, size_t timeline_entries, unsigned* op_count, unsigned* ctas,
                            uint32_t* op_kinds);
/* Copies the last token's final hidden state (fp16 [hidden]) and logits of the
 * local vocabulary shard (fp32) to host memory, for parity checks. */
int gfxb_session_read_state(gfxb_session* session, uint16_t* hidden, float* logits, size_t logits_count);

#ifdef __cplusplus
}
#endif
#endif
