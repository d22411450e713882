/*
 * CPU oracle for the gfxinfer-b200 decode path. TEST INFRASTRUCTURE ONLY.
 *
 * This library restates, in plain C, the arithmetic of the reference engine's
 * decode token loop (H-Sami/gfxinfer: src/quantization.cpp,
 * src/kernels/lowbit_gemv.hip, src/kernels/qwen_ops.hip,
 * src/qwen_runtime.cpp). It is linked only by tests/, by
 * __graft_entry__.smoke() and by bench.py's CPU-baseline leg, always as the
 * checker or the timed CPU baseline, never as part of the product path.
 *
 * Every floating-point reduction below follows one fixed order (documented at
 * each function) and the CUDA kernels follow the same order, so outputs are
 * compared bit-for-bit. exp/log1p are the engine's own published-method
 * implementations (Cody-Waite reduction + Taylor polynomial; atanh series),
 * restated here independently.
 *
 * Parity pins: the quantizer/tiler restatement is checked bit-exactly against
 * the reference's own src/quantization.cpp compiled into oracle/_ref, and
 * against golden fixtures in tests/golden generated from it.
 */
#ifndef GFXB_ORACLE_H
#define GFXB_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Quantization ids follow the reference enum (include/gfxinfer/artifact.h:22-29). */
enum { OR_W2 = 1, OR_W3 = 2, OR_W4 = 3 };

/* ---- scalar helpers ------------------------------------------------------ */
uint16_t or_f32_to_f16(float value);
float or_f16_to_f32(uint16_t bits);
uint16_t or_f32_to_bf16(float value);
float or_bf16_to_f32(uint16_t bits);
float or_expf(float x);
float or_log1pf(float x);
uint64_t or_hash(uint64_t seed, uint64_t stream, uint64_t index);

/* ---- packing (src/quantization.cpp) -------------------------------------- */
size_t or_packed_row_bytes(int format, size_t columns);
int or_quantize_group128(const float* weights, size_t rows, size_t columns, int format,
                         uint8_t* codes, float* scales);
uint8_t or_load_code(const uint8_t* row, size_t column, int format);
int or_decode_value(uint8_t code, int format);
float or_dequantized_weight(const uint8_t* codes, const float* scales, size_t rows,
                            size_t columns, int format, size_t row, size_t column);
int or_tile_gfx12(const uint8_t* codes, const float* scales, size_t rows, size_t columns,
                  int format, uint8_t* tiled_codes, float* tiled_scales);
void or_unpack_logical(const uint8_t* codes, size_t rows, size_t columns, int format,
                       int8_t* logical);

/* ---- activation quantizers (lowbit_gemv.hip:373-436) --------------------- */
void or_quantize_activation_i4(const uint16_t* input, size_t columns, unsigned batch,
                               uint8_t* packed, uint16_t* scales);
void or_quantize_activation_i8(const uint16_t* input, size_t columns, unsigned batch,
                               int8_t* quantized, uint16_t* scales);
void or_unpack_a4(const uint8_t* packed, size_t count, int8_t* values);

/* ---- GEMV (lowbit_gemv.hip:461-553, 682-755) ------------------------------ */
void or_gemv_int(const int8_t* weights, const uint16_t* weight_scales, size_t rows,
                 size_t columns, const int8_t* activations, const uint16_t* activation_scales,
                 unsigned batch, float* output);
void or_gemv_f16(const int8_t* weights, const uint16_t* weight_scales, size_t rows,
                 size_t columns, const uint16_t* activations, unsigned batch, double* output);

/* ---- qwen ops (qwen_ops.hip) ---------------------------------------------- */
float or_tree32(const float* values);
void or_rms_norm(const uint16_t* input, const uint16_t* weight, size_t elements, float eps,
                 int unit_offset, uint16_t* output);
void or_residual_add_rms_norm(const uint16_t* residual, const float* update,
                              const uint16_t* weight, size_t elements, float eps,
                              int unit_offset, uint16_t* residual_out, uint16_t* normalized);
void or_silu_multiply_f16(const float* gate, const float* up, size_t elements,
                          uint16_t* output);
void or_gdn_conv_update(const float* projected, const uint16_t* weight, uint16_t* state,
                        uint16_t* output, uint16_t* appended_log, size_t channels,
                        unsigned batch);
void or_gdn_recurrent(const uint16_t* qkv, const float* z, const float* a, const float* b,
                      const uint16_t* a_log, const uint16_t* dt_bias,
                      const uint16_t* norm_weight, float* state, uint16_t* output,
                      float* key_log, float* delta_log, float* decay_log, unsigned key_heads,
                      unsigned value_heads, unsigned batch);
void or_gdn_restore(uint16_t* conv_state, float* state, const uint16_t* conv_log,
                    const float* key_log, const float* delta_log, const float* decay_log,
                    size_t channels, unsigned key_heads, unsigned value_heads,
                    unsigned accepted);
void or_rope_table(size_t positions, unsigned rotary, float theta, float* cos_table,
                   float* sin_table);
void or_qk_norm_rope(const float* input, size_t stride, const uint16_t* weight,
                     unsigned heads, size_t position, const float* cos_table,
                     const float* sin_table, unsigned rotary, uint16_t* output);
void or_gated_attention(const uint16_t* query, const float* gate_projection,
                        const uint16_t* key_cache, const uint16_t* value_cache,
                        size_t token_count, unsigned q_heads, unsigned kv_heads,
                        uint16_t* output);
uint32_t or_argmax(const float* logits, size_t count);

/* ---- synthetic model and scalar forward ----------------------------------- */
typedef struct {
  uint32_t hidden, intermediate, layers, attention_interval;
  uint32_t gdn_key_heads, gdn_value_heads, q_heads, kv_heads;
  uint32_t vocab, draft_vocab;
  uint32_t mlp_bits, proj_bits, head_bits, emb_bits;
  uint32_t activation_bits; /* 4 (A4) or 8 (A8) */
  uint32_t max_context;
  uint64_t seed;
} or_model_config;

typedef struct or_model or_model;
or_model* or_model_create(const or_model_config* config, int include_mtp);
/* Every layer runs, but only the first resident_layers hold their own weights
 * (layer i reuses layer i % resident_layers): the full model's per-token
 * work in the host memory of a few layers, for CPU-baseline timing. */
or_model* or_model_create_cycled(const or_model_config* config, unsigned resident_layers);
void or_model_destroy(or_model* model);
int or_model_greedy_step(or_model* model, uint32_t token, uint32_t* next_token);
/* block_step: count <= 64 tokens, layer-major, one argmax per token. */
int or_model_block_step(or_model* model, const uint32_t* tokens, unsigned count,
                        uint32_t* outputs);
/* Any number of prompt tokens without the LM head. */
int or_model_prefill(or_model* model, const uint32_t* tokens, size_t count);
int or_model_mtp_draft(or_model* model, uint32_t token, int use_mtp_hidden,
                       uint32_t* draft);
size_t or_model_position(const or_model* model);
void or_model_timing(const or_model* model, double* layer_seconds, double* head_seconds, size_t* tokens);
int or_set_threads(int threads);
const uint16_t* or_model_last_hidden(const or_model* model);
const float* or_model_logits(const or_model* model);
uint32_t or_prompt_token(uint64_t seed, uint32_t vocab, uint32_t index);

/* Synthetic weight generators (the engine's generator follows the same rules). */
void or_gen_codes_rowmajor(uint64_t seed, uint32_t tensor, size_t rows, size_t columns,
                           int format, uint8_t* codes);
void or_gen_scales(uint64_t seed, uint32_t tensor, size_t count, int format,
                   uint16_t* scales);
void or_gen_bf16(uint64_t seed, uint32_t tensor, size_t count, float lo, float hi,
                 uint16_t* values);

#ifdef __cplusplus
}
#endif
#endif
