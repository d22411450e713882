// Argument blocks and launchers of the decode-path operators (ops.cu).
// Shared by the C ABI wrappers and the C++ runtime.
#pragma once

#include <cstddef>
#include <cstdint>

#include <cuda_fp16.h>
#include <cuda_runtime.h>

namespace gfxb {

constexpr unsigned kAttentionChunk = 128;

struct NormPackArgs {
  const __half* residual = nullptr;      // [B][H] input (or residual when update != null)
  const float* update = nullptr;         // [B][H] fp32 update added to residual first
  __half* residual_out = nullptr;        // [B][H] fp16(residual + update) (or gathered embedding)
  const std::uint16_t* weight = nullptr; // bf16 [H]
  int unit_offset = 1;
  float epsilon = 1.0e-6f;
  std::uint32_t elements = 0;            // H
  __half* normalized_out = nullptr;      // [B][H] optional
  std::int8_t* act_codes = nullptr;      // activation pack (fragment order)
  __half* act_scales = nullptr;
  std::int32_t* act_sums = nullptr;
  std::uint8_t* packed_a4 = nullptr;     // optional reference packed A4
  // embedding gather as the input (row-major W4/W2 codes + fp16 scales [V][H/128])
  const std::uint8_t* embedding_codes = nullptr;
  const __half* embedding_scales = nullptr;
  std::uint32_t embedding_rows = 0;
  int embedding_bits = 4;
  const std::uint32_t* device_tokens = nullptr;
  std::uint32_t host_token = 0;
};

struct SiluPackArgs {
  const float* gate = nullptr;
  const float* up = nullptr;
  std::uint32_t elements = 0;  // per row
  std::uint32_t batch = 0;
  __half* product_out = nullptr;
  std::int8_t* act_codes = nullptr;
  __half* act_scales = nullptr;
  std::int32_t* act_sums = nullptr;
  std::uint8_t* packed_a4 = nullptr;
};

struct GdnConvArgs {
  const float* projected = nullptr;        // [B][C]
  const std::uint16_t* weight = nullptr;   // bf16 [C][4]
  const __half* initial_state = nullptr;   // [C][4]
  __half* final_state = nullptr;           // [C][4] (may alias initial_state)
  __half* output = nullptr;                // [B][C]
  __half* appended_log = nullptr;          // [B][C] optional
  std::uint32_t channels = 0;
  std::uint32_t batch = 0;
};

struct GdnRecurrentArgs {
  const __half* qkv = nullptr;             // [B][2*Hk*128 + Hv*128] conv output
  const float* z = nullptr;                // [B][Hv*128]
  const float* a = nullptr;                // [B][Hv]
  const float* b = nullptr;                // [B][Hv]
  const std::uint16_t* a_log = nullptr;    // bf16 [Hv]
  const std::uint16_t* dt_bias = nullptr;  // bf16 [Hv]
  const std::uint16_t* norm_weight = nullptr;  // bf16 [128]
  const float* initial_state = nullptr;    // [Hv][128][128]
  float* final_state = nullptr;            // may alias initial_state
  __half* output = nullptr;                // [B][Hv*128]
  float* key_log = nullptr;                // [B][Hk*128]
  float* delta_log = nullptr;              // [B][Hv*128]
  float* decay_log = nullptr;              // [B][Hv]
  std::uint32_t key_heads = 0;
  std::uint32_t value_heads = 0;
  std::uint32_t batch = 0;
  std::uint32_t ab_stride = 0;             // per-token stride of a/b (0: value_heads)
  // optional activation pack of the output (one 128-group per value head)
  int act_bits = 0;
  std::int8_t* act_codes = nullptr;
  __half* act_scales = nullptr;
  std::int32_t* act_sums = nullptr;
  // optional causal conv fused in front (conv.projected != nullptr): the CTAs
  // of one key head's value heads run as a cluster, each convolves the q/k/v
  // channels it reads, and `qkv` is unused; conv.output and conv.channels are
  // ignored (the channel count follows from the head counts)
  GdnConvArgs conv;
};

struct GdnRestoreArgs {
  __half* conv_states = nullptr;           // [L][C][4]
  float* states = nullptr;                 // [L][Hv][128][128]
  const __half* conv_logs = nullptr;       // [L][max_logged][C]
  const float* key_logs = nullptr;         // [L][max_logged][Hk*128]
  const float* delta_logs = nullptr;       // [L][max_logged][Hv*128]
  const float* decay_logs = nullptr;       // [L][max_logged][Hv]
  std::uint32_t channels = 0;
  std::uint32_t key_heads = 0;
  std::uint32_t value_heads = 0;
  std::uint32_t layers = 0;
  std::uint32_t max_logged = 0;
  std::uint32_t accepted = 0;
};

struct QkRopeArgs {
  const float* q_input = nullptr;          // [B][q_heads][q_stride] (q_proj output, first 256 of each head)
  const std::uint16_t* q_weight = nullptr;
  __half* q_output = nullptr;              // [B][q_heads][256]
  const float* k_input = nullptr;          // [B][k_heads][k_stride]
  const std::uint16_t* k_weight = nullptr;
  __half* k_output = nullptr;              // [B][k_heads][256] optional
  const float* v_input = nullptr;          // [B][k_heads][256] for the fused KV append
  __half* key_cache = nullptr;             // [capacity][k_heads][256] optional
  __half* value_cache = nullptr;
  std::size_t capacity = 0;
  std::uint32_t q_heads = 0, k_heads = 0;
  std::uint32_t q_stride = 512, k_stride = 256;
  std::uint32_t rotary = 64;
  const float* cos_table = nullptr;        // [positions][rotary/2]
  const float* sin_table = nullptr;
  std::uint64_t table_positions = 0;
  std::uint64_t base_position = 0;
  const std::uint64_t* device_base_position = nullptr;
};

struct AttentionArgs {
  const __half* query = nullptr;           // [B][q_heads][256]
  const float* gate = nullptr;             // [B][q_heads][512] (q_proj output; gate = second half)
  const __half* key_cache = nullptr;       // [capacity][kv_heads][256]
  const __half* value_cache = nullptr;
  __half* output = nullptr;                // [B][q_heads][256]
  float* partials = nullptr;               // [B][q_heads][max_chunks][258]
  std::uint32_t max_chunks = 0;
  std::size_t capacity = 0;
  std::uint64_t base_token_count = 0;      // visible positions for token 0 (position + 1)
  const std::uint64_t* device_base_position = nullptr;  // if set, base_token_count = *p + 1
  std::uint32_t q_heads = 0, kv_heads = 0;
  // optional activation pack of the output (two 128-groups per query head)
  int act_bits = 0;
  std::int8_t* act_codes = nullptr;
  __half* act_scales = nullptr;
  std::int32_t* act_sums = nullptr;
};

// Single-token decode attention: the Q/K RMSNorm + RoPE with the KV append
// (rope) and the gated attention over the cache (attention) in one launch.
// `tickets` holds one zero-initialised counter per query head; each launch
// leaves it at zero again.
struct AttentionDecodeArgs {
  QkRopeArgs rope;
  AttentionArgs attention;
  std::uint32_t* tickets = nullptr;
};

struct ArgmaxArgs {
  const float* logits = nullptr;
  std::size_t row_stride = 0;
  std::uint32_t vocab = 0;
  const std::uint32_t* token_ids = nullptr;
  std::uint32_t* tokens = nullptr;
  float* partial_values = nullptr;
  std::uint32_t* partial_indices = nullptr;
};

int launch_norm_pack(const NormPackArgs& args, int act_bits, unsigned batch, cudaStream_t stream);
int launch_silu_pack(const SiluPackArgs& args, int act_bits, cudaStream_t stream);
int launch_gdn_conv(const GdnConvArgs& args, cudaStream_t stream);
int launch_gdn_recurrent(const GdnRecurrentArgs& args, cudaStream_t stream);
int launch_gdn_restore(const GdnRestoreArgs& args, cudaStream_t stream);
int launch_qk_rope(const QkRopeArgs& args, unsigned batch, cudaStream_t stream);
std::size_t attention_partial_bytes(unsigned q_heads, std::size_t capacity, unsigned batch);
int launch_attention(const AttentionArgs& args, unsigned batch, cudaStream_t stream);
int launch_attention_decode(const AttentionDecodeArgs& args, cudaStream_t stream);
bool attention_decode_enabled();
std::size_t argmax_scratch_bytes(unsigned batch);
int launch_argmax(const ArgmaxArgs& args, unsigned batch, cudaStream_t stream);
int launch_float_to_half(const float* input, __half* output, std::size_t n, cudaStream_t stream);
int read_ops_error(std::uint32_t* value, bool clear);

}  // namespace gfxb
