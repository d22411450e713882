// C ABI wrappers of the decode-path operators (include/gfxb/gfxb.h), the
// counterparts of the reference's qwen_ops.h launchers.
#include <mutex>

#include "common.cuh"
#include "ops.cuh"

using namespace gfxb;

namespace {
__half* as_half(std::uint16_t* p) { return reinterpret_cast<__half*>(p); }
const __half* as_half(const std::uint16_t* p) { return reinterpret_cast<const __half*>(p); }
}  // namespace

extern "C" int gfxb_residual_rms_norm_pack(const std::uint16_t* input, const float* update, std::uint16_t* residual_out,
                                           const std::uint16_t* bf16_weight, std::uint16_t* normalized_out,
                                           std::size_t elements, unsigned batch, float epsilon, int add_unit_offset,
                                           int act_bits, std::int8_t* act_codes, std::uint16_t* act_scales,
                                           std::int32_t* act_sums, std::uint8_t* packed_a4, void* stream) {
  GFXB_REQUIRE(input != nullptr, "RMSNorm input is null");
  GFXB_REQUIRE(update == nullptr || residual_out != nullptr || normalized_out != nullptr || act_codes != nullptr,
               "RMSNorm has no output");
  NormPackArgs a;
  a.residual = as_half(input);
  a.update = update;
  a.residual_out = as_half(residual_out);
  a.weight = bf16_weight;
  a.unit_offset = add_unit_offset;
  a.epsilon = epsilon;
  a.elements = static_cast<std::uint32_t>(elements);
  a.normalized_out = as_half(normalized_out);
  a.act_codes = act_codes;
  a.act_scales = as_half(act_scales);
  a.act_sums = act_sums;
  a.packed_a4 = packed_a4;
  return launch_norm_pack(a, act_bits, batch, as_stream(stream));
}

extern "C" int gfxb_silu_multiply_pack(const float* gate, const float* up, std::size_t elements_per_row,
                                       unsigned batch, std::uint16_t* product_out, int act_bits,
                                       std::int8_t* act_codes, std::uint16_t* act_scales, std::int32_t* act_sums,
                                       std::uint8_t* packed_a4, void* stream) {
  GFXB_REQUIRE(act_bits == 0 || act_bits == 4 || act_bits == 8, "activation bits must be 0, 4 or 8");
  GFXB_REQUIRE(act_bits != 0 || product_out != nullptr, "SiLU multiply has no output");
  SiluPackArgs a;
  a.gate = gate;
  a.up = up;
  a.elements = static_cast<std::uint32_t>(elements_per_row);
  a.batch = batch;
  a.product_out = as_half(product_out);
  if (act_bits != 0) {
    a.act_codes = act_codes;
    a.act_scales = as_half(act_scales);
    a.act_sums = act_sums;
    a.packed_a4 = packed_a4;
  }
  return launch_silu_pack(a, act_bits == 0 ? 4 : act_bits, as_stream(stream));
}

extern "C" int gfxb_gdn_conv_update(const float* projected, const std::uint16_t* bf16_weight,
                                    const std::uint16_t* initial_state, std::uint16_t* final_state,
                                    std::uint16_t* output, std::uint16_t* appended_log, std::size_t channels,
                                    unsigned batch, void* stream) {
  GdnConvArgs a;
  a.projected = projected;
  a.weight = bf16_weight;
  a.initial_state = as_half(initial_state);
  a.final_state = as_half(final_state);
  a.output = as_half(output);
  a.appended_log = as_half(appended_log);
  a.channels = static_cast<std::uint32_t>(channels);
  a.batch = batch;
  return launch_gdn_conv(a, as_stream(stream));
}

extern "C" int gfxb_gdn_recurrent(const std::uint16_t* qkv, const float* z, const float* a, const float* b,
                                  const std::uint16_t* a_log, const std::uint16_t* dt_bias,
                                  const std::uint16_t* norm_weight, const float* initial_state, float* final_state,
                                  std::uint16_t* output, float* key_log, float* delta_log, float* decay_log,
                                  unsigned key_heads, unsigned value_heads, unsigned batch, void* stream) {
  GdnRecurrentArgs g;
  g.qkv = as_half(qkv);
  g.z = z;
  g.a = a;
  g.b = b;
  g.a_log = a_log;
  g.dt_bias = dt_bias;
  g.norm_weight = norm_weight;
  g.initial_state = initial_state;
  g.final_state = final_state;
  g.output = as_half(output);
  g.key_log = key_log;
  g.delta_log = delta_log;
  g.decay_log = decay_log;
  g.key_heads = key_heads;
  g.value_heads = value_heads;
  g.batch = batch;
  return launch_gdn_recurrent(g, as_stream(stream));
}

extern "C" int gfxb_gdn_restore_prefix_all(std::uint16_t* conv_states, float* recurrent_states,
                                           const std::uint16_t* conv_logs, const float* key_logs,
                                           const float* delta_logs, const float* decay_logs, std::size_t channels,
                                           unsigned key_heads, unsigned value_heads, unsigned layers,
                                           unsigned maximum_logged_tokens, unsigned accepted_tokens, void* stream) {
  GdnRestoreArgs r;
  r.conv_states = as_half(conv_states);
  r.states = recurrent_states;
  r.conv_logs = as_half(conv_logs);
  r.key_logs = key_logs;
  r.delta_logs = delta_logs;
  r.decay_logs = decay_logs;
  r.channels = static_cast<std::uint32_t>(channels);
  r.key_heads = key_heads;
  r.value_heads = value_heads;
  r.layers = layers;
  r.max_logged = maximum_logged_tokens;
  r.accepted = accepted_tokens;
  return launch_gdn_restore(r, as_stream(stream));
}

extern "C" int gfxb_qk_rms_norm_rope(const float* q_input, const std::uint16_t* q_weight, std::uint16_t* q_output,
                                     unsigned q_heads, std::size_t q_stride, const float* k_input,
                                     const std::uint16_t* k_weight, std::uint16_t* k_output, unsigned k_heads,
                                     std::size_t k_stride, unsigned rotary, const float* cos_table,
                                     const float* sin_table, std::size_t table_positions, std::uint64_t base_position,
                                     const std::uint64_t* device_base_position, unsigned batch, const float* v_input,
                                     std::uint16_t* key_cache, std::uint16_t* value_cache, std::size_t capacity,
                                     void* stream) {
  QkRopeArgs r;
  r.q_input = q_input;
  r.q_weight = q_weight;
  r.q_output = as_half(q_output);
  r.k_input = k_input;
  r.k_weight = k_weight;
  r.k_output = as_half(k_output);
  r.v_input = v_input;
  r.key_cache = as_half(key_cache);
  r.value_cache = as_half(value_cache);
  r.capacity = capacity;
  r.q_heads = q_heads;
  r.k_heads = k_heads;
  r.q_stride = static_cast<std::uint32_t>(q_stride);
  r.k_stride = static_cast<std::uint32_t>(k_stride);
  r.rotary = rotary;
  r.cos_table = cos_table;
  r.sin_table = sin_table;
  r.table_positions = table_positions;
  r.base_position = base_position;
  r.device_base_position = device_base_position;
  if (device_base_position == nullptr && base_position + batch > table_positions) {
    return fail(GFXB_INVALID_ARGUMENT, "RoPE positions exceed the table");
  }
  return launch_qk_rope(r, batch, as_stream(stream));
}

extern "C" std::size_t gfxb_gated_attention_scratch_bytes(unsigned q_heads, std::size_t capacity, unsigned batch) {
  return attention_partial_bytes(q_heads, capacity, batch);
}

extern "C" int gfxb_gated_attention(const std::uint16_t* query, const float* gate_projection,
                                    const std::uint16_t* key_cache, const std::uint16_t* value_cache,
                                    std::uint16_t* output, std::size_t base_token_count,
                                    const std::uint64_t* device_base_position, std::size_t capacity, unsigned q_heads,
                                    unsigned kv_heads, unsigned batch, void* scratch, std::size_t scratch_bytes,
                                    void* stream) {
  GFXB_REQUIRE(scratch != nullptr && scratch_bytes >= attention_partial_bytes(q_heads, capacity, batch),
               "attention scratch is too small");
  AttentionArgs a;
  a.query = as_half(query);
  a.gate = gate_projection;
  a.key_cache = as_half(key_cache);
  a.value_cache = as_half(value_cache);
  a.output = as_half(output);
  a.partials = static_cast<float*>(scratch);
  a.max_chunks = static_cast<std::uint32_t>((capacity + kAttentionChunk - 1) / kAttentionChunk);
  a.capacity = capacity;
  a.base_token_count = base_token_count;
  a.device_base_position = device_base_position;
  a.q_heads = q_heads;
  a.kv_heads = kv_heads;
  return launch_attention(a, batch, as_stream(stream));
}

extern "C" std::size_t gfxb_decode_attention_scratch_bytes(unsigned q_heads, std::size_t capacity) {
  return attention_partial_bytes(q_heads, capacity, 1) + static_cast<std::size_t>(q_heads) * sizeof(std::uint32_t);
}

extern "C" int gfxb_decode_attention(const float* q_input, const std::uint16_t* q_weight, std::size_t q_stride,
                                     const float* k_input, const std::uint16_t* k_weight, std::size_t k_stride,
                                     const float* v_input, unsigned rotary, const float* cos_table,
                                     const float* sin_table, std::size_t table_positions, std::uint16_t* key_cache,
                                     std::uint16_t* value_cache, std::size_t capacity, std::uint64_t position,
                                     const std::uint64_t* device_position, unsigned q_heads, unsigned kv_heads,
                                     std::uint16_t* output, void* scratch, std::size_t scratch_bytes, void* stream) {
  GFXB_REQUIRE(q_heads != 0 && capacity != 0 && scratch != nullptr &&
                   scratch_bytes >= gfxb_decode_attention_scratch_bytes(q_heads, capacity),
               "decode attention scratch is too small");
  GFXB_REQUIRE(q_stride <= 0xffffffffull && k_stride <= 0xffffffffull, "row strides exceed 32 bits");
  GFXB_REQUIRE(device_position != nullptr || (position < capacity && position < table_positions),
               "position is outside the cache or the RoPE table");
  AttentionDecodeArgs d;
  QkRopeArgs& r = d.rope;
  r.q_input = q_input;
  r.q_weight = q_weight;
  r.k_input = k_input;
  r.k_weight = k_weight;
  r.v_input = v_input;
  r.key_cache = as_half(key_cache);
  r.value_cache = as_half(value_cache);
  r.capacity = capacity;
  r.q_heads = q_heads;
  r.k_heads = kv_heads;
  r.q_stride = static_cast<std::uint32_t>(q_stride);
  r.k_stride = static_cast<std::uint32_t>(k_stride);
  r.rotary = rotary;
  r.cos_table = cos_table;
  r.sin_table = sin_table;
  r.table_positions = table_positions;
  r.base_position = position;
  r.device_base_position = device_position;
  AttentionArgs& a = d.attention;
  a.gate = q_input;
  a.key_cache = r.key_cache;
  a.value_cache = r.value_cache;
  a.output = as_half(output);
  a.partials = static_cast<float*>(scratch);
  a.max_chunks = static_cast<std::uint32_t>((capacity + kAttentionChunk - 1) / kAttentionChunk);
  a.capacity = capacity;
  a.base_token_count = position + 1;
  a.device_base_position = device_position;
  a.q_heads = q_heads;
  a.kv_heads = kv_heads;
  d.tickets = reinterpret_cast<std::uint32_t*>(static_cast<std::uint8_t*>(scratch) +
                                               attention_partial_bytes(q_heads, capacity, 1));
  return launch_attention_decode(d, as_stream(stream));
}

extern "C" std::size_t gfxb_argmax_scratch_bytes(unsigned batch) { return argmax_scratch_bytes(batch); }

extern "C" int gfxb_argmax(const float* logits, const std::uint32_t* token_ids, std::uint32_t* tokens,
                           std::size_t vocabulary_size, std::size_t row_stride, unsigned batch, void* scratch,
                           std::size_t scratch_bytes, void* stream) {
  GFXB_REQUIRE(scratch != nullptr && scratch_bytes >= argmax_scratch_bytes(batch), "argmax scratch is too small");
  GFXB_REQUIRE(vocabulary_size <= 0xffffffffull, "vocabulary exceeds 32-bit token ids");
  ArgmaxArgs a;
  a.logits = logits;
  a.row_stride = row_stride;
  a.vocab = static_cast<std::uint32_t>(vocabulary_size);
  a.token_ids = token_ids;
  a.tokens = tokens;
  a.partial_values = static_cast<float*>(scratch);
  a.partial_indices = reinterpret_cast<std::uint32_t*>(static_cast<float*>(scratch) + static_cast<std::size_t>(batch) * 64);
  return launch_argmax(a, batch, as_stream(stream));
}

// ---------------------------------------------------------------------------
// Gated attention without allocation.
//
// Some callers cannot call cudaMalloc: code that runs inside another
// framework's memory budget (an inference server or plugin host that owns
// all device memory), latency-critical loops that cannot afford the implicit
// device synchronisation an allocation may cause, or embedded deployments that
// fix their memory map at start-up. For them this entry point keeps the
// attention chunk partials in a fixed array compiled into the library, so it
// allocates nothing. The array is 4 MiB; every GPU that loads the library
// holds it until the process exits.
// ---------------------------------------------------------------------------

namespace {

constexpr std::size_t kStaticAttentionScratchBytes = std::size_t{4} << 20;

static __device__ __align__(256) float g_static_attention_scratch[kStaticAttentionScratchBytes / sizeof(float)];

std::mutex g_static_scratch_mutex;
void* g_static_scratch_address[kMaxDevices] = {};

// Host code cannot pass the array's name to a kernel (it is a host-side
// stand-in, not a device address), so the device address is looked up once
// per device, with that device current, and cached.
int static_scratch_address(void** address) {
  int device = 0;
  GFXB_TRY(current_device(&device));
  std::lock_guard<std::mutex> lock(g_static_scratch_mutex);
  if (g_static_scratch_address[device] == nullptr) {
    void* pointer = nullptr;
    const cudaError_t error = cudaGetSymbolAddress(&pointer, g_static_attention_scratch);
    if (error != cudaSuccess) {
      set_error_cuda(error, "cudaGetSymbolAddress of the static attention scratch failed");
      return GFXB_CUDA_ERROR;
    }
    g_static_scratch_address[device] = pointer;
  }
  *address = g_static_scratch_address[device];
  return GFXB_OK;
}

}  // namespace

extern "C" int gfxb_gated_attention_static_scratch(const std::uint16_t* query, const float* gate_projection,
                                                   const std::uint16_t* key_cache, const std::uint16_t* value_cache,
                                                   std::uint16_t* output, std::size_t base_token_count,
                                                   const std::uint64_t* device_base_position, std::size_t capacity,
                                                   unsigned q_heads, unsigned kv_heads, unsigned batch,
                                                   void* stream) {
  // the shape limits of launch_attention first, so that the size product below cannot wrap
  if (batch == 0 || batch > 32 || kv_heads == 0 || q_heads == 0 || q_heads % kv_heads != 0 ||
      q_heads / kv_heads > 8 || capacity == 0 || capacity > (std::size_t{1} << 32)) {
    return fail(GFXB_INVALID_ARGUMENT, "invalid gated attention arguments");
  }
  const std::size_t needed = attention_partial_bytes(q_heads, capacity, batch);
  if (needed > kStaticAttentionScratchBytes) {
    return fail(GFXB_INVALID_ARGUMENT,
                "attention scratch (batch x q_heads x ceil(capacity / 128) x 258 floats) exceeds the 4 MiB "
                "static array of gfxb_gated_attention_static_scratch; use gfxb_gated_attention with a caller buffer");
  }
  void* scratch = nullptr;
  const int status = static_scratch_address(&scratch);
  if (status != GFXB_OK) return status;
  return gfxb_gated_attention(query, gate_projection, key_cache, value_cache, output, base_token_count,
                              device_base_position, capacity, q_heads, kv_heads, batch, scratch,
                              kStaticAttentionScratchBytes, stream);
}
