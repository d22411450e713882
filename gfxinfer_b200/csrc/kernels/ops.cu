// Decode-path operators for sm_100a: fused residual/RMSNorm/activation
// packing, SwiGLU + packing, Gated-DeltaNet conv and recurrence with rollback
// replay, fused Q/K RMSNorm + RoPE + KV append, chunked gated attention,
// argmax and embedding gathers.
//
// Replaces the reference's qwen_ops.hip kernels. Each kernel follows the
// reference arithmetic (file:line at each kernel) with one fixed reduction
// order that the CPU oracle restates, so outputs compare bit for bit.
#include <type_traits>

#include "common.cuh"
#include "ops.cuh"
#include "ops_device.cuh"

namespace gfxb {

__device__ std::uint32_t g_ops_error;

namespace {

// residual add + RMSNorm (+ activation pack): blockIdx.y = token; the
// blockIdx.x-th CTA of a token writes kNormSplitIters iterations (8 groups)
// of the outputs, each CTA computing the row's whole sum of squares, so one
// token's normalisation and packing is spread over several SMs.
constexpr unsigned kNormSplitIters = 4;

template <int ActBits, unsigned Iterations>
__global__ __launch_bounds__(kNormThreads) void residual_norm_pack_kernel(NormPackArgs args) {
  pdl_trigger();
  pdl_wait();
  __shared__ float warp_sums[8];
  __shared__ float warp_max[Iterations][8];
  __shared__ int warp_code_sums[Iterations][8];
  const unsigned begin = blockIdx.x * kNormSplitIters;
  const unsigned end = begin + kNormSplitIters < Iterations ? begin + kNormSplitIters : Iterations;
  norm_pack_body<ActBits, Iterations>(args, blockIdx.y, threadIdx.x, BlockSync{}, warp_sums, warp_max, warp_code_sums,
                                      begin, end);
}

// ---------------------------------------------------------------------------
// SiLU(gate) * up -> fp16 -> activation pack (qwen_ops.hip:108-163). One warp
// per 128-group; lane l owns elements 4l..4l+3 (one 32-bit fragment word).
// ---------------------------------------------------------------------------

template <int ActBits>
__global__ __launch_bounds__(256) void silu_pack_kernel(SiluPackArgs args) {
  pdl_trigger();
  pdl_wait();
  const unsigned lane = threadIdx.x & 31u, warp = threadIdx.x >> 5;
  const std::uint32_t groups = args.elements / kGroup;
  const std::uint32_t linear = blockIdx.x * 8u + warp;
  if (linear >= groups * args.batch) return;
  const std::uint32_t token = linear / groups, group = linear - token * groups;
  const std::size_t base = static_cast<std::size_t>(token) * args.elements + group * kGroup + 4u * lane;
  const float4 g4 = ld_cg_f4(args.gate + base);
  const float4 u4 = ld_cg_f4(args.up + base);
  const float gs[4] = {g4.x, g4.y, g4.z, g4.w};
  const float us[4] = {u4.x, u4.y, u4.z, u4.w};
  float x[4];
  float amax = 0.0f;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const __half product = silu_product(gs[j], us[j]);
    if (args.product_out != nullptr) args.product_out[base + j] = product;
    x[j] = h2f(product);
    amax = fmaxf(amax, fabsf(x[j]));
  }
  if (args.act_codes == nullptr) return;
  amax = warp_amax(amax);
  const __half scale_h = act_scale_of<ActBits>(amax);
  const float scale = h2f(scale_h);
  const float recip = __frcp_rn(scale);
  std::uint32_t word = 0;
  int code_sum = 0;
  int q[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    q[j] = act_code_fast<ActBits>(x[j], scale, recip);
    word |= (static_cast<std::uint32_t>(q[j]) & 0xffu) << (8 * j);
    code_sum += q[j];
  }
  const std::size_t group_base = static_cast<std::size_t>(token) * args.elements + group * kGroup;
  *reinterpret_cast<std::uint32_t*>(args.act_codes + group_base + fragment_offset(4u * lane)) = word;
  if (ActBits == 4 && args.packed_a4 != nullptr) {
    const std::uint32_t packed = static_cast<std::uint32_t>((q[0] & 15) | ((q[1] & 15) << 4)) |
                                 (static_cast<std::uint32_t>((q[2] & 15) | ((q[3] & 15) << 4)) << 8);
    *reinterpret_cast<std::uint16_t*>(args.packed_a4 + group_base / 2u + 2u * lane) =
        static_cast<std::uint16_t>(packed);
  }
  code_sum = warp_sum_int(code_sum);
  if (lane == 0) {
    args.act_scales[static_cast<std::size_t>(token) * groups + group] = scale_h;
    args.act_sums[static_cast<std::size_t>(token) * groups + group] = code_sum;
  }
}

// ---------------------------------------------------------------------------
// GDN causal conv (qwen_ops.hip:219-261): fp16 4-tap state per channel.
// ---------------------------------------------------------------------------

__global__ void gdn_conv_kernel(GdnConvArgs args) {
  pdl_trigger();
  pdl_wait();
  const std::uint32_t channel = blockIdx.x * blockDim.x + threadIdx.x;
  if (channel >= args.channels) return;
  __half taps[4];
  const __half* initial = args.initial_state + static_cast<std::size_t>(channel) * 4u;
#pragma unroll
  for (int i = 0; i < 4; ++i) taps[i] = initial[i];
  float w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) w[i] = bf2f(args.weight[static_cast<std::size_t>(channel) * 4u + i]);
  for (std::uint32_t token = 0; token < args.batch; ++token) {
    const std::size_t index = static_cast<std::size_t>(token) * args.channels + channel;
    args.output[index] = gdn_conv_step(taps, w, ld_cg(args.projected + index));
    if (args.appended_log != nullptr) args.appended_log[index] = taps[3];
  }
  __half* final_state = args.final_state + static_cast<std::size_t>(channel) * 4u;
#pragma unroll
  for (int i = 0; i < 4; ++i) final_state[i] = taps[i];
}

// ---------------------------------------------------------------------------
// GDN recurrent step (qwen_ops.hip:263-411). One CTA of 128 threads per value
// head; thread v keeps column S[:, v] of the 128x128 fp32 state in registers
// across the whole token block (read once, written once). Per token: q/k
// L2 norms (warp tree + tree of the four warp sums), decay/beta gates, the
// delta-rule column update as two ordered fma chains over k, output RMSNorm
// and SiLU(z) gate.
// ---------------------------------------------------------------------------

template <bool FusedConv, bool Block>
__global__ __launch_bounds__(kGdnThreads) void gdn_recurrent_kernel(GdnRecurrentArgs args) {
  pdl_trigger();
  // The head's 64 KB state slice is pulled into L2 before waiting for the
  // previous kernel: a prefetch is only a hint (L2 stays coherent with any
  // later write, e.g. a rollback replay), and the loads below then hit L2.
  if (threadIdx.x < 4u) {
    const std::uint8_t* slice = reinterpret_cast<const std::uint8_t*>(args.initial_state) +
                                (static_cast<std::size_t>(blockIdx.x) * kGdnHead * kGdnHead + threadIdx.x * 4096u) * 4u;
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(slice), "r"(16384u) : "memory");
  }
  pdl_wait();
  const unsigned vh = blockIdx.x, t = threadIdx.x;
  float S[kGdnRows];
  gdn_load_state(args, vh, t, S);
  if constexpr (Block) {  // up to kGdnBlockMax tokens: the three-phase form
    __shared__ GdnBlockScratch scratch;
    gdn_recurrent_block<FusedConv>(args, vh, t, S, scratch);
  } else {
    __shared__ GdnScratch scratch;
    gdn_recurrent_tokens<BlockSync, FusedConv>(args, vh, t, S, BlockSync{}, scratch);
  }
  gdn_store_state(args, vh, t, S);
}

// Rollback replay (qwen_ops.hip:467-539): conv inputs and delta-rule updates of
// the accepted prefix are re-applied to the untouched pre-block state, for all
// GDN layers in one launch. Bit-identical to the forward's update order.
__global__ void gdn_restore_conv_kernel(GdnRestoreArgs args) {
  pdl_trigger();
  pdl_wait();
  const std::uint64_t linear = static_cast<std::uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const std::uint64_t total = static_cast<std::uint64_t>(args.layers) * args.channels;
  if (linear >= total) return;
  const std::uint64_t layer = linear / args.channels, channel = linear % args.channels;
  __half* taps = args.conv_states + (layer * args.channels + channel) * 4u;
  const __half* log = args.conv_logs + layer * args.max_logged * args.channels;
  for (std::uint32_t t = 0; t < args.accepted; ++t) {
    taps[0] = taps[1];
    taps[1] = taps[2];
    taps[2] = taps[3];
    taps[3] = log[static_cast<std::size_t>(t) * args.channels + channel];
  }
}

__global__ __launch_bounds__(128) void gdn_restore_state_kernel(GdnRestoreArgs args) {
  pdl_trigger();
  pdl_wait();
  constexpr unsigned kHead = 128;
  const unsigned layer = blockIdx.x / args.value_heads, vh = blockIdx.x % args.value_heads;
  const unsigned v = threadIdx.x;
  const unsigned ratio = args.value_heads / args.key_heads, kh = vh / ratio;
  const std::size_t key_elements = static_cast<std::size_t>(args.key_heads) * kHead;
  const std::size_t value_elements = static_cast<std::size_t>(args.value_heads) * kHead;
  float* S = args.states + (static_cast<std::size_t>(layer) * args.value_heads + vh) * kHead * kHead;
  const float* key_log = args.key_logs + static_cast<std::size_t>(layer) * args.max_logged * key_elements;
  const float* delta_log = args.delta_logs + static_cast<std::size_t>(layer) * args.max_logged * value_elements;
  const float* decay_log = args.decay_logs + static_cast<std::size_t>(layer) * args.max_logged * args.value_heads;
  float column[kHead];
#pragma unroll
  for (unsigned k = 0; k < kHead; ++k) column[k] = S[k * kHead + v];
  for (std::uint32_t t = 0; t < args.accepted; ++t) {
    const float decay = decay_log[static_cast<std::size_t>(t) * args.value_heads + vh];
    const float delta = delta_log[static_cast<std::size_t>(t) * value_elements + vh * kHead + v];
    const float* keys = key_log + static_cast<std::size_t>(t) * key_elements + kh * kHead;
#pragma unroll
    for (unsigned k = 0; k < kHead; ++k) column[k] = fmaf(keys[k], delta, __fmul_rn(column[k], decay));
  }
#pragma unroll
  for (unsigned k = 0; k < kHead; ++k) S[k * kHead + v] = column[k];
}

// ---------------------------------------------------------------------------
// Q/K RMSNorm(1+w) + NeoX RoPE (+ KV append), qwen_ops.hip:599-696. One
// 256-thread CTA per (token, head); angles come from a host-built table.
// ---------------------------------------------------------------------------

__global__ __launch_bounds__(256) void qk_norm_rope_kernel(QkRopeArgs args) {
  pdl_trigger();
  pdl_wait();
  const unsigned heads = args.q_heads + args.k_heads;
  const unsigned token = blockIdx.x / heads, local = blockIdx.x % heads;
  const bool is_key = local >= args.q_heads;
  const unsigned head = is_key ? local - args.q_heads : local;
  const unsigned d = threadIdx.x;
  const std::uint64_t base = args.device_base_position != nullptr ? *args.device_base_position : args.base_position;
  const std::uint64_t position = base + token;
  const float* input = is_key ? args.k_input + (static_cast<std::size_t>(token) * args.k_heads + head) * args.k_stride
                              : args.q_input + (static_cast<std::size_t>(token) * args.q_heads + head) * args.q_stride;
  __shared__ float normalized[256];
  __shared__ float warp_sums[8];
  bool out_of_range = false;
  const __half result = qk_norm_rope_value(ld_cg(input + d), is_key ? args.k_weight : args.q_weight, position, args, d,
                                           BlockSync{}, normalized, warp_sums, out_of_range);
  if (out_of_range && d == 0) atomicOr(&g_ops_error, 2u);
  if (!is_key) {
    args.q_output[(static_cast<std::size_t>(token) * args.q_heads + head) * 256u + d] = result;
    return;
  }
  if (args.k_output != nullptr) args.k_output[(static_cast<std::size_t>(token) * args.k_heads + head) * 256u + d] = result;
  if (args.key_cache != nullptr) {
    if (position >= args.capacity) {
      if (d == 0) atomicOr(&g_ops_error, 4u);
      return;
    }
    const std::size_t slot = (static_cast<std::size_t>(position) * args.k_heads + head) * 256u + d;
    args.key_cache[slot] = result;
    args.value_cache[slot] = f2h(ld_cg(args.v_input + (static_cast<std::size_t>(token) * args.k_heads + head) * 256u + d));
  }
}

// ---------------------------------------------------------------------------
// Gated attention decode (qwen_ops.hip:698-766) as chunked online softmax:
// pass 1 handles one 128-position chunk per (token, kv head) CTA with one warp
// per query head; pass 2 merges chunks in ascending order and applies the
// sigmoid gate. Scores: lane l owns dims 8l..8l+7 (fma chain) + xor tree,
// times 1/16. Within a chunk the running maximum is an exact prefix max, so
// the per-position rescale factors equal the reference's serial update.
// ---------------------------------------------------------------------------

constexpr unsigned kChunk = kAttentionChunk;

// One CTA per (chunk of 128 positions, KV head, token); warp w < group is
// query head kvh * group + w. The chunk's key and value rows (512 B each)
// are staged into shared memory once for the whole GQA group by bulk copies
// that every thread helps issue, so the CTA waits for one memory round trip
// instead of one per eight rows and warp; the values land while the scores
// and the softmax run.
constexpr std::uint32_t kAttentionStageBytes = 2u * kChunk * 256u * 2u;

__global__ __launch_bounds__(256) void attention_chunk_kernel(AttentionArgs args) {
  extern __shared__ __align__(128) std::uint8_t stage[];
  pdl_trigger();
  pdl_wait();
  const unsigned group = args.q_heads / args.kv_heads;
  const unsigned warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
  const unsigned chunk = blockIdx.x, kvh = blockIdx.y, token = blockIdx.z;
  const std::uint64_t base = args.device_base_position != nullptr ? *args.device_base_position + 1u
                                                                  : args.base_token_count;
  const std::uint64_t count = base + token;  // positions 0 .. count-1 are visible
  const std::uint32_t chunks = static_cast<std::uint32_t>((count + kChunk - 1) / kChunk);
  __shared__ float scores[8][kChunk];
  __shared__ float alphas[8][kChunk];
  __shared__ float betas[8][kChunk];
  __shared__ __align__(8) std::uint64_t bars[2];  // keys, values
  if (chunk >= chunks) return;
  if (count > args.capacity) {
    if (threadIdx.x == 0) atomicOr(&g_ops_error, 8u);
    return;
  }
  const std::uint64_t begin = static_cast<std::uint64_t>(chunk) * kChunk;
  const std::uint64_t remaining = count - begin;
  const std::uint32_t n = remaining < kChunk ? static_cast<std::uint32_t>(remaining) : kChunk;
  __half* keys = reinterpret_cast<__half*>(stage);
  __half* values = keys + kChunk * 256u;
  if (threadIdx.x == 0) {
    mbar_init(&bars[0], 1);
    mbar_init(&bars[1], 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    mbar_expect_tx(&bars[0], n * 512u);
    mbar_expect_tx(&bars[1], n * 512u);
  }
  const std::size_t row_stride = static_cast<std::size_t>(args.kv_heads) * 256u;
  for (std::uint32_t i = threadIdx.x; i < 2u * n; i += blockDim.x) {
    const bool is_value = i >= n;
    const std::uint32_t row = is_value ? i - n : i;
    const __half* source = (is_value ? args.value_cache : args.key_cache) + (begin + row) * row_stride + kvh * 256u;
    bulk_g2s((is_value ? values : keys) + row * 256u, source, 512u, &bars[is_value ? 1 : 0]);
  }
  if (warp < group) {
    const unsigned h = kvh * group + warp;
    float* partial =
        args.partials + ((static_cast<std::size_t>(token) * args.q_heads + h) * args.max_chunks + chunk) * 258u;
    if (mbar_wait_bounded(&bars[0], 0, &g_ops_error)) {
      attention_chunk_warp<true>(args.query + (static_cast<std::size_t>(token) * args.q_heads + h) * 256u, keys,
                                 values, 256u, n, lane, scores[warp], alphas[warp], betas[warp], partial, &bars[1]);
      if (lane == 0 && !mbar_try_wait(&bars[1], 0)) atomicOr(&g_ops_error, kDeviceErrorTimeout);
    }
  }
  // no copy may still be landing when the CTA exits (only after a failed wait)
  if (threadIdx.x == 0) {
    mbar_wait_bounded(&bars[0], 0, nullptr);
    mbar_wait_bounded(&bars[1], 0, nullptr);
  }
}

__global__ __launch_bounds__(256) void attention_merge_kernel(AttentionArgs args) {
  pdl_trigger();
  pdl_wait();
  const unsigned h = blockIdx.x, token = blockIdx.y, d = threadIdx.x;
  const std::uint64_t base = args.device_base_position != nullptr ? *args.device_base_position + 1u
                                                                  : args.base_token_count;
  const std::uint64_t count = base + token;
  if (count > args.capacity) return;
  const std::uint32_t chunks = static_cast<std::uint32_t>((count + kChunk - 1) / kChunk);
  __shared__ float pack_max[2][4];
  __shared__ int pack_sum[2][4];
  attention_merge_head(args, h, token, d, chunks, BlockSync{}, pack_max, pack_sum);
}

// ---------------------------------------------------------------------------
// argmax with the lowest index on ties (qwen_ops.hip:768-807): per-block
// partial maxima, then one reduction per token (and an optional id map).
// ---------------------------------------------------------------------------

constexpr unsigned kArgmaxBlocks = 64;


__global__ __launch_bounds__(256) void argmax_partial_kernel(ArgmaxArgs args) {
  pdl_trigger();
  pdl_wait();
  const unsigned token = blockIdx.y;
  const float* logits = args.logits + static_cast<std::size_t>(token) * args.row_stride;
  float best = -__int_as_float(0x7f800000);
  std::uint32_t index = 0xffffffffu;
  for (std::uint32_t i = blockIdx.x * 256u + threadIdx.x; i < args.vocab; i += kArgmaxBlocks * 256u) {
    better(best, index, logits[i], i);
  }
#pragma unroll
  for (unsigned offset = 16; offset != 0; offset >>= 1) {
    const float other_value = __shfl_xor_sync(0xffffffffu, best, offset);
    const std::uint32_t other_index = __shfl_xor_sync(0xffffffffu, index, offset);
    better(best, index, other_value, other_index);
  }
  __shared__ float values[8];
  __shared__ std::uint32_t indices[8];
  if ((threadIdx.x & 31u) == 0) {
    values[threadIdx.x >> 5] = best;
    indices[threadIdx.x >> 5] = index;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < 8; ++w) better(best, index, values[w], indices[w]);
    args.partial_values[token * kArgmaxBlocks + blockIdx.x] = best;
    args.partial_indices[token * kArgmaxBlocks + blockIdx.x] = index;
  }
}

__global__ void argmax_final_kernel(ArgmaxArgs args) {
  pdl_trigger();
  pdl_wait();
  const unsigned token = blockIdx.x, lane = threadIdx.x;
  float best = -__int_as_float(0x7f800000);
  std::uint32_t index = 0xffffffffu;
  for (unsigned b = lane; b < kArgmaxBlocks; b += 32) {
    better(best, index, args.partial_values[token * kArgmaxBlocks + b], args.partial_indices[token * kArgmaxBlocks + b]);
  }
#pragma unroll
  for (unsigned offset = 16; offset != 0; offset >>= 1) {
    const float other_value = __shfl_xor_sync(0xffffffffu, best, offset);
    const std::uint32_t other_index = __shfl_xor_sync(0xffffffffu, index, offset);
    better(best, index, other_value, other_index);
  }
  if (lane == 0) {
    if (index >= args.vocab) index = 0;  // all NaN: the reference also returns 0
    args.tokens[token] = args.token_ids != nullptr ? args.token_ids[index] : index;
  }
}

// ---------------------------------------------------------------------------
// small elementwise helpers (qwen_ops.hip:809-828)
// ---------------------------------------------------------------------------

__global__ void float_to_half_kernel(const float* __restrict__ input, __half* __restrict__ output, std::size_t n) {
  pdl_trigger();
  pdl_wait();
  const std::size_t i = static_cast<std::size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i < n) output[i] = f2h(input[i]);
}

}  // namespace

// ===========================================================================
// launchers (C++ API used by the runtime; the C ABI wraps them)
// ===========================================================================

int launch_norm_pack(const NormPackArgs& args, int act_bits, unsigned batch, cudaStream_t stream) {
  if (args.weight == nullptr || batch == 0 || args.elements == 0 || args.elements % kNormThreads != 0 ||
      args.elements / kNormThreads > kNormMaxIter || !(args.epsilon > 0.0f)) {
    return fail(GFXB_INVALID_ARGUMENT, "invalid RMSNorm arguments (H must be a multiple of 256, at most 16384)");
  }
  if (args.embedding_codes == nullptr && args.residual == nullptr) {
    return fail(GFXB_INVALID_ARGUMENT, "RMSNorm needs an input");
  }
  if (act_bits != 0 && (args.act_codes == nullptr || args.act_scales == nullptr || args.act_sums == nullptr)) {
    return fail(GFXB_INVALID_ARGUMENT, "activation pack outputs are required");
  }
  if (act_bits != 0 && act_bits != 4 && act_bits != 8) {
    return fail(GFXB_INVALID_ARGUMENT, "activation bits must be 0, 4 or 8");
  }
  const unsigned iterations = args.elements / kNormThreads;
  bool launched = false;
  auto try_launch = [&](auto iter_tag) {
    constexpr unsigned kIter = decltype(iter_tag)::value;
    if (iterations != kIter) return;
    launched = true;
    const dim3 grid((kIter + kNormSplitIters - 1) / kNormSplitIters, batch);
    if (act_bits == 0) launch_kernel(residual_norm_pack_kernel<0, kIter>, grid, dim3(kNormThreads), 0, stream, 0, args);
    else if (act_bits == 4) launch_kernel(residual_norm_pack_kernel<4, kIter>, grid, dim3(kNormThreads), 0, stream, 0, args);
    else launch_kernel(residual_norm_pack_kernel<8, kIter>, grid, dim3(kNormThreads), 0, stream, 0, args);
  };
  try_launch(std::integral_constant<unsigned, 1>{});
  try_launch(std::integral_constant<unsigned, 2>{});
  try_launch(std::integral_constant<unsigned, 4>{});
  try_launch(std::integral_constant<unsigned, 8>{});
  try_launch(std::integral_constant<unsigned, 16>{});
  try_launch(std::integral_constant<unsigned, 20>{});
  try_launch(std::integral_constant<unsigned, 40>{});
  if (!launched) return fail(GFXB_UNSUPPORTED, "RMSNorm width must be 256 x {1,2,4,8,16,20,40}");
  return launch_status("RMSNorm launch failed");
}

int launch_silu_pack(const SiluPackArgs& args, int act_bits, cudaStream_t stream) {
  if (args.gate == nullptr || args.up == nullptr || args.elements == 0 || args.elements % kGroup != 0 ||
      args.batch == 0 || args.batch > 32) {
    return fail(GFXB_INVALID_ARGUMENT, "invalid SiLU/pack arguments");
  }
  if (args.act_codes != nullptr && (args.act_scales == nullptr || args.act_sums == nullptr)) {
    return fail(GFXB_INVALID_ARGUMENT, "activation pack outputs are required");
  }
  const std::uint32_t groups = args.elements / kGroup * args.batch;
  const unsigned grid = (groups + 7u) / 8u;
  if (act_bits == 8) {
    launch_kernel(silu_pack_kernel<8>, dim3(grid), dim3(256), 0, stream, 0, args);
  } else {
    launch_kernel(silu_pack_kernel<4>, dim3(grid), dim3(256), 0, stream, 0, args);
  }
  return launch_status("SiLU/pack launch failed");
}

int launch_gdn_conv(const GdnConvArgs& args, cudaStream_t stream) {
  if (args.projected == nullptr || args.weight == nullptr || args.initial_state == nullptr ||
      args.final_state == nullptr || args.output == nullptr || args.channels == 0 || args.batch == 0) {
    return fail(GFXB_INVALID_ARGUMENT, "invalid GDN convolution arguments");
  }
  launch_kernel(gdn_conv_kernel, dim3((args.channels + 255u) / 256u), dim3(256), 0, stream, 0, args);
  return launch_status("GDN convolution launch failed");
}

int launch_gdn_recurrent(const GdnRecurrentArgs& args, cudaStream_t stream) {
  if (args.z == nullptr || args.a == nullptr || args.b == nullptr || args.a_log == nullptr ||
      args.dt_bias == nullptr || args.norm_weight == nullptr || args.initial_state == nullptr ||
      args.final_state == nullptr || args.output == nullptr || args.batch == 0 || args.key_heads == 0 ||
      args.value_heads == 0 || args.value_heads % args.key_heads != 0) {
    return fail(GFXB_INVALID_ARGUMENT, "invalid GDN recurrent arguments");
  }
  if (args.conv.projected != nullptr) {
    // one cluster per key head: its value heads share the q/k conv channels
    const unsigned ratio = args.value_heads / args.key_heads;
    if (ratio > 8 || args.conv.weight == nullptr || args.conv.initial_state == nullptr ||
        args.conv.final_state == nullptr) {
      return fail(GFXB_INVALID_ARGUMENT, "fused GDN conv needs its weights and states and at most 8 value heads "
                                         "per key head");
    }
    if (args.batch >= 2u && args.batch <= kGdnBlockMax) {  // a verifier block: the three-phase form
      launch_kernel(gdn_recurrent_kernel<true, true>, dim3(args.value_heads), dim3(kGdnThreads), 0, stream, ratio,
                    args);
    } else {
      launch_kernel(gdn_recurrent_kernel<true, false>, dim3(args.value_heads), dim3(kGdnThreads), 0, stream, ratio,
                    args);
    }
  } else {
    if (args.qkv == nullptr) return fail(GFXB_INVALID_ARGUMENT, "invalid GDN recurrent arguments");
    if (args.batch >= 2u && args.batch <= kGdnBlockMax) {  // a verifier block: the three-phase form
      launch_kernel(gdn_recurrent_kernel<false, true>, dim3(args.value_heads), dim3(kGdnThreads), 0, stream, 0, args);
    } else {
      launch_kernel(gdn_recurrent_kernel<false, false>, dim3(args.value_heads), dim3(kGdnThreads), 0, stream, 0, args);
    }
  }
  return launch_status("GDN recurrent launch failed");
}

int launch_gdn_restore(const GdnRestoreArgs& args, cudaStream_t stream) {
  if (args.conv_states == nullptr || args.states == nullptr || args.conv_logs == nullptr || args.key_logs == nullptr ||
      args.delta_logs == nullptr || args.decay_logs == nullptr || args.channels == 0 || args.layers == 0 ||
      args.max_logged == 0 || args.accepted == 0 || args.accepted > args.max_logged || args.key_heads == 0 ||
      args.value_heads % args.key_heads != 0) {
    return fail(GFXB_INVALID_ARGUMENT, "invalid GDN prefix restore arguments");
  }
  const std::uint64_t total = static_cast<std::uint64_t>(args.layers) * args.channels;
  launch_kernel(gdn_restore_conv_kernel, dim3(static_cast<unsigned>((total + 255u) / 256u)), dim3(256), 0, stream, 0,
                args);
  int status = launch_status("GDN convolution restore launch failed");
  if (status != GFXB_OK) return status;
  launch_kernel(gdn_restore_state_kernel, dim3(args.layers * args.value_heads), dim3(128), 0, stream, 0, args);
  return launch_status("GDN recurrent restore launch failed");
}

int launch_qk_rope(const QkRopeArgs& args, unsigned batch, cudaStream_t stream) {
  if (args.q_input == nullptr || args.q_weight == nullptr || args.q_output == nullptr || args.k_input == nullptr ||
      args.k_weight == nullptr || args.q_heads == 0 || args.k_heads == 0 || batch == 0 || args.rotary == 0 ||
      args.rotary > 256 || (args.rotary & 1u) != 0 || args.cos_table == nullptr || args.sin_table == nullptr ||
      args.q_stride < 256 || args.k_stride < 256) {
    return fail(GFXB_INVALID_ARGUMENT, "invalid Q/K RMSNorm/RoPE arguments");
  }
  if (args.key_cache != nullptr && (args.value_cache == nullptr || args.v_input == nullptr)) {
    return fail(GFXB_INVALID_ARGUMENT, "KV append needs value input and cache");
  }
  if (args.device_base_position == nullptr && args.key_cache != nullptr &&
      args.base_position + batch > args.capacity) {
    return fail(GFXB_INVALID_ARGUMENT, "KV append exceeds the cache capacity");
  }
  launch_kernel(qk_norm_rope_kernel, dim3((args.q_heads + args.k_heads) * batch), dim3(256), 0, stream, 0, args);
  return launch_status("Q/K RMSNorm/RoPE launch failed");
}

std::size_t attention_partial_bytes(unsigned q_heads, std::size_t capacity, unsigned batch) {
  const std::size_t chunks = (capacity + kChunk - 1) / kChunk;
  return static_cast<std::size_t>(batch) * q_heads * chunks * 258u * sizeof(float);
}

int launch_attention(const AttentionArgs& args, unsigned batch, cudaStream_t stream) {
  if (args.query == nullptr || args.gate == nullptr || args.key_cache == nullptr || args.value_cache == nullptr ||
      args.output == nullptr || args.partials == nullptr || batch == 0 || batch > 32 || args.kv_heads == 0 ||
      args.q_heads % args.kv_heads != 0 || args.q_heads / args.kv_heads > 8) {
    return fail(GFXB_INVALID_ARGUMENT, "invalid gated attention arguments");
  }
  if (args.max_chunks < (args.capacity + kChunk - 1) / kChunk) {
    return fail(GFXB_INVALID_ARGUMENT, "attention partial buffer is too small for the capacity");
  }
  if (args.device_base_position == nullptr &&
      (args.base_token_count == 0 || args.base_token_count + batch - 1 > args.capacity)) {
    return fail(GFXB_INVALID_ARGUMENT, "attention token count exceeds the cache capacity");
  }
  const std::uint32_t max_chunks = args.device_base_position != nullptr
                                       ? args.max_chunks
                                       : static_cast<std::uint32_t>((args.base_token_count + batch - 1 + kChunk - 1) / kChunk);
  static DeviceOnce configured;
  GFXB_TRY(configured.run([](int) {
    const cudaError_t error = cudaFuncSetAttribute(attention_chunk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                   static_cast<int>(kAttentionStageBytes));
    if (error != cudaSuccess) {
      set_error_cuda(error, "attention shared-memory configuration failed");
      return static_cast<int>(GFXB_CUDA_ERROR);
    }
    return static_cast<int>(GFXB_OK);
  }));
  launch_kernel(attention_chunk_kernel, dim3(dim3(max_chunks, args.kv_heads, batch)), dim3(256),
                kAttentionStageBytes, stream, 0, args);
  int status = launch_status("attention chunk launch failed");
  if (status != GFXB_OK) return status;
  launch_kernel(attention_merge_kernel, dim3(dim3(args.q_heads, batch)), dim3(256), 0, stream, 0, args);
  return launch_status("attention merge launch failed");
}

std::size_t argmax_scratch_bytes(unsigned batch) {
  return static_cast<std::size_t>(batch) * kArgmaxBlocks * (sizeof(float) + sizeof(std::uint32_t));
}

int launch_argmax(const ArgmaxArgs& args, unsigned batch, cudaStream_t stream) {
  if (args.logits == nullptr || args.tokens == nullptr || args.partial_values == nullptr ||
      args.partial_indices == nullptr || args.vocab == 0 || args.row_stride < args.vocab || batch == 0 ||
      batch > 32) {
    return fail(GFXB_INVALID_ARGUMENT, "invalid argmax arguments");
  }
  launch_kernel(argmax_partial_kernel, dim3(dim3(kArgmaxBlocks, batch)), dim3(256), 0, stream, 0, args);
  int status = launch_status("argmax launch failed");
  if (status != GFXB_OK) return status;
  launch_kernel(argmax_final_kernel, dim3(batch), dim3(32), 0, stream, 0, args);
  return launch_status("argmax launch failed");
}

int launch_float_to_half(const float* input, __half* output, std::size_t n, cudaStream_t stream) {
  if (input == nullptr || output == nullptr || n == 0) return fail(GFXB_INVALID_ARGUMENT, "invalid float-to-half arguments");
  launch_kernel(float_to_half_kernel, dim3(static_cast<unsigned>((n + 255) / 256)), dim3(256), 0, stream, 0, input,
                output, n);
  return launch_status("float-to-half launch failed");
}

int read_ops_error(std::uint32_t* value, bool clear) {
  cudaError_t error = cudaMemcpyFromSymbol(value, g_ops_error, sizeof(std::uint32_t));
  if (error == cudaSuccess && clear) {
    const std::uint32_t zero = 0;
    error = cudaMemcpyToSymbol(g_ops_error, &zero, sizeof zero);
  }
  if (error != cudaSuccess) {
    set_error_cuda(error, "device error word access failed");
    return GFXB_CUDA_ERROR;
  }
  return GFXB_OK;
}

}  // namespace gfxb
