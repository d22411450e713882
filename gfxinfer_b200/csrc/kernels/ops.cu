// Decode-path operators for sm_100a: fused residual/RMSNorm/activation
// packing, SwiGLU + packing, Gated-DeltaNet conv and recurrence with rollback
// replay, fused Q/K RMSNorm + RoPE + KV append, chunked gated attention,
// argmax and embedding gathers.
//
// Replaces the reference's qwen_ops.hip kernels. Each kernel follows the
// reference arithmetic (file:line at each kernel) with one fixed reduction
// order that the CPU oracle restates, so outputs compare bit for bit.
#include <type_traits>

#include <cstdlib>

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
  __shared__ float warp_sums[8];
  __shared__ float warp_max[Iterations][8];
  __shared__ int warp_code_sums[Iterations][8];
  const unsigned begin = blockIdx.x * kNormSplitIters;
  const unsigned end = begin + kNormSplitIters < Iterations ? begin + kNormSplitIters : Iterations;
  norm_pack_body<ActBits, Iterations>(args, blockIdx.y, threadIdx.x, BlockSync{}, warp_sums, warp_max, warp_code_sums,
                                      begin, end, true);
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
    extern __shared__ __align__(16) std::uint8_t block_scratch[];
    gdn_recurrent_block<FusedConv>(args, vh, t, S, *reinterpret_cast<GdnBlockScratch*>(block_scratch));
  } else {
    __shared__ GdnScratch scratch;
    gdn_recurrent_tokens<BlockSync, FusedConv>(args, vh, t, S, BlockSync{}, scratch);
  }
  gdn_store_state(args, vh, t, S);
}

// ---------------------------------------------------------------------------
// The single-token GDN step with the conv fused in, its 128 state columns split
// over kGdnParts CTAs per value head (4 x 48 CTAs for config 2 instead of 48).
// CTA (vh, part) holds columns [32 part, 32 part + 32): lane = column, warp w =
// rows [32 w, 32 w + 32), so every state load and store is one 128-byte line
// per warp. Each CTA convolves and normalises the key head's q/k itself; the
// two ordered fma chains over the 128 rows (memory = sum_k S[k][v] key[k],
// then mixed = sum_k S'[k][v] query[k]) pass from warp to warp in row order,
// the same operations in the same order as gdn_recurrent_tokens, hence the
// same bits. Parts 1..3 send their 32 mixed values to part 0 (st.async on one
// mbarrier) and exit; part 0 runs the output RMSNorm, SiLU(z) gate and pack
// for the whole head. The CTAs of one key head form one cluster: one cluster
// barrier, arrived right after the conv taps are read, orders every CTA's
// read of the shared q/k conv state before its single writer updates it and
// shows that part 0's mbarrier is initialised before the first remote store.
// ---------------------------------------------------------------------------

constexpr unsigned kGdnParts = 4;
constexpr unsigned kGdnPartColumns = kGdnHead / kGdnParts;
constexpr unsigned kGdnPartThreads = 128;

struct GdnPartScratch {
  float query[kGdnHead];
  float key[kGdnHead];
  float mixed[kGdnHead];  // part 0: the head's mixed values (own warp 0 + received)
  float value[kGdnPartColumns];
  float carry[kGdnPartColumns];
  float delta[kGdnPartColumns];
  float sums[3][4];
  float gates[2];
  float pack_max[4];
  int pack_sum[4];
  std::uint64_t bar;
};

__global__ __launch_bounds__(kGdnPartThreads) void gdn_parts_kernel(GdnRecurrentArgs args) {
  __shared__ __align__(16) GdnPartScratch sc;
  pdl_trigger();
  const unsigned t = threadIdx.x, lane = t & 31u, warp = t >> 5;
  const unsigned vh = blockIdx.x / kGdnParts, part = blockIdx.x % kGdnParts;
  const unsigned column = part * kGdnPartColumns + lane;  // this thread's state column
  const unsigned ratio = args.value_heads / args.key_heads, kh = vh / ratio;
  const unsigned key_elements = args.key_heads * kGdnHead;
  const unsigned value_elements = args.value_heads * kGdnHead;
  const bool qk_owner = vh % ratio == 0 && part == 0;  // writes the shared q/k conv state
  const std::size_t q_channel = kh * kGdnHead + t, k_channel = key_elements + kh * kGdnHead + t;
  const std::size_t v_channel = 2u * key_elements + vh * kGdnHead + column;
  const float* initial = args.initial_state + static_cast<std::size_t>(vh) * kGdnHead * kGdnHead;
  float* final_state = args.final_state + static_cast<std::size_t>(vh) * kGdnHead * kGdnHead;
  // weights never change: read before the dependency wait; the state slice is pulled into L2
  const float neg_exp_a_log = -gx_expf(bf2f(args.a_log[vh]));
  const float dt_bias = bf2f(args.dt_bias[vh]);
  const float norm_weight = part == 0 ? bf2f(args.norm_weight[t]) : 0.0f;
  ConvChannel cq, ck, cv;
  cq.load_weights(args.conv, q_channel);
  ck.load_weights(args.conv, k_channel);
  if (warp == 0) cv.load_weights(args.conv, v_channel);
  asm volatile("prefetch.global.L2 [%0];" ::"l"(initial + static_cast<std::size_t>(t) * kGdnHead +
                                                part * kGdnPartColumns)
               : "memory");
  if (part == 0 && t == 0) {
    mbar_init(&sc.bar, 1);
    fence_mbar_init();
    mbar_expect_tx(&sc.bar, (kGdnParts - 1u) * kGdnPartColumns * 4u);
  }
  pdl_wait();
  // every input of the step is requested at once (one memory round trip instead of one per use)
  const float xq = ld_cg(args.conv.projected + q_channel);
  const float xk = ld_cg(args.conv.projected + k_channel);
  const float xv = warp == 0 ? ld_cg(args.conv.projected + v_channel) : 0.0f;
  const float z = part == 0 ? ld_cg(args.z + static_cast<std::size_t>(vh) * kGdnHead + t) : 0.0f;
  const float a_in = t == 0 ? ld_cg(args.a + vh) : 0.0f;
  const float b_in = t == 32u ? ld_cg(args.b + vh) : 0.0f;
  cq.load_taps(args.conv, q_channel);
  ck.load_taps(args.conv, k_channel);
  if (warp == 0) cv.load_taps(args.conv, v_channel);
  float S[kGdnPartColumns];
#pragma unroll
  for (unsigned j = 0; j < kGdnPartColumns; ++j) S[j] = initial[(warp * kGdnPartColumns + j) * kGdnHead + column];
  cluster_arrive();  // this CTA has read the conv taps; part 0's barrier is initialised
  // q/k conv and norms (element t of the key head), the value conv of this part's columns, the gates
  const float q = cq.step_input(xq);
  const float k = ck.step_input(xk);
  if (warp == 0) sc.value[lane] = cv.step_input(xv);
  const float qs = warp_sum_down(__fmul_rn(q, q));
  const float ks = warp_sum_down(__fmul_rn(k, k));
  if (lane == 0) {
    sc.sums[0][warp] = qs;
    sc.sums[1][warp] = ks;
  }
  if (t == 0) {  // the decay's dependent exp / log1p / exp chain
    const float a_value = __fadd_rn(a_in, dt_bias);
    const float softplus = a_value > 20.0f ? a_value : gx_log1pf(gx_expf(a_value));
    sc.gates[0] = gx_expf(__fmul_rn(neg_exp_a_log, softplus));
  }
  if (t == 32u) sc.gates[1] = gx_sigmoid(b_in);  // beta, on another warp in parallel
  __syncthreads();
  {
    const float inv_q = __fmul_rn(inv_sqrt_rn(__fadd_rn(tree_of_eight(sc.sums[0], 4), 1.0e-6f)), 0.08838834764831845f);
    const float inv_k = inv_sqrt_rn(__fadd_rn(tree_of_eight(sc.sums[1], 4), 1.0e-6f));
    sc.query[t] = __fmul_rn(q, inv_q);
    sc.key[t] = __fmul_rn(k, inv_k);
  }
  __syncthreads();
  const float decay = sc.gates[0], beta = sc.gates[1];
  const unsigned row0 = warp * kGdnPartColumns;
#pragma unroll
  for (unsigned j = 0; j < kGdnPartColumns; ++j) S[j] = __fmul_rn(S[j], decay);
  // memory = sum over k in row order of S[k][v] * key[k], warp by warp
  for (unsigned w = 0; w < 4u; ++w) {
    if (warp == w) {
      float memory = w == 0 ? 0.0f : sc.carry[lane];
#pragma unroll
      for (unsigned j = 0; j < kGdnPartColumns; ++j) memory = fmaf(S[j], sc.key[row0 + j], memory);
      sc.carry[lane] = memory;
    }
    __syncthreads();
  }
  if (warp == 0) sc.delta[lane] = __fmul_rn(__fsub_rn(sc.value[lane], sc.carry[lane]), beta);
  __syncthreads();
  const float delta = sc.delta[lane];
#pragma unroll
  for (unsigned j = 0; j < kGdnPartColumns; ++j) S[j] = fmaf(sc.key[row0 + j], delta, S[j]);
  // mixed = sum over k in row order of S'[k][v] * query[k], warp by warp; a warp
  // stores its rows of the new state while another warp runs the chain (warps
  // 1-3 during warp 0's turn, warp 0 during warp 1's)
  for (unsigned w = 0; w < 4u; ++w) {
    if (warp == w) {
      float mixed = w == 0 ? 0.0f : sc.carry[lane];
#pragma unroll
      for (unsigned j = 0; j < kGdnPartColumns; ++j) mixed = fmaf(S[j], sc.query[row0 + j], mixed);
      sc.carry[lane] = mixed;
    } else if (w == (warp == 0 ? 1u : 0u)) {
#pragma unroll
      for (unsigned j = 0; j < kGdnPartColumns; ++j) final_state[(row0 + j) * kGdnHead + column] = S[j];
    }
    __syncthreads();
  }
  cluster_wait();  // every CTA of the key head has read the conv taps and part 0 can take stores
  if (warp == 0) cv.store(args.conv, v_channel);
  if (qk_owner) {
    cq.store(args.conv, q_channel);
    ck.store(args.conv, k_channel);
  }
  const std::uint32_t leader = (vh % ratio) * kGdnParts;  // cluster rank of this head's part 0
  if (part != 0) {
    if (warp == 0) {
      st_async_s32(map_shared_rank(smem_addr(&sc.mixed[column]), leader), __float_as_int(sc.carry[lane]),
                   map_shared_rank(smem_addr(&sc.bar), leader));
    }
    return;
  }
  if (warp == 0) sc.mixed[lane] = sc.carry[lane];
  bool arrived = false;
  for (std::uint32_t i = 0; i < kWaitLimit && !arrived; ++i) arrived = mbar_try_wait_cluster(&sc.bar, 0);
  if (!arrived && t == 0) atomicOr(&g_ops_error, kDeviceErrorTimeout);
  __syncthreads();
  // output RMSNorm, SiLU(z) gate and pack of the head (thread t = column t), as gdn_recurrent_tokens
  const float m = arrived ? sc.mixed[t] : 0.0f;
  const float os = warp_sum_down(__fmul_rn(m, m));
  if (lane == 0) sc.sums[2][warp] = os;
  __syncthreads();
  const float inv_o = inv_sqrt_rn(__fadd_rn(__fdiv_rn(tree_of_eight(sc.sums[2], 4), 128.0f), 1.0e-6f));
  const float normalized = __fmul_rn(__fmul_rn(m, inv_o), norm_weight);
  const __half y = f2h(__fmul_rn(normalized, gx_silu(z)));
  args.output[static_cast<std::size_t>(vh) * kGdnHead + t] = y;
  if (args.act_bits != 0) {
    const float y_value = h2f(y);
    const std::size_t row = static_cast<std::size_t>(vh) * kGdnHead;
    float amax = warp_amax(y_value);
    if (lane == 0) sc.pack_max[warp] = amax;
    __syncthreads();
    amax = fmaxf(fmaxf(sc.pack_max[0], sc.pack_max[1]), fmaxf(sc.pack_max[2], sc.pack_max[3]));
    const __half scale_h = args.act_bits == 8 ? act_scale_of<8>(amax) : act_scale_of<4>(amax);
    const float scale = h2f(scale_h), recip = __frcp_rn(scale);
    const int code = args.act_bits == 8 ? act_code_fast<8>(y_value, scale, recip) : act_code_fast<4>(y_value, scale, recip);
    args.act_codes[row + fragment_offset(t)] = static_cast<std::int8_t>(code);
    const int total = warp_sum_int(code);
    if (lane == 0) sc.pack_sum[warp] = total;
    __syncthreads();
    if (t == 0) {
      args.act_scales[vh] = scale_h;
      args.act_sums[vh] = sc.pack_sum[0] + sc.pack_sum[1] + sc.pack_sum[2] + sc.pack_sum[3];
    }
  }
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
    mbar_init(&bars[0], blockDim.x);
    mbar_init(&bars[1], blockDim.x);
    fence_mbar_init();
  }
  __syncthreads();
  // the chunk's key rows, then its value rows (512 bytes each), copied 16 bytes per thread
  // (consecutive threads take consecutive pieces of a row); each thread's copies arrive on
  // the rows' barrier as they land
  const std::size_t row_stride = static_cast<std::size_t>(args.kv_heads) * 256u;
  for (int which = 0; which < 2; ++which) {
    const __half* cache = which == 0 ? args.key_cache : args.value_cache;
    __half* dest = which == 0 ? keys : values;
    for (std::uint32_t i = threadIdx.x; i < n * 32u; i += blockDim.x) {
      const std::uint32_t row = i >> 5, piece = i & 31u;
      cp_async_16(dest + row * 256u + piece * 8u, cache + (begin + row) * row_stride + kvh * 256u + piece * 8u);
    }
    cp_async_arrive_noinc(&bars[which]);
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
// Single-token decode attention in one launch: the Q/K RMSNorm + RoPE, the
// KV append, the chunked online softmax and the merge. One CTA per (chunk of
// 128 positions, query head), so a head's chunk is spread over the whole CTA
// instead of one warp:
//  - the CTA normalises and rotates its query head; the CTA of the last chunk
//    also builds the new key/value row in shared memory (and one CTA per KV
//    head appends it to the cache), while the chunk's cached rows land by
//    cp.async;
//  - warp w scores positions 16w..16w+15: lane l runs the same 8-term fma
//    chain over dims 8l..8l+7 for each, and a transposed butterfly (each
//    exchange halves the positions a lane carries) adds the 32 lane partials
//    in the xor tree's pairs, 31 shuffles for 16 scores instead of 80;
//  - 128 threads scan the exact prefix maximum and form the rescale factors;
//  - thread t runs the accumulation chains of dims 2t and 2t+1 (thread 128
//    the denominator's);
//  - with one chunk the CTA finishes the head; otherwise the last CTA of the
//    head to arrive (ticket counter) merges the partials in ascending chunk
//    order.
// Every float operation and its order is that of qk_norm_rope_kernel,
// attention_chunk_kernel and attention_merge_kernel, so the outputs and the
// cache rows are bit-identical to the three-launch path.
// ---------------------------------------------------------------------------

constexpr std::uint32_t kDecodeStageBytes = 2u * kChunk * 256u * 2u;  // the chunk's key and value rows

// Shared: the keys and then the values of the chunk pass through one 64 KB stage (the values are copied in
// once the scores are done), so that three CTAs fit on an SM: for long contexts, where the grid holds several
// CTAs per SM. Otherwise both are staged at once into 128 KB.
template <bool Shared>
__global__ __launch_bounds__(256) void attention_decode_kernel(const AttentionDecodeArgs args) {
  extern __shared__ __align__(128) std::uint8_t stage[];
  __shared__ float normalized[256];
  __shared__ float warp_sums[8];
  __shared__ __align__(16) float query[256];
  __shared__ float scores[kChunk];
  __shared__ __align__(8) float2 rescale[kChunk];  // (alpha, beta) of each position
  __shared__ float warp_max[kChunk / 32u];
  __shared__ float head_max, head_den;
  __shared__ float pack_max[2][4];
  __shared__ int pack_sum[2][4];
  __shared__ bool merge_here;
  pdl_trigger();
  pdl_wait();
  const QkRopeArgs& R = args.rope;
  const AttentionArgs& A = args.attention;
  const unsigned chunk = blockIdx.x, h = blockIdx.y;
  const unsigned group = A.q_heads / A.kv_heads, kvh = h / group;
  const unsigned tid = threadIdx.x, warp = tid >> 5, lane = tid & 31u;
  const std::uint64_t count =
      A.device_base_position != nullptr ? *A.device_base_position + 1u : A.base_token_count;
  const std::uint64_t position = count - 1u;
  const std::uint32_t chunks = static_cast<std::uint32_t>((count + kChunk - 1) / kChunk);
  if (chunk >= chunks) return;
  if (count > A.capacity) {
    if (tid == 0 && chunk == 0) atomicOr(&g_ops_error, 4u | 8u);
    return;
  }
  const std::uint64_t begin = static_cast<std::uint64_t>(chunk) * kChunk;
  const std::uint32_t n = static_cast<std::uint32_t>(min(static_cast<std::uint64_t>(kChunk), count - begin));
  const bool holds_new = chunk + 1u == chunks;  // row n - 1 is `position`
  const std::uint32_t cached = holds_new ? n - 1u : n;
  __half* keys = reinterpret_cast<__half*>(stage);
  __half* values = Shared ? keys : keys + kChunk * 256u;
  const std::size_t row_stride = static_cast<std::size_t>(A.kv_heads) * 256u;
  const std::size_t first = (begin * A.kv_heads + kvh) * 256u;
  auto stage_values = [&]() {
    for (std::uint32_t i = tid; i < cached * 32u; i += blockDim.x) {
      const std::uint32_t row = i >> 5, piece = i & 31u;
      cp_async_16(values + row * 256u + piece * 8u, A.value_cache + first + row * row_stride + piece * 8u);
    }
    cp_async_commit();
  };
  for (std::uint32_t i = tid; i < cached * 32u; i += blockDim.x) {
    const std::uint32_t row = i >> 5, piece = i & 31u;
    cp_async_16(keys + row * 256u + piece * 8u, A.key_cache + first + row * row_stride + piece * 8u);
  }
  cp_async_commit();
  if constexpr (!Shared) stage_values();
  bool out_of_range = false;
  __half new_value = __ushort_as_half(0);
  query[tid] = h2f(qk_norm_rope_value(ld_cg(R.q_input + static_cast<std::size_t>(h) * R.q_stride + tid), R.q_weight,
                                      position, R, tid, BlockSync{}, normalized, warp_sums, out_of_range));
  if (holds_new) {
    const __half key = qk_norm_rope_value(ld_cg(R.k_input + static_cast<std::size_t>(kvh) * R.k_stride + tid),
                                          R.k_weight, position, R, tid, BlockSync{}, normalized, warp_sums,
                                          out_of_range);
    new_value = f2h(ld_cg(R.v_input + static_cast<std::size_t>(kvh) * 256u + tid));
    const __half value = new_value;
    keys[(n - 1u) * 256u + tid] = key;
    if constexpr (!Shared) values[(n - 1u) * 256u + tid] = value;
    if (h % group == 0) {  // one writer per KV head appends the row
      const std::size_t slot = (position * A.kv_heads + kvh) * 256u + tid;
      R.key_cache[slot] = key;
      R.value_cache[slot] = value;
    }
  }
  if (out_of_range && tid == 0) atomicOr(&g_ops_error, 2u);
  if constexpr (Shared) {
    cp_async_wait<0>();  // this thread's key copies
  } else {
    cp_async_wait<1>();  // this thread's key copies
  }
  __syncthreads();  // everyone's, the new row and the query

  if (16u * warp < n) {
    float qf[8];
    {
      const float4 q0 = *reinterpret_cast<const float4*>(query + 8u * lane);
      const float4 q1 = *reinterpret_cast<const float4*>(query + 8u * lane + 4u);
      qf[0] = q0.x, qf[1] = q0.y, qf[2] = q0.z, qf[3] = q0.w;
      qf[4] = q1.x, qf[5] = q1.y, qf[6] = q1.z, qf[7] = q1.w;
    }
    float part[16];
#pragma unroll
    for (unsigned i = 0; i < 16; ++i) {
      const std::uint32_t p = 16u * warp + i;
      const uint4 raw = *reinterpret_cast<const uint4*>(keys + (p < n ? p : 0u) * 256u + 8u * lane);
      const __half* hv = reinterpret_cast<const __half*>(&raw);
      float sum = 0.0f;
#pragma unroll
      for (int j = 0; j < 8; ++j) sum = fmaf(qf[j], h2f(hv[j]), sum);
      part[i] = sum;
    }
    // transposed xor butterfly: after the exchange at distance d a lane keeps
    // the half of its positions selected by its lane bit d, summed with the
    // partner's partials of the same positions (the tree's pair at that level)
#pragma unroll
    for (unsigned i = 0; i < 8; ++i) {
      const bool upper = (lane & 16u) != 0;
      const float send = upper ? part[i] : part[i + 8];
      const float keep = upper ? part[i + 8] : part[i];
      part[i] = __fadd_rn(keep, __shfl_xor_sync(0xffffffffu, send, 16));
    }
#pragma unroll
    for (unsigned i = 0; i < 4; ++i) {
      const bool upper = (lane & 8u) != 0;
      const float send = upper ? part[i] : part[i + 4];
      const float keep = upper ? part[i + 4] : part[i];
      part[i] = __fadd_rn(keep, __shfl_xor_sync(0xffffffffu, send, 8));
    }
#pragma unroll
    for (unsigned i = 0; i < 2; ++i) {
      const bool upper = (lane & 4u) != 0;
      const float send = upper ? part[i] : part[i + 2];
      const float keep = upper ? part[i + 2] : part[i];
      part[i] = __fadd_rn(keep, __shfl_xor_sync(0xffffffffu, send, 4));
    }
    {
      const bool upper = (lane & 2u) != 0;
      const float send = upper ? part[0] : part[1];
      const float keep = upper ? part[1] : part[0];
      part[0] = __fadd_rn(keep, __shfl_xor_sync(0xffffffffu, send, 2));
    }
    part[0] = __fadd_rn(part[0], __shfl_xor_sync(0xffffffffu, part[0], 1));
    const std::uint32_t p = 16u * warp + (lane >> 1);  // lane bits 4..1 name the position
    if ((lane & 1u) == 0 && p < n) scores[p] = __fmul_rn(part[0], 0.0625f);
  }
  __syncthreads();
  if constexpr (Shared) {  // every key has been read: the values take the stage
    stage_values();
    if (holds_new) values[(n - 1u) * 256u + tid] = new_value;
  }

  // exact prefix maximum over the chunk and the rescale factors
  const float negative_infinity = -__int_as_float(0x7f800000);
  float score = negative_infinity, inclusive = negative_infinity;
  if (tid < kChunk) {
    score = tid < n ? scores[tid] : negative_infinity;
    inclusive = fmaxf(negative_infinity, score);
#pragma unroll
    for (unsigned offset = 1; offset < 32; offset <<= 1) {
      const float other = __shfl_up_sync(0xffffffffu, inclusive, offset);
      if (lane >= offset) inclusive = fmaxf(inclusive, other);
    }
    if (lane == 31) warp_max[warp] = inclusive;
  }
  __syncthreads();
  if (tid < kChunk) {
    float before = negative_infinity;
    for (unsigned w = 0; w < warp; ++w) before = fmaxf(before, warp_max[w]);
    inclusive = fmaxf(before, inclusive);
    float previous = __shfl_up_sync(0xffffffffu, inclusive, 1);
    if (lane == 0) previous = before;
    if (tid < n) rescale[tid] = make_float2(gx_expf(__fsub_rn(previous, inclusive)), gx_expf(__fsub_rn(score, inclusive)));
    if (tid + 1u == n) head_max = inclusive;
  }
  cp_async_wait<0>();  // this thread's value copies
  __syncthreads();

  // scalar IEEE operations: packed f32x2 multiplies feeding packed adds are fused
  // into fma by the assembler, which would change the reference's rounding
  float2 acc = make_float2(0.0f, 0.0f);
  float den = 0.0f;
  if (tid < 128u) {
    const __half2* column = reinterpret_cast<const __half2*>(values) + tid;  // dims 2 tid, 2 tid + 1
#pragma unroll 8
    for (std::uint32_t p = 0; p < n; ++p) {
      const float2 ab = rescale[p];
      const float2 v = __half22float2(column[p * 128u]);
      acc.x = __fadd_rn(__fmul_rn(acc.x, ab.x), __fmul_rn(v.x, ab.y));
      acc.y = __fadd_rn(__fmul_rn(acc.y, ab.x), __fmul_rn(v.y, ab.y));
    }
  } else if (tid == 128u) {
    for (std::uint32_t p = 0; p < n; ++p) den = __fadd_rn(__fmul_rn(den, rescale[p].x), rescale[p].y);
  }

  if (chunks == 1u) {
    if (tid < 128u) {
      normalized[2u * tid] = acc.x;
      normalized[2u * tid + 1u] = acc.y;
    } else if (tid == 128u) {
      head_den = den;
    }
    __syncthreads();
    attention_finish_head(A, h, 0, tid, normalized[tid], head_den, BlockSync{}, pack_max, pack_sum);
    return;
  }
  float* partial = A.partials + (static_cast<std::size_t>(h) * A.max_chunks + chunk) * 258u;
  if (tid < 128u) {
    *reinterpret_cast<float2*>(partial + 2u + 2u * tid) = acc;
  } else if (tid == 128u) {
    partial[0] = head_max;
    partial[1] = den;
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    const std::uint32_t ticket = atomicAdd(&args.tickets[h], 1u);
    merge_here = ticket + 1u == chunks;
    if (merge_here) atomicExch(&args.tickets[h], 0u);  // every chunk of this launch has counted
  }
  __syncthreads();
  if (!merge_here) return;
  __threadfence();
  attention_merge_head(A, h, 0, tid, chunks, BlockSync{}, pack_max, pack_sum);
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

// GFXB_ATTENTION_FUSED=0 keeps single-token attention on the three-launch path (for A/B timing).
bool attention_decode_enabled() {
  static const bool enabled = [] {
    const char* value = std::getenv("GFXB_ATTENTION_FUSED");
    return value == nullptr || value[0] != '0';
  }();
  return enabled;
}

// GFXB_GDN_PARTS=0 keeps single-token steps on the one-CTA-per-head kernel (for A/B timing).
bool gdn_parts_enabled() {
  static const bool enabled = [] {
    const char* value = std::getenv("GFXB_GDN_PARTS");
    return value == nullptr || value[0] != '0';
  }();
  return enabled;
}

// The block form keeps every token's vectors in dynamic shared memory (above the 48 KB default).
int configure_gdn_block() {
  static DeviceOnce configured;
  return configured.run([](int) {
    cudaError_t error = cudaFuncSetAttribute(gdn_recurrent_kernel<true, true>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(sizeof(GdnBlockScratch)));
    if (error == cudaSuccess) {
      error = cudaFuncSetAttribute(gdn_recurrent_kernel<false, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   static_cast<int>(sizeof(GdnBlockScratch)));
    }
    if (error != cudaSuccess) {
      set_error_cuda(error, "GDN block shared-memory configuration failed");
      return static_cast<int>(GFXB_CUDA_ERROR);
    }
    return static_cast<int>(GFXB_OK);
  });
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
    if (args.batch == 1u && ratio * kGdnParts <= 16u && args.key_log == nullptr && args.delta_log == nullptr &&
        args.decay_log == nullptr && args.conv.appended_log == nullptr && gdn_parts_enabled()) {
      // one token: the head's columns over kGdnParts CTAs, the key head's CTAs one cluster
      static DeviceOnce configured;
      GFXB_TRY(configured.run([](int) {
        const cudaError_t error =
            cudaFuncSetAttribute(gdn_parts_kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
        if (error != cudaSuccess) {
          set_error_cuda(error, "GDN cluster configuration failed");
          return static_cast<int>(GFXB_CUDA_ERROR);
        }
        return static_cast<int>(GFXB_OK);
      }));
      launch_kernel(gdn_parts_kernel, dim3(args.value_heads * kGdnParts), dim3(kGdnPartThreads), 0, stream,
                    ratio * kGdnParts, args);
    } else if (args.batch >= 2u && args.batch <= kGdnBlockMax) {  // a verifier block: the three-phase form
      GFXB_TRY(configure_gdn_block());
      launch_kernel(gdn_recurrent_kernel<true, true>, dim3(args.value_heads), dim3(kGdnThreads),
                    sizeof(GdnBlockScratch), stream, ratio, args);
    } else {
      launch_kernel(gdn_recurrent_kernel<true, false>, dim3(args.value_heads), dim3(kGdnThreads), 0, stream, ratio,
                    args);
    }
  } else {
    if (args.qkv == nullptr) return fail(GFXB_INVALID_ARGUMENT, "invalid GDN recurrent arguments");
    if (args.batch >= 2u && args.batch <= kGdnBlockMax) {  // a verifier block: the three-phase form
      GFXB_TRY(configure_gdn_block());
      launch_kernel(gdn_recurrent_kernel<false, true>, dim3(args.value_heads), dim3(kGdnThreads),
                    sizeof(GdnBlockScratch), stream, 0, args);
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

int launch_attention_decode(const AttentionDecodeArgs& args, cudaStream_t stream) {
  const QkRopeArgs& r = args.rope;
  const AttentionArgs& a = args.attention;
  if (r.q_input == nullptr || r.q_weight == nullptr || r.k_input == nullptr || r.k_weight == nullptr ||
      r.v_input == nullptr || r.key_cache == nullptr || r.value_cache == nullptr || r.cos_table == nullptr ||
      r.sin_table == nullptr || r.q_stride < 256 || r.k_stride < 256 || r.rotary == 0 || r.rotary > 256 ||
      (r.rotary & 1u) != 0 || a.gate == nullptr || a.output == nullptr || a.partials == nullptr ||
      args.tickets == nullptr || a.kv_heads == 0 || a.q_heads % a.kv_heads != 0 || r.q_heads != a.q_heads ||
      r.k_heads != a.kv_heads || a.key_cache != r.key_cache || a.value_cache != r.value_cache ||
      a.capacity != r.capacity || a.device_base_position != r.device_base_position) {
    return fail(GFXB_INVALID_ARGUMENT, "invalid single-token attention arguments");
  }
  if (a.max_chunks < (a.capacity + kChunk - 1) / kChunk) {
    return fail(GFXB_INVALID_ARGUMENT, "attention partial buffer is too small for the capacity");
  }
  if (a.device_base_position == nullptr &&
      (a.base_token_count == 0 || a.base_token_count > a.capacity || r.base_position + 1u != a.base_token_count)) {
    return fail(GFXB_INVALID_ARGUMENT, "attention token count exceeds the cache capacity");
  }
  const std::uint32_t grid_chunks = a.device_base_position != nullptr
                                        ? a.max_chunks
                                        : static_cast<std::uint32_t>((a.base_token_count + kChunk - 1) / kChunk);
  static DeviceOnce configured;
  GFXB_TRY(configured.run([](int) {
    cudaError_t error = cudaFuncSetAttribute(attention_decode_kernel<false>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(kDecodeStageBytes));
    if (error == cudaSuccess) {
      error = cudaFuncSetAttribute(attention_decode_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   static_cast<int>(kDecodeStageBytes / 2u));
    }
    if (error != cudaSuccess) {
      set_error_cuda(error, "attention shared-memory configuration failed");
      return static_cast<int>(GFXB_CUDA_ERROR);
    }
    return static_cast<int>(GFXB_OK);
  }));
  // more CTAs than two per SM (long contexts): the shared 64 KB stage, three CTAs per SM
  int sms = 0;
  GFXB_TRY(device_sm_count(&sms));
  if (static_cast<std::uint64_t>(grid_chunks) * a.q_heads > 2ull * static_cast<std::uint64_t>(sms)) {
    launch_kernel(attention_decode_kernel<true>, dim3(grid_chunks, a.q_heads), dim3(256), kDecodeStageBytes / 2u,
                  stream, 0, args);
  } else {
    launch_kernel(attention_decode_kernel<false>, dim3(grid_chunks, a.q_heads), dim3(256), kDecodeStageBytes, stream,
                  0, args);
  }
  return launch_status("single-token attention launch failed");
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
