// Device bodies of the decode-path operators, shared by the standalone
// kernels (ops.cu) and the persistent token kernel (token_loop.cu), so that
// both run the same arithmetic in the same order.
//
// Each body takes a synchronisation policy: the standalone kernels pass
// BlockSync (__syncthreads); the persistent kernel passes a named barrier
// covering only its compute warps. Inputs that another CTA of the same grid
// may have written are read with ld.global.cg (L2), never through L1.
#pragma once

#include "common.cuh"
#include "ops.cuh"

namespace gfxb {

struct BlockSync {
  __device__ __forceinline__ void operator()() const { __syncthreads(); }
};

template <unsigned Id, unsigned Threads>
struct NamedSync {
  __device__ __forceinline__ void operator()() const {
    asm volatile("bar.sync %0, %1;" ::"n"(Id), "n"(Threads) : "memory");
  }
};

// ---- L2 loads for data produced inside the running grid --------------------

__device__ __forceinline__ float ld_cg(const float* p) {
  float v;
  asm volatile("ld.global.cg.f32 %0, [%1];" : "=f"(v) : "l"(p));
  return v;
}
__device__ __forceinline__ __half ld_cg(const __half* p) {
  unsigned short v;
  asm volatile("ld.global.cg.u16 %0, [%1];" : "=h"(v) : "l"(p));
  return __ushort_as_half(v);
}
__device__ __forceinline__ int ld_cg(const int* p) {
  int v;
  asm volatile("ld.global.cg.s32 %0, [%1];" : "=r"(v) : "l"(p));
  return v;
}
__device__ __forceinline__ std::uint32_t ld_cg(const std::uint32_t* p) {
  std::uint32_t v;
  asm volatile("ld.global.cg.u32 %0, [%1];" : "=r"(v) : "l"(p));
  return v;
}
__device__ __forceinline__ uint4 ld_cg16(const void* p) {
  uint4 v;
  asm volatile("ld.global.cg.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
  return v;
}
__device__ __forceinline__ float4 ld_cg_f4(const float* p) {
  float4 v;
  asm volatile("ld.global.cg.v4.f32 {%0,%1,%2,%3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "l"(p));
  return v;
}

// Position of logical column k (0..127) of a 128-group in the GEMV activation
// pack's fragment order.
__device__ __forceinline__ std::uint32_t fragment_offset(std::uint32_t k) {
  const std::uint32_t s = k >> 5, rest = k & 31u, half = rest >> 4, t = (rest & 15u) >> 2, j = k & 3u;
  return t * 32u + s * 8u + half * 4u + j;
}

// Reference A4/A8 rule (lowbit_gemv.hip:373-436): scale = fp16(amax / 7 or
// 127), 1 when the group is all zero; code = clamp(round_even(x / scale)).
template <int ActBits>
__device__ __forceinline__ __half act_scale_of(float amax) {
  constexpr float kDivisor = ActBits == 4 ? 7.0f : 127.0f;
  return f2h(amax == 0.0f ? 1.0f : __fdiv_rn(amax, kDivisor));
}
template <int ActBits>
__device__ __forceinline__ int act_code_of(float x, float scale) {
  constexpr int kLimit = ActBits == 4 ? 7 : 127;
  return max(-kLimit, min(kLimit, f2i_rn(__fdiv_rn(x, scale))));
}

// The same code without a division per element, for fp16 values x and fp16
// scales (`recip` = __frcp_rn(scale), computed once per group). Exactness:
// x and (k + 1/2) * scale lie on a common grid, so a quotient x / scale that
// is not exactly k + 1/2 lies at least 2^-12 from it, while the fp32
// quotient the reference rounds is within 2^-17 of the exact one; the
// reference's rint(fp32(x / scale)) is therefore round-half-even of the exact
// quotient. That is decided here from k = floor(x * recip) (at most one off,
// and only next to an integer, where either k resolves the same way) and the
// exactly rounded sign of x - (k + 1/2) * scale (one fma). Non-finite inputs
// and zero or non-finite scales take the division.
template <int ActBits>
__device__ __forceinline__ int act_code_fast(float x, float scale, float recip) {
  constexpr float kLimit = ActBits == 4 ? 7.0f : 127.0f;
  if (!(scale > 0.0f) || !isfinite(scale) || !isfinite(x)) return act_code_of<ActBits>(x, scale);
  const float k = floorf(__fmul_rn(x, recip));
  const float e = fmaf(-__fadd_rn(k, 0.5f), scale, x);
  float q = e > 0.0f ? __fadd_rn(k, 1.0f) : k;
  if (e == 0.0f && (__float2int_rz(k) & 1) != 0) q = __fadd_rn(k, 1.0f);  // tie: the even neighbour (|k| < 2^23 here)
  return static_cast<int>(fminf(fmaxf(q, -kLimit), kLimit));
}

// Largest |v| over the warp (NaN lanes count as 0, as fmaxf ignores NaN):
// one redux on the bit patterns, which order like the non-negative values.
__device__ __forceinline__ float warp_amax(float v) {
  const float a = fabsf(v);
  const std::uint32_t bits = a == a ? __float_as_uint(a) : 0u;
  return __uint_as_float(__reduce_max_sync(0xffffffffu, bits));
}
__device__ __forceinline__ int warp_sum_int(int v) { return __reduce_add_sync(0xffffffffu, v); }

// Quantize one 128-group held by four consecutive warps (element = thread
// index within the 128) and store it into a GEMV activation pack. `max_slot`
// and `sum_slot` hold 4 values of shared scratch per group.
template <int ActBits, class Sync>
__device__ __forceinline__ void pack_group_128(float x, unsigned element, std::int8_t* codes, __half* scale_out,
                                               std::int32_t* sum_out, float* max_slot, int* sum_slot, Sync sync) {
  const unsigned lane = element & 31u, warp = element >> 5;
  float amax = warp_amax(x);
  if (lane == 0) max_slot[warp] = amax;
  sync();
  amax = fmaxf(fmaxf(max_slot[0], max_slot[1]), fmaxf(max_slot[2], max_slot[3]));
  const __half scale_h = act_scale_of<ActBits>(amax);
  const float scale = h2f(scale_h);
  const int q = act_code_fast<ActBits>(x, scale, __frcp_rn(scale));
  codes[fragment_offset(element)] = static_cast<std::int8_t>(q);
  const int total = warp_sum_int(q);
  if (lane == 0) sum_slot[warp] = total;
  sync();
  if (element == 0) {
    *scale_out = scale_h;
    *sum_out = sum_slot[0] + sum_slot[1] + sum_slot[2] + sum_slot[3];
  }
}

// ---------------------------------------------------------------------------
// residual add + RMSNorm (+ activation pack), qwen_ops.hip:31-63, 176-217.
// 256 threads per token; thread t owns elements t, t+256, ...; the sum of
// squares is an fma chain per thread, the warp tree and the tree of the eight
// warp sums. The normalized fp16 value is quantized per 128-group with the
// reference's A4/A8 rule into a GEMV pack (global or shared memory).
// ---------------------------------------------------------------------------

constexpr unsigned kNormThreads = 256;
constexpr unsigned kNormMaxIter = 64;  // H <= 16384

// [it_begin, it_end) limits the outputs (residual, normalized values, pack)
// to elements it * 256 + t of those iterations, i.e. 128-groups 2 it_begin ..
// 2 it_end - 1; every thread still reads the whole row for the sum of squares.
// With dependency_wait the body waits for the previous kernel (pdl_wait) itself,
// after loading the norm weights, which never depend on it.
template <int ActBits, unsigned Iterations, class Sync>
__device__ __forceinline__ void norm_pack_body(const NormPackArgs& args, std::uint32_t token, unsigned t, Sync sync,
                                               float* warp_sums, float (*warp_max)[8], int (*warp_code_sums)[8],
                                               unsigned it_begin = 0, unsigned it_end = Iterations,
                                               bool dependency_wait = false) {
  const std::uint32_t H = args.elements;
  const unsigned lane = t & 31u, warp = t >> 5;
  constexpr unsigned iterations = Iterations;
  auto mine = [&](unsigned it) { return it >= it_begin && it < it_end; };
  const std::size_t row = static_cast<std::size_t>(token) * H;

  float values[Iterations];
  float weights[Iterations];
  float square_sum = 0.0f;
  // Every global load is issued before any store: the outputs may alias the
  // inputs as far as the compiler knows, so interleaving them would serialise
  // one memory round trip per element.
#pragma unroll
  for (unsigned it = 0; it < iterations; ++it) {
    const std::uint32_t column = it * kNormThreads + t;
    float scale = bf2f(args.weight[column]);
    if (args.unit_offset) scale = __fadd_rn(scale, 1.0f);
    weights[it] = scale;
  }
  if (dependency_wait) pdl_wait();
  if (args.embedding_codes != nullptr) {
    // Embedding row gather fused as the input (lowbit_gemv.hip:158-189, W4/W2 row-major).
    const std::uint32_t id = args.device_tokens != nullptr ? ld_cg(args.device_tokens + token) : args.host_token;
    const bool valid = id < args.embedding_rows;
    const std::uint32_t groups = H / kGroup;
#pragma unroll
    for (unsigned it = 0; it < iterations; ++it) {
      const std::uint32_t column = it * kNormThreads + t;
      float value = 0.0f;
      if (valid) {
        int q;
        if (args.embedding_bits == 2) {
          const std::uint8_t packed = args.embedding_codes[static_cast<std::size_t>(id) * (H / 4u) + column / 4u];
          q = static_cast<int>((packed >> ((column & 3u) * 2u)) & 3u) * 2 - 3;
        } else {
          const std::uint8_t packed = args.embedding_codes[static_cast<std::size_t>(id) * (H / 2u) + column / 2u];
          const int code = (packed >> ((column & 1u) * 4u)) & 15;
          q = code >= 8 ? code - 16 : code;
        }
        value = h2f(f2h(__fmul_rn(static_cast<float>(q),
                                  h2f(args.embedding_scales[static_cast<std::size_t>(id) * groups + column / kGroup]))));
      }
      values[it] = value;
    }
    if (args.residual_out != nullptr) {
#pragma unroll
      for (unsigned it = 0; it < iterations; ++it) {
        if (mine(it)) args.residual_out[row + it * kNormThreads + t] = f2h(values[it]);
      }
    }
  } else if (args.update != nullptr) {
    float updates[Iterations];
#pragma unroll
    for (unsigned it = 0; it < iterations; ++it) {
      const std::size_t index = row + it * kNormThreads + t;
      values[it] = h2f(ld_cg(args.residual + index));
      updates[it] = ld_cg(args.update + index);
    }
#pragma unroll
    for (unsigned it = 0; it < iterations; ++it) {
      const __half rounded = f2h(__fadd_rn(values[it], updates[it]));
      values[it] = h2f(rounded);
      if (args.residual_out != nullptr && mine(it)) args.residual_out[row + it * kNormThreads + t] = rounded;
    }
  } else {
#pragma unroll
    for (unsigned it = 0; it < iterations; ++it) values[it] = h2f(ld_cg(args.residual + row + it * kNormThreads + t));
  }
#pragma unroll
  for (unsigned it = 0; it < iterations; ++it) square_sum = fmaf(values[it], values[it], square_sum);
  square_sum = warp_sum_down(square_sum);
  if (lane == 0) warp_sums[warp] = square_sum;
  sync();
  const float total = tree_of_eight(warp_sums, 8);
  const float inverse = inv_sqrt_rn(__fadd_rn(__fdiv_rn(total, static_cast<float>(H)), args.epsilon));
#pragma unroll
  for (unsigned it = 0; it < iterations; ++it) {
    const std::uint32_t column = it * kNormThreads + t;
    const __half y = f2h(__fmul_rn(__fmul_rn(values[it], inverse), weights[it]));
    if (args.normalized_out != nullptr && mine(it)) args.normalized_out[row + column] = y;
    values[it] = h2f(y);
  }
  if constexpr (ActBits != 0) {
    // groups: element (it, t) belongs to group 2*it + (t >= 128), lane-local index t % 128
#pragma unroll
    for (unsigned it = 0; it < iterations; ++it) {
      if (!mine(it)) continue;
      const float amax = warp_amax(values[it]);
      if (lane == 0) warp_max[it][warp] = amax;
    }
    sync();
    const unsigned half = warp >> 2;
    const std::uint32_t groups = H / kGroup;
    // one thread per group turns the four warp maxima into the group's scale
    // and its reciprocal, left in the group's first two slots
    if (t < groups && mine(t >> 1)) {
      float* slot = warp_max[t >> 1] + 4 * (t & 1u);
      const float amax = fmaxf(fmaxf(slot[0], slot[1]), fmaxf(slot[2], slot[3]));
      const float scale = h2f(act_scale_of<ActBits>(amax));
      slot[0] = scale;
      slot[1] = __frcp_rn(scale);
    }
    sync();
#pragma unroll
    for (unsigned it = 0; it < iterations; ++it) {
      if (!mine(it)) continue;
      const float scale = warp_max[it][4 * half], recip = warp_max[it][4 * half + 1];
      const __half scale_h = f2h(scale);
      const int q = act_code_fast<ActBits>(values[it], scale, recip);
      const std::uint32_t group = 2u * it + half;
      const std::uint32_t local = t & 127u;
      args.act_codes[row + group * kGroup + fragment_offset(local)] = static_cast<std::int8_t>(q);
      if (ActBits == 4 && args.packed_a4 != nullptr) {
        const int neighbour = __shfl_down_sync(0xffffffffu, q, 1);
        if ((local & 1u) == 0) {
          args.packed_a4[static_cast<std::size_t>(token) * (H / 2u) + group * 64u + local / 2u] =
              static_cast<std::uint8_t>((q & 0x0f) | ((neighbour & 0x0f) << 4));
        }
      }
      const int code_sum = warp_sum_int(q);
      if (lane == 0) warp_code_sums[it][warp] = code_sum;
      if (local == 0) args.act_scales[static_cast<std::size_t>(token) * groups + group] = scale_h;
    }
    sync();
    for (std::uint32_t group = 2 * it_begin + t; group < 2 * it_end && group < groups; group += kNormThreads) {
      const unsigned it = group >> 1, h = group & 1u;
      args.act_sums[static_cast<std::size_t>(token) * groups + group] =
          warp_code_sums[it][4 * h] + warp_code_sums[it][4 * h + 1] + warp_code_sums[it][4 * h + 2] +
          warp_code_sums[it][4 * h + 3];
    }
  }
}

// SiLU(gate) * up rounded to fp16 (qwen_ops.hip:108-163).
__device__ __forceinline__ __half silu_product(float gate, float up) { return f2h(__fmul_rn(gx_silu(gate), up)); }

// One 128-group of fp16 values held four per lane (lane l: elements 4l..4l+3)
// -> fragment-order codes, scale and code sum. Every lane returns the sum.
template <int ActBits>
__device__ __forceinline__ void pack_warp_group(const float (&x)[4], unsigned lane, std::int8_t* group_codes,
                                                __half* scale_out, std::int32_t* sum_out) {
  const float amax = warp_amax(fmaxf(fmaxf(fabsf(x[0]), fabsf(x[1])), fmaxf(fabsf(x[2]), fabsf(x[3]))));
  const __half scale_h = act_scale_of<ActBits>(amax);
  const float scale = h2f(scale_h);
  const float recip = __frcp_rn(scale);
  std::uint32_t word = 0;
  int code_sum = 0;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int q = act_code_fast<ActBits>(x[j], scale, recip);
    word |= (static_cast<std::uint32_t>(q) & 0xffu) << (8 * j);
    code_sum += q;
  }
  *reinterpret_cast<std::uint32_t*>(group_codes + fragment_offset(4u * lane)) = word;
  code_sum = warp_sum_int(code_sum);
  if (lane == 0) {
    *scale_out = scale_h;
    *sum_out = code_sum;
  }
}

// GDN causal conv tap update for one channel (qwen_ops.hip:219-261): shift in
// fp16(projected), fma chain over the four taps, SiLU, fp16.
__device__ __forceinline__ __half gdn_conv_step(__half (&taps)[4], const float (&w)[4], float projected) {
  taps[0] = taps[1];
  taps[1] = taps[2];
  taps[2] = taps[3];
  taps[3] = f2h(projected);
  float conv = 0.0f;
#pragma unroll
  for (int i = 0; i < 4; ++i) conv = fmaf(h2f(taps[i]), w[i], conv);
  return f2h(gx_silu(conv));
}

// ---------------------------------------------------------------------------
// GDN recurrent step (qwen_ops.hip:263-411) for one value head, 256 threads.
// Thread t holds rows [64*(t&1), 64*(t&1)+64) of state column t>>1 in
// registers across the token block (read once, written once). Per token:
// q/k L2 norms on threads 0-127 (element v = t: warp tree + tree of the four
// warp sums), decay/beta gates, the delta-rule column update as two ordered
// fma chains over k, each run by the even lane over rows 0-63 and continued
// by the odd lane over rows 64-127 (the same chain, hence the same bits),
// then output RMSNorm and SiLU(z) gate on threads 0-127.
// ---------------------------------------------------------------------------

constexpr unsigned kGdnHead = 128;
constexpr unsigned kGdnThreads = 256;
constexpr unsigned kGdnRows = kGdnHead / 2;  // state rows per thread

struct GdnScratch {
  float query[kGdnHead];
  float key[kGdnHead];
  float mixed[kGdnHead];
  float value[kGdnHead];  // fused conv: this token's value vector
  float sums[3][4];
  float gates[2];  // decay, beta
  float pack_max[4];
  int pack_sum[4];
};

__device__ __forceinline__ void gdn_load_state(const GdnRecurrentArgs& args, unsigned vh, unsigned t,
                                               float (&S)[kGdnRows]) {
  const unsigned column = t >> 1, row0 = (t & 1u) * kGdnRows;
  const float* initial = args.initial_state + static_cast<std::size_t>(vh) * kGdnHead * kGdnHead;
#pragma unroll
  for (unsigned k = 0; k < kGdnRows; ++k) S[k] = initial[(row0 + k) * kGdnHead + column];
}

__device__ __forceinline__ void gdn_store_state(const GdnRecurrentArgs& args, unsigned vh, unsigned t,
                                                const float (&S)[kGdnRows]) {
  const unsigned column = t >> 1, row0 = (t & 1u) * kGdnRows;
  float* final_state = args.final_state + static_cast<std::size_t>(vh) * kGdnHead * kGdnHead;
#pragma unroll
  for (unsigned k = 0; k < kGdnRows; ++k) final_state[(row0 + k) * kGdnHead + column] = S[k];
}

// Causal-conv taps and weights of one channel, for the fused conv.
struct ConvChannel {
  __half taps[4];
  float w[4];
  __device__ __forceinline__ void load(const GdnConvArgs& conv, std::size_t channel) {
#pragma unroll
    for (int i = 0; i < 4; ++i) taps[i] = conv.initial_state[channel * 4u + i];
#pragma unroll
    for (int i = 0; i < 4; ++i) w[i] = bf2f(conv.weight[channel * 4u + i]);
  }
  __device__ __forceinline__ void store(const GdnConvArgs& conv, std::size_t channel) const {
#pragma unroll
    for (int i = 0; i < 4; ++i) conv.final_state[channel * 4u + i] = taps[i];
  }
  // the same loads as two 8-byte reads (weights, then taps): the weights never
  // change and may be read before the dependency wait, the taps may not
  __device__ __forceinline__ void load_weights(const GdnConvArgs& conv, std::size_t channel) {
    const uint2 raw = *reinterpret_cast<const uint2*>(conv.weight + channel * 4u);
    w[0] = bf2f(static_cast<std::uint16_t>(raw.x & 0xffffu));
    w[1] = bf2f(static_cast<std::uint16_t>(raw.x >> 16));
    w[2] = bf2f(static_cast<std::uint16_t>(raw.y & 0xffffu));
    w[3] = bf2f(static_cast<std::uint16_t>(raw.y >> 16));
  }
  __device__ __forceinline__ void load_taps(const GdnConvArgs& conv, std::size_t channel) {
    const uint2 raw = *reinterpret_cast<const uint2*>(conv.initial_state + channel * 4u);
    const __half* h = reinterpret_cast<const __half*>(&raw);
#pragma unroll
    for (int i = 0; i < 4; ++i) taps[i] = h[i];
  }
  // one token with its projected input already loaded
  __device__ __forceinline__ float step_input(float projected) { return h2f(gdn_conv_step(taps, w, projected)); }
  // one token: the same step as gdn_conv_kernel, including its log entry
  __device__ __forceinline__ float step(const GdnConvArgs& conv, std::size_t index, bool log) {
    const float y = h2f(gdn_conv_step(taps, w, ld_cg(conv.projected + index)));
    if (log && conv.appended_log != nullptr) conv.appended_log[index] = taps[3];
    return y;
  }
};

// With FusedConv the CTA convolves its own channels (element thread t: q and
// k channel t of key head kh, value channel t of head vh) instead of reading
// a conv output; the conv state of the shared q/k channels is written by the
// first value head of the key head only, after a cluster barrier that every
// CTA of the key head reaches once it has read the initial state.
template <class Sync, bool FusedConv = false>
__device__ __forceinline__ void gdn_recurrent_tokens(const GdnRecurrentArgs& args, unsigned vh, unsigned t,
                                                     float (&S)[kGdnRows], Sync sync, GdnScratch& sc) {
  const unsigned lane = t & 31u, warp = t >> 5;
  const bool element_thread = t < kGdnHead;  // threads 0-127: element v = t of the head vectors
  const unsigned column = t >> 1, half = t & 1u, row0 = half * kGdnRows;
  const unsigned ratio = args.value_heads / args.key_heads;
  const unsigned kh = vh / ratio;
  const unsigned key_elements = args.key_heads * kGdnHead;
  const unsigned value_elements = args.value_heads * kGdnHead;
  const unsigned channels = 2u * key_elements + value_elements;
  const float a_log = bf2f(args.a_log[vh]);
  const float dt_bias = bf2f(args.dt_bias[vh]);
  const float norm_weight = element_thread ? bf2f(args.norm_weight[t]) : 0.0f;
  const std::uint32_t ab_stride = args.ab_stride != 0 ? args.ab_stride : args.value_heads;
  const bool qk_owner = vh % ratio == 0;  // writes the shared q/k conv state and logs
  const std::size_t q_channel = kh * kGdnHead + t, k_channel = key_elements + kh * kGdnHead + t;
  const std::size_t v_channel = 2u * key_elements + vh * kGdnHead + t;
  ConvChannel cq, ck, cv;
  if constexpr (FusedConv) {
    if (element_thread) {
      cq.load(args.conv, q_channel);
      ck.load(args.conv, k_channel);
      cv.load(args.conv, v_channel);
    }
    cluster_arrive();  // this CTA has read the initial conv state
  }

  for (std::uint32_t token = 0; token < args.batch; ++token) {
    const __half* qkv = args.qkv + static_cast<std::size_t>(token) * channels;
    float q = 0.0f, k = 0.0f;
    if (element_thread) {
      if constexpr (FusedConv) {
        const std::size_t row = static_cast<std::size_t>(token) * channels;
        q = cq.step(args.conv, row + q_channel, qk_owner);
        k = ck.step(args.conv, row + k_channel, qk_owner);
        sc.value[t] = cv.step(args.conv, row + v_channel, true);
      } else {
        q = h2f(ld_cg(qkv + kh * kGdnHead + t));
        k = h2f(ld_cg(qkv + key_elements + kh * kGdnHead + t));
      }
      const float qs = warp_sum_down(__fmul_rn(q, q));
      const float ks = warp_sum_down(__fmul_rn(k, k));
      if (lane == 0) {
        sc.sums[0][warp] = qs;
        sc.sums[1][warp] = ks;
      }
    }
    sync();
    if (element_thread) {
      const float inv_q = __fmul_rn(inv_sqrt_rn(__fadd_rn(tree_of_eight(sc.sums[0], 4), 1.0e-6f)), 0.08838834764831845f);
      const float inv_k = inv_sqrt_rn(__fadd_rn(tree_of_eight(sc.sums[1], 4), 1.0e-6f));
      const float kn = __fmul_rn(k, inv_k);
      sc.query[t] = __fmul_rn(q, inv_q);
      sc.key[t] = kn;
      if (args.key_log != nullptr && vh % ratio == 0) {
        args.key_log[static_cast<std::size_t>(token) * key_elements + kh * kGdnHead + t] = kn;
      }
      if (t == 0) {
        const float a_value = __fadd_rn(ld_cg(args.a + static_cast<std::size_t>(token) * ab_stride + vh), dt_bias);
        const float softplus = a_value > 20.0f ? a_value : gx_log1pf(gx_expf(a_value));
        const float g = __fmul_rn(-gx_expf(a_log), softplus);
        const float decay = gx_expf(g);
        sc.gates[0] = decay;
        sc.gates[1] = gx_sigmoid(ld_cg(args.b + static_cast<std::size_t>(token) * ab_stride + vh));
        if (args.decay_log != nullptr) args.decay_log[static_cast<std::size_t>(token) * args.value_heads + vh] = decay;
      }
    }
    sync();
    const float decay = sc.gates[0], beta = sc.gates[1];
    // memory = sum_k (S[k][v] * decay) * key[k], one fma chain in k order
    float memory = 0.0f;
#pragma unroll
    for (unsigned kk = 0; kk < kGdnRows; ++kk) {
      S[kk] = __fmul_rn(S[kk], decay);
      if (half == 0) memory = fmaf(S[kk], sc.key[kk], memory);
    }
    const float carried = __shfl_up_sync(0xffffffffu, memory, 1);
    if (half == 1) {
      memory = carried;
#pragma unroll
      for (unsigned kk = 0; kk < kGdnRows; ++kk) memory = fmaf(S[kk], sc.key[kGdnRows + kk], memory);
    }
    float delta = 0.0f;
    if (half == 1) {
      float value;
      if constexpr (FusedConv) {
        value = sc.value[column];
      } else {
        value = h2f(ld_cg(qkv + 2u * key_elements + vh * kGdnHead + column));
      }
      delta = __fmul_rn(__fsub_rn(value, memory), beta);
      if (args.delta_log != nullptr) {
        args.delta_log[static_cast<std::size_t>(token) * value_elements + vh * kGdnHead + column] = delta;
      }
    }
    delta = __shfl_sync(0xffffffffu, delta, lane | 1u);
    // S[k][v] += key[k] * delta, then mixed = sum_k S[k][v] * query[k] (one chain)
    float mixed = 0.0f;
#pragma unroll
    for (unsigned kk = 0; kk < kGdnRows; ++kk) {
      S[kk] = fmaf(sc.key[row0 + kk], delta, S[kk]);
      if (half == 0) mixed = fmaf(S[kk], sc.query[kk], mixed);
    }
    const float mixed_carried = __shfl_up_sync(0xffffffffu, mixed, 1);
    if (half == 1) {
      mixed = mixed_carried;
#pragma unroll
      for (unsigned kk = 0; kk < kGdnRows; ++kk) mixed = fmaf(S[kk], sc.query[kGdnRows + kk], mixed);
      sc.mixed[column] = mixed;
    }
    sync();
    float y_value = 0.0f;
    if (element_thread) {
      const float m = sc.mixed[t];
      const float os = warp_sum_down(__fmul_rn(m, m));
      if (lane == 0) sc.sums[2][warp] = os;
    }
    sync();
    if (element_thread) {
      const float m = sc.mixed[t];
      const float inv_o = inv_sqrt_rn(__fadd_rn(__fdiv_rn(tree_of_eight(sc.sums[2], 4), 128.0f), 1.0e-6f));
      const float z = ld_cg(args.z + static_cast<std::size_t>(token) * value_elements + vh * kGdnHead + t);
      const float normalized = __fmul_rn(__fmul_rn(m, inv_o), norm_weight);
      const __half y = f2h(__fmul_rn(normalized, gx_silu(z)));
      args.output[static_cast<std::size_t>(token) * value_elements + vh * kGdnHead + t] = y;
      y_value = h2f(y);
    }
    if (args.act_bits != 0) {
      // one 128-group per value head, quantized by threads 0-127 (all threads meet the barriers)
      const std::size_t row = static_cast<std::size_t>(token) * value_elements + vh * kGdnHead;
      const std::size_t group = static_cast<std::size_t>(token) * args.value_heads + vh;
      float amax = warp_amax(y_value);
      if (element_thread && lane == 0) sc.pack_max[warp] = amax;
      sync();
      amax = fmaxf(fmaxf(sc.pack_max[0], sc.pack_max[1]), fmaxf(sc.pack_max[2], sc.pack_max[3]));
      const __half scale_h = args.act_bits == 8 ? act_scale_of<8>(amax) : act_scale_of<4>(amax);
      const float scale = h2f(scale_h), recip = __frcp_rn(scale);
      const int code = args.act_bits == 8 ? act_code_fast<8>(y_value, scale, recip) : act_code_fast<4>(y_value, scale, recip);
      if (element_thread) args.act_codes[row + fragment_offset(t)] = static_cast<std::int8_t>(code);
      const int total = warp_sum_int(code);
      if (element_thread && lane == 0) sc.pack_sum[warp] = total;
      sync();
      if (t == 0) {
        args.act_scales[group] = scale_h;
        args.act_sums[group] = sc.pack_sum[0] + sc.pack_sum[1] + sc.pack_sum[2] + sc.pack_sum[3];
      }
    }
    sync();  // query/key/mixed/sums are rewritten by the next token
  }
  if constexpr (FusedConv) {
    cluster_wait();  // every CTA of the key head has read the initial conv state
    if (element_thread) {
      cv.store(args.conv, v_channel);
      if (qk_owner) {
        cq.store(args.conv, q_channel);
        ck.store(args.conv, k_channel);
      }
    }
  }
}

// ---------------------------------------------------------------------------
// The same GDN step for a block of up to kGdnBlockMax tokens, in three phases:
// (1) for every token, the conv (serial over tokens per channel), the q/k
// L2 norms and the decay/beta gates, none of which depend on the state; (2)
// the delta-rule recurrence, the only serial part, which each (column, half)
// thread pair runs for all tokens without a CTA barrier; (3) for every token,
// the output RMSNorm, SiLU(z) gate and A4/A8 pack. Every value is computed
// by the same operations in the same order as gdn_recurrent_tokens, so the
// results are identical; only the barriers per token are gone.
// ---------------------------------------------------------------------------

constexpr unsigned kGdnBlockMax = 32;  // the scratch (66 KB) lives in dynamic shared memory

struct GdnBlockScratch {
  float query[kGdnBlockMax][kGdnHead];  // raw, then normalized
  float key[kGdnBlockMax][kGdnHead];
  float value[kGdnBlockMax][kGdnHead];
  float mixed[kGdnBlockMax][kGdnHead];
  float sums[kGdnBlockMax][3][4];       // q, k, output sums of squares per warp
  float gates[kGdnBlockMax][2];         // decay, beta
  float pack_max[kGdnBlockMax][4];
  int pack_sum[kGdnBlockMax][4];
};

template <bool FusedConv>
__device__ __forceinline__ void gdn_recurrent_block(const GdnRecurrentArgs& args, unsigned vh, unsigned t,
                                                    float (&S)[kGdnRows], GdnBlockScratch& sc) {
  const unsigned lane = t & 31u, warp = t >> 5;
  const bool element_thread = t < kGdnHead;
  const unsigned column = t >> 1, half = t & 1u, row0 = half * kGdnRows;
  const unsigned ratio = args.value_heads / args.key_heads;
  const unsigned kh = vh / ratio;
  const unsigned key_elements = args.key_heads * kGdnHead;
  const unsigned value_elements = args.value_heads * kGdnHead;
  const unsigned channels = 2u * key_elements + value_elements;
  const std::uint32_t B = args.batch;
  const float a_log = bf2f(args.a_log[vh]);
  const float dt_bias = bf2f(args.dt_bias[vh]);
  const float norm_weight = element_thread ? bf2f(args.norm_weight[t]) : 0.0f;
  const std::uint32_t ab_stride = args.ab_stride != 0 ? args.ab_stride : args.value_heads;
  const bool qk_owner = vh % ratio == 0;
  const std::size_t q_channel = kh * kGdnHead + t, k_channel = key_elements + kh * kGdnHead + t;
  const std::size_t v_channel = 2u * key_elements + vh * kGdnHead + t;
  ConvChannel cq, ck, cv;
  if constexpr (FusedConv) {
    if (element_thread) {
      cq.load(args.conv, q_channel);
      ck.load(args.conv, k_channel);
      cv.load(args.conv, v_channel);
    }
    cluster_arrive();  // this CTA has read the initial conv state
  }
  // ---- phase 1: inputs, norms and gates of every token ----
  if (element_thread) {
    for (std::uint32_t token = 0; token < B; ++token) {
      float q, k, v;
      if constexpr (FusedConv) {
        const std::size_t row = static_cast<std::size_t>(token) * channels;
        q = cq.step(args.conv, row + q_channel, qk_owner);
        k = ck.step(args.conv, row + k_channel, qk_owner);
        v = cv.step(args.conv, row + v_channel, true);
      } else {
        const __half* qkv = args.qkv + static_cast<std::size_t>(token) * channels;
        q = h2f(ld_cg(qkv + kh * kGdnHead + t));
        k = h2f(ld_cg(qkv + key_elements + kh * kGdnHead + t));
        v = h2f(ld_cg(qkv + 2u * key_elements + vh * kGdnHead + t));
      }
      sc.query[token][t] = q;
      sc.key[token][t] = k;
      sc.value[token][t] = v;
      const float qs = warp_sum_down(__fmul_rn(q, q));
      const float ks = warp_sum_down(__fmul_rn(k, k));
      if (lane == 0) {
        sc.sums[token][0][warp] = qs;
        sc.sums[token][1][warp] = ks;
      }
    }
  } else if (t - kGdnHead < B) {
    // thread 128 + i: the gates of token i, meanwhile
    const std::uint32_t token = t - kGdnHead;
    const float a_value = __fadd_rn(ld_cg(args.a + static_cast<std::size_t>(token) * ab_stride + vh), dt_bias);
    const float softplus = a_value > 20.0f ? a_value : gx_log1pf(gx_expf(a_value));
    const float g = __fmul_rn(-gx_expf(a_log), softplus);
    const float decay = gx_expf(g);
    sc.gates[token][0] = decay;
    sc.gates[token][1] = gx_sigmoid(ld_cg(args.b + static_cast<std::size_t>(token) * ab_stride + vh));
    if (args.decay_log != nullptr) args.decay_log[static_cast<std::size_t>(token) * args.value_heads + vh] = decay;
  }
  __syncthreads();
  if (element_thread) {
    for (std::uint32_t token = 0; token < B; ++token) {
      const float inv_q =
          __fmul_rn(inv_sqrt_rn(__fadd_rn(tree_of_eight(sc.sums[token][0], 4), 1.0e-6f)), 0.08838834764831845f);
      const float inv_k = inv_sqrt_rn(__fadd_rn(tree_of_eight(sc.sums[token][1], 4), 1.0e-6f));
      const float kn = __fmul_rn(sc.key[token][t], inv_k);
      sc.query[token][t] = __fmul_rn(sc.query[token][t], inv_q);
      sc.key[token][t] = kn;
      if (args.key_log != nullptr && qk_owner) {
        args.key_log[static_cast<std::size_t>(token) * key_elements + kh * kGdnHead + t] = kn;
      }
    }
  }
  __syncthreads();
  // ---- phase 2: the recurrence (one thread pair per state column, no CTA barrier) ----
  for (std::uint32_t token = 0; token < B; ++token) {
    const float decay = sc.gates[token][0], beta = sc.gates[token][1];
    const float* key = sc.key[token];
    const float* query = sc.query[token];
    float memory = 0.0f;
#pragma unroll
    for (unsigned kk = 0; kk < kGdnRows; ++kk) {
      S[kk] = __fmul_rn(S[kk], decay);
      if (half == 0) memory = fmaf(S[kk], key[kk], memory);
    }
    const float carried = __shfl_up_sync(0xffffffffu, memory, 1);
    if (half == 1) {
      memory = carried;
#pragma unroll
      for (unsigned kk = 0; kk < kGdnRows; ++kk) memory = fmaf(S[kk], key[kGdnRows + kk], memory);
    }
    float delta = 0.0f;
    if (half == 1) {
      delta = __fmul_rn(__fsub_rn(sc.value[token][column], memory), beta);
      if (args.delta_log != nullptr) {
        args.delta_log[static_cast<std::size_t>(token) * value_elements + vh * kGdnHead + column] = delta;
      }
    }
    delta = __shfl_sync(0xffffffffu, delta, lane | 1u);
    float mixed = 0.0f;
#pragma unroll
    for (unsigned kk = 0; kk < kGdnRows; ++kk) {
      S[kk] = fmaf(key[row0 + kk], delta, S[kk]);
      if (half == 0) mixed = fmaf(S[kk], query[kk], mixed);
    }
    const float mixed_carried = __shfl_up_sync(0xffffffffu, mixed, 1);
    if (half == 1) {
      mixed = mixed_carried;
#pragma unroll
      for (unsigned kk = 0; kk < kGdnRows; ++kk) mixed = fmaf(S[kk], query[kGdnRows + kk], mixed);
      sc.mixed[token][column] = mixed;
    }
  }
  __syncthreads();
  // ---- phase 3: output norm, gate and pack of every token ----
  if (element_thread) {
    for (std::uint32_t token = 0; token < B; ++token) {
      const float m = sc.mixed[token][t];
      const float os = warp_sum_down(__fmul_rn(m, m));
      if (lane == 0) sc.sums[token][2][warp] = os;
    }
  }
  __syncthreads();
  for (std::uint32_t token = 0; token < B; ++token) {
    float y_value = 0.0f;
    if (element_thread) {
      const float m = sc.mixed[token][t];
      const float inv_o = inv_sqrt_rn(__fadd_rn(__fdiv_rn(tree_of_eight(sc.sums[token][2], 4), 128.0f), 1.0e-6f));
      const float z = ld_cg(args.z + static_cast<std::size_t>(token) * value_elements + vh * kGdnHead + t);
      const float normalized = __fmul_rn(__fmul_rn(m, inv_o), norm_weight);
      const __half y = f2h(__fmul_rn(normalized, gx_silu(z)));
      args.output[static_cast<std::size_t>(token) * value_elements + vh * kGdnHead + t] = y;
      y_value = h2f(y);
    }
    if (element_thread) sc.mixed[token][t] = y_value;  // its own slot: the packer reads y here
    if (args.act_bits != 0) {
      const float amax = warp_amax(y_value);
      if (element_thread && lane == 0) sc.pack_max[token][warp] = amax;
    }
  }
  if (args.act_bits != 0) {
    __syncthreads();
    if (element_thread) {
      for (std::uint32_t token = 0; token < B; ++token) {
        const std::size_t row = static_cast<std::size_t>(token) * value_elements + vh * kGdnHead;
        const float* pm = sc.pack_max[token];
        const float amax = fmaxf(fmaxf(pm[0], pm[1]), fmaxf(pm[2], pm[3]));
        const __half scale_h = args.act_bits == 8 ? act_scale_of<8>(amax) : act_scale_of<4>(amax);
        const float scale = h2f(scale_h), recip = __frcp_rn(scale);
        const float y_value = sc.mixed[token][t];
        const int code =
            args.act_bits == 8 ? act_code_fast<8>(y_value, scale, recip) : act_code_fast<4>(y_value, scale, recip);
        args.act_codes[row + fragment_offset(t)] = static_cast<std::int8_t>(code);
        const int total = warp_sum_int(code);
        if (lane == 0) sc.pack_sum[token][warp] = total;
      }
    }
    __syncthreads();
    if (t < B) {
      const std::uint32_t token = t;
      const float* pm = sc.pack_max[token];
      const float amax = fmaxf(fmaxf(pm[0], pm[1]), fmaxf(pm[2], pm[3]));
      const std::size_t group = static_cast<std::size_t>(token) * args.value_heads + vh;
      args.act_scales[group] = args.act_bits == 8 ? act_scale_of<8>(amax) : act_scale_of<4>(amax);
      args.act_sums[group] = sc.pack_sum[token][0] + sc.pack_sum[token][1] + sc.pack_sum[token][2] +
                             sc.pack_sum[token][3];
    }
  }
  if constexpr (FusedConv) {
    cluster_wait();  // every CTA of the key head has read the initial conv state
    if (element_thread) {
      cv.store(args.conv, v_channel);
      if (qk_owner) {
        cq.store(args.conv, q_channel);
        ck.store(args.conv, k_channel);
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Q/K RMSNorm(1+w) + NeoX RoPE for one 256-wide head (qwen_ops.hip:599-696).
// 256 threads; thread d returns output element d. `normalized` (256 floats)
// and `warp_sums` (8) are shared scratch, free again when this returns.
// ---------------------------------------------------------------------------

template <class Sync>
__device__ __forceinline__ __half qk_norm_rope_value(float value, const std::uint16_t* weight, std::uint64_t position,
                                                     const QkRopeArgs& args, unsigned d, Sync sync, float* normalized,
                                                     float* warp_sums, bool& out_of_range) {
  const unsigned lane = d & 31u, warp = d >> 5;
  const float square = warp_sum_down(__fmul_rn(value, value));
  if (lane == 0) warp_sums[warp] = square;
  sync();
  const float inverse = inv_sqrt_rn(__fadd_rn(__fdiv_rn(tree_of_eight(warp_sums, 8), 256.0f), 1.0e-6f));
  normalized[d] = __fmul_rn(value, __fmul_rn(inverse, __fadd_rn(1.0f, bf2f(weight[d]))));
  sync();
  float out = normalized[d];
  const unsigned half = args.rotary / 2u;
  out_of_range = false;
  if (d < args.rotary) {
    const bool in_range = position < args.table_positions;
    out_of_range = !in_range;
    const std::uint64_t p = in_range ? position : 0;
    const unsigned f = d % half;
    const float partner = d < half ? normalized[d + half] : normalized[d - half];
    const float rotated = d < half ? -partner : partner;
    out = fmaf(out, args.cos_table[p * half + f], __fmul_rn(rotated, args.sin_table[p * half + f]));
  }
  sync();  // scratch reuse by the next head
  return f2h(out);
}

// ---------------------------------------------------------------------------
// Gated attention decode (qwen_ops.hip:698-766) as chunked online softmax.
// One warp handles one query head over one chunk of at most 128 positions:
// scores (lane l owns dims 8l..8l+7, fma chain + xor tree, times 1/16), the
// exact prefix max, then the rescaled accumulation; the partial (max, den,
// acc[256]) goes to `partial`. Within a chunk the running maximum is an exact
// prefix max, so the per-position rescale factors equal the reference's
// serial update.
// ---------------------------------------------------------------------------

// K/V rows come from global memory (L2 loads: the cache was appended inside
// the running grid or just before) or, with Staged, from shared memory where
// the caller has placed them; the arithmetic is the same either way.
template <bool Staged = false>
__device__ __forceinline__ uint4 kv_row_load(const __half* p) {
  if constexpr (Staged) {
    return *reinterpret_cast<const uint4*>(p);
  } else {
    return ld_cg16(p);
  }
}

template <bool Staged = false>
__device__ __forceinline__ void attention_chunk_warp(const __half* q_row, const __half* key_base,
                                                     const __half* value_base, std::size_t row_stride, std::uint32_t n,
                                                     unsigned lane, float* scores, float* alphas, float* betas,
                                                     float* partial, std::uint64_t* value_ready = nullptr) {
  float qf[8];
  {
    const uint4 raw = *reinterpret_cast<const uint4*>(q_row + 8u * lane);
    const __half* hv = reinterpret_cast<const __half*>(&raw);
#pragma unroll
    for (int j = 0; j < 8; ++j) qf[j] = h2f(hv[j]);
  }
  const __half* keys = key_base + 8u * lane;
  // eight key rows in flight per step; positions past n read row 0 (valid) and are dropped
  for (std::uint32_t p0 = 0; p0 < n; p0 += 8) {
    uint4 raw[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const std::uint32_t p = p0 + i < n ? p0 + i : 0u;
      raw[i] = kv_row_load<Staged>(keys + p * row_stride);
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const __half* hv = reinterpret_cast<const __half*>(&raw[i]);
      float s = 0.0f;
#pragma unroll
      for (int j = 0; j < 8; ++j) s = fmaf(qf[j], h2f(hv[j]), s);
      s = warp_sum_xor(s);
      if (lane == 0 && p0 + i < n) scores[p0 + i] = __fmul_rn(s, 0.0625f);
    }
  }
  __syncwarp();
  // prefix maximum: lane owns positions 4l..4l+3
  float local_max[4];
  float running = -__int_as_float(0x7f800000);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const std::uint32_t p = 4u * lane + j;
    if (p < n) running = fmaxf(running, scores[p]);
    local_max[j] = running;
  }
  float exclusive = __shfl_up_sync(0xffffffffu, running, 1);
  if (lane == 0) exclusive = -__int_as_float(0x7f800000);
#pragma unroll
  for (unsigned offset = 1; offset < 32; offset <<= 1) {
    const float other = __shfl_up_sync(0xffffffffu, exclusive, offset);
    if (lane >= offset) exclusive = fmaxf(exclusive, other);
  }
  float previous = exclusive;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const std::uint32_t p = 4u * lane + j;
    const float m = fmaxf(exclusive, local_max[j]);
    if (p < n) {
      alphas[p] = gx_expf(__fsub_rn(previous, m));
      betas[p] = gx_expf(__fsub_rn(scores[p], m));
    }
    previous = m;
  }
  const float chunk_max = __shfl_sync(0xffffffffu, previous, 31);
  __syncwarp();
  if (value_ready != nullptr && !mbar_wait_bounded(value_ready, 0, nullptr)) n = 0;  // staged values landed
  float den = 0.0f;
  float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  const __half* values = value_base + 8u * lane;
  for (std::uint32_t p0 = 0; p0 < n; p0 += 8) {
    uint4 raw[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const std::uint32_t p = p0 + i < n ? p0 + i : 0u;
      raw[i] = kv_row_load<Staged>(values + p * row_stride);
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      if (p0 + i < n) {
        const float alpha = alphas[p0 + i], beta = betas[p0 + i];
        const __half* hv = reinterpret_cast<const __half*>(&raw[i]);
        den = __fadd_rn(__fmul_rn(den, alpha), beta);
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[j] = __fadd_rn(__fmul_rn(acc[j], alpha), __fmul_rn(h2f(hv[j]), beta));
      }
    }
  }
  if (lane == 0) {
    partial[0] = chunk_max;
    partial[1] = den;
  }
#pragma unroll
  for (int j = 0; j < 8; ++j) partial[2 + 8 * lane + j] = acc[j];
}

// Merge of one query head's chunk partials in ascending chunk order, sigmoid
// gate, fp16 output and (optionally) the o_proj activation pack: 256 threads,
// thread d owns output dimension d.
template <class Sync>
__device__ __forceinline__ void attention_finish_head(const AttentionArgs& args, unsigned h, unsigned token, unsigned d,
                                                      float Acc, float Den, Sync sync, float (*pack_max)[4],
                                                      int (*pack_sum)[4]);

// Batch chunks' loads are issued before their part of the ordered chain (one memory round trip per batch);
// Batch = 1 keeps the register footprint of a single step.
template <class Sync, unsigned Batch = 8>
__device__ __forceinline__ void attention_merge_head(const AttentionArgs& args, unsigned h, unsigned token, unsigned d,
                                                     std::uint32_t chunks, Sync sync, float (*pack_max)[4],
                                                     int (*pack_sum)[4]) {
  const float* partial = args.partials + (static_cast<std::size_t>(token) * args.q_heads + h) * args.max_chunks * 258u;
  float M = ld_cg(partial), Den = ld_cg(partial + 1), Acc = ld_cg(partial + 2 + d);
  for (std::uint32_t c0 = 1; c0 < chunks; c0 += Batch) {
    float m[Batch], den[Batch], acc[Batch];
#pragma unroll
    for (unsigned i = 0; i < Batch; ++i) {
      if (c0 + i < chunks) {
        const float* p = partial + static_cast<std::size_t>(c0 + i) * 258u;
        m[i] = ld_cg(p);
        den[i] = ld_cg(p + 1);
        acc[i] = ld_cg(p + 2 + d);
      }
    }
#pragma unroll
    for (unsigned i = 0; i < Batch; ++i) {
      if (c0 + i < chunks) {
        const float next = fmaxf(M, m[i]);
        const float a1 = gx_expf(__fsub_rn(M, next));
        const float a2 = gx_expf(__fsub_rn(m[i], next));
        Den = __fadd_rn(__fmul_rn(Den, a1), __fmul_rn(den[i], a2));
        Acc = __fadd_rn(__fmul_rn(Acc, a1), __fmul_rn(acc[i], a2));
        M = next;
      }
    }
  }
  attention_finish_head(args, h, token, d, Acc, Den, sync, pack_max, pack_sum);
}

// Output element d of query head h from its merged accumulator and
// denominator: Acc / Den times the sigmoid gate, fp16, and (optionally) the
// o_proj activation pack. 256 threads, thread d owns dimension d.
template <class Sync>
__device__ __forceinline__ void attention_finish_head(const AttentionArgs& args, unsigned h, unsigned token, unsigned d,
                                                      float Acc, float Den, Sync sync, float (*pack_max)[4],
                                                      int (*pack_sum)[4]) {
  const float gate = ld_cg(args.gate + (static_cast<std::size_t>(token) * args.q_heads + h) * 512u + 256u + d);
  const __half y = f2h(__fmul_rn(__fdiv_rn(Acc, Den), gx_sigmoid(gate)));
  args.output[(static_cast<std::size_t>(token) * args.q_heads + h) * 256u + d] = y;
  if (args.act_bits != 0) {
    const unsigned half = d >> 7, element = d & 127u;
    const std::size_t row = (static_cast<std::size_t>(token) * args.q_heads + h) * 256u + half * 128u;
    const std::size_t group = static_cast<std::size_t>(token) * args.q_heads * 2u + h * 2u + half;
    if (args.act_bits == 8) {
      pack_group_128<8>(h2f(y), element, args.act_codes + row, args.act_scales + group, args.act_sums + group,
                        pack_max[half], pack_sum[half], sync);
    } else {
      pack_group_128<4>(h2f(y), element, args.act_codes + row, args.act_scales + group, args.act_sums + group,
                        pack_max[half], pack_sum[half], sync);
    }
  }
}

// argmax order (qwen_ops.hip:768-807): larger value wins, lower index on
// ties; NaN never wins.
__device__ __forceinline__ void better(float& best, std::uint32_t& index, float value, std::uint32_t other) {
  if (value > best || (value == best && other < index)) {
    best = value;
    index = other;
  }
}

}  // namespace gfxb
