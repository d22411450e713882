// Low-bit dequant-GEMV for sm_100a: W2/W3/W4 group-128 weights x A4/A8
// activations on the int8 tensor cores (mma.sync m16n8k32 s8).
//
// Replaces the reference's RDNA4 WMMA kernels (lowbit_gemv.hip:461-755). The
// arithmetic contract is the reference's: per 128-column group an exact int32
// dot of weight codes and activation codes, then an fp32 fma chain over
// groups in ascending order with the product of the two fp16 scales
// (lowbit_gemv.hip:525-536). The result is therefore bit-identical to the
// reference's, independent of how this kernel splits the work.
//
// Codes enter the tensor core unsigned (u = q - beta/alpha): W3 u = q + 4,
// W4 u = q + 8, W2 u = (q + 3) / 2, and the exact correction
// dot = alpha * mma(u, a) + beta * sum(a) uses a per-group activation sum
// carried in the activation pack.
#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <map>
#include <mutex>
#include <tuple>

#include "codec.cuh"
#include "common.cuh"

namespace gfxb {
namespace {

// ---------------------------------------------------------------------------
// GEMV over the b200 layout
// ---------------------------------------------------------------------------

struct MatrixArg {
  const std::uint8_t* codes;
  const __half* scales;
  void* output;
  std::uint32_t tiles;
  std::uint32_t output_f16;
};

struct GemvArgs {
  MatrixArg m[4];
  std::uint32_t count;
  const std::int8_t* act;
  const __half* act_scales;
  const std::int32_t* act_sums;
  std::uint32_t columns;
  std::uint32_t groups;
  std::uint32_t batch;
  std::uint32_t act_stride;  // elements between tokens in the activation pack (>= columns)
};

// Locate the matrix a CTA's global tile index belongs to.
__device__ __forceinline__ MatrixArg select_matrix(const GemvArgs& args, std::uint32_t& tile) {
  MatrixArg m = args.m[0];
#pragma unroll
  for (int i = 1; i < 4; ++i) {
    if (static_cast<std::uint32_t>(i) < args.count && tile >= m.tiles) {
      tile -= m.tiles;
      m = args.m[i];
    }
  }
  return m;
}

// One CTA (8 warps) per 16-row tile. Round r: warp w computes the int32 dots
// of group 8r+w with 4 mma per 8-token block, writes them to shared memory;
// then each (row, token) thread extends its fp32 fma chain by the round's
// groups in ascending order. Weights are prefetched two rounds ahead.
template <int Bits, int NB>
__global__ __launch_bounds__(256) void gemv_b200_kernel(const GemvArgs args) {
  pdl_trigger();
  pdl_wait();
  std::uint32_t tile = blockIdx.x;
  const MatrixArg m = select_matrix(args, tile);
  const unsigned warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
  const unsigned gl = lane >> 2, tq = lane & 3u;
  const std::uint32_t G = args.groups, B = args.batch, K = args.columns;
  constexpr std::uint32_t kBlock = Bits * 256u;
  constexpr int kAlpha = Codec<Bits>::alpha, kBeta = Codec<Bits>::beta;
  const std::uint8_t* tile_codes = m.codes + static_cast<std::size_t>(tile) * G * kBlock;
  const __half* tile_scales = m.scales + static_cast<std::size_t>(tile) * G * 16u;

  // one padding word per row: the chain's reads (16 rows x 2 tokens per warp) and the mma lanes' writes
  // (8 rows per warp) then fall into distinct banks instead of 8-16 on one
  __shared__ std::int32_t dots[8][16][NB * 8 + 1];

  const std::uint32_t pairs = 16u * B;
  float accumulator[2] = {0.0f, 0.0f};

  LaneWords<Bits> w_cur{}, w_next{}, w_after{};
  if (warp < G) load_lane(tile_codes + warp * kBlock, lane, w_cur);
  if (warp + 8 < G) load_lane(tile_codes + (warp + 8) * kBlock, lane, w_next);

  const std::uint32_t rounds = (G + 7u) / 8u;
  for (std::uint32_t r = 0; r < rounds; ++r) {
    const std::uint32_t g = 8u * r + warp;
    if (g + 16u < G) load_lane(tile_codes + (g + 16u) * kBlock, lane, w_after);

    // Scales this thread's chain needs for the round, issued early.
    const std::uint32_t round_groups = min(8u, G - 8u * r);
    float scale_product[2][8];
#pragma unroll
    for (int p = 0; p < 2; ++p) {
      const std::uint32_t pair = threadIdx.x + 256u * p;
      if (pair < pairs) {
        const std::uint32_t row = pair & 15u, token = pair >> 4;
#pragma unroll
        for (unsigned w = 0; w < 8; ++w) {
          if (w < round_groups) {
            const std::uint32_t gg = 8u * r + w;
            scale_product[p][w] = __fmul_rn(h2f(tile_scales[gg * 16u + row]),
                                            h2f(args.act_scales[token * (args.act_stride / kGroup) + gg]));
          }
        }
      }
    }

    if (g < G) {
      std::uint32_t a[4][4];
      unpack(w_cur, a);
#pragma unroll
      for (int nb = 0; nb < NB; ++nb) {
        std::uint32_t token = nb * 8u + gl;
        token = token < B ? token : B - 1u;
        const std::int8_t* ap = args.act + static_cast<std::size_t>(token) * args.act_stride +
                                static_cast<std::size_t>(g) * kGroup + tq * 32u;
        const uint4 b0 = __ldg(reinterpret_cast<const uint4*>(ap));
        const uint4 b1 = __ldg(reinterpret_cast<const uint4*>(ap + 16));
        int c[4] = {0, 0, 0, 0};
        mma_s8_16832(c, a[0], b0.x, b0.y);
        mma_s8_16832(c, a[1], b0.z, b0.w);
        mma_s8_16832(c, a[2], b1.x, b1.y);
        mma_s8_16832(c, a[3], b1.z, b1.w);
        const std::uint32_t t0 = nb * 8u + 2u * tq, t1 = t0 + 1u;
        if (t0 < B) {
          const int s0 = args.act_sums[t0 * (args.act_stride / kGroup) + g];
          dots[warp][gl][t0] = kAlpha * c[0] + kBeta * s0;
          dots[warp][gl + 8][t0] = kAlpha * c[2] + kBeta * s0;
        }
        if (t1 < B) {
          const int s1 = args.act_sums[t1 * (args.act_stride / kGroup) + g];
          dots[warp][gl][t1] = kAlpha * c[1] + kBeta * s1;
          dots[warp][gl + 8][t1] = kAlpha * c[3] + kBeta * s1;
        }
      }
    }
    __syncthreads();
#pragma unroll
    for (int p = 0; p < 2; ++p) {
      const std::uint32_t pair = threadIdx.x + 256u * p;
      if (pair < pairs) {
        const std::uint32_t row = pair & 15u, token = pair >> 4;
#pragma unroll
        for (unsigned w = 0; w < 8; ++w) {
          if (w < round_groups) {
            accumulator[p] = fmaf(static_cast<float>(dots[w][row][token]), scale_product[p][w],
                                  accumulator[p]);
          }
        }
      }
    }
    __syncthreads();
    w_cur = w_next;
    w_next = w_after;
  }

  const std::uint32_t rows = m.tiles * 16u;
#pragma unroll
  for (int p = 0; p < 2; ++p) {
    const std::uint32_t pair = threadIdx.x + 256u * p;
    if (pair < pairs) {
      const std::uint32_t row = pair & 15u, token = pair >> 4;
      const std::size_t index = static_cast<std::size_t>(token) * rows + tile * 16u + row;
      if (m.output_f16) {
        static_cast<__half*>(m.output)[index] = f2h(accumulator[p]);
      } else {
        static_cast<float*>(m.output)[index] = accumulator[p];
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Streaming GEMV for batch <= 8 (the decode regime).
//
// A cluster of P CTAs owns one 16-row tile; CTA p owns a contiguous range of
// its 128-column groups. One thread stages the CTA's whole weight range into
// shared memory with bulk copies (one mbarrier per 8 groups), so every byte
// the CTA needs is in flight from the first cycle. Warps turn staged groups
// into exact int32 dots on the tensor cores; the other CTAs send theirs to
// the cluster leader with asynchronous shared-memory stores whose bytes are
// counted on one leader mbarrier, and exit. The leader then runs the
// reference's ordered fp32 chain over all groups of the tile. No cluster
// barrier is needed after the dots: the leader alone waits, and only for the
// bytes it expects.
// ---------------------------------------------------------------------------

__device__ std::uint32_t g_gemv_error;
constexpr std::uint32_t kGemvErrorCluster = 16u;  // cluster size differs from the split the host chose
constexpr std::uint32_t kGemvErrorSmem = 32u;     // shared-memory layout exceeds the launch's dynamic size
constexpr std::uint32_t kGemvErrorTile = 64u;     // CTA maps past the last tile of its matrix

struct StreamLayout {
  std::uint32_t per_part;     // groups per cluster rank
  std::uint32_t weight_bytes;  // per_part * block
  std::uint32_t scale_bytes;   // G * 32
  std::uint32_t dot_bytes;     // G * 16 * B * 4
  std::uint32_t act_scale_bytes;  // G * B * 2, rounded up to 16
  std::uint32_t bar_offset;    // chunk barriers, the scale barrier, the dots barrier
  std::uint32_t total;
};

__host__ __device__ inline StreamLayout stream_layout(int bits, std::uint32_t groups, std::uint32_t parts,
                                                      std::uint32_t batch, std::uint32_t chunk) {
  StreamLayout s{};
  s.per_part = (groups + parts - 1) / parts;
  s.weight_bytes = s.per_part * static_cast<std::uint32_t>(bits) * 256u;
  s.scale_bytes = groups * 32u;
  s.dot_bytes = groups * 16u * batch * 4u;
  s.act_scale_bytes = (groups * batch * 2u + 15u) & ~15u;
  s.bar_offset = (s.weight_bytes + s.scale_bytes + s.dot_bytes + s.act_scale_bytes + 15u) & ~15u;
  const std::uint32_t bars = (s.per_part + chunk - 1u) / chunk + 2u;
  s.total = s.bar_offset + bars * 8u;
  return s;
}

// One: batch 1 (token 0 only: one mma chain, no second-token lanes). Long: the
// leader forms the scale products first (wide K; a separate instantiation so
// that the short-chain one keeps its lower register count and occupancy).
template <int Bits, bool One, bool Long = false>
__global__ __launch_bounds__(256) void gemv_stream_kernel(const GemvArgs args, std::uint32_t parts,
                                                          std::uint32_t chunk) {
  extern __shared__ __align__(128) std::uint8_t smem[];
  pdl_trigger();
  const std::uint32_t part = cluster_ctarank();
  std::uint32_t tile = blockIdx.x / parts;
  const MatrixArg m = select_matrix(args, tile);
  const unsigned warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
  const unsigned gl = lane >> 2, tq = lane & 3u;
  const std::uint32_t G = args.groups, B = args.batch;
  constexpr std::uint32_t kBlock = Bits * 256u;
  constexpr int kAlpha = Codec<Bits>::alpha, kBeta = Codec<Bits>::beta;
  const StreamLayout layout = stream_layout(Bits, G, parts, B, chunk);
  const std::uint32_t g_begin = min(G, part * layout.per_part);
  const std::uint32_t n = min(G, g_begin + layout.per_part) - g_begin;
  const std::uint32_t chunks = (n + chunk - 1u) / chunk;
  const std::uint32_t chunk_shift = static_cast<std::uint32_t>(__ffs(static_cast<int>(chunk)) - 1);  // chunk: a power of two

  std::uint8_t* stage = smem;
  __half* tile_scales = reinterpret_cast<__half*>(smem + layout.weight_bytes);
  std::int32_t* dots = reinterpret_cast<std::int32_t*>(smem + layout.weight_bytes + layout.scale_bytes);
  __half* act_scale_stage =
      reinterpret_cast<__half*>(smem + layout.weight_bytes + layout.scale_bytes + layout.dot_bytes);
  std::uint64_t* bars = reinterpret_cast<std::uint64_t*>(smem + layout.bar_offset);
  const std::uint32_t max_chunks = (layout.per_part + chunk - 1u) / chunk;
  const std::uint32_t scale_bar = max_chunks, dots_bar = max_chunks + 1u;

  // Self-check of the launch geometry: every CTA of the grid sees the same
  // values, so all of them return together, before any barrier or copy.
  {
    std::uint32_t bad = 0;
    if (cluster_nctarank() != parts || part >= parts) bad |= kGemvErrorCluster;
    if (layout.total > dynamic_smem_bytes()) bad |= kGemvErrorSmem;
    if (tile >= m.tiles) bad |= kGemvErrorTile;
    if (bad != 0) {
      if (threadIdx.x == 0) atomicOr(&g_gemv_error, bad);
      return;
    }
  }

  if (threadIdx.x == 0) {
    for (std::uint32_t c = 0; c <= dots_bar; ++c) mbar_init(&bars[c], 1);
    fence_mbar_init();
    const std::uint8_t* source = m.codes + (static_cast<std::size_t>(tile) * G + g_begin) * kBlock;
    for (std::uint32_t c = 0; c < chunks; ++c) {
      const std::uint32_t bytes = min(chunk, n - chunk * c) * kBlock;
      mbar_expect_tx(&bars[c], bytes);
      bulk_g2s(stage + chunk * c * kBlock, source + chunk * c * kBlock, bytes, &bars[c]);
    }
    if (part == 0) {
      mbar_expect_tx(&bars[scale_bar], layout.scale_bytes);
      bulk_g2s(tile_scales, m.scales + static_cast<std::size_t>(tile) * G * 16u, layout.scale_bytes,
               &bars[scale_bar]);
      // the other ranks' dots: (G - own groups) x 16 rows x B tokens x 4 bytes
      if (parts > 1u) mbar_expect_tx(&bars[dots_bar], (G - n) * 16u * B * 4u);
    }
  }

  // Every CTA of the cluster announces it is running with its barriers
  // initialised; the wait below (before the first store into the leader's
  // shared memory) completes this phase.
  cluster_arrive_relaxed();
  // Weights and their scales never depend on the previous kernel; the
  // activation pack does.
  pdl_wait();
  if (part == 0) {
    const std::uint32_t act_groups = args.act_stride / kGroup;
    for (std::uint32_t i = threadIdx.x; i < G * B; i += blockDim.x) {
      const std::uint32_t tok = i / G, g = i - tok * G;
      act_scale_stage[i] = args.act_scales[static_cast<std::size_t>(tok) * act_groups + g];
    }
  }
  const std::uint32_t leader_dots = map_shared_rank(smem_addr(dots), 0);
  const std::uint32_t leader_bar = map_shared_rank(smem_addr(&bars[dots_bar]), 0);
  const std::uint32_t token = min(gl, B - 1u);
  cluster_wait();
  // stores dot (row, tok) of group g: locally in the leader, asynchronously elsewhere
  auto put = [&](std::uint32_t g, std::uint32_t row, std::uint32_t tok, int value) {
    const std::uint32_t index = (g * 16u + row) * B + tok;
    if (part == 0) {
      dots[index] = value;
    } else {
      st_async_s32(leader_dots + index * 4u, value, leader_bar);
    }
  };
  if constexpr (One) {
    // token 0 only: lanes with tq = 0 hold its column of the mma; the four
    // k-steps accumulate in one chain (exact integer sums, the same dot)
    for (std::uint32_t local = warp; local < n; local += 8u) {
      const std::uint32_t g = g_begin + local;
      const std::int8_t* ap = args.act + static_cast<std::size_t>(g) * kGroup + tq * 32u;
      const uint4 b0 = __ldg(reinterpret_cast<const uint4*>(ap));
      const uint4 b1 = __ldg(reinterpret_cast<const uint4*>(ap + 16));
      const int beta_sum = tq == 0 ? kBeta * __ldg(args.act_sums + g) : 0;
      if (!mbar_wait_bounded(&bars[local >> chunk_shift], 0, &g_gemv_error)) break;
      LaneWords<Bits> w;
      load_lane_shared<Bits>(stage + local * kBlock, lane, w);
      std::uint32_t a[4][4];
      unpack(w, a);
      int c[4];
      mma_s8_16832_zero(c, a[0], b0.x, b0.y);
      mma_s8_16832(c, a[1], b0.z, b0.w);
      mma_s8_16832(c, a[2], b1.x, b1.y);
      mma_s8_16832(c, a[3], b1.z, b1.w);
      if (tq == 0) {
        put(g, gl, 0, kAlpha * c[0] + beta_sum);
        put(g, gl + 8u, 0, kAlpha * c[2] + beta_sum);
      }
    }
  }
  for (std::uint32_t local = warp; !One && local < n; local += 8u) {
    const std::uint32_t g = g_begin + local;
    const std::int8_t* ap = args.act + static_cast<std::size_t>(token) * args.act_stride +
                            static_cast<std::size_t>(g) * kGroup + tq * 32u;
    const uint4 b0 = __ldg(reinterpret_cast<const uint4*>(ap));
    const uint4 b1 = __ldg(reinterpret_cast<const uint4*>(ap + 16));
    const std::uint32_t t0 = 2u * tq, t1 = t0 + 1u;
    const std::uint32_t act_groups = args.act_stride / kGroup;
    const int s0 = t0 < B ? __ldg(args.act_sums + t0 * act_groups + g) : 0;
    const int s1 = t1 < B ? __ldg(args.act_sums + t1 * act_groups + g) : 0;
    if (!mbar_wait_bounded(&bars[local >> chunk_shift], 0, &g_gemv_error)) break;
    LaneWords<Bits> w;
    load_lane_shared<Bits>(stage + local * kBlock, lane, w);
    std::uint32_t a[4][4];
    unpack(w, a);
    int c0[4] = {0, 0, 0, 0}, c1[4] = {0, 0, 0, 0};
    mma_s8_16832(c0, a[0], b0.x, b0.y);
    mma_s8_16832(c1, a[1], b0.z, b0.w);
    mma_s8_16832(c0, a[2], b1.x, b1.y);
    mma_s8_16832(c1, a[3], b1.z, b1.w);
    if (t0 < B) {
      put(g, gl, t0, kAlpha * (c0[0] + c1[0]) + kBeta * s0);
      put(g, gl + 8u, t0, kAlpha * (c0[2] + c1[2]) + kBeta * s0);
    }
    if (t1 < B) {
      put(g, gl, t1, kAlpha * (c0[1] + c1[1]) + kBeta * s1);
      put(g, gl + 8u, t1, kAlpha * (c0[3] + c1[3]) + kBeta * s1);
    }
  }
  if (part != 0) return;
  __syncthreads();  // the leader's own dots and staged activation scales
  if constexpr (One && Long) {
    // Long chains (wide K): the whole CTA forms the tile's scale products
    // (weight scale x activation scale, the chain's multiplier) in the consumed
    // weight stage while the peers' dots arrive; the 16 chain threads then only
    // load and fma.
    float* products = reinterpret_cast<float*>(stage);
    const bool scales_ready = mbar_wait_bounded(&bars[scale_bar], 0, &g_gemv_error);
    if (scales_ready) {
      for (std::uint32_t i = threadIdx.x; i < G * 16u; i += blockDim.x) {
        products[i] = __fmul_rn(h2f(tile_scales[i]), h2f(act_scale_stage[i >> 4]));
      }
    }
    __syncthreads();
    if (threadIdx.x >= 16u || !scales_ready) return;
    if (parts > 1u) {
      bool arrived = false;  // outlast every peer's bounded waits, as below
      for (std::uint32_t r = 0; r < max_chunks + 2u && !arrived; ++r) {
        for (std::uint32_t i = 0; i < kWaitLimit && !arrived; ++i) arrived = mbar_try_wait_cluster(&bars[dots_bar], 0);
      }
      if (!arrived) {
        atomicOr(&g_gemv_error, kDeviceErrorTimeout);
        return;
      }
    }
    const std::uint32_t row = threadIdx.x;
    float accumulator = 0.0f;
    std::uint32_t g = 0;
    // the next eight groups' operands load while the current eight fma
    float product[8];
    int dot[8];
#pragma unroll
    for (unsigned i = 0; i < 8; ++i) {
      const std::uint32_t gi = min(i, G - 1u);
      product[i] = products[gi * 16u + row];
      dot[i] = dots[gi * 16u + row];
    }
    for (; g + 8u <= G; g += 8u) {
      float next_product[8];
      int next_dot[8];
#pragma unroll
      for (unsigned i = 0; i < 8; ++i) {
        const std::uint32_t gi = min(g + 8u + i, G - 1u);
        next_product[i] = products[gi * 16u + row];
        next_dot[i] = dots[gi * 16u + row];
      }
#pragma unroll
      for (unsigned i = 0; i < 8; ++i) accumulator = fmaf(static_cast<float>(dot[i]), product[i], accumulator);
#pragma unroll
      for (unsigned i = 0; i < 8; ++i) {
        product[i] = next_product[i];
        dot[i] = next_dot[i];
      }
    }
#pragma unroll
    for (unsigned i = 0; i < 8; ++i) {
      if (g + i < G) accumulator = fmaf(static_cast<float>(dot[i]), product[i], accumulator);
    }
    const std::size_t index = static_cast<std::size_t>(tile) * 16u + row;
    if (m.output_f16) {
      static_cast<__half*>(m.output)[index] = f2h(accumulator);
    } else {
      static_cast<float*>(m.output)[index] = accumulator;
    }
    return;
  }
  const std::uint32_t pairs = 16u * B;
  if (threadIdx.x >= pairs) return;
  if (!mbar_wait_bounded(&bars[scale_bar], 0, &g_gemv_error)) return;
  if (parts > 1u) {
    // Outlast every peer's own bounded waits (at most max_chunks of them), so
    // that no peer can still be storing when this CTA exits.
    bool arrived = false;
    for (std::uint32_t r = 0; r < max_chunks + 2u && !arrived; ++r) {
      for (std::uint32_t i = 0; i < kWaitLimit && !arrived; ++i) arrived = mbar_try_wait_cluster(&bars[dots_bar], 0);
    }
    if (!arrived) {
      atomicOr(&g_gemv_error, kDeviceErrorTimeout);
      return;
    }
  }
  const std::uint32_t row = threadIdx.x & 15u, tok = threadIdx.x >> 4;
  const __half* act_scales = act_scale_stage + static_cast<std::size_t>(tok) * G;
  float accumulator = 0.0f;
  std::uint32_t g = 0;
  for (; g + 8u <= G; g += 8u) {
    float product[8];
    int dot[8];
#pragma unroll
    for (unsigned i = 0; i < 8; ++i) {
      product[i] = __fmul_rn(h2f(tile_scales[(g + i) * 16u + row]), h2f(act_scales[g + i]));
      dot[i] = dots[((g + i) * 16u + row) * B + tok];
    }
#pragma unroll
    for (unsigned i = 0; i < 8; ++i) accumulator = fmaf(static_cast<float>(dot[i]), product[i], accumulator);
  }
  for (; g < G; ++g) {
    const float product = __fmul_rn(h2f(tile_scales[g * 16u + row]), h2f(act_scales[g]));
    accumulator = fmaf(static_cast<float>(dots[(g * 16u + row) * B + tok]), product, accumulator);
  }
  const std::size_t index = static_cast<std::size_t>(tok) * (m.tiles * 16u) + tile * 16u + row;
  if (m.output_f16) {
    static_cast<__half*>(m.output)[index] = f2h(accumulator);
  } else {
    static_cast<float*>(m.output)[index] = accumulator;
  }
}

// ---------------------------------------------------------------------------
// Cascaded split-K GEMV for 2 <= batch <= 16 (the causal verifier's widths).
//
// Same split as gemv_stream_kernel (a cluster of P CTAs per 16-row tile, CTA p
// owns a contiguous range of the tile's groups), but no CTA gathers the whole
// tile's dots, whose buffer grows with the batch (70 KB at 136 groups x 8
// tokens) and would cut the CTAs per SM. CTA p keeps the dots of its own
// groups, and its 16 x B chain threads run their segment of the ordered fp32
// chain: CTA 0 starts it at zero, CTA p > 0 starts from the accumulators CTA
// p - 1 sends with st.async (bytes counted on this CTA's mbarrier) and sends
// its own on; the last CTA writes the outputs. The fma sequence per (row,
// token) is the one over all groups in ascending order, hence identical bits.
// ---------------------------------------------------------------------------

struct CascadeLayout {
  std::uint32_t per_part;      // groups per cluster rank
  std::uint32_t weight_bytes;  // per_part * block
  std::uint32_t scale_offset;  // own groups' scales [per_part][16] fp16
  std::uint32_t dot_offset;    // own groups' dots [per_part][16][B] int32
  std::uint32_t act_offset;    // own groups' activation scales [B][per_part] fp16
  std::uint32_t acc_offset;    // incoming accumulators [16 * B] fp32
  std::uint32_t bar_offset;    // chunk barriers, the scale barrier, the accumulator barrier
  std::uint32_t total;
};

__host__ __device__ inline CascadeLayout cascade_layout(int bits, std::uint32_t groups, std::uint32_t parts,
                                                        std::uint32_t batch, std::uint32_t chunk) {
  CascadeLayout l{};
  l.per_part = (groups + parts - 1u) / parts;
  l.weight_bytes = l.per_part * static_cast<std::uint32_t>(bits) * 256u;
  l.scale_offset = l.weight_bytes;
  l.dot_offset = l.scale_offset + ((l.per_part * 32u + 15u) & ~15u);
  l.act_offset = l.dot_offset + l.per_part * 16u * batch * 4u;
  l.acc_offset = (l.act_offset + l.per_part * batch * 2u + 15u) & ~15u;
  l.bar_offset = (l.acc_offset + 16u * batch * 4u + 15u) & ~15u;
  const std::uint32_t bars = (l.per_part + chunk - 1u) / chunk + 2u;
  l.total = l.bar_offset + bars * 8u;
  return l;
}

template <int Bits, int NB>  // NB blocks of 8 tokens
__global__ __launch_bounds__(256) void gemv_cascade_kernel(const GemvArgs args, std::uint32_t parts,
                                                           std::uint32_t chunk) {
  extern __shared__ __align__(128) std::uint8_t smem[];
  pdl_trigger();
  const std::uint32_t part = cluster_ctarank();
  std::uint32_t tile = blockIdx.x / parts;
  const MatrixArg m = select_matrix(args, tile);
  const unsigned warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
  const unsigned gl = lane >> 2, tq = lane & 3u;
  const std::uint32_t G = args.groups, B = args.batch;
  constexpr std::uint32_t kBlock = Bits * 256u;
  constexpr int kAlpha = Codec<Bits>::alpha, kBeta = Codec<Bits>::beta;
  const CascadeLayout layout = cascade_layout(Bits, G, parts, B, chunk);
  const std::uint32_t g_begin = min(G, part * layout.per_part);
  const std::uint32_t n = min(G, g_begin + layout.per_part) - g_begin;
  const std::uint32_t chunks = (n + chunk - 1u) / chunk;
  const std::uint32_t chunk_shift = static_cast<std::uint32_t>(__ffs(static_cast<int>(chunk)) - 1);  // chunk: a power of two
  const std::uint32_t max_chunks = (layout.per_part + chunk - 1u) / chunk;
  std::uint8_t* stage = smem;
  __half* own_scales = reinterpret_cast<__half*>(smem + layout.scale_offset);
  std::int32_t* dots = reinterpret_cast<std::int32_t*>(smem + layout.dot_offset);
  __half* act_scale_stage = reinterpret_cast<__half*>(smem + layout.act_offset);
  float* acc_in = reinterpret_cast<float*>(smem + layout.acc_offset);
  std::uint64_t* bars = reinterpret_cast<std::uint64_t*>(smem + layout.bar_offset);
  const std::uint32_t scale_bar = max_chunks, acc_bar = max_chunks + 1u;

  // Self-check of the launch geometry (uniform over the cluster: all return together).
  {
    std::uint32_t bad = 0;
    if (cluster_nctarank() != parts || part >= parts || B < 1u || (B + 7u) / 8u != NB) bad |= kGemvErrorCluster;
    if (layout.total > dynamic_smem_bytes()) bad |= kGemvErrorSmem;
    if (tile >= m.tiles) bad |= kGemvErrorTile;
    if (bad != 0) {
      if (threadIdx.x == 0) atomicOr(&g_gemv_error, bad);
      return;
    }
  }

  if (threadIdx.x == 0) {
    for (std::uint32_t c = 0; c <= acc_bar; ++c) mbar_init(&bars[c], 1);
    fence_mbar_init();
    const std::uint8_t* source = m.codes + (static_cast<std::size_t>(tile) * G + g_begin) * kBlock;
    for (std::uint32_t c = 0; c < chunks; ++c) {
      const std::uint32_t bytes = min(chunk, n - chunk * c) * kBlock;
      mbar_expect_tx(&bars[c], bytes);
      bulk_g2s(stage + chunk * c * kBlock, source + chunk * c * kBlock, bytes, &bars[c]);
    }
    if (n != 0u) {
      mbar_expect_tx(&bars[scale_bar], n * 32u);
      bulk_g2s(own_scales, m.scales + (static_cast<std::size_t>(tile) * G + g_begin) * 16u, n * 32u,
               &bars[scale_bar]);
    }
    // the previous rank's accumulators: 16 rows x B tokens x 4 bytes
    if (part > 0u) mbar_expect_tx(&bars[acc_bar], 16u * B * 4u);
  }
  // every CTA of the cluster is running with its barriers initialised before
  // the first store into another CTA's shared memory (the wait below)
  cluster_arrive_relaxed();
  pdl_wait();
  const std::uint32_t act_groups = args.act_stride / kGroup;
  for (std::uint32_t i = threadIdx.x; i < n * B; i += blockDim.x) {
    const std::uint32_t tok = i / n, local = i - tok * n;
    act_scale_stage[i] = args.act_scales[static_cast<std::size_t>(tok) * act_groups + g_begin + local];
  }
  const std::uint32_t next_acc = map_shared_rank(smem_addr(acc_in), part + 1u < parts ? part + 1u : part);
  const std::uint32_t next_bar = map_shared_rank(smem_addr(&bars[acc_bar]), part + 1u < parts ? part + 1u : part);
  cluster_wait();
  bool ok = true;
  for (std::uint32_t local = warp; local < n; local += 8u) {
    const std::uint32_t g = g_begin + local;
    if (!mbar_wait_bounded(&bars[local >> chunk_shift], 0, &g_gemv_error)) {
      ok = false;
      break;
    }
    LaneWords<Bits> w;
    load_lane_shared<Bits>(stage + local * kBlock, lane, w);
    std::uint32_t a[4][4];
    unpack(w, a);
    const std::uint32_t row_base = local * 16u;
    // tokens in blocks of 8 (the mma's N), the unpacked weights reused
#pragma unroll
    for (std::uint32_t tb = 0; tb < 8u * NB; tb += 8u) {
      const std::uint32_t token = min(tb + gl, B - 1u);
      const std::int8_t* ap = args.act + static_cast<std::size_t>(token) * args.act_stride +
                              static_cast<std::size_t>(g) * kGroup + tq * 32u;
      const uint4 b0 = __ldg(reinterpret_cast<const uint4*>(ap));
      const uint4 b1 = __ldg(reinterpret_cast<const uint4*>(ap + 16));
      const std::uint32_t t0 = tb + 2u * tq, t1 = t0 + 1u;
      const int s0 = t0 < B ? __ldg(args.act_sums + t0 * act_groups + g) : 0;
      const int s1 = t1 < B ? __ldg(args.act_sums + t1 * act_groups + g) : 0;
      int c0[4] = {0, 0, 0, 0}, c1[4] = {0, 0, 0, 0};
      mma_s8_16832(c0, a[0], b0.x, b0.y);
      mma_s8_16832(c1, a[1], b0.z, b0.w);
      mma_s8_16832(c0, a[2], b1.x, b1.y);
      mma_s8_16832(c1, a[3], b1.z, b1.w);
      if (t0 < B) {
        dots[(row_base + gl) * B + t0] = kAlpha * (c0[0] + c1[0]) + kBeta * s0;
        dots[(row_base + gl + 8u) * B + t0] = kAlpha * (c0[2] + c1[2]) + kBeta * s0;
      }
      if (t1 < B) {
        dots[(row_base + gl) * B + t1] = kAlpha * (c0[1] + c1[1]) + kBeta * s1;
        dots[(row_base + gl + 8u) * B + t1] = kAlpha * (c0[3] + c1[3]) + kBeta * s1;
      }
    }
  }
  ok = __syncthreads_and(ok);  // also publishes the dots and the staged activation scales
  if (threadIdx.x >= 16u * B) return;
  const std::uint32_t row = threadIdx.x & 15u, tok = threadIdx.x >> 4;
  if (ok && n != 0u && !mbar_wait_bounded(&bars[scale_bar], 0, &g_gemv_error)) ok = false;
  float accumulator = 0.0f;
  if (part > 0u) {
    // Outlast the bounded waits of every earlier rank (their copies and their
    // own accumulator waits, each longer than the one before), so that none
    // can still be sending when this CTA exits.
    bool arrived = false;
    for (std::uint32_t r = 0; r < (max_chunks + 3u) * (part + 1u) && !arrived; ++r) {
      for (std::uint32_t i = 0; i < kWaitLimit && !arrived; ++i) arrived = mbar_try_wait_cluster(&bars[acc_bar], 0);
    }
    if (!arrived) {
      atomicOr(&g_gemv_error, kDeviceErrorTimeout);
      return;
    }
    accumulator = acc_in[threadIdx.x];
  }
  if (ok) {
    const __half* as = act_scale_stage + static_cast<std::size_t>(tok) * n;
    for (std::uint32_t local = 0; local < n; ++local) {
      const float product = __fmul_rn(h2f(own_scales[local * 16u + row]), h2f(as[local]));
      accumulator = fmaf(static_cast<float>(dots[(local * 16u + row) * B + tok]), product, accumulator);
    }
  }
  if (part + 1u < parts) {
    // the next rank continues the chain (sent even after a failed wait, so that it does not stall)
    st_async_s32(next_acc + threadIdx.x * 4u, __float_as_int(accumulator), next_bar);
    return;
  }
  if (!ok) return;
  const std::size_t index = static_cast<std::size_t>(tok) * (m.tiles * 16u) + tile * 16u + row;
  if (m.output_f16) {
    static_cast<__half*>(m.output)[index] = f2h(accumulator);
  } else {
    static_cast<float*>(m.output)[index] = accumulator;
  }
}

// ---------------------------------------------------------------------------
// Pipelined multi-tile GEMV for batch <= 8 and tall matrices.
//
// A grid of a few CTAs per SM; CTA c handles tiles c, c + grid, c + 2 grid,
// ... with two shared-memory stages: while the warps turn one tile's staged
// groups into int32 dots and the fp32 chain runs, the next tile's codes and
// scales are already landing (one bulk copy each, mbarrier completion). Every
// CTA is resident from the start, so there is no second wave and no tail of
// CTAs that only start when others exit; the weights stream continuously.
// Arithmetic as gemv_stream_kernel (per-group int32 dots, the ordered fp32
// chain per row), hence identical bits.
// ---------------------------------------------------------------------------

struct PipeLayout {
  std::uint32_t weight_bytes;  // G * block
  std::uint32_t scale_bytes;   // G * 32
  std::uint32_t dot_bytes;     // G * 16 * B * 4
  std::uint32_t stage_bytes;   // the three, 128-byte aligned
  std::uint32_t act_offset;    // fp16 activation scales [B][G]
  std::uint32_t pair_offset;   // one token: (float(dot), scale product) of the tile being chained [G][16]
  std::uint32_t bar_offset;
  std::uint32_t total;
};

constexpr std::uint32_t kPipeStages = 2;

__host__ __device__ inline PipeLayout pipe_layout(int bits, std::uint32_t groups, std::uint32_t batch) {
  PipeLayout l{};
  l.weight_bytes = groups * static_cast<std::uint32_t>(bits) * 256u;
  l.scale_bytes = groups * 32u;
  l.dot_bytes = groups * 16u * batch * 4u;
  l.stage_bytes = (l.weight_bytes + l.scale_bytes + l.dot_bytes + 127u) & ~127u;
  l.act_offset = kPipeStages * l.stage_bytes;
  l.pair_offset = (l.act_offset + groups * batch * 2u + 15u) & ~15u;
  l.bar_offset = l.pair_offset + (batch == 1u ? groups * 16u * 8u : 0u);
  l.total = l.bar_offset + kPipeStages * 8u;
  return l;
}

template <int Bits, bool One>  // One: batch 1 (token 0 only: one mma chain, no second-token lanes)
__global__ __launch_bounds__(256) void gemv_pipe_kernel(const GemvArgs args, std::uint32_t total_tiles) {
  extern __shared__ __align__(128) std::uint8_t smem[];
  pdl_trigger();
  const unsigned warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
  const unsigned gl = lane >> 2, tq = lane & 3u;
  const std::uint32_t G = args.groups, B = args.batch;
  constexpr std::uint32_t kBlock = Bits * 256u;
  constexpr int kAlpha = Codec<Bits>::alpha, kBeta = Codec<Bits>::beta;
  const PipeLayout layout = pipe_layout(Bits, G, B);
  const std::uint32_t count = blockIdx.x < total_tiles ? (total_tiles - blockIdx.x + gridDim.x - 1u) / gridDim.x : 0u;
  if (layout.total > dynamic_smem_bytes()) {
    if (threadIdx.x == 0) atomicOr(&g_gemv_error, kGemvErrorSmem);
    return;
  }
  std::uint64_t* bars = reinterpret_cast<std::uint64_t*>(smem + layout.bar_offset);
  __half* act_scales = reinterpret_cast<__half*>(smem + layout.act_offset);
  auto stage_base = [&](std::uint32_t stage) { return smem + stage * layout.stage_bytes; };
  // one thread stages tile i's codes and scales into stage i % 2
  auto issue = [&](std::uint32_t i) {
    std::uint32_t tile = blockIdx.x + i * gridDim.x;
    const MatrixArg m = select_matrix(args, tile);
    std::uint8_t* base = stage_base(i % kPipeStages);
    std::uint64_t* bar = &bars[i % kPipeStages];
    mbar_expect_tx(bar, layout.weight_bytes + layout.scale_bytes);
    bulk_g2s(base, m.codes + static_cast<std::size_t>(tile) * G * kBlock, layout.weight_bytes, bar);
    bulk_g2s(base + layout.weight_bytes, m.scales + static_cast<std::size_t>(tile) * G * 16u, layout.scale_bytes, bar);
  };
  if (threadIdx.x == 0) {
    for (std::uint32_t s = 0; s < kPipeStages; ++s) mbar_init(&bars[s], 1);
    fence_mbar_init();
    for (std::uint32_t i = 0; i < kPipeStages && i < count; ++i) issue(i);
  }
  // weights never depend on the previous kernel; the activation pack does
  pdl_wait();
  const std::uint32_t act_groups = args.act_stride / kGroup;
  for (std::uint32_t i = threadIdx.x; i < G * B; i += blockDim.x) {
    const std::uint32_t tok = i / G, g = i - tok * G;
    act_scales[i] = args.act_scales[static_cast<std::size_t>(tok) * act_groups + g];
  }
  __syncthreads();
  const std::uint32_t token = min(gl, B - 1u);
  for (std::uint32_t i = 0; i < count; ++i) {
    const std::uint32_t stage = i % kPipeStages;
    std::uint32_t tile = blockIdx.x + i * gridDim.x;
    const MatrixArg m = select_matrix(args, tile);
    std::uint8_t* base = stage_base(stage);
    const __half* tile_scales = reinterpret_cast<const __half*>(base + layout.weight_bytes);
    std::int32_t* dots = reinterpret_cast<std::int32_t*>(base + layout.weight_bytes + layout.scale_bytes);
    const bool ready = mbar_wait_bounded(&bars[stage], (i / kPipeStages) & 1u, &g_gemv_error);
    if (ready && One) {
      for (std::uint32_t g = warp; g < G; g += 8u) {
        const std::int8_t* ap = args.act + static_cast<std::size_t>(g) * kGroup + tq * 32u;
        const uint4 b0 = __ldg(reinterpret_cast<const uint4*>(ap));
        const uint4 b1 = __ldg(reinterpret_cast<const uint4*>(ap + 16));
        const int beta_sum = tq == 0 ? kBeta * __ldg(args.act_sums + g) : 0;
        LaneWords<Bits> w;
        load_lane_shared<Bits>(base + g * kBlock, lane, w);
        std::uint32_t a[4][4];
        unpack(w, a);
        int c[4];
        mma_s8_16832_zero(c, a[0], b0.x, b0.y);
        mma_s8_16832(c, a[1], b0.z, b0.w);
        mma_s8_16832(c, a[2], b1.x, b1.y);
        mma_s8_16832(c, a[3], b1.z, b1.w);
        if (tq == 0) {
          dots[g * 16u + gl] = kAlpha * c[0] + beta_sum;
          dots[g * 16u + gl + 8u] = kAlpha * c[2] + beta_sum;
        }
      }
    } else if (ready) {
      for (std::uint32_t g = warp; g < G; g += 8u) {
        const std::int8_t* ap = args.act + static_cast<std::size_t>(token) * args.act_stride +
                                static_cast<std::size_t>(g) * kGroup + tq * 32u;
        const uint4 b0 = __ldg(reinterpret_cast<const uint4*>(ap));
        const uint4 b1 = __ldg(reinterpret_cast<const uint4*>(ap + 16));
        const std::uint32_t t0 = 2u * tq, t1 = t0 + 1u;
        const int s0 = t0 < B ? __ldg(args.act_sums + t0 * act_groups + g) : 0;
        const int s1 = t1 < B ? __ldg(args.act_sums + t1 * act_groups + g) : 0;
        LaneWords<Bits> w;
        load_lane_shared<Bits>(base + g * kBlock, lane, w);
        std::uint32_t a[4][4];
        unpack(w, a);
        int c0[4] = {0, 0, 0, 0}, c1[4] = {0, 0, 0, 0};
        mma_s8_16832(c0, a[0], b0.x, b0.y);
        mma_s8_16832(c1, a[1], b0.z, b0.w);
        mma_s8_16832(c0, a[2], b1.x, b1.y);
        mma_s8_16832(c1, a[3], b1.z, b1.w);
        const std::uint32_t row_base = g * 16u;
        if (t0 < B) {
          dots[(row_base + gl) * B + t0] = kAlpha * (c0[0] + c1[0]) + kBeta * s0;
          dots[(row_base + gl + 8u) * B + t0] = kAlpha * (c0[2] + c1[2]) + kBeta * s0;
        }
        if (t1 < B) {
          dots[(row_base + gl) * B + t1] = kAlpha * (c0[1] + c1[1]) + kBeta * s1;
          dots[(row_base + gl + 8u) * B + t1] = kAlpha * (c0[3] + c1[3]) + kBeta * s1;
        }
      }
    }
    __syncthreads();
    if constexpr (One) {
      // every thread forms (float(dot), scale product) pairs of the tile, so that the 16 chain threads only load
      // and fma: the same conversions and products as the chain below, in parallel
      float2* pairs = reinterpret_cast<float2*>(smem + layout.pair_offset);
      if (ready) {
        for (std::uint32_t idx = threadIdx.x; idx < G * 16u; idx += blockDim.x) {
          pairs[idx] = make_float2(static_cast<float>(dots[idx]),
                                   __fmul_rn(h2f(tile_scales[idx]), h2f(act_scales[idx >> 4])));
        }
      }
      __syncthreads();
      if (ready && threadIdx.x < 16u) {
        const std::uint32_t row = threadIdx.x;
        float accumulator = 0.0f;
#pragma unroll 8
        for (std::uint32_t g = 0; g < G; ++g) {
          const float2 pair = pairs[g * 16u + row];
          accumulator = fmaf(pair.x, pair.y, accumulator);
        }
        const std::size_t index = static_cast<std::size_t>(tile) * 16u + row;
        if (m.output_f16) {
          static_cast<__half*>(m.output)[index] = f2h(accumulator);
        } else {
          static_cast<float*>(m.output)[index] = accumulator;
        }
      }
    }
    if (!One && ready && threadIdx.x < 16u * B) {
      const std::uint32_t row = threadIdx.x & 15u, tok = threadIdx.x >> 4;
      const __half* as = act_scales + static_cast<std::size_t>(tok) * G;
      float accumulator = 0.0f;
      std::uint32_t g = 0;
      for (; g + 8u <= G; g += 8u) {
        float product[8];
        int dot[8];
#pragma unroll
        for (unsigned k = 0; k < 8; ++k) {
          product[k] = __fmul_rn(h2f(tile_scales[(g + k) * 16u + row]), h2f(as[g + k]));
          dot[k] = dots[((g + k) * 16u + row) * B + tok];
        }
#pragma unroll
        for (unsigned k = 0; k < 8; ++k) accumulator = fmaf(static_cast<float>(dot[k]), product[k], accumulator);
      }
      for (; g < G; ++g) {
        const float product = __fmul_rn(h2f(tile_scales[g * 16u + row]), h2f(as[g]));
        accumulator = fmaf(static_cast<float>(dots[(g * 16u + row) * B + tok]), product, accumulator);
      }
      const std::size_t index = static_cast<std::size_t>(tok) * (m.tiles * 16u) + tile * 16u + row;
      if (m.output_f16) {
        static_cast<__half*>(m.output)[index] = f2h(accumulator);
      } else {
        static_cast<float*>(m.output)[index] = accumulator;
      }
    }
    __syncthreads();  // the stage's codes, scales and dots are free again
    if (threadIdx.x == 0 && i + kPipeStages < count) issue(i + kPipeStages);
  }
  // no copy may still be landing when the CTA exits (only after a failed wait)
  if (threadIdx.x == 0) {
    for (std::uint32_t i = count > kPipeStages ? count - kPipeStages : 0u; i < count; ++i) {
      mbar_wait_bounded(&bars[i % kPipeStages], (i / kPipeStages) & 1u, nullptr);
    }
  }
}

// ---------------------------------------------------------------------------
// Warp-specialised persistent GEMV for one token (the decode regime).
//
// A cluster of P CTAs walks the tiles c, c + C, c + 2C, ... (C resident
// clusters); CTA p owns the 128-column groups [p n, p n + n) of every tile.
// In each CTA:
//  - one producer lane streams the CTA's share of each tile's codes through a
//    ring of S stages (full / empty mbarriers), starting before the previous
//    kernel has finished;
//  - eight compute warps (warp w takes the stage's groups w, w + 8, ...) turn
//    the staged codes into exact int32 group dots against the activation
//    codes and group sums, which were staged once in shared memory, and put
//    the dots of token 0 into the cluster leader's dot buffer of the tile:
//    locally, or by st.async whose bytes count on the leader's dots-full
//    mbarrier;
//  - in the leader two chain warps (even and odd tiles) run the reference's
//    ordered fp32 chain over the tile's groups as soon as its dots are
//    complete, write the 16 outputs, fetch the scales of the tile D ahead into
//    the freed slot and hand the dot buffer back to every CTA of the cluster
//    (a local and P - 1 remote mbarrier arrivals).
// No warp waits at a CTA barrier inside the loop. The per-group dots and the
// chain are those of the other GEMV kernels, so every bit is the same.
// ---------------------------------------------------------------------------

constexpr std::uint32_t kLeanComputeWarps = 8;
constexpr std::uint32_t kLeanChainWarps = 2;
constexpr std::uint32_t kLeanThreads = (kLeanComputeWarps + 1u + kLeanChainWarps) * 32u;
constexpr std::uint32_t kLeanSlots = 3;  // dot buffers / scale slots of the leader
constexpr std::uint32_t kLeanMaxStages = 8;

struct LeanLayout {
  std::uint32_t per_part;     // groups per CTA
  std::uint32_t stage_bytes;  // per_part * block, 128-aligned
  std::uint32_t stages;
  std::uint32_t dots_offset;  // [slots][G][16] int32
  std::uint32_t scales_offset;  // [slots][G][16] fp16
  std::uint32_t act_offset;   // [per_part][128] int8 activation codes
  std::uint32_t beta_offset;  // [per_part] int32: beta * group code sum
  std::uint32_t ascale_offset;  // [G] float activation scales
  std::uint32_t bar_offset;   // full[S], empty[S], dots_full[D], dots_free[D], scale_full[D]
  std::uint32_t total;
};

__host__ __device__ inline LeanLayout lean_layout(int bits, std::uint32_t groups, std::uint32_t parts,
                                                  std::uint32_t stages) {
  LeanLayout l{};
  l.per_part = (groups + parts - 1u) / parts;
  l.stage_bytes = (l.per_part * static_cast<std::uint32_t>(bits) * 256u + 127u) & ~127u;
  l.stages = stages;
  l.dots_offset = stages * l.stage_bytes;
  l.scales_offset = l.dots_offset + kLeanSlots * groups * 64u;
  l.act_offset = (l.scales_offset + kLeanSlots * groups * 32u + 15u) & ~15u;
  l.beta_offset = l.act_offset + l.per_part * kGroup;
  l.ascale_offset = l.beta_offset + l.per_part * 4u;
  l.bar_offset = (l.ascale_offset + groups * 4u + 7u) & ~7u;
  l.total = l.bar_offset + (2u * stages + 3u * kLeanSlots) * 8u;
  return l;
}

template <int Bits>
__global__ __launch_bounds__(kLeanThreads, 2) void gemv_lean_kernel(const GemvArgs args, std::uint32_t total_tiles,
                                                                     std::uint32_t parts, std::uint32_t stages) {
  extern __shared__ __align__(128) std::uint8_t smem[];
  pdl_trigger();
  const unsigned warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
  const std::uint32_t G = args.groups;
  constexpr std::uint32_t kBlock = Bits * 256u;
  constexpr int kAlpha = Codec<Bits>::alpha, kBeta = Codec<Bits>::beta;
  const LeanLayout layout = lean_layout(Bits, G, parts, stages);
  const std::uint32_t part = parts > 1u ? cluster_ctarank() : 0u;
  const std::uint32_t clusters = gridDim.x / parts, cluster = blockIdx.x / parts;
  const std::uint32_t count = cluster < total_tiles ? (total_tiles - cluster + clusters - 1u) / clusters : 0u;
  const std::uint32_t g_begin = min(G, part * layout.per_part);
  const std::uint32_t n = min(G, g_begin + layout.per_part) - g_begin;
  const std::uint32_t remote_bytes = (G - min(G, layout.per_part)) * 64u;  // the peers' dots of one tile
  {
    std::uint32_t bad = 0;
    if (parts > 1u && (cluster_nctarank() != parts || part >= parts)) bad |= kGemvErrorCluster;
    if (layout.total > dynamic_smem_bytes() || stages > kLeanMaxStages || stages < 2u) bad |= kGemvErrorSmem;
    if (args.batch != 1u) bad |= kGemvErrorTile;
    if (bad != 0) {  // every CTA sees the same values: all return together, before any barrier
      if (threadIdx.x == 0) atomicOr(&g_gemv_error, bad);
      return;
    }
  }
  std::uint8_t* ring = smem;
  std::int32_t* dots = reinterpret_cast<std::int32_t*>(smem + layout.dots_offset);
  __half* tile_scales = reinterpret_cast<__half*>(smem + layout.scales_offset);
  std::int8_t* act = reinterpret_cast<std::int8_t*>(smem + layout.act_offset);
  std::int32_t* beta_sums = reinterpret_cast<std::int32_t*>(smem + layout.beta_offset);
  float* act_scales = reinterpret_cast<float*>(smem + layout.ascale_offset);
  std::uint64_t* full = reinterpret_cast<std::uint64_t*>(smem + layout.bar_offset);
  std::uint64_t* empty = full + stages;
  std::uint64_t* dots_full = empty + stages;
  std::uint64_t* dots_free = dots_full + kLeanSlots;
  std::uint64_t* scale_full = dots_free + kLeanSlots;
  auto tile_of = [&](std::uint32_t i) { return cluster + i * clusters; };

  if (threadIdx.x == 0) {
    for (std::uint32_t s = 0; s < stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kLeanComputeWarps);
    }
    for (std::uint32_t d = 0; d < kLeanSlots; ++d) {
      mbar_init(&dots_full[d], kLeanComputeWarps + 1u);  // the leader's warps + the chain warp's expect-tx
      mbar_init(&dots_free[d], 1);
      mbar_init(&scale_full[d], 1);
    }
    fence_mbar_init();
  }
  __syncthreads();
  const bool leader = part == 0;
  const bool chain_warp = warp > kLeanComputeWarps;
  if (chain_warp && leader && lane == 0) {
    // the first slots: the tiles' scales and the expected peer bytes (before any peer can store)
    for (std::uint32_t i = warp - kLeanComputeWarps - 1u; i < kLeanSlots && i < count; i += kLeanChainWarps) {
      std::uint32_t tile = tile_of(i);
      const MatrixArg m = select_matrix(args, tile);
      mbar_expect_tx(&scale_full[i], G * 32u);
      bulk_g2s(tile_scales + static_cast<std::size_t>(i) * G * 16u, m.scales + static_cast<std::size_t>(tile) * G * 16u,
               G * 32u, &scale_full[i]);
      mbar_expect_tx(&dots_full[i], remote_bytes);
    }
  }
  __syncwarp();
  if (parts > 1u) {
    cluster_arrive_relaxed();  // barriers initialised, first expect-tx posted
    cluster_wait();
  }

  if (warp == kLeanComputeWarps) {
    // producer: the weight ring (no dependence on the previous kernel); the
    // whole warp waits, lane 0 issues, so the warp stays converged
    for (std::uint32_t i = 0; i < count; ++i) {
      const std::uint32_t s = i % stages;
      if (!warp_wait_bounded<WaitKind::kPoll>(&empty[s], ((i / stages) & 1u) ^ 1u, &g_gemv_error)) break;
      if (lane == 0) {
        std::uint32_t tile = tile_of(i);
        const MatrixArg m = select_matrix(args, tile);
        mbar_expect_tx(&full[s], n * kBlock);
        bulk_g2s(ring + s * layout.stage_bytes, m.codes + (static_cast<std::size_t>(tile) * G + g_begin) * kBlock,
                 n * kBlock, &full[s]);
      }
      __syncwarp();
    }
  } else if (warp < kLeanComputeWarps) {
    pdl_wait();
    {
      const std::uint32_t act_groups = args.act_stride / kGroup;
      const uint4* source = reinterpret_cast<const uint4*>(args.act + static_cast<std::size_t>(g_begin) * kGroup);
      for (std::uint32_t v = threadIdx.x; v < n * 8u; v += kLeanComputeWarps * 32u) {
        reinterpret_cast<uint4*>(act)[v] = __ldg(source + v);
      }
      for (std::uint32_t l = threadIdx.x; l < n; l += kLeanComputeWarps * 32u) {
        beta_sums[l] = kBeta * __ldg(args.act_sums + g_begin + l);
      }
      (void)act_groups;
    }
    named_barrier(1, kLeanComputeWarps * 32u);
    const unsigned gl = lane >> 2, tq = lane & 3u;
    const std::uint32_t leader_dots = parts > 1u ? map_shared_rank(smem_addr(dots), 0) : 0u;
    const std::uint32_t leader_full = parts > 1u ? map_shared_rank(smem_addr(dots_full), 0) : 0u;
    for (std::uint32_t i = 0; i < count; ++i) {
      const std::uint32_t s = i % stages, d = i % kLeanSlots;
      if (!warp_wait_bounded<WaitKind::kSuspend>(&full[s], (i / stages) & 1u, &g_gemv_error)) break;
      if (!warp_wait_bounded<WaitKind::kPollCluster>(&dots_free[d], ((i / kLeanSlots) & 1u) ^ 1u, &g_gemv_error)) break;
      const std::uint8_t* stage = ring + s * layout.stage_bytes;
      for (std::uint32_t l = warp; l < n; l += kLeanComputeWarps) {
        const uint4 b0 = *reinterpret_cast<const uint4*>(act + l * kGroup + tq * 32u);
        const uint4 b1 = *reinterpret_cast<const uint4*>(act + l * kGroup + tq * 32u + 16u);
        const int beta_sum = beta_sums[l];
        LaneWords<Bits> w;
        load_lane_shared<Bits>(stage + l * kBlock, lane, w);
        std::uint32_t a[4][4];
        unpack(w, a);
        int c[4];
        mma_s8_16832_zero(c, a[0], b0.x, b0.y);
        mma_s8_16832(c, a[1], b0.z, b0.w);
        mma_s8_16832(c, a[2], b1.x, b1.y);
        mma_s8_16832(c, a[3], b1.z, b1.w);
        if (tq == 0) {  // token 0: rows gl and gl + 8
          const std::uint32_t index = (d * G + g_begin + l) * 16u + gl;
          const int low = kAlpha * c[0] + beta_sum, high = kAlpha * c[2] + beta_sum;
          if (leader) {
            dots[index] = low;
            dots[index + 8u] = high;
          } else {
            st_async_s32(leader_dots + index * 4u, low, leader_full + d * 8u);
            st_async_s32(leader_dots + (index + 8u) * 4u, high, leader_full + d * 8u);
          }
        }
      }
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&empty[s]);
        if (leader) mbar_arrive(&dots_full[d]);
      }
    }
  } else if (leader) {
    // chain warps: tiles k, k + 2, ... of this cluster
    pdl_wait();
    const std::uint32_t k = warp - kLeanComputeWarps - 1u;
    {
      const std::uint32_t t = threadIdx.x - (kLeanComputeWarps + 1u) * 32u;
      for (std::uint32_t g = t; g < G; g += kLeanChainWarps * 32u) act_scales[g] = h2f(args.act_scales[g]);
    }
    named_barrier(2, kLeanChainWarps * 32u);
    for (std::uint32_t i = k; i < count; i += kLeanChainWarps) {
      const std::uint32_t d = i % kLeanSlots, phase = (i / kLeanSlots) & 1u;
      if (!warp_wait_bounded<WaitKind::kSuspend>(&scale_full[d], phase, &g_gemv_error)) break;
      if (!warp_wait_bounded<WaitKind::kPollCluster>(&dots_full[d], phase, &g_gemv_error)) break;
      std::uint32_t tile = tile_of(i);
      const MatrixArg m = select_matrix(args, tile);
      float accumulator = 0.0f;
      if (lane < 16u) {
        const std::int32_t* tile_dots = dots + d * G * 16u + lane;
        const __half* scales = tile_scales + d * G * 16u + lane;
        std::uint32_t g = 0;
        for (; g + 8u <= G; g += 8u) {
          float product[8];
          int dot[8];
#pragma unroll
          for (unsigned j = 0; j < 8; ++j) {
            product[j] = __fmul_rn(h2f(scales[(g + j) * 16u]), act_scales[g + j]);
            dot[j] = tile_dots[(g + j) * 16u];
          }
#pragma unroll
          for (unsigned j = 0; j < 8; ++j) accumulator = fmaf(static_cast<float>(dot[j]), product[j], accumulator);
        }
        for (; g < G; ++g) {
          accumulator = fmaf(static_cast<float>(tile_dots[g * 16u]), __fmul_rn(h2f(scales[g * 16u]), act_scales[g]),
                             accumulator);
        }
      }
      __syncwarp();
      // hand the slot back before the output stores, so that the releases below
      // do not wait for them
      if (lane == 0 && i + kLeanSlots < count) {
        // slot d now serves tile i + D: its scales, its expected peer bytes, then the buffer goes back
        std::uint32_t next = tile_of(i + kLeanSlots);
        const MatrixArg nm = select_matrix(args, next);
        fence_proxy_async_shared();
        mbar_expect_tx(&scale_full[d], G * 32u);
        bulk_g2s(tile_scales + static_cast<std::size_t>(d) * G * 16u, nm.scales + static_cast<std::size_t>(next) * G * 16u,
                 G * 32u, &scale_full[d]);
        mbar_expect_tx(&dots_full[d], remote_bytes);
        mbar_arrive(&dots_free[d]);
        for (std::uint32_t r = 1; r < parts; ++r) mbar_arrive_remote(map_shared_rank(smem_addr(&dots_free[d]), r));
      }
      if (lane < 16u) {
        const std::size_t index = static_cast<std::size_t>(tile) * 16u + lane;
        if (m.output_f16) {
          static_cast<__half*>(m.output)[index] = f2h(accumulator);
        } else {
          static_cast<float*>(m.output)[index] = accumulator;
        }
      }
      __syncwarp();
    }
  }
  // No CTA of the cluster leaves while a peer may still address its shared memory.
  __syncthreads();
  if (parts > 1u) {
    cluster_arrive();
    cluster_wait();
  }
}

template <int Bits>
int launch_pipe(const GemvArgs& args, std::uint32_t total_tiles, cudaStream_t stream) {
  const PipeLayout layout = pipe_layout(Bits, args.groups, args.batch);
  static DeviceOnce configured;
  GFXB_TRY(configured.run([](int) {
    cudaError_t error = cudaFuncSetAttribute(gemv_pipe_kernel<Bits, false>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    if (error == cudaSuccess) {
      error = cudaFuncSetAttribute(gemv_pipe_kernel<Bits, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   200 * 1024);
    }
    if (error != cudaSuccess) {
      set_error_cuda(error, "pipelined GEMV shared-memory configuration failed");
      return static_cast<int>(GFXB_CUDA_ERROR);
    }
    return static_cast<int>(GFXB_OK);
  }));
  int sms = 0;
  GFXB_TRY(device_sm_count(&sms));
  // resident CTAs per SM for each (device, shared-memory size) seen
  static std::mutex occupancy_mutex;
  static std::map<std::pair<int, std::uint32_t>, int> occupancy;
  int device = 0;
  GFXB_TRY(current_device(&device));
  int cached_blocks = 0;
  {
    std::lock_guard<std::mutex> lock(occupancy_mutex);
    const auto found = occupancy.find({device, layout.total});
    if (found != occupancy.end()) {
      cached_blocks = found->second;
    } else {
      const cudaError_t error =
          cudaOccupancyMaxActiveBlocksPerMultiprocessor(&cached_blocks, gemv_pipe_kernel<Bits, false>, 256, layout.total);
      if (error != cudaSuccess || cached_blocks < 1) {
        set_error_cuda(error, "pipelined GEMV occupancy query failed");
        return GFXB_CUDA_ERROR;
      }
      occupancy[{device, layout.total}] = cached_blocks;
    }
  }
  const std::uint32_t grid = std::min<std::uint32_t>(total_tiles, static_cast<std::uint32_t>(sms * cached_blocks));
  const cudaError_t launch =
      args.batch == 1u ? launch_kernel(gemv_pipe_kernel<Bits, true>, dim3(grid), dim3(256), layout.total, stream, 0u,
                                       args, total_tiles)
                       : launch_kernel(gemv_pipe_kernel<Bits, false>, dim3(grid), dim3(256), layout.total, stream, 0u,
                                       args, total_tiles);
  if (launch != cudaSuccess) {
    set_error_cuda(launch, "pipelined GEMV launch failed");
    return GFXB_CUDA_ERROR;
  }
  return GFXB_OK;
}

std::uint32_t env_value(const char* name, std::uint32_t fallback) {
  const char* value = std::getenv(name);
  return value != nullptr && value[0] != '\0' ? static_cast<std::uint32_t>(std::strtoul(value, nullptr, 10)) : fallback;
}

// Tuning knobs (read once): cluster split override and groups per bulk copy.
struct StreamTuning {
  std::uint32_t parts = env_value("GFXB_GEMV_PARTS", 0);
  // groups per bulk copy: a power of two (the kernels find a group's barrier by a shift)
  std::uint32_t chunk = 1u << (31 - __builtin_clz(std::max<std::uint32_t>(1u, env_value("GFXB_GEMV_CHUNK", 8))));
  std::uint32_t min_tiles_p1 = env_value("GFXB_GEMV_P1_TILES", 1024);
  std::uint32_t cascade = env_value("GFXB_GEMV_CASCADE", 1);  // 0: several tokens gather in one CTA too
  std::uint32_t tall_cascade = std::max<std::uint32_t>(2u, env_value("GFXB_GEMV_TALL_CASCADE", 9));  // tokens from which tall matrices split in two
};

const StreamTuning& tuning() {
  static const StreamTuning t;
  return t;
}

// launch_stream's answer when no streaming kernel takes the shape (more than 8
// tokens without a cluster split): the caller uses the one-CTA-per-tile kernel.
constexpr int kNoStreamPath = -1;

template <int Bits>
int launch_stream(const GemvArgs& args, std::uint32_t total_tiles, cudaStream_t stream) {
  const StreamTuning& tune = tuning();
  std::uint32_t parts = total_tiles >= tune.min_tiles_p1 ? 1u : (total_tiles >= tune.min_tiles_p1 / 2 ? 2u : 4u);
  if (tune.parts != 0) parts = tune.parts;
  while (parts > 1u && parts > args.groups) parts >>= 1;
  const std::uint32_t chunk = tune.chunk;
  // beyond 8 tokens tall matrices split in two as well: the cascade then takes them
  if (args.batch >= tune.tall_cascade && parts == 1u && tune.parts == 0 && args.groups >= 2u) parts = 2u;
  if (args.batch > 8u && (parts == 1u || tune.cascade == 0)) return kNoStreamPath;
  if (parts > 1u && tune.cascade != 0 && (args.batch >= 3u || (args.batch == 2u && args.groups > 64u))) {
    // several tokens: the chain passes from rank to rank instead of gathering every dot in one CTA
    // (measured on B200: faster from 3 tokens on, and at 2 tokens for long K)
    const CascadeLayout layout = cascade_layout(Bits, args.groups, parts, args.batch, chunk);
    static DeviceOnce cascade_configured;
    GFXB_TRY(cascade_configured.run([](int) {
      cudaError_t error = cudaFuncSetAttribute(gemv_cascade_kernel<Bits, 1>,
                                               cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
      if (error == cudaSuccess) {
        error = cudaFuncSetAttribute(gemv_cascade_kernel<Bits, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     200 * 1024);
      }
      if (error != cudaSuccess) {
        set_error_cuda(error, "GEMV shared-memory configuration failed");
        return static_cast<int>(GFXB_CUDA_ERROR);
      }
      return static_cast<int>(GFXB_OK);
    }));
    if (layout.total > 200u * 1024u) return fail(GFXB_UNSUPPORTED, "GEMV shape exceeds shared memory");
    const cudaError_t error =
        args.batch > 8u ? launch_kernel(gemv_cascade_kernel<Bits, 2>, dim3(total_tiles * parts), dim3(256),
                                        layout.total, stream, parts, args, parts, chunk)
                        : launch_kernel(gemv_cascade_kernel<Bits, 1>, dim3(total_tiles * parts), dim3(256),
                                        layout.total, stream, parts, args, parts, chunk);
    if (error != cudaSuccess) {
      set_error_cuda(error, "cascaded GEMV launch failed");
      return GFXB_CUDA_ERROR;
    }
    return GFXB_OK;
  }
  const StreamLayout layout = stream_layout(Bits, args.groups, parts, args.batch, chunk);
  static DeviceOnce configured;
  GFXB_TRY(configured.run([](int) {
    cudaError_t error = cudaFuncSetAttribute(gemv_stream_kernel<Bits, false>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    if (error == cudaSuccess) {
      error = cudaFuncSetAttribute(gemv_stream_kernel<Bits, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   200 * 1024);
    }
    if (error == cudaSuccess) {
      error = cudaFuncSetAttribute(gemv_stream_kernel<Bits, true, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   200 * 1024);
    }
    if (error != cudaSuccess) {
      set_error_cuda(error, "GEMV shared-memory configuration failed");
      return static_cast<int>(GFXB_CUDA_ERROR);
    }
    return static_cast<int>(GFXB_OK);
  }));
  if (layout.total > 200u * 1024u) return fail(GFXB_UNSUPPORTED, "GEMV shape exceeds shared memory");
  cudaLaunchConfig_t config{};
  config.gridDim = dim3(total_tiles * parts);
  config.blockDim = dim3(256);
  config.dynamicSmemBytes = layout.total;
  config.stream = stream;
  cudaLaunchAttribute attribute[1];
  attribute[0].id = cudaLaunchAttributeClusterDimension;
  attribute[0].val.clusterDim.x = parts;
  attribute[0].val.clusterDim.y = 1;
  attribute[0].val.clusterDim.z = 1;
  config.attrs = attribute;
  config.numAttrs = 1;
  // the product-first chain from 64 groups on (measured: faster on the 136-group down projection, slower on
  // 40-group matrices, whose CTAs are limited by registers rather than shared memory)
  const cudaError_t error =
      args.batch != 1u ? launch_kernel(gemv_stream_kernel<Bits, false>, config.gridDim, config.blockDim,
                                       config.dynamicSmemBytes, stream, parts, args, parts, chunk)
      : args.groups >= 64u ? launch_kernel(gemv_stream_kernel<Bits, true, true>, config.gridDim, config.blockDim,
                                           config.dynamicSmemBytes, stream, parts, args, parts, chunk)
                           : launch_kernel(gemv_stream_kernel<Bits, true>, config.gridDim, config.blockDim,
                                           config.dynamicSmemBytes, stream, parts, args, parts, chunk);
  if (error != cudaSuccess) {
    set_error_cuda(error, "streaming GEMV launch failed");
    return GFXB_CUDA_ERROR;
  }
  return GFXB_OK;
}

// Warp-specialised persistent GEMV for one token: two CTAs per SM, the
// deepest ring that fits. Which shapes take it follows what measured fastest
// on B200 against the older kernels: P = 1 for very tall matrices (the LM
// head: 73 -> 60 us alone), P = 2 for small matrices (the output projections:
// 7.1 -> 6.5 us); decode 199.9 -> 202.0 tok/s with both. Wide K at P = 4 (the
// MLP down projection) is faster alone (16.5 -> 14.5 us) but slowed the whole
// decode (192.7 tok/s: its two large CTAs per SM cannot start until the
// previous kernel has left the SMs), so it is off by default (bit 1 of
// GFXB_GEMV_LEAN_SHAPES turns it on); other shapes keep the pipelined and
// streaming kernels, which were faster there. Larger clusters were slower on
// every shape (each tile waits for its slowest CTA); one CTA per SM (room for
// the next kernel) lost bandwidth: 163 tok/s.
struct LeanPlan {
  std::uint32_t parts = 0, stages = 0, clusters = 0;
  std::uint32_t smem = 0;
};

constexpr std::uint32_t kLeanSmemBudget = 110u * 1024u;
constexpr std::uint32_t kLeanOneCtaSmem = 120u * 1024u;  // occupancy query size: at most one CTA per SM

template <int Bits>
int lean_plan(const GemvArgs& args, std::uint32_t total_tiles, LeanPlan* out) {
  static DeviceOnce configured;
  GFXB_TRY(configured.run([](int) {
    const cudaError_t error = cudaFuncSetAttribute(gemv_lean_kernel<Bits>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                   static_cast<int>(kLeanOneCtaSmem));
    if (error != cudaSuccess) {
      set_error_cuda(error, "persistent GEMV shared-memory configuration failed");
      return static_cast<int>(GFXB_CUDA_ERROR);
    }
    return static_cast<int>(GFXB_OK);
  }));
  int device = 0;
  GFXB_TRY(current_device(&device));
  static std::mutex plan_mutex;
  static std::map<std::tuple<int, std::uint32_t, std::uint32_t>, LeanPlan> plans;
  const auto key = std::make_tuple(device, args.groups, total_tiles);
  std::lock_guard<std::mutex> lock(plan_mutex);
  const auto found = plans.find(key);
  if (found != plans.end()) {
    *out = found->second;
    return GFXB_OK;
  }
  static const std::uint32_t forced = env_value("GFXB_GEMV_LEAN_PARTS", 0);
  static const std::uint32_t ctas_per_sm = env_value("GFXB_GEMV_LEAN_CTAS", 2) == 1u ? 1u : 2u;
  // shape classes that take this kernel (bit 0 very tall, bit 1 wide K, bit 2 small)
  static const std::uint32_t classes = env_value("GFXB_GEMV_LEAN_SHAPES", 5);
  std::uint32_t wanted = forced;
  if (wanted == 0) {
    if (total_tiles >= 4096u) {
      wanted = (classes & 1u) != 0 ? 1u : 0u;
    } else if (args.groups >= 96u) {
      wanted = (classes & 2u) != 0 ? 4u : 0u;
    } else if (total_tiles <= 640u) {
      wanted = (classes & 4u) != 0 ? 2u : 0u;
    }
  }
  LeanPlan best;
  for (std::uint32_t parts = 1; parts <= 8u && wanted != 0; parts <<= 1) {
    if (parts != wanted) continue;
    const std::uint32_t per_part = (args.groups + parts - 1u) / parts;
    if (parts > 1u && (per_part < 4u || per_part * (parts - 1u) >= args.groups)) continue;
    std::uint32_t stages = 0;
    for (std::uint32_t s = kLeanMaxStages; s >= 2u; --s) {
      if (lean_layout(Bits, args.groups, parts, s).total <= kLeanSmemBudget) {
        stages = s;
        break;
      }
    }
    if (stages == 0) continue;
    const std::uint32_t smem = lean_layout(Bits, args.groups, parts, stages).total;
    cudaLaunchConfig_t config{};
    config.gridDim = dim3(parts);
    config.blockDim = dim3(kLeanThreads);
    config.dynamicSmemBytes = ctas_per_sm == 1u ? kLeanOneCtaSmem : smem;
    cudaLaunchAttribute attribute[1];
    attribute[0].id = cudaLaunchAttributeClusterDimension;
    attribute[0].val.clusterDim.x = parts;
    attribute[0].val.clusterDim.y = 1;
    attribute[0].val.clusterDim.z = 1;
    config.attrs = attribute;
    config.numAttrs = 1;
    int clusters = 0;
    const cudaError_t error = cudaOccupancyMaxActiveClusters(&clusters, gemv_lean_kernel<Bits>, &config);
    if (error != cudaSuccess || clusters < 1) {
      cudaGetLastError();
      continue;
    }
    const std::uint32_t c = static_cast<std::uint32_t>(clusters);
    {
      best.parts = parts;
      best.stages = stages;
      best.clusters = std::min(c, total_tiles);
      best.smem = smem;
    }
  }
  plans[key] = best;
  *out = best;
  return GFXB_OK;
}

template <int Bits>
int launch_lean(const GemvArgs& args, std::uint32_t total_tiles, cudaStream_t stream) {
  LeanPlan plan;
  GFXB_TRY(lean_plan<Bits>(args, total_tiles, &plan));
  if (plan.parts == 0) return kNoStreamPath;
  const cudaError_t error = launch_kernel(gemv_lean_kernel<Bits>, dim3(plan.clusters * plan.parts), dim3(kLeanThreads),
                                          plan.smem, stream, plan.parts > 1u ? plan.parts : 0u, args, total_tiles,
                                          plan.parts, plan.stages);
  if (error != cudaSuccess) {
    set_error_cuda(error, "persistent GEMV launch failed");
    return GFXB_CUDA_ERROR;
  }
  return GFXB_OK;
}

// ---------------------------------------------------------------------------
// Reference-layout GEMM (drop-in for launch_gfx12_i4_gemm / _i8_gemm): gfx12
// tiled weights staged per warp in shared memory, activations read in the
// reference's packed-A4 or row-major A8 layout, group sums formed on the fly.
// ---------------------------------------------------------------------------

// Spread four consecutive 3-bit codes (a 12-bit field) into four bytes.
__device__ __forceinline__ std::uint32_t spread3(std::uint32_t f) {
  f &= 0xfffu;
  std::uint32_t x = (f & 0x3fu) | ((f & 0xfc0u) << 10);
  return (x & 0x00070007u) | ((x & 0x00380038u) << 5);
}
__device__ __forceinline__ std::uint32_t spread4(std::uint32_t f) {
  f &= 0xffffu;
  std::uint32_t x = (f & 0xffu) | ((f & 0xff00u) << 8);
  return (x & 0x000f000fu) | ((x & 0x00f000f0u) << 4);
}
__device__ __forceinline__ std::uint32_t spread2(std::uint32_t f) {
  f &= 0xffu;
  std::uint32_t x = (f & 0xfu) | ((f & 0xf0u) << 12);
  return (x & 0x00030003u) | ((x & 0x000c000cu) << 6);
}

// Signed nibbles (two's complement) -> signed bytes, four at a time.
__device__ __forceinline__ std::uint32_t nibbles_to_s8(std::uint32_t packed16) {
  const std::uint32_t biased = spread4(packed16) ^ 0x08080808u;   // v + 8 in [0, 15]
  return ((biased | 0x80808080u) - 0x08080808u) ^ 0x80808080u;    // per-byte v
}

template <int Bits, bool Act8, int NB>
__global__ __launch_bounds__(256) void gemm_gfx12_kernel(
    const std::uint8_t* __restrict__ weights, const __half* __restrict__ weight_scales,
    const std::uint8_t* __restrict__ activations, const __half* __restrict__ activation_scales,
    float* __restrict__ output, std::uint32_t rows, std::uint32_t columns, std::uint32_t batch) {
  pdl_trigger();
  pdl_wait();
  const std::uint32_t tile = blockIdx.x;
  const unsigned warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
  const unsigned gl = lane >> 2, tq = lane & 3u;
  const std::uint32_t G = columns / kGroup, B = batch, K = columns;
  constexpr std::uint32_t kBlock = Bits * 256u;
  constexpr std::uint32_t kFrag = Bits == 2 ? 8u : (Bits == 3 ? 12u : 16u);
  constexpr int kAlpha = Codec<Bits>::alpha, kBeta = Codec<Bits>::beta;
  __shared__ std::uint32_t stage[8][kBlock / 4 + 4];
  // one padding word per row: the chain's reads (16 rows x 2 tokens per warp) and the mma lanes' writes
  // (8 rows per warp) then fall into distinct banks instead of 8-16 on one
  __shared__ std::int32_t dots[8][16][NB * 8 + 1];
  const std::uint32_t pairs = 16u * B;
  float accumulator[2] = {0.0f, 0.0f};
  const std::uint32_t rounds = (G + 7u) / 8u;
  for (std::uint32_t r = 0; r < rounds; ++r) {
    const std::uint32_t g = 8u * r + warp;
    const std::uint32_t round_groups = min(8u, G - 8u * r);
    if (g < G) {
      const std::uint8_t* block = weights + (static_cast<std::size_t>(tile) * G + g) * kBlock;
      for (std::uint32_t offset = lane * 16u; offset < kBlock; offset += 512u) {
        const uint4 v = ldg_stream16(block + offset);
        stage[warp][offset / 4 + 0] = v.x;
        stage[warp][offset / 4 + 1] = v.y;
        stage[warp][offset / 4 + 2] = v.z;
        stage[warp][offset / 4 + 3] = v.w;
      }
      __syncwarp();
      std::uint32_t a[4][4];
#pragma unroll
      for (unsigned s = 0; s < 4; ++s) {
#pragma unroll
        for (unsigned q = 0; q < 4; ++q) {
          const unsigned row = gl + 8u * (q & 1u), half = q >> 1;
          const std::uint32_t frag_bit = ((s * 16u + row) * kFrag) * 8u;
          const std::uint32_t bit = frag_bit + (Bits * (16u * half + 4u * tq));
          const std::uint32_t lo = stage[warp][bit / 32u];
          const std::uint32_t hi = stage[warp][bit / 32u + 1u];
          const std::uint32_t field = __funnelshift_r(lo, hi, bit & 31u);
          if constexpr (Bits == 3) {
            a[s][q] = spread3(field);
          } else if constexpr (Bits == 4) {
            a[s][q] = spread4(field) ^ 0x08080808u;
          } else {
            a[s][q] = spread2(field);
          }
        }
      }
#pragma unroll
      for (int nb = 0; nb < NB; ++nb) {
        std::uint32_t token = nb * 8u + gl;
        token = token < B ? token : B - 1u;
        std::uint32_t bregs[4][2];
        int partial = 0;
#pragma unroll
        for (unsigned s = 0; s < 4; ++s) {
#pragma unroll
          for (unsigned h = 0; h < 2; ++h) {
            const std::uint32_t k = g * kGroup + 32u * s + 16u * h + 4u * tq;
            std::uint32_t value;
            if constexpr (Act8) {
              value = __ldg(reinterpret_cast<const std::uint32_t*>(
                  activations + static_cast<std::size_t>(token) * K + k));
            } else {
              const std::uint16_t packed = __ldg(reinterpret_cast<const std::uint16_t*>(
                  activations + static_cast<std::size_t>(token) * (K / 2u) + k / 2u));
              value = nibbles_to_s8(packed);
            }
            bregs[s][h] = value;
            partial = __dp4a(static_cast<int>(value), 0x01010101, partial);
          }
        }
        partial += __shfl_xor_sync(0xffffffffu, partial, 1);
        partial += __shfl_xor_sync(0xffffffffu, partial, 2);
        const int sum0 = __shfl_sync(0xffffffffu, partial, (2u * tq) * 4u);
        const int sum1 = __shfl_sync(0xffffffffu, partial, (2u * tq + 1u) * 4u);
        int c[4] = {0, 0, 0, 0};
#pragma unroll
        for (unsigned s = 0; s < 4; ++s) mma_s8_16832(c, a[s], bregs[s][0], bregs[s][1]);
        const std::uint32_t t0 = nb * 8u + 2u * tq, t1 = t0 + 1u;
        if (t0 < B) {
          dots[warp][gl][t0] = kAlpha * c[0] + kBeta * sum0;
          dots[warp][gl + 8][t0] = kAlpha * c[2] + kBeta * sum0;
        }
        if (t1 < B) {
          dots[warp][gl][t1] = kAlpha * c[1] + kBeta * sum1;
          dots[warp][gl + 8][t1] = kAlpha * c[3] + kBeta * sum1;
        }
      }
    }
    __syncthreads();
#pragma unroll
    for (int p = 0; p < 2; ++p) {
      const std::uint32_t pair = threadIdx.x + 256u * p;
      if (pair < pairs) {
        const std::uint32_t row = pair & 15u, token = pair >> 4;
        for (unsigned w = 0; w < round_groups; ++w) {
          const std::uint32_t gg = 8u * r + w;
          const float product = __fmul_rn(h2f(weight_scales[(tile * G + gg) * 16u + row]),
                                          h2f(activation_scales[token * G + gg]));
          accumulator[p] = fmaf(static_cast<float>(dots[w][row][token]), product, accumulator[p]);
        }
      }
    }
    __syncthreads();
  }
#pragma unroll
  for (int p = 0; p < 2; ++p) {
    const std::uint32_t pair = threadIdx.x + 256u * p;
    if (pair < pairs) {
      const std::uint32_t row = pair & 15u, token = pair >> 4;
      output[static_cast<std::size_t>(token) * rows + tile * 16u + row] = accumulator[p];
    }
  }
}

// ---------------------------------------------------------------------------
// activation packs
// ---------------------------------------------------------------------------

__device__ __forceinline__ std::uint32_t fragment_offset(std::uint32_t k) {
  const std::uint32_t s = k >> 5, rest = k & 31u, half = rest >> 4, t = (rest & 15u) >> 2, j = k & 3u;
  return t * 32u + s * 8u + half * 4u + j;
}

template <int Bits>
__global__ __launch_bounds__(128) void pack_activation_kernel(
    const __half* __restrict__ input, std::int8_t* __restrict__ codes, __half* __restrict__ scales,
    std::int32_t* __restrict__ sums, std::uint8_t* __restrict__ packed_a4,
    std::uint32_t columns, std::uint32_t groups) {
  pdl_trigger();
  pdl_wait();
  const std::uint32_t linear = blockIdx.x;
  const std::uint32_t token = linear / groups, group = linear - token * groups;
  const unsigned i = threadIdx.x, lane = i & 31u, warp = i >> 5;
  const std::size_t base = static_cast<std::size_t>(token) * columns + group * kGroup;
  const float x = h2f(input[base + i]);
  float amax = fabsf(x);
#pragma unroll
  for (unsigned offset = 16; offset != 0; offset >>= 1) {
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, offset));
  }
  __shared__ float warp_max[4];
  __shared__ int warp_sum[4];
  if (lane == 0) warp_max[warp] = amax;
  __syncthreads();
  amax = fmaxf(fmaxf(warp_max[0], warp_max[1]), fmaxf(warp_max[2], warp_max[3]));
  constexpr float kDivisor = Bits == 4 ? 7.0f : 127.0f;
  constexpr int kLimit = Bits == 4 ? 7 : 127;
  const __half scale_h = f2h(amax == 0.0f ? 1.0f : __fdiv_rn(amax, kDivisor));
  const float scale = h2f(scale_h);
  int q = f2i_rn(__fdiv_rn(x, scale));
  q = max(-kLimit, min(kLimit, q));
  codes[base + fragment_offset(i)] = static_cast<std::int8_t>(q);
  int total = q;
#pragma unroll
  for (unsigned offset = 16; offset != 0; offset >>= 1) total += __shfl_xor_sync(0xffffffffu, total, offset);
  if (lane == 0) warp_sum[warp] = total;
  const int neighbour = __shfl_down_sync(0xffffffffu, q, 1);
  if (Bits == 4 && packed_a4 != nullptr && (i & 1u) == 0) {
    packed_a4[static_cast<std::size_t>(token) * (columns / 2u) + group * 64u + i / 2u] =
        static_cast<std::uint8_t>((q & 0x0f) | ((neighbour & 0x0f) << 4));
  }
  __syncthreads();
  if (i == 0) {
    scales[linear] = scale_h;
    sums[linear] = warp_sum[0] + warp_sum[1] + warp_sum[2] + warp_sum[3];
  }
}

template <int Bits>
__global__ __launch_bounds__(128) void quantize_reference_kernel(
    const __half* __restrict__ input, std::uint8_t* __restrict__ output, __half* __restrict__ scales,
    std::uint32_t columns, std::uint32_t groups) {
  pdl_trigger();
  pdl_wait();
  const std::uint32_t linear = blockIdx.x;
  const std::uint32_t token = linear / groups, group = linear - token * groups;
  const unsigned i = threadIdx.x, lane = i & 31u, warp = i >> 5;
  const std::size_t base = static_cast<std::size_t>(token) * columns + group * kGroup;
  const float x = h2f(input[base + i]);
  float amax = fabsf(x);
#pragma unroll
  for (unsigned offset = 16; offset != 0; offset >>= 1) {
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, offset));
  }
  __shared__ float warp_max[4];
  if (lane == 0) warp_max[warp] = amax;
  __syncthreads();
  amax = fmaxf(fmaxf(warp_max[0], warp_max[1]), fmaxf(warp_max[2], warp_max[3]));
  constexpr float kDivisor = Bits == 4 ? 7.0f : 127.0f;
  constexpr int kLimit = Bits == 4 ? 7 : 127;
  const __half scale_h = f2h(amax == 0.0f ? 1.0f : __fdiv_rn(amax, kDivisor));
  int q = f2i_rn(__fdiv_rn(x, h2f(scale_h)));
  q = max(-kLimit, min(kLimit, q));
  if constexpr (Bits == 8) {
    output[base + i] = static_cast<std::uint8_t>(static_cast<std::int8_t>(q));
  } else {
    const int neighbour = __shfl_down_sync(0xffffffffu, q, 1);
    if ((i & 1u) == 0) {
      output[static_cast<std::size_t>(token) * (columns / 2u) + group * 64u + i / 2u] =
          static_cast<std::uint8_t>((q & 0x0f) | ((neighbour & 0x0f) << 4));
    }
  }
  if (i == 0) scales[linear] = scale_h;
}

// ---------------------------------------------------------------------------
// layout conversion and synthetic weights
// ---------------------------------------------------------------------------

// Code sources: each yields the unsigned code u (reference code mapping of
// quantization.cpp:29-56, W4 biased by +8) of logical (row, column).
struct RowMajorSource {
  const std::uint8_t* codes;
  std::uint32_t columns;
  int bits;
  __device__ std::uint32_t operator()(std::uint32_t row, std::uint32_t column) const {
    if (bits == 2) {
      const std::uint8_t* r = codes + static_cast<std::size_t>(row) * (columns / 4u);
      return (r[column / 4u] >> ((column & 3u) * 2u)) & 3u;
    }
    if (bits == 4) {
      const std::uint8_t* r = codes + static_cast<std::size_t>(row) * (columns / 2u);
      return ((r[column / 2u] >> ((column & 1u) * 4u)) & 15u) ^ 8u;
    }
    const std::uint8_t* r = codes + static_cast<std::size_t>(row) * (columns * 3u / 8u);
    const std::uint32_t group = column / kGroup, local = column % kGroup;
    const std::uint32_t byte = local / 8u, bit = local & 7u;
    std::uint32_t code = 0;
#pragma unroll
    for (std::uint32_t plane = 0; plane < 3; ++plane) {
      code |= ((r[group * 48u + plane * 16u + byte] >> bit) & 1u) << plane;
    }
    return code;
  }
};

struct Gfx12Source {
  const std::uint8_t* codes;
  std::uint32_t columns;
  int bits;
  __device__ std::uint32_t operator()(std::uint32_t row, std::uint32_t column) const {
    const std::uint32_t groups = columns / kGroup;
    const std::uint32_t fragment_bytes = bits == 2 ? 8u : (bits == 3 ? 12u : 16u);
    const std::uint32_t tile = row / 16u, local_row = row & 15u;
    const std::uint32_t group = column / kGroup, k_tile = (column % kGroup) / 32u, item = column & 31u;
    const std::uint8_t* fragment =
        codes + (((static_cast<std::size_t>(tile) * groups + group) * 4u + k_tile) * 16u + local_row) *
                    fragment_bytes;
    const std::uint32_t bit = item * static_cast<std::uint32_t>(bits);
    std::uint32_t word = fragment[bit / 8u];
    if (bit / 8u + 1u < fragment_bytes) word |= static_cast<std::uint32_t>(fragment[bit / 8u + 1u]) << 8;
    const std::uint32_t code = (word >> (bit & 7u)) & ((1u << bits) - 1u);
    return bits == 4 ? (code ^ 8u) : code;
  }
};

__device__ __forceinline__ std::uint64_t mix64(std::uint64_t z) {
  z += 0x9e3779b97f4a7c15ULL;
  z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ULL;
  z = (z ^ (z >> 27)) * 0x94d049bb133111ebULL;
  return z ^ (z >> 31);
}

__device__ __forceinline__ std::uint64_t hash3(std::uint64_t seed, std::uint64_t stream, std::uint64_t index) {
  return mix64(mix64(seed ^ (stream * 0xd1b54a32d192ed03ULL)) + index);
}

// Synthetic weights: the reference code of global (row, column) is the top
// `bits` bits of hash(seed, 2*tensor, row*K + column). A shard generates its
// local rows/columns through a row map (up to three contiguous segments of
// global rows) and a column offset, so every tensor-parallel rank holds
// exactly its slice of the same global model.
struct RowMap {
  std::uint32_t segments;
  std::uint32_t local_begin[4];
  std::uint32_t global_begin[3];
  __host__ __device__ std::uint32_t operator()(std::uint32_t row) const {
    std::uint32_t i = 0;
    while (i + 1 < segments && row >= local_begin[i + 1]) ++i;
    return global_begin[i] + (row - local_begin[i]);
  }
};

// Zero-mean synthetic reference codes: W2 levels {-3,-1,1,3}, W3 q uniform on
// {-3..3}, W4 q uniform on {-7..7} (two's-complement nibble).
__host__ __device__ __forceinline__ std::uint32_t synthetic_code(std::uint64_t h, int bits) {
  if (bits == 2) return static_cast<std::uint32_t>(h >> 62);
  if (bits == 3) return static_cast<std::uint32_t>((h >> 32) % 7u + 1u);
  return static_cast<std::uint32_t>((static_cast<int>((h >> 32) % 15u) - 7) & 0x0f);
}

struct HashSource {
  std::uint64_t seed;
  std::uint32_t tensor;
  std::uint32_t global_columns;
  std::uint32_t column_offset;
  RowMap rows;
  int bits;
  __device__ std::uint32_t operator()(std::uint32_t row, std::uint32_t column) const {
    const std::uint64_t index = static_cast<std::uint64_t>(rows(row)) * global_columns + column + column_offset;
    return synthetic_code(hash3(seed, 2ull * tensor, index), bits) ^ (bits == 4 ? 8u : 0u);
  }
};

template <class Source>
__global__ void write_b200_kernel(Source source, std::uint8_t* __restrict__ out, std::uint32_t groups,
                                  std::uint64_t lanes_total, int bits) {
  const std::uint64_t index = static_cast<std::uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (index >= lanes_total) return;
  const std::uint32_t lane = static_cast<std::uint32_t>(index & 31u);
  const std::uint64_t block_index = index >> 5;
  const std::uint32_t tile = static_cast<std::uint32_t>(block_index / groups);
  const std::uint32_t group = static_cast<std::uint32_t>(block_index % groups);
  const std::uint32_t gl = lane >> 2, tq = lane & 3u;
  auto code = [&](std::uint32_t s, std::uint32_t q, std::uint32_t j) -> std::uint32_t {
    const std::uint32_t row = tile * 16u + gl + 8u * (q & 1u);
    const std::uint32_t column = group * kGroup + 32u * s + 16u * (q >> 1) + 4u * tq + j;
    return source(row, column);
  };
  std::uint8_t* block = out + block_index * static_cast<std::uint64_t>(bits) * 256u;
  if (bits == 3) {
    std::uint32_t words[6] = {0, 0, 0, 0, 0, 0};
#pragma unroll
    for (std::uint32_t triple = 0; triple < 2; ++triple) {
      const std::uint32_t sa = 2u * triple, sb = sa + 1u;
      std::uint32_t x0 = 0, x1 = 0, x2 = 0;
#pragma unroll
      for (std::uint32_t j = 0; j < 4; ++j) {
        const std::uint32_t shift = 8u * j;
        x0 |= (code(sa, 0, j) | (code(sa, 1, j) << 3) | ((code(sb, 2, j) & 3u) << 6)) << shift;
        x1 |= (code(sa, 2, j) | (code(sa, 3, j) << 3) | ((code(sb, 3, j) & 3u) << 6)) << shift;
        x2 |= (code(sb, 0, j) | (code(sb, 1, j) << 3) | ((code(sb, 2, j) >> 2) << 6) |
               ((code(sb, 3, j) >> 2) << 7))
              << shift;
      }
      words[3 * triple] = x0;
      words[3 * triple + 1] = x1;
      words[3 * triple + 2] = x2;
    }
    std::uint32_t* p0 = reinterpret_cast<std::uint32_t*>(block + 16u * lane);
    std::uint32_t* p1 = reinterpret_cast<std::uint32_t*>(block + 512u + 8u * lane);
    p0[0] = words[0];
    p0[1] = words[1];
    p0[2] = words[2];
    p0[3] = words[3];
    p1[0] = words[4];
    p1[1] = words[5];
  } else if (bits == 4) {
    std::uint32_t words[8];
#pragma unroll
    for (std::uint32_t s = 0; s < 4; ++s) {
      std::uint32_t lo = 0, hi = 0;
#pragma unroll
      for (std::uint32_t j = 0; j < 4; ++j) {
        lo |= (code(s, 0, j) | (code(s, 1, j) << 4)) << (8u * j);
        hi |= (code(s, 2, j) | (code(s, 3, j) << 4)) << (8u * j);
      }
      words[2 * s] = lo;
      words[2 * s + 1] = hi;
    }
    std::uint32_t* p0 = reinterpret_cast<std::uint32_t*>(block + 16u * lane);
    std::uint32_t* p1 = reinterpret_cast<std::uint32_t*>(block + 512u + 16u * lane);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      p0[i] = words[i];
      p1[i] = words[4 + i];
    }
  } else {
    std::uint32_t* p0 = reinterpret_cast<std::uint32_t*>(block + 16u * lane);
#pragma unroll
    for (std::uint32_t s = 0; s < 4; ++s) {
      std::uint32_t word = 0;
#pragma unroll
      for (std::uint32_t j = 0; j < 4; ++j) {
        word |= (code(s, 0, j) | (code(s, 1, j) << 2) | (code(s, 2, j) << 4) | (code(s, 3, j) << 6))
                << (8u * j);
      }
      p0[s] = word;
    }
  }
}

__global__ void tile_scales_kernel(const __half* __restrict__ rowmajor, __half* __restrict__ tiled,
                                   std::uint32_t rows, std::uint32_t groups) {
  const std::uint64_t index = static_cast<std::uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (index >= static_cast<std::uint64_t>(rows) * groups) return;
  const std::uint32_t row = static_cast<std::uint32_t>(index / groups);
  const std::uint32_t group = static_cast<std::uint32_t>(index % groups);
  tiled[(static_cast<std::size_t>(row / 16u) * groups + group) * 16u + (row & 15u)] = rowmajor[index];
}

template <class Source>
int launch_write_b200(const Source& source, std::uint8_t* out, std::size_t rows, std::size_t columns,
                      int bits, cudaStream_t stream) {
  const std::uint64_t groups = columns / kGroup;
  const std::uint64_t lanes = (rows / 16u) * groups * 32u;
  const unsigned threads = 256;
  const std::uint64_t blocks = (lanes + threads - 1) / threads;
  write_b200_kernel<Source><<<static_cast<unsigned>(blocks), threads, 0, stream>>>(
      source, out, static_cast<std::uint32_t>(groups), lanes, bits);
  return launch_status("b200 weight layout kernel launch failed");
}

// gfx12 tiled W2/W4 codes and tiled scales -> row-major codes and scales
// (quantization.cpp:278-314 in reverse). For W2 and W4 a fragment holds the
// row's 32 codes of one k-tile in row-major byte order, so each fragment is
// one contiguous piece of the row.
__global__ void untile_gfx12_kernel(const std::uint8_t* __restrict__ tiled, std::uint8_t* __restrict__ rowmajor,
                                    std::uint64_t bytes, std::uint32_t groups, std::uint32_t fragment) {
  const std::uint64_t index = static_cast<std::uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (index >= bytes) return;
  const std::uint64_t piece = index / fragment;
  const std::uint32_t byte = static_cast<std::uint32_t>(index % fragment);
  const std::uint32_t local_row = static_cast<std::uint32_t>(piece & 15u);
  const std::uint64_t k_group = piece >> 4;  // (tile * groups + group) * 4 + k_tile
  const std::uint32_t k_tile = static_cast<std::uint32_t>(k_group & 3u);
  const std::uint64_t tile_group = k_group >> 2;
  const std::uint64_t tile = tile_group / groups;
  const std::uint32_t group = static_cast<std::uint32_t>(tile_group % groups);
  const std::uint64_t row = tile * 16u + local_row;
  rowmajor[row * groups * 4u * fragment + (group * 4u + k_tile) * fragment + byte] = tiled[index];
}

__global__ void untile_scales_kernel(const __half* __restrict__ tiled, __half* __restrict__ rowmajor,
                                     std::uint64_t count, std::uint32_t groups) {
  const std::uint64_t index = static_cast<std::uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (index >= count) return;
  const std::uint32_t local_row = static_cast<std::uint32_t>(index & 15u);
  const std::uint64_t tile_group = index >> 4;
  const std::uint64_t tile = tile_group / groups;
  const std::uint32_t group = static_cast<std::uint32_t>(tile_group % groups);
  rowmajor[(tile * 16u + local_row) * groups + group] = tiled[index];
}

int validate_matrix_shape(int format, std::size_t rows, std::size_t columns) {
  if (format != GFXB_W2 && format != GFXB_W3 && format != GFXB_W4) {
    return fail(GFXB_UNSUPPORTED, "weight format must be W2G128, W3G128 or W4G128");
  }
  if (rows == 0 || rows % 16 != 0 || columns == 0 || columns % kGroup != 0) {
    return fail(GFXB_INVALID_ARGUMENT, "weight matrix needs N divisible by 16 and K divisible by 128");
  }
  if (rows > (1ull << 31) || columns > (1ull << 24)) {
    return fail(GFXB_INVALID_ARGUMENT, "weight matrix dimensions exceed the supported range");
  }
  return GFXB_OK;
}

template <int Bits, int NB>
void launch_gemv_typed(const GemvArgs& args, unsigned grid, cudaStream_t stream) {
  launch_kernel(gemv_b200_kernel<Bits, NB>, dim3(grid), dim3(256), 0, stream, 0, args);
}

template <int Bits>
void launch_gemv_bits(const GemvArgs& args, unsigned grid, cudaStream_t stream) {
  const unsigned nb = (args.batch + 7u) / 8u;
  switch (nb) {
    case 1: launch_gemv_typed<Bits, 1>(args, grid, stream); break;
    case 2: launch_gemv_typed<Bits, 2>(args, grid, stream); break;
    case 3: launch_gemv_typed<Bits, 3>(args, grid, stream); break;
    default: launch_gemv_typed<Bits, 4>(args, grid, stream); break;
  }
}

template <int Bits, bool Act8>
void launch_gfx12_bits(const std::uint8_t* w, const __half* ws, const std::uint8_t* act, const __half* as,
                       float* out, std::uint32_t rows, std::uint32_t columns, std::uint32_t batch,
                       cudaStream_t stream) {
  const unsigned nb = (batch + 7u) / 8u;
  const unsigned grid = rows / 16u;
  switch (nb) {
    case 1: gemm_gfx12_kernel<Bits, Act8, 1><<<grid, 256, 0, stream>>>(w, ws, act, as, out, rows, columns, batch); break;
    case 2: gemm_gfx12_kernel<Bits, Act8, 2><<<grid, 256, 0, stream>>>(w, ws, act, as, out, rows, columns, batch); break;
    case 3: gemm_gfx12_kernel<Bits, Act8, 3><<<grid, 256, 0, stream>>>(w, ws, act, as, out, rows, columns, batch); break;
    default: gemm_gfx12_kernel<Bits, Act8, 4><<<grid, 256, 0, stream>>>(w, ws, act, as, out, rows, columns, batch); break;
  }
}

int gfx12_gemm(int format, const std::uint8_t* w, const std::uint16_t* ws, const std::uint8_t* act,
               const std::uint16_t* as, float* out, std::size_t rows, std::size_t columns,
               unsigned batch, bool act8, cudaStream_t stream) {
  const int shape = validate_matrix_shape(format, rows, columns);
  if (shape != GFXB_OK) return shape;
  GFXB_REQUIRE(w != nullptr && ws != nullptr && act != nullptr && as != nullptr && out != nullptr,
               "gfx12 GEMM requires non-null buffers");
  GFXB_REQUIRE(batch >= 1 && batch <= 32, "gfx12 GEMM batch must be in [1, 32]");
  const auto* scales = reinterpret_cast<const __half*>(ws);
  const auto* act_scales = reinterpret_cast<const __half*>(as);
  const auto r = static_cast<std::uint32_t>(rows), k = static_cast<std::uint32_t>(columns);
  const int bits = bits_of(format);
  if (act8) {
    if (bits == 2) launch_gfx12_bits<2, true>(w, scales, act, act_scales, out, r, k, batch, stream);
    else if (bits == 3) launch_gfx12_bits<3, true>(w, scales, act, act_scales, out, r, k, batch, stream);
    else launch_gfx12_bits<4, true>(w, scales, act, act_scales, out, r, k, batch, stream);
  } else {
    if (bits == 2) launch_gfx12_bits<2, false>(w, scales, act, act_scales, out, r, k, batch, stream);
    else if (bits == 3) launch_gfx12_bits<3, false>(w, scales, act, act_scales, out, r, k, batch, stream);
    else launch_gfx12_bits<4, false>(w, scales, act, act_scales, out, r, k, batch, stream);
  }
  return launch_status("gfx12 GEMM launch failed");
}

}  // namespace

// ---------------------------------------------------------------------------
// synthetic weight generation for the engine (see HashSource)
// ---------------------------------------------------------------------------

namespace {

__device__ __forceinline__ float unit_float(std::uint64_t h) {
  return __fmul_rn(static_cast<float>(h >> 40), 1.0f / 16777216.0f);
}

__global__ void gen_tiled_scales_kernel(std::uint64_t seed, std::uint32_t tensor, RowMap rows,
                                        std::uint32_t global_groups, std::uint32_t group_offset,
                                        std::uint32_t local_rows, std::uint32_t local_groups, float lo,
                                        float hi, __half* __restrict__ tiled) {
  const std::uint64_t index = static_cast<std::uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (index >= static_cast<std::uint64_t>(local_rows) * local_groups) return;
  const std::uint32_t row = static_cast<std::uint32_t>(index / local_groups);
  const std::uint32_t group = static_cast<std::uint32_t>(index % local_groups);
  const std::uint64_t global = static_cast<std::uint64_t>(rows(row)) * global_groups + group + group_offset;
  const float value = fmaf(__fsub_rn(hi, lo), unit_float(hash3(seed, 2ull * tensor + 1, global)), lo);
  tiled[(static_cast<std::size_t>(row / 16u) * local_groups + group) * 16u + (row & 15u)] = f2h(value);
}

__global__ void gen_rowmajor_kernel(std::uint64_t seed, std::uint32_t tensor, std::uint32_t rows,
                                    std::uint32_t columns, int bits, float lo, float hi,
                                    std::uint8_t* __restrict__ codes, __half* __restrict__ scales) {
  // one thread per output byte of the reference row-major layout (W2/W4)
  const std::uint32_t per_byte = 8u / static_cast<std::uint32_t>(bits);
  const std::uint64_t bytes = static_cast<std::uint64_t>(rows) * columns / per_byte;
  const std::uint64_t index = static_cast<std::uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (index < bytes) {
    std::uint32_t value = 0;
    for (std::uint32_t i = 0; i < per_byte; ++i) {
      const std::uint64_t element = index * per_byte + i;
      const std::uint32_t code = synthetic_code(hash3(seed, 2ull * tensor, element), bits);
      value |= code << (i * static_cast<std::uint32_t>(bits));
    }
    codes[index] = static_cast<std::uint8_t>(value);
  }
  const std::uint64_t groups = static_cast<std::uint64_t>(rows) * (columns / kGroup);
  if (index < groups) {
    scales[index] = f2h(fmaf(__fsub_rn(hi, lo), unit_float(hash3(seed, 2ull * tensor + 1, index)), lo));
  }
}

__global__ void gen_bf16_kernel(std::uint64_t seed, std::uint32_t tensor, std::uint64_t offset,
                                std::uint64_t count, float lo, float hi, std::uint16_t* __restrict__ out) {
  const std::uint64_t index = static_cast<std::uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (index >= count) return;
  const float value = fmaf(__fsub_rn(hi, lo), unit_float(hash3(seed, 2ull * tensor, index + offset)), lo);
  std::uint32_t bits = __float_as_uint(value);
  bits += 0x7fffu + ((bits >> 16) & 1u);
  out[index] = static_cast<std::uint16_t>(bits >> 16);
}

}  // namespace

void scale_range(int format, float* lo, float* hi) {
  switch (format) {
    case GFXB_W2: *lo = 0.0045f; *hi = 0.0134f; break;
    case GFXB_W3: *lo = 0.0050f; *hi = 0.0150f; break;
    default: *lo = 0.0023f; *hi = 0.0069f; break;
  }
}

int generate_b200_weights(std::uint64_t seed, std::uint32_t tensor, int format, std::uint8_t* codes,
                          std::uint16_t* tiled_scales, std::size_t rows, std::size_t columns,
                          std::size_t global_columns, std::size_t column_offset, const std::uint32_t* segment_local,
                          const std::uint32_t* segment_global, std::uint32_t segments, cudaStream_t stream) {
  const int shape = validate_matrix_shape(format, rows, columns);
  if (shape != GFXB_OK) return shape;
  if (segments == 0 || segments > 3 || column_offset % kGroup != 0) {
    return fail(GFXB_INVALID_ARGUMENT, "invalid shard map");
  }
  RowMap map{};
  map.segments = segments;
  for (std::uint32_t i = 0; i < segments; ++i) {
    map.local_begin[i] = segment_local[i];
    map.global_begin[i] = segment_global[i];
  }
  const int bits = bits_of(format);
  int status = launch_write_b200(
      HashSource{seed, tensor, static_cast<std::uint32_t>(global_columns), static_cast<std::uint32_t>(column_offset),
                 map, bits},
      codes, rows, columns, bits, stream);
  if (status != GFXB_OK) return status;
  float lo, hi;
  scale_range(format, &lo, &hi);
  const std::uint64_t total = rows * (columns / kGroup);
  gen_tiled_scales_kernel<<<static_cast<unsigned>((total + 255) / 256), 256, 0, stream>>>(
      seed, tensor, map, static_cast<std::uint32_t>(global_columns / kGroup),
      static_cast<std::uint32_t>(column_offset / kGroup), static_cast<std::uint32_t>(rows),
      static_cast<std::uint32_t>(columns / kGroup), lo, hi, reinterpret_cast<__half*>(tiled_scales));
  return launch_status("synthetic scale generation failed");
}

int generate_rowmajor_weights(std::uint64_t seed, std::uint32_t tensor, int format, std::uint8_t* codes,
                              std::uint16_t* scales, std::size_t rows, std::size_t columns, cudaStream_t stream) {
  if (format != GFXB_W2 && format != GFXB_W4) return fail(GFXB_UNSUPPORTED, "row-major generation supports W2/W4");
  const int bits = bits_of(format);
  float lo, hi;
  scale_range(format, &lo, &hi);
  const std::uint64_t bytes = rows * columns * bits / 8u;
  gen_rowmajor_kernel<<<static_cast<unsigned>((bytes + 255) / 256), 256, 0, stream>>>(
      seed, tensor, static_cast<std::uint32_t>(rows), static_cast<std::uint32_t>(columns), bits, lo, hi, codes,
      reinterpret_cast<__half*>(scales));
  return launch_status("synthetic row-major generation failed");
}

int generate_bf16(std::uint64_t seed, std::uint32_t tensor, std::uint64_t offset, std::uint64_t count, float lo,
                  float hi, std::uint16_t* out, cudaStream_t stream) {
  gen_bf16_kernel<<<static_cast<unsigned>((count + 255) / 256), 256, 0, stream>>>(seed, tensor, offset, count, lo, hi,
                                                                                   out);
  return launch_status("synthetic bf16 generation failed");
}

int untile_gfx12_rowmajor(int format, const std::uint8_t* tiled_codes, const std::uint16_t* tiled_scales,
                          std::uint8_t* codes, std::uint16_t* scales, std::size_t rows, std::size_t columns,
                          cudaStream_t stream) {
  if (format != GFXB_W2 && format != GFXB_W4) return fail(GFXB_UNSUPPORTED, "row-major untiling takes W2 or W4 codes");
  if (rows == 0 || rows % 16 != 0 || columns == 0 || columns % kGroup != 0) {
    return fail(GFXB_INVALID_ARGUMENT, "untiling requires N divisible by 16 and K by 128");
  }
  const std::uint32_t groups = static_cast<std::uint32_t>(columns / kGroup);
  const std::uint32_t fragment = format == GFXB_W2 ? 8u : 16u;
  const std::uint64_t bytes = static_cast<std::uint64_t>(rows) * groups * 4u * fragment;
  untile_gfx12_kernel<<<static_cast<unsigned>((bytes + 255) / 256), 256, 0, stream>>>(tiled_codes, codes, bytes, groups,
                                                                                       fragment);
  GFXB_TRY(launch_status("untiling launch failed"));
  const std::uint64_t count = static_cast<std::uint64_t>(rows) * groups;
  untile_scales_kernel<<<static_cast<unsigned>((count + 255) / 256), 256, 0, stream>>>(
      reinterpret_cast<const __half*>(tiled_scales), reinterpret_cast<__half*>(scales), count, groups);
  return launch_status("scale untiling launch failed");
}

int read_gemv_error(std::uint32_t* value, bool clear) {
  cudaError_t error = cudaMemcpyFromSymbol(value, g_gemv_error, sizeof(std::uint32_t));
  if (error == cudaSuccess && clear) {
    const std::uint32_t zero = 0;
    error = cudaMemcpyToSymbol(g_gemv_error, &zero, sizeof zero);
  }
  if (error != cudaSuccess) {
    set_error_cuda(error, "device error word access failed");
    return GFXB_CUDA_ERROR;
  }
  return GFXB_OK;
}

}  // namespace gfxb

using namespace gfxb;

extern "C" int gfxb_repack_rowmajor_to_b200(int format, const std::uint8_t* rowmajor_codes,
                                            std::uint8_t* b200_codes, std::size_t rows,
                                            std::size_t columns, void* stream) {
  const int shape = validate_matrix_shape(format, rows, columns);
  if (shape != GFXB_OK) return shape;
  GFXB_REQUIRE(rowmajor_codes != nullptr && b200_codes != nullptr, "repack requires non-null buffers");
  const int bits = bits_of(format);
  return launch_write_b200(RowMajorSource{rowmajor_codes, static_cast<std::uint32_t>(columns), bits},
                           b200_codes, rows, columns, bits, as_stream(stream));
}

extern "C" int gfxb_repack_gfx12_to_b200(int format, const std::uint8_t* gfx12_codes,
                                         std::uint8_t* b200_codes, std::size_t rows,
                                         std::size_t columns, void* stream) {
  const int shape = validate_matrix_shape(format, rows, columns);
  if (shape != GFXB_OK) return shape;
  GFXB_REQUIRE(gfx12_codes != nullptr && b200_codes != nullptr, "repack requires non-null buffers");
  const int bits = bits_of(format);
  return launch_write_b200(Gfx12Source{gfx12_codes, static_cast<std::uint32_t>(columns), bits},
                           b200_codes, rows, columns, bits, as_stream(stream));
}

extern "C" int gfxb_tile_scales(const std::uint16_t* rowmajor_scales, std::uint16_t* tiled_scales,
                                std::size_t rows, std::size_t columns, void* stream) {
  GFXB_REQUIRE(rowmajor_scales != nullptr && tiled_scales != nullptr, "scale tiling requires buffers");
  GFXB_REQUIRE(rows % 16 == 0 && rows > 0 && columns % kGroup == 0 && columns > 0,
               "scale tiling needs N divisible by 16 and K divisible by 128");
  const std::uint64_t total = rows * (columns / kGroup);
  tile_scales_kernel<<<static_cast<unsigned>((total + 255) / 256), 256, 0, as_stream(stream)>>>(
      reinterpret_cast<const __half*>(rowmajor_scales), reinterpret_cast<__half*>(tiled_scales),
      static_cast<std::uint32_t>(rows), static_cast<std::uint32_t>(columns / kGroup));
  return launch_status("scale tiling launch failed");
}

extern "C" int gfxb_pack_activation(int activation_bits, const std::uint16_t* input, std::int8_t* codes,
                                    std::uint16_t* scales, std::int32_t* sums, std::uint8_t* packed_a4,
                                    std::size_t columns, unsigned batch, void* stream) {
  GFXB_REQUIRE(activation_bits == 4 || activation_bits == 8, "activation bits must be 4 or 8");
  GFXB_REQUIRE(input != nullptr && codes != nullptr && scales != nullptr && sums != nullptr,
               "activation packing requires non-null buffers");
  GFXB_REQUIRE(columns > 0 && columns % kGroup == 0 && batch >= 1 && batch <= 32,
               "activation packing requires batch in [1,32] and K divisible by 128");
  const std::uint32_t groups = static_cast<std::uint32_t>(columns / kGroup);
  const dim3 grid(groups * batch);
  const auto* in = reinterpret_cast<const __half*>(input);
  auto* s = reinterpret_cast<__half*>(scales);
  if (activation_bits == 4) {
    launch_kernel(pack_activation_kernel<4>, grid, dim3(128), 0, as_stream(stream), 0, in, codes, s, sums,
                  packed_a4, static_cast<std::uint32_t>(columns), groups);
  } else {
    launch_kernel(pack_activation_kernel<8>, grid, dim3(128), 0, as_stream(stream), 0, in, codes, s, sums,
                  static_cast<std::uint8_t*>(nullptr), static_cast<std::uint32_t>(columns), groups);
  }
  return launch_status("activation packing launch failed");
}

namespace gfxb {
int lowbit_gemv(int format, const gfxb_gemv_matrix* matrices, unsigned matrix_count, const std::int8_t* act_codes,
                const std::uint16_t* act_scales, const std::int32_t* act_sums, std::size_t columns,
                std::size_t act_stride, unsigned batch, cudaStream_t stream) {
  GFXB_REQUIRE(matrices != nullptr && matrix_count >= 1 && matrix_count <= 4,
               "GEMV takes between one and four matrices");
  GFXB_REQUIRE(act_codes != nullptr && act_scales != nullptr && act_sums != nullptr,
               "GEMV requires an activation pack");
  GFXB_REQUIRE(batch >= 1 && batch <= 32, "GEMV batch must be in [1, 32]");
  GemvArgs args{};
  std::uint64_t total_tiles = 0;
  for (unsigned i = 0; i < matrix_count; ++i) {
    const int shape = validate_matrix_shape(format, matrices[i].rows, columns);
    if (shape != GFXB_OK) return shape;
    GFXB_REQUIRE(matrices[i].codes != nullptr && matrices[i].scales != nullptr &&
                     matrices[i].output != nullptr,
                 "GEMV matrix binding is invalid");
    args.m[i].codes = matrices[i].codes;
    args.m[i].scales = reinterpret_cast<const __half*>(matrices[i].scales);
    args.m[i].output = matrices[i].output;
    args.m[i].tiles = static_cast<std::uint32_t>(matrices[i].rows / 16);
    args.m[i].output_f16 = matrices[i].output_f16 != 0;
    total_tiles += args.m[i].tiles;
  }
  GFXB_REQUIRE(total_tiles <= 0x7fffffffull, "GEMV grid is too large");
  args.count = matrix_count;
  args.act = act_codes;
  args.act_scales = reinterpret_cast<const __half*>(act_scales);
  args.act_sums = act_sums;
  args.columns = static_cast<std::uint32_t>(columns);
  args.groups = static_cast<std::uint32_t>(columns / kGroup);
  args.batch = batch;
  args.act_stride = act_stride == 0 ? static_cast<std::uint32_t>(columns) : static_cast<std::uint32_t>(act_stride);
  GFXB_REQUIRE(args.act_stride >= args.columns && args.act_stride % kGroup == 0, "activation stride is invalid");
  const int bits = bits_of(format);
  const unsigned grid = static_cast<unsigned>(total_tiles);
  static const bool force_v1 = env_value("GFXB_GEMV_V1", 0) != 0;
  static const std::uint32_t pipe_mode = env_value("GFXB_GEMV_PIPE", 1);  // 0: never, 1: tall matrices, 2: always
  static const bool lean = env_value("GFXB_GEMV_LEAN", 1) != 0;           // the persistent kernel for one token
  if (batch == 1 && lean && !force_v1) {
    const int status = bits == 2   ? launch_lean<2>(args, grid, stream)
                       : bits == 3 ? launch_lean<3>(args, grid, stream)
                                   : launch_lean<4>(args, grid, stream);
    if (status != kNoStreamPath) return status;
  }
  if (batch <= 8 && batch < tuning().tall_cascade && !force_v1 && pipe_mode != 0) {
    // tall matrices (one CTA per tile would need several waves) whose two stages leave room for two CTAs per SM
    const PipeLayout pipe = pipe_layout(bits, args.groups, batch);
    if ((pipe_mode == 2 || total_tiles >= tuning().min_tiles_p1) && pipe.total <= 100u * 1024u) {
      if (bits == 2) return launch_pipe<2>(args, grid, stream);
      if (bits == 3) return launch_pipe<3>(args, grid, stream);
      return launch_pipe<4>(args, grid, stream);
    }
  }
  if (batch <= 16 && !force_v1) {
    const int status = bits == 2   ? launch_stream<2>(args, grid, stream)
                       : bits == 3 ? launch_stream<3>(args, grid, stream)
                                   : launch_stream<4>(args, grid, stream);
    if (status != kNoStreamPath) return status;
  }
  if (bits == 2) launch_gemv_bits<2>(args, grid, stream);
  else if (bits == 3) launch_gemv_bits<3>(args, grid, stream);
  else launch_gemv_bits<4>(args, grid, stream);
  return launch_status("low-bit GEMV launch failed");
}
}  // namespace gfxb

extern "C" int gfxb_lowbit_gemv(int format, const gfxb_gemv_matrix* matrices, unsigned matrix_count,
                                const std::int8_t* act_codes, const std::uint16_t* act_scales,
                                const std::int32_t* act_sums, std::size_t columns, unsigned batch,
                                void* stream) {
  return gfxb::lowbit_gemv(format, matrices, matrix_count, act_codes, act_scales, act_sums, columns, 0, batch,
                           as_stream(stream));
}

extern "C" int gfxb_quantize_activation_i4(const std::uint16_t* input, std::uint8_t* packed_output,
                                           std::uint16_t* scales, std::size_t columns, unsigned batch,
                                           void* stream) {
  GFXB_REQUIRE(input != nullptr && packed_output != nullptr && scales != nullptr && columns > 0 &&
                   columns % kGroup == 0 && batch >= 1 && batch <= 32,
               "A4 quantization requires non-null buffers, batch in [1,32], and K divisible by 128");
  const std::uint32_t groups = static_cast<std::uint32_t>(columns / kGroup);
  quantize_reference_kernel<4><<<groups * batch, 128, 0, as_stream(stream)>>>(
      reinterpret_cast<const __half*>(input), packed_output, reinterpret_cast<__half*>(scales),
      static_cast<std::uint32_t>(columns), groups);
  return launch_status("A4 activation quantization launch failed");
}

extern "C" int gfxb_quantize_activation_i8(const std::uint16_t* input, std::int8_t* quantized_output,
                                           std::uint16_t* scales, std::size_t columns, unsigned batch,
                                           void* stream) {
  GFXB_REQUIRE(input != nullptr && quantized_output != nullptr && scales != nullptr && columns > 0 &&
                   columns % kGroup == 0 && batch >= 1 && batch <= 32,
               "A8 quantization requires non-null buffers, batch in [1,32], and K divisible by 128");
  const std::uint32_t groups = static_cast<std::uint32_t>(columns / kGroup);
  quantize_reference_kernel<8><<<groups * batch, 128, 0, as_stream(stream)>>>(
      reinterpret_cast<const __half*>(input), reinterpret_cast<std::uint8_t*>(quantized_output),
      reinterpret_cast<__half*>(scales), static_cast<std::uint32_t>(columns), groups);
  return launch_status("A8 activation quantization launch failed");
}

extern "C" int gfxb_gfx12_i4_gemm(int format, const std::uint8_t* tiled_weights,
                                  const std::uint16_t* tiled_weight_scales,
                                  const std::uint8_t* packed_activations,
                                  const std::uint16_t* activation_scales, float* output, std::size_t rows,
                                  std::size_t columns, unsigned batch, int sequential_w3, void* stream) {
  if (format == GFXB_W3 && !sequential_w3) {
    return fail(GFXB_UNSUPPORTED, "only the sequential W3 fragment order is supported");
  }
  return gfx12_gemm(format, tiled_weights, tiled_weight_scales, packed_activations, activation_scales,
                    output, rows, columns, batch, false, as_stream(stream));
}

extern "C" int gfxb_gfx12_i8_gemm(int format, const std::uint8_t* tiled_weights,
                                  const std::uint16_t* tiled_weight_scales,
                                  const std::int8_t* quantized_activations,
                                  const std::uint16_t* activation_scales, float* output, std::size_t rows,
                                  std::size_t columns, unsigned batch, void* stream) {
  return gfx12_gemm(format, tiled_weights, tiled_weight_scales,
                    reinterpret_cast<const std::uint8_t*>(quantized_activations), activation_scales,
                    output, rows, columns, batch, true, as_stream(stream));
}
