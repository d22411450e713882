// FP16-activation dequant-GEMV for sm_100a: W2/W3/W4 group-128 weights x
// fp16 activations on the f16 tensor cores (mma.sync m16n8k16, fp32
// accumulate).
//
// Replaces the reference's gfx12_f16_gemm (lowbit_gemv.hip:757-834,
// launched by launch_gfx12_f16_gemm :1328-1363), its `--activation f16`
// path. The reference arithmetic: every weight is dequantized to fp16 as
// fp16(q * scale) with the fp16 group scale widened to fp32, then multiplied
// by the fp16 activation with fp32 accumulation on the matrix cores. Here q
// is formed exactly in fp16 from the stored code and multiplied by the scale
// with one fp16 rounding (__hmul2), which equals fp16(fp32(q) * fp32(scale))
// because |q| <= 8 makes the fp32 product exact. The fp32 summation order
// inside the tensor cores is the hardware's, as on the reference GPU, so
// outputs are compared to an exact (double) sum within a relative tolerance.
//
// Two weight layouts share one kernel body:
//  - b200 (gfxb_lowbit_gemv_f16): lane L (g = L/4, t = L%4) of a warp holds,
//    for k-step s, codes of rows g and g+8 at k = 32s + 4t + j (register
//    pair 0/1) and k = 32s + 16 + 4t + j (pair 2/3), j = 0..3;
//  - gfx12 tiled (gfxb_gfx12_f16_gemm, the reference artifact layout,
//    quantization.cpp:253-318): the same lane takes k = 32s + 8t + j for
//    j = 0..3 and 4..7, which is one contiguous piece of each row fragment.
// A dot product does not depend on how k is dealt out to the lanes, only on
// activations being fetched at the same k as the weights.
#include <algorithm>
#include <cstdint>

#include "codec.cuh"
#include "common.cuh"

namespace gfxb {
namespace {

constexpr unsigned kF16Warps = 8;

struct F16Matrix {
  const std::uint8_t* codes;
  const __half* scales;
  void* output;
  std::uint32_t tiles;
  std::uint32_t output_f16;
};

struct F16GemvArgs {
  F16Matrix m[4];
  std::uint32_t count;
  const __half* act;   // [B][K] fp16
  std::uint32_t groups;
  std::uint32_t batch;
  std::uint32_t act_stride;
};

__device__ __forceinline__ F16Matrix select_f16_matrix(const F16GemvArgs& args, std::uint32_t& tile) {
  F16Matrix m = args.m[0];
#pragma unroll
  for (int i = 1; i < 4; ++i) {
    if (static_cast<std::uint32_t>(i) < args.count && tile >= m.tiles) {
      tile -= m.tiles;
      m = args.m[i];
    }
  }
  return m;
}

__device__ __forceinline__ void mma_f16_16816(float (&c)[4], const std::uint32_t (&a)[4], std::uint32_t b0,
                                              std::uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Two byte codes (bytes `sel` of `word`, unsigned u = (q - beta) / alpha) ->
// fp16 pair of fp16(q * scale). 0x6400 | u is the fp16 value 1024 + u.
template <int Bits>
__device__ __forceinline__ std::uint32_t dequant_pair(std::uint32_t word, std::uint32_t sel, __half2 scale) {
  const std::uint32_t biased = __byte_perm(word, 0x64646464u, sel);
  const __half2 h = *reinterpret_cast<const __half2*>(&biased);
  __half2 q;
  if constexpr (Bits == 2) {
    // 2u - 3 from u = h - 1024 (2051 itself is not an fp16 value)
    q = __hfma2(__hsub2(h, __float2half2_rn(1024.0f)), __float2half2_rn(2.0f), __float2half2_rn(-3.0f));
  } else if constexpr (Bits == 3) {
    q = __hsub2(h, __float2half2_rn(1028.0f));  // u - 4
  } else {
    q = __hsub2(h, __float2half2_rn(1032.0f));  // u - 8
  }
  const __half2 w = __hmul2(q, scale);
  return *reinterpret_cast<const std::uint32_t*>(&w);
}

// Four byte codes of row g (word_lo) and row g+8 (word_hi) -> the A fragment
// of one m16n8k16: (row g, k 0-1), (row g+8, k 0-1), (row g, k 2-3), (row g+8, k 2-3).
template <int Bits>
__device__ __forceinline__ void a_fragment(std::uint32_t word_lo, std::uint32_t word_hi, __half2 s_lo, __half2 s_hi,
                                           std::uint32_t (&a)[4]) {
  a[0] = dequant_pair<Bits>(word_lo, 0x4140u, s_lo);
  a[1] = dequant_pair<Bits>(word_hi, 0x4140u, s_hi);
  a[2] = dequant_pair<Bits>(word_lo, 0x4342u, s_lo);
  a[3] = dequant_pair<Bits>(word_hi, 0x4342u, s_hi);
}

// ---- layouts: one group's codes for a lane -> words[s][r] (4 byte codes each)
// words[s][0] = row g, first k-quad; [1] = row g+8, first quad; [2] = row g,
// second quad; [3] = row g+8, second quad. kq(s, h) = the quad's first k.

struct B200Layout {
  template <int Bits>
  struct Fetch {
    LaneWords<Bits> w;
  };
  template <int Bits>
  __device__ __forceinline__ static void load(const std::uint8_t* tile_codes, std::uint32_t group,
                                              std::uint32_t groups, unsigned lane, Fetch<Bits>& f) {
    (void)groups;
    load_lane(tile_codes + static_cast<std::size_t>(group) * Bits * 256u, lane, f.w);
  }
  template <int Bits>
  __device__ __forceinline__ static void words(const Fetch<Bits>& f, unsigned lane, std::uint32_t (&w)[4][4]) {
    (void)lane;
    unpack(f.w, w);
  }
  __device__ __forceinline__ static std::uint32_t quad(std::uint32_t s, std::uint32_t h, unsigned tq) {
    return 32u * s + 16u * h + 4u * tq;
  }
};

// Spread four 3-bit (12-bit field), 4-bit (16-bit field) or 2-bit (8-bit
// field) codes into four bytes.
__device__ __forceinline__ std::uint32_t spread_codes3(std::uint32_t f) {
  f &= 0xfffu;
  const std::uint32_t x = (f & 0x3fu) | ((f & 0xfc0u) << 10);
  return (x & 0x00070007u) | ((x & 0x00380038u) << 5);
}
__device__ __forceinline__ std::uint32_t spread_codes4(std::uint32_t f) {
  f &= 0xffffu;
  const std::uint32_t x = (f & 0xffu) | ((f & 0xff00u) << 8);
  return (x & 0x000f000fu) | ((x & 0x00f000f0u) << 4);
}
__device__ __forceinline__ std::uint32_t spread_codes2(std::uint32_t f) {
  f &= 0xffu;
  const std::uint32_t x = (f & 0xfu) | ((f & 0xf0u) << 12);
  return (x & 0x00030003u) | ((x & 0x000c000cu) << 6);
}

// gfx12 tiled layout: per (tile, group) [4 k-tiles][16 rows][fragment], the
// fragment holding the row's 32 codes of the k-tile (W2 8 bytes, code i at
// bit 2i; W3 12 bytes, bit 3i; W4 16 bytes, nibble i). Codes are the
// reference's (W2 (q+3)/2, W3 q+4, W4 two's-complement nibble), turned into
// the offset form u here (W4: u = code ^ 8).
struct Gfx12Layout {
  template <int Bits>
  struct Fetch {
    std::uint32_t piece[4][2];  // [k-tile][row g / g+8]: the lane's 8 codes
  };
  template <int Bits>
  __device__ __forceinline__ static void load(const std::uint8_t* tile_codes, std::uint32_t group,
                                              std::uint32_t groups, unsigned lane, Fetch<Bits>& f) {
    (void)groups;
    constexpr std::uint32_t kFragment = Bits == 2 ? 8u : (Bits == 3 ? 12u : 16u);
    const unsigned gl = lane >> 2, tq = lane & 3u;
    const std::uint8_t* base = tile_codes + static_cast<std::size_t>(group) * 64u * kFragment;
#pragma unroll
    for (unsigned s = 0; s < 4; ++s) {
#pragma unroll
      for (unsigned r = 0; r < 2; ++r) {
        const std::uint8_t* fragment = base + (s * 16u + gl + 8u * r) * kFragment;
        if constexpr (Bits == 4) {
          f.piece[s][r] = __ldg(reinterpret_cast<const std::uint32_t*>(fragment) + tq);
        } else if constexpr (Bits == 2) {
          f.piece[s][r] = __ldg(reinterpret_cast<const std::uint16_t*>(fragment) + tq);
        } else {
          // bits 24t .. 24t+23 of the 96-bit fragment (4-byte aligned words)
          const std::uint32_t* w = reinterpret_cast<const std::uint32_t*>(fragment);
          const std::uint32_t word = (24u * tq) >> 5, shift = (24u * tq) & 31u;
          const std::uint32_t lo = __ldg(w + word);
          const std::uint32_t hi = word + 1u < 3u ? __ldg(w + word + 1u) : 0u;
          f.piece[s][r] = __funnelshift_r(lo, hi, shift) & 0xffffffu;
        }
      }
    }
  }
  template <int Bits>
  __device__ __forceinline__ static void words(const Fetch<Bits>& f, unsigned lane, std::uint32_t (&w)[4][4]) {
    (void)lane;
#pragma unroll
    for (unsigned s = 0; s < 4; ++s) {
#pragma unroll
      for (unsigned r = 0; r < 2; ++r) {
        const std::uint32_t p = f.piece[s][r];
        std::uint32_t first, second;
        if constexpr (Bits == 4) {
          first = spread_codes4(p) ^ 0x08080808u;
          second = spread_codes4(p >> 16) ^ 0x08080808u;
        } else if constexpr (Bits == 3) {
          first = spread_codes3(p);
          second = spread_codes3(p >> 12);
        } else {
          first = spread_codes2(p);
          second = spread_codes2(p >> 8);
        }
        w[s][r] = first;
        w[s][2u + r] = second;
      }
    }
  }
  __device__ __forceinline__ static std::uint32_t quad(std::uint32_t s, std::uint32_t h, unsigned tq) {
    return 32u * s + 8u * tq + 4u * h;
  }
};

// One CTA (8 warps) per 16-row tile; warp w accumulates groups w, w+8, ...
// for up to NB blocks of 8 tokens in fp32 tensor-core accumulators, with the
// next group's weights prefetched. Partials of the 8 warps are then added in
// warp order by one thread per (row, token).
template <class Layout, int Bits, int NB>
__global__ __launch_bounds__(256) void gemv_f16_kernel(const F16GemvArgs args) {
  std::uint32_t tile = blockIdx.x;
  const F16Matrix m = select_f16_matrix(args, tile);
  const unsigned warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
  const unsigned gl = lane >> 2, tq = lane & 3u;
  const std::uint32_t G = args.groups, B = args.batch;
  const std::uint8_t* tile_codes = m.codes + static_cast<std::size_t>(tile) * G * Bits * 256u;
  const __half* tile_scales = m.scales + static_cast<std::size_t>(tile) * G * 16u;
  __shared__ float partial[kF16Warps][16][NB * 8];

  float acc[NB][4];
#pragma unroll
  for (int nb = 0; nb < NB; ++nb) {
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[nb][i] = 0.0f;
  }
  const __half* token_act[NB];
#pragma unroll
  for (int nb = 0; nb < NB; ++nb) {
    const std::uint32_t token = min(static_cast<std::uint32_t>(nb) * 8u + gl, B - 1u);
    token_act[nb] = args.act + static_cast<std::size_t>(token) * args.act_stride;
  }

  typename Layout::template Fetch<Bits> cur, next;
  if (warp < G) Layout::template load<Bits>(tile_codes, warp, G, lane, cur);
  for (std::uint32_t g = warp; g < G; g += kF16Warps) {
    if (g + kF16Warps < G) Layout::template load<Bits>(tile_codes, g + kF16Warps, G, lane, next);
    const __half2 s_lo = __half2half2(tile_scales[g * 16u + gl]);
    const __half2 s_hi = __half2half2(tile_scales[g * 16u + gl + 8u]);
    std::uint32_t w[4][4];
    Layout::template words<Bits>(cur, lane, w);
#pragma unroll
    for (std::uint32_t s = 0; s < 4; ++s) {
#pragma unroll
      for (std::uint32_t h = 0; h < 2; ++h) {
        std::uint32_t a[4];
        a_fragment<Bits>(w[s][2u * h], w[s][2u * h + 1u], s_lo, s_hi, a);
        const std::uint32_t k = g * kGroup + Layout::quad(s, h, tq);
#pragma unroll
        for (int nb = 0; nb < NB; ++nb) {
          const uint2 x = __ldg(reinterpret_cast<const uint2*>(token_act[nb] + k));
          mma_f16_16816(acc[nb], a, x.x, x.y);
        }
      }
    }
    cur = next;
  }
#pragma unroll
  for (int nb = 0; nb < NB; ++nb) {
    const unsigned t0 = nb * 8u + 2u * tq;
    partial[warp][gl][t0] = acc[nb][0];
    partial[warp][gl][t0 + 1u] = acc[nb][1];
    partial[warp][gl + 8u][t0] = acc[nb][2];
    partial[warp][gl + 8u][t0 + 1u] = acc[nb][3];
  }
  __syncthreads();
  const std::uint32_t rows = m.tiles * 16u;
  for (std::uint32_t pair = threadIdx.x; pair < 16u * B; pair += blockDim.x) {
    const std::uint32_t row = pair & 15u, token = pair >> 4;
    float sum = 0.0f;
#pragma unroll
    for (unsigned w8 = 0; w8 < kF16Warps; ++w8) sum = __fadd_rn(sum, partial[w8][row][token]);
    const std::size_t index = static_cast<std::size_t>(token) * rows + tile * 16u + row;
    if (m.output_f16) {
      static_cast<__half*>(m.output)[index] = f2h(sum);
    } else {
      static_cast<float*>(m.output)[index] = sum;
    }
  }
}

template <class Layout, int Bits>
void launch_f16_bits(const F16GemvArgs& args, unsigned grid, cudaStream_t stream) {
  const unsigned nb = (args.batch + 7u) / 8u;
  if (nb == 1) gemv_f16_kernel<Layout, Bits, 1><<<grid, 256, 0, stream>>>(args);
  else if (nb == 2) gemv_f16_kernel<Layout, Bits, 2><<<grid, 256, 0, stream>>>(args);
  else if (nb == 3) gemv_f16_kernel<Layout, Bits, 3><<<grid, 256, 0, stream>>>(args);
  else gemv_f16_kernel<Layout, Bits, 4><<<grid, 256, 0, stream>>>(args);
}

template <class Layout>
int launch_f16(int format, const F16GemvArgs& args, unsigned grid, cudaStream_t stream) {
  const int bits = bits_of(format);
  if (bits == 2) launch_f16_bits<Layout, 2>(args, grid, stream);
  else if (bits == 3) launch_f16_bits<Layout, 3>(args, grid, stream);
  else launch_f16_bits<Layout, 4>(args, grid, stream);
  return launch_status("fp16-activation GEMV launch failed");
}

bool aligned(const void* pointer, std::uintptr_t alignment) {
  return reinterpret_cast<std::uintptr_t>(pointer) % alignment == 0;
}

int check_format(int format) {
  return format == GFXB_W2 || format == GFXB_W3 || format == GFXB_W4
             ? GFXB_OK
             : fail(GFXB_UNSUPPORTED, "fp16-activation GEMV supports W2, W3 and W4 group-128 weights");
}

}  // namespace
}  // namespace gfxb

using namespace gfxb;

extern "C" int gfxb_lowbit_gemv_f16(int format, const gfxb_gemv_matrix* matrices, unsigned matrix_count,
                                    const std::uint16_t* activations, std::size_t columns, unsigned batch,
                                    void* stream) {
  GFXB_REQUIRE(matrices != nullptr && matrix_count >= 1 && matrix_count <= 4,
               "GEMV takes between one and four matrices");
  GFXB_REQUIRE(activations != nullptr && aligned(activations, 8), "GEMV requires 8-byte aligned fp16 activations");
  GFXB_REQUIRE(batch >= 1 && batch <= 32, "GEMV batch must be in [1, 32]");
  GFXB_REQUIRE(columns != 0 && columns % kGroup == 0 && columns <= 0xffffffffull, "GEMV K must be a multiple of 128");
  GFXB_TRY(check_format(format));
  F16GemvArgs args{};
  std::uint64_t total_tiles = 0;
  for (unsigned i = 0; i < matrix_count; ++i) {
    const gfxb_gemv_matrix& mat = matrices[i];
    GFXB_REQUIRE(mat.codes != nullptr && mat.scales != nullptr && mat.output != nullptr && mat.rows != 0 &&
                     mat.rows % 16 == 0,
                 "GEMV matrix binding is invalid (rows must be a positive multiple of 16)");
    GFXB_REQUIRE(aligned(mat.codes, 16) && aligned(mat.scales, 2) && aligned(mat.output, 4),
                 "GEMV weight codes must be 16-byte aligned");
    args.m[i].codes = mat.codes;
    args.m[i].scales = reinterpret_cast<const __half*>(mat.scales);
    args.m[i].output = mat.output;
    args.m[i].tiles = static_cast<std::uint32_t>(mat.rows / 16);
    args.m[i].output_f16 = mat.output_f16 != 0;
    total_tiles += args.m[i].tiles;
  }
  GFXB_REQUIRE(total_tiles <= 0x7fffffffull, "GEMV grid is too large");
  args.count = matrix_count;
  args.act = reinterpret_cast<const __half*>(activations);
  args.groups = static_cast<std::uint32_t>(columns / kGroup);
  args.batch = batch;
  args.act_stride = static_cast<std::uint32_t>(columns);
  return launch_f16<B200Layout>(format, args, static_cast<unsigned>(total_tiles), as_stream(stream));
}

extern "C" int gfxb_gfx12_f16_gemm(int format, const std::uint8_t* tiled_weights,
                                   const std::uint16_t* tiled_weight_scales, const std::uint16_t* activations,
                                   float* output, std::size_t rows, std::size_t columns, unsigned batch,
                                   void* stream) {
  if (tiled_weights == nullptr || tiled_weight_scales == nullptr || activations == nullptr || output == nullptr ||
      rows == 0 || rows % 16 != 0 || columns == 0 || columns % kGroup != 0 || batch == 0 || batch > 32 ||
      rows / 16 > 0x7fffffffull || columns > 0xffffffffull) {
    return fail(GFXB_INVALID_ARGUMENT,
                "FP16 GEMM requires tiled buffers, N divisible by 16, K divisible by 128, and batch in [1,32]");
  }
  GFXB_REQUIRE(aligned(tiled_weights, 4) && aligned(tiled_weight_scales, 2) && aligned(activations, 8) &&
                   aligned(output, 4),
               "FP16 GEMM buffers are misaligned (weights 4, activations 8 bytes)");
  GFXB_TRY(check_format(format));
  F16GemvArgs args{};
  args.m[0].codes = tiled_weights;
  args.m[0].scales = reinterpret_cast<const __half*>(tiled_weight_scales);
  args.m[0].output = output;
  args.m[0].tiles = static_cast<std::uint32_t>(rows / 16);
  args.count = 1;
  args.act = reinterpret_cast<const __half*>(activations);
  args.groups = static_cast<std::uint32_t>(columns / kGroup);
  args.batch = batch;
  args.act_stride = static_cast<std::uint32_t>(columns);
  return launch_f16<Gfx12Layout>(format, args, static_cast<unsigned>(rows / 16), as_stream(stream));
}
