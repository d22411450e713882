// Group-128 weight packing on the device: the reference's host packing rules
// (src/quantization.cpp) as sm_100a kernels, and the conversion of fp32 or
// bf16 weights into the layouts the engines load.
//
//  - quantize_group128 (quantization.cpp:163-220): per (row, 128-column
//    group) one thread runs choose_scale (:67-92; amax / {3, 4, 8}, four
//    least-squares refits with double accumulators in column order, floor at
//    FLT_MIN, 1 for an all-zero group) and encode_value (:29-46), then writes
//    the group's row-major codes (store_code, :94-124) as whole words. The
//    CTA's 128 groups are one contiguous 64 KB range of the input, staged in
//    shared memory with coalesced loads; each thread then reads its group six
//    times from a padded shared-memory row.
//  - tile_group128_for_gfx12 (:253-318): one thread per 16-row x 32-column
//    fragment (W3 re-packed from bit planes to sequential 3-bit codes).
//  - dequantize_group128 (:222-251): one thread per weight.
// Every float operation is the reference's (IEEE division, round-half-even
// nearbyint, double products and sums in the same order), so codes and
// scales are bit-identical to the reference's host code.
#include <cfloat>
#include <cmath>

#include "common.cuh"
#include "gfxb/artifact.h"

namespace gfxb {
namespace {

constexpr unsigned kItems = 128;           // (row, group) items per CTA, one per thread
constexpr unsigned kRowPitch = kGroup + 1;  // padded shared-memory row: thread t, column c at t*129 + c
constexpr std::size_t kStageBytes = std::size_t{kItems} * kRowPitch * sizeof(float);

__device__ std::uint32_t bf16_bits_to_float_bits(std::uint16_t value) { return static_cast<std::uint32_t>(value) << 16; }

// quantization.cpp:15-27: the closest of {-3, -1, 1, 3}, the lower one on ties.
__device__ __forceinline__ int nearest_w2(float normalized) {
  int best = -3;
  float best_error = __int_as_float(0x7f800000);
  for (int level = -3; level <= 3; level += 2) {
    const float error = fabsf(__fsub_rn(normalized, static_cast<float>(level)));
    if (error < best_error) {
      best = level;
      best_error = error;
    }
  }
  return best;
}

// encode_value then decode_value (quantization.cpp:29-56): the signed level.
template <int Format>
__device__ __forceinline__ int quantize_level(float value, float scale) {
  const float normalized = scale == 0.0f ? 0.0f : __fdiv_rn(value, scale);
  if constexpr (Format == GFXB_W2) {
    return nearest_w2(normalized);
  } else {
    constexpr int lo = Format == GFXB_W3 ? -4 : -8;
    constexpr int hi = Format == GFXB_W3 ? 3 : 7;
    return min(max(static_cast<int>(rintf(normalized)), lo), hi);
  }
}

template <int Format>
__host__ __device__ constexpr float divisor() {
  return Format == GFXB_W2 ? 3.0f : (Format == GFXB_W3 ? 4.0f : 8.0f);
}

template <int Format>
__host__ __device__ constexpr unsigned group_words() {
  return Format == GFXB_W2 ? 8u : (Format == GFXB_W3 ? 12u : 16u);
}

template <int Format, typename Input>
__global__ __launch_bounds__(kItems) void quantize_group128_kernel(const Input* __restrict__ weights,
                                                                   std::uint64_t items,
                                                                   std::uint8_t* __restrict__ codes,
                                                                   float* __restrict__ scales,
                                                                   std::uint32_t* __restrict__ non_finite) {
  extern __shared__ float stage[];
  const std::uint64_t first = static_cast<std::uint64_t>(blockIdx.x) * kItems;
  const unsigned count = items - first < kItems ? static_cast<unsigned>(items - first) : kItems;
  // coalesced staging of the CTA's count * 128 consecutive values
  const Input* source = weights + first * kGroup;
  for (unsigned i = threadIdx.x; i < count * kGroup; i += kItems) {
    float value;
    if constexpr (sizeof(Input) == 2) {
      value = __uint_as_float(bf16_bits_to_float_bits(source[i]));
    } else {
      value = source[i];
    }
    stage[(i / kGroup) * kRowPitch + (i % kGroup)] = value;
  }
  __syncthreads();
  if (threadIdx.x >= count) return;
  const float* v = stage + threadIdx.x * kRowPitch;
  // quantization.cpp:186-197: the largest finite magnitude
  float maximum = 0.0f;
  bool finite = true;
  for (unsigned c = 0; c < kGroup; ++c) {
    const float value = v[c];
    if (!isfinite(value)) {
      finite = false;
      continue;
    }
    const float magnitude = fabsf(value);
    if (maximum < magnitude) maximum = magnitude;
  }
  if (!finite) atomicOr(non_finite, 1u);
  // choose_scale (quantization.cpp:67-92)
  float scale = 1.0f;
  if (maximum != 0.0f) {
    scale = __fdiv_rn(maximum, divisor<Format>());
    for (int iteration = 0; iteration < 4; ++iteration) {
      double numerator = 0.0, denominator = 0.0;
      for (unsigned c = 0; c < kGroup; ++c) {
        const int level = quantize_level<Format>(v[c], scale);
        numerator = __dadd_rn(numerator, __dmul_rn(static_cast<double>(v[c]), static_cast<double>(level)));
        denominator = __dadd_rn(denominator, __dmul_rn(static_cast<double>(level), static_cast<double>(level)));
      }
      if (denominator == 0.0) break;
      scale = __double2float_rn(__ddiv_rn(numerator, denominator));
    }
    if (scale < FLT_MIN) scale = FLT_MIN;  // std::max(scale, FLT_MIN), NaN kept as it is
  }
  const std::uint64_t item = first + threadIdx.x;
  scales[item] = scale;
  // encode and store_code (quantization.cpp:94-124, 208-213), one 32-bit word
  // of the group's packed bytes at a time
  uint4* out = reinterpret_cast<uint4*>(codes + item * (group_words<Format>() * 4u));
  if constexpr (Format == GFXB_W3) {
    // three bit planes of 16 bytes; word k of plane p holds bit p of codes 32k .. 32k + 31
    std::uint32_t planes[3][4];
#pragma unroll
    for (unsigned k = 0; k < 4; ++k) {
      std::uint32_t p0 = 0, p1 = 0, p2 = 0;
      for (unsigned j = 0; j < 32; ++j) {
        const std::uint32_t code = static_cast<std::uint32_t>(quantize_level<Format>(v[32 * k + j], scale) + 4);
        p0 |= (code & 1u) << j;
        p1 |= ((code >> 1) & 1u) << j;
        p2 |= ((code >> 2) & 1u) << j;
      }
      planes[0][k] = p0;
      planes[1][k] = p1;
      planes[2][k] = p2;
    }
#pragma unroll
    for (unsigned p = 0; p < 3; ++p) out[p] = make_uint4(planes[p][0], planes[p][1], planes[p][2], planes[p][3]);
  } else {
    constexpr unsigned per_word = Format == GFXB_W2 ? 16u : 8u, bits = 32u / per_word;
    std::uint32_t words[group_words<Format>()];
#pragma unroll
    for (unsigned w = 0; w < group_words<Format>(); ++w) {
      std::uint32_t word = 0;
      for (unsigned j = 0; j < per_word; ++j) {
        const int level = quantize_level<Format>(v[per_word * w + j], scale);
        const std::uint32_t code = Format == GFXB_W2 ? static_cast<std::uint32_t>((level + 3) / 2)
                                                     : static_cast<std::uint32_t>(level) & 0x0fu;
        word |= code << (bits * j);
      }
      words[w] = word;
    }
#pragma unroll
    for (unsigned w = 0; w < group_words<Format>(); w += 4) {
      out[w / 4] = make_uint4(words[w], words[w + 1], words[w + 2], words[w + 3]);
    }
  }
}

// load_code (quantization.cpp:126-150).
__device__ __forceinline__ std::uint32_t load_code(const std::uint8_t* row, std::uint32_t column, int format) {
  if (format == GFXB_W2) return (row[column / 4] >> ((column & 3u) * 2u)) & 3u;
  if (format == GFXB_W4) return (row[column / 2] >> ((column & 1u) * 4u)) & 15u;
  const std::uint32_t group_base = (column / kGroup) * 48u, local = column % kGroup;
  std::uint32_t code = 0;
  for (std::uint32_t plane = 0; plane < 3; ++plane) {
    code |= ((row[group_base + plane * 16u + local / 8u] >> (local & 7u)) & 1u) << plane;
  }
  return code;
}

// decode_value (quantization.cpp:48-56).
__device__ __forceinline__ int decode_level(std::uint32_t code, int format) {
  if (format == GFXB_W2) return static_cast<int>(code) * 2 - 3;
  if (format == GFXB_W3) return static_cast<int>(code) - 4;
  return (code & 8u) != 0 ? static_cast<int>(code) - 16 : static_cast<int>(code);
}

// tile_group128_for_gfx12 (quantization.cpp:253-318): fragment f =
// ((tile * groups + group) * 4 + k_tile) * 16 + local_row holds the row's 32
// codes of that k-tile: the row-major bytes for W2 and W4, sequential 3-bit
// codes (code i at bit 3i) for W3. The thread of k-tile 0 also moves the
// row's scale of the group.
__global__ void tile_gfx12_kernel(const std::uint8_t* __restrict__ codes, const float* __restrict__ scales,
                                  std::uint8_t* __restrict__ tiled, float* __restrict__ tiled_scales,
                                  std::uint64_t fragments, std::uint32_t groups, std::uint32_t row_bytes, int format) {
  const std::uint64_t f = static_cast<std::uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (f >= fragments) return;
  const std::uint32_t local_row = static_cast<std::uint32_t>(f & 15u);
  const std::uint32_t k_tile = static_cast<std::uint32_t>((f >> 4) & 3u);
  const std::uint64_t tile_group = f >> 6;
  const std::uint64_t tile = tile_group / groups;
  const std::uint32_t group = static_cast<std::uint32_t>(tile_group % groups);
  const std::uint64_t row = tile * 16u + local_row;
  const std::uint8_t* source = codes + row * row_bytes;
  if (format == GFXB_W3) {
    std::uint32_t planes[3];
    for (std::uint32_t p = 0; p < 3; ++p) {
      const std::uint8_t* b = source + group * 48u + p * 16u + k_tile * 4u;
      planes[p] = b[0] | (b[1] << 8) | (b[2] << 16) | (static_cast<std::uint32_t>(b[3]) << 24);
    }
    std::uint32_t out[3] = {0, 0, 0};
    for (std::uint32_t i = 0; i < 32; ++i) {
      const std::uint32_t code = ((planes[0] >> i) & 1u) | (((planes[1] >> i) & 1u) << 1) | (((planes[2] >> i) & 1u) << 2);
      const std::uint32_t bit = 3u * i;
      out[bit / 32] |= code << (bit % 32);
      if (bit % 32 > 29) out[bit / 32 + 1] |= code >> (32u - bit % 32);
    }
    std::uint8_t* dest = tiled + f * 12u;
    for (std::uint32_t b = 0; b < 12; ++b) dest[b] = static_cast<std::uint8_t>(out[b / 4] >> (8u * (b % 4)));
  } else {
    const std::uint32_t fragment = format == GFXB_W2 ? 8u : 16u;
    const std::uint8_t* from = source + (group * 4u + k_tile) * fragment;
    std::uint8_t* dest = tiled + f * fragment;
    for (std::uint32_t b = 0; b < fragment; ++b) dest[b] = from[b];
  }
  if (k_tile == 0 && tiled_scales != nullptr) tiled_scales[tile_group * 16u + local_row] = scales[row * groups + group];
}

__global__ void dequantize_kernel(const std::uint8_t* __restrict__ codes, const float* __restrict__ scales,
                                  float* __restrict__ out, std::uint64_t count, std::uint32_t columns,
                                  std::uint32_t row_bytes, int format) {
  const std::uint64_t index = static_cast<std::uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (index >= count) return;
  const std::uint64_t row = index / columns;
  const std::uint32_t column = static_cast<std::uint32_t>(index % columns);
  const int level = decode_level(load_code(codes + row * row_bytes, column, format), format);
  out[index] = __fmul_rn(static_cast<float>(level), scales[row * (columns / kGroup) + column / kGroup]);
}

// fp32 group scales [N][K/128] -> fp16 (round to nearest even, converter.cpp:385-386)
// in the tiled order [N/16][K/128][16] (tiled) or row-major (not tiled).
__global__ void scales_to_f16_kernel(const float* __restrict__ scales, __half* __restrict__ out, std::uint64_t count,
                                     std::uint32_t groups, int tiled) {
  const std::uint64_t index = static_cast<std::uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (index >= count) return;
  const std::uint64_t row = index / groups;
  const std::uint32_t group = static_cast<std::uint32_t>(index % groups);
  const std::uint64_t to = tiled ? ((row / 16u) * groups + group) * 16u + (row & 15u) : index;
  out[to] = __float2half_rn(scales[index]);
}

bool aligned16(const void* pointer) { return (reinterpret_cast<std::uintptr_t>(pointer) & 15u) == 0; }

unsigned blocks_for(std::uint64_t count, unsigned threads) {
  return static_cast<unsigned>((count + threads - 1) / threads);
}

template <int Format, typename Input>
int launch_quantize(const Input* weights, std::uint64_t items, std::uint8_t* codes, float* scales,
                    std::uint32_t* flag, cudaStream_t stream) {
  static DeviceOnce configured;
  GFXB_TRY(configured.run([](int) {
    const cudaError_t error = cudaFuncSetAttribute(quantize_group128_kernel<Format, Input>,
                                                   cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                   static_cast<int>(kStageBytes));
    if (error != cudaSuccess) {
      set_error_cuda(error, "quantizer shared-memory configuration failed");
      return static_cast<int>(GFXB_CUDA_ERROR);
    }
    return static_cast<int>(GFXB_OK);
  }));
  quantize_group128_kernel<Format, Input><<<blocks_for(items, kItems), kItems, kStageBytes, stream>>>(
      weights, items, codes, scales, flag);
  return launch_status("group-128 quantizer launch failed");
}

template <typename Input>
int dispatch_quantize(int format, const Input* weights, std::uint64_t items, std::uint8_t* codes, float* scales,
                      std::uint32_t* flag, cudaStream_t stream) {
  if (format == GFXB_W2) return launch_quantize<GFXB_W2>(weights, items, codes, scales, flag, stream);
  if (format == GFXB_W3) return launch_quantize<GFXB_W3>(weights, items, codes, scales, flag, stream);
  return launch_quantize<GFXB_W4>(weights, items, codes, scales, flag, stream);
}

int check_quantizer_shape(int format, std::size_t rows, std::size_t columns) {
  if (rows == 0 || columns == 0 || columns % kGroup != 0) {
    return fail(GFXB_INVALID_ARGUMENT,
                "group-128 quantization requires nonzero dimensions, K divisible by 128, and an exact input span");
  }
  if (format != GFXB_W2 && format != GFXB_W3 && format != GFXB_W4) {
    return fail(GFXB_UNSUPPORTED, "only W2G128, W3G128, and W4G128 are implemented");
  }
  if (rows > (1ull << 31) || columns > (1ull << 24)) return fail(GFXB_UNSUPPORTED, "matrix is too large");
  return GFXB_OK;
}

// Quantizes and waits for the stream: returns GFXB_INVALID_ARGUMENT when the
// matrix holds a non-finite value (the reference's rejection, :215-218).
int quantize_and_check(int format, int input_dtype, const void* weights, std::size_t rows, std::size_t columns,
                       std::uint8_t* codes, float* scales, std::uint32_t* flag, cudaStream_t stream) {
  const std::uint64_t items = static_cast<std::uint64_t>(rows) * (columns / kGroup);
  cudaError_t error = cudaMemsetAsync(flag, 0, sizeof(std::uint32_t), stream);
  if (error != cudaSuccess) {
    set_error_cuda(error, "quantizer flag clear failed");
    return GFXB_CUDA_ERROR;
  }
  if (input_dtype == GFXB_DTYPE_BF16) {
    GFXB_TRY(dispatch_quantize(format, static_cast<const std::uint16_t*>(weights), items, codes, scales, flag, stream));
  } else {
    GFXB_TRY(dispatch_quantize(format, static_cast<const float*>(weights), items, codes, scales, flag, stream));
  }
  std::uint32_t host_flag = 0;
  error = cudaMemcpyAsync(&host_flag, flag, sizeof host_flag, cudaMemcpyDeviceToHost, stream);
  if (error == cudaSuccess) error = cudaStreamSynchronize(stream);
  if (error != cudaSuccess) {
    set_error_cuda(error, "group-128 quantization failed");
    return GFXB_CUDA_ERROR;
  }
  if (host_flag != 0) return fail(GFXB_INVALID_ARGUMENT, "weight matrix contains a non-finite value");
  return GFXB_OK;
}

std::size_t round_up(std::size_t value, std::size_t alignment) { return (value + alignment - 1) / alignment * alignment; }

}  // namespace

// The DType values of the reference artifact (artifact.h:18-25) name the input type.
std::size_t convert_scratch_bytes(int format, std::size_t rows, std::size_t columns) {
  const std::size_t codes = rows * (columns / kGroup) * (format == GFXB_W2 ? 32u : (format == GFXB_W3 ? 48u : 64u));
  const std::size_t scales = rows * (columns / kGroup) * sizeof(float);
  return round_up(codes, 256) + round_up(scales, 256) + 256;
}

}  // namespace gfxb

using namespace gfxb;

extern "C" std::size_t gfxb_packed_row_bytes(int format, std::size_t columns) {
  // quantization.cpp:154-161
  switch (format) {
    case GFXB_W2: return (columns + 3) / 4;
    case GFXB_W3: return (columns * 3 + 7) / 8;
    case GFXB_W4: return (columns + 1) / 2;
    default: return 0;
  }
}

extern "C" int gfxb_quantize_group128(int format, int input_dtype, const void* weights, std::size_t rows,
                                      std::size_t columns, std::uint8_t* codes, float* scales, void* stream) {
  GFXB_TRY(check_quantizer_shape(format, rows, columns));
  GFXB_REQUIRE(input_dtype == GFXB_DTYPE_F32 || input_dtype == GFXB_DTYPE_BF16, "weights must be fp32 or bf16");
  GFXB_REQUIRE(weights != nullptr && codes != nullptr && scales != nullptr, "quantization requires buffers");
  GFXB_REQUIRE(aligned16(codes), "packed codes must be 16-byte aligned");
  std::uint32_t* flag = nullptr;
  const cudaStream_t s = as_stream(stream);
  cudaError_t error = cudaMallocAsync(reinterpret_cast<void**>(&flag), sizeof(std::uint32_t), s);
  if (error != cudaSuccess) {
    set_error_cuda(error, "quantizer flag allocation failed");
    return GFXB_OUT_OF_MEMORY;
  }
  const int status = quantize_and_check(format, input_dtype, weights, rows, columns, codes, scales, flag, s);
  cudaFreeAsync(flag, s);
  return status;
}

extern "C" int gfxb_tile_group128_for_gfx12(int format, const std::uint8_t* codes, const float* scales,
                                            std::size_t rows, std::size_t columns, std::uint8_t* tiled_codes,
                                            float* tiled_scales, void* stream) {
  if ((format != GFXB_W2 && format != GFXB_W3 && format != GFXB_W4) || rows == 0 || rows % 16 != 0 ||
      columns == 0 || columns % kGroup != 0) {
    return fail(GFXB_INVALID_ARGUMENT,
                "gfx12 tiling requires valid W2G128/W3G128/W4G128 storage, N divisible by 16, and K divisible by 128");
  }
  GFXB_REQUIRE(codes != nullptr && scales != nullptr && tiled_codes != nullptr && tiled_scales != nullptr,
               "tiling requires buffers");
  const std::uint32_t groups = static_cast<std::uint32_t>(columns / kGroup);
  const std::uint64_t fragments = static_cast<std::uint64_t>(rows) * groups * 4u;
  tile_gfx12_kernel<<<blocks_for(fragments, 256), 256, 0, as_stream(stream)>>>(
      codes, scales, tiled_codes, tiled_scales, fragments, groups,
      static_cast<std::uint32_t>(gfxb_packed_row_bytes(format, columns)), format);
  return launch_status("gfx12 tiling launch failed");
}

extern "C" int gfxb_dequantize_group128(int format, const std::uint8_t* codes, const float* scales, std::size_t rows,
                                        std::size_t columns, float* output, void* stream) {
  if (rows == 0 || columns == 0 || columns % kGroup != 0 ||
      (format != GFXB_W2 && format != GFXB_W3 && format != GFXB_W4)) {
    return fail(GFXB_INVALID_ARGUMENT, "packed matrix metadata or storage is invalid");
  }
  GFXB_REQUIRE(codes != nullptr && scales != nullptr && output != nullptr, "dequantization requires buffers");
  const std::uint64_t count = static_cast<std::uint64_t>(rows) * columns;
  dequantize_kernel<<<blocks_for(count, 256), 256, 0, as_stream(stream)>>>(
      codes, scales, output, count, static_cast<std::uint32_t>(columns),
      static_cast<std::uint32_t>(gfxb_packed_row_bytes(format, columns)), format);
  return launch_status("dequantization launch failed");
}

extern "C" float gfxb_dequantized_weight(int format, const std::uint8_t* codes, const float* scales, std::size_t rows,
                                         std::size_t columns, std::size_t row, std::size_t column) {
  // quantization.cpp:222-235 on host memory
  if (codes == nullptr || scales == nullptr || row >= rows || column >= columns || columns % kGroup != 0 ||
      (format != GFXB_W2 && format != GFXB_W3 && format != GFXB_W4)) {
    return std::nanf("");
  }
  const std::uint8_t* r = codes + row * gfxb_packed_row_bytes(format, columns);
  std::uint32_t code = 0;
  if (format == GFXB_W2) {
    code = (r[column / 4] >> ((column & 3u) * 2u)) & 3u;
  } else if (format == GFXB_W4) {
    code = (r[column / 2] >> ((column & 1u) * 4u)) & 15u;
  } else {
    const std::size_t base = (column / kGroup) * 48u, local = column % kGroup;
    for (unsigned plane = 0; plane < 3; ++plane) code |= ((r[base + plane * 16u + local / 8u] >> (local & 7u)) & 1u) << plane;
  }
  const int level = format == GFXB_W2 ? static_cast<int>(code) * 2 - 3
                                      : (format == GFXB_W3 ? static_cast<int>(code) - 4
                                                           : ((code & 8u) != 0 ? static_cast<int>(code) - 16
                                                                               : static_cast<int>(code)));
  return static_cast<float>(level) * scales[row * (columns / kGroup) + column / kGroup];
}

extern "C" std::size_t gfxb_convert_scratch_bytes(int format, std::size_t rows, std::size_t columns) {
  return convert_scratch_bytes(format, rows, columns);
}

extern "C" int gfxb_convert_group128(int format, int input_dtype, const void* weights, std::size_t rows,
                                     std::size_t columns, int layout, std::uint8_t* codes, std::uint16_t* scales,
                                     void* scratch, std::size_t scratch_bytes, void* stream) {
  GFXB_TRY(check_quantizer_shape(format, rows, columns));
  GFXB_REQUIRE(input_dtype == GFXB_DTYPE_F32 || input_dtype == GFXB_DTYPE_BF16, "weights must be fp32 or bf16");
  GFXB_REQUIRE(layout == GFXB_LAYOUT_B200 || layout == GFXB_LAYOUT_GFX12 || layout == GFXB_LAYOUT_ROWMAJOR,
               "unknown weight layout");
  GFXB_REQUIRE(layout == GFXB_LAYOUT_ROWMAJOR || rows % 16 == 0, "tiled layouts need N divisible by 16");
  GFXB_REQUIRE(weights != nullptr && codes != nullptr && scales != nullptr && scratch != nullptr,
               "conversion requires buffers");
  GFXB_REQUIRE(scratch_bytes >= convert_scratch_bytes(format, rows, columns) && aligned16(scratch),
               "conversion scratch is too small or misaligned");
  const cudaStream_t s = as_stream(stream);
  const std::size_t groups = columns / kGroup;
  const std::size_t code_bytes = rows * gfxb_packed_row_bytes(format, columns);
  auto* base = static_cast<std::uint8_t*>(scratch);
  std::uint8_t* rowmajor = layout == GFXB_LAYOUT_ROWMAJOR ? codes : base;
  float* fp32_scales = reinterpret_cast<float*>(base + round_up(code_bytes, 256));
  auto* flag = reinterpret_cast<std::uint32_t*>(base + round_up(code_bytes, 256) + round_up(rows * groups * 4, 256));
  GFXB_REQUIRE(aligned16(rowmajor), "packed codes must be 16-byte aligned");
  GFXB_TRY(quantize_and_check(format, input_dtype, weights, rows, columns, rowmajor, fp32_scales, flag, s));
  if (layout == GFXB_LAYOUT_B200) {
    GFXB_TRY(gfxb_repack_rowmajor_to_b200(format, rowmajor, codes, rows, columns, stream));
  } else if (layout == GFXB_LAYOUT_GFX12) {
    // codes only: the fp16 scales are tiled below, in the same [N/16][K/128][16] order
    const std::uint64_t fragments = static_cast<std::uint64_t>(rows) * groups * 4u;
    tile_gfx12_kernel<<<blocks_for(fragments, 256), 256, 0, s>>>(
        rowmajor, fp32_scales, codes, nullptr, fragments, static_cast<std::uint32_t>(groups),
        static_cast<std::uint32_t>(gfxb_packed_row_bytes(format, columns)), format);
    GFXB_TRY(launch_status("gfx12 tiling launch failed"));
  }
  const std::uint64_t count = static_cast<std::uint64_t>(rows) * groups;
  scales_to_f16_kernel<<<blocks_for(count, 256), 256, 0, s>>>(fp32_scales, reinterpret_cast<__half*>(scales), count,
                                                             static_cast<std::uint32_t>(groups),
                                                             layout == GFXB_LAYOUT_ROWMAJOR ? 0 : 1);
  return launch_status("scale conversion launch failed");
}
