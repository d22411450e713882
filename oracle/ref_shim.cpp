// C entry points over the reference's own packing routines, for parity tests.
// TEST INFRASTRUCTURE ONLY. This file is compiled together with the
// reference's unmodified src/quantization.cpp (read in place from the
// reference checkout; never copied) into oracle/_ref/libgfxref.so.
#include <cstdint>
#include <cstring>
#include <span>

#include "gfxinfer/quantization.h"

namespace {
gfxinfer::Quantization to_format(int format) {
  return static_cast<gfxinfer::Quantization>(format);
}
}  // namespace

extern "C" {

// Wraps gfxinfer::quantize_group128 (src/quantization.cpp:163-220).
// Returns the reference ErrorCode value (0 = ok).
int ref_quantize_group128(const float* weights, std::size_t rows, std::size_t columns,
                          int format, std::uint8_t* codes, float* scales) {
  auto result = gfxinfer::quantize_group128(
      std::span<const float>(weights, rows * columns), rows, columns, to_format(format));
  if (!result.ok()) return static_cast<int>(result.status().code());
  const auto& packed = result.value();
  std::memcpy(codes, packed.codes.data(), packed.codes.size());
  std::memcpy(scales, packed.scales.data(), packed.scales.size() * sizeof(float));
  return 0;
}

// Wraps gfxinfer::tile_group128_for_gfx12 (src/quantization.cpp:253-318).
int ref_tile_gfx12(const std::uint8_t* codes, const float* scales, std::size_t rows,
                   std::size_t columns, int format, std::uint8_t* tiled_codes,
                   float* tiled_scales) {
  gfxinfer::PackedMatrix matrix;
  matrix.rows = rows;
  matrix.columns = columns;
  matrix.format = to_format(format);
  matrix.codes.assign(codes, codes + rows * gfxinfer::packed_row_bytes(matrix.format, columns));
  matrix.scales.assign(scales, scales + rows * (columns / 128));
  auto result = gfxinfer::tile_group128_for_gfx12(matrix);
  if (!result.ok()) return static_cast<int>(result.status().code());
  std::memcpy(tiled_codes, result.value().codes.data(), result.value().codes.size());
  std::memcpy(tiled_scales, result.value().scales.data(),
              result.value().scales.size() * sizeof(float));
  return 0;
}

// Wraps gfxinfer::dequantized_weight (src/quantization.cpp:222-235).
float ref_dequantized_weight(const std::uint8_t* codes, const float* scales, std::size_t rows,
                             std::size_t columns, int format, std::size_t row,
                             std::size_t column) {
  gfxinfer::PackedMatrix matrix;
  matrix.rows = rows;
  matrix.columns = columns;
  matrix.format = to_format(format);
  matrix.codes.assign(codes, codes + rows * gfxinfer::packed_row_bytes(matrix.format, columns));
  matrix.scales.assign(scales, scales + rows * (columns / 128));
  return gfxinfer::dequantized_weight(matrix, row, column);
}

std::size_t ref_packed_row_bytes(int format, std::size_t columns) {
  return gfxinfer::packed_row_bytes(to_format(format), columns);
}

}  // extern "C"

#include <random>

extern "C" {

// The exact input matrices of the reference's tests/quantization_test.cpp
// (std::mt19937 + std::normal_distribution<float>, :12-22 and :49-56).
void ref_test_matrix(unsigned seed, float stddev, std::size_t count, float* values) {
  std::mt19937 generator(seed);
  std::normal_distribution<float> distribution(0.0F, stddev);
  for (std::size_t i = 0; i < count; ++i) values[i] = distribution(generator);
}

}  // extern "C"
