// C entry points over the reference's own packing routines and `.gfxi`
// container, for parity tests. TEST INFRASTRUCTURE ONLY. This file is
// compiled together with the reference's unmodified src/quantization.cpp and
// src/artifact.cpp (read in place from the reference checkout; never copied)
// into oracle/_ref/libgfxref.so.
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <span>
#include <vector>

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

#include "gfxinfer/artifact.h"

extern "C" {

// Writes an artifact with the reference's own ArtifactWriter::write
// (src/artifact.cpp:426-562). dims is [count][4]. Returns the ErrorCode.
int ref_artifact_write(const char* path, const char* target, const char* model, const char* weights,
                       const char* recipe, std::size_t count, const char* const* names,
                       const std::uint16_t* dtypes, const std::uint16_t* quantizations,
                       const std::uint16_t* ranks, const std::uint64_t* dims, const void* const* data,
                       const std::uint64_t* data_bytes, const void* const* aux,
                       const std::uint64_t* aux_bytes, const std::uint32_t* alignments) {
  std::vector<gfxinfer::TensorWriteRequest> requests(count);
  for (std::size_t i = 0; i < count; ++i) {
    auto& r = requests[i];
    r.name = names[i];
    r.dtype = static_cast<gfxinfer::DType>(dtypes[i]);
    r.quantization = static_cast<gfxinfer::Quantization>(quantizations[i]);
    r.dimensions.assign(dims + 4 * i, dims + 4 * i + ranks[i]);
    r.alignment = alignments[i];
    r.data = {static_cast<const std::byte*>(data[i]), static_cast<std::size_t>(data_bytes[i])};
    if (aux_bytes[i] != 0) {
      r.auxiliary = {static_cast<const std::byte*>(aux[i]), static_cast<std::size_t>(aux_bytes[i])};
    }
  }
  const gfxinfer::ArtifactIdentity identity{target, model, weights, recipe};
  const auto status = gfxinfer::ArtifactWriter::write(path, identity, requests);
  return static_cast<int>(status.code());
}

// Opens an artifact with the reference's ArtifactView::open
// (src/artifact.cpp:274-407); returns the ErrorCode and, when it opens, the
// tensor count and file size.
int ref_artifact_open(const char* path, int verify, std::size_t* count, std::uint64_t* file_bytes) {
  auto view = gfxinfer::ArtifactView::open(path, {.verify_checksums = verify != 0});
  if (!view.ok()) return static_cast<int>(view.status().code());
  *count = view.value().tensors().size();
  *file_bytes = view.value().file_bytes();
  return 0;
}

// Tensor `index` as the reference reader sees it: name (NUL-terminated,
// truncated to 255 bytes), dims[4], meta = {dtype, quantization, rank},
// spans = {data_offset, data_bytes, aux_offset, aux_bytes, data_crc64}.
int ref_artifact_tensor(const char* path, std::size_t index, char* name, std::uint64_t* dims,
                        std::uint16_t* meta, std::uint64_t* spans) {
  auto view = gfxinfer::ArtifactView::open(path, {.verify_checksums = true});
  if (!view.ok()) return static_cast<int>(view.status().code());
  const auto& tensors = view.value().tensors();
  if (index >= tensors.size()) return 1;
  const auto& t = tensors[index];
  std::snprintf(name, 256, "%s", t.name.c_str());
  for (int d = 0; d < 4; ++d) dims[d] = t.dimensions[d];
  meta[0] = static_cast<std::uint16_t>(t.dtype);
  meta[1] = static_cast<std::uint16_t>(t.quantization);
  meta[2] = t.rank;
  spans[0] = t.data_offset;
  spans[1] = t.data_bytes;
  spans[2] = t.aux_offset;
  spans[3] = t.aux_bytes;
  spans[4] = t.data_crc64;
  return 0;
}

}  // extern "C"
