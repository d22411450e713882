// Model conversion to `.gfxi` artifacts: the reference converter's plan and
// write_quantized pipeline (src/converter.cpp:98-119, 186-330, 345-393)
// over in-memory source tensors, with the group-128 quantizer running on the
// device.
//
// Per tensor, choose_quantization's rules pick the format: a 2-D tensor with
// N % 16 == 0 and K % 128 == 0 is quantized (lm_head to head_bits, the MLPs of
// decoder layers below layers - w4_tail_layers to mlp_bits, W3 only from
// w3_start_layer on and W2 before it, everything else W4); any other tensor
// is stored as bf16. Quantized tensors are uploaded `chunk_rows` rows at a
// time, quantized (bit-identical to quantize_group128), laid out for the
// chosen recipe and streamed to the writer with fp16 scales rounded to
// nearest even, as the reference writes them.
#include <algorithm>
#include <cstdio>
#include <cstring>
#include <string>
#include <string_view>
#include <vector>

#include "artifact_internal.h"
#include "gfxb/artifact.h"
#include "kernels/common.cuh"

namespace gfxb {
namespace {

int cuda_status(cudaError_t error, const char* context) {
  if (error == cudaSuccess) return GFXB_OK;
  set_error_cuda(error, context);
  return error == cudaErrorMemoryAllocation ? GFXB_OUT_OF_MEMORY : GFXB_CUDA_ERROR;
}

int format_of_bits(std::uint32_t bits) { return bits == 2 ? GFXB_W2 : (bits == 3 ? GFXB_W3 : GFXB_W4); }

// converter.cpp:77-96: the layer index of a decoder-layer MLP tensor, if it is one.
bool decoder_mlp_layer(std::string_view name, std::uint32_t* layer) {
  constexpr std::string_view prefix = "model.language_model.layers.";
  if (name.substr(0, prefix.size()) != prefix) return false;
  const std::size_t end = name.find('.', prefix.size());
  if (end == std::string_view::npos || name.find(".mlp.", end) == std::string_view::npos) return false;
  std::uint32_t value = 0;
  for (const char digit : name.substr(prefix.size(), end - prefix.size())) {
    if (digit < '0' || digit > '9') return false;
    value = value * 10u + static_cast<std::uint32_t>(digit - '0');
  }
  *layer = value;
  return true;
}

// converter.cpp:98-119: 0 for a tensor stored as bf16, else GFXB_W2/W3/W4.
int choose_format(const gfxb_convert_source& t, const gfxb_convert_options& o) {
  if (t.rank != 2 || t.dimensions[0] % 16 != 0 || t.dimensions[1] % 128 != 0) return 0;
  const std::string_view name(t.name);
  if (name == "lm_head.weight") return format_of_bits(o.head_bits);
  std::uint32_t layer = 0;
  if (!decoder_mlp_layer(name, &layer) || layer + o.w4_tail_layers >= o.layers) return GFXB_W4;
  if (o.mlp_bits == 4) return GFXB_W4;
  return o.mlp_bits == 3 && layer >= o.w3_start_layer ? GFXB_W3 : GFXB_W2;
}

std::uint16_t f32_to_bf16(float value) {
  std::uint32_t bits;
  std::memcpy(&bits, &value, sizeof bits);
  if ((bits & 0x7fffffffu) > 0x7f800000u) return static_cast<std::uint16_t>((bits >> 16) | 0x40u);  // quiet NaN
  bits += 0x7fffu + ((bits >> 16) & 1u);
  return static_cast<std::uint16_t>(bits >> 16);
}

std::uint64_t elements_of(const gfxb_convert_source& t) {
  std::uint64_t count = 1;
  for (std::uint16_t d = 0; d < t.rank; ++d) count *= t.dimensions[d];
  return count;
}

int element_bytes(std::uint16_t dtype) { return dtype == GFXB_DTYPE_F32 ? 4 : (dtype == GFXB_DTYPE_BF16 ? 2 : 0); }

}  // namespace
}  // namespace gfxb

using namespace gfxb;

extern "C" int gfxb_convert_to_artifact(const char* path, const gfxb_artifact_identity* identity,
                                        const gfxb_convert_source* sources, size_t count,
                                        const gfxb_convert_options* options, int device) {
  if (path == nullptr || identity == nullptr || sources == nullptr || options == nullptr || count == 0) {
    return fail(GFXB_INVALID_ARGUMENT, "null argument");
  }
  const gfxb_convert_options& o = *options;
  if ((o.layout != GFXB_LAYOUT_B200 && o.layout != GFXB_LAYOUT_GFX12) || o.mlp_bits < 2 || o.mlp_bits > 4 ||
      o.head_bits < 2 || o.head_bits > 4 || o.chunk_rows == 0 || o.chunk_rows % 16 != 0 || o.chunk_rows > 4096) {
    return fail(GFXB_INVALID_ARGUMENT, "conversion options are invalid (chunk rows: a multiple of 16 up to 4096)");
  }
  const std::string recipe(identity->recipe_id, strnlen(identity->recipe_id, sizeof identity->recipe_id));
  const bool b200_recipe = recipe == "b200-v1";
  const bool tiled_recipe = recipe.find("tiled-v") != std::string::npos;
  if ((o.layout == GFXB_LAYOUT_B200) != b200_recipe || (o.layout == GFXB_LAYOUT_GFX12 && !tiled_recipe)) {
    return fail(GFXB_INVALID_ARGUMENT, "recipe id does not name the requested layout (b200-v1 or a tiled-v recipe)");
  }
  // plan (converter.cpp:186-330), in name order as the writer lays out the directory
  std::vector<std::size_t> order(count);
  for (std::size_t i = 0; i < count; ++i) {
    const gfxb_convert_source& t = sources[i];
    if (t.name == nullptr || t.data == nullptr || t.rank == 0 || t.rank > 4 || element_bytes(t.dtype) == 0 ||
        t.data_bytes != elements_of(t) * static_cast<std::uint64_t>(element_bytes(t.dtype))) {
      return fail(GFXB_INVALID_ARGUMENT, "source tensors need a name, fp32 or bf16 data and matching sizes");
    }
    order[i] = i;
  }
  std::sort(order.begin(), order.end(),
            [&](std::size_t a, std::size_t b) { return std::strcmp(sources[a].name, sources[b].name) < 0; });
  std::vector<gfxi::Plan> plans;
  std::vector<int> formats;
  std::vector<int> layouts;
  bool has_w3 = false;
  std::uint64_t widest = 0;
  for (const std::size_t i : order) {
    const gfxb_convert_source& t = sources[i];
    gfxi::Plan plan;
    plan.name = t.name;
    plan.dimensions.assign(t.dimensions, t.dimensions + t.rank);
    const int format = choose_format(t, o);
    // the b200 recipe keeps the embedding row-major (the gather reads one row); the tiled recipes tile it
    const bool embedding = plan.name == "model.language_model.embed_tokens.weight";
    if (format != 0 && embedding && format == GFXB_W3) {
      return fail(GFXB_UNSUPPORTED, "the embedding must be W2 or W4");
    }
    if (format == 0) {
      plan.dtype = GFXB_DTYPE_BF16;
      plan.quantization = GFXB_QUANT_NONE;
      plan.data_bytes = elements_of(t) * 2;
    } else {
      const std::uint64_t rows = t.dimensions[0], cols = t.dimensions[1];
      plan.dtype = GFXB_DTYPE_U8;
      plan.quantization = static_cast<std::uint16_t>(format);  // GFXB_W* equal the Quantization values
      plan.data_bytes = rows * gfxb_packed_row_bytes(format, cols);
      plan.aux_bytes = rows * (cols / 128) * 2;
      has_w3 = has_w3 || format == GFXB_W3;
      widest = std::max<std::uint64_t>(widest, cols);
    }
    plans.push_back(std::move(plan));
    formats.push_back(format);
    layouts.push_back(o.layout == GFXB_LAYOUT_B200 && embedding ? GFXB_LAYOUT_ROWMAJOR : static_cast<int>(o.layout));
  }
  if (o.layout == GFXB_LAYOUT_GFX12 && has_w3 && recipe.find("w3seq") == std::string::npos) {
    return fail(GFXB_INVALID_ARGUMENT, "a tiled recipe with W3 tensors must name the sequential W3 form (w3seq)");
  }
  GFXB_TRY(cuda_status(cudaSetDevice(device), "cudaSetDevice failed"));
  gfxi::StreamWriter writer;
  GFXB_TRY(writer.create(path, *identity, plans));
  // device staging for one chunk: fp32 input, codes, fp16 scales, conversion scratch
  const std::uint64_t chunk_values = static_cast<std::uint64_t>(o.chunk_rows) * std::max<std::uint64_t>(widest, 128);
  const std::size_t scratch_bytes = gfxb_convert_scratch_bytes(GFXB_W4, o.chunk_rows, std::max<std::uint64_t>(widest, 128));
  const std::size_t input_bytes = chunk_values * 4, code_bytes = chunk_values / 2, scale_bytes = chunk_values / 128 * 2;
  const std::size_t device_bytes = input_bytes + code_bytes + scale_bytes + scratch_bytes + 1024;
  std::byte* device_buffer = nullptr;
  std::byte* host_buffer = nullptr;
  cudaStream_t stream = nullptr;
  int status = cuda_status(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking), "stream creation failed");
  if (status == GFXB_OK) {
    status = cuda_status(cudaMalloc(reinterpret_cast<void**>(&device_buffer), device_bytes), "staging allocation failed");
  }
  if (status == GFXB_OK) {
    status = cuda_status(cudaMallocHost(reinterpret_cast<void**>(&host_buffer), code_bytes + scale_bytes + 256),
                         "staging allocation failed");
  }
  auto align = [](std::size_t v) { return (v + 255) & ~std::size_t{255}; };
  std::byte* d_input = device_buffer;
  auto* d_codes = reinterpret_cast<std::uint8_t*>(device_buffer + align(input_bytes));
  auto* d_scales = reinterpret_cast<std::uint16_t*>(device_buffer + align(input_bytes) + align(code_bytes));
  std::byte* d_scratch = device_buffer + align(input_bytes) + align(code_bytes) + align(scale_bytes);
  std::vector<std::uint16_t> bf16;
  for (std::size_t p = 0; p < plans.size() && status == GFXB_OK; ++p) {
    const gfxb_convert_source& t = sources[order[p]];
    const int format = formats[p];
    if (format == 0) {
      // stored as bf16 (fp32 sources rounded to nearest even)
      if (t.dtype == GFXB_DTYPE_BF16) {
        status = writer.append(p, false, t.data, t.data_bytes);
      } else {
        const std::uint64_t n = elements_of(t);
        bf16.resize(n);
        const float* values = static_cast<const float*>(t.data);
        for (std::uint64_t i = 0; i < n; ++i) bf16[i] = f32_to_bf16(values[i]);
        status = writer.append(p, false, bf16.data(), n * 2);
      }
      continue;
    }
    const std::uint64_t rows = t.dimensions[0], cols = t.dimensions[1];
    const std::uint64_t row_bytes = gfxb_packed_row_bytes(format, cols);
    const int bytes_per_value = element_bytes(t.dtype);
    for (std::uint64_t row = 0; row < rows && status == GFXB_OK; row += o.chunk_rows) {
      const std::uint64_t n = std::min<std::uint64_t>(o.chunk_rows, rows - row);
      status = cuda_status(cudaMemcpyAsync(d_input, static_cast<const std::byte*>(t.data) + row * cols * bytes_per_value,
                                           n * cols * bytes_per_value, cudaMemcpyHostToDevice, stream),
                           "weight upload failed");
      if (status == GFXB_OK) {
        status = gfxb_convert_group128(format, t.dtype, d_input, n, cols, layouts[p], d_codes, d_scales, d_scratch,
                                       scratch_bytes, stream);
      }
      if (status == GFXB_OK) {
        status = cuda_status(cudaMemcpyAsync(host_buffer, d_codes, n * row_bytes, cudaMemcpyDeviceToHost, stream),
                             "code download failed");
      }
      if (status == GFXB_OK) {
        status = cuda_status(cudaMemcpyAsync(host_buffer + align(n * row_bytes), d_scales, n * (cols / 128) * 2,
                                             cudaMemcpyDeviceToHost, stream),
                             "scale download failed");
      }
      if (status == GFXB_OK) status = cuda_status(cudaStreamSynchronize(stream), "conversion failed");
      if (status == GFXB_OK) status = writer.append(p, false, host_buffer, n * row_bytes);
      if (status == GFXB_OK) status = writer.append(p, true, host_buffer + align(n * row_bytes), n * (cols / 128) * 2);
    }
  }
  if (status == GFXB_OK) status = writer.finalize();
  if (host_buffer != nullptr) cudaFreeHost(host_buffer);
  if (device_buffer != nullptr) cudaFree(device_buffer);
  if (stream != nullptr) cudaStreamDestroy(stream);
  return status;
}
