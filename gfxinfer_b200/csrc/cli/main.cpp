// gfxinfer-b200 command line: the reference CLI's benchmark and check
// commands (src/cli/main.cpp:38-67, 790-1000, 1529-1700) over the C ABI.
//
//   gfxinfer-b200 probe
//   gfxinfer-b200 inspect ARTIFACT [--no-verify]
//   gfxinfer-b200 bench-gemv [--format w2|w3|w4] [--rows N] [--columns K] [--batch B]
//                            [--activation a4|a8|f16] [--iterations I]
//   gfxinfer-b200 decode-bench [MODEL] [--steps S] [--persistent]
//   gfxinfer-b200 block-bench [MODEL] [--width W]
//   gfxinfer-b200 spec-bench [MODEL] [--depth D] [--tokens N] [--eager]
//   gfxinfer-b200 export PATH [MODEL]
//
// MODEL: --artifact PATH (a .gfxi file), or seeded random-init weights of the
// config-2 shape (default) or the scaled-down test shape (--small), with
// --layers L, --context C and --a8 to vary them.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <array>
#include <chrono>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <random>
#include <string>
#include <vector>

#include "gfxb/artifact.h"
#include "gfxb/gfxb.h"

namespace {

struct Args {
  std::vector<std::string> positional;
  std::vector<std::pair<std::string, std::string>> options;
  bool flag(const char* name) const {
    return std::any_of(options.begin(), options.end(), [&](const auto& o) { return o.first == name; });
  }
  std::string get(const char* name, const std::string& fallback) const {
    for (const auto& o : options) {
      if (o.first == name) return o.second;
    }
    return fallback;
  }
  long number(const char* name, long fallback) const {
    const std::string value = get(name, "");
    return value.empty() ? fallback : std::strtol(value.c_str(), nullptr, 10);
  }
};

Args parse(int argc, char** argv, int first) {
  static const char* kValued[] = {"--format", "--rows", "--columns", "--batch", "--activation", "--iterations",
                                  "--steps", "--width", "--depth", "--tokens", "--artifact", "--layers",
                                  "--context", "--device"};
  Args args;
  for (int i = first; i < argc; ++i) {
    const std::string a = argv[i];
    if (a.rfind("--", 0) != 0) {
      args.positional.push_back(a);
      continue;
    }
    const bool valued = std::any_of(std::begin(kValued), std::end(kValued), [&](const char* v) { return a == v; });
    if (valued && i + 1 < argc) {
      args.options.emplace_back(a, argv[++i]);
    } else {
      args.options.emplace_back(a, "");
    }
  }
  return args;
}

int fail(int status) {
  std::fprintf(stderr, "error: %s (status %d)\n", gfxb_last_error_message(), status);
  return 1;
}

#define CLI_TRY(expression)              \
  do {                                   \
    const int status_ = (expression);    \
    if (status_ != GFXB_OK) return fail(status_); \
  } while (0)

bool cuda_ok(cudaError_t error, const char* what) {
  if (error == cudaSuccess) return true;
  std::fprintf(stderr, "error: %s: %s\n", what, cudaGetErrorString(error));
  return false;
}

template <class T>
struct DeviceBuffer {
  T* p = nullptr;
  std::size_t count = 0;
  explicit DeviceBuffer(std::size_t n) : count(n) {
    if (cudaMalloc(&p, std::max<std::size_t>(n, 1) * sizeof(T)) != cudaSuccess) p = nullptr;
  }
  ~DeviceBuffer() { cudaFree(p); }
  DeviceBuffer(const DeviceBuffer&) = delete;
  DeviceBuffer& operator=(const DeviceBuffer&) = delete;
};

double now_ms() {
  return std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now().time_since_epoch()).count();
}

// ---- probe / inspect --------------------------------------------------------

int probe(const Args& args) {
  gfxb_device_info info{};
  CLI_TRY(gfxb_require_sm100_device(static_cast<int>(args.number("--device", 0)), &info));
  std::printf("device %d: %s (sm_%d%d), %d SMs, %.1f GiB\n", info.index, info.name, info.compute_major,
              info.compute_minor, info.multiprocessors, info.global_memory_bytes / 1073741824.0);
  return 0;
}

int inspect(const Args& args) {
  if (args.positional.empty()) {
    std::fprintf(stderr, "usage: inspect ARTIFACT [--no-verify]\n");
    return 2;
  }
  gfxb_artifact* artifact = nullptr;
  CLI_TRY(gfxb_artifact_open(args.positional[0].c_str(), args.flag("--no-verify") ? 0 : 1, &artifact));
  gfxb_artifact_identity id{};
  gfxb_artifact_identity_of(artifact, &id);
  std::uint64_t bytes = 0;
  std::size_t count = 0;
  gfxb_artifact_file_bytes(artifact, &bytes);
  gfxb_artifact_tensor_count(artifact, &count);
  std::printf("target %s  model %s  weights %s  recipe %s\n%zu tensors, %llu bytes\n", id.target_arch, id.model_id,
              id.weights_id, id.recipe_id, count, static_cast<unsigned long long>(bytes));
  static const char* kDtype[] = {"?", "u8", "i32", "f16", "bf16", "f32"};
  static const char* kQuant[] = {"none", "w2g128", "w3g128", "w4g128", "w8g128", "fp8-row"};
  for (std::size_t i = 0; i < count; ++i) {
    gfxb_tensor_view t{};
    gfxb_artifact_tensor_at(artifact, i, &t);
    std::printf("  %-60s %-5s %-7s [", t.name, kDtype[t.dtype <= 5 ? t.dtype : 0],
                kQuant[t.quantization <= 5 ? t.quantization : 0]);
    for (unsigned d = 0; d < t.rank; ++d) std::printf(d ? ",%llu" : "%llu", static_cast<unsigned long long>(t.dimensions[d]));
    std::printf("] %llu+%llu bytes\n", static_cast<unsigned long long>(t.data_bytes),
                static_cast<unsigned long long>(t.aux_bytes));
  }
  gfxb_artifact_close(artifact);
  return 0;
}

// ---- bench-gemv -----------------------------------------------------------------

// Reference row-major packing rules (quantization.cpp:126-150, 29-56): signed level of column c.
int level(const std::uint8_t* row, std::size_t c, int bits) {
  if (bits == 2) return static_cast<int>((row[c / 4] >> ((c & 3u) * 2u)) & 3u) * 2 - 3;
  if (bits == 4) {
    const int code = (row[c / 2] >> ((c & 1u) * 4u)) & 15;
    return code >= 8 ? code - 16 : code;
  }
  const std::size_t group = c / 128, local = c % 128;
  int code = 0;
  for (int plane = 0; plane < 3; ++plane) code |= ((row[group * 48 + plane * 16 + local / 8] >> (local & 7u)) & 1) << plane;
  return code - 4;
}

// Position of column k of a 128-group in the activation pack (fragment order).
std::size_t fragment_offset(std::size_t k) {
  const std::size_t s = k >> 5, rest = k & 31u, half = rest >> 4, t = (rest & 15u) >> 2, j = k & 3u;
  return t * 32u + s * 8u + half * 4u + j;
}

int bench_gemv(const Args& args) {
  const std::string fmt_name = args.get("--format", "w3");
  const int bits = fmt_name == "w2" ? 2 : (fmt_name == "w4" ? 4 : 3);
  const int format = bits == 2 ? GFXB_W2 : (bits == 3 ? GFXB_W3 : GFXB_W4);
  const std::size_t rows = static_cast<std::size_t>(args.number("--rows", 17408));
  const std::size_t cols = static_cast<std::size_t>(args.number("--columns", 5120));
  const unsigned batch = static_cast<unsigned>(args.number("--batch", 1));
  const std::string activation = args.get("--activation", "a4");
  const int iterations = static_cast<int>(args.number("--iterations", 200));
  if (rows == 0 || rows % 16 != 0 || cols == 0 || cols % 128 != 0 || batch == 0 || batch > 32 || iterations <= 0) {
    std::fprintf(stderr, "error: rows must be a multiple of 16, columns of 128, batch in [1, 32]\n");
    return 2;
  }
  CLI_TRY(gfxb_require_sm100_device(0, nullptr));
  // seeded inputs as the reference bench (main.cpp:1540-1563)
  std::mt19937 generator(0x1200u);
  std::uniform_int_distribution<int> byte(0, 255);
  std::uniform_real_distribution<float> scale_dist(0.002f, 0.08f), input_dist(-2.0f, 2.0f);
  const std::size_t row_bytes = cols * bits / 8, groups = cols / 128;
  std::vector<std::uint8_t> codes(rows * row_bytes);
  for (auto& c : codes) c = static_cast<std::uint8_t>(byte(generator));
  std::vector<__half> scales(rows * groups);
  for (auto& s : scales) s = __float2half(scale_dist(generator));
  std::vector<__half> x(static_cast<std::size_t>(batch) * cols);
  for (auto& v : x) v = __float2half(input_dist(generator));

  DeviceBuffer<std::uint8_t> d_rowmajor(codes.size()), d_codes(codes.size());
  DeviceBuffer<__half> d_scales_rm(scales.size()), d_scales(scales.size()), d_x(x.size());
  DeviceBuffer<std::int8_t> d_act(x.size());
  DeviceBuffer<__half> d_act_scales(static_cast<std::size_t>(batch) * groups);
  DeviceBuffer<std::int32_t> d_act_sums(static_cast<std::size_t>(batch) * groups);
  DeviceBuffer<float> d_out(static_cast<std::size_t>(batch) * rows);
  if (!d_rowmajor.p || !d_codes.p || !d_scales.p || !d_out.p) return fail(GFXB_OUT_OF_MEMORY);
  if (!cuda_ok(cudaMemcpy(d_rowmajor.p, codes.data(), codes.size(), cudaMemcpyHostToDevice), "upload") ||
      !cuda_ok(cudaMemcpy(d_scales_rm.p, scales.data(), scales.size() * 2, cudaMemcpyHostToDevice), "upload") ||
      !cuda_ok(cudaMemcpy(d_x.p, x.data(), x.size() * 2, cudaMemcpyHostToDevice), "upload")) {
    return 1;
  }
  CLI_TRY(gfxb_repack_rowmajor_to_b200(format, d_rowmajor.p, d_codes.p, rows, cols, nullptr));
  CLI_TRY(gfxb_tile_scales(reinterpret_cast<const std::uint16_t*>(d_scales_rm.p),
                           reinterpret_cast<std::uint16_t*>(d_scales.p), rows, cols, nullptr));
  const bool f16 = activation == "f16";
  const int act_bits = activation == "a8" ? 8 : 4;
  if (!f16) {
    CLI_TRY(gfxb_pack_activation(act_bits, reinterpret_cast<const std::uint16_t*>(d_x.p), d_act.p,
                                 reinterpret_cast<std::uint16_t*>(d_act_scales.p), d_act_sums.p, nullptr, cols,
                                 batch, nullptr));
  }
  gfxb_gemv_matrix matrix{d_codes.p, reinterpret_cast<const std::uint16_t*>(d_scales.p), d_out.p, rows, 0};
  auto launch = [&]() {
    return f16 ? gfxb_lowbit_gemv_f16(format, &matrix, 1, reinterpret_cast<const std::uint16_t*>(d_x.p), cols, batch,
                                      nullptr)
               : gfxb_lowbit_gemv(format, &matrix, 1, d_act.p, reinterpret_cast<const std::uint16_t*>(d_act_scales.p),
                                  d_act_sums.p, cols, batch, nullptr);
  };
  for (int i = 0; i < 10; ++i) CLI_TRY(launch());
  cudaEvent_t start, stop;
  cudaEventCreate(&start);
  cudaEventCreate(&stop);
  cudaEventRecord(start);
  for (int i = 0; i < iterations; ++i) CLI_TRY(launch());
  cudaEventRecord(stop);
  if (!cuda_ok(cudaEventSynchronize(stop), "timing")) return 1;
  float ms = 0.0f;
  cudaEventElapsedTime(&ms, start, stop);
  cudaEventDestroy(start);
  cudaEventDestroy(stop);

  std::vector<float> out(static_cast<std::size_t>(batch) * rows);
  if (!cuda_ok(cudaMemcpy(out.data(), d_out.p, out.size() * 4, cudaMemcpyDeviceToHost), "download")) return 1;
  // the activation the GPU multiplied: fp16 values, or the device's A4/A8 codes times their scales
  std::vector<double> a(x.size());
  if (f16) {
    for (std::size_t i = 0; i < x.size(); ++i) a[i] = __half2float(x[i]);
  } else {
    std::vector<std::int8_t> act(x.size());
    std::vector<__half> act_scales(static_cast<std::size_t>(batch) * groups);
    cudaMemcpy(act.data(), d_act.p, act.size(), cudaMemcpyDeviceToHost);
    cudaMemcpy(act_scales.data(), d_act_scales.p, act_scales.size() * 2, cudaMemcpyDeviceToHost);
    for (unsigned b = 0; b < batch; ++b) {
      for (std::size_t c = 0; c < cols; ++c) {
        const std::size_t g = c / 128;
        a[b * cols + c] = act[b * cols + g * 128 + fragment_offset(c % 128)] *
                          static_cast<double>(__half2float(act_scales[b * groups + g]));
      }
    }
  }
  const double tolerance = f16 ? 0.003 : 0.008;  // the reference's sampled check (main.cpp:1499, 1674)
  double max_error = 0.0;
  for (unsigned b = 0; b < batch; ++b) {
    for (const std::size_t row : {std::size_t{0}, rows / 2, rows - 1}) {
      double expected = 0.0;
      for (std::size_t c = 0; c < cols; ++c) {
        double w = level(codes.data() + row * row_bytes, c, bits) * static_cast<double>(__half2float(scales[row * groups + c / 128]));
        if (f16) w = __half2float(__float2half(static_cast<float>(w)));  // fp16(q * scale), lowbit_gemv.hip:800-815
        expected += w * a[b * cols + c];
      }
      const double actual = out[b * rows + row], error = std::fabs(expected - actual);
      max_error = std::max(max_error, error);
      if (!std::isfinite(actual) || error > tolerance * std::max(1.0, std::fabs(expected))) {
        std::fprintf(stderr, "error: validation failed at batch %u row %zu: expected %.6f actual %.6f\n", b, row,
                     expected, actual);
        return 1;
      }
    }
  }
  const double seconds = ms / 1000.0;
  const double algorithmic = static_cast<double>(codes.size()) + scales.size() * 2.0 +
                             batch * (f16 ? cols * 2.0 : cols * act_bits / 8.0 + groups * 2.0) + batch * rows * 4.0;
  gfxb_device_info info{};
  gfxb_require_sm100_device(0, &info);
  std::printf("device:             %s\nformat:             %s x %s\nshape:              [%zu,%zu]\nbatch:              %u\n"
              "packed weights:     %zu bytes\nmean launch:        %.3f us\npacked bandwidth:   %.1f GB/s\n"
              "algorithmic bw:     %.1f GB/s (codes + scales + activation + output)\nmax sampled error:  %.3g\n"
              "validation:         pass\n",
              info.name, fmt_name.c_str(), activation.c_str(), rows, cols, batch, codes.size(), ms * 1000.0 / iterations,
              codes.size() * iterations / seconds / 1e9, algorithmic * iterations / seconds / 1e9, max_error);
  return 0;
}

// ---- models -----------------------------------------------------------------------

gfxb_model_config model_config(const Args& args) {
  gfxb_model_config c{};
  if (args.flag("--small")) {
    c = {1024, 2048, 8, 4, 4, 16, 8, 2, 4096, 3072, 3, 4, 4, 4, 4, 320, 0x5EED};
  } else {
    c = {5120, 17408, 64, 4, 16, 48, 24, 4, 151936, 98304, 3, 4, 4, 4, 4, 512, 0x5EED};
  }
  c.layers = static_cast<std::uint32_t>(args.number("--layers", c.layers));
  c.max_context = static_cast<std::uint32_t>(args.number("--context", c.max_context));
  if (args.flag("--a8")) c.activation_bits = 8;
  return c;
}

struct Model {
  gfxb_engine* engine = nullptr;
  gfxb_model_config config{};
  ~Model() { gfxb_engine_destroy(engine); }
};

int open_model(const Args& args, bool mtp, Model& model) {
  const std::string path = args.get("--artifact", "");
  const int device = static_cast<int>(args.number("--device", 0));
  if (!path.empty()) {
    gfxb_artifact_load_options options{args.flag("--a8") ? 8u : 4u,
                                       static_cast<std::uint32_t>(args.number("--context", 512)), 0, mtp ? 1u : 0u, 1u};
    const int status = gfxb_engine_create_from_artifact(path.c_str(), &options, device, 0, 1, nullptr, &model.engine);
    if (status != GFXB_OK) return status;
    return gfxb_engine_config(model.engine, &model.config);
  }
  model.config = model_config(args);
  return gfxb_engine_create_synthetic(&model.config, device, 0, 1, nullptr, mtp ? 1 : 0, &model.engine);
}

std::uint32_t prompt_token(std::uint64_t index, std::uint32_t vocab) {
  std::uint64_t z = 0x9E3779B97F4A7C15ull * (index + 1) + 0x1200;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return static_cast<std::uint32_t>((z ^ (z >> 31)) % vocab);
}

struct Session {
  gfxb_session* s = nullptr;
  ~Session() { gfxb_session_destroy(s); }
};

int make_session(Model& model, std::uint32_t context, std::uint32_t verifier, std::uint32_t step_kernel, Session& out) {
  gfxb_session_config config{context, verifier, 1, step_kernel};
  return gfxb_session_create(model.engine, &config, &out.s);
}

// decode-bench (main.cpp:790-844): serial prefill of a 64-token prompt, then timed greedy steps.
int decode_bench(const Args& args) {
  Model model;
  CLI_TRY(open_model(args, false, model));
  Session session;
  CLI_TRY(make_session(model, model.config.max_context, 0,
                       args.flag("--persistent") ? GFXB_STEP_PERSISTENT : GFXB_STEP_AUTO, session));
  const unsigned prompt = std::min(64u, model.config.max_context / 4);
  const unsigned steps = static_cast<unsigned>(
      std::min<long>(args.number("--steps", 128), model.config.max_context - prompt - 8));
  std::uint32_t token = 0;
  for (unsigned i = 0; i < prompt; ++i) CLI_TRY(gfxb_session_greedy_step(session.s, prompt_token(i, model.config.vocab), &token));
  for (int i = 0; i < 3; ++i) CLI_TRY(gfxb_session_greedy_step(session.s, token, &token));
  const double begin = now_ms();
  for (unsigned i = 0; i < steps; ++i) CLI_TRY(gfxb_session_greedy_step(session.s, token, &token));
  const double elapsed = now_ms() - begin;
  std::uint64_t weights = 0;
  gfxb_engine_weight_bytes(model.engine, &weights);
  std::printf("decode: %u layers, hidden %u, vocab %u, %u prompt tokens, %u timed greedy steps\n"
              "  time per token:   %.3f ms\n  decode speed:     %.2f tokens/s\n  weight stream:    %.1f GB/s\n"
              "  last token:       %u\n",
              model.config.layers, model.config.hidden, model.config.vocab, prompt, steps, elapsed / steps,
              steps * 1000.0 / elapsed, weights / (elapsed / steps / 1000.0) / 1e9, token);
  return 0;
}

// block-bench (main.cpp:846-915): a W-token causal block must emit the tokens of W serial steps.
int block_bench(const Args& args) {
  Model model;
  CLI_TRY(open_model(args, false, model));
  const unsigned width = static_cast<unsigned>(args.number("--width", 32));
  if (width == 0 || width > 32) {
    std::fprintf(stderr, "error: --width must be in [1, 32]\n");
    return 2;
  }
  Session block, serial;
  CLI_TRY(make_session(model, model.config.max_context, 0, GFXB_STEP_AUTO, block));
  CLI_TRY(make_session(model, model.config.max_context, 0, GFXB_STEP_AUTO, serial));
  std::vector<std::uint32_t> tokens(width), got(width), want(width);
  for (unsigned i = 0; i < width; ++i) tokens[i] = prompt_token(i, model.config.vocab);
  CLI_TRY(gfxb_session_block_step(block.s, tokens.data(), width, got.data()));  // warm-up and parity
  for (unsigned i = 0; i < width; ++i) CLI_TRY(gfxb_session_greedy_step(serial.s, tokens[i], &want[i]));
  if (got != want) {
    const auto at = std::mismatch(got.begin(), got.end(), want.begin()).first - got.begin();
    std::fprintf(stderr, "error: block token %td differs: block %u serial %u\n", at, got[at], want[at]);
    return 1;
  }
  const int rounds = 8;
  const double begin = now_ms();
  for (int r = 0; r < rounds; ++r) {
    for (unsigned i = 0; i < width; ++i) tokens[i] = got[(i + 1) % width];
    CLI_TRY(gfxb_session_block_step(block.s, tokens.data(), width, got.data()));
  }
  const double elapsed = now_ms() - begin;
  std::printf("causal verifier block passed\n  width:            %u\n  time per block:   %.3f ms\n"
              "  evaluated speed:  %.2f tokens/s\n  serial parity:    exact token IDs\n",
              width, elapsed / rounds, width * rounds * 1000.0 / elapsed);
  return 0;
}

// spec-bench (main.cpp:917-998): the speculative stream must equal the serial greedy stream.
int spec_bench(const Args& args) {
  Model model;
  CLI_TRY(open_model(args, true, model));
  const unsigned depth = static_cast<unsigned>(args.number("--depth", 4));
  const std::size_t minimum = static_cast<std::size_t>(args.number("--tokens", 64));
  if (depth == 0 || depth > 31 || minimum + depth + 2 > model.config.max_context) {
    std::fprintf(stderr, "error: --depth must be in [1, 31] and the stream must fit the context\n");
    return 2;
  }
  Session spec, serial;
  CLI_TRY(make_session(model, model.config.max_context, args.flag("--eager") ? 0 : depth + 1, GFXB_STEP_AUTO, spec));
  CLI_TRY(make_session(model, model.config.max_context, 0, GFXB_STEP_AUTO, serial));
  const std::uint32_t start = prompt_token(0, model.config.vocab);
  std::uint32_t first = 0;
  CLI_TRY(gfxb_session_greedy_step(spec.s, start, &first));
  std::vector<std::uint32_t> stream{first};
  std::size_t proposed = 0, accepted = 0, rounds = 0;
  std::uint32_t seed = first, out[32];
  const double begin = now_ms();
  while (stream.size() < minimum) {
    unsigned count = 0, ok = 0;
    CLI_TRY(gfxb_session_speculative_step(spec.s, seed, depth, out, &count, &ok));
    proposed += depth;
    accepted += ok;
    ++rounds;
    stream.insert(stream.end(), out, out + count);
    seed = out[count - 1];
  }
  const double elapsed = now_ms() - begin;
  std::vector<std::uint32_t> reference;
  std::uint32_t token = 0;
  CLI_TRY(gfxb_session_greedy_step(serial.s, start, &token));
  reference.push_back(token);
  while (reference.size() < stream.size()) {
    CLI_TRY(gfxb_session_greedy_step(serial.s, token, &token));
    reference.push_back(token);
  }
  if (reference != stream) {
    const auto at = std::mismatch(reference.begin(), reference.end(), stream.begin()).first - reference.begin();
    std::fprintf(stderr, "error: speculative stream differs from serial target at token %td: serial %u speculative %u\n",
                 at, reference[at], stream[at]);
    return 1;
  }
  const std::size_t measured = stream.size() - 1;
  std::printf("MTP speculative decode passed\n  draft depth:      %u (%s)\n  rounds:           %zu\n"
              "  measured tokens:  %zu\n  proposed drafts:  %zu\n  accepted drafts:  %zu\n  acceptance:       %.3f%%\n"
              "  tokens/round:     %.3f\n  total time:       %.3f ms\n  effective speed:  %.3f tokens/s\n"
              "  serial parity:    exact token IDs\n",
              depth, args.flag("--eager") ? "eager" : "CUDA graph", rounds, measured, proposed, accepted,
              proposed ? accepted * 100.0 / proposed : 0.0, rounds ? double(measured) / rounds : 0.0, elapsed,
              measured * 1000.0 / elapsed);
  return 0;
}

int export_artifact(const Args& args) {
  if (args.positional.empty()) {
    std::fprintf(stderr, "usage: export PATH [--small] [--layers L]\n");
    return 2;
  }
  Model model;
  CLI_TRY(open_model(args, true, model));
  CLI_TRY(gfxb_engine_export_artifact(model.engine, args.positional[0].c_str(), "seeded-random-init"));
  std::printf("wrote %s\n", args.positional[0].c_str());
  return 0;
}

void usage() {
  std::fprintf(stderr,
               "usage: gfxinfer-b200 <probe|inspect|bench-gemv|decode-bench|block-bench|spec-bench|export> [options]\n");
}

}  // namespace

int main(int argc, char** argv) {
  if (argc < 2) {
    usage();
    return 2;
  }
  const std::string command = argv[1];
  const Args args = parse(argc, argv, 2);
  if (command == "probe") return probe(args);
  if (command == "inspect") return inspect(args);
  if (command == "bench-gemv") return bench_gemv(args);
  if (command == "decode-bench") return decode_bench(args);
  if (command == "block-bench") return block_bench(args);
  if (command == "spec-bench") return spec_bench(args);
  if (command == "export") return export_artifact(args);
  usage();
  return 2;
}
