// Engine and decode session: the B200 counterpart of the reference's
// src/engine.cpp and src/qwen_runtime.cpp.
//
// Engine: one device arena per GPU holding every weight of the model (or of
// this rank's tensor-parallel shard), generated on the device from a seed.
// Session: one arena of activations, recurrent states, KV caches and logs;
// the 64-layer forward for a causal block of 1..32 tokens; the greedy step as
// a replayed CUDA graph that reads its token and position from device memory;
// MTP drafting and the speculative verify/rollback transaction.
//
// Tensor parallelism (absent in the reference): column-parallel projections
// (GDN qkv/z, attention q/k/v, MLP gate/up, LM-head vocabulary rows) and
// row-parallel ones (GDN out, attention o, MLP down, MTP fc) with one NCCL
// all-reduce of the fp32 partial output, captured inside the graph.
#include <dlfcn.h>
#include <nccl.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <memory>
#include <string>
#include <vector>

#include "gfxb/artifact.h"
#include "gfxb/gfxb.h"
#include "host/artifact_internal.h"
#include "kernels/common.cuh"
#include "kernels/ops.cuh"
#include "kernels/peer.cuh"
#include "kernels/token_loop.cuh"

namespace gfxb {

int lowbit_gemv(int format, const gfxb_gemv_matrix* matrices, unsigned matrix_count, const std::int8_t* act_codes,
                const std::uint16_t* act_scales, const std::int32_t* act_sums, std::size_t columns,
                std::size_t act_stride, unsigned batch, cudaStream_t stream);
int generate_b200_weights(std::uint64_t seed, std::uint32_t tensor, int format, std::uint8_t* codes,
                          std::uint16_t* tiled_scales, std::size_t rows, std::size_t columns,
                          std::size_t global_columns, std::size_t column_offset, const std::uint32_t* segment_local,
                          const std::uint32_t* segment_global, std::uint32_t segments, cudaStream_t stream);
int generate_rowmajor_weights(std::uint64_t seed, std::uint32_t tensor, int format, std::uint8_t* codes,
                              std::uint16_t* scales, std::size_t rows, std::size_t columns, cudaStream_t stream);
int generate_bf16(std::uint64_t seed, std::uint32_t tensor, std::uint64_t offset, std::uint64_t count, float lo,
                  float hi, std::uint16_t* out, cudaStream_t stream);
int read_gemv_error(std::uint32_t* value, bool clear);
int untile_gfx12_rowmajor(int format, const std::uint8_t* tiled_codes, const std::uint16_t* tiled_scales,
                          std::uint8_t* codes, std::uint16_t* scales, std::size_t rows, std::size_t columns,
                          cudaStream_t stream);

namespace {

int cuda_check(cudaError_t error, const char* context) {
  if (error == cudaSuccess) return GFXB_OK;
  set_error_cuda(error, context);
  return error == cudaErrorMemoryAllocation ? GFXB_OUT_OF_MEMORY : GFXB_CUDA_ERROR;
}

// ---------------------------------------------------------------------------
// NCCL, resolved at run time (the process usually has it loaded already).
// ---------------------------------------------------------------------------

struct NcclApi {
  void* handle = nullptr;
  ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
  ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
  ncclResult_t (*comm_abort)(ncclComm_t) = nullptr;
  ncclResult_t (*all_reduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                             cudaStream_t) = nullptr;
  ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
  const char* (*error_string)(ncclResult_t) = nullptr;
};

int load_nccl(NcclApi& api) {
  if (api.handle != nullptr) return GFXB_OK;
  const char* names[] = {"libnccl.so.2", "libnccl.so"};
  for (const char* name : names) {
    api.handle = dlopen(name, RTLD_NOW | RTLD_GLOBAL);
    if (api.handle != nullptr) break;
  }
  if (api.handle == nullptr) return fail(GFXB_UNSUPPORTED, "NCCL (libnccl.so.2) could not be loaded");
  api.get_unique_id = reinterpret_cast<decltype(api.get_unique_id)>(dlsym(api.handle, "ncclGetUniqueId"));
  api.comm_init_rank = reinterpret_cast<decltype(api.comm_init_rank)>(dlsym(api.handle, "ncclCommInitRank"));
  api.comm_destroy = reinterpret_cast<decltype(api.comm_destroy)>(dlsym(api.handle, "ncclCommDestroy"));
  api.comm_abort = reinterpret_cast<decltype(api.comm_abort)>(dlsym(api.handle, "ncclCommAbort"));
  api.all_reduce = reinterpret_cast<decltype(api.all_reduce)>(dlsym(api.handle, "ncclAllReduce"));
  api.all_gather = reinterpret_cast<decltype(api.all_gather)>(dlsym(api.handle, "ncclAllGather"));
  api.error_string = reinterpret_cast<decltype(api.error_string)>(dlsym(api.handle, "ncclGetErrorString"));
  if (!api.get_unique_id || !api.comm_init_rank || !api.comm_destroy || !api.all_reduce || !api.all_gather) {
    return fail(GFXB_UNSUPPORTED, "NCCL is missing required entry points");
  }
  return GFXB_OK;
}

NcclApi& nccl() {
  static NcclApi api;
  return api;
}

int nccl_check(ncclResult_t result, const char* context) {
  if (result == ncclSuccess) return GFXB_OK;
  std::string message = std::string(context) + ": " +
                        (nccl().error_string ? nccl().error_string(result) : "NCCL error");
  set_error(message.c_str());
  return GFXB_CUDA_ERROR;
}

// ---------------------------------------------------------------------------
// synthetic model: tensor ids shared with the CPU oracle
// ---------------------------------------------------------------------------

enum Kind : std::uint32_t {
  kInputNorm = 0, kPostNorm, kGate, kUp, kDown,
  kQkv, kZ, kA, kB, kConv, kALog, kDtBias, kGdnNorm, kGdnOut,
  kQ, kK, kV, kQNorm, kKNorm, kO,
  kFc, kPreEmbNorm, kPreHiddenNorm, kMtpFinalNorm
};
constexpr std::uint32_t kLayerGlobal = 4096, kLayerMtp = 4097;
constexpr std::uint32_t kEmbedding = 0, kFinalNorm = 1, kLmHead = 2;
constexpr unsigned kMaxBlock = 32;

std::uint32_t tensor_id(std::uint32_t layer, std::uint32_t kind) { return layer * 32u + kind; }
int format_of(std::uint32_t bits) { return bits == 2 ? GFXB_W2 : (bits == 3 ? GFXB_W3 : GFXB_W4); }
int bits_of_format(int format) { return format == GFXB_W2 ? 2 : (format == GFXB_W3 ? 3 : 4); }

struct QMatrix {
  std::uint8_t* codes = nullptr;
  std::uint16_t* scales = nullptr;
  std::uint32_t rows = 0, cols = 0;
  int format = 0;
};

struct Layer {
  bool attention = false;
  std::uint32_t state_index = 0;
  std::uint16_t *input_norm = nullptr, *post_norm = nullptr;
  QMatrix gate, up, down;
  QMatrix qkv, z, a, b, out;
  std::uint16_t *conv = nullptr, *a_log = nullptr, *dt_bias = nullptr, *gdn_norm = nullptr;
  QMatrix q, k, v;
  std::uint16_t *q_norm = nullptr, *k_norm = nullptr;
};

struct Shard {
  std::uint32_t tp = 1, rank = 0;
  std::uint32_t nk = 0, kh0 = 0, nv = 0, vh0 = 0;   // GDN key/value heads of this rank
  std::uint32_t nq = 0, qh0 = 0, nkv = 0, kv0 = 0;  // attention heads of this rank
  std::uint32_t inter = 0, i0 = 0;                  // MLP intermediate slice
  std::uint32_t vocab = 0, v0 = 0;                  // LM-head rows
  std::uint32_t fc_cols = 0, fc0 = 0;               // MTP fc K slice
  std::uint32_t channels = 0;                       // GDN conv channels of this rank
};

struct Planner {
  std::byte* base = nullptr;
  std::size_t offset = 0;
  template <class T>
  T* take(std::size_t count) {
    const std::size_t at = (offset + 255u) & ~static_cast<std::size_t>(255u);
    offset = at + count * sizeof(T);
    return base != nullptr ? reinterpret_cast<T*>(base + at) : nullptr;
  }
};

}  // namespace
}  // namespace gfxb

struct gfxb_engine {
  gfxb_model_config cfg{};
  int device = 0;
  bool has_mtp = false;
  gfxb::Shard shard;
  std::byte* arena = nullptr;
  std::size_t arena_bytes = 0;
  std::vector<gfxb::Layer> layers;
  gfxb::Layer mtp;
  std::uint8_t* emb_codes = nullptr;
  std::uint16_t* emb_scales = nullptr;
  gfxb::QMatrix lm_head, fc;
  std::uint16_t *final_norm = nullptr, *pre_emb_norm = nullptr, *pre_hidden_norm = nullptr,
                *mtp_final_norm = nullptr;
  cudaStream_t stream = nullptr;
  ncclComm_t comm = nullptr;
  std::uint32_t gdn_layers = 0, attention_layers = 0;
};

namespace gfxb {
namespace {

int validate_config(const gfxb_model_config& c, std::uint32_t tp) {
  auto bad = [](const char* message) { return fail(GFXB_INVALID_ARGUMENT, message); };
  if (c.hidden == 0 || c.hidden % 256 != 0 || c.hidden / 256 > 40) return bad("hidden must be a multiple of 256");
  if (c.intermediate % (128 * tp) != 0 || (c.intermediate / tp) % 16 != 0) return bad("intermediate must split into 128-column shards");
  if (c.layers == 0 || c.attention_interval == 0) return bad("layer count must be positive");
  if (c.gdn_key_heads == 0 || c.gdn_value_heads % c.gdn_key_heads != 0) return bad("GDN value heads must be a multiple of key heads");
  if (c.gdn_key_heads % tp != 0 || c.gdn_value_heads % tp != 0) return bad("GDN heads must divide by the TP size");
  if (c.gdn_value_heads % 16 != 0) return bad("GDN value heads must be a multiple of 16 (a/b projection tiles)");
  if (c.q_heads % tp != 0 || c.kv_heads == 0 || c.q_heads % c.kv_heads != 0 || c.q_heads / c.kv_heads > 8) return bad("invalid attention head counts");
  if (c.vocab % (16 * tp) != 0) return bad("vocabulary must split into 16-row shards");
  if ((2 * c.hidden / tp) % 128 != 0) return bad("MTP fc input must split into 128-column shards");
  if (c.activation_bits != 4 && c.activation_bits != 8) return bad("activation bits must be 4 or 8");
  for (std::uint32_t bits : {c.mlp_bits, c.proj_bits, c.head_bits}) {
    if (bits < 2 || bits > 4) return bad("weight bits must be 2, 3 or 4");
  }
  if (c.emb_bits != 2 && c.emb_bits != 4) return bad("embedding bits must be 2 or 4");
  if (c.max_context == 0) return bad("maximum context must be positive");
  return GFXB_OK;
}

Shard make_shard(const gfxb_model_config& c, std::uint32_t tp, std::uint32_t rank) {
  Shard s;
  s.tp = tp;
  s.rank = rank;
  s.nk = c.gdn_key_heads / tp;
  s.kh0 = rank * s.nk;
  s.nv = c.gdn_value_heads / tp;
  s.vh0 = rank * s.nv;
  s.nq = c.q_heads / tp;
  s.qh0 = rank * s.nq;
  const std::uint32_t group = c.q_heads / c.kv_heads;
  s.kv0 = s.qh0 / group;
  s.nkv = (s.qh0 + s.nq - 1) / group - s.kv0 + 1;
  s.inter = c.intermediate / tp;
  s.i0 = rank * s.inter;
  s.vocab = c.vocab / tp;
  s.v0 = rank * s.vocab;
  s.fc_cols = 2 * c.hidden / tp;
  s.fc0 = rank * s.fc_cols;
  s.channels = 2 * s.nk * 128 + s.nv * 128;
  return s;
}

// Where the weights come from: seeded synthetic generation on the device, or
// a `.gfxi` artifact (mapped on the host; copied shard by shard, repacked to
// the b200 layout when the recipe is a reference gfx12 tiled one).
struct WeightSource {
  const gfxi::View* view = nullptr;   // null: synthetic weights
  bool gfx12 = false;                 // reference tiled recipe (else "b200-v1")
  bool sequential_w3 = false;         // the tiled recipe's W3 fragments are sequential 3-bit
  std::uint8_t* scratch = nullptr;    // device staging for repacks (placement pass)
  std::size_t scratch_bytes = 0;      // largest staging need (planning pass)
};

std::string layer_name(std::uint32_t id, const char* suffix) {
  if (id == kLayerMtp) return std::string("mtp.layers.0.") + suffix;
  return "model.language_model.layers." + std::to_string(id) + "." + suffix;
}

int bits_of_quantization(std::uint16_t quantization) {
  return quantization == GFXB_QUANT_W2G128 ? 2 : (quantization == GFXB_QUANT_W3G128 ? 3 : (quantization == GFXB_QUANT_W4G128 ? 4 : 0));
}

int artifact_error(const std::string& message) { return fail(GFXB_CORRUPT_ARTIFACT, message.c_str()); }

// Checks a 2-D low-bit tensor of the artifact against the expected global shape.
int check_matrix_tensor(const gfxi::View& view, const WeightSource& src, const std::string& name,
                        std::uint32_t global_rows, std::uint32_t global_cols, int* bits) {
  const gfxi::Tensor* t = view.find(name);
  if (t == nullptr) return artifact_error("artifact lacks " + name);
  const int b = bits_of_quantization(t->quantization);
  if (t->rank != 2 || t->dtype != GFXB_DTYPE_U8 || b == 0 || t->dimensions[0] != global_rows ||
      t->dimensions[1] != global_cols) {
    return artifact_error("artifact tensor has an unexpected shape or format: " + name);
  }
  const std::uint64_t code_bytes = static_cast<std::uint64_t>(global_rows) * global_cols * b / 8;
  const std::uint64_t scale_bytes = static_cast<std::uint64_t>(global_rows) * (global_cols / 128) * 2;
  if (t->data_bytes != code_bytes || t->aux_bytes != scale_bytes) {
    return artifact_error("artifact tensor payload sizes do not match its shape: " + name);
  }
  if (src.gfx12 && b == 3 && !src.sequential_w3) {
    return fail(GFXB_UNSUPPORTED, "bit-plane W3 tiles (recipes without w3seq) are not supported");
  }
  *bits = b;
  return GFXB_OK;
}

// Copies this shard's rows (row segments) and columns (one 128-group range)
// of a [global_rows][global_cols] tensor stored as [N/16][K/128][block] (both
// the b200 and the gfx12 tiled layouts, and the tiled scales, have this
// blocking) into a packed local block array.
int copy_blocks(const std::byte* source, std::uint32_t global_cols, std::uint32_t block_bytes, std::uint8_t* dest,
                std::uint32_t cols, std::uint32_t col_offset, const std::vector<std::uint32_t>& local_begin,
                const std::vector<std::uint32_t>& global_begin, std::uint32_t rows, cudaStream_t stream) {
  const std::size_t G = global_cols / 128, g0 = col_offset / 128, ng = cols / 128;
  for (std::size_t i = 0; i < local_begin.size(); ++i) {
    const std::uint32_t end = i + 1 < local_begin.size() ? local_begin[i + 1] : rows;
    const std::size_t tiles = (end - local_begin[i]) / 16, t_src = global_begin[i] / 16, t_dst = local_begin[i] / 16;
    if (tiles == 0) continue;
    GFXB_TRY(cuda_check(cudaMemcpy2DAsync(dest + t_dst * ng * block_bytes, ng * block_bytes,
                                          source + (t_src * G + g0) * block_bytes, G * block_bytes, ng * block_bytes,
                                          tiles, cudaMemcpyHostToDevice, stream),
                        "weight upload failed"));
  }
  return GFXB_OK;
}

// Plans (pass 1) or places and fills (pass 2) every weight of the shard.
int build_weights(gfxb_engine& e, Planner& plan, bool generate, WeightSource& src) {
  const gfxb_model_config& c = e.cfg;
  const Shard& s = e.shard;
  const cudaStream_t stream = e.stream;
  const std::uint64_t seed = c.seed;
  auto matrix = [&](QMatrix& m, std::uint32_t tensor, const std::string& name, std::uint32_t bits, std::uint32_t rows,
                    std::uint32_t cols, std::uint32_t global_rows, std::uint32_t global_cols, std::uint32_t col_offset,
                    std::vector<std::uint32_t> local_begin, std::vector<std::uint32_t> global_begin) -> int {
    if (src.view != nullptr) {
      int b = 0;
      GFXB_TRY(check_matrix_tensor(*src.view, src, name, global_rows, global_cols, &b));
      bits = static_cast<std::uint32_t>(b);
    }
    m.format = format_of(bits);
    m.rows = rows;
    m.cols = cols;
    const std::size_t code_bytes = static_cast<std::size_t>(rows) * cols * bits / 8;
    m.codes = plan.take<std::uint8_t>(code_bytes);
    m.scales = plan.take<std::uint16_t>(static_cast<std::size_t>(rows) * (cols / 128));
    if (src.view != nullptr && src.gfx12) src.scratch_bytes = std::max(src.scratch_bytes, code_bytes);
    if (!generate) return GFXB_OK;
    if (src.view == nullptr) {
      return generate_b200_weights(seed, tensor, m.format, m.codes, m.scales, rows, cols, global_cols, col_offset,
                                   local_begin.data(), global_begin.data(),
                                   static_cast<std::uint32_t>(local_begin.size()), stream);
    }
    const gfxi::Tensor& t = *src.view->find(name);
    std::uint8_t* codes = src.gfx12 ? src.scratch : m.codes;
    GFXB_TRY(copy_blocks(src.view->data(t), global_cols, bits * 256u, codes, cols, col_offset, local_begin,
                         global_begin, rows, stream));
    GFXB_TRY(copy_blocks(src.view->aux(t), global_cols, 32u, reinterpret_cast<std::uint8_t*>(m.scales), cols,
                         col_offset, local_begin, global_begin, rows, stream));
    if (src.gfx12) return gfxb_repack_gfx12_to_b200(m.format, src.scratch, m.codes, rows, cols, stream);
    return GFXB_OK;
  };
  auto simple = [&](QMatrix& m, std::uint32_t tensor, const std::string& name, std::uint32_t bits, std::uint32_t rows,
                    std::uint32_t cols, std::uint32_t row0, std::uint32_t global_rows, std::uint32_t global_cols,
                    std::uint32_t col0) -> int {
    return matrix(m, tensor, name, bits, rows, cols, global_rows, global_cols, col0, {0}, {row0});
  };
  // bf16 vectors: `count` values from element `offset` (of `total`) of the tensor
  auto vector_bf16 = [&](std::uint16_t*& out, std::uint32_t tensor, const std::string& name, std::uint64_t count,
                         std::uint64_t offset, std::uint64_t total, float lo, float hi) -> int {
    out = plan.take<std::uint16_t>(count);
    if (src.view != nullptr) {
      const gfxi::Tensor* t = src.view->find(name);
      if (t == nullptr) return artifact_error("artifact lacks " + name);
      std::uint64_t elements = t->rank == 0 ? 0 : 1;
      for (std::uint16_t d = 0; d < t->rank; ++d) elements *= t->dimensions[d];
      if (t->dtype != GFXB_DTYPE_BF16 || t->quantization != GFXB_QUANT_NONE || elements != total ||
          t->data_bytes != total * 2) {
        return artifact_error("artifact tensor has an unexpected shape or type: " + name);
      }
      if (!generate) return GFXB_OK;
      return cuda_check(cudaMemcpyAsync(out, src.view->data(*t) + offset * 2, count * 2, cudaMemcpyHostToDevice, stream),
                        "weight upload failed");
    }
    if (!generate) return GFXB_OK;
    return generate_bf16(seed, tensor, offset, count, lo, hi, out, stream);
  };
  const std::uint32_t H = c.hidden;
  auto mlp = [&](Layer& L, std::uint32_t id) -> int {
    GFXB_TRY(vector_bf16(L.input_norm, tensor_id(id, kInputNorm), layer_name(id, "input_layernorm.weight"), H, 0, H,
                         -0.1f, 0.1f));
    GFXB_TRY(vector_bf16(L.post_norm, tensor_id(id, kPostNorm), layer_name(id, "post_attention_layernorm.weight"), H, 0,
                         H, -0.1f, 0.1f));
    GFXB_TRY(simple(L.gate, tensor_id(id, kGate), layer_name(id, "mlp.gate_proj.weight"), c.mlp_bits, s.inter, H, s.i0,
                    c.intermediate, H, 0));
    GFXB_TRY(simple(L.up, tensor_id(id, kUp), layer_name(id, "mlp.up_proj.weight"), c.mlp_bits, s.inter, H, s.i0,
                    c.intermediate, H, 0));
    GFXB_TRY(simple(L.down, tensor_id(id, kDown), layer_name(id, "mlp.down_proj.weight"), c.mlp_bits, H, s.inter, 0, H,
                    c.intermediate, s.i0));
    if (L.gate.format != L.up.format) return artifact_error("gate and up projections differ in format");
    return GFXB_OK;
  };
  auto attention = [&](Layer& L, std::uint32_t id) -> int {
    GFXB_TRY(simple(L.q, tensor_id(id, kQ), layer_name(id, "self_attn.q_proj.weight"), c.proj_bits, s.nq * 512, H,
                    s.qh0 * 512, c.q_heads * 512, H, 0));
    GFXB_TRY(simple(L.k, tensor_id(id, kK), layer_name(id, "self_attn.k_proj.weight"), c.proj_bits, s.nkv * 256, H,
                    s.kv0 * 256, c.kv_heads * 256, H, 0));
    GFXB_TRY(simple(L.v, tensor_id(id, kV), layer_name(id, "self_attn.v_proj.weight"), c.proj_bits, s.nkv * 256, H,
                    s.kv0 * 256, c.kv_heads * 256, H, 0));
    GFXB_TRY(simple(L.out, tensor_id(id, kO), layer_name(id, "self_attn.o_proj.weight"), c.proj_bits, H, s.nq * 256, 0,
                    H, c.q_heads * 256, s.qh0 * 256));
    GFXB_TRY(vector_bf16(L.q_norm, tensor_id(id, kQNorm), layer_name(id, "self_attn.q_norm.weight"), 256, 0, 256,
                         -0.1f, 0.1f));
    GFXB_TRY(vector_bf16(L.k_norm, tensor_id(id, kKNorm), layer_name(id, "self_attn.k_norm.weight"), 256, 0, 256,
                         -0.1f, 0.1f));
    if (L.q.format != L.k.format || L.q.format != L.v.format) {
      return artifact_error("q/k/v projections differ in format");
    }
    return GFXB_OK;
  };
  auto gdn = [&](Layer& L, std::uint32_t id) -> int {
    const std::uint32_t nk_all = c.gdn_key_heads * 128, nv_all = c.gdn_value_heads * 128;
    const std::uint32_t channels_all = 2 * nk_all + nv_all;
    GFXB_TRY(matrix(L.qkv, tensor_id(id, kQkv), layer_name(id, "linear_attn.in_proj_qkv.weight"), c.proj_bits,
                    s.channels, H, channels_all, H, 0, {0, s.nk * 128, 2 * s.nk * 128},
                    {s.kh0 * 128, nk_all + s.kh0 * 128, 2 * nk_all + s.vh0 * 128}));
    GFXB_TRY(simple(L.z, tensor_id(id, kZ), layer_name(id, "linear_attn.in_proj_z.weight"), c.proj_bits, s.nv * 128, H,
                    s.vh0 * 128, nv_all, H, 0));
    GFXB_TRY(simple(L.a, tensor_id(id, kA), layer_name(id, "linear_attn.in_proj_a.weight"), c.proj_bits,
                    c.gdn_value_heads, H, 0, c.gdn_value_heads, H, 0));
    GFXB_TRY(simple(L.b, tensor_id(id, kB), layer_name(id, "linear_attn.in_proj_b.weight"), c.proj_bits,
                    c.gdn_value_heads, H, 0, c.gdn_value_heads, H, 0));
    GFXB_TRY(simple(L.out, tensor_id(id, kGdnOut), layer_name(id, "linear_attn.out_proj.weight"), c.proj_bits, H,
                    s.nv * 128, 0, H, nv_all, s.vh0 * 128));
    if (L.qkv.format != L.z.format || L.qkv.format != L.a.format || L.qkv.format != L.b.format) {
      return artifact_error("GDN input projections differ in format");
    }
    // conv weights [channels][4] (reference [channels][1][4]) follow the qkv channel map
    L.conv = plan.take<std::uint16_t>(static_cast<std::size_t>(s.channels) * 4);
    const std::uint64_t starts[3] = {static_cast<std::uint64_t>(s.kh0) * 128, nk_all + static_cast<std::uint64_t>(s.kh0) * 128,
                                     2ull * nk_all + static_cast<std::uint64_t>(s.vh0) * 128};
    const std::uint64_t counts[3] = {s.nk * 128ull, s.nk * 128ull, s.nv * 128ull};
    const std::string conv_name = layer_name(id, "linear_attn.conv1d.weight");
    const gfxi::Tensor* conv = nullptr;
    if (src.view != nullptr) {
      conv = src.view->find(conv_name);
      if (conv == nullptr || conv->dtype != GFXB_DTYPE_BF16 || conv->data_bytes != channels_all * 8ull) {
        return artifact_error("artifact lacks a valid " + conv_name);
      }
    }
    if (generate) {
      const std::uint32_t tensor = tensor_id(id, kConv);
      std::uint64_t local = 0;
      for (int i = 0; i < 3; ++i) {
        if (conv != nullptr) {
          GFXB_TRY(cuda_check(cudaMemcpyAsync(L.conv + local * 4, src.view->data(*conv) + starts[i] * 8, counts[i] * 8,
                                              cudaMemcpyHostToDevice, stream),
                              "weight upload failed"));
        } else {
          GFXB_TRY(generate_bf16(seed, tensor, starts[i] * 4, counts[i] * 4, -0.5f, 0.5f, L.conv + local * 4, stream));
        }
        local += counts[i];
      }
    }
    GFXB_TRY(vector_bf16(L.a_log, tensor_id(id, kALog), layer_name(id, "linear_attn.A_log"), s.nv, s.vh0,
                         c.gdn_value_heads, -1.0f, 1.0f));
    GFXB_TRY(vector_bf16(L.dt_bias, tensor_id(id, kDtBias), layer_name(id, "linear_attn.dt_bias"), s.nv, s.vh0,
                         c.gdn_value_heads, -1.0f, 1.0f));
    GFXB_TRY(vector_bf16(L.gdn_norm, tensor_id(id, kGdnNorm), layer_name(id, "linear_attn.norm.weight"), 128, 0, 128,
                         0.8f, 1.2f));
    return GFXB_OK;
  };
  e.layers.resize(c.layers);
  e.gdn_layers = e.attention_layers = 0;
  for (std::uint32_t i = 0; i < c.layers; ++i) {
    Layer& L = e.layers[i];
    L.attention = (i + 1) % c.attention_interval == 0;
    L.state_index = L.attention ? e.attention_layers++ : e.gdn_layers++;
    GFXB_TRY(mlp(L, i));
    GFXB_TRY(L.attention ? attention(L, i) : gdn(L, i));
  }
  // embedding (row-major, replicated), LM head (vocabulary rows), final norm
  {
    std::uint32_t emb_bits = c.emb_bits;
    const char* emb_name = "model.language_model.embed_tokens.weight";
    if (src.view != nullptr) {
      int b = 0;
      GFXB_TRY(check_matrix_tensor(*src.view, src, emb_name, c.vocab, H, &b));
      if (b == 3) return fail(GFXB_UNSUPPORTED, "the embedding must be W2 or W4");
      emb_bits = static_cast<std::uint32_t>(b);
    }
    const int format = format_of(emb_bits);
    const std::size_t code_bytes = static_cast<std::size_t>(c.vocab) * H * emb_bits / 8;
    const std::size_t scale_bytes = static_cast<std::size_t>(c.vocab) * (H / 128) * 2;
    e.emb_codes = plan.take<std::uint8_t>(code_bytes);
    e.emb_scales = plan.take<std::uint16_t>(static_cast<std::size_t>(c.vocab) * (H / 128));
    if (src.view != nullptr && src.gfx12) src.scratch_bytes = std::max(src.scratch_bytes, code_bytes + scale_bytes + 256);
    if (generate && src.view == nullptr) {
      GFXB_TRY(generate_rowmajor_weights(seed, tensor_id(kLayerGlobal, kEmbedding), format, e.emb_codes, e.emb_scales,
                                         c.vocab, H, stream));
    } else if (generate) {
      const gfxi::Tensor& t = *src.view->find(emb_name);
      if (src.gfx12) {
        std::uint8_t* staged_scales = src.scratch + ((code_bytes + 255) & ~std::size_t{255});
        GFXB_TRY(cuda_check(cudaMemcpyAsync(src.scratch, src.view->data(t), code_bytes, cudaMemcpyHostToDevice, stream),
                            "weight upload failed"));
        GFXB_TRY(cuda_check(cudaMemcpyAsync(staged_scales, src.view->aux(t), scale_bytes, cudaMemcpyHostToDevice, stream),
                            "weight upload failed"));
        GFXB_TRY(untile_gfx12_rowmajor(format, src.scratch, reinterpret_cast<const std::uint16_t*>(staged_scales),
                                       e.emb_codes, e.emb_scales, c.vocab, H, stream));
      } else {
        GFXB_TRY(cuda_check(cudaMemcpyAsync(e.emb_codes, src.view->data(t), code_bytes, cudaMemcpyHostToDevice, stream),
                            "weight upload failed"));
        GFXB_TRY(cuda_check(cudaMemcpyAsync(e.emb_scales, src.view->aux(t), scale_bytes, cudaMemcpyHostToDevice, stream),
                            "weight upload failed"));
      }
    }
    e.cfg.emb_bits = emb_bits;
  }
  GFXB_TRY(simple(e.lm_head, tensor_id(kLayerGlobal, kLmHead), "lm_head.weight", c.head_bits, s.vocab, H, s.v0, c.vocab,
                  H, 0));
  GFXB_TRY(vector_bf16(e.final_norm, tensor_id(kLayerGlobal, kFinalNorm), "model.language_model.norm.weight", H, 0, H,
                       -0.1f, 0.1f));
  if (e.has_mtp) {
    e.mtp.attention = true;
    GFXB_TRY(mlp(e.mtp, kLayerMtp));
    GFXB_TRY(attention(e.mtp, kLayerMtp));
    GFXB_TRY(simple(e.fc, tensor_id(kLayerMtp, kFc), "mtp.fc.weight", c.proj_bits, H, s.fc_cols, 0, H, 2 * H, s.fc0));
    GFXB_TRY(vector_bf16(e.pre_emb_norm, tensor_id(kLayerMtp, kPreEmbNorm), "mtp.pre_fc_norm_embedding.weight", H, 0, H,
                         -0.1f, 0.1f));
    GFXB_TRY(vector_bf16(e.pre_hidden_norm, tensor_id(kLayerMtp, kPreHiddenNorm), "mtp.pre_fc_norm_hidden.weight", H, 0,
                         H, -0.1f, 0.1f));
    GFXB_TRY(vector_bf16(e.mtp_final_norm, tensor_id(kLayerMtp, kMtpFinalNorm), "mtp.norm.weight", H, 0, H, -0.1f,
                         0.1f));
  }
  return GFXB_OK;
}

}  // namespace
}  // namespace gfxb

// ===========================================================================
// session
// ===========================================================================

struct gfxb_session {
  gfxb_engine* e = nullptr;
  gfxb_session_config cfg{};
  // tensor parallelism: the peer all-reduce's exchange buffers (own + mapped peers) and call counters
  std::uint8_t* peer_buffer = nullptr;
  std::uint8_t* exchange_peers[8] = {};
  std::uint32_t* peer_epochs = nullptr;
  std::uint32_t exchange_slot_floats = 0;
  bool peer_reduce = false;
  std::byte* arena = nullptr;
  std::size_t arena_bytes = 0;
  cudaStream_t stream = nullptr;
  // activations (capacity kMaxBlock tokens)
  __half* hidden[2] = {nullptr, nullptr};
  __half* post_attention = nullptr;
  std::int8_t* act_codes = nullptr;
  __half* act_scales = nullptr;
  std::int32_t* act_sums = nullptr;
  std::uint32_t act_width = 0;
  float *proj_main = nullptr, *proj_z = nullptr, *proj_a = nullptr, *proj_b = nullptr, *proj_k = nullptr,
        *proj_v = nullptr, *update = nullptr, *gate = nullptr, *up = nullptr, *logits = nullptr;
  __half *conv_out = nullptr, *gdn_out = nullptr, *query = nullptr, *attn_out = nullptr;
  float* attention_partials = nullptr;
  std::uint32_t* attention_tickets = nullptr;  // [nq] merge counters of the single-token attention
  std::uint32_t attention_chunks = 0;
  float* argmax_values = nullptr;
  std::uint32_t* argmax_indices = nullptr;
  std::uint32_t* gathered = nullptr;  // TP argmax exchange [tp][kMaxBlock][2]
  std::uint32_t* exchange = nullptr;  // [kMaxBlock][2]
  std::uint32_t* selected = nullptr;  // [kMaxBlock] target tokens
  std::uint32_t* tokens = nullptr;    // [kMaxBlock] input tokens
  std::uint64_t* position = nullptr;  // base position of the block
  // MTP
  __half *mtp_hidden = nullptr, *mtp_input = nullptr, *mtp_embed = nullptr, *target_snapshot = nullptr;
  std::uint32_t* draft_tokens = nullptr;  // [kMaxBlock]
  std::uint32_t* external_drafts = nullptr;  // [kMaxBlock] caller-supplied drafts
  std::uint64_t* mtp_positions = nullptr; // [kMaxBlock]
  std::uint32_t* seed_token = nullptr;
  // states
  __half *conv_states = nullptr, *conv_snapshot = nullptr, *conv_log = nullptr;
  float *gdn_states = nullptr, *gdn_snapshot = nullptr, *key_log = nullptr, *delta_log = nullptr,
        *decay_log = nullptr;
  __half *key_cache = nullptr, *value_cache = nullptr, *mtp_keys = nullptr, *mtp_values = nullptr;
  float *rope_cos = nullptr, *rope_sin = nullptr;
  // host state
  std::uint64_t host_position = 0, mtp_position = 0;
  bool mtp_chain_active = false;
  bool have_last_hidden = false;
  const __half* last_hidden = nullptr;
  std::uint32_t* pinned = nullptr;  // host staging
  cudaGraphExec_t greedy_graph = nullptr;
  cudaGraphExec_t spec_graph = nullptr;  // the speculative round for spec_drafts drafts
  unsigned spec_drafts = 0;
  // persistent token kernel
  __half* mlp_product = nullptr;  // fp16 SiLU(gate) * up of the token kernel's MLP
  gfxb::LoopOp* loop_ops = nullptr;
  gfxb::LoopControl* loop_control = nullptr;
  gfxb::LoopLaunch loop{};
  bool loop_ready = false;
  std::uint64_t* loop_trace = nullptr;  // timeline buffer, allocated on the first traced step
};

namespace gfxb {
namespace {

constexpr float kEps = 1.0e-6f;

struct Pack {
  std::int8_t* codes;
  __half* scales;
  std::int32_t* sums;
};

Pack pack_of(gfxb_session& s) { return Pack{s.act_codes, s.act_scales, s.act_sums}; }

int gemv(gfxb_session& s, const std::vector<std::pair<const QMatrix*, void*>>& mats, unsigned batch,
         std::size_t act_offset = 0, std::size_t act_stride = 0, bool f16_first = false) {
  gfxb_gemv_matrix items[4];
  for (std::size_t i = 0; i < mats.size(); ++i) {
    const QMatrix& m = *mats[i].first;
    items[i] = gfxb_gemv_matrix{m.codes, m.scales, mats[i].second, m.rows, (i == 0 && f16_first) ? 1 : 0};
  }
  const QMatrix& first = *mats[0].first;
  const std::size_t stride = act_stride != 0 ? act_stride : first.cols;
  return lowbit_gemv(first.format, items, static_cast<unsigned>(mats.size()), s.act_codes + act_offset,
                     reinterpret_cast<const std::uint16_t*>(s.act_scales) + act_offset / 128,
                     s.act_sums + act_offset / 128, first.cols, stride, batch, s.stream);
}

int all_reduce(gfxb_session& s, float* buffer, std::size_t count) {
  if (s.e->shard.tp == 1) return GFXB_OK;
  if (s.peer_reduce && count % 4 == 0 && count <= s.exchange_slot_floats) {
    PeerReduceArgs a;
    a.data = buffer;
    a.count = static_cast<std::uint32_t>(count);
    a.rank = s.e->shard.rank;
    a.ranks = s.e->shard.tp;
    for (std::uint32_t r = 0; r < a.ranks; ++r) a.buffers[r] = s.exchange_peers[r];
    a.epochs = s.peer_epochs;
    a.slot_floats = s.exchange_slot_floats;
    return launch_peer_all_reduce(a, s.stream);
  }
  return nccl_check(nccl().all_reduce(buffer, buffer, count, ncclFloat, ncclSum, s.e->comm, s.stream),
                    "NCCL all-reduce failed");
}

// Peer all-reduce setup (collective over the TP ranks, NCCL for the exchange):
// allocate and clear this rank's exchange buffer, gather every rank's IPC
// handle, map the peers' buffers, then agree (a min-reduction of a success
// flag) so that either every rank uses the peer path or none does.
// GFXB_PEER_ALLREDUCE=1 selects it; NCCL otherwise.
int setup_peer_reduce(gfxb_session& s) {
  const Shard& sh = s.e->shard;
  if (sh.tp == 1) return GFXB_OK;
  const char* env = std::getenv("GFXB_PEER_ALLREDUCE");
  if (env == nullptr || env[0] != '1') return GFXB_OK;
  int ok = 1;
  s.exchange_slot_floats = kMaxBlock * s.e->cfg.hidden;
  const std::size_t bytes = peer_exchange_bytes(sh.tp, s.exchange_slot_floats);
  cudaIpcMemHandle_t mine{};
  if (ok) ok = cudaMalloc(&s.peer_buffer, bytes) == cudaSuccess ? 1 : 0;
  if (ok) ok = cudaMalloc(&s.peer_epochs, kPeerCtas * sizeof(std::uint32_t)) == cudaSuccess ? 1 : 0;
  if (ok) ok = cudaMemset(s.peer_buffer, 0, bytes) == cudaSuccess ? 1 : 0;
  if (ok) ok = cudaMemset(s.peer_epochs, 0, kPeerCtas * sizeof(std::uint32_t)) == cudaSuccess ? 1 : 0;
  if (ok) ok = cudaIpcGetMemHandle(&mine, s.peer_buffer) == cudaSuccess ? 1 : 0;
  cudaGetLastError();
  // gather the handles (64 bytes each) and the flags through device memory
  std::uint8_t* staging = nullptr;
  const std::size_t handle_bytes = sizeof(cudaIpcMemHandle_t);
  GFXB_TRY(cuda_check(cudaMalloc(&staging, handle_bytes * (sh.tp + 1) + 8), "peer setup staging failed"));
  std::vector<std::uint8_t> handles(handle_bytes * sh.tp);
  int status = cuda_check(cudaMemcpy(staging + handle_bytes * sh.tp, &mine, handle_bytes, cudaMemcpyHostToDevice),
                          "peer setup copy failed");
  if (status == GFXB_OK) {
    status = nccl_check(nccl().all_gather(staging + handle_bytes * sh.tp, staging, handle_bytes, ncclUint8,
                                          s.e->comm, s.stream),
                        "NCCL all-gather of IPC handles failed");
  }
  if (status == GFXB_OK) status = cuda_check(cudaStreamSynchronize(s.stream), "peer setup failed");
  if (status == GFXB_OK) {
    status = cuda_check(cudaMemcpy(handles.data(), staging, handles.size(), cudaMemcpyDeviceToHost),
                        "peer setup copy failed");
  }
  for (std::uint32_t r = 0; status == GFXB_OK && ok && r < sh.tp; ++r) {
    if (r == sh.rank) {
      s.exchange_peers[r] = s.peer_buffer;
      continue;
    }
    cudaIpcMemHandle_t handle;
    std::memcpy(&handle, handles.data() + handle_bytes * r, handle_bytes);
    void* mapped = nullptr;
    if (cudaIpcOpenMemHandle(&mapped, handle, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
      cudaGetLastError();
      ok = 0;
      break;
    }
    s.exchange_peers[r] = static_cast<std::uint8_t*>(mapped);
  }
  // every rank must take the same path
  std::int32_t agreed = ok;
  if (status == GFXB_OK) {
    status = cuda_check(cudaMemcpy(staging, &agreed, sizeof agreed, cudaMemcpyHostToDevice), "peer setup copy failed");
  }
  if (status == GFXB_OK) {
    status = nccl_check(nccl().all_reduce(staging, staging, 1, ncclInt32, ncclMin, s.e->comm, s.stream),
                        "NCCL agreement on the peer all-reduce failed");
  }
  if (status == GFXB_OK) status = cuda_check(cudaStreamSynchronize(s.stream), "peer setup failed");
  if (status == GFXB_OK) {
    status = cuda_check(cudaMemcpy(&agreed, staging, sizeof agreed, cudaMemcpyDeviceToHost), "peer setup copy failed");
  }
  cudaFree(staging);
  s.peer_reduce = status == GFXB_OK && agreed == 1;
  return status;
}

void release_peer_reduce(gfxb_session& s) {
  for (std::uint32_t r = 0; r < 8; ++r) {
    if (s.exchange_peers[r] != nullptr && s.exchange_peers[r] != s.peer_buffer) cudaIpcCloseMemHandle(s.exchange_peers[r]);
    s.exchange_peers[r] = nullptr;
  }
  if (s.peer_buffer != nullptr) cudaFree(s.peer_buffer);
  if (s.peer_epochs != nullptr) cudaFree(s.peer_epochs);
  s.peer_buffer = nullptr;
  s.peer_epochs = nullptr;
  s.peer_reduce = false;
}

int norm_pack(gfxb_session& s, const __half* residual, const float* update, __half* residual_out,
              const std::uint16_t* weight, unsigned batch, __half* normalized_out = nullptr,
              std::size_t act_offset = 0) {
  NormPackArgs a;
  a.residual = residual;
  a.update = update;
  a.residual_out = residual_out;
  a.weight = weight;
  a.unit_offset = 1;
  a.epsilon = kEps;
  a.elements = s.e->cfg.hidden;
  a.normalized_out = normalized_out;
  a.act_codes = s.act_codes + act_offset;
  a.act_scales = s.act_scales + act_offset / 128;
  a.act_sums = s.act_sums + act_offset / 128;
  return launch_norm_pack(a, static_cast<int>(s.e->cfg.activation_bits), batch, s.stream);
}

int embed_norm_pack(gfxb_session& s, const std::uint32_t* device_tokens, __half* residual_out,
                    const std::uint16_t* weight, unsigned batch, std::size_t act_offset = 0) {
  NormPackArgs a;
  a.weight = weight;
  a.unit_offset = 1;
  a.epsilon = kEps;
  a.elements = s.e->cfg.hidden;
  a.residual_out = residual_out;
  a.act_codes = s.act_codes + act_offset;
  a.act_scales = s.act_scales + act_offset / 128;
  a.act_sums = s.act_sums + act_offset / 128;
  a.embedding_codes = s.e->emb_codes;
  a.embedding_scales = reinterpret_cast<const __half*>(s.e->emb_scales);
  a.embedding_rows = s.e->cfg.vocab;
  a.embedding_bits = static_cast<int>(s.e->cfg.emb_bits);
  a.device_tokens = device_tokens;
  return launch_norm_pack(a, static_cast<int>(s.e->cfg.activation_bits), batch, s.stream);
}

int mlp_block(gfxb_session& s, const Layer& L, unsigned batch) {
  GFXB_TRY(gemv(s, {{&L.gate, s.gate}, {&L.up, s.up}}, batch));
  SiluPackArgs a;
  a.gate = s.gate;
  a.up = s.up;
  a.elements = s.e->shard.inter;
  a.batch = batch;
  a.act_codes = s.act_codes;
  a.act_scales = s.act_scales;
  a.act_sums = s.act_sums;
  GFXB_TRY(launch_silu_pack(a, static_cast<int>(s.e->cfg.activation_bits), s.stream));
  GFXB_TRY(gemv(s, {{&L.down, s.update}}, batch));
  return all_reduce(s, s.update, static_cast<std::size_t>(batch) * s.e->cfg.hidden);
}

// Fused Q/K norm + RoPE + KV append, then chunked gated attention with the
// o_proj input pack fused in its epilogue (the attention mixer between its
// q/k/v and o projections).
int attention_core(gfxb_session& s, const Layer& L, __half* key_cache, __half* value_cache,
                   const std::uint64_t* device_position, unsigned batch) {
  const Shard& sh = s.e->shard;
  QkRopeArgs r;
  r.q_input = s.proj_main;
  r.q_weight = L.q_norm;
  r.q_output = s.query;
  r.k_input = s.proj_k;
  r.k_weight = L.k_norm;
  r.v_input = s.proj_v;
  r.key_cache = key_cache;
  r.value_cache = value_cache;
  r.capacity = s.cfg.maximum_context_tokens;
  r.q_heads = sh.nq;
  r.k_heads = sh.nkv;
  r.q_stride = 512;
  r.k_stride = 256;
  r.rotary = 64;
  r.cos_table = s.rope_cos;
  r.sin_table = s.rope_sin;
  r.table_positions = s.cfg.maximum_context_tokens;
  r.device_base_position = device_position;
  AttentionArgs a;
  a.query = s.query;
  a.gate = s.proj_main;
  a.key_cache = key_cache;
  a.value_cache = value_cache;
  a.output = s.attn_out;
  a.partials = s.attention_partials;
  a.max_chunks = s.attention_chunks;
  a.capacity = s.cfg.maximum_context_tokens;
  a.device_base_position = device_position;
  a.q_heads = sh.nq;
  a.kv_heads = sh.nkv;
  a.act_bits = static_cast<int>(s.e->cfg.activation_bits);
  a.act_codes = s.act_codes;
  a.act_scales = s.act_scales;
  a.act_sums = s.act_sums;
  if (batch == 1 && attention_decode_enabled()) {
    AttentionDecodeArgs d;
    d.rope = r;
    d.attention = a;
    d.tickets = s.attention_tickets;
    return launch_attention_decode(d, s.stream);
  }
  GFXB_TRY(launch_qk_rope(r, batch, s.stream));
  return launch_attention(a, batch, s.stream);
}

// Attention mixer: q/k/v GEMV, the attention core, o_proj.
int attention_mixer(gfxb_session& s, const Layer& L, __half* key_cache, __half* value_cache,
                    const std::uint64_t* device_position, unsigned batch) {
  GFXB_TRY(gemv(s, {{&L.q, s.proj_main}, {&L.k, s.proj_k}, {&L.v, s.proj_v}}, batch));
  GFXB_TRY(attention_core(s, L, key_cache, value_cache, device_position, batch));
  GFXB_TRY(gemv(s, {{&L.out, s.update}}, batch));
  return all_reduce(s, s.update, static_cast<std::size_t>(batch) * s.e->cfg.hidden);
}

// The GDN step between the in- and out-projections: conv and recurrence
// (+ out_proj pack). With `record` the final states go to the snapshot
// buffers and the per-token logs are written for a later rollback replay.
int gdn_recurrent_step(gfxb_session& s, const Layer& L, unsigned batch, bool record) {
  const Shard& sh = s.e->shard;
  const gfxb_model_config& c = s.e->cfg;
  const std::size_t conv_elems = static_cast<std::size_t>(sh.channels) * 4;
  const std::size_t state_elems = static_cast<std::size_t>(sh.nv) * 128 * 128;
  __half* conv_state = s.conv_states + L.state_index * conv_elems;
  float* state = s.gdn_states + L.state_index * state_elems;
  GdnConvArgs cv;
  cv.projected = s.proj_main;
  cv.weight = L.conv;
  cv.initial_state = conv_state;
  cv.final_state = record ? s.conv_snapshot + L.state_index * conv_elems : conv_state;
  cv.output = s.conv_out;
  cv.appended_log = record ? s.conv_log + static_cast<std::size_t>(L.state_index) * kMaxBlock * sh.channels : nullptr;
  cv.channels = sh.channels;
  cv.batch = batch;
  GdnRecurrentArgs g;
  // the conv runs inside the recurrent kernel when a key head's value heads fit one cluster
  if (sh.nv / sh.nk <= 8) {
    g.conv = cv;
  } else {
    GFXB_TRY(launch_gdn_conv(cv, s.stream));
    g.qkv = s.conv_out;
  }
  g.z = s.proj_z;
  g.a = s.proj_a + sh.vh0;
  g.b = s.proj_b + sh.vh0;
  g.ab_stride = c.gdn_value_heads;
  g.a_log = L.a_log;
  g.dt_bias = L.dt_bias;
  g.norm_weight = L.gdn_norm;
  g.initial_state = state;
  g.final_state = record ? s.gdn_snapshot + L.state_index * state_elems : state;
  g.output = s.gdn_out;
  if (record) {
    g.key_log = s.key_log + static_cast<std::size_t>(L.state_index) * kMaxBlock * sh.nk * 128;
    g.delta_log = s.delta_log + static_cast<std::size_t>(L.state_index) * kMaxBlock * sh.nv * 128;
    g.decay_log = s.decay_log + static_cast<std::size_t>(L.state_index) * kMaxBlock * sh.nv;
  }
  g.key_heads = sh.nk;
  g.value_heads = sh.nv;
  g.batch = batch;
  g.act_bits = static_cast<int>(c.activation_bits);
  g.act_codes = s.act_codes;
  g.act_scales = s.act_scales;
  g.act_sums = s.act_sums;
  return launch_gdn_recurrent(g, s.stream);
}

// Gated-DeltaNet mixer: fused qkv/z/a/b GEMV, the GDN step, out_proj.
int gdn_mixer(gfxb_session& s, const Layer& L, unsigned batch, bool record) {
  GFXB_TRY(gemv(s, {{&L.qkv, s.proj_main}, {&L.z, s.proj_z}, {&L.a, s.proj_a}, {&L.b, s.proj_b}}, batch));
  GFXB_TRY(gdn_recurrent_step(s, L, batch, record));
  GFXB_TRY(gemv(s, {{&L.out, s.update}}, batch));
  return all_reduce(s, s.update, static_cast<std::size_t>(batch) * s.e->cfg.hidden);
}

__global__ void advance_kernel(std::uint64_t* position, std::uint32_t* tokens, const std::uint32_t* selected,
                               unsigned batch) {
  *position += batch;
  tokens[0] = selected[batch - 1];
}

// TP argmax: each rank contributes (value bits, global index) per token; the
// winner is the largest value, lowest global index on ties.
__global__ void select_across_ranks_kernel(const std::uint32_t* gathered, unsigned ranks, unsigned batch,
                                           std::uint32_t* tokens) {
  const unsigned t = threadIdx.x;
  if (t >= batch) return;
  float best = -__int_as_float(0x7f800000);
  std::uint32_t index = 0xffffffffu;
  for (unsigned r = 0; r < ranks; ++r) {
    const float value = __uint_as_float(gathered[(r * kMaxBlock + t) * 2]);
    const std::uint32_t other = gathered[(r * kMaxBlock + t) * 2 + 1];
    if (value > best || (value == best && other < index)) {
      best = value;
      index = other;
    }
  }
  tokens[t] = index;
}

__global__ void exchange_kernel(const float* values, const std::uint32_t* indices, const std::uint32_t* local_tokens,
                                std::uint32_t offset, unsigned batch, unsigned blocks, std::uint32_t* exchange) {
  // local winner per token: recompute its value from the partials (first block carrying the index)
  const unsigned t = threadIdx.x;
  if (t >= batch) return;
  const std::uint32_t local = local_tokens[t];
  float value = -__int_as_float(0x7f800000);
  for (unsigned b = 0; b < blocks; ++b) {
    if (indices[t * blocks + b] == local) {
      value = values[t * blocks + b];
      break;
    }
  }
  exchange[t * 2] = __float_as_uint(value);
  exchange[t * 2 + 1] = local + offset;
}

int head_argmax(gfxb_session& s, const QMatrix& head_rows, std::uint32_t rows, std::uint32_t* out_tokens,
                unsigned batch, std::size_t act_offset = 0) {
  const Shard& sh = s.e->shard;
  QMatrix head = head_rows;
  if (rows == 0) {
    // this rank holds none of the requested vocabulary rows
    if (sh.tp == 1) return fail(GFXB_INTERNAL, "empty vocabulary range");
    // NaN value bits never win the comparison in select_across_ranks_kernel
    GFXB_TRY(cuda_check(cudaMemsetAsync(s.exchange, 0xff, kMaxBlock * 2 * sizeof(std::uint32_t), s.stream), "memset"));
  } else {
    head.rows = rows;
    GFXB_TRY(gemv(s, {{&head, s.logits}}, batch, act_offset));
    ArgmaxArgs a;
    a.logits = s.logits;
    a.row_stride = rows;
    a.vocab = rows;
    a.tokens = sh.tp == 1 ? out_tokens : s.exchange + kMaxBlock * 2;  // local winners scratch
    a.partial_values = s.argmax_values;
    a.partial_indices = s.argmax_indices;
    GFXB_TRY(launch_argmax(a, batch, s.stream));
    if (sh.tp == 1) return GFXB_OK;
    exchange_kernel<<<1, kMaxBlock, 0, s.stream>>>(s.argmax_values, s.argmax_indices, s.exchange + kMaxBlock * 2,
                                                   sh.v0, batch, 64, s.exchange);
    GFXB_TRY(launch_status("argmax exchange failed"));
  }
  GFXB_TRY(nccl_check(nccl().all_gather(s.exchange, s.gathered, kMaxBlock * 2, ncclUint32, s.e->comm, s.stream),
                      "NCCL all-gather failed"));
  select_across_ranks_kernel<<<1, kMaxBlock, 0, s.stream>>>(s.gathered, sh.tp, batch, out_tokens);
  return launch_status("argmax selection failed");
}

// Which tokens of a block get the LM head and argmax: all of them (greedy and
// block steps, the verifier), the last one only (the final block of a
// prefill) or none (the other prefill blocks).
enum class Head { all, last, none };

// The causal block forward (qwen_runtime.cpp:349-544, 1264-1392): tokens and
// base position are read from device memory, so the same launch sequence
// serves the eager path and captured graphs.
int enqueue_forward(gfxb_session& s, unsigned batch, const std::uint32_t* device_tokens,
                    const std::uint64_t* device_position, bool record, Head head = Head::all) {
  gfxb_engine& e = *s.e;
  const gfxb_model_config& c = e.cfg;
  __half* current = s.hidden[0];
  __half* next = s.hidden[1];
  GFXB_TRY(embed_norm_pack(s, device_tokens, current, e.layers[0].input_norm, batch));
  const std::size_t kv_stride = static_cast<std::size_t>(s.cfg.maximum_context_tokens) * e.shard.nkv * 256;
  for (std::uint32_t i = 0; i < c.layers; ++i) {
    const Layer& L = e.layers[i];
    if (L.attention) {
      GFXB_TRY(attention_mixer(s, L, s.key_cache + L.state_index * kv_stride, s.value_cache + L.state_index * kv_stride,
                               device_position, batch));
    } else {
      GFXB_TRY(gdn_mixer(s, L, batch, record));
    }
    GFXB_TRY(norm_pack(s, current, s.update, s.post_attention, L.post_norm, batch));
    GFXB_TRY(mlp_block(s, L, batch));
    const std::uint16_t* next_norm = i + 1 < c.layers ? e.layers[i + 1].input_norm : e.final_norm;
    GFXB_TRY(norm_pack(s, s.post_attention, s.update, next, next_norm, batch));
    std::swap(current, next);
  }
  s.last_hidden = current + static_cast<std::size_t>(batch - 1) * c.hidden;
  if (head == Head::none) return GFXB_OK;
  if (head == Head::last) {
    return head_argmax(s, e.lm_head, e.shard.vocab, s.selected, 1, static_cast<std::size_t>(batch - 1) * c.hidden);
  }
  return head_argmax(s, e.lm_head, e.shard.vocab, s.selected, batch);
}

// MTP proposal (qwen_runtime.cpp:715-867) for one token: embedding of
// *device_token and the conditioning hidden state -> dual RMSNorm -> fc ->
// one attention layer + MLP on the MTP KV cache -> draft head (first
// draft_vocab LM-head rows) -> argmax into *output_token (or nothing when
// output_token is null: cache advance only).
int enqueue_mtp(gfxb_session& s, const std::uint32_t* device_token, const __half* conditioning,
                const std::uint64_t* device_position, std::uint32_t* output_token) {
  gfxb_engine& e = *s.e;
  const gfxb_model_config& c = e.cfg;
  const Shard& sh = e.shard;
  const std::uint32_t H = c.hidden;
  GFXB_TRY(embed_norm_pack(s, device_token, s.mtp_embed, e.pre_emb_norm, 1, 0));
  GFXB_TRY(norm_pack(s, conditioning, nullptr, nullptr, e.pre_hidden_norm, 1, nullptr, H));
  if (sh.tp == 1) {
    GFXB_TRY(gemv(s, {{&e.fc, s.mtp_input}}, 1, 0, 2 * H, true));
  } else {
    GFXB_TRY(gemv(s, {{&e.fc, s.update}}, 1, sh.fc0, 2 * H));
    GFXB_TRY(all_reduce(s, s.update, H));
    GFXB_TRY(launch_float_to_half(s.update, s.mtp_input, H, s.stream));
  }
  GFXB_TRY(norm_pack(s, s.mtp_input, nullptr, nullptr, e.mtp.input_norm, 1));
  if (output_token == nullptr) {
    // advance the MTP KV cache only (qwen_runtime.cpp:826-829)
    GFXB_TRY(gemv(s, {{&e.mtp.q, s.proj_main}, {&e.mtp.k, s.proj_k}, {&e.mtp.v, s.proj_v}}, 1));
    QkRopeArgs r;
    r.q_input = s.proj_main;
    r.q_weight = e.mtp.q_norm;
    r.q_output = s.query;
    r.k_input = s.proj_k;
    r.k_weight = e.mtp.k_norm;
    r.v_input = s.proj_v;
    r.key_cache = s.mtp_keys;
    r.value_cache = s.mtp_values;
    r.capacity = s.cfg.maximum_context_tokens;
    r.q_heads = sh.nq;
    r.k_heads = sh.nkv;
    r.cos_table = s.rope_cos;
    r.sin_table = s.rope_sin;
    r.table_positions = s.cfg.maximum_context_tokens;
    r.device_base_position = device_position;
    return launch_qk_rope(r, 1, s.stream);
  }
  GFXB_TRY(attention_mixer(s, e.mtp, s.mtp_keys, s.mtp_values, device_position, 1));
  GFXB_TRY(norm_pack(s, s.mtp_input, s.update, s.post_attention, e.mtp.post_norm, 1));
  GFXB_TRY(mlp_block(s, e.mtp, 1));
  GFXB_TRY(norm_pack(s, s.post_attention, s.update, s.mtp_hidden, e.mtp_final_norm, 1));
  const std::uint32_t draft = std::min(c.draft_vocab, c.vocab);
  const std::uint32_t local_rows = sh.v0 >= draft ? 0 : std::min(sh.vocab, draft - sh.v0);
  return head_argmax(s, e.lm_head, local_rows, output_token, 1);
}

__global__ void set_positions_kernel(std::uint64_t* position, std::uint64_t value, std::uint64_t* mtp_positions,
                                     std::uint64_t mtp_base, unsigned count, std::uint32_t* seed_slot,
                                     std::uint32_t seed, std::uint32_t* tokens) {
  *position = value;
  for (unsigned i = 0; i < count; ++i) mtp_positions[i] = mtp_base + i;
  *seed_slot = seed;
  tokens[0] = seed;
}

__global__ void copy_drafts_kernel(const std::uint32_t* drafts, std::uint32_t* tokens, unsigned count) {
  const unsigned i = threadIdx.x;
  if (i < count) tokens[i + 1] = drafts[i];
}

// The batch-1 greedy step as one token-kernel operation list. Operation i
// reads only outputs of operations before it (the kernel puts a grid barrier
// in front of each); buffers follow enqueue_forward so both paths leave the
// same state behind (hidden[0/1], post_attention, update, caches, logits).
int build_token_loop(gfxb_session& s) {
  gfxb_engine& e = *s.e;
  const gfxb_model_config& c = e.cfg;
  const Shard& sh = e.shard;
  if (sh.tp != 1) return fail(GFXB_UNSUPPORTED, "token kernel: tensor-parallel sessions use per-operation launches");
  if (!token_loop_supported_hidden(c.hidden)) return fail(GFXB_UNSUPPORTED, "token kernel: unsupported hidden size");
  if (sh.nkv > kLoopMaxKvHeads) return fail(GFXB_UNSUPPORTED, "token kernel: too many KV heads");
  std::uint32_t ctas = 0;
  GFXB_TRY(token_loop_grid(e.device, &ctas));
  const std::size_t ctx = s.cfg.maximum_context_tokens;
  std::vector<LoopOp> ops;
  std::uint32_t rotation = 0, max_groups = 0, dots_half = 0;
  auto matrix = [](const QMatrix& q, void* output, std::uint32_t epilogue) {
    LoopMatrix m{};
    m.codes = q.codes;
    m.scales = reinterpret_cast<const __half*>(q.scales);
    m.output = output;
    m.tiles = q.rows / 16u;
    m.epilogue = epilogue;
    return m;
  };
  auto add_op = [&](LoopOp& op, std::uint32_t units) {
    op.rotation = rotation;
    rotation = (rotation + units) % ctas;
    ops.push_back(op);
  };
  auto add_gemv = [&](LoopGemv g, const std::vector<LoopMatrix>& mats, std::uint32_t columns, std::uint32_t bits) {
    g.bits = bits;
    g.groups = columns / 128u;
    g.count = static_cast<std::uint32_t>(mats.size());
    g.units = 0;
    for (std::size_t i = 0; i < mats.size(); ++i) {
      g.m[i] = mats[i];
      g.units += mats[i].tiles;
    }
    if (g.paired) g.units = mats[0].tiles;
    max_groups = std::max(max_groups, g.groups);
    dots_half = std::max(dots_half, (g.paired ? 2u : 1u) * g.groups * 16u);
    LoopOp op{};
    op.kind = kLoopGemv;
    op.gemv = g;
    add_op(op, g.units);
  };
  auto residual_norm = [&](const __half* residual, __half* residual_out, const std::uint16_t* weight) {
    LoopGemv g{};
    g.act_source = kActResidualNorm;
    g.residual = residual;
    g.update = s.update;
    g.residual_out = residual_out;
    g.norm_weight = weight;
    return g;
  };
  auto global_pack = [&]() {
    LoopGemv g{};
    g.act_source = kActGlobalPack;
    g.pack_codes = s.act_codes;
    g.pack_scales = s.act_scales;
    g.pack_sums = s.act_sums;
    return g;
  };
  const std::size_t kv_stride = ctx * sh.nkv * 256;
  const std::size_t conv_elems = static_cast<std::size_t>(sh.channels) * 4;
  const std::size_t state_elems = static_cast<std::size_t>(sh.nv) * 128 * 128;
  const int act_bits = static_cast<int>(c.activation_bits);
  for (std::uint32_t i = 0; i < c.layers; ++i) {
    const Layer& L = e.layers[i];
    __half* current = s.hidden[i % 2];
    // input RMSNorm + mixer projections
    LoopGemv in{};
    if (i == 0) {
      in.act_source = kActEmbedNorm;
      in.embedding_codes = e.emb_codes;
      in.embedding_scales = reinterpret_cast<const __half*>(e.emb_scales);
      in.embedding_rows = c.vocab;
      in.embedding_bits = c.emb_bits;
      in.tokens = s.tokens;
      in.residual_out = current;
      in.norm_weight = L.input_norm;
    } else {
      in = residual_norm(s.post_attention, current, L.input_norm);
    }
    if (L.attention) {
      add_gemv(in, {matrix(L.q, s.proj_main, kEpiF32), matrix(L.k, s.proj_k, kEpiF32), matrix(L.v, s.proj_v, kEpiF32)},
               c.hidden, static_cast<std::uint32_t>(bits_of_format(L.q.format)));
      LoopOp op{};
      op.kind = kLoopAttention;
      QkRopeArgs& r = op.rope;
      r.q_input = s.proj_main;
      r.q_weight = L.q_norm;
      r.k_input = s.proj_k;
      r.k_weight = L.k_norm;
      r.v_input = s.proj_v;
      r.key_cache = s.key_cache + L.state_index * kv_stride;
      r.value_cache = s.value_cache + L.state_index * kv_stride;
      r.capacity = ctx;
      r.q_heads = sh.nq;
      r.k_heads = sh.nkv;
      r.q_stride = 512;
      r.k_stride = 256;
      r.rotary = 64;
      r.cos_table = s.rope_cos;
      r.sin_table = s.rope_sin;
      r.table_positions = ctx;
      r.device_base_position = s.position;
      AttentionArgs& a = op.attention;
      a.gate = s.proj_main;
      a.key_cache = r.key_cache;
      a.value_cache = r.value_cache;
      a.output = s.attn_out;
      a.partials = s.attention_partials;
      a.max_chunks = s.attention_chunks;
      a.capacity = ctx;
      a.device_base_position = s.position;
      a.q_heads = sh.nq;
      a.kv_heads = sh.nkv;
      a.act_bits = act_bits;
      a.act_codes = s.act_codes;
      a.act_scales = s.act_scales;
      a.act_sums = s.act_sums;
      add_op(op, sh.nkv * s.attention_chunks);
      add_gemv(global_pack(), {matrix(L.out, s.update, kEpiF32)}, sh.nq * 256,
               static_cast<std::uint32_t>(bits_of_format(L.out.format)));
    } else {
      LoopMatrix qkv = matrix(L.qkv, s.conv_out, kEpiConv);
      qkv.conv_state = s.conv_states + L.state_index * conv_elems;
      qkv.conv_weight = L.conv;
      add_gemv(in, {qkv, matrix(L.z, s.proj_z, kEpiF32), matrix(L.a, s.proj_a, kEpiF32), matrix(L.b, s.proj_b, kEpiF32)},
               c.hidden, static_cast<std::uint32_t>(bits_of_format(L.qkv.format)));
      LoopOp op{};
      op.kind = kLoopGdn;
      GdnRecurrentArgs& g = op.gdn;
      g.qkv = s.conv_out;
      g.z = s.proj_z;
      g.a = s.proj_a;
      g.b = s.proj_b;
      g.ab_stride = c.gdn_value_heads;
      g.a_log = L.a_log;
      g.dt_bias = L.dt_bias;
      g.norm_weight = L.gdn_norm;
      g.initial_state = s.gdn_states + L.state_index * state_elems;
      g.final_state = s.gdn_states + L.state_index * state_elems;
      g.output = s.gdn_out;
      g.key_heads = sh.nk;
      g.value_heads = sh.nv;
      g.batch = 1;
      g.act_bits = act_bits;
      g.act_codes = s.act_codes;
      g.act_scales = s.act_scales;
      g.act_sums = s.act_sums;
      add_op(op, sh.nv);
      add_gemv(global_pack(), {matrix(L.out, s.update, kEpiF32)}, sh.nv * 128,
               static_cast<std::uint32_t>(bits_of_format(L.out.format)));
    }
    // post-mixer RMSNorm + SwiGLU gate/up (fused SiLU product), then down
    LoopGemv gate_up = residual_norm(current, s.post_attention, L.post_norm);
    gate_up.paired = 1;
    add_gemv(gate_up, {matrix(L.gate, s.mlp_product, kEpiSiluPair), matrix(L.up, nullptr, kEpiSiluPair)}, c.hidden,
             static_cast<std::uint32_t>(bits_of_format(L.gate.format)));
    LoopGemv down{};
    down.act_source = kActPackF16;
    down.f16_input = s.mlp_product;
    add_gemv(down, {matrix(L.down, s.update, kEpiF32)}, sh.inter, static_cast<std::uint32_t>(bits_of_format(L.down.format)));
  }
  // final RMSNorm + LM head + argmax
  add_gemv(residual_norm(s.post_attention, s.hidden[c.layers % 2], e.final_norm), {matrix(e.lm_head, s.logits, kEpiLogits)},
           c.hidden, static_cast<std::uint32_t>(bits_of_format(e.lm_head.format)));
  LoopOp argmax{};
  argmax.kind = kLoopArgmax;
  add_op(argmax, 0);
  if (ops.size() > 5ull * c.layers + 4) return fail(GFXB_INTERNAL, "token kernel operation list overflow");

  LoopLaunch& launch = s.loop;
  launch = LoopLaunch{};
  launch.ops = s.loop_ops;
  launch.op_count = static_cast<std::uint32_t>(ops.size());
  launch.control = s.loop_control;
  launch.hidden = c.hidden;
  launch.vocab = sh.vocab;
  launch.selected = s.selected;
  launch.tokens = s.tokens;
  launch.position = s.position;
  launch.act_bits = c.activation_bits;
  GFXB_TRY(plan_token_loop(launch, max_groups, dots_half, e.device));
  if (launch.ctas != ctas) return fail(GFXB_INTERNAL, "token kernel grid changed");
  GFXB_TRY(cuda_check(cudaMemcpyAsync(s.loop_ops, ops.data(), ops.size() * sizeof(LoopOp), cudaMemcpyHostToDevice,
                                      s.stream),
                      "token kernel operation upload failed"));
  GFXB_TRY(cuda_check(cudaMemsetAsync(s.loop_control, 0, sizeof(LoopControl), s.stream), "token kernel control reset failed"));
  GFXB_TRY(cuda_check(cudaStreamSynchronize(s.stream), "token kernel setup failed"));
  s.loop_ready = true;
  return GFXB_OK;
}

// Error bits the token kernel left in the control block (0: none).
int check_token_loop(gfxb_session& s) {
  if (!s.loop_ready) return GFXB_OK;
  std::uint32_t error = 0;
  GFXB_TRY(cuda_check(cudaMemcpy(&error, &s.loop_control->error, sizeof error, cudaMemcpyDeviceToHost),
                      "token kernel status read failed"));
  if (error == 0) return GFXB_OK;
  // clear the abort state so later steps run (their results follow the failed step's state)
  GFXB_TRY(cuda_check(cudaMemset(s.loop_control, 0, sizeof(LoopControl)), "token kernel control reset failed"));
  std::string message = "token kernel failed:";
  if (error & kLoopErrorBarrier) message += " grid barrier wait expired;";
  if (error & kLoopErrorRing) message += " weight ring wait expired;";
  if (error & kLoopErrorContext) message += " position outside the KV cache or RoPE table;";
  return fail((error & kLoopErrorContext) && !(error & (kLoopErrorBarrier | kLoopErrorRing)) ? GFXB_INVALID_ARGUMENT
                                                                                             : GFXB_INTERNAL,
              message.c_str());
}

int enqueue_greedy_step(gfxb_session& s) {
  if (s.loop_ready) return launch_token_loop(s.loop, s.stream);
  GFXB_TRY(enqueue_forward(s, 1, s.tokens, s.position, false));
  advance_kernel<<<1, 1, 0, s.stream>>>(s.position, s.tokens, s.selected, 1);
  return launch_status("advance launch failed");
}

// The device part of a speculative round (qwen_runtime.cpp:546-640, 715-867):
// `drafts` MTP proposals chained through device token ids, the drafts copied
// behind the seed, the causal verifier block with rollback logs, and the
// drafts and verifier tokens copied to pinned host memory. Reads only device
// scalars (positions, seed) set before it runs, so it can be captured once
// and replayed every round (prepare_speculative_graphs, :642-713).
int enqueue_speculative_body(gfxb_session& s, unsigned drafts, bool external = false) {
  for (unsigned i = 0; i < drafts; ++i) {
    const std::uint32_t* token = i == 0 ? s.seed_token : s.draft_tokens + i - 1;
    const __half* conditioning = i == 0 ? s.target_snapshot : s.mtp_hidden;
    GFXB_TRY(enqueue_mtp(s, token, conditioning, s.mtp_positions + i, s.draft_tokens + i));
  }
  if (external) {
    // the caller's drafts replace the MTP proposals; the MTP cache keeps the chain's entries
    GFXB_TRY(cuda_check(cudaMemcpyAsync(s.draft_tokens, s.external_drafts, drafts * sizeof(std::uint32_t),
                                        cudaMemcpyDeviceToDevice, s.stream),
                        "external draft copy failed"));
  }
  copy_drafts_kernel<<<1, kMaxBlock, 0, s.stream>>>(s.draft_tokens, s.tokens, drafts);
  GFXB_TRY(launch_status("draft copy failed"));
  GFXB_TRY(enqueue_forward(s, drafts + 1, s.tokens, s.position, true));
  GFXB_TRY(cuda_check(cudaMemcpyAsync(s.pinned + 128, s.draft_tokens, drafts * 4, cudaMemcpyDeviceToHost, s.stream),
                      "draft download failed"));
  return cuda_check(cudaMemcpyAsync(s.pinned + 160, s.selected, (drafts + 1) * 4, cudaMemcpyDeviceToHost, s.stream),
                    "verifier download failed");
}

int capture_speculative(gfxb_session& s, unsigned drafts) {
  cudaGraph_t graph = nullptr;
  GFXB_TRY(cuda_check(cudaStreamBeginCapture(s.stream, cudaStreamCaptureModeThreadLocal), "graph capture start failed"));
  const int status = enqueue_speculative_body(s, drafts);
  const cudaError_t end = cudaStreamEndCapture(s.stream, &graph);
  if (status != GFXB_OK) {
    if (graph) cudaGraphDestroy(graph);
    return status;
  }
  GFXB_TRY(cuda_check(end, "graph capture end failed"));
  const cudaError_t inst = cudaGraphInstantiate(&s.spec_graph, graph, 0);
  cudaGraphDestroy(graph);
  GFXB_TRY(cuda_check(inst, "graph instantiation failed"));
  s.spec_drafts = drafts;
  return GFXB_OK;
}

int capture_greedy(gfxb_session& s) {
  cudaGraph_t graph = nullptr;
  GFXB_TRY(cuda_check(cudaStreamBeginCapture(s.stream, cudaStreamCaptureModeThreadLocal), "graph capture start failed"));
  const int status = enqueue_greedy_step(s);
  const cudaError_t end = cudaStreamEndCapture(s.stream, &graph);
  if (status != GFXB_OK) {
    if (graph) cudaGraphDestroy(graph);
    return status;
  }
  GFXB_TRY(cuda_check(end, "graph capture end failed"));
  const cudaError_t inst = cudaGraphInstantiate(&s.greedy_graph, graph, 0);
  cudaGraphDestroy(graph);
  return cuda_check(inst, "graph instantiation failed");
}

int allocate_session(gfxb_session& s, bool place) {
  gfxb_engine& e = *s.e;
  const gfxb_model_config& c = e.cfg;
  const Shard& sh = e.shard;
  Planner plan;
  plan.base = place ? s.arena : nullptr;
  const std::size_t B = kMaxBlock, H = c.hidden, ctx = s.cfg.maximum_context_tokens;
  const std::size_t proj_main = std::max<std::size_t>(sh.channels, static_cast<std::size_t>(sh.nq) * 512);
  s.act_width = static_cast<std::uint32_t>(std::max<std::size_t>({2 * H, sh.inter, sh.nv * 128ull, sh.nq * 256ull}));
  s.hidden[0] = plan.take<__half>(B * H);
  s.hidden[1] = plan.take<__half>(B * H);
  s.post_attention = plan.take<__half>(B * H);
  s.act_codes = plan.take<std::int8_t>(B * s.act_width);
  s.act_scales = plan.take<__half>(B * s.act_width / 128);
  s.act_sums = plan.take<std::int32_t>(B * s.act_width / 128);
  s.proj_main = plan.take<float>(B * proj_main);
  s.proj_z = plan.take<float>(B * sh.nv * 128);
  s.proj_a = plan.take<float>(B * c.gdn_value_heads);
  s.proj_b = plan.take<float>(B * c.gdn_value_heads);
  s.proj_k = plan.take<float>(B * sh.nkv * 256);
  s.proj_v = plan.take<float>(B * sh.nkv * 256);
  s.update = plan.take<float>(B * H);
  s.gate = plan.take<float>(B * sh.inter);
  s.up = plan.take<float>(B * sh.inter);
  s.logits = plan.take<float>(B * sh.vocab);
  s.conv_out = plan.take<__half>(B * sh.channels);
  s.gdn_out = plan.take<__half>(B * sh.nv * 128);
  s.query = plan.take<__half>(B * sh.nq * 256);
  s.attn_out = plan.take<__half>(B * sh.nq * 256);
  s.attention_chunks = static_cast<std::uint32_t>((ctx + kAttentionChunk - 1) / kAttentionChunk);
  s.attention_partials = plan.take<float>(attention_partial_bytes(sh.nq, ctx, kMaxBlock) / sizeof(float));
  s.attention_tickets = plan.take<std::uint32_t>(sh.nq);
  s.argmax_values = plan.take<float>(argmax_scratch_bytes(kMaxBlock) / 8);
  s.argmax_indices = plan.take<std::uint32_t>(argmax_scratch_bytes(kMaxBlock) / 8);
  s.gathered = plan.take<std::uint32_t>(static_cast<std::size_t>(sh.tp) * B * 2);
  s.exchange = plan.take<std::uint32_t>(B * 4);
  s.selected = plan.take<std::uint32_t>(B);
  s.tokens = plan.take<std::uint32_t>(B);
  s.position = plan.take<std::uint64_t>(1);
  s.mtp_hidden = plan.take<__half>(H);
  s.mtp_input = plan.take<__half>(H);
  s.mtp_embed = plan.take<__half>(H);
  s.target_snapshot = plan.take<__half>(H);
  s.draft_tokens = plan.take<std::uint32_t>(B);
  s.external_drafts = plan.take<std::uint32_t>(B);
  s.mtp_positions = plan.take<std::uint64_t>(B);
  s.seed_token = plan.take<std::uint32_t>(1);
  const std::size_t conv_elems = static_cast<std::size_t>(e.gdn_layers) * sh.channels * 4;
  const std::size_t state_elems = static_cast<std::size_t>(e.gdn_layers) * sh.nv * 128 * 128;
  s.conv_states = plan.take<__half>(conv_elems);
  s.conv_snapshot = plan.take<__half>(conv_elems);
  s.gdn_states = plan.take<float>(state_elems);
  s.gdn_snapshot = plan.take<float>(state_elems);
  s.conv_log = plan.take<__half>(static_cast<std::size_t>(e.gdn_layers) * B * sh.channels);
  s.key_log = plan.take<float>(static_cast<std::size_t>(e.gdn_layers) * B * sh.nk * 128);
  s.delta_log = plan.take<float>(static_cast<std::size_t>(e.gdn_layers) * B * sh.nv * 128);
  s.decay_log = plan.take<float>(static_cast<std::size_t>(e.gdn_layers) * B * sh.nv);
  const std::size_t kv = static_cast<std::size_t>(e.attention_layers) * ctx * sh.nkv * 256;
  s.key_cache = plan.take<__half>(kv);
  s.value_cache = plan.take<__half>(kv);
  s.mtp_keys = plan.take<__half>(ctx * sh.nkv * 256);
  s.mtp_values = plan.take<__half>(ctx * sh.nkv * 256);
  s.rope_cos = plan.take<float>(ctx * 32);
  s.rope_sin = plan.take<float>(ctx * 32);
  s.mlp_product = plan.take<__half>(B * sh.inter);
  s.loop_control = plan.take<LoopControl>(1);
  s.loop_ops = plan.take<LoopOp>(5ull * c.layers + 4);
  s.arena_bytes = plan.offset;
  return GFXB_OK;
}

}  // namespace
}  // namespace gfxb

// ===========================================================================
// C ABI
// ===========================================================================

using namespace gfxb;

extern "C" int gfxb_nccl_unique_id(void* id128) {
  if (id128 == nullptr) return fail(GFXB_INVALID_ARGUMENT, "NCCL id buffer is null");
  GFXB_TRY(load_nccl(nccl()));
  ncclUniqueId id;
  GFXB_TRY(nccl_check(nccl().get_unique_id(&id), "ncclGetUniqueId failed"));
  std::memcpy(id128, &id, sizeof id);
  return GFXB_OK;
}

extern "C" int gfxb_tp_shard(const gfxb_model_config* config, int tp_rank, int tp_size, gfxb_tp_shard_info* out) {
  if (config == nullptr || out == nullptr) return fail(GFXB_INVALID_ARGUMENT, "null argument");
  if (tp_size < 1 || tp_size > 8 || tp_rank < 0 || tp_rank >= tp_size) {
    return fail(GFXB_INVALID_ARGUMENT, "tensor-parallel rank/size are invalid");
  }
  GFXB_TRY(validate_config(*config, static_cast<std::uint32_t>(tp_size)));
  const Shard s = make_shard(*config, static_cast<std::uint32_t>(tp_size), static_cast<std::uint32_t>(tp_rank));
  *out = gfxb_tp_shard_info{s.nk, s.kh0, s.nv, s.vh0, s.nq, s.qh0, s.nkv, s.kv0, s.inter, s.i0,
                            s.vocab, s.v0, s.fc_cols, s.fc0, s.channels};
  return GFXB_OK;
}

namespace gfxb {
namespace {

int create_engine(const gfxb_model_config& config, int device, int tp_rank, int tp_size, const void* nccl_id128,
                  bool include_mtp, WeightSource& src, gfxb_engine** out) {
  *out = nullptr;
  if (tp_size < 1 || tp_size > 8 || tp_rank < 0 || tp_rank >= tp_size) {
    return fail(GFXB_INVALID_ARGUMENT, "tensor-parallel rank/size are invalid");
  }
  if (tp_size > 1 && nccl_id128 == nullptr) return fail(GFXB_INVALID_ARGUMENT, "TP > 1 requires an NCCL id");
  GFXB_TRY(validate_config(config, static_cast<std::uint32_t>(tp_size)));
  GFXB_TRY(gfxb_require_sm100_device(device, nullptr));
  GFXB_TRY(cuda_check(cudaSetDevice(device), "cudaSetDevice failed"));
  auto e = std::make_unique<gfxb_engine>();
  e->cfg = config;
  e->device = device;
  e->has_mtp = include_mtp;
  e->shard = make_shard(config, static_cast<std::uint32_t>(tp_size), static_cast<std::uint32_t>(tp_rank));
  GFXB_TRY(cuda_check(cudaStreamCreateWithFlags(&e->stream, cudaStreamNonBlocking), "stream creation failed"));
  Planner plan;
  int status = build_weights(*e, plan, false, src);
  if (status != GFXB_OK) {
    cudaStreamDestroy(e->stream);
    return status;
  }
  e->arena_bytes = plan.offset;
  void* arena = nullptr;
  status = cuda_check(cudaMalloc(&arena, e->arena_bytes), "weight arena allocation failed");
  if (status == GFXB_OK && src.scratch_bytes != 0) {
    void* scratch = nullptr;
    status = cuda_check(cudaMalloc(&scratch, src.scratch_bytes), "repack staging allocation failed");
    src.scratch = static_cast<std::uint8_t*>(scratch);
  }
  e->arena = static_cast<std::byte*>(arena);
  if (status == GFXB_OK) {
    Planner place;
    place.base = e->arena;
    status = build_weights(*e, place, true, src);
  }
  if (status == GFXB_OK) status = cuda_check(cudaStreamSynchronize(e->stream), "weight upload failed");
  if (src.scratch != nullptr) {
    cudaStreamSynchronize(e->stream);
    cudaFree(src.scratch);
    src.scratch = nullptr;
  }
  if (status == GFXB_OK && tp_size > 1) {
    status = load_nccl(nccl());
    if (status == GFXB_OK) {
      ncclUniqueId id;
      std::memcpy(&id, nccl_id128, sizeof id);
      status = nccl_check(nccl().comm_init_rank(&e->comm, tp_size, id, tp_rank), "ncclCommInitRank failed");
    }
  }
  if (status != GFXB_OK) {
    cudaFree(e->arena);
    cudaStreamDestroy(e->stream);
    return status;
  }
  *out = e.release();
  return GFXB_OK;
}

// Model shape of an artifact from its tensor shapes (the reference inventory,
// qwen38_spec.cpp:32-102): hidden and vocabulary from the embedding, layer
// count and attention placement from the per-layer names, head counts from
// the projection heights.
int derive_config(const gfxi::View& view, const gfxb_artifact_load_options& options, gfxb_model_config& c) {
  c = gfxb_model_config{};
  const gfxi::Tensor* emb = view.find("model.language_model.embed_tokens.weight");
  const gfxi::Tensor* head = view.find("lm_head.weight");
  if (emb == nullptr || head == nullptr || view.find("model.language_model.norm.weight") == nullptr) {
    return artifact_error("artifact lacks embedding, final norm, or LM head");
  }
  if (emb->rank != 2 || head->rank != 2 || head->dimensions[0] != emb->dimensions[0] ||
      head->dimensions[1] != emb->dimensions[1] || emb->dimensions[0] > 0xffffffffull ||
      emb->dimensions[1] > 0xffffffffull) {
    return artifact_error("embedding and LM head shapes disagree");
  }
  c.vocab = static_cast<std::uint32_t>(emb->dimensions[0]);
  c.hidden = static_cast<std::uint32_t>(emb->dimensions[1]);
  c.emb_bits = static_cast<std::uint32_t>(bits_of_quantization(emb->quantization));
  c.head_bits = static_cast<std::uint32_t>(bits_of_quantization(head->quantization));
  while (view.find(layer_name(c.layers, "input_layernorm.weight")) != nullptr) ++c.layers;
  if (c.layers == 0) return artifact_error("artifact has no decoder layers");
  std::int64_t first_attention = -1, first_gdn = -1;
  for (std::uint32_t i = 0; i < c.layers; ++i) {
    const bool attention = view.find(layer_name(i, "self_attn.q_proj.weight")) != nullptr;
    if (attention && first_attention < 0) first_attention = i;
    if (!attention && first_gdn < 0) first_gdn = i;
  }
  c.attention_interval = first_attention < 0 ? c.layers + 1 : static_cast<std::uint32_t>(first_attention) + 1;
  for (std::uint32_t i = 0; i < c.layers; ++i) {
    const bool attention = view.find(layer_name(i, "self_attn.q_proj.weight")) != nullptr;
    if (attention != ((i + 1) % c.attention_interval == 0)) {
      return fail(GFXB_UNSUPPORTED, "attention layers must repeat with a fixed interval");
    }
  }
  const gfxi::Tensor* gate = view.find(layer_name(0, "mlp.gate_proj.weight"));
  if (gate == nullptr || gate->rank != 2) return artifact_error("artifact lacks layer 0's MLP");
  c.intermediate = static_cast<std::uint32_t>(gate->dimensions[0]);
  c.mlp_bits = static_cast<std::uint32_t>(bits_of_quantization(gate->quantization));
  c.gdn_key_heads = 16;  // placeholders for models without GDN or attention layers
  c.gdn_value_heads = 48;
  c.q_heads = 24;
  c.kv_heads = 4;
  c.proj_bits = 4;
  if (first_gdn >= 0) {
    const std::uint32_t id = static_cast<std::uint32_t>(first_gdn);
    const gfxi::Tensor* qkv = view.find(layer_name(id, "linear_attn.in_proj_qkv.weight"));
    const gfxi::Tensor* a_log = view.find(layer_name(id, "linear_attn.A_log"));
    if (qkv == nullptr || a_log == nullptr || a_log->rank != 1) return artifact_error("artifact lacks a GDN layer's tensors");
    c.gdn_value_heads = static_cast<std::uint32_t>(a_log->dimensions[0]);
    const std::uint64_t key_rows = qkv->dimensions[0] - static_cast<std::uint64_t>(c.gdn_value_heads) * 128;
    if (qkv->dimensions[0] <= static_cast<std::uint64_t>(c.gdn_value_heads) * 128 || key_rows % 256 != 0) {
      return artifact_error("GDN qkv projection height is inconsistent with its heads");
    }
    c.gdn_key_heads = static_cast<std::uint32_t>(key_rows / 256);
    c.proj_bits = static_cast<std::uint32_t>(bits_of_quantization(qkv->quantization));
  }
  const std::uint32_t attention_id = first_attention >= 0 ? static_cast<std::uint32_t>(first_attention) : kLayerMtp;
  const gfxi::Tensor* q = view.find(layer_name(attention_id, "self_attn.q_proj.weight"));
  const gfxi::Tensor* k = view.find(layer_name(attention_id, "self_attn.k_proj.weight"));
  if (q != nullptr && k != nullptr) {
    c.q_heads = static_cast<std::uint32_t>(q->dimensions[0] / 512);
    c.kv_heads = static_cast<std::uint32_t>(k->dimensions[0] / 256);
    if (first_gdn < 0) c.proj_bits = static_cast<std::uint32_t>(bits_of_quantization(q->quantization));
  } else if (first_attention >= 0) {
    return artifact_error("artifact lacks an attention layer's projections");
  }
  c.activation_bits = options.activation_bits;
  c.max_context = options.max_context;
  c.draft_vocab = options.draft_vocab != 0 ? options.draft_vocab : std::min<std::uint32_t>(98304u, c.vocab);
  if (c.draft_vocab > c.vocab || c.draft_vocab % 16 != 0) return fail(GFXB_INVALID_ARGUMENT, "invalid MTP draft vocabulary");
  c.seed = 0;
  return GFXB_OK;
}

bool has_substring(const char* text, const char* part) { return std::strstr(text, part) != nullptr; }

}  // namespace
}  // namespace gfxb

extern "C" int gfxb_engine_create_synthetic(const gfxb_model_config* config, int device, int tp_rank, int tp_size,
                                            const void* nccl_id128, int include_mtp, gfxb_engine** out) {
  if (config == nullptr || out == nullptr) return fail(GFXB_INVALID_ARGUMENT, "engine arguments are null");
  WeightSource synthetic;
  return create_engine(*config, device, tp_rank, tp_size, nccl_id128, include_mtp != 0, synthetic, out);
}

extern "C" int gfxb_engine_create_from_artifact(const char* path, const gfxb_artifact_load_options* options,
                                                int device, int tp_rank, int tp_size, const void* nccl_id128,
                                                gfxb_engine** out) {
  if (path == nullptr || options == nullptr || out == nullptr) return fail(GFXB_INVALID_ARGUMENT, "null argument");
  *out = nullptr;
  gfxi::View view;
  GFXB_TRY(view.open(path, options->verify_checksums != 0));
  const gfxb_artifact_identity& id = view.identity();
  if (std::strcmp(id.target_arch, "sm_100a") != 0 && std::strcmp(id.target_arch, "gfx1200") != 0) {
    const std::string message = std::string("artifact target is ") + id.target_arch + "; expected sm_100a or gfx1200";
    return fail(GFXB_UNSUPPORTED, message.c_str());
  }
  if (std::strcmp(id.model_id, "qwen3.8-27b") != 0 && std::strcmp(id.model_id, "qwen-hybrid") != 0) {
    const std::string message = std::string("artifact model is ") + id.model_id + "; expected qwen3.8-27b or qwen-hybrid";
    return fail(GFXB_UNSUPPORTED, message.c_str());
  }
  WeightSource src;
  src.view = &view;
  if (std::strcmp(id.recipe_id, "b200-v1") == 0) {
    src.gfx12 = false;
  } else if (has_substring(id.recipe_id, "tiled-v")) {
    src.gfx12 = true;
    src.sequential_w3 = has_substring(id.recipe_id, "w3seq");
  } else {
    const std::string message = std::string("artifact recipe ") + id.recipe_id + " is not a tiled or b200 recipe";
    return fail(GFXB_UNSUPPORTED, message.c_str());
  }
  gfxb_model_config config{};
  GFXB_TRY(derive_config(view, *options, config));
  if (options->include_mtp != 0 && view.find("mtp.fc.weight") == nullptr) {
    return fail(GFXB_CORRUPT_ARTIFACT, "artifact lacks the MTP layer");
  }
  return create_engine(config, device, tp_rank, tp_size, nccl_id128, options->include_mtp != 0, src, out);
}

namespace gfxb {
namespace {

struct ExportItem {
  gfxi::Plan plan;
  const void* data = nullptr;  // device
  const void* aux = nullptr;   // device
};

void export_matrix(std::vector<ExportItem>& items, const std::string& name, const QMatrix& m) {
  ExportItem item;
  item.plan.name = name;
  item.plan.dtype = GFXB_DTYPE_U8;
  item.plan.quantization = static_cast<std::uint16_t>(m.format);  // GFXB_W* equal the Quantization values
  item.plan.dimensions = {m.rows, m.cols};
  const int bits = m.format == GFXB_W2 ? 2 : (m.format == GFXB_W3 ? 3 : 4);
  item.plan.data_bytes = static_cast<std::uint64_t>(m.rows) * m.cols * bits / 8;
  item.plan.aux_bytes = static_cast<std::uint64_t>(m.rows) * (m.cols / 128) * 2;
  item.data = m.codes;
  item.aux = m.scales;
  items.push_back(std::move(item));
}

void export_bf16(std::vector<ExportItem>& items, const std::string& name, const std::uint16_t* values,
                 std::vector<std::uint64_t> dimensions) {
  ExportItem item;
  item.plan.name = name;
  item.plan.dtype = GFXB_DTYPE_BF16;
  item.plan.quantization = GFXB_QUANT_NONE;
  std::uint64_t count = 1;
  for (std::uint64_t d : dimensions) count *= d;
  item.plan.dimensions = std::move(dimensions);
  item.plan.data_bytes = count * 2;
  item.data = values;
  items.push_back(std::move(item));
}

std::vector<ExportItem> export_items(const gfxb_engine& e) {
  const gfxb_model_config& c = e.cfg;
  const std::uint64_t H = c.hidden;
  std::vector<ExportItem> items;
  auto mlp = [&](const Layer& L, std::uint32_t id) {
    export_bf16(items, layer_name(id, "input_layernorm.weight"), L.input_norm, {H});
    export_bf16(items, layer_name(id, "post_attention_layernorm.weight"), L.post_norm, {H});
    export_matrix(items, layer_name(id, "mlp.gate_proj.weight"), L.gate);
    export_matrix(items, layer_name(id, "mlp.up_proj.weight"), L.up);
    export_matrix(items, layer_name(id, "mlp.down_proj.weight"), L.down);
  };
  auto attention = [&](const Layer& L, std::uint32_t id) {
    export_matrix(items, layer_name(id, "self_attn.q_proj.weight"), L.q);
    export_matrix(items, layer_name(id, "self_attn.k_proj.weight"), L.k);
    export_matrix(items, layer_name(id, "self_attn.v_proj.weight"), L.v);
    export_matrix(items, layer_name(id, "self_attn.o_proj.weight"), L.out);
    export_bf16(items, layer_name(id, "self_attn.q_norm.weight"), L.q_norm, {256});
    export_bf16(items, layer_name(id, "self_attn.k_norm.weight"), L.k_norm, {256});
  };
  for (std::uint32_t i = 0; i < c.layers; ++i) {
    const Layer& L = e.layers[i];
    mlp(L, i);
    if (L.attention) {
      attention(L, i);
    } else {
      const std::uint64_t channels = e.shard.channels;
      export_matrix(items, layer_name(i, "linear_attn.in_proj_qkv.weight"), L.qkv);
      export_matrix(items, layer_name(i, "linear_attn.in_proj_z.weight"), L.z);
      export_matrix(items, layer_name(i, "linear_attn.in_proj_a.weight"), L.a);
      export_matrix(items, layer_name(i, "linear_attn.in_proj_b.weight"), L.b);
      export_matrix(items, layer_name(i, "linear_attn.out_proj.weight"), L.out);
      export_bf16(items, layer_name(i, "linear_attn.conv1d.weight"), L.conv, {channels, 1, 4});
      export_bf16(items, layer_name(i, "linear_attn.A_log"), L.a_log, {c.gdn_value_heads});
      export_bf16(items, layer_name(i, "linear_attn.dt_bias"), L.dt_bias, {c.gdn_value_heads});
      export_bf16(items, layer_name(i, "linear_attn.norm.weight"), L.gdn_norm, {128});
    }
  }
  {
    ExportItem emb;
    emb.plan.name = "model.language_model.embed_tokens.weight";
    emb.plan.dtype = GFXB_DTYPE_U8;
    emb.plan.quantization = static_cast<std::uint16_t>(format_of(c.emb_bits));
    emb.plan.dimensions = {c.vocab, H};
    emb.plan.data_bytes = static_cast<std::uint64_t>(c.vocab) * H * c.emb_bits / 8;
    emb.plan.aux_bytes = static_cast<std::uint64_t>(c.vocab) * (H / 128) * 2;
    emb.data = e.emb_codes;
    emb.aux = e.emb_scales;
    items.push_back(std::move(emb));
  }
  export_matrix(items, "lm_head.weight", e.lm_head);
  export_bf16(items, "model.language_model.norm.weight", e.final_norm, {H});
  if (e.has_mtp) {
    mlp(e.mtp, kLayerMtp);
    attention(e.mtp, kLayerMtp);
    export_matrix(items, "mtp.fc.weight", e.fc);
    export_bf16(items, "mtp.pre_fc_norm_embedding.weight", e.pre_emb_norm, {H});
    export_bf16(items, "mtp.pre_fc_norm_hidden.weight", e.pre_hidden_norm, {H});
    export_bf16(items, "mtp.norm.weight", e.mtp_final_norm, {H});
  }
  std::sort(items.begin(), items.end(), [](const ExportItem& a, const ExportItem& b) { return a.plan.name < b.plan.name; });
  return items;
}

int copy_out(gfxi::StreamWriter& writer, std::size_t index, bool aux, const void* device, std::uint64_t bytes,
             std::byte* staging, std::size_t staging_bytes, cudaStream_t stream) {
  const std::byte* source = static_cast<const std::byte*>(device);
  for (std::uint64_t done = 0; done < bytes;) {
    const std::size_t chunk = static_cast<std::size_t>(std::min<std::uint64_t>(staging_bytes, bytes - done));
    GFXB_TRY(cuda_check(cudaMemcpyAsync(staging, source + done, chunk, cudaMemcpyDeviceToHost, stream),
                        "weight download failed"));
    GFXB_TRY(cuda_check(cudaStreamSynchronize(stream), "weight download failed"));
    GFXB_TRY(writer.append(index, aux, staging, chunk));
    done += chunk;
  }
  return GFXB_OK;
}

}  // namespace
}  // namespace gfxb

extern "C" int gfxb_engine_export_artifact(gfxb_engine* engine, const char* path, const char* weights_id) {
  if (engine == nullptr || path == nullptr) return fail(GFXB_INVALID_ARGUMENT, "null argument");
  if (engine->shard.tp != 1) return fail(GFXB_UNSUPPORTED, "export needs a single-GPU engine (the whole model)");
  gfxb_artifact_identity identity{};
  std::snprintf(identity.target_arch, sizeof identity.target_arch, "%s", "sm_100a");
  std::snprintf(identity.model_id, sizeof identity.model_id, "%s", "qwen-hybrid");
  std::snprintf(identity.recipe_id, sizeof identity.recipe_id, "%s", "b200-v1");
  const char* weights = weights_id != nullptr && weights_id[0] != '\0' ? weights_id : "synthetic";
  if (std::strlen(weights) >= sizeof identity.weights_id) return fail(GFXB_INVALID_ARGUMENT, "weights id is too long");
  std::snprintf(identity.weights_id, sizeof identity.weights_id, "%s", weights);
  GFXB_TRY(cuda_check(cudaSetDevice(engine->device), "cudaSetDevice failed"));
  const std::vector<ExportItem> items = export_items(*engine);
  std::vector<gfxi::Plan> plans;
  plans.reserve(items.size());
  for (const ExportItem& item : items) plans.push_back(item.plan);
  gfxi::StreamWriter writer;
  GFXB_TRY(writer.create(path, identity, plans));
  constexpr std::size_t kStaging = 64u << 20;
  std::byte* staging = nullptr;
  GFXB_TRY(cuda_check(cudaMallocHost(reinterpret_cast<void**>(&staging), kStaging), "staging allocation failed"));
  int status = GFXB_OK;
  for (std::size_t i = 0; i < items.size() && status == GFXB_OK; ++i) {
    status = copy_out(writer, i, false, items[i].data, items[i].plan.data_bytes, staging, kStaging, engine->stream);
    if (status == GFXB_OK && items[i].plan.aux_bytes != 0) {
      status = copy_out(writer, i, true, items[i].aux, items[i].plan.aux_bytes, staging, kStaging, engine->stream);
    }
  }
  cudaFreeHost(staging);
  GFXB_TRY(status);
  return writer.finalize();
}

extern "C" int gfxb_engine_config(const gfxb_engine* engine, gfxb_model_config* config) {
  if (engine == nullptr || config == nullptr) return fail(GFXB_INVALID_ARGUMENT, "null argument");
  *config = engine->cfg;
  return GFXB_OK;
}

extern "C" int gfxb_engine_destroy(gfxb_engine* engine) {
  if (engine == nullptr) return GFXB_OK;
  cudaSetDevice(engine->device);
  if (engine->comm != nullptr) nccl().comm_destroy(engine->comm);
  cudaFree(engine->arena);
  cudaStreamDestroy(engine->stream);
  delete engine;
  cudaGetLastError();  // teardown errors are not reported; keep them from surfacing in a later launch check
  return GFXB_OK;
}

extern "C" int gfxb_engine_abort(gfxb_engine* engine) {
  if (engine == nullptr) return fail(GFXB_INVALID_ARGUMENT, "null engine");
  if (engine->comm == nullptr || nccl().comm_abort == nullptr) return GFXB_OK;
  const ncclComm_t comm = engine->comm;
  engine->comm = nullptr;
  return nccl_check(nccl().comm_abort(comm), "ncclCommAbort failed");
}

extern "C" int gfxb_engine_weight_bytes(const gfxb_engine* engine, std::uint64_t* bytes) {
  if (engine == nullptr || bytes == nullptr) return fail(GFXB_INVALID_ARGUMENT, "null argument");
  *bytes = engine->arena_bytes;
  return GFXB_OK;
}

extern "C" int gfxb_session_create(gfxb_engine* engine, const gfxb_session_config* config, gfxb_session** out) {
  if (engine == nullptr || config == nullptr || out == nullptr) return fail(GFXB_INVALID_ARGUMENT, "null argument");
  *out = nullptr;
  if (config->maximum_context_tokens == 0 || config->maximum_context_tokens > engine->cfg.max_context ||
      (config->graph_verifier_batch != 0 &&
       (config->graph_verifier_batch < 2 || config->graph_verifier_batch > kMaxBlock))) {
    return fail(GFXB_INVALID_ARGUMENT, "invalid decode session configuration");
  }
  GFXB_TRY(cuda_check(cudaSetDevice(engine->device), "cudaSetDevice failed"));
  auto s = std::make_unique<gfxb_session>();
  s->e = engine;
  s->cfg = *config;
  s->stream = engine->stream;
  GFXB_TRY(allocate_session(*s, false));
  void* arena = nullptr;
  GFXB_TRY(cuda_check(cudaMalloc(&arena, s->arena_bytes), "session arena allocation failed"));
  s->arena = static_cast<std::byte*>(arena);
  allocate_session(*s, true);
  int status = cuda_check(cudaMemsetAsync(s->arena, 0, s->arena_bytes, s->stream), "session arena clear failed");
  const std::size_t ctx = config->maximum_context_tokens;
  std::vector<float> cos_table(ctx * 32), sin_table(ctx * 32);
  gfxb_rope_table(ctx, 64, 10000000.0f, cos_table.data(), sin_table.data());
  if (status == GFXB_OK) {
    status = cuda_check(cudaMemcpy(s->rope_cos, cos_table.data(), ctx * 32 * sizeof(float), cudaMemcpyHostToDevice),
                        "RoPE table upload failed");
  }
  if (status == GFXB_OK) {
    status = cuda_check(cudaMemcpy(s->rope_sin, sin_table.data(), ctx * 32 * sizeof(float), cudaMemcpyHostToDevice),
                        "RoPE table upload failed");
  }
  if (status == GFXB_OK) {
    status = cuda_check(cudaMallocHost(reinterpret_cast<void**>(&s->pinned), 256 * sizeof(std::uint32_t)),
                        "pinned staging allocation failed");
  }
  if (status == GFXB_OK) status = setup_peer_reduce(*s);
  if (status == GFXB_OK && config->step_kernel > GFXB_STEP_PERSISTENT) {
    status = fail(GFXB_INVALID_ARGUMENT, "unknown step kernel");
  }
  if (status == GFXB_OK && config->step_kernel == GFXB_STEP_PERSISTENT) status = build_token_loop(*s);
  if (status == GFXB_OK && config->use_graphs) status = capture_greedy(*s);
  if (status == GFXB_OK && config->graph_verifier_batch != 0 && engine->has_mtp) {
    status = capture_speculative(*s, config->graph_verifier_batch - 1);
  }
  if (status == GFXB_OK) status = cuda_check(cudaStreamSynchronize(s->stream), "session setup failed");
  if (status != GFXB_OK) {
    if (s->greedy_graph) cudaGraphExecDestroy(s->greedy_graph);
    if (s->spec_graph) cudaGraphExecDestroy(s->spec_graph);
    if (s->pinned) cudaFreeHost(s->pinned);
    release_peer_reduce(*s);
    cudaFree(s->arena);
    return status;
  }
  *out = s.release();
  return GFXB_OK;
}

extern "C" int gfxb_session_destroy(gfxb_session* session) {
  if (session == nullptr) return GFXB_OK;
  cudaSetDevice(session->e->device);
  cudaStreamSynchronize(session->stream);
  if (session->greedy_graph) cudaGraphExecDestroy(session->greedy_graph);
  if (session->spec_graph) cudaGraphExecDestroy(session->spec_graph);
  if (session->pinned) cudaFreeHost(session->pinned);
  if (session->loop_trace) cudaFree(session->loop_trace);
  release_peer_reduce(*session);
  cudaFree(session->arena);
  delete session;
  cudaGetLastError();  // teardown errors are not reported; keep them from surfacing in a later launch check
  return GFXB_OK;
}

namespace {

int upload_step(gfxb_session& s, const std::uint32_t* tokens, unsigned count) {
  std::memcpy(s.pinned, tokens, count * sizeof(std::uint32_t));
  std::uint64_t position = s.host_position;
  std::memcpy(s.pinned + 64, &position, sizeof position);
  GFXB_TRY(cuda_check(cudaMemcpyAsync(s.tokens, s.pinned, count * sizeof(std::uint32_t), cudaMemcpyHostToDevice, s.stream),
                      "token upload failed"));
  return cuda_check(cudaMemcpyAsync(s.position, s.pinned + 64, sizeof position, cudaMemcpyHostToDevice, s.stream),
                    "position upload failed");
}

int download_tokens(gfxb_session& s, const std::uint32_t* device, std::uint32_t* host, unsigned count) {
  GFXB_TRY(cuda_check(cudaMemcpyAsync(s.pinned + 128, device, count * sizeof(std::uint32_t), cudaMemcpyDeviceToHost,
                                      s.stream),
                      "token download failed"));
  GFXB_TRY(cuda_check(cudaStreamSynchronize(s.stream), "decode step failed"));
  std::memcpy(host, s.pinned + 128, count * sizeof(std::uint32_t));
  return GFXB_OK;
}

bool valid_tokens(const gfxb_session& s, const std::uint32_t* tokens, unsigned count) {
  for (unsigned i = 0; i < count; ++i) {
    if (tokens[i] >= s.e->cfg.vocab) return false;
  }
  return true;
}

}  // namespace

extern "C" int gfxb_session_greedy_step(gfxb_session* session, std::uint32_t input_token, std::uint32_t* output) {
  if (session == nullptr || output == nullptr) return fail(GFXB_INVALID_ARGUMENT, "null argument");
  gfxb_session& s = *session;
  if (s.host_position >= s.cfg.maximum_context_tokens || input_token >= s.e->cfg.vocab) {
    return fail(GFXB_INVALID_ARGUMENT, "decode token or session position is invalid");
  }
  GFXB_TRY(upload_step(s, &input_token, 1));
  if (s.greedy_graph != nullptr) {
    GFXB_TRY(cuda_check(cudaGraphLaunch(s.greedy_graph, s.stream), "graph launch failed"));
  } else if (s.loop_ready) {
    GFXB_TRY(launch_token_loop(s.loop, s.stream));
  } else {
    GFXB_TRY(enqueue_forward(s, 1, s.tokens, s.position, false));
  }
  s.last_hidden = s.hidden[s.e->cfg.layers % 2];
  GFXB_TRY(download_tokens(s, s.selected, output, 1));
  GFXB_TRY(check_token_loop(s));
  s.host_position += 1;
  s.have_last_hidden = true;
  s.mtp_chain_active = false;
  return GFXB_OK;
}

extern "C" int gfxb_session_enqueue_greedy(gfxb_session* session, std::uint32_t first_token, unsigned steps) {
  if (session == nullptr) return fail(GFXB_INVALID_ARGUMENT, "null session");
  gfxb_session& s = *session;
  if (s.greedy_graph == nullptr) return fail(GFXB_UNSUPPORTED, "device-resident decode needs use_graphs");
  if (s.host_position + steps > s.cfg.maximum_context_tokens || first_token >= s.e->cfg.vocab) {
    return fail(GFXB_INVALID_ARGUMENT, "decode loop exceeds the context or the token is invalid");
  }
  set_positions_kernel<<<1, 1, 0, s.stream>>>(s.position, s.host_position, s.mtp_positions, 0, 0, s.seed_token,
                                               first_token, s.tokens);
  GFXB_TRY(launch_status("decode loop setup failed"));
  for (unsigned i = 0; i < steps; ++i) {
    GFXB_TRY(cuda_check(cudaGraphLaunch(s.greedy_graph, s.stream), "graph launch failed"));
  }
  s.last_hidden = s.hidden[s.e->cfg.layers % 2];
  s.host_position += steps;
  s.have_last_hidden = steps > 0;
  s.mtp_chain_active = false;
  return GFXB_OK;
}

extern "C" int gfxb_session_sync(gfxb_session* session) {
  if (session == nullptr) return fail(GFXB_INVALID_ARGUMENT, "null session");
  GFXB_TRY(cuda_check(cudaStreamSynchronize(session->stream), "session synchronisation failed"));
  return check_token_loop(*session);
}

extern "C" int gfxb_session_last_token(gfxb_session* session, std::uint32_t* token) {
  if (session == nullptr || token == nullptr) return fail(GFXB_INVALID_ARGUMENT, "null argument");
  return download_tokens(*session, session->selected, token, 1);
}

extern "C" void* gfxb_session_stream(gfxb_session* session) { return session != nullptr ? session->stream : nullptr; }

extern "C" int gfxb_session_block_step(gfxb_session* session, const std::uint32_t* input_tokens, unsigned count,
                                       std::uint32_t* output_tokens) {
  if (session == nullptr || input_tokens == nullptr || output_tokens == nullptr) {
    return fail(GFXB_INVALID_ARGUMENT, "null argument");
  }
  gfxb_session& s = *session;
  if (count == 0 || count > kMaxBlock || count > s.cfg.maximum_context_tokens - s.host_position ||
      !valid_tokens(s, input_tokens, count)) {
    return fail(GFXB_INVALID_ARGUMENT,
                "decode block must contain a supported number of valid tokens within the context limit");
  }
  GFXB_TRY(upload_step(s, input_tokens, count));
  GFXB_TRY(enqueue_forward(s, count, s.tokens, s.position, false));
  GFXB_TRY(download_tokens(s, s.selected, output_tokens, count));
  s.host_position += count;
  s.have_last_hidden = true;
  s.mtp_chain_active = false;
  return GFXB_OK;
}

extern "C" int gfxb_session_mtp_draft(gfxb_session* session, std::uint32_t next_token, std::uint32_t* draft) {
  if (session == nullptr || draft == nullptr) return fail(GFXB_INVALID_ARGUMENT, "null argument");
  gfxb_session& s = *session;
  if (!s.e->has_mtp) return fail(GFXB_UNSUPPORTED, "engine was created without the MTP layer");
  if (!s.have_last_hidden || (!s.mtp_chain_active && s.mtp_position + 1 != s.host_position) ||
      next_token >= s.e->cfg.vocab || s.mtp_position >= s.cfg.maximum_context_tokens) {
    return fail(GFXB_INVALID_ARGUMENT, "MTP drafting is not aligned with the target state");
  }
  const __half* conditioning = s.mtp_chain_active ? s.mtp_hidden : s.last_hidden;
  s.pinned[0] = next_token;
  const std::uint64_t position = s.mtp_position;
  std::memcpy(s.pinned + 64, &position, sizeof position);
  GFXB_TRY(cuda_check(cudaMemcpyAsync(s.seed_token, s.pinned, 4, cudaMemcpyHostToDevice, s.stream), "upload failed"));
  GFXB_TRY(cuda_check(cudaMemcpyAsync(s.mtp_positions, s.pinned + 64, 8, cudaMemcpyHostToDevice, s.stream),
                      "upload failed"));
  GFXB_TRY(enqueue_mtp(s, s.seed_token, conditioning, s.mtp_positions, s.draft_tokens));
  GFXB_TRY(download_tokens(s, s.draft_tokens, draft, 1));
  s.mtp_position += 1;
  return GFXB_OK;
}

namespace {

// One speculative round (qwen_runtime.cpp:1421-1544). drafts == nullptr: the
// MTP chain's proposals are verified; otherwise the caller's.
int speculative_round(gfxb_session& s, std::uint32_t seed_token, unsigned draft_count, const std::uint32_t* drafts,
                      std::uint32_t* tokens, unsigned* token_count, unsigned* accepted_out) {
  if (!s.e->has_mtp) return fail(GFXB_UNSUPPORTED, "engine was created without the MTP layer");
  if (!s.have_last_hidden || draft_count == 0 || draft_count >= kMaxBlock || seed_token >= s.e->cfg.vocab ||
      s.mtp_position + 1 != s.host_position ||
      draft_count + 1 > s.cfg.maximum_context_tokens - s.host_position) {
    return fail(GFXB_INVALID_ARGUMENT, "speculative step requires 1..31 drafts and aligned target/MTP state");
  }
  const std::uint64_t base = s.host_position, mtp_base = s.mtp_position;
  const gfxb_model_config& c = s.e->cfg;
  // snapshot the conditioning hidden state (qwen_runtime.cpp:236-247)
  GFXB_TRY(cuda_check(cudaMemcpyAsync(s.target_snapshot, s.last_hidden, c.hidden * sizeof(__half),
                                      cudaMemcpyDeviceToDevice, s.stream),
                      "hidden snapshot failed"));
  set_positions_kernel<<<1, 1, 0, s.stream>>>(s.position, base, s.mtp_positions, mtp_base, draft_count, s.seed_token,
                                               seed_token, s.tokens);
  GFXB_TRY(launch_status("position setup failed"));
  if (drafts != nullptr) {
    std::memcpy(s.pinned + 192, drafts, draft_count * sizeof(std::uint32_t));
    GFXB_TRY(cuda_check(cudaMemcpyAsync(s.external_drafts, s.pinned + 192, draft_count * sizeof(std::uint32_t),
                                        cudaMemcpyHostToDevice, s.stream),
                        "draft upload failed"));
    GFXB_TRY(enqueue_speculative_body(s, draft_count, true));
  } else if (s.spec_graph != nullptr && draft_count == s.spec_drafts) {
    // the captured round when its draft count matches (launch_prepared_speculative_graph, :888-934)
    GFXB_TRY(cuda_check(cudaGraphLaunch(s.spec_graph, s.stream), "speculative graph launch failed"));
  } else {
    GFXB_TRY(enqueue_speculative_body(s, draft_count));
  }
  const unsigned batch = draft_count + 1;
  std::uint32_t host[2 * kMaxBlock];
  GFXB_TRY(cuda_check(cudaStreamSynchronize(s.stream), "speculative round failed"));
  std::memcpy(host, s.pinned + 128, draft_count * 4);
  std::memcpy(host + kMaxBlock, s.pinned + 160, batch * 4);
  unsigned accepted = 0;
  while (accepted < draft_count && host[accepted] == host[kMaxBlock + accepted]) ++accepted;
  const std::size_t conv_elems = static_cast<std::size_t>(s.e->gdn_layers) * s.e->shard.channels * 4;
  const std::size_t state_elems = static_cast<std::size_t>(s.e->gdn_layers) * s.e->shard.nv * 128 * 128;
  if (accepted != draft_count) {
    // replay the accepted prefix (+ the correction's own input) onto the untouched states
    GdnRestoreArgs r;
    r.conv_states = s.conv_states;
    r.states = s.gdn_states;
    r.conv_logs = s.conv_log;
    r.key_logs = s.key_log;
    r.delta_logs = s.delta_log;
    r.decay_logs = s.decay_log;
    r.channels = s.e->shard.channels;
    r.key_heads = s.e->shard.nk;
    r.value_heads = s.e->shard.nv;
    r.layers = s.e->gdn_layers;
    r.max_logged = kMaxBlock;
    r.accepted = accepted + 1;
    GFXB_TRY(launch_gdn_restore(r, s.stream));
    s.host_position = base + accepted + 1;
    s.mtp_position = mtp_base + accepted + 1;
    s.last_hidden = s.hidden[c.layers % 2] + static_cast<std::size_t>(accepted) * c.hidden;
  } else {
    // The verifier's final states become current. Copied rather than swapped
    // because the captured greedy graph holds the state addresses.
    GFXB_TRY(cuda_check(cudaMemcpyAsync(s.conv_states, s.conv_snapshot, conv_elems * sizeof(__half),
                                        cudaMemcpyDeviceToDevice, s.stream),
                        "conv state commit failed"));
    GFXB_TRY(cuda_check(cudaMemcpyAsync(s.gdn_states, s.gdn_snapshot, state_elems * sizeof(float),
                                        cudaMemcpyDeviceToDevice, s.stream),
                        "recurrent state commit failed"));
    s.host_position = base + batch;
    s.mtp_position = mtp_base + draft_count;
    s.last_hidden = s.hidden[c.layers % 2] + static_cast<std::size_t>(draft_count) * c.hidden;
    // advance only the MTP KV cache through the final draft (qwen_runtime.cpp:1520-1534)
    const std::uint64_t position = s.mtp_position;
    std::memcpy(s.pinned + 64, &position, sizeof position);
    GFXB_TRY(cuda_check(cudaMemcpyAsync(s.mtp_positions, s.pinned + 64, 8, cudaMemcpyHostToDevice, s.stream),
                        "upload failed"));
    GFXB_TRY(enqueue_mtp(s, s.draft_tokens + draft_count - 1, s.last_hidden - c.hidden, s.mtp_positions, nullptr));
    GFXB_TRY(cuda_check(cudaStreamSynchronize(s.stream), "MTP cache advance failed"));
    s.mtp_position += 1;
  }
  s.mtp_chain_active = false;
  for (unsigned i = 0; i < accepted; ++i) tokens[i] = host[i];
  tokens[accepted] = host[kMaxBlock + accepted];
  *token_count = accepted + 1;
  *accepted_out = accepted;
  return GFXB_OK;
}

}  // namespace

extern "C" int gfxb_session_speculative_step(gfxb_session* session, std::uint32_t seed_token, unsigned draft_count,
                                             std::uint32_t* tokens, unsigned* token_count, unsigned* accepted_out) {
  if (session == nullptr || tokens == nullptr || token_count == nullptr || accepted_out == nullptr) {
    return fail(GFXB_INVALID_ARGUMENT, "null argument");
  }
  return speculative_round(*session, seed_token, draft_count, nullptr, tokens, token_count, accepted_out);
}

extern "C" int gfxb_session_speculative_step_with_drafts(gfxb_session* session, std::uint32_t seed_token,
                                                         const std::uint32_t* drafts, unsigned draft_count,
                                                         std::uint32_t* tokens, unsigned* token_count,
                                                         unsigned* accepted_out) {
  if (session == nullptr || drafts == nullptr || tokens == nullptr || token_count == nullptr ||
      accepted_out == nullptr) {
    return fail(GFXB_INVALID_ARGUMENT, "null argument");
  }
  if (draft_count >= kMaxBlock || !valid_tokens(*session, drafts, draft_count)) {
    return fail(GFXB_INVALID_ARGUMENT, "drafts must be 1..31 valid token ids");
  }
  return speculative_round(*session, seed_token, draft_count, drafts, tokens, token_count, accepted_out);
}

extern "C" int gfxb_session_prefill(gfxb_session* session, const std::uint32_t* tokens, std::size_t count,
                                    std::uint32_t* next_token) {
  if (session == nullptr || tokens == nullptr || next_token == nullptr) {
    return fail(GFXB_INVALID_ARGUMENT, "null argument");
  }
  gfxb_session& s = *session;
  if (count == 0 || count > s.cfg.maximum_context_tokens - s.host_position || !valid_tokens(s, tokens, static_cast<unsigned>(count))) {
    return fail(GFXB_INVALID_ARGUMENT, "prompt must hold valid tokens within the context limit");
  }
  // causal blocks of up to 32 tokens; the LM head runs for the prompt's last token only
  for (std::size_t done = 0; done < count;) {
    const unsigned n = static_cast<unsigned>(std::min<std::size_t>(kMaxBlock, count - done));
    const bool last = done + n == count;
    GFXB_TRY(upload_step(s, tokens + done, n));
    GFXB_TRY(enqueue_forward(s, n, s.tokens, s.position, false, last ? Head::last : Head::none));
    if (!last) GFXB_TRY(cuda_check(cudaStreamSynchronize(s.stream), "prefill block failed"));
    s.host_position += n;
    done += n;
  }
  GFXB_TRY(download_tokens(s, s.selected, next_token, 1));
  s.have_last_hidden = true;
  s.mtp_chain_active = false;
  return GFXB_OK;
}

extern "C" int gfxb_session_position(const gfxb_session* session, std::uint64_t* position) {
  if (session == nullptr || position == nullptr) return fail(GFXB_INVALID_ARGUMENT, "null argument");
  *position = session->host_position;
  return GFXB_OK;
}

extern "C" int gfxb_session_read_state(gfxb_session* session, std::uint16_t* hidden, float* logits,
                                       std::size_t logits_count) {
  if (session == nullptr) return fail(GFXB_INVALID_ARGUMENT, "null session");
  gfxb_session& s = *session;
  GFXB_TRY(cuda_check(cudaStreamSynchronize(s.stream), "session synchronisation failed"));
  if (hidden != nullptr && s.last_hidden != nullptr) {
    GFXB_TRY(cuda_check(cudaMemcpy(hidden, s.last_hidden, s.e->cfg.hidden * sizeof(__half), cudaMemcpyDeviceToHost),
                        "hidden download failed"));
  }
  if (logits != nullptr) {
    const std::size_t n = std::min<std::size_t>(logits_count, s.e->shard.vocab);
    GFXB_TRY(cuda_check(cudaMemcpy(logits, s.logits, n * sizeof(float), cudaMemcpyDeviceToHost), "logit download failed"));
  }
  return GFXB_OK;
}

extern "C" int gfxb_session_enqueue_operation(gfxb_session* session, int kind, unsigned launches,
                                              std::uint64_t* bytes) {
  if (session == nullptr || launches == 0 || kind < 0 || kind > GFXB_OP_SILU_PACK) {
    return fail(GFXB_INVALID_ARGUMENT, "invalid operation benchmark arguments");
  }
  gfxb_session& s = *session;
  gfxb_engine& e = *s.e;
  const gfxb_model_config& c = e.cfg;
  const Shard& sh = e.shard;
  const std::uint64_t H = c.hidden;
  const bool gdn_kind = kind == GFXB_OP_GDN_IN || kind == GFXB_OP_GDN_OUT || kind == GFXB_OP_GDN_STEP;
  const bool attention_kind = kind == GFXB_OP_ATTN_QKV || kind == GFXB_OP_ATTN_O || kind == GFXB_OP_ATTENTION;
  // Cycle over the layers that carry the operation so every launch reads its
  // own weights or states from HBM (one layer's fit in L2; all of them do not).
  std::vector<const Layer*> layers;
  for (const Layer& L : e.layers) {
    if ((!gdn_kind && !attention_kind) || (gdn_kind && !L.attention) || (attention_kind && L.attention)) {
      layers.push_back(&L);
    }
  }
  if (layers.empty()) return fail(GFXB_INVALID_ARGUMENT, "no layer carries the requested operation");
  const std::uint64_t act_bytes_per_column = c.activation_bits == 8 ? 1 : 0;  // A8: one byte; A4: half a byte
  auto act_bytes = [&](std::uint64_t cols) {
    return (act_bytes_per_column != 0 ? cols : cols / 2) + cols / 128 * 2;
  };
  auto matrix_bytes = [&](const QMatrix& m) {
    const std::uint64_t bits = m.format == GFXB_W2 ? 2 : (m.format == GFXB_W3 ? 3 : 4);
    return static_cast<std::uint64_t>(m.rows) * m.cols * bits / 8 + static_cast<std::uint64_t>(m.rows) * (m.cols / 128) * 2 +
           static_cast<std::uint64_t>(m.rows) * 4;
  };
  const std::size_t kv_stride = static_cast<std::size_t>(s.cfg.maximum_context_tokens) * sh.nkv * 256;
  const std::uint64_t position = std::min<std::uint64_t>(s.host_position, s.cfg.maximum_context_tokens - 1);
  if (kind == GFXB_OP_ATTENTION) {
    // from pinned memory and without a synchronisation, so the launches can be captured in a graph
    std::memcpy(s.pinned + 64, &position, sizeof position);
    GFXB_TRY(cuda_check(cudaMemcpyAsync(s.position, s.pinned + 64, sizeof position, cudaMemcpyHostToDevice, s.stream),
                        "position upload failed"));
  }
  std::uint64_t total = 0;
  for (unsigned i = 0; i < launches; ++i) {
    const Layer& L = *layers[i % layers.size()];
    std::vector<std::pair<const QMatrix*, void*>> mats;
    std::uint64_t b = 0;
    switch (kind) {
      case GFXB_OP_MLP_GATE_UP: mats = {{&L.gate, s.gate}, {&L.up, s.up}}; break;
      case GFXB_OP_MLP_DOWN: mats = {{&L.down, s.update}}; break;
      case GFXB_OP_GDN_IN: mats = {{&L.qkv, s.proj_main}, {&L.z, s.proj_z}, {&L.a, s.proj_a}, {&L.b, s.proj_b}}; break;
      case GFXB_OP_GDN_OUT: mats = {{&L.out, s.update}}; break;
      case GFXB_OP_ATTN_QKV: mats = {{&L.q, s.proj_main}, {&L.k, s.proj_k}, {&L.v, s.proj_v}}; break;
      case GFXB_OP_ATTN_O: mats = {{&L.out, s.update}}; break;
      case GFXB_OP_LM_HEAD: {
        static thread_local QMatrix head;
        head = e.lm_head;
        head.rows = sh.vocab;
        mats = {{&head, s.logits}};
        break;
      }
      case GFXB_OP_GDN_STEP: {
        GFXB_TRY(gdn_recurrent_step(s, L, 1, false));
        const std::uint64_t state = static_cast<std::uint64_t>(sh.nv) * 128 * 128 * 4;
        b = 2 * state + static_cast<std::uint64_t>(sh.channels) * (4 * 2 * 2 + 4 * 2 + 4) +
            static_cast<std::uint64_t>(sh.nv) * 128 * (4 + 2) + 2ull * sh.nv * 4 + act_bytes(sh.nv * 128ull) +
            sh.nv * 128ull / 128 * 4;
        break;
      }
      case GFXB_OP_ATTENTION: {
        GFXB_TRY(attention_core(s, L, s.key_cache + L.state_index * kv_stride, s.value_cache + L.state_index * kv_stride,
                                s.position, 1));
        b = (position + 1) * sh.nkv * 256ull * 2 * 2 + sh.nq * 512ull * 4 + 2ull * sh.nkv * 256 * 4 +
            act_bytes(sh.nq * 256ull) + sh.nq * 256ull / 128 * 4;
        break;
      }
      case GFXB_OP_NORM_PACK:
        GFXB_TRY(norm_pack(s, s.hidden[0], s.update, s.hidden[1], L.post_norm, 1));
        b = H * 2 + H * 4 + H * 2 + H * 2 + act_bytes(H) + H / 128 * 4;
        break;
      default: {  // GFXB_OP_SILU_PACK
        SiluPackArgs a;
        a.gate = s.gate;
        a.up = s.up;
        a.elements = sh.inter;
        a.batch = 1;
        a.act_codes = s.act_codes;
        a.act_scales = s.act_scales;
        a.act_sums = s.act_sums;
        GFXB_TRY(launch_silu_pack(a, static_cast<int>(c.activation_bits), s.stream));
        b = sh.inter * 8ull + act_bytes(sh.inter) + sh.inter / 128 * 4ull;
        break;
      }
    }
    if (!mats.empty()) {
      GFXB_TRY(gemv(s, mats, 1));
      for (const auto& m : mats) b += matrix_bytes(*m.first);
      b += act_bytes(mats[0].first->cols) + mats[0].first->cols / 128 * 4;
    }
    if (i == 0) total = b;
  }
  if (bytes != nullptr) *bytes = total;
  return GFXB_OK;
}

extern "C" int gfxb_session_time_operation(gfxb_session* session, int kind, unsigned launches, int use_graph,
                                           float* microseconds, std::uint64_t* bytes) {
  if (session == nullptr || microseconds == nullptr || launches == 0) {
    return fail(GFXB_INVALID_ARGUMENT, "invalid operation timing arguments");
  }
  gfxb_session& s = *session;
  GFXB_TRY(cuda_check(cudaSetDevice(s.e->device), "cudaSetDevice failed"));
  GFXB_TRY(gfxb_session_enqueue_operation(session, kind, std::min(launches, 8u), nullptr));  // warm-up
  cudaEvent_t start = nullptr, stop = nullptr;
  cudaGraphExec_t exec = nullptr;
  int status = cuda_check(cudaEventCreate(&start), "event creation failed");
  if (status == GFXB_OK) status = cuda_check(cudaEventCreate(&stop), "event creation failed");
  if (status == GFXB_OK && use_graph) {
    // the launches captured once and replayed: host launch cost stays out of the timing
    cudaGraph_t graph = nullptr;
    status = cuda_check(cudaStreamBeginCapture(s.stream, cudaStreamCaptureModeThreadLocal), "graph capture start failed");
    if (status == GFXB_OK) {
      const int enqueued = gfxb_session_enqueue_operation(session, kind, launches, bytes);
      const cudaError_t end = cudaStreamEndCapture(s.stream, &graph);
      status = enqueued != GFXB_OK ? enqueued : cuda_check(end, "graph capture end failed");
    }
    if (status == GFXB_OK) status = cuda_check(cudaGraphInstantiate(&exec, graph, 0), "graph instantiation failed");
    if (graph != nullptr) cudaGraphDestroy(graph);
    if (status == GFXB_OK) status = cuda_check(cudaGraphLaunch(exec, s.stream), "graph launch failed");
    if (status == GFXB_OK) status = cuda_check(cudaEventRecord(start, s.stream), "event record failed");
    if (status == GFXB_OK) status = cuda_check(cudaGraphLaunch(exec, s.stream), "graph launch failed");
  } else if (status == GFXB_OK) {
    status = cuda_check(cudaStreamSynchronize(s.stream), "warm-up failed");
    if (status == GFXB_OK) status = cuda_check(cudaEventRecord(start, s.stream), "event record failed");
    if (status == GFXB_OK) status = gfxb_session_enqueue_operation(session, kind, launches, bytes);
  }
  if (status == GFXB_OK) status = cuda_check(cudaEventRecord(stop, s.stream), "event record failed");
  if (status == GFXB_OK) status = cuda_check(cudaEventSynchronize(stop), "timed launches failed");
  float ms = 0.0f;
  if (status == GFXB_OK) status = cuda_check(cudaEventElapsedTime(&ms, start, stop), "event timing failed");
  if (status == GFXB_OK) *microseconds = ms * 1000.0f / static_cast<float>(launches);
  if (exec != nullptr) cudaGraphExecDestroy(exec);
  if (start != nullptr) cudaEventDestroy(start);
  if (stop != nullptr) cudaEventDestroy(stop);
  return status;
}

extern "C" int gfxb_session_enqueue_gemv(gfxb_session* session, int kind, unsigned launches, std::uint64_t* bytes) {
  if (session == nullptr || launches == 0) return fail(GFXB_INVALID_ARGUMENT, "invalid GEMV benchmark arguments");
  gfxb_session& s = *session;
  gfxb_engine& e = *s.e;
  // Cycle over the layers that carry the requested projection so every launch
  // streams its weights from HBM (one layer's matrices fit in L2; 48 do not).
  std::vector<const Layer*> layers;
  for (const Layer& L : e.layers) {
    if (kind == 0 || kind == 1 || (kind == 2 && !L.attention)) layers.push_back(&L);
  }
  if (layers.empty()) return fail(GFXB_INVALID_ARGUMENT, "no layer carries the requested projection");
  std::uint64_t total = 0;
  for (unsigned i = 0; i < launches; ++i) {
    const Layer& L = *layers[i % layers.size()];
    std::vector<std::pair<const QMatrix*, void*>> mats;
    if (kind == 0) mats = {{&L.gate, s.gate}, {&L.up, s.up}};
    else if (kind == 1) mats = {{&L.down, s.update}};
    else mats = {{&L.qkv, s.proj_main}, {&L.z, s.proj_z}, {&L.a, s.proj_a}, {&L.b, s.proj_b}};
    GFXB_TRY(gemv(s, mats, 1));
    if (i == 0) {
      const QMatrix& first = *mats[0].first;
      const std::uint32_t bits = first.format == GFXB_W2 ? 2 : (first.format == GFXB_W3 ? 3 : 4);
      for (const auto& m : mats) {
        const std::uint64_t rows = m.first->rows, cols = m.first->cols;
        total += rows * cols * bits / 8 + rows * (cols / 128) * 2 + rows * 4;  // codes + fp16 scales + fp32 out
      }
      const std::uint64_t cols = first.cols;
      total += cols / 2 + cols / 128 * 2;  // A4 activation + its fp16 group scales
    }
  }
  if (bytes != nullptr) *bytes = total;
  return GFXB_OK;
}

extern "C" int gfxb_session_trace_step(gfxb_session* session, std::uint32_t input_token, std::uint32_t* output_token,
                                       std::uint64_t* timeline, std::size_t timeline_entries, unsigned* op_count,
                                       unsigned* ctas, std::uint32_t* op_kinds) {
  if (session == nullptr || output_token == nullptr || op_count == nullptr || ctas == nullptr) {
    return fail(GFXB_INVALID_ARGUMENT, "null argument");
  }
  gfxb_session& s = *session;
  if (!s.loop_ready) return fail(GFXB_UNSUPPORTED, "the session does not run the persistent token kernel");
  *op_count = s.loop.op_count;
  *ctas = s.loop.ctas;
  const std::size_t entries = (static_cast<std::size_t>(s.loop.op_count) + 1u) * 2u * s.loop.ctas;
  if (timeline == nullptr || timeline_entries < entries) {
    return fail(GFXB_INVALID_ARGUMENT, "timeline buffer must hold (op_count + 1) * 2 * ctas entries");
  }
  if (s.host_position >= s.cfg.maximum_context_tokens || input_token >= s.e->cfg.vocab) {
    return fail(GFXB_INVALID_ARGUMENT, "decode token or session position is invalid");
  }
  cudaSetDevice(s.e->device);
  if (s.loop_trace == nullptr) {
    GFXB_TRY(cuda_check(cudaMalloc(reinterpret_cast<void**>(&s.loop_trace), entries * sizeof(std::uint64_t)),
                        "timeline allocation failed"));
  }
  GFXB_TRY(cuda_check(cudaMemsetAsync(s.loop_trace, 0, entries * sizeof(std::uint64_t), s.stream), "timeline reset failed"));
  GFXB_TRY(upload_step(s, &input_token, 1));
  LoopLaunch traced = s.loop;
  traced.trace = s.loop_trace;
  GFXB_TRY(launch_token_loop(traced, s.stream));
  s.last_hidden = s.hidden[s.e->cfg.layers % 2];
  GFXB_TRY(download_tokens(s, s.selected, output_token, 1));
  GFXB_TRY(check_token_loop(s));
  s.host_position += 1;
  s.have_last_hidden = true;
  s.mtp_chain_active = false;
  GFXB_TRY(cuda_check(cudaMemcpy(timeline, s.loop_trace, entries * sizeof(std::uint64_t), cudaMemcpyDeviceToHost),
                      "timeline download failed"));
  if (op_kinds != nullptr) {
    std::vector<LoopOp> ops(s.loop.op_count);
    GFXB_TRY(cuda_check(cudaMemcpy(ops.data(), s.loop_ops, ops.size() * sizeof(LoopOp), cudaMemcpyDeviceToHost),
                        "operation list download failed"));
    for (std::size_t i = 0; i < ops.size(); ++i) {
      op_kinds[i] = ops[i].kind == kLoopGemv ? (ops[i].gemv.bits << 8) | (ops[i].gemv.act_source << 4) | kLoopGemv
                                             : ops[i].kind;
    }
  }
  return GFXB_OK;
}

extern "C" int gfxb_read_device_errors(std::uint32_t* flags) {
  if (flags == nullptr) return fail(GFXB_INVALID_ARGUMENT, "null argument");
  std::uint32_t a = 0, b = 0, c = 0;
  GFXB_TRY(read_gemv_error(&a, true));
  GFXB_TRY(read_ops_error(&b, true));
  GFXB_TRY(read_peer_errors(&c));
  *flags = a | b | c;
  return GFXB_OK;
}

extern "C" int gfxb_rope_table(std::size_t positions, unsigned rotary, float theta, float* cos_table,
                               float* sin_table) {
  if (cos_table == nullptr || sin_table == nullptr || rotary == 0 || (rotary & 1u) != 0 || !(theta > 1.0f)) {
    return fail(GFXB_INVALID_ARGUMENT, "invalid RoPE table arguments");
  }
  const unsigned half = rotary / 2;
  for (std::size_t p = 0; p < positions; ++p) {
    for (unsigned f = 0; f < half; ++f) {
      const float exponent = (2.0f * static_cast<float>(f)) / static_cast<float>(rotary);
      const float inv_freq = static_cast<float>(std::pow(static_cast<double>(theta), -static_cast<double>(exponent)));
      const float angle = static_cast<float>(p) * inv_freq;
      cos_table[p * half + f] = static_cast<float>(std::cos(static_cast<double>(angle)));
      sin_table[p * half + f] = static_cast<float>(std::sin(static_cast<double>(angle)));
    }
  }
  return GFXB_OK;
}
