// Persistent token kernel: one launch runs a whole batch-1 decode step (all
// layers, the LM head and the argmax) as a list of operations executed by one
// CTA per SM.
//
// Each CTA has four producer warps and eight compute warps. The producers walk
// the CTA's share of every weight matrix of the step, in step order, and
// streams it into shared memory with bulk copies (cp.async.bulk, mbarrier
// completion): weight codes into a ring of 16 KB slots, each tile's fp16
// scales into a small ring of its own (a tile's scales stay until its fp32
// chain is done, while its code slots are released as soon as they are
// read). The four producers (lane 0 of each producer warp) issue alternate
// copies, so one producer's wait for a free slot never stalls the stream; a
// waiting producer may be suspended in hardware, which is why each has a
// warp of its own. Weights never depend on activations,
// so the stream runs ahead across operation and layer boundaries while the
// compute warps wait at grid barriers. Compute warps run each operation's units (16-row
// weight tiles, GDN value heads, attention chunks) and meet at a grid barrier
// before every operation that reads another CTA's output.
//
// Arithmetic is the standalone kernels' (ops_device.cuh, codec.cuh): the
// same reductions in the same order, so both paths produce identical bits.
#pragma once

#include <cstddef>
#include <cstdint>

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "ops.cuh"

namespace gfxb {

constexpr unsigned kLoopComputeWarps = 8;
constexpr unsigned kLoopComputeThreads = kLoopComputeWarps * 32;
constexpr unsigned kLoopSlotBytes = 16384;                   // one code-ring slot
constexpr unsigned kLoopProducerLanes = 4;                   // producer warps (lane 0 of each issues copies)
constexpr unsigned kLoopThreads = kLoopComputeThreads + 32 * kLoopProducerLanes;
constexpr unsigned kLoopScaleSlots = 4;                      // scale-ring slots (one tile's scales each)
constexpr unsigned kLoopMaxGroups = 512;                     // K <= 65536
constexpr unsigned kLoopMaxCtas = 1024;
constexpr unsigned kLoopMaxKvHeads = 64;
constexpr unsigned kLoopMaxNormIterations = 40;  // hidden <= 10240

enum LoopOpKind : std::uint32_t { kLoopGemv = 1, kLoopGdn = 2, kLoopAttention = 3, kLoopArgmax = 4 };

// Where a GEMV's activation pack comes from (built in shared memory by every CTA).
enum LoopActSource : std::uint32_t {
  kActEmbedNorm = 1,     // embedding row of tokens[0] -> RMSNorm -> pack (residual_out = the row)
  kActResidualNorm = 2,  // fp16(residual + update) -> RMSNorm -> pack (residual_out = the sum)
  kActPackF16 = 3,       // fp16 vector -> pack
  kActGlobalPack = 4,    // copy of a pack another operation wrote
};

// What a matrix's fp32 outputs turn into.
enum LoopEpilogue : std::uint32_t {
  kEpiF32 = 0,       // fp32 rows
  kEpiConv = 1,      // GDN causal conv of each channel -> fp16 conv output, conv state update
  kEpiSiluPair = 2,  // matrix 0 = gate, matrix 1 = up: fp16 SiLU(gate) * up into matrix 0's output
  kEpiLogits = 3,    // fp32 logits + this CTA's running argmax
};

struct LoopMatrix {
  const std::uint8_t* codes;
  const __half* scales;
  void* output;
  std::uint32_t tiles;
  std::uint32_t epilogue;
  __half* conv_state;                // kEpiConv: [rows][4] fp16 taps
  const std::uint16_t* conv_weight;  // kEpiConv: [rows][4] bf16
};

struct LoopGemv {
  std::uint32_t bits;     // 2, 3 or 4
  std::uint32_t groups;   // K / 128
  std::uint32_t count;    // matrices (1..4)
  std::uint32_t paired;   // units are (tile of matrix 0, same tile of matrix 1)
  std::uint32_t units;    // tiles (or tile pairs)
  LoopMatrix m[4];
  std::uint32_t act_source;
  const __half* residual;
  const float* update;
  __half* residual_out;  // written by CTA 0 only
  const std::uint16_t* norm_weight;
  const std::uint8_t* embedding_codes;
  const __half* embedding_scales;
  std::uint32_t embedding_rows, embedding_bits;
  const std::uint32_t* tokens;
  const __half* f16_input;
  const std::int8_t* pack_codes;
  const __half* pack_scales;
  const std::int32_t* pack_sums;
};

struct LoopOp {
  std::uint32_t kind;
  std::uint32_t rotation;  // unit u runs on CTA (u + rotation) % grid
  LoopGemv gemv;
  GdnRecurrentArgs gdn;    // batch 1
  QkRopeArgs rope;         // batch 1, device position
  AttentionArgs attention; // batch 1, device position
};

// Device-side control block of one session (zeroed at creation).
struct LoopControl {
  std::uint32_t arrive;  // grid-barrier arrivals, never reset
  std::uint32_t epoch;   // value of `arrive` when the next launch starts
  std::uint32_t abort;   // set when a wait expired: every later wait returns at once
  std::uint32_t error;   // kLoopError* bits
  std::uint32_t attention_arrivals[kLoopMaxKvHeads];
  float argmax_value[kLoopMaxCtas];
  std::uint32_t argmax_index[kLoopMaxCtas];
};

constexpr std::uint32_t kLoopErrorBarrier = 1u;   // a grid barrier wait expired
constexpr std::uint32_t kLoopErrorRing = 2u;      // a weight-ring wait expired
constexpr std::uint32_t kLoopErrorContext = 4u;   // position outside the KV cache or RoPE table

struct LoopLaunch {
  const LoopOp* ops;
  std::uint32_t op_count;
  LoopControl* control;
  std::uint32_t hidden;
  std::uint32_t vocab;        // logits rows of the LM head (argmax range)
  std::uint32_t* selected;    // argmax result
  std::uint32_t* tokens;      // next input token
  std::uint64_t* position;    // advanced by one per step
  std::uint32_t slots;        // code-ring slots
  std::uint32_t ring_offset, bars_offset, act_offset, act_scales_offset, act_sums_offset, dots_offset;
  std::uint32_t scale_offset, scale_bars_offset;
  std::uint32_t scale_slot_bytes;  // largest K / 128 * 32, rounded to 128
  std::uint32_t dots_half;    // int32 words per dots buffer (two buffers)
  std::uint32_t smem_bytes;   // dynamic shared memory of the launch
  std::uint32_t ctas;         // grid: one CTA per SM
  std::uint32_t act_bits;     // 4 or 8
  // Optional timeline ([op_count + 1][2][ctas] globaltimer ns, null: off).
  // Entry (i, 0, cta): the CTA's compute warps finished operation i - 1 and
  // reached the grid barrier in front of operation i; (i, 1, cta): the
  // barrier released. Entry i = 0 is the kernel start, i = op_count its end.
  std::uint64_t* trace;
};

// Shared-memory plan for the given largest K (groups) and dots buffer; also
// configures the kernel and checks that one CTA fits each SM. Call outside
// stream capture; launch_token_loop then only launches.
int plan_token_loop(LoopLaunch& launch, std::uint32_t max_groups, std::uint32_t dots_half, int device);
// Grid size (one CTA per SM).
int token_loop_grid(int device, std::uint32_t* ctas);
int launch_token_loop(const LoopLaunch& launch, cudaStream_t stream);
bool token_loop_supported_hidden(std::uint32_t hidden);

}  // namespace gfxb
