// Persistent token kernel (see token_loop.cuh for the design).
//
// Ring protocol. Slot s of the code ring carries a `full` mbarrier (issuing
// lane's arrival + bulk-copy bytes) and an `empty` mbarrier (one arrival per
// compute warp). Producer lanes and compute warps walk the same sequence of
// slot uses: for every GEMV operation, for each of this CTA's units, for each
// matrix tile of the unit, ceil(G / groups-per-slot) slots of weight codes;
// use n is issued by producer n % kLoopProducerLanes. A compute warp
// waits for `full` before it reads a slot and arrives on `empty` after, even
// when the slot holds none of its groups, so a slot is refilled only after
// every warp is done with it. Each tile's fp16 scales travel through the
// scale ring (same protocol, one `empty` arrival: the warp that runs the
// tile's fp32 chain releases it).
//
// Every wait is bounded by the global timer. A wait that expires sets the
// control block's abort word; every later wait of every CTA then returns at
// once, the kernel runs to its end without waiting, and the host reports the
// error. Control flow between named barriers never depends on data, so an
// abort cannot leave a barrier short of threads.
#include <algorithm>

#include "codec.cuh"
#include "common.cuh"
#include "ops_device.cuh"
#include "token_loop.cuh"

namespace gfxb {
namespace {

constexpr std::uint64_t kLoopWaitNs = 1000000000ull;  // 1 s, far above any legitimate wait


using ComputeSync = NamedSync<1, kLoopComputeThreads>;

union LoopScratch {
  struct {
    __half query[8 * 256];
    float scores[8][kAttentionChunk];
    float alphas[8][kAttentionChunk];
    float betas[8][kAttentionChunk];
    float normalized[256];
    float warp_sums[8];
    float pack_max[2][4];
    int pack_sum[2][4];
  } attention;
  GdnScratch gdn;
  struct {
    float warp_sums[8];
    float warp_max[kLoopMaxNormIterations][8];
    int code_sums[kLoopMaxNormIterations][8];
  } norm;
};

__device__ __forceinline__ std::uint64_t global_ns() {
  std::uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ std::uint32_t ld_volatile(const std::uint32_t* p) {
  return *reinterpret_cast<const volatile std::uint32_t*>(p);
}
__device__ __forceinline__ std::uint32_t ld_acquire(const std::uint32_t* p) {
  std::uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ std::uint64_t ld_cg_u64(const std::uint64_t* p) {
  std::uint64_t v;
  asm volatile("ld.global.cg.u64 %0, [%1];" : "=l"(v) : "l"(p));
  return v;
}
__device__ __forceinline__ uint2 ld_cg8(const void* p) {
  uint2 v;
  asm volatile("ld.global.cg.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p));
  return v;
}
__device__ __forceinline__ void mbar_arrive(std::uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

struct Ctx {
  LoopControl* ctl;
  std::uint8_t* ring;
  std::uint64_t* full;
  std::uint64_t* empty;
  std::uint8_t* scale_ring;
  std::uint64_t* scale_full;
  std::uint64_t* scale_empty;
  std::uint32_t scale_slot_bytes;
  std::uint32_t sn;            // scale-ring position
  std::int8_t* act_codes;
  __half* act_scales;
  std::int32_t* act_sums;
  std::int32_t* dots;
  std::uint32_t dots_half;
  std::uint32_t slots;
  std::uint32_t cta, ctas;
  std::uint32_t n;             // ring position
  std::uint32_t unit_counter;  // GEMV units done by this CTA
  volatile std::uint32_t* abort;
  std::uint64_t* trace;        // LoopLaunch::trace
};

// Timeline entry (see LoopLaunch::trace); thread 0 only.
__device__ __forceinline__ void trace_mark(const Ctx& c, std::uint32_t op, std::uint32_t which) {
  if (c.trace != nullptr) c.trace[(2ull * op + which) * c.ctas + c.cta] = global_ns();
}

__device__ __forceinline__ std::uint32_t first_unit(const Ctx& c, std::uint32_t rotation) {
  return (c.cta + c.ctas - rotation % c.ctas) % c.ctas;
}

// Matrix index and tile of part `part` of unit `unit`.
__device__ __forceinline__ std::uint32_t locate(const LoopGemv& g, std::uint32_t unit, std::uint32_t part,
                                                std::uint32_t& tile) {
  if (g.paired) {
    tile = unit;
    return part;
  }
  std::uint32_t i = 0;
  tile = unit;
  while (i + 1 < g.count && tile >= g.m[i].tiles) {
    tile -= g.m[i].tiles;
    ++i;
  }
  return i;
}

__device__ __forceinline__ void raise_abort(Ctx& c, std::uint32_t error) {
  atomicOr(&c.ctl->error, error);
  atomicExch(&c.ctl->abort, 1u);
  *c.abort = 1u;
}

// Another CTA's abort is polled from global memory at most every
// kLoopAbortPollNs while a wait lasts: a global load on every spin would
// delay each wake-up by an L2 round trip.
constexpr std::uint64_t kLoopAbortPollNs = 20000;

// Warp-uniform bounded wait for a ring slot's `full` phase (`round`: the slot's use count).
__device__ __forceinline__ bool ring_wait(Ctx& c, std::uint64_t* bar, std::uint32_t round, unsigned lane) {
  if (*c.abort != 0) return false;
  const std::uint32_t parity = round & 1u;
  std::uint64_t start = 0, next_poll = 0;
  for (std::uint32_t spin = 0;; ++spin) {
    const bool done = mbar_try_wait(bar, parity);
    if (__all_sync(0xffffffffu, done)) return true;
    std::uint32_t stop = 0;
    if (lane == 0) {
      const std::uint64_t now = global_ns();
      if (spin == 0) {
        start = now;
        next_poll = now + kLoopAbortPollNs;
      }
      if (*c.abort != 0) {
        stop = 1;
      } else if (now >= next_poll) {
        next_poll = now + kLoopAbortPollNs;
        if (ld_volatile(&c.ctl->abort) != 0) {
          *c.abort = 1u;
          stop = 1;
        } else if (now - start > kLoopWaitNs) {
          raise_abort(c, kLoopErrorRing);
          stop = 1;
        }
      }
    }
    if (__shfl_sync(0xffffffffu, stop, 0) != 0) return false;
  }
}

// Grid barrier over all CTAs (compute warps only). Returns false once the
// step is aborted.
__device__ __forceinline__ bool grid_barrier(Ctx& c, std::uint32_t target, std::uint32_t op) {
  ComputeSync{}();
  if (threadIdx.x == 0) trace_mark(c, op, 0);
  if (threadIdx.x == 0 && *c.abort == 0) {
    __threadfence();
    atomicAdd(&c.ctl->arrive, 1u);
    const std::uint64_t start = global_ns();
    std::uint64_t next_poll = start + kLoopAbortPollNs;
    while (true) {
      const std::uint32_t v = ld_acquire(&c.ctl->arrive);
      if (static_cast<std::int32_t>(v - target) >= 0) break;
      const std::uint64_t now = global_ns();
      if (now >= next_poll) {
        next_poll = now + kLoopAbortPollNs;
        if (ld_volatile(&c.ctl->abort) != 0) {
          *c.abort = 1u;
          break;
        }
        if (now - start > kLoopWaitNs) {
          raise_abort(c, kLoopErrorBarrier);
          break;
        }
      }
    }
    __threadfence();
  }
  if (threadIdx.x == 0) trace_mark(c, op, 1);
  ComputeSync{}();
  return *c.abort == 0;
}

// ---------------------------------------------------------------------------
// producers: lane 0 of each of the last kLoopProducerLanes warps
// ---------------------------------------------------------------------------

__device__ __forceinline__ bool producer_wait(Ctx& c, std::uint64_t* bar, std::uint32_t parity, bool honour_abort) {
  const std::uint64_t start = global_ns();
  std::uint64_t next_poll = start + kLoopAbortPollNs;
  while (!mbar_try_wait(bar, parity)) {
    if (honour_abort && *c.abort != 0) return false;
    const std::uint64_t now = global_ns();
    if (now >= next_poll) {
      next_poll = now + kLoopAbortPollNs;
      if (honour_abort && ld_volatile(&c.ctl->abort) != 0) return false;
      if (now - start > kLoopWaitNs) {
        raise_abort(c, kLoopErrorRing);
        return false;
      }
    }
  }
  return true;
}

// Groups of weight codes one code slot carries.
__device__ __forceinline__ std::uint32_t groups_per_slot(std::uint32_t bits) { return kLoopSlotBytes / (bits * 256u); }

// Every producer walks the whole copy sequence and issues the copies it owns
// (sequence position % kLoopProducerLanes == lane, `lane` = producer index).
__device__ __forceinline__ void produce(const LoopLaunch& L, Ctx& c, unsigned lane) {
  std::uint32_t code_n = 0, scale_n = 0;
  bool ok = true;
  auto issue = [&](std::uint32_t n, std::uint32_t slots, std::uint64_t* full, std::uint64_t* empty,
                   std::uint8_t* ring, std::uint32_t slot_bytes, const void* source, std::uint32_t bytes) {
    if (!ok || n % kLoopProducerLanes != lane) return;
    const std::uint32_t slot = n % slots, round = n / slots;
    if (round > 0 && !producer_wait(c, &empty[slot], (round - 1u) & 1u, true)) {
      ok = false;
      return;
    }
    mbar_expect_tx(&full[slot], bytes);
    bulk_g2s(ring + static_cast<std::size_t>(slot) * slot_bytes, source, bytes, &full[slot]);
  };
  for (std::uint32_t i = 0; ok && i < L.op_count; ++i) {
    const LoopOp& op = L.ops[i];
    if (op.kind != kLoopGemv) continue;
    const LoopGemv& g = op.gemv;
    const std::uint32_t block = g.bits * 256u, G = g.groups, per_slot = groups_per_slot(g.bits);
    const std::uint32_t parts = g.paired ? 2u : 1u;
    for (std::uint32_t u = first_unit(c, op.rotation); ok && u < g.units; u += c.ctas) {
      for (std::uint32_t p = 0; ok && p < parts; ++p) {
        std::uint32_t tile;
        const LoopMatrix& m = g.m[locate(g, u, p, tile)];
        issue(scale_n++, kLoopScaleSlots, c.scale_full, c.scale_empty, c.scale_ring, c.scale_slot_bytes,
              m.scales + static_cast<std::size_t>(tile) * G * 16u, G * 32u);
        for (std::uint32_t g0 = 0; g0 < G; g0 += per_slot) {
          issue(code_n++, c.slots, c.full, c.empty, c.ring, kLoopSlotBytes,
                m.codes + (static_cast<std::size_t>(tile) * G + g0) * block, min(per_slot, G - g0) * block);
        }
      }
    }
  }
  // No copy may still be landing in shared memory when the CTA exits.
  for (std::uint32_t k = code_n > c.slots ? code_n - c.slots : 0u; k < code_n; ++k) {
    if (k % kLoopProducerLanes == lane) producer_wait(c, &c.full[k % c.slots], (k / c.slots) & 1u, false);
  }
  for (std::uint32_t k = scale_n > kLoopScaleSlots ? scale_n - kLoopScaleSlots : 0u; k < scale_n; ++k) {
    if (k % kLoopProducerLanes == lane) {
      producer_wait(c, &c.scale_full[k % kLoopScaleSlots], (k / kLoopScaleSlots) & 1u, false);
    }
  }
}

// ---------------------------------------------------------------------------
// GEMV
// ---------------------------------------------------------------------------

// int32 dots of this warp's groups of one code slot (groups g0..g1-1 of the
// tile; warp w takes first = g0 + (w - g0) mod 8, first + 8, ...), token 0:
// lanes with t = lane % 4 == 0 hold rows lane/4 and lane/4 + 8. All of the
// warp's groups are loaded, unpacked and multiplied together (indices past
// g1 repeat the last group and are not stored), and each group's four mma
// run as two independent chains, so the tensor-core latency overlaps.
template <int Bits>
__device__ __forceinline__ void slot_dots(const std::uint8_t* base, std::uint32_t g0, std::uint32_t g1,
                                          const std::int8_t* act_codes, const std::int32_t* act_sums,
                                          unsigned warp, unsigned lane, std::int32_t* out) {
  constexpr int kAlpha = Codec<Bits>::alpha, kBeta = Codec<Bits>::beta;
  constexpr std::uint32_t kBlock = Bits * 256u;
  constexpr std::uint32_t kPerWarp = (kLoopSlotBytes / kBlock + kLoopComputeWarps - 1u) / kLoopComputeWarps;
  const unsigned tq = lane & 3u, gl = lane >> 2;
  const std::uint32_t first = g0 + ((warp + kLoopComputeWarps - g0 % kLoopComputeWarps) % kLoopComputeWarps);
  if (first >= g1) return;
  std::uint32_t group[kPerWarp];
  LaneWords<Bits> w[kPerWarp];
  uint4 b0[kPerWarp], b1[kPerWarp];
#pragma unroll
  for (std::uint32_t j = 0; j < kPerWarp; ++j) {
    group[j] = min(first + kLoopComputeWarps * j, g1 - 1u);
    load_lane_shared<Bits>(base + (group[j] - g0) * kBlock, lane, w[j]);
    const std::int8_t* act = act_codes + group[j] * kGroup + tq * 32u;
    b0[j] = *reinterpret_cast<const uint4*>(act);
    b1[j] = *reinterpret_cast<const uint4*>(act + 16u);
  }
  int acc[kPerWarp][2][4];
#pragma unroll
  for (std::uint32_t j = 0; j < kPerWarp; ++j) {
    std::uint32_t a[4][4];
    unpack(w[j], a);
#pragma unroll
    for (int h = 0; h < 2; ++h) {
#pragma unroll
      for (int r = 0; r < 4; ++r) acc[j][h][r] = 0;
    }
    mma_s8_16832(acc[j][0], a[0], b0[j].x, b0[j].y);
    mma_s8_16832(acc[j][1], a[1], b0[j].z, b0[j].w);
    mma_s8_16832(acc[j][0], a[2], b1[j].x, b1[j].y);
    mma_s8_16832(acc[j][1], a[3], b1[j].z, b1[j].w);
  }
#pragma unroll
  for (std::uint32_t j = 0; j < kPerWarp; ++j) {
    if (tq == 0 && first + kLoopComputeWarps * j < g1) {
      const std::int32_t sum = act_sums[group[j]];
      out[group[j] * 16u + gl] = kAlpha * (acc[j][0][0] + acc[j][1][0]) + kBeta * sum;
      out[group[j] * 16u + gl + 8u] = kAlpha * (acc[j][0][2] + acc[j][1][2]) + kBeta * sum;
    }
  }
}

template <int ActBits, unsigned NormIters>
__device__ __forceinline__ void gemv_prologue(const LoopLaunch& L, Ctx& c, const LoopGemv& g, LoopScratch& sc) {
  const unsigned t = threadIdx.x;
  const std::uint32_t G = g.groups;
  if (g.act_source == kActEmbedNorm || g.act_source == kActResidualNorm) {
    NormPackArgs a;
    a.residual = g.residual;
    a.update = g.act_source == kActResidualNorm ? g.update : nullptr;
    a.residual_out = c.cta == 0 ? g.residual_out : nullptr;
    a.weight = g.norm_weight;
    a.unit_offset = 1;
    a.epsilon = 1.0e-6f;
    a.elements = L.hidden;
    a.act_codes = c.act_codes;
    a.act_scales = c.act_scales;
    a.act_sums = c.act_sums;
    if (g.act_source == kActEmbedNorm) {
      a.embedding_codes = g.embedding_codes;
      a.embedding_scales = g.embedding_scales;
      a.embedding_rows = g.embedding_rows;
      a.embedding_bits = static_cast<int>(g.embedding_bits);
      a.device_tokens = g.tokens;
    }
    norm_pack_body<ActBits, NormIters>(a, 0, t, ComputeSync{}, sc.norm.warp_sums, sc.norm.warp_max,
                                       sc.norm.code_sums);
  } else if (g.act_source == kActPackF16) {
    // Batches of eight groups per warp: all eight L2 loads are in flight
    // before the first group's reductions.
    const unsigned warp = t >> 5, lane = t & 31u;
    constexpr std::uint32_t kBatch = 8;
    for (std::uint32_t first = warp; first < G; first += kBatch * kLoopComputeWarps) {
      uint2 raw[kBatch];
#pragma unroll
      for (std::uint32_t j = 0; j < kBatch; ++j) {
        const std::uint32_t group = min(first + j * kLoopComputeWarps, G - 1u);
        raw[j] = ld_cg8(g.f16_input + static_cast<std::size_t>(group) * kGroup + 4u * lane);
      }
#pragma unroll
      for (std::uint32_t j = 0; j < kBatch; ++j) {
        const std::uint32_t group = first + j * kLoopComputeWarps;
        if (group >= G) break;
        const __half* hv = reinterpret_cast<const __half*>(&raw[j]);
        const float x[4] = {h2f(hv[0]), h2f(hv[1]), h2f(hv[2]), h2f(hv[3])};
        pack_warp_group<ActBits>(x, lane, c.act_codes + group * kGroup, c.act_scales + group, c.act_sums + group);
      }
    }
  } else {
    for (std::uint32_t i = t; i < G * 8u; i += kLoopComputeThreads) {
      reinterpret_cast<uint4*>(c.act_codes)[i] = ld_cg16(g.pack_codes + static_cast<std::size_t>(i) * 16u);
    }
    for (std::uint32_t i = t; i < G; i += kLoopComputeThreads) {
      c.act_scales[i] = ld_cg(g.pack_scales + i);
      c.act_sums[i] = ld_cg(g.pack_sums + i);
    }
  }
  ComputeSync{}();
}

template <int Bits>
__device__ __forceinline__ void gemv_units(Ctx& c, const LoopOp& op, float* best, std::uint32_t* best_index) {
  const LoopGemv& g = op.gemv;
  const unsigned t = threadIdx.x, warp = t >> 5, lane = t & 31u;
  constexpr std::uint32_t kPerSlot = kLoopSlotBytes / (Bits * 256u);
  const std::uint32_t G = g.groups;
  const std::uint32_t parts = g.paired ? 2u : 1u;
  for (std::uint32_t u = first_unit(c, op.rotation); u < g.units; u += c.ctas, ++c.unit_counter) {
    std::int32_t* dbuf = c.dots + (c.unit_counter & 1u) * c.dots_half;
    const unsigned chain_warp = c.unit_counter % kLoopComputeWarps;
    std::uint32_t scale_pos[2] = {0, 0}, tiles[2] = {0, 0}, mats[2] = {0, 0};
#pragma unroll
    for (std::uint32_t p = 0; p < 2; ++p) {
      if (p >= parts) break;
      mats[p] = locate(g, u, p, tiles[p]);
      scale_pos[p] = c.sn++;
      std::int32_t* dpart = dbuf + p * G * 16u;
      for (std::uint32_t g0 = 0; g0 < G; g0 += kPerSlot) {
        const std::uint32_t pos = c.n++, slot = pos % c.slots;
        const bool ok = ring_wait(c, &c.full[slot], pos / c.slots, lane);
        if (ok) {
          slot_dots<Bits>(c.ring + static_cast<std::size_t>(slot) * kLoopSlotBytes, g0, min(G, g0 + kPerSlot),
                          c.act_codes, c.act_sums, warp, lane, dpart);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&c.empty[slot]);
      }
    }
    ComputeSync{}();
    if (warp != chain_warp) continue;
    // fp32 chain over groups in ascending order (lowbit_gemv.hip:525-536);
    // lanes 0-15 run part 0's rows, lanes 16-31 part 1's.
    const std::uint32_t p = lane >> 4, row = lane & 15u;
    bool ok = true;
    ok = ring_wait(c, &c.scale_full[scale_pos[0] % kLoopScaleSlots], scale_pos[0] / kLoopScaleSlots, lane);
    if (parts == 2) {
      ok = ring_wait(c, &c.scale_full[scale_pos[1] % kLoopScaleSlots], scale_pos[1] / kLoopScaleSlots, lane) && ok;
    }
    const std::uint32_t my_scale = p == 0 ? scale_pos[0] : scale_pos[1];
    const std::uint32_t my_tile = p == 0 ? tiles[0] : tiles[1];
    const std::uint32_t my_mat = p == 0 ? mats[0] : mats[1];
    float acc = 0.0f;
    if (ok && p < parts) {
      const __half* ws = reinterpret_cast<const __half*>(
          c.scale_ring + static_cast<std::size_t>(my_scale % kLoopScaleSlots) * c.scale_slot_bytes);
      const std::int32_t* d = dbuf + p * G * 16u;
      std::uint32_t gg = 0;
      for (; gg + 8u <= G; gg += 8u) {
        float product[8];
        int dot[8];
#pragma unroll
        for (unsigned i = 0; i < 8; ++i) {
          product[i] = __fmul_rn(h2f(ws[(gg + i) * 16u + row]), h2f(c.act_scales[gg + i]));
          dot[i] = d[(gg + i) * 16u + row];
        }
#pragma unroll
        for (unsigned i = 0; i < 8; ++i) acc = fmaf(static_cast<float>(dot[i]), product[i], acc);
      }
      for (; gg < G; ++gg) {
        const float product = __fmul_rn(h2f(ws[gg * 16u + row]), h2f(c.act_scales[gg]));
        acc = fmaf(static_cast<float>(d[gg * 16u + row]), product, acc);
      }
    }
    const LoopMatrix& m = g.m[my_mat];
    const std::uint32_t epilogue = g.m[mats[0]].epilogue;
    const std::uint32_t r = my_tile * 16u + row;
    if (epilogue == kEpiSiluPair) {
      const float up = __shfl_down_sync(0xffffffffu, acc, 16);
      if (ok && p == 0) static_cast<__half*>(m.output)[r] = silu_product(acc, up);
    } else if (epilogue == kEpiLogits) {
      float value = -__int_as_float(0x7f800000);
      std::uint32_t index = 0xffffffffu;
      if (ok && p == 0) {
        static_cast<float*>(m.output)[r] = acc;
        value = acc;
        index = r;
      }
#pragma unroll
      for (unsigned offset = 8; offset != 0; offset >>= 1) {
        const float other_value = __shfl_xor_sync(0xffffffffu, value, offset);
        const std::uint32_t other_index = __shfl_xor_sync(0xffffffffu, index, offset);
        better(value, index, other_value, other_index);
      }
      if (lane == 0) better(*best, *best_index, value, index);
    } else if (ok && p < parts) {
      if (epilogue == kEpiConv) {
        const uint2 raw = *reinterpret_cast<const uint2*>(m.conv_state + static_cast<std::size_t>(r) * 4u);
        __half taps[4];
        *reinterpret_cast<uint2*>(taps) = raw;
        float w[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) w[i] = bf2f(m.conv_weight[static_cast<std::size_t>(r) * 4u + i]);
        static_cast<__half*>(m.output)[r] = gdn_conv_step(taps, w, acc);
        *reinterpret_cast<uint2*>(m.conv_state + static_cast<std::size_t>(r) * 4u) = *reinterpret_cast<uint2*>(taps);
      } else {
        static_cast<float*>(m.output)[r] = acc;
      }
    }
    __syncwarp();
    if (lane == 0) {
      mbar_arrive(&c.scale_empty[scale_pos[0] % kLoopScaleSlots]);
      if (parts == 2) mbar_arrive(&c.scale_empty[scale_pos[1] % kLoopScaleSlots]);
    }
  }
}

// ---------------------------------------------------------------------------
// attention: one unit = (kv head, 128-position chunk); the last arriving
// chunk of a kv head merges the partials of its query heads.
// ---------------------------------------------------------------------------

__device__ __forceinline__ void attention_units(const LoopLaunch& L, Ctx& c, const LoopOp& op, LoopScratch& sc,
                                std::uint32_t* flag) {
  const AttentionArgs& A = op.attention;
  const QkRopeArgs& R = op.rope;
  const unsigned t = threadIdx.x, warp = t >> 5, lane = t & 31u;
  const std::uint32_t group = A.q_heads / A.kv_heads;
  const std::uint64_t position = ld_cg_u64(A.device_base_position);
  const std::uint64_t count = position + 1u;
  const std::uint32_t chunks = static_cast<std::uint32_t>((count + kAttentionChunk - 1u) / kAttentionChunk);
  const std::uint32_t units = A.kv_heads * A.max_chunks;
  const std::size_t row_stride = static_cast<std::size_t>(A.kv_heads) * 256u;
  for (std::uint32_t u = first_unit(c, op.rotation); u < units; u += c.ctas) {
    const std::uint32_t kvh = u / A.max_chunks, chunk = u % A.max_chunks;
    if (chunk >= chunks) continue;
    if (count > A.capacity) {
      if (t == 0) atomicOr(&c.ctl->error, kLoopErrorContext);
      continue;
    }
    bool out_of_range = false;
    for (std::uint32_t j = 0; j < group; ++j) {
      const std::uint32_t h = kvh * group + j;
      const float value = ld_cg(R.q_input + static_cast<std::size_t>(h) * R.q_stride + t);
      bool oor = false;
      sc.attention.query[j * 256u + t] = qk_norm_rope_value(value, R.q_weight, position, R, t, ComputeSync{},
                                                            sc.attention.normalized, sc.attention.warp_sums, oor);
      out_of_range = out_of_range || oor;
    }
    if (chunk == chunks - 1u) {
      // this chunk holds the new position: K RMSNorm/RoPE and the KV append
      const float value = ld_cg(R.k_input + static_cast<std::size_t>(kvh) * R.k_stride + t);
      bool oor = false;
      const __half key = qk_norm_rope_value(value, R.k_weight, position, R, t, ComputeSync{},
                                            sc.attention.normalized, sc.attention.warp_sums, oor);
      out_of_range = out_of_range || oor;
      const std::size_t slot = (static_cast<std::size_t>(position) * A.kv_heads + kvh) * 256u + t;
      R.key_cache[slot] = key;
      R.value_cache[slot] = f2h(ld_cg(R.v_input + static_cast<std::size_t>(kvh) * 256u + t));
    }
    if (out_of_range && t == 0) atomicOr(&c.ctl->error, kLoopErrorContext);
    ComputeSync{}();
    if (warp < group) {
      const std::uint32_t h = kvh * group + warp;
      const std::uint64_t begin = static_cast<std::uint64_t>(chunk) * kAttentionChunk;
      const std::uint64_t remaining = count - begin;
      const std::uint32_t n = remaining < kAttentionChunk ? static_cast<std::uint32_t>(remaining) : kAttentionChunk;
      float* partial = A.partials + (static_cast<std::size_t>(h) * A.max_chunks + chunk) * 258u;
      attention_chunk_warp(sc.attention.query + warp * 256u, A.key_cache + (begin * A.kv_heads + kvh) * 256u,
                           A.value_cache + (begin * A.kv_heads + kvh) * 256u, row_stride, n, lane,
                           sc.attention.scores[warp], sc.attention.alphas[warp], sc.attention.betas[warp], partial);
    }
    ComputeSync{}();
    if (t == 0) {
      __threadfence();
      const std::uint32_t arrived = atomicAdd(&c.ctl->attention_arrivals[kvh], 1u) + 1u;
      const bool last = arrived == chunks;
      if (last) atomicExch(&c.ctl->attention_arrivals[kvh], 0u);
      __threadfence();
      *flag = last ? 1u : 0u;
    }
    ComputeSync{}();
    if (*flag != 0) {
      for (std::uint32_t j = 0; j < group; ++j) {
        attention_merge_head<ComputeSync, 1>(A, kvh * group + j, 0, t, chunks, ComputeSync{}, sc.attention.pack_max,
                             sc.attention.pack_sum);
        ComputeSync{}();
      }
    }
  }
}

// ---------------------------------------------------------------------------
// the kernel
// ---------------------------------------------------------------------------

template <int ActBits, unsigned NormIters>
__global__ void __launch_bounds__(kLoopThreads, 1) token_loop_kernel(const __grid_constant__ LoopLaunch L) {
  extern __shared__ __align__(1024) std::uint8_t smem[];
  __shared__ LoopScratch scratch;
  __shared__ std::uint32_t s_abort, s_flag, s_best_index;
  __shared__ float s_best;

  Ctx c;
  c.ctl = L.control;
  c.ring = smem + L.ring_offset;
  c.full = reinterpret_cast<std::uint64_t*>(smem + L.bars_offset);
  c.empty = c.full + L.slots;
  c.act_codes = reinterpret_cast<std::int8_t*>(smem + L.act_offset);
  c.act_scales = reinterpret_cast<__half*>(smem + L.act_scales_offset);
  c.act_sums = reinterpret_cast<std::int32_t*>(smem + L.act_sums_offset);
  c.dots = reinterpret_cast<std::int32_t*>(smem + L.dots_offset);
  c.scale_ring = smem + L.scale_offset;
  c.scale_full = reinterpret_cast<std::uint64_t*>(smem + L.scale_bars_offset);
  c.scale_empty = c.scale_full + kLoopScaleSlots;
  c.scale_slot_bytes = L.scale_slot_bytes;
  c.sn = 0;
  c.dots_half = L.dots_half;
  c.slots = L.slots;
  c.cta = blockIdx.x;
  c.ctas = gridDim.x;
  c.n = 0;
  c.unit_counter = 0;
  c.abort = &s_abort;
  c.trace = L.trace;

  if (threadIdx.x == 0) {
    trace_mark(c, 0, 0);
    trace_mark(c, 0, 1);
    for (std::uint32_t s = 0; s < L.slots; ++s) {
      mbar_init(&c.full[s], 1);
      mbar_init(&c.empty[s], kLoopComputeWarps);
    }
    for (std::uint32_t s = 0; s < kLoopScaleSlots; ++s) {
      mbar_init(&c.scale_full[s], 1);
      mbar_init(&c.scale_empty[s], 1);
    }
    fence_mbar_init();
    s_abort = 0;
  }
  __syncthreads();
  if (threadIdx.x >= kLoopComputeThreads) {
    const unsigned producer = (threadIdx.x - kLoopComputeThreads) >> 5;
    if ((threadIdx.x & 31u) == 0) produce(L, c, producer);
    return;
  }

  const unsigned t = threadIdx.x, warp = t >> 5, lane = t & 31u;
  const std::uint32_t base = t == 0 ? ld_volatile(&L.control->epoch) : 0u;
  for (std::uint32_t i = 0; i < L.op_count; ++i) {
    const LoopOp& op = L.ops[i];
    const std::uint32_t target = base + i * c.ctas;
    const std::uint32_t kind = op.kind;
    if (kind == kLoopGemv) {
      const LoopGemv& g = op.gemv;
      if (i > 0) grid_barrier(c, target, i);
      const bool logits = g.m[0].epilogue == kEpiLogits;
      if (logits && t == 0) {
        s_best = -__int_as_float(0x7f800000);
        s_best_index = 0xffffffffu;
      }
      gemv_prologue<ActBits, NormIters>(L, c, g, scratch);
      if (g.bits == 3) {
        gemv_units<3>(c, op, &s_best, &s_best_index);
      } else if (g.bits == 4) {
        gemv_units<4>(c, op, &s_best, &s_best_index);
      } else {
        gemv_units<2>(c, op, &s_best, &s_best_index);
      }
      if (logits) {
        ComputeSync{}();
        if (t == 0) {
          L.control->argmax_value[c.cta] = s_best;
          L.control->argmax_index[c.cta] = s_best_index;
        }
      }
    } else if (kind == kLoopGdn) {
      const GdnRecurrentArgs& a = op.gdn;
      std::uint32_t u = first_unit(c, op.rotation);
      float S[kGdnRows];
      // The state does not depend on this step: load it before the barrier.
      if (u < a.value_heads) gdn_load_state(a, u, t, S);
      const bool alive = i == 0 || grid_barrier(c, target, i);
      for (; u < a.value_heads; u += c.ctas) {
        if (alive) {
          gdn_recurrent_tokens(a, u, t, S, ComputeSync{}, scratch.gdn);
          gdn_store_state(a, u, t, S);
        }
        if (u + c.ctas < a.value_heads) gdn_load_state(a, u + c.ctas, t, S);
      }
    } else if (kind == kLoopAttention) {
      const bool alive = i == 0 || grid_barrier(c, target, i);
      if (alive) attention_units(L, c, op, scratch, &s_flag);
    } else if (kind == kLoopArgmax) {
      grid_barrier(c, target, i);
      if (c.cta == 0 && warp == 0) {
        float best = -__int_as_float(0x7f800000);
        std::uint32_t index = 0xffffffffu;
        for (std::uint32_t j = lane; j < c.ctas; j += 32u) {
          better(best, index, ld_cg(&L.control->argmax_value[j]), ld_cg(&L.control->argmax_index[j]));
        }
#pragma unroll
        for (unsigned offset = 16; offset != 0; offset >>= 1) {
          const float other_value = __shfl_xor_sync(0xffffffffu, best, offset);
          const std::uint32_t other_index = __shfl_xor_sync(0xffffffffu, index, offset);
          better(best, index, other_value, other_index);
        }
        if (lane == 0) {
          if (index >= L.vocab) index = 0;  // all NaN: the reference also returns 0
          L.selected[0] = index;
          L.tokens[0] = index;
          *L.position += 1u;
        }
      }
    }
  }
  if (c.cta == 0 && t == 0) L.control->epoch = base + (L.op_count - 1u) * c.ctas;
  if (t == 0) {
    trace_mark(c, L.op_count, 0);
    trace_mark(c, L.op_count, 1);
  }
}

using LoopKernel = void (*)(LoopLaunch);


LoopKernel select_kernel(int act_bits, std::uint32_t hidden) {
  const std::uint32_t iterations = hidden / 256u;
  if (hidden % 256u != 0) return nullptr;
#define GFXB_LOOP_CASE(IT)                                                              \
  if (iterations == IT) return act_bits == 8 ? token_loop_kernel<8, IT> : token_loop_kernel<4, IT>;
  GFXB_LOOP_CASE(4)
  GFXB_LOOP_CASE(8)
  GFXB_LOOP_CASE(16)
  GFXB_LOOP_CASE(20)
#undef GFXB_LOOP_CASE
  return nullptr;
}

std::uint32_t align_up(std::uint32_t value, std::uint32_t alignment) {
  return (value + alignment - 1u) / alignment * alignment;
}

}  // namespace

bool token_loop_supported_hidden(std::uint32_t hidden) { return select_kernel(4, hidden) != nullptr; }

int token_loop_grid(int device, std::uint32_t* ctas) {
  int sms = 0;
  const cudaError_t error = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
  if (error != cudaSuccess) {
    set_error_cuda(error, "SM count query failed");
    return GFXB_CUDA_ERROR;
  }
  *ctas = static_cast<std::uint32_t>(std::min<int>(sms, static_cast<int>(kLoopMaxCtas)));
  return GFXB_OK;
}

int plan_token_loop(LoopLaunch& L, std::uint32_t max_groups, std::uint32_t dots_half, int device) {
  if (max_groups == 0 || max_groups > kLoopMaxGroups) return fail(GFXB_UNSUPPORTED, "token kernel: K out of range");
  LoopKernel kernel = select_kernel(static_cast<int>(L.act_bits), L.hidden);
  if (kernel == nullptr) return fail(GFXB_UNSUPPORTED, "token kernel: unsupported hidden size");
  int optin = 0;
  cudaError_t error = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, device);
  if (error != cudaSuccess) {
    set_error_cuda(error, "shared-memory limit query failed");
    return GFXB_CUDA_ERROR;
  }
  cudaFuncAttributes attributes{};
  error = cudaFuncGetAttributes(&attributes, kernel);
  if (error != cudaSuccess) {
    set_error_cuda(error, "token kernel attribute query failed");
    return GFXB_CUDA_ERROR;
  }
  const std::uint32_t available =
      static_cast<std::uint32_t>(optin) - static_cast<std::uint32_t>(attributes.sharedSizeBytes) - 1024u;
  std::uint32_t offset = 0;
  L.act_offset = offset;
  offset = align_up(offset + max_groups * kGroup, 16);
  L.act_scales_offset = offset;
  offset = align_up(offset + max_groups * 2u, 16);
  L.act_sums_offset = offset;
  offset = align_up(offset + max_groups * 4u, 16);
  L.dots_offset = offset;
  L.dots_half = dots_half;
  offset = align_up(offset + 2u * dots_half * 4u, 128);
  L.scale_slot_bytes = align_up(max_groups * 32u, 128);
  L.scale_offset = offset;
  offset += kLoopScaleSlots * L.scale_slot_bytes;
  L.scale_bars_offset = offset;
  offset = align_up(offset + kLoopScaleSlots * 16u, 1024);
  if (offset >= available) return fail(GFXB_UNSUPPORTED, "token kernel: shared memory exhausted");
  L.slots = std::min<std::uint32_t>((available - offset) / (kLoopSlotBytes + 16u), 64u);
  if (L.slots < 4) return fail(GFXB_UNSUPPORTED, "token kernel: weight ring too small");
  L.ring_offset = offset;
  offset += L.slots * kLoopSlotBytes;
  L.bars_offset = offset;
  offset += L.slots * 16u;
  L.smem_bytes = offset;
  GFXB_TRY(token_loop_grid(device, &L.ctas));
  error = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(L.smem_bytes));
  if (error != cudaSuccess) {
    set_error_cuda(error, "token kernel shared-memory configuration failed");
    return GFXB_CUDA_ERROR;
  }
  int per_sm = 0;
  error = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, kLoopThreads, L.smem_bytes);
  if (error != cudaSuccess) {
    set_error_cuda(error, "token kernel occupancy query failed");
    return GFXB_CUDA_ERROR;
  }
  if (per_sm < 1) return fail(GFXB_UNSUPPORTED, "token kernel does not fit one CTA per SM");
  return GFXB_OK;
}

int launch_token_loop(const LoopLaunch& L, cudaStream_t stream) {
  LoopKernel kernel = select_kernel(static_cast<int>(L.act_bits), L.hidden);
  if (kernel == nullptr || L.ctas == 0 || L.smem_bytes == 0) return fail(GFXB_INTERNAL, "token kernel is not planned");
  cudaLaunchConfig_t config{};
  config.gridDim = dim3(L.ctas);
  config.blockDim = dim3(kLoopThreads);
  config.dynamicSmemBytes = L.smem_bytes;
  config.stream = stream;
  cudaLaunchAttribute attribute[1];
  attribute[0].id = cudaLaunchAttributeCooperative;
  attribute[0].val.cooperative = 1;
  config.attrs = attribute;
  config.numAttrs = 1;
  const cudaError_t error = cudaLaunchKernelEx(&config, kernel, L);
  if (error != cudaSuccess) {
    set_error_cuda(error, "token kernel launch failed");
    return GFXB_CUDA_ERROR;
  }
  return GFXB_OK;
}

}  // namespace gfxb
