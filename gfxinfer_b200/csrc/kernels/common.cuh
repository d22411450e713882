// Shared device helpers for the gfxinfer-b200 kernels (sm_100a).
//
// Numerics contract: this library is compiled with -fmad=false, -prec-div=true,
// -prec-sqrt=true and -ftz=false, so each float operation written here is one
// IEEE round-to-nearest-even operation. Fused multiply-adds appear only where
// written as fmaf(). Every reduction uses a fixed order, which lets the CPU
// oracle reproduce kernel outputs bit for bit.
#pragma once

#include <atomic>
#include <cstddef>
#include <cstdint>
#include <mutex>
#include <utility>

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "gfxb/gfxb.h"

namespace gfxb {

constexpr unsigned kGroup = 128;
constexpr unsigned kWarp = 32;

// ---- status plumbing ------------------------------------------------------

void set_error(const char* message);
void set_error_cuda(cudaError_t error, const char* context);
int fail(int status, const char* message);
int launch_status(const char* context);

#define GFXB_TRY(expression)                \
  do {                                      \
    const int status_ = (expression);       \
    if (status_ != GFXB_OK) return status_; \
  } while (0)

#define GFXB_REQUIRE(condition, message) \
  do {                                   \
    if (!(condition)) return ::gfxb::fail(GFXB_INVALID_ARGUMENT, message); \
  } while (0)

// ---- scalar conversions ---------------------------------------------------

__device__ __forceinline__ float h2f(__half value) { return __half2float(value); }
__device__ __forceinline__ __half f2h(float value) { return __float2half_rn(value); }
__device__ __forceinline__ float bf2f(std::uint16_t bits) {
  return __uint_as_float(static_cast<std::uint32_t>(bits) << 16);
}

// __float2int_rn: NaN -> 0, saturating, ties to even.
__device__ __forceinline__ int f2i_rn(float value) { return __float2int_rn(value); }

// ---- exp / log1p ----------------------------------------------------------
// e^x by Cody-Waite two-constant reduction x = n*ln2 + r (W. J. Cody and
// W. Waite, "Software Manual for the Elementary Functions", 1980), e^r by its
// degree-7 Taylor polynomial in Horner form, then exact scaling by 2^n.

__device__ __forceinline__ float pow2i(int k) {
  return __uint_as_float(static_cast<std::uint32_t>(k + 127) << 23);
}

__device__ __forceinline__ float gx_expf(float x) {
  if (x != x) return x;
  if (x > 88.7228394f) return __uint_as_float(0x7f800000u);
  if (x < -104.0f) return 0.0f;
  const float n = rintf(__fmul_rn(x, 1.44269502f));
  float r = fmaf(n, -0.693145751953125f, x);
  r = fmaf(n, -1.428606765330187e-6f, r);
  float p = 1.98412698e-4f;
  p = fmaf(p, r, 1.38888889e-3f);
  p = fmaf(p, r, 8.33333333e-3f);
  p = fmaf(p, r, 4.16666667e-2f);
  p = fmaf(p, r, 1.66666667e-1f);
  p = fmaf(p, r, 0.5f);
  p = fmaf(p, r, 1.0f);
  p = fmaf(p, r, 1.0f);
  const int e = static_cast<int>(n);
  if (e > 127) return __fmul_rn(__fmul_rn(p, pow2i(127)), pow2i(e - 127));
  if (e < -126) return __fmul_rn(__fmul_rn(p, pow2i(e + 64)), pow2i(-64));
  return __fmul_rn(p, pow2i(e));
}

// ln(u), u >= 1: u = m*2^e, m in [sqrt(1/2), sqrt(2)], ln(m) = 2*atanh(s),
// s = (m-1)/(m+1), odd series to s^11.
__device__ __forceinline__ float gx_log_ge1(float u) {
  const std::uint32_t bits = __float_as_uint(u);
  int e = static_cast<int>((bits >> 23) & 0xffu) - 127;
  float m = __uint_as_float((bits & 0x007fffffu) | 0x3f800000u);
  if (m > 1.41421356f) {
    m = __fmul_rn(m, 0.5f);
    e += 1;
  }
  const float s = __fdiv_rn(__fsub_rn(m, 1.0f), __fadd_rn(m, 1.0f));
  const float s2 = __fmul_rn(s, s);
  float p = 0.0909090909f;
  p = fmaf(p, s2, 0.111111111f);
  p = fmaf(p, s2, 0.142857143f);
  p = fmaf(p, s2, 0.2f);
  p = fmaf(p, s2, 0.333333333f);
  p = fmaf(p, s2, 1.0f);
  const float lm = __fmul_rn(__fmul_rn(2.0f, s), p);
  return fmaf(static_cast<float>(e), 0.693147181f, lm);
}

// log(1+x), x >= 0 (D. Goldberg 1991, Theorem 4).
__device__ __forceinline__ float gx_log1pf(float x) {
  if (x != x) return x;
  if (x == __uint_as_float(0x7f800000u)) return x;
  const float u = __fadd_rn(1.0f, x);
  if (u == 1.0f) return x;
  return __fmul_rn(gx_log_ge1(u), __fdiv_rn(x, __fsub_rn(u, 1.0f)));
}

__device__ __forceinline__ float gx_sigmoid(float x) {
  return __fdiv_rn(1.0f, __fadd_rn(1.0f, gx_expf(-x)));
}

__device__ __forceinline__ float gx_silu(float x) {
  return __fdiv_rn(x, __fadd_rn(1.0f, gx_expf(-x)));
}

// 1 / sqrt(x), both steps correctly rounded (stands in for rsqrtf so the CPU
// oracle can reproduce it).
__device__ __forceinline__ float inv_sqrt_rn(float x) {
  return __fdiv_rn(1.0f, __fsqrt_rn(x));
}

// ---- fixed-order reductions -----------------------------------------------

// Lane 0 receives the pairwise tree of the shuffle-down sequence 16, 8, 4, 2, 1.
__device__ __forceinline__ float warp_sum_down(float value) {
  value = __fadd_rn(value, __shfl_down_sync(0xffffffffu, value, 16));
  value = __fadd_rn(value, __shfl_down_sync(0xffffffffu, value, 8));
  value = __fadd_rn(value, __shfl_down_sync(0xffffffffu, value, 4));
  value = __fadd_rn(value, __shfl_down_sync(0xffffffffu, value, 2));
  value = __fadd_rn(value, __shfl_down_sync(0xffffffffu, value, 1));
  return value;
}

// Every lane receives the same pairwise tree (xor butterfly 16, 8, 4, 2, 1);
// identical to warp_sum_down's lane-0 value because float addition commutes.
__device__ __forceinline__ float warp_sum_xor(float value) {
  value = __fadd_rn(value, __shfl_xor_sync(0xffffffffu, value, 16));
  value = __fadd_rn(value, __shfl_xor_sync(0xffffffffu, value, 8));
  value = __fadd_rn(value, __shfl_xor_sync(0xffffffffu, value, 4));
  value = __fadd_rn(value, __shfl_xor_sync(0xffffffffu, value, 2));
  value = __fadd_rn(value, __shfl_xor_sync(0xffffffffu, value, 1));
  return value;
}

// Tree over up to eight per-warp sums padded with zeros to 32 lanes (the
// second stage of the reference's 256-thread block reduction).
__device__ __forceinline__ float tree_of_eight(const float* sums, unsigned count) {
  float a[8];
#pragma unroll
  for (unsigned i = 0; i < 8; ++i) a[i] = i < count ? sums[i] : 0.0f;
  // padding lanes 8..31 are zero: x + 0 == x, so only offsets 4, 2, 1 change values
#pragma unroll
  for (unsigned i = 0; i < 4; ++i) a[i] = __fadd_rn(a[i], a[i + 4]);
#pragma unroll
  for (unsigned i = 0; i < 2; ++i) a[i] = __fadd_rn(a[i], a[i + 2]);
  return __fadd_rn(a[0], a[1]);
}

// ---- streaming loads --------------------------------------------------------

__device__ __forceinline__ uint4 ldg_stream16(const void* pointer) {
  uint4 value;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(value.x), "=r"(value.y), "=r"(value.z), "=r"(value.w)
               : "l"(pointer));
  return value;
}

__device__ __forceinline__ uint2 ldg_stream8(const void* pointer) {
  uint2 value;
  asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];"
               : "=r"(value.x), "=r"(value.y)
               : "l"(pointer));
  return value;
}

__device__ __forceinline__ void mma_s8_16832(int (&c)[4], const std::uint32_t (&a)[4],
                                             std::uint32_t b0, std::uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// The same mma with a zero accumulator input (no register clearing).
__device__ __forceinline__ void mma_s8_16832_zero(int (&d)[4], const std::uint32_t (&a)[4], std::uint32_t b0,
                                                  std::uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%10,%10,%10,%10};"
      : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "r"(0));
}

inline cudaStream_t as_stream(void* stream) { return static_cast<cudaStream_t>(stream); }

// ---- per-device set-up -------------------------------------------------------
// cudaFuncSetAttribute and occupancy answers belong to the device that is
// current when they are made, so launchers keep them per device. Thread-safe:
// the first caller on a device runs the set-up under a lock, later callers
// only read an atomic flag.

constexpr int kMaxDevices = 64;

// The current device, checked against kMaxDevices.
int current_device(int* device);

class DeviceOnce {
 public:
  // Runs configure(device) once for the current device; a failed set-up is
  // retried by the next call.
  template <typename Configure>
  int run(Configure&& configure) {
    int device = 0;
    const int status = current_device(&device);
    if (status != GFXB_OK) return status;
    if (done_[device].load(std::memory_order_acquire) != 0) return GFXB_OK;
    std::lock_guard<std::mutex> lock(mutex_);
    if (done_[device].load(std::memory_order_relaxed) != 0) return GFXB_OK;
    const int result = configure(device);
    if (result == GFXB_OK) done_[device].store(1, std::memory_order_release);
    return result;
  }

 private:
  std::mutex mutex_;
  std::atomic<std::uint8_t> done_[kMaxDevices] = {};
};

// The current device's SM count (queried once per device).
int device_sm_count(int* sms);

// ---- programmatic dependent launch -------------------------------------------
// Every kernel of the decode chain lets its successor launch early
// (pdl_trigger) and waits for its predecessor's completion and memory
// (pdl_wait) before it reads a predecessor's output or writes any global
// memory. Work that depends on neither (weight prefetch) goes in between.

__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

bool pdl_enabled();

template <typename... KernelArgs, typename... Args>
cudaError_t launch_kernel(void (*kernel)(KernelArgs...), dim3 grid, dim3 block, std::size_t shared_bytes,
                          cudaStream_t stream, unsigned cluster, Args&&... args) {
  cudaLaunchConfig_t config{};
  config.gridDim = grid;
  config.blockDim = block;
  config.dynamicSmemBytes = shared_bytes;
  config.stream = stream;
  cudaLaunchAttribute attributes[2];
  unsigned count = 0;
  if (pdl_enabled()) {
    attributes[count].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attributes[count].val.programmaticStreamSerializationAllowed = 1;
    ++count;
  }
  if (cluster > 0) {
    attributes[count].id = cudaLaunchAttributeClusterDimension;
    attributes[count].val.clusterDim.x = cluster;
    attributes[count].val.clusterDim.y = 1;
    attributes[count].val.clusterDim.z = 1;
    ++count;
  }
  config.attrs = attributes;
  config.numAttrs = count;
  return cudaLaunchKernelEx(&config, kernel, std::forward<Args>(args)...);
}

// ---- shared-memory staging: mbarriers, bulk copies, clusters ---------------

constexpr std::uint32_t kSuspendHintNs = 20000;

__device__ __forceinline__ std::uint32_t smem_addr(const void* pointer) {
  return static_cast<std::uint32_t>(__cvta_generic_to_shared(pointer));
}

__device__ __forceinline__ void mbar_init(std::uint64_t* bar, std::uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}

// 16-byte asynchronous global -> shared copy (L2 only), 16-byte aligned addresses.
__device__ __forceinline__ void cp_async_16(void* shared_dst, const void* global_src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(shared_dst)), "l"(global_src) : "memory");
}

__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }

// Wait until at most N of this thread's committed cp.async groups are pending.
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// The mbarrier counts one arrival of this thread once all of its earlier
// cp.async copies have landed (the barrier is initialised with one expected
// arrival per thread).
__device__ __forceinline__ void cp_async_arrive_noinc(std::uint64_t* bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_expect_tx(std::uint64_t* bar, std::uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
               : "memory");
}

// Global -> this CTA's shared memory, completion counted on `bar` (no multicast).
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, std::uint32_t bytes, std::uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}

// The waiting thread is suspended in hardware until the phase completes or
// the hint (ns) expires, so waiting warps do not compete for issue slots.
__device__ __forceinline__ bool mbar_try_wait(std::uint64_t* bar, std::uint32_t parity) {
  std::uint32_t done;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n selp.u32 %0, 1, 0, p;\n}"
      : "=r"(done)
      : "r"(smem_addr(bar)), "r"(parity), "r"(kSuspendHintNs)
      : "memory");
  return done != 0;
}

// Non-blocking test of a phase (test_wait never suspends the thread). For
// phases completed by other threads' arrivals, local or remote, whose waiters
// are not reliably woken before a suspension expires.
__device__ __forceinline__ bool mbar_poll(std::uint64_t* bar, std::uint32_t parity) {
  std::uint32_t done;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
      : "=r"(done)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return done != 0;
}

__device__ __forceinline__ bool mbar_poll_cluster(std::uint64_t* bar, std::uint32_t parity) {
  std::uint32_t done;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.test_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}"
      : "=r"(done)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return done != 0;
}

// Every wait is bounded: on expiry the kernel records kDeviceErrorTimeout in
// `error` (when given) and the caller skips the work instead of hanging.
constexpr std::uint32_t kDeviceErrorTimeout = 1u;
constexpr std::uint32_t kWaitLimit = 1u << 16;

__device__ __forceinline__ bool mbar_wait_bounded(std::uint64_t* bar, std::uint32_t parity,
                                                  std::uint32_t* error) {
  for (std::uint32_t i = 0; i < kWaitLimit; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
  }
  if (error != nullptr) atomicOr(error, kDeviceErrorTimeout);
  return false;
}

constexpr std::uint32_t kPollLimit = 1u << 26;

__device__ __forceinline__ bool mbar_poll_bounded(std::uint64_t* bar, std::uint32_t parity, std::uint32_t* error,
                                                  bool cluster_scope = false) {
  for (std::uint32_t i = 0; i < kPollLimit; ++i) {
    if (cluster_scope ? mbar_poll_cluster(bar, parity) : mbar_poll(bar, parity)) return true;
  }
  if (error != nullptr) atomicOr(error, kDeviceErrorTimeout);
  return false;
}

// Whole-warp bounded wait (every lane calls it): the answer is the same in all
// lanes, so a warp that gives up leaves its loop together.
enum class WaitKind { kSuspend, kPoll, kPollCluster };

template <WaitKind Kind>
__device__ __forceinline__ bool warp_wait_bounded(std::uint64_t* bar, std::uint32_t parity, std::uint32_t* error) {
  const std::uint32_t limit = Kind == WaitKind::kSuspend ? kWaitLimit : kPollLimit;
  for (std::uint32_t i = 0; i < limit; ++i) {
    const bool done = Kind == WaitKind::kSuspend ? mbar_try_wait(bar, parity)
                      : Kind == WaitKind::kPoll  ? mbar_poll(bar, parity)
                                                 : mbar_poll_cluster(bar, parity);
    if (__all_sync(0xffffffffu, done)) return true;
  }
  if (error != nullptr && (threadIdx.x & 31u) == 0) atomicOr(error, kDeviceErrorTimeout);
  return false;
}

__device__ __forceinline__ std::uint32_t cluster_ctarank() {
  std::uint32_t rank;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(rank));
  return rank;
}

__device__ __forceinline__ std::uint32_t cluster_nctarank() {
  std::uint32_t count;
  asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(count));
  return count;
}

__device__ __forceinline__ std::uint32_t dynamic_smem_bytes() {
  std::uint32_t bytes;
  asm volatile("mov.u32 %0, %%dynamic_smem_size;" : "=r"(bytes));
  return bytes;
}

__device__ __forceinline__ std::uint32_t map_shared_rank(std::uint32_t address, std::uint32_t rank) {
  std::uint32_t mapped;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(mapped) : "r"(address), "r"(rank));
  return mapped;
}

__device__ __forceinline__ void st_cluster_s32(std::uint32_t address, int value) {
  asm volatile("st.shared::cluster.s32 [%0], %1;" ::"r"(address), "r"(value) : "memory");
}

// Asynchronous 4-byte store into a cluster peer's shared memory whose arrival
// is counted (4 transaction bytes) on the peer's mbarrier `remote_bar`.
__device__ __forceinline__ void st_async_s32(std::uint32_t address, int value, std::uint32_t remote_bar) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.s32 [%0], %1, [%2];" ::"r"(address),
               "r"(value), "r"(remote_bar)
               : "memory");
}

// Plain arrival on this CTA's mbarrier (release at CTA scope).
__device__ __forceinline__ void mbar_arrive(std::uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

// Arrival on a cluster peer's mbarrier (address from map_shared_rank).
__device__ __forceinline__ void mbar_arrive_remote(std::uint32_t remote_bar) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(remote_bar) : "memory");
}

// Order this thread's earlier generic-proxy shared-memory accesses before its
// later asynchronous-proxy (bulk copy) writes to the same memory.
__device__ __forceinline__ void fence_proxy_async_shared() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Named barrier over `threads` threads (a multiple of 32) of this CTA.
__device__ __forceinline__ void named_barrier(std::uint32_t id, std::uint32_t threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

__device__ __forceinline__ bool mbar_wait_cluster_bounded(std::uint64_t* bar, std::uint32_t parity,
                                                          std::uint32_t* error);

// Wait for a phase completed by peers' st.async (cluster-scope acquire).
__device__ __forceinline__ bool mbar_try_wait_cluster(std::uint64_t* bar, std::uint32_t parity) {
  std::uint32_t done;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2, %3;\n"
      " selp.u32 %0, 1, 0, p;\n}"
      : "=r"(done)
      : "r"(smem_addr(bar)), "r"(parity), "r"(kSuspendHintNs)
      : "memory");
  return done != 0;
}

__device__ __forceinline__ bool mbar_wait_cluster_bounded(std::uint64_t* bar, std::uint32_t parity,
                                                          std::uint32_t* error) {
  for (std::uint32_t i = 0; i < kWaitLimit; ++i) {
    if (mbar_try_wait_cluster(bar, parity)) return true;
  }
  if (error != nullptr) atomicOr(error, kDeviceErrorTimeout);
  return false;
}

// Split cluster barrier. A CTA must not touch another CTA's shared memory
// before a cluster barrier has shown that every CTA of the cluster is running.
__device__ __forceinline__ void cluster_arrive() {
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
// Arrive without ordering memory: enough when the only thing the peers must
// see is an mbarrier initialised before a fence.mbarrier_init.
__device__ __forceinline__ void cluster_arrive_relaxed() {
  asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() {
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

}  // namespace gfxb
