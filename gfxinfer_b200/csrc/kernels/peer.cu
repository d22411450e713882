// One-shot all-reduce of a row-parallel partial over NVLink peer memory,
// replacing the NCCL all-reduce after each row-parallel projection (o_proj,
// GDN out_proj, MLP down, the MTP fc) for tensor parallelism on one node.
//
// Every rank owns an exchange buffer that every other rank has mapped (CUDA
// IPC): data slots [2 parities][ranks][slot_floats] fp32, then flags
// [ranks][kPeerCtas] u32. CTA c of call k (its own counter, identical on all
// ranks because every rank makes the same calls) pushes its slice of the
// partial into slot [k & 1][rank] of every rank, then raises flag
// [rank][c] = k on every peer with a system-scope release; it waits (bounded)
// for flag [p][c] >= k from every peer with a system-scope acquire, and sums
// the slice's slots in rank order, so every rank computes the same bits. Two
// parities suffice: a rank can only start call k + 2 after every peer has
// raised its flag for call k + 1, i.e. has finished reading call k.
#include <cstdint>

#include "common.cuh"
#include "peer.cuh"

namespace gfxb {
namespace {

__device__ std::uint32_t g_peer_error;

__device__ __forceinline__ std::uint32_t ld_acquire_sys(const std::uint32_t* p) {
  std::uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys(std::uint32_t* p, std::uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

constexpr std::uint32_t kPeerWaitLimit = 1u << 22;  // polls of ~100 ns: about half a second

__global__ __launch_bounds__(256) void peer_all_reduce_kernel(PeerReduceArgs args) {
  pdl_trigger();
  pdl_wait();
  __shared__ std::uint32_t epoch_shared;
  const std::uint32_t cta = blockIdx.x;
  if (threadIdx.x == 0) {
    const std::uint32_t epoch = args.epochs[cta] + 1u;
    args.epochs[cta] = epoch;
    epoch_shared = epoch;
  }
  __syncthreads();
  const std::uint32_t epoch = epoch_shared;
  const std::uint32_t parity = epoch & 1u;
  // this CTA's slice, in float4 units
  const std::uint32_t vectors = args.count / 4u;
  const std::uint32_t per = (vectors + gridDim.x - 1u) / gridDim.x;
  const std::uint32_t begin = min(vectors, cta * per), end = min(vectors, begin + per);
  const std::size_t slot_bytes = static_cast<std::size_t>(args.slot_floats) * 4u;
  auto slot = [&](std::uint32_t owner, std::uint32_t source) {
    return reinterpret_cast<float4*>(args.buffers[owner] + (static_cast<std::size_t>(parity) * args.ranks + source) *
                                                               slot_bytes);
  };
  auto flags = [&](std::uint32_t owner) {
    return reinterpret_cast<std::uint32_t*>(args.buffers[owner] + 2u * args.ranks * slot_bytes);
  };
  const float4* data = reinterpret_cast<const float4*>(args.data);
  for (std::uint32_t p = 0; p < args.ranks; ++p) {
    float4* dst = slot(p, args.rank);
    for (std::uint32_t i = begin + threadIdx.x; i < end; i += blockDim.x) dst[i] = data[i];
  }
  __syncthreads();
  if (threadIdx.x < args.ranks && threadIdx.x != args.rank) {
    __threadfence_system();
    st_release_sys(flags(threadIdx.x) + args.rank * kPeerCtas + cta, epoch);
  }
  if (threadIdx.x < args.ranks && threadIdx.x != args.rank) {
    const std::uint32_t* flag = flags(args.rank) + threadIdx.x * kPeerCtas + cta;
    std::uint32_t polls = 0;
    while (ld_acquire_sys(flag) < epoch) {
      if (++polls == kPeerWaitLimit) {
        atomicOr(&g_peer_error, kDeviceErrorTimeout);
        break;
      }
      __nanosleep(100);
    }
  }
  __syncthreads();
  float4* out = reinterpret_cast<float4*>(args.data);
  for (std::uint32_t i = begin + threadIdx.x; i < end; i += blockDim.x) {
    float4 acc = slot(args.rank, 0)[i];
    for (std::uint32_t r = 1; r < args.ranks; ++r) {
      const float4 v = slot(args.rank, r)[i];
      acc.x = __fadd_rn(acc.x, v.x);
      acc.y = __fadd_rn(acc.y, v.y);
      acc.z = __fadd_rn(acc.z, v.z);
      acc.w = __fadd_rn(acc.w, v.w);
    }
    out[i] = acc;
  }
}

}  // namespace

std::size_t peer_exchange_bytes(std::uint32_t ranks, std::uint32_t slot_floats) {
  return 2u * ranks * static_cast<std::size_t>(slot_floats) * 4u + static_cast<std::size_t>(ranks) * kPeerCtas * 4u;
}

int launch_peer_all_reduce(const PeerReduceArgs& args, cudaStream_t stream) {
  if (args.data == nullptr || args.epochs == nullptr || args.ranks < 2 || args.ranks > 8 || args.rank >= args.ranks ||
      args.count == 0 || args.count % 4u != 0 || args.count > args.slot_floats || args.slot_floats % 4u != 0) {
    return fail(GFXB_INVALID_ARGUMENT, "invalid peer all-reduce arguments");
  }
  for (std::uint32_t r = 0; r < args.ranks; ++r) {
    if (args.buffers[r] == nullptr) return fail(GFXB_INVALID_ARGUMENT, "peer exchange buffer is not mapped");
  }
  launch_kernel(peer_all_reduce_kernel, dim3(kPeerCtas), dim3(256), 0, stream, 0, args);
  return launch_status("peer all-reduce launch failed");
}

// Reads and clears the peer all-reduce's error word (kDeviceErrorTimeout: a
// peer's flag never came).
int read_peer_errors(std::uint32_t* value) {
  cudaError_t error = cudaMemcpyFromSymbol(value, g_peer_error, sizeof(std::uint32_t));
  const std::uint32_t zero = 0;
  if (error == cudaSuccess) error = cudaMemcpyToSymbol(g_peer_error, &zero, sizeof(std::uint32_t));
  if (error != cudaSuccess) {
    set_error_cuda(error, "peer error word access failed");
    return GFXB_CUDA_ERROR;
  }
  return GFXB_OK;
}

}  // namespace gfxb
