// One-shot peer all-reduce over NVLink (see peer.cu).
#pragma once

#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

namespace gfxb {

constexpr std::uint32_t kPeerCtas = 16;  // slices of one call, one CTA each

struct PeerReduceArgs {
  float* data = nullptr;                 // [count] this rank's partial in, the sum over ranks out
  std::uint32_t count = 0;               // multiple of 4, <= slot_floats
  std::uint32_t rank = 0, ranks = 0;
  std::uint8_t* buffers[8] = {};         // every rank's exchange buffer as mapped here (own one included)
  std::uint32_t* epochs = nullptr;       // [kPeerCtas] this rank's call counters (zero at start)
  std::uint32_t slot_floats = 0;         // floats per (parity, source) slot
};

std::size_t peer_exchange_bytes(std::uint32_t ranks, std::uint32_t slot_floats);
int launch_peer_all_reduce(const PeerReduceArgs& args, cudaStream_t stream);
int read_peer_errors(std::uint32_t* value);

}  // namespace gfxb
