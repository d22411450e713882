// Weight codec of the b200 GEMV layout: unsigned code offsets per format and
// the in-register unpacking of one lane's words into int8 tensor-core A
// fragments. Shared by the standalone GEMV kernels (gemv.cu) and the
// persistent token kernel (token_loop.cu).
#pragma once

#include "common.cuh"

namespace gfxb {

constexpr std::uint32_t kM7 = 0x07070707u;
constexpr std::uint32_t kM3 = 0x03030303u;
constexpr std::uint32_t kM4 = 0x04040404u;
constexpr std::uint32_t kM15 = 0x0f0f0f0fu;

template <int Bits>
struct Codec;

template <>
struct Codec<2> {
  static constexpr int alpha = 2, beta = -3;
};
template <>
struct Codec<3> {
  static constexpr int alpha = 1, beta = -4;
};
template <>
struct Codec<4> {
  static constexpr int alpha = 1, beta = -8;
};

__host__ __device__ constexpr int bits_of(int format) {
  return format == GFXB_W2 ? 2 : (format == GFXB_W3 ? 3 : 4);
}

// ---------------------------------------------------------------------------
// b200 layout. For lane L (g = L/4, t = L%4) the tensor-core A fragment of
// k-step s (0..3) holds registers q = 0..3, byte j = 0..3, covering
//   row = g + 8*(q & 1),  k = 32*s + 16*(q >> 1) + 4*t + j.
// ---------------------------------------------------------------------------

template <int Bits>
struct LaneWords;

template <>
struct LaneWords<3> {
  uint4 p0;  // block + 16*L        : words w0..w3
  uint2 p1;  // block + 512 + 8*L   : words w4..w5
};
template <>
struct LaneWords<4> {
  uint4 p0;  // block + 16*L
  uint4 p1;  // block + 512 + 16*L
};
template <>
struct LaneWords<2> {
  uint4 p0;  // block + 16*L
};

__device__ __forceinline__ void load_lane(const std::uint8_t* block, unsigned lane, LaneWords<3>& w) {
  w.p0 = ldg_stream16(block + 16u * lane);
  w.p1 = ldg_stream8(block + 512u + 8u * lane);
}
__device__ __forceinline__ void load_lane(const std::uint8_t* block, unsigned lane, LaneWords<4>& w) {
  w.p0 = ldg_stream16(block + 16u * lane);
  w.p1 = ldg_stream16(block + 512u + 16u * lane);
}
__device__ __forceinline__ void load_lane(const std::uint8_t* block, unsigned lane, LaneWords<2>& w) {
  w.p0 = ldg_stream16(block + 16u * lane);
}

// W3: a word triple (x0, x1, x2) carries the 32 codes of k-steps (sa, sb):
// six registers from 3-bit fields at bits 0-2 / 3-5 of each byte, two more
// assembled from the spare bits 6-7 (low bits) and x2's bits 6 / 7 (high bit).
__device__ __forceinline__ void unpack_w3_triple(std::uint32_t x0, std::uint32_t x1, std::uint32_t x2,
                                                 std::uint32_t (&ra)[4], std::uint32_t (&rb)[4]) {
  ra[0] = x0 & kM7;
  ra[1] = (x0 >> 3) & kM7;
  ra[2] = x1 & kM7;
  ra[3] = (x1 >> 3) & kM7;
  rb[0] = x2 & kM7;
  rb[1] = (x2 >> 3) & kM7;
  rb[2] = ((x0 >> 6) & kM3) | ((x2 >> 4) & kM4);
  rb[3] = ((x1 >> 6) & kM3) | ((x2 >> 5) & kM4);
}

__device__ __forceinline__ void unpack(const LaneWords<3>& w, std::uint32_t (&a)[4][4]) {
  unpack_w3_triple(w.p0.x, w.p0.y, w.p0.z, a[0], a[1]);
  unpack_w3_triple(w.p0.w, w.p1.x, w.p1.y, a[2], a[3]);
}

__device__ __forceinline__ void unpack_w4_pair(std::uint32_t lo, std::uint32_t hi, std::uint32_t (&r)[4]) {
  r[0] = lo & kM15;
  r[1] = (lo >> 4) & kM15;
  r[2] = hi & kM15;
  r[3] = (hi >> 4) & kM15;
}

__device__ __forceinline__ void unpack(const LaneWords<4>& w, std::uint32_t (&a)[4][4]) {
  unpack_w4_pair(w.p0.x, w.p0.y, a[0]);
  unpack_w4_pair(w.p0.z, w.p0.w, a[1]);
  unpack_w4_pair(w.p1.x, w.p1.y, a[2]);
  unpack_w4_pair(w.p1.z, w.p1.w, a[3]);
}

__device__ __forceinline__ void unpack_w2_word(std::uint32_t x, std::uint32_t (&r)[4]) {
  r[0] = x & kM3;
  r[1] = (x >> 2) & kM3;
  r[2] = (x >> 4) & kM3;
  r[3] = (x >> 6) & kM3;
}

__device__ __forceinline__ void unpack(const LaneWords<2>& w, std::uint32_t (&a)[4][4]) {
  unpack_w2_word(w.p0.x, a[0]);
  unpack_w2_word(w.p0.y, a[1]);
  unpack_w2_word(w.p0.z, a[2]);
  unpack_w2_word(w.p0.w, a[3]);
}

// Same lane words staged in shared memory.
template <int Bits>
__device__ __forceinline__ void load_lane_shared(const std::uint8_t* block, unsigned lane, LaneWords<Bits>& w) {
  if constexpr (Bits == 3) {
    w.p0 = *reinterpret_cast<const uint4*>(block + 16u * lane);
    w.p1 = *reinterpret_cast<const uint2*>(block + 512u + 8u * lane);
  } else if constexpr (Bits == 4) {
    w.p0 = *reinterpret_cast<const uint4*>(block + 16u * lane);
    w.p1 = *reinterpret_cast<const uint4*>(block + 512u + 16u * lane);
  } else {
    w.p0 = *reinterpret_cast<const uint4*>(block + 16u * lane);
  }
}

}  // namespace gfxb
