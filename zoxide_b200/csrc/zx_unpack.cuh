// zx_unpack.cuh — s4 -> s8 weight unpacking in shared memory (W4A8 path).
//
// Storage convention (the reference's packS4, src/examples_abi.zig:54-56, applied along K as
// BASELINE config 3 asks): byte i of a weight row holds k = 2i in its low nibble and k = 2i + 1 in
// its high nibble, each a 4-bit two's-complement value; s4At (src/bench.zig:753-759) reads it back.
#pragma once
#include <cstdint>

#include "zx_ptx.cuh"

namespace zx {

// Four bytes each holding a value in [0, 15] -> the same bytes sign-extended from bit 3:
// v | 0xF0 where bit 3 is set (v - 16 mod 256), v otherwise. No carries cross bytes.
__device__ __forceinline__ uint32_t sext4x4(uint32_t v) {
  return v | (((v & 0x08080808u) >> 3) * 0xF0u);
}

// 8 packed s4 (one little-endian word, k = 0..7 low nibble first) -> 8 s8 bytes in k order.
__device__ __forceinline__ void unpack8(uint32_t w, uint32_t& o0, uint32_t& o1) {
  const uint32_t lo = sext4x4(w & 0x0F0F0F0Fu);         // k0 k2 k4 k6
  const uint32_t hi = sext4x4((w >> 4) & 0x0F0F0F0Fu);  // k1 k3 k5 k7
  o0 = __byte_perm(lo, hi, 0x5140);                     // k0 k1 k2 k3
  o1 = __byte_perm(lo, hi, 0x7362);                     // k4 k5 k6 k7
}

__device__ __forceinline__ void ld_shared_v4(uint32_t addr, uint32_t& a, uint32_t& b, uint32_t& c,
                                             uint32_t& d) {
  asm volatile("ld.shared.v4.b32 {%0,%1,%2,%3}, [%4];"
               : "=r"(a), "=r"(b), "=r"(c), "=r"(d)
               : "r"(addr)
               : "memory");
}

// One stage: `rows` x 64 packed bytes (row-major, no swizzle: 128 k values per row) at `src`
// -> rows x 128 int8 bytes in the tcgen05 K-major 128B-swizzle layout at `dst` (16-byte chunk c
// of row r at (c ^ (r & 7))), the layout TMA would have written for an int8 tile.
// Executed by `nthreads` threads with ids tid in [0, nthreads); each takes (row, 16-byte packed
// chunk) units u = tid, tid + nthreads, ...: a warp reads 512 contiguous bytes (row u >> 2,
// chunk u & 3 sits at byte 16 u) and its 8-thread store phases hit 8 distinct 16-byte bank groups.
template <int kRows, int kThreads>
__device__ __forceinline__ void unpack_s4_stage(uint32_t src, uint32_t dst, uint32_t tid) {
  constexpr int kUnits = kRows * 4 / kThreads;
  // all shared loads first (issued back to back), then the arithmetic, then the stores
  uint32_t w[kUnits][4];
#pragma unroll
  for (int i = 0; i < kUnits; ++i)
    ld_shared_v4(src + (tid + i * kThreads) * 16u, w[i][0], w[i][1], w[i][2], w[i][3]);
#pragma unroll
  for (int i = 0; i < kUnits; ++i) {
    const uint32_t u = tid + i * kThreads;
    const uint32_t row = u >> 2, cp = u & 3u;
    uint32_t o[8];
#pragma unroll
    for (int j = 0; j < 4; ++j) unpack8(w[i][j], o[2 * j], o[2 * j + 1]);
    const uint32_t rbase = dst + row * 128u;
    const uint32_t sw = row & 7u;
    st_shared_v4(rbase + (((2u * cp) ^ sw) << 4), o[0], o[1], o[2], o[3]);
    st_shared_v4(rbase + (((2u * cp + 1u) ^ sw) << 4), o[4], o[5], o[6], o[7]);
  }
}

}  // namespace zx
