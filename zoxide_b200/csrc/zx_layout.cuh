// zx_layout.cuh — operand layout passes that let the reference's own operand layouts run on the
// K-major tcgen05 kernels (HBM-bound byte work, no tensor cores).
//
//   - transpose_u8_kernel: B row-major K x N int8 (the reference's imma_s8 / imma_sp_s8 layout,
//     src/examples/imma_sp_s8.zig:144-187) -> N x K (K contiguous), the layout the 2:4 sparse
//     kernels read.
//   - s4_repack_kernel: B K x N signed int4 packed two per byte along N (imma_s4's layout,
//     src/examples/imma_s4.zig:89-101, low nibble = even n) -> N x K/2 packed along K (low
//     nibble = even k), the W4A8 kernels' weight layout.
//   - unpack_s4_kernel: A M x K signed int4 packed along K -> M x K int8 (sign-extended), the
//     W4A8 kernels' activation operand.
//   - sp48_a_kernel / sp48_b_kernel: imma_sp_s4's 4:8 pair-clustered s4 A with its metadata, and
//     its B K x N s4 packed along N (src/examples/imma_sp_s4.zig:153-196, examples_abi.zig:83-96)
//     -> the int8 2:4 operands of the sparse kernels, with k reordered inside every 8-wide chunk
//     (logical 2p + e -> position 4e + p, the same for A and B, so C is unchanged): in each group
//     of four positions exactly the reference's two kept sub-chunks p0 < p1 survive, and both
//     groups of a chunk carry the reference nibble p0 | p1 << 2 unchanged.
// Each kernel reads and writes every byte once with 16-byte (or 8-byte) coalesced accesses;
// tiles go through shared memory. Bounds are checked per access.
#pragma once
#include <cstdint>

namespace zx {

// rows x cols bytes -> cols x rows bytes; rows % 16 == 0, cols % 16 == 0, 16-byte aligned bases.
// 64 x 64 tiles, 256 threads: 16-byte row loads, 4 x 4 byte blocks transposed in registers with
// byte permutes, 16-byte row stores.
__global__ void __launch_bounds__(256) transpose_u8_kernel(const uint8_t* __restrict__ in, uint8_t* __restrict__ out,
                                                           uint32_t rows, uint32_t cols) {
  __shared__ uint32_t tile[64][17];  // [row][word of 4 columns], one word of padding
  __shared__ uint32_t tt[64][17];    // [column][word of 4 rows]
  const uint32_t r0 = blockIdx.y * 64u, c0 = blockIdx.x * 64u, t = threadIdx.x;
  {
    const uint32_t r = r0 + t / 4u, c = c0 + (t % 4u) * 16u;
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if (r < rows && c < cols) v = *reinterpret_cast<const uint4*>(in + static_cast<uint64_t>(r) * cols + c);
    uint32_t* w = &tile[t / 4u][(t % 4u) * 4u];
    w[0] = v.x;
    w[1] = v.y;
    w[2] = v.z;
    w[3] = v.w;
  }
  __syncthreads();
  {
    const uint32_t br = t / 16u, bc = t % 16u;  // rows 4 br .. +3, columns 4 bc .. +3
    const uint32_t w0 = tile[4u * br][bc], w1 = tile[4u * br + 1u][bc];
    const uint32_t w2 = tile[4u * br + 2u][bc], w3 = tile[4u * br + 3u][bc];
    const uint32_t a_lo = __byte_perm(w0, w1, 0x5140), a_hi = __byte_perm(w0, w1, 0x7362);
    const uint32_t b_lo = __byte_perm(w2, w3, 0x5140), b_hi = __byte_perm(w2, w3, 0x7362);
    tt[4u * bc][br] = __byte_perm(a_lo, b_lo, 0x5410);       // column 4 bc: rows 4 br .. +3
    tt[4u * bc + 1u][br] = __byte_perm(a_lo, b_lo, 0x7632);
    tt[4u * bc + 2u][br] = __byte_perm(a_hi, b_hi, 0x5410);
    tt[4u * bc + 3u][br] = __byte_perm(a_hi, b_hi, 0x7632);
  }
  __syncthreads();
  {
    const uint32_t oc = c0 + t / 4u, orow = r0 + (t % 4u) * 16u;
    if (oc < cols && orow < rows) {
      const uint32_t* w = &tt[t / 4u][(t % 4u) * 4u];
      *reinterpret_cast<uint4*>(out + static_cast<uint64_t>(oc) * rows + orow) = make_uint4(w[0], w[1], w[2], w[3]);
    }
  }
}

// B K x N s4 packed along N (K x N/2 bytes) -> N x K/2 bytes packed along K; K % 64 == 0,
// N % 16 == 0. 64 (k) x 64 (n) tiles: 8-byte loads of 16 nibbles, nibbles unpacked into a
// [k][n] byte tile, then each output byte packs k, k + 1 of one n.
__global__ void __launch_bounds__(256) s4_repack_kernel(const uint8_t* __restrict__ in, uint8_t* __restrict__ out,
                                                        uint32_t K, uint32_t N) {
  __shared__ uint8_t nib[64][64 + 4];
  const uint32_t k0 = blockIdx.y * 64u, n0 = blockIdx.x * 64u, t = threadIdx.x;
  {
    const uint32_t k = k0 + t / 4u, nb = n0 + (t % 4u) * 16u;  // 16 nibbles of row k from n = nb
    uint2 v = make_uint2(0u, 0u);
    if (k < K && nb < N) v = *reinterpret_cast<const uint2*>(in + static_cast<uint64_t>(k) * (N / 2u) + nb / 2u);
    uint8_t* dst = &nib[t / 4u][(t % 4u) * 16u];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const uint32_t byte = ((i < 4 ? v.x : v.y) >> (8 * (i & 3))) & 0xFFu;
      dst[2 * i] = static_cast<uint8_t>(byte & 0xFu);
      dst[2 * i + 1] = static_cast<uint8_t>(byte >> 4);
    }
  }
  __syncthreads();
  {
    const uint32_t n = n0 + t / 4u, kb = k0 + (t % 4u) * 16u;  // 16 k values of column n
    if (n < N && kb < K) {
      const uint32_t col = t / 4u, kr = (t % 4u) * 16u;
      uint32_t w[2] = {0u, 0u};
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const uint32_t byte = static_cast<uint32_t>(nib[kr + 2 * i][col]) | (static_cast<uint32_t>(nib[kr + 2 * i + 1][col]) << 4);
        w[i >> 2] |= byte << (8 * (i & 3));
      }
      *reinterpret_cast<uint2*>(out + static_cast<uint64_t>(n) * (K / 2u) + kb / 2u) = make_uint2(w[0], w[1]);
    }
  }
}

// A M x K s4 packed along K (M x K/2 bytes) -> M x K int8; `groups` = M * K / 16 groups of 8
// input bytes (16 values), K % 16 == 0.
__global__ void __launch_bounds__(256) unpack_s4_kernel(const uint8_t* __restrict__ in, int8_t* __restrict__ out,
                                                        uint64_t groups) {
  for (uint64_t g = blockIdx.x * 256ull + threadIdx.x; g < groups; g += static_cast<uint64_t>(gridDim.x) * 256ull) {
    const uint2 v = *reinterpret_cast<const uint2*>(in + g * 8u);
    uint32_t w[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t src = i < 2 ? v.x : v.y;
      const uint32_t b0 = (src >> (16 * (i & 1))) & 0xFFu, b1 = (src >> (16 * (i & 1) + 8)) & 0xFFu;
      // sign-extended nibbles: low nibble first (even index)
      const uint32_t e0 = static_cast<uint32_t>(static_cast<uint8_t>(static_cast<int8_t>(b0 << 4) >> 4));
      const uint32_t e1 = static_cast<uint32_t>(static_cast<uint8_t>(static_cast<int8_t>(b0 & 0xF0u) >> 4));
      const uint32_t e2 = static_cast<uint32_t>(static_cast<uint8_t>(static_cast<int8_t>(b1 << 4) >> 4));
      const uint32_t e3 = static_cast<uint32_t>(static_cast<uint8_t>(static_cast<int8_t>(b1 & 0xF0u) >> 4));
      w[i] = e0 | (e1 << 8) | (e2 << 16) | (e3 << 24);
    }
    *reinterpret_cast<uint4*>(out + g * 16u) = make_uint4(w[0], w[1], w[2], w[3]);
  }
}

// A: per row and 64 dense k, 16 bytes of 4:8 pair-clustered s4 (two packed bytes b0, b1 per 8-wide
// chunk j: the kept sub-chunks p0 < p1, low nibble = element 0) and one metadata word (nibble j =
// p0 | p1 << 2) -> 32 bytes of int8 2:4-compressed A (chunk j: lo(b0) lo(b1) hi(b0) hi(b1), the
// kept values of groups 2j and 2j + 1) and two int8 metadata words (one per 32 dense k; groups
// 2j and 2j + 1 both get nibble j). `units` = M * K / 64.
__global__ void __launch_bounds__(256) sp48_a_kernel(const uint8_t* __restrict__ a4, const uint32_t* __restrict__ meta4,
                                                     int8_t* __restrict__ a8, uint32_t* __restrict__ meta8,
                                                     uint64_t units) {
  for (uint64_t u = blockIdx.x * 256ull + threadIdx.x; u < units; u += static_cast<uint64_t>(gridDim.x) * 256ull) {
    const uint4 v = *reinterpret_cast<const uint4*>(a4 + u * 16u);
    const uint32_t in[4] = {v.x, v.y, v.z, v.w};
    uint32_t out[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const uint32_t b0 = (in[j >> 1] >> (16 * (j & 1))) & 0xFFu, b1 = (in[j >> 1] >> (16 * (j & 1) + 8)) & 0xFFu;
      const uint32_t l0 = static_cast<uint32_t>(static_cast<uint8_t>(static_cast<int8_t>(b0 << 4) >> 4));
      const uint32_t l1 = static_cast<uint32_t>(static_cast<uint8_t>(static_cast<int8_t>(b1 << 4) >> 4));
      const uint32_t h0 = static_cast<uint32_t>(static_cast<uint8_t>(static_cast<int8_t>(b0 & 0xF0u) >> 4));
      const uint32_t h1 = static_cast<uint32_t>(static_cast<uint8_t>(static_cast<int8_t>(b1 & 0xF0u) >> 4));
      out[j] = l0 | (l1 << 8) | (h0 << 16) | (h1 << 24);
    }
    uint4* dst = reinterpret_cast<uint4*>(a8 + u * 32u);
    dst[0] = make_uint4(out[0], out[1], out[2], out[3]);
    dst[1] = make_uint4(out[4], out[5], out[6], out[7]);
    const uint32_t w = meta4[u];
    uint32_t m[2] = {0u, 0u};
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const uint32_t nib = (w >> (4 * j)) & 0xFu;
      m[j >> 2] |= (nib | (nib << 4)) << (8 * (j & 3));
    }
    *reinterpret_cast<uint2*>(meta8 + 2u * u) = make_uint2(m[0], m[1]);
  }
}

// B K x N s4 packed along N (K x N/2 bytes) -> N x K int8 with k reordered inside every 8-wide
// chunk (position 4e + p of chunk c holds logical k = 8c + 2p + e); K % 64 == 0, N % 16 == 0.
// 64 (k) x 64 (n) tiles: 8-byte loads of 16 nibbles into a [k][n] tile, 16-byte stores of 16 k.
__global__ void __launch_bounds__(256) sp48_b_kernel(const uint8_t* __restrict__ in, int8_t* __restrict__ out,
                                                     uint32_t K, uint32_t N) {
  __shared__ uint8_t nib[64][64 + 4];
  const uint32_t k0 = blockIdx.y * 64u, n0 = blockIdx.x * 64u, t = threadIdx.x;
  {
    const uint32_t k = k0 + t / 4u, nb = n0 + (t % 4u) * 16u;  // 16 nibbles of row k from n = nb
    uint2 v = make_uint2(0u, 0u);
    if (k < K && nb < N) v = *reinterpret_cast<const uint2*>(in + static_cast<uint64_t>(k) * (N / 2u) + nb / 2u);
    uint8_t* dst = &nib[t / 4u][(t % 4u) * 16u];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const uint32_t byte = ((i < 4 ? v.x : v.y) >> (8 * (i & 3))) & 0xFFu;
      dst[2 * i] = static_cast<uint8_t>(byte & 0xFu);
      dst[2 * i + 1] = static_cast<uint8_t>(byte >> 4);
    }
  }
  __syncthreads();
  {
    const uint32_t n = n0 + t / 4u, kb = k0 + (t % 4u) * 16u;  // positions kb .. kb + 15 of row n
    if (n < N && kb < K) {
      const uint32_t col = t / 4u, kr = (t % 4u) * 16u;
      uint32_t w[4] = {0u, 0u, 0u, 0u};
#pragma unroll
      for (int q = 0; q < 16; ++q) {
        const uint32_t src = kr + 8u * (q >> 3) + 2u * (q & 3) + ((q >> 2) & 1);  // logical k of position q
        const uint32_t v = static_cast<uint32_t>(static_cast<uint8_t>(static_cast<int8_t>(nib[src][col] << 4) >> 4));
        w[q >> 2] |= v << (8 * (q & 3));
      }
      *reinterpret_cast<uint4*>(out + static_cast<uint64_t>(n) * K + kb) = make_uint4(w[0], w[1], w[2], w[3]);
    }
  }
}

}  // namespace zx
