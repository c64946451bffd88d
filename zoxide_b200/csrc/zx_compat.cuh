// zx_compat.cuh — kernels that keep the reference's own launch contract, so they drop into the
// reference's module/launch flow unchanged (src/host.zig:342-349 Module.kernel, :498-565
// Kernel.launchOn; src/cuda_driver.zig:820-845 cuLaunchKernel). Entry names are the reference's
// `<stem>_$_<decl>` symbols (src/host.zig:100-123) and parameter lists its examples_abi.zig
// signatures; every one is launched with block 128, no dynamic shared memory and no cluster:
//
//   imma_s8_$_immaS8(a: *const i8, b: *const i8, c: *i32, n)             examples_abi.zig:42
//       grid (n/128, n/128) (src/bench.zig:671-682). A, B, C n x n row-major (B is K x N).
//   imma_s4_$_immaS4(a: *const u8, b: *const u8, c: *i32, n)             examples_abi.zig:44-56
//       grid (n/128, n/128). A packed two s4 per byte along K, B (K x N) packed along N.
//   imma_sp_s8_$_immaSpS8(a: *const i8, b: *const i8, meta: *const u32, c: *i32, n)
//       examples_abi.zig:71-81; grid (n/128, n/128). A 2:4-compressed (n/2 per row), meta one
//       word per row per 32 dense k, B dense K x N.
//   imma_sp_s4_$_immaSpS4(a: *const u8, b: *const u8, meta: *const u32, c: *i32, n)
//       examples_abi.zig:83-96; grid (n/128, n/128). A 4:8 pair-clustered (n/4 bytes per row),
//       meta one word per row per 64 dense k, B dense K x N packed along N.
//   hgemm_bf16_$_hgemmBf16 / hgemm_wgmma_bf16_$_hgemmWgmmaBf16(a: *const u16, b: *const u16,
//       c: *f32, n)  examples_abi.zig:33-36; grid (n/128, n/128) resp. (n/128, n/64)
//       (src/bench.zig:77-78 tile choice, :589-600).
//   hgemm_tma_$_hgemmTma(a: *const f16, b: *const f16, c: *f32, n, desc_a: u64, desc_b: u64)
//       examples_abi.zig:168-190; grid (n/128, n/64). The descriptors (reference-built tensor
//       maps of the same A and B) are accepted and not dereferenced: the tiles are read through
//       a and b, which the reference binds to the same buffers (src/bench.zig:1475-1512).
//
// Under that contract there is no tensor-map argument to use and no room for warp
// specialisation, so each CTA copies its operand tiles with cp.async into the tcgen05 shared-
// memory layouts itself, double-buffered in static shared memory (<= 40 KB); thread 0 issues
// tcgen05.mma (M = 128, cta_group::1) and the four warps drain TMEM. s4 operands land in a
// staging buffer and are unpacked to s8 by all 128 threads. These are slower by construction
// than the zx_gemm_* paths; they exist to be a literal drop-in for the reference's cubin
// loader. Every wait is bounded; a wait that gives up records its site in g_status and the
// whole CTA leaves the K loop together.
//
// 4:8 pair-clustered s4 on the int8 2:4 sparse MMA (imma_sp_s4). Blackwell has no s4 MMA kind.
// Within each 8-wide dense k chunk the reference keeps two of four 2-wide sub-chunks p0 < p1
// (metadata nibble p0 | p1 << 2). Reordering k inside every chunk, logical 2p + e -> position
// 4e + p, turns that into plain 2:4: positions 0..3 hold element 0 of sub-chunks 0..3, positions
// 4..7 element 1, and in each group of four exactly p0 and p1 survive, so both groups carry the
// reference nibble unchanged. A GEMM sums over k, so applying the same reorder to B's k rows
// leaves C unchanged. The compressed row per chunk is therefore [lo(b0), lo(b1), hi(b0), hi(b1)]
// for the two kept bytes b0, b1 (packS4: low nibble = element 0), and each reference word
// (8 chunks) expands to two int8 metadata words with every nibble doubled.
#pragma once
#include "zx_ptx.cuh"
#include "zx_unpack.cuh"

namespace zx {

__device__ __forceinline__ void cp_async_16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_8(uint32_t dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void st_shared_v2(uint32_t addr, uint32_t a, uint32_t b) {
  asm volatile("st.shared.v2.b32 [%0], {%1, %2};" ::"r"(addr), "r"(a), "r"(b) : "memory");
}
__device__ __forceinline__ void ld_shared_v2(uint32_t addr, uint32_t& a, uint32_t& b) {
  asm volatile("ld.shared.v2.b32 {%0, %1}, [%2];" : "=r"(a), "=r"(b) : "r"(addr) : "memory");
}

// Matrix descriptor with an explicit layout type (0 none, 2 = 128B swizzle, 4 = 64B, 6 = 32B).
__device__ __forceinline__ uint64_t smem_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo,
                                              uint32_t layout) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32;
  d |= 1ull << 46;
  d |= static_cast<uint64_t>(layout) << 61;
  return d;
}

// 128 TMEM lanes x 128 bits from a no-swizzle K-major shared tile (16 B per row, rows 16 B apart).
__device__ __forceinline__ void tmem_cp_128x128b(uint32_t taddr, uint32_t saddr) {
  asm volatile("tcgen05.cp.cta_group::1.128x128b [%0], %1;" ::"r"(taddr), "l"(smem_desc(saddr, 128, 128, 0))
               : "memory");
}

// Byte offset of 16-byte chunk `ch` of row `row` in the tcgen05 K-major / MN-major swizzled
// layouts with `rowb`-byte rows (128: 128B swizzle, 64: 64B, 32: 32B).
__device__ __forceinline__ uint32_t swz_off(uint32_t row, uint32_t ch, uint32_t rowb) {
  const uint32_t x = rowb == 128 ? (row & 7u) : rowb == 64 ? ((row >> 1) & 3u) : ((row >> 2) & 1u);
  return row * rowb + ((ch ^ x) << 4);
}

// Every CTA: 128 threads, TMEM (`cols` columns) allocated by warp 0, two MMA-done barriers.
struct CompatCta {
  uint32_t tmem;
  uint32_t bar_base;  // two consecutive 8-byte mbarriers
  __device__ __forceinline__ uint32_t bar(uint32_t s) const { return bar_base + 8u * s; }
};

__device__ __forceinline__ void compat_setup(CompatCta& cta, uint64_t* bars, uint32_t* tslot,
                                             uint32_t cols, uint32_t nbars = 2) {
  const uint32_t tid = threadIdx.x;
  if ((tid >> 5) == 0) {
    tmem_alloc(smem_u32(tslot), cols);
    tmem_relinquish();
  }
  if (tid == 0) {
    for (uint32_t i = 0; i < nbars; ++i) mbar_init(smem_u32(&bars[i]), 1);
    fence_mbar_init();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  cta.tmem = *tslot;
  cta.bar_base = smem_u32(&bars[0]);
}

// After the K loop: wait for the last commit (all MMAs), drain TMEM rows [0, tile_m) of the
// 128 x 128 accumulator to C (32-bit elements, row pitch n), release TMEM.
__device__ __forceinline__ void compat_finish(const CompatCta& cta, bool ok, uint32_t nk,
                                              uint32_t* c, uint32_t n, uint32_t m0, uint32_t n0,
                                              uint32_t tile_m, uint32_t cols, uint32_t nbuf = 2) {
  const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  cp_async_wait<0>();  // no copy may still be landing when the CTA leaves
  if (ok && nk > 0) {
    const bool w = mbar_wait(cta.bar((nk - 1) % nbuf), ((nk - 1) / nbuf) & 1u, 0xA2, nullptr);
    ok = !__syncthreads_or(!w);
  }
  if (ok) {
    tc_fence_after();
    const uint32_t row = warp * 32u + lane;
#pragma unroll 1
    for (int j = 0; j < 4; ++j) {
      uint32_t v[32];
      tmem_ld_32x32b_x32(cta.tmem + ((warp * 32u) << 16) + j * 32, v);
      tmem_ld_wait();
      if (row < tile_m) {
        uint4* dst = reinterpret_cast<uint4*>(c + static_cast<size_t>(m0 + row) * n + n0 + j * 32);
#pragma unroll
        for (int q = 0; q < 8; ++q) dst[q] = make_uint4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(cta.tmem, cols);
  }
}

// Waits until the MMAs of step kb - nbuf (the last readers of operand buffer kb % nbuf) are done.
// Uniform across the CTA: false if any thread's bounded wait gave up.
__device__ __forceinline__ bool compat_wait_buffer(const CompatCta& cta, uint32_t kb, uint32_t site,
                                                   uint32_t nbuf = 2) {
  if (kb < nbuf) return true;
  const bool w = mbar_wait(cta.bar(kb % nbuf), ((kb - nbuf) / nbuf) & 1u, site, nullptr);
  return !__syncthreads_or(!w);
}

// ------------------------------------------------------------------------------------------
// Dense body. ESZ = element bytes (1: s8 -> s32, 2: bf16 / f16 -> f32), FMT = tcgen05 operand
// format (s8: 1 signed; 16-bit: 0 f16, 1 bf16). Tile = 128 (M, only TILE_M rows stored) x 128
// (N); K step per stage = 64 bytes of A row.
template <int ESZ, int TILE_M, uint32_t FMT>
__device__ __forceinline__ void compat_gemm_body(const uint8_t* a, const uint8_t* b, uint32_t* c,
                                                 uint32_t n, uint32_t m0, uint32_t n0) {
  constexpr int BK = 64 / ESZ;              // K elements per stage
  constexpr int A_STAGE = 128 * 64;         // 128 rows x 64 B (rows >= TILE_M never stored)
  constexpr int B_ROWB = 128 * ESZ;         // bytes of N per k row
  constexpr int B_STAGE = BK * B_ROWB;
  constexpr int MMA_K = 32 / ESZ;
  constexpr int KSTEPS = BK / MMA_K;        // 2
  constexpr uint32_t IDESC = idesc_make(ESZ == 1 ? 2 : 1, FMT, FMT, 0, 1, 128, 128);  // B MN-major
  __shared__ __align__(1024) uint8_t sA[2][A_STAGE];
  __shared__ __align__(1024) uint8_t sB[2][B_STAGE];
  __shared__ __align__(8) uint64_t bars[2];
  __shared__ uint32_t tslot;

  CompatCta cta;
  compat_setup(cta, bars, &tslot, 128);
  const uint32_t tid = threadIdx.x;
  const uint32_t nk = n / BK;
  const uint32_t rowb = n * ESZ;  // global row pitch in bytes

  auto load = [&](uint32_t st, uint32_t kb) {
    const uint32_t sa = smem_u32(sA[st]), sb = smem_u32(sB[st]);
#pragma unroll
    for (int i = 0; i < 4; ++i) {  // A: TILE_M rows x 4 chunks of 16 B (64B swizzle)
      const uint32_t u = tid + 128u * i, row = u >> 2, ch = u & 3u;
      if (row < TILE_M)
        cp_async_16(sa + swz_off(row, ch, 64), a + static_cast<size_t>(m0 + row) * rowb + kb * 64u + ch * 16u);
    }
#pragma unroll
    for (int i = 0; i < B_STAGE / 16 / 128; ++i) {  // B: BK k-rows x B_ROWB bytes (128B swizzle)
      const uint32_t u = tid + 128u * i, kr = u / (B_ROWB / 16), ch = u % (B_ROWB / 16);
      const uint32_t atom = ch >> 3, cin = ch & 7u;
      cp_async_16(sb + atom * (BK * 128u) + swz_off(kr, cin, 128),
                  b + static_cast<size_t>(kb * BK + kr) * rowb + n0 * ESZ + ch * 16u);
    }
    cp_async_commit();
  };

  load(0, 0);
  bool ok = true;
  for (uint32_t kb = 0; kb < nk; ++kb) {
    const uint32_t s = kb & 1u;
    if (kb + 1 < nk) {
      if (!compat_wait_buffer(cta, kb + 1, 0xA1)) { ok = false; break; }  // MMAs of kb - 1
      load(s ^ 1u, kb + 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    fence_proxy_async_smem();  // cp.async (generic proxy) writes -> visible to tcgen05.mma
    __syncthreads();
    if (tid == 0) {
      tc_fence_after();
#pragma unroll
      for (int kk = 0; kk < KSTEPS; ++kk) {
        const uint64_t ad = smem_desc(smem_u32(sA[s]) + kk * 32, 16, 512, 4);
        const uint64_t bd = smem_desc(smem_u32(sB[s]) + kk * MMA_K * 128, BK * 128, 1024, 2);
        if constexpr (ESZ == 1)
          mma_i8_ss(cta.tmem, ad, bd, IDESC, (kb | kk) != 0u);
        else
          mma_f16_ss(cta.tmem, ad, bd, IDESC, (kb | kk) != 0u);
      }
      mma_commit(cta.bar(s));
    }
  }
  compat_finish(cta, ok, nk, c, n, m0, n0, TILE_M, 128);
}

// ------------------------------------------------------------------------------------------
// imma_s4: s4 x s4 -> s32, 128 x 128 tile, 64 logical k per stage. Packed A (128 rows x 32 B)
// and packed B (64 k rows x 64 B) are copied to a staging buffer, then unpacked by all threads
// into the s8 operand layouts (A K-major 64B swizzle, B MN-major 128B swizzle).
__device__ __forceinline__ void compat_s4_body(const uint8_t* a, const uint8_t* b, uint32_t* c,
                                               uint32_t n, uint32_t m0, uint32_t n0) {
  constexpr uint32_t IDESC = idesc_make(2, 1, 1, 0, 1, 128, 128);
  __shared__ __align__(1024) uint8_t sA[2][128 * 64];
  __shared__ __align__(1024) uint8_t sB[2][64 * 128];
  __shared__ __align__(128) uint8_t pA[128 * 32];
  __shared__ __align__(128) uint8_t pB[64 * 64];
  __shared__ __align__(8) uint64_t bars[2];
  __shared__ uint32_t tslot;

  CompatCta cta;
  compat_setup(cta, bars, &tslot, 128);
  const uint32_t tid = threadIdx.x;
  const uint32_t nk = n / 64;
  const size_t pitch = n / 2;  // packed bytes per row of A and of B

  auto load_staging = [&](uint32_t kb) {
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const uint32_t u = tid + 128u * i;
      const uint32_t row = u >> 1, ch = u & 1u;  // A: 128 rows x 2 chunks
      cp_async_16(smem_u32(pA) + row * 32u + ch * 16u, a + (m0 + row) * pitch + kb * 32u + ch * 16u);
      const uint32_t kr = u >> 2, cb = u & 3u;  // B: 64 k rows x 4 chunks
      cp_async_16(smem_u32(pB) + kr * 64u + cb * 16u, b + (kb * 64u + kr) * pitch + n0 / 2 + cb * 16u);
    }
    cp_async_commit();
  };
  auto unpack = [&](uint32_t s) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t u = tid + 128u * i;
      uint32_t w0, w1, o0, o1, o2, o3;
      const uint32_t row = u >> 2, ch = u & 3u;  // A: 16 k of row `row` from 8 packed bytes
      ld_shared_v2(smem_u32(pA) + row * 32u + ch * 8u, w0, w1);
      unpack8(w0, o0, o1);
      unpack8(w1, o2, o3);
      st_shared_v4(smem_u32(sA[s]) + swz_off(row, ch, 64), o0, o1, o2, o3);
      const uint32_t kr = u >> 3, cb = u & 7u;  // B: 16 n of k row `kr`
      ld_shared_v2(smem_u32(pB) + kr * 64u + cb * 8u, w0, w1);
      unpack8(w0, o0, o1);
      unpack8(w1, o2, o3);
      st_shared_v4(smem_u32(sB[s]) + swz_off(kr, cb, 128), o0, o1, o2, o3);
    }
  };

  load_staging(0);
  bool ok = true;
  for (uint32_t kb = 0; kb < nk; ++kb) {
    const uint32_t s = kb & 1u;
    if (!compat_wait_buffer(cta, kb, 0xA3)) { ok = false; break; }
    cp_async_wait<0>();
    __syncthreads();  // staging of step kb complete for every thread
    unpack(s);
    fence_proxy_async_smem();
    __syncthreads();  // operands visible to the MMA; staging free
    if (kb + 1 < nk) load_staging(kb + 1);
    if (tid == 0) {
      tc_fence_after();
#pragma unroll
      for (int kk = 0; kk < 2; ++kk)
        mma_i8_ss(cta.tmem, smem_desc(smem_u32(sA[s]) + kk * 32, 16, 512, 4),
                  smem_desc(smem_u32(sB[s]) + kk * 32 * 128, 64 * 128, 1024, 2), IDESC, (kb | kk) != 0u);
      mma_commit(cta.bar(s));
    }
  }
  compat_finish(cta, ok, nk, c, n, m0, n0, 128, 128);
}

// ------------------------------------------------------------------------------------------
// Sparse bodies: one tcgen05.mma.sp kind::i8 (M 128, N 128, 64 dense k) per stage. Operands per
// stage: A_c 128 rows x 32 B (K-major 32B swizzle), B 64 k rows x 128 B (MN-major 128B swizzle),
// metadata 128 rows x 16 B (two words used), copied to TMEM columns [128, 132) by tcgen05.cp
// before the MMA (tcgen05 operations of one thread execute in issue order).
//   S4 = false: imma_sp_s8 — A_c, B and metadata are copied straight into the operand buffers.
//   S4 = true:  imma_sp_s4 — packed A_c (128 x 16 B) and B (64 x 64 B) go to staging and are
//               unpacked with the k reorder described at the top of this file; metadata words
//               are read and expanded per thread.
template <bool S4>
__device__ __forceinline__ void compat_sp_body(const uint8_t* a, const uint8_t* b, const uint32_t* meta,
                                               uint32_t* c, uint32_t n, uint32_t m0, uint32_t n0) {
  constexpr uint32_t IDESC = idesc_make(2, 1, 1, 0, 1, 128, 128, /*sparse*/ 1);
  constexpr uint32_t META_COL = 128;
  // imma_sp_s8 keeps three stages in flight (42 KB of the 48 KB of static shared memory): with
  // two, a CTA waited on each stage's copies; imma_sp_s4 needs its staging buffers and keeps two
  constexpr uint32_t NS = S4 ? 2 : 3;
  __shared__ __align__(1024) uint8_t sA[NS][128 * 32];
  __shared__ __align__(1024) uint8_t sB[NS][64 * 128];
  __shared__ __align__(128) uint8_t sE[NS][128 * 16];
  __shared__ __align__(128) uint8_t pA[S4 ? 128 * 16 : 16];
  __shared__ __align__(128) uint8_t pB[S4 ? 64 * 64 : 16];
  __shared__ __align__(8) uint64_t bars[NS];
  __shared__ uint32_t tslot;

  CompatCta cta;
  compat_setup(cta, bars, &tslot, 256, NS);
  const uint32_t tid = threadIdx.x;
  const uint32_t nk = n / 64;

  // S4 = false: straight into operand buffer s.
  auto load_direct = [&](uint32_t s, uint32_t kb) {
    const size_t apitch = n / 2;
#pragma unroll
    for (int i = 0; i < 2; ++i) {  // A_c: 128 rows x 2 chunks
      const uint32_t u = tid + 128u * i, row = u >> 1, ch = u & 1u;
      cp_async_16(smem_u32(sA[s]) + swz_off(row, ch, 32), a + (m0 + row) * apitch + kb * 32u + ch * 16u);
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {  // B: 64 k rows x 8 chunks
      const uint32_t u = tid + 128u * i, kr = u >> 3, ch = u & 7u;
      cp_async_16(smem_u32(sB[s]) + swz_off(kr, ch, 128), b + static_cast<size_t>(kb * 64u + kr) * n + n0 + ch * 16u);
    }
    // metadata: words 2 kb, 2 kb + 1 of row `tid` (n/32 words per row)
    cp_async_8(smem_u32(sE[s]) + tid * 16u, meta + static_cast<size_t>(m0 + tid) * (n / 32) + 2u * kb);
    cp_async_commit();
  };
  // S4 = true: packed operands into staging.
  auto load_staging = [&](uint32_t kb) {
    cp_async_16(smem_u32(pA) + tid * 16u, a + static_cast<size_t>(m0 + tid) * (n / 4) + kb * 16u);
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const uint32_t u = tid + 128u * i, kr = u >> 2, cb = u & 3u;
      cp_async_16(smem_u32(pB) + kr * 64u + cb * 16u, b + static_cast<size_t>(kb * 64u + kr) * (n / 2) + n0 / 2 + cb * 16u);
    }
    cp_async_commit();
  };
  auto unpack = [&](uint32_t s, uint32_t kb) {
    // A_c row `tid`: 8 chunks x 2 kept bytes -> 8 x [lo(b0), lo(b1), hi(b0), hi(b1)]
    uint32_t w[4];
    ld_shared_v4(smem_u32(pA) + tid * 16u, w[0], w[1], w[2], w[3]);
    uint32_t o[8];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const uint32_t lo = sext4x4(w[q] & 0x0F0F0F0Fu), hi = sext4x4((w[q] >> 4) & 0x0F0F0F0Fu);
      o[2 * q] = __byte_perm(lo, hi, 0x5410);      // chunk 2q:   lo(b0) lo(b1) hi(b0) hi(b1)
      o[2 * q + 1] = __byte_perm(lo, hi, 0x7632);  // chunk 2q+1: lo(b2) lo(b3) hi(b2) hi(b3)
    }
    st_shared_v4(smem_u32(sA[s]) + swz_off(tid, 0, 32), o[0], o[1], o[2], o[3]);
    st_shared_v4(smem_u32(sA[s]) + swz_off(tid, 1, 32), o[4], o[5], o[6], o[7]);
    // metadata: each reference nibble serves both 4-groups of its chunk
    const uint32_t mw = __ldg(meta + static_cast<size_t>(m0 + tid) * (n / 64) + kb);
    auto spread = [](uint32_t x) {  // 4 nibbles -> 8 nibbles, each repeated
      const uint32_t t = (x & 0xFu) | ((x & 0xF0u) << 4) | ((x & 0xF00u) << 8) | ((x & 0xF000u) << 12);
      return t | (t << 4);
    };
    st_shared_v2(smem_u32(sE[s]) + tid * 16u, spread(mw & 0xFFFFu), spread(mw >> 16));
    // B: logical k row kr = 8j + 2p + e of the stage goes to row 8j + 4e + p
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t u = tid + 128u * i, kr = u >> 3, cb = u & 7u;
      const uint32_t pos = (kr & ~7u) | ((kr & 1u) << 2) | ((kr >> 1) & 3u);
      uint32_t w0, w1, o0, o1, o2, o3;
      ld_shared_v2(smem_u32(pB) + kr * 64u + cb * 8u, w0, w1);
      unpack8(w0, o0, o1);
      unpack8(w1, o2, o3);
      st_shared_v4(smem_u32(sB[s]) + swz_off(pos, cb, 128), o0, o1, o2, o3);
    }
  };
  auto issue = [&](uint32_t s, uint32_t kb) {
    tc_fence_after();
    tmem_cp_128x128b(cta.tmem + META_COL, smem_u32(sE[s]));
    mma_sp_i8_ss(cta.tmem, smem_desc(smem_u32(sA[s]), 16, 256, 6), smem_desc(smem_u32(sB[s]), 64 * 128, 1024, 2),
                 cta.tmem + META_COL, IDESC, kb != 0u);
    mma_commit(cta.bar(s));
  };

  bool ok = true;
  if constexpr (!S4) {
    load_direct(0, 0);
    if (nk > 1) load_direct(1, 1);
    for (uint32_t kb = 0; kb < nk; ++kb) {
      const uint32_t s = kb % NS;
      if (kb + 2 < nk) {
        if (!compat_wait_buffer(cta, kb + 2, 0xA4, NS)) { ok = false; break; }  // MMAs of kb - 1
        load_direct((kb + 2) % NS, kb + 2);
        cp_async_wait<2>();
      } else if (kb + 1 < nk) {
        cp_async_wait<1>();
      } else {
        cp_async_wait<0>();
      }
      fence_proxy_async_smem();
      __syncthreads();
      if (tid == 0) issue(s, kb);
    }
  } else {
    load_staging(0);
    for (uint32_t kb = 0; kb < nk; ++kb) {
      const uint32_t s = kb & 1u;
      if (!compat_wait_buffer(cta, kb, 0xA5)) { ok = false; break; }
      cp_async_wait<0>();
      __syncthreads();
      unpack(s, kb);
      fence_proxy_async_smem();
      __syncthreads();
      if (kb + 1 < nk) load_staging(kb + 1);
      if (tid == 0) issue(s, kb);
    }
  }
  compat_finish(cta, ok, nk, c, n, m0, n0, 128, 256, NS);
}

}  // namespace zx

// Exact reference entry names (src/host.zig:100-123 symbol mangling: <stem>_$_<decl>).
extern "C" __global__ void __launch_bounds__(128)
    imma_s8_$_immaS8(const int8_t* a, const int8_t* b, int32_t* c, uint32_t n) {
  zx::compat_gemm_body<1, 128, 1>(reinterpret_cast<const uint8_t*>(a), reinterpret_cast<const uint8_t*>(b),
                                  reinterpret_cast<uint32_t*>(c), n, blockIdx.y * 128u, blockIdx.x * 128u);
}

extern "C" __global__ void __launch_bounds__(128)
    imma_s4_$_immaS4(const uint8_t* a, const uint8_t* b, int32_t* c, uint32_t n) {
  zx::compat_s4_body(a, b, reinterpret_cast<uint32_t*>(c), n, blockIdx.y * 128u, blockIdx.x * 128u);
}

extern "C" __global__ void __launch_bounds__(128)
    imma_sp_s8_$_immaSpS8(const int8_t* a, const int8_t* b, const uint32_t* meta, int32_t* c, uint32_t n) {
  zx::compat_sp_body<false>(reinterpret_cast<const uint8_t*>(a), reinterpret_cast<const uint8_t*>(b), meta,
                            reinterpret_cast<uint32_t*>(c), n, blockIdx.y * 128u, blockIdx.x * 128u);
}

extern "C" __global__ void __launch_bounds__(128)
    imma_sp_s4_$_immaSpS4(const uint8_t* a, const uint8_t* b, const uint32_t* meta, int32_t* c, uint32_t n) {
  zx::compat_sp_body<true>(a, b, meta, reinterpret_cast<uint32_t*>(c), n, blockIdx.y * 128u, blockIdx.x * 128u);
}

extern "C" __global__ void __launch_bounds__(128)
    hgemm_bf16_$_hgemmBf16(const uint16_t* a, const uint16_t* b, float* c, uint32_t n) {
  zx::compat_gemm_body<2, 128, 1>(reinterpret_cast<const uint8_t*>(a), reinterpret_cast<const uint8_t*>(b),
                                  reinterpret_cast<uint32_t*>(c), n, blockIdx.y * 128u, blockIdx.x * 128u);
}

extern "C" __global__ void __launch_bounds__(128)
    hgemm_wgmma_bf16_$_hgemmWgmmaBf16(const uint16_t* a, const uint16_t* b, float* c, uint32_t n) {
  zx::compat_gemm_body<2, 64, 1>(reinterpret_cast<const uint8_t*>(a), reinterpret_cast<const uint8_t*>(b),
                                 reinterpret_cast<uint32_t*>(c), n, blockIdx.y * 64u, blockIdx.x * 128u);
}

extern "C" __global__ void __launch_bounds__(128)
    hgemm_tma_$_hgemmTma(const uint16_t* a, const uint16_t* b, float* c, uint32_t n, uint64_t desc_a,
                         uint64_t desc_b) {
  (void)desc_a;
  (void)desc_b;
  zx::compat_gemm_body<2, 64, 0>(reinterpret_cast<const uint8_t*>(a), reinterpret_cast<const uint8_t*>(b),
                                 reinterpret_cast<uint32_t*>(c), n, blockIdx.y * 64u, blockIdx.x * 128u);
}
