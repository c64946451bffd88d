// zx_compat.cuh — kernels that keep the reference's own launch contract, so they drop into the
// reference's module/launch flow unchanged (src/host.zig:342-349 Module.kernel, :498-565
// Kernel.launchOn; src/cuda_driver.zig:820-845 cuLaunchKernel):
//
//   imma_s8_$_immaS8(a: *const i8, b: *const i8, c: *i32, n: u32)
//       src/examples_abi.zig:42; launched by src/bench.zig:671-682 with grid (n/128, n/128),
//       block 128, no dynamic shared memory, no cluster. A, B, C n x n row-major (B is K x N).
//   hgemm_wgmma_bf16_$_hgemmWgmmaBf16(a: *const u16, b: *const u16, c: *f32, n: u32)
//       src/examples_abi.zig:33-36 (hgemm_bf16.signature, launch_bounds 128); launched by
//       src/bench.zig:589-600 with grid (n/128, n/64), block 128: a 64 x 128 tile per CTA.
//
// Entry names are the reference's `<stem>_$_<decl>` symbols (src/host.zig:100-123). Under that
// contract there is no tensor-map argument and no room for warp specialisation, so each CTA
// copies its operand tiles with 16-byte cp.async into the tcgen05 swizzled layouts itself
// (A K-major 64B swizzle, B MN-major 128B swizzle), double-buffered in 32 KB of static shared
// memory; thread 0 issues tcgen05.mma (M=128, cta_group::1) and the four warps drain TMEM.
// These are slower by construction than the zx_gemm_* paths; they exist to be a literal
// drop-in for the reference's cubin loader. Every wait is bounded; a wait that gives up
// records its site in g_status and the whole CTA leaves the K loop together.
#pragma once
#include "zx_ptx.cuh"

namespace zx {

__device__ __forceinline__ void cp_async_16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Matrix descriptor with an explicit layout type (2 = 128B swizzle, 4 = 64B swizzle).
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

// Shared body. ESZ = element bytes (1: s8 -> s32, 2: bf16 -> f32). Tile = 128 (M, only TILE_M
// rows stored) x 128 (N); K step per stage = 64 bytes of A row.
template <int ESZ, int TILE_M>
__device__ __forceinline__ void compat_gemm_body(const uint8_t* a, const uint8_t* b, uint32_t* c,
                                                 uint32_t n, uint32_t m0, uint32_t n0) {
  constexpr int BK = 64 / ESZ;              // K elements per stage
  constexpr int A_STAGE = 128 * 64;         // 128 rows x 64 B (rows >= TILE_M never stored)
  constexpr int B_ROWB = 128 * ESZ;         // bytes of N per k row
  constexpr int B_ATOMS = B_ROWB / 128;     // 128-byte swizzle atoms along N
  constexpr int B_STAGE = BK * B_ROWB;
  constexpr int MMA_K = 32 / ESZ;
  constexpr int KSTEPS = BK / MMA_K;        // 2
  constexpr uint32_t IDESC = ESZ == 1 ? idesc_make(2, 1, 1, 0, 1, 128, 128)   // s8, B MN-major
                                      : idesc_make(1, 1, 1, 0, 1, 128, 128);  // bf16 -> f32
  __shared__ __align__(1024) uint8_t sA[2][A_STAGE];
  __shared__ __align__(1024) uint8_t sB[2][B_STAGE];
  __shared__ __align__(8) uint64_t bars[2];
  __shared__ uint32_t tslot;

  const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (warp == 0) {
    tmem_alloc(smem_u32(&tslot), 128);
    tmem_relinquish();
  }
  if (tid == 0) {
    mbar_init(smem_u32(&bars[0]), 1);
    mbar_init(smem_u32(&bars[1]), 1);
    fence_mbar_init();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tslot;
  const uint32_t nk = n / BK;
  const uint32_t rowb = n * ESZ;  // global row pitch in bytes

  auto load = [&](uint32_t st, uint32_t kb) {
    const uint32_t sa = smem_u32(sA[st]), sb = smem_u32(sB[st]);
#pragma unroll
    for (int i = 0; i < 4; ++i) {  // A: TILE_M rows x 4 chunks of 16 B (64B swizzle)
      const uint32_t u = tid + 128u * i, row = u >> 2, ch = u & 3u;
      if (row < TILE_M)
        cp_async_16(sa + row * 64u + ((ch ^ ((row >> 1) & 3u)) << 4),
                    a + static_cast<size_t>(m0 + row) * rowb + kb * 64u + ch * 16u);
    }
#pragma unroll
    for (int i = 0; i < B_STAGE / 16 / 128; ++i) {  // B: BK k-rows x B_ROWB bytes (128B swizzle)
      const uint32_t u = tid + 128u * i, kr = u / (B_ROWB / 16), ch = u % (B_ROWB / 16);
      const uint32_t atom = ch >> 3, cin = ch & 7u;
      cp_async_16(sb + atom * (BK * 128u) + kr * 128u + ((cin ^ (kr & 7u)) << 4),
                  b + static_cast<size_t>(kb * BK + kr) * rowb + n0 * ESZ + ch * 16u);
    }
    cp_async_commit();
  };

  load(0, 0);
  bool ok = true;
  for (uint32_t kb = 0; kb < nk; ++kb) {
    const uint32_t s = kb & 1u;
    if (kb + 1 < nk) {
      if (kb >= 1) {  // the other stage was read by the MMAs of step kb - 1
        const bool w = mbar_wait(smem_u32(&bars[s ^ 1u]), ((kb - 1) >> 1) & 1u, 0xA1, nullptr);
        if (__syncthreads_or(!w)) { ok = false; break; }
      }
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
          mma_i8_ss(tmem, ad, bd, IDESC, (kb | kk) != 0u);
        else
          mma_f16_ss(tmem, ad, bd, IDESC, (kb | kk) != 0u);
      }
      mma_commit(smem_u32(&bars[s]));
    }
  }
  cp_async_wait<0>();  // no copy may still be landing when the CTA leaves
  if (ok && nk > 0) {
    const bool w = mbar_wait(smem_u32(&bars[(nk - 1) & 1u]), ((nk - 1) >> 1) & 1u, 0xA2, nullptr);
    ok = !__syncthreads_or(!w);
  }
  if (ok) {
    tc_fence_after();
    const uint32_t row = warp * 32u + lane;
#pragma unroll 1
    for (int j = 0; j < 4; ++j) {
      uint32_t v[32];
      tmem_ld_32x32b_x32(tmem + ((warp * 32u) << 16) + j * 32, v);
      tmem_ld_wait();
      if (row < TILE_M) {
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
    tmem_dealloc(tmem, 128);
  }
}

}  // namespace zx

// Exact reference entry names (src/host.zig:100-123 symbol mangling: <stem>_$_<decl>).
extern "C" __global__ void __launch_bounds__(128)
    imma_s8_$_immaS8(const int8_t* a, const int8_t* b, int32_t* c, uint32_t n) {
  zx::compat_gemm_body<1, 128>(reinterpret_cast<const uint8_t*>(a), reinterpret_cast<const uint8_t*>(b),
                               reinterpret_cast<uint32_t*>(c), n, blockIdx.y * 128u, blockIdx.x * 128u);
}

extern "C" __global__ void __launch_bounds__(128)
    hgemm_wgmma_bf16_$_hgemmWgmmaBf16(const uint16_t* a, const uint16_t* b, float* c, uint32_t n) {
  zx::compat_gemm_body<2, 64>(reinterpret_cast<const uint8_t*>(a), reinterpret_cast<const uint8_t*>(b),
                              reinterpret_cast<uint32_t*>(c), n, blockIdx.y * 64u, blockIdx.x * 128u);
}
