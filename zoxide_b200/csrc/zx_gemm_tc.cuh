// zx_gemm_tc.cuh — persistent, warp-specialised tcgen05 GEMM for sm_100a.
//
// One template covers the dense paths of the quantised-GEMM family:
//   kind::i8  s8 x s8 -> s32, stored as int32       (reference imma_s8, src/examples/imma_s8.zig:130-173)
//   kind::i8  s8 x s8 -> s32 -> fp32 row/col scale -> bf16  (BASELINE config-2 epilogue; no ref kernel)
//   kind::f16 bf16 x bf16 -> f32                    (reference hgemm_wgmma_bf16, src/examples/hgemm_wgmma_bf16.zig:105-169)
// with B either K-major ("NT": B stored N x K, K contiguous) or MN-major ("NN": B stored K x N,
// N contiguous — the reference's own layout, src/examples/imma_s8.zig:75 and src/bench.zig:726).
//
// CTA = 6 warps, one CTA per SM, persistent over output tiles (BM x BN):
//   warp 0      TMA producer: A and B stage tiles (128-byte rows, 128B swizzle) into a ring of
//               kStages shared-memory stages, completion on full[s] (expect-tx bytes).
//   warp 1      TMEM owner + MMA issuer: one thread issues tcgen05.mma (M=128, N=BN, K=32 bytes)
//               into one of two TMEM accumulators; tcgen05.commit frees a stage (empty[s]) and
//               publishes a finished accumulator (tfull[b]).
//   warps 2..5  epilogue: tcgen05.ld 32 lanes x 32 columns, convert, write a 32-row x 128-byte
//               swizzled staging tile, TMA store. Releases the accumulator (tempty[b]) as soon as
//               its last column is in registers, so tile i's epilogue overlaps tile i+1's MMAs.
// Every mbarrier wait is bounded (zx::mbar_wait); a timeout records a code in zx::g_status, raises
// a CTA-wide abort flag, and every role drains and falls through to the TMEM dealloc.
#pragma once
#include <cuda_bf16.h>

#include "zx_ptx.cuh"

namespace zx {

// I8: s8 x s8; BF16: bf16 x bf16; W4: s8 activations x s4 weights (B packed two per byte along
// K, low nibble = even k), unpacked to s8 in shared memory and run on kind::i8.
enum class Kind : int { I8 = 0, BF16 = 1, W4 = 2 };
enum class Out : int { S32 = 0, F32 = 1, BF16_SCALED = 2 };

struct GemmParams {
  CUtensorMap tmA;  // A  M x K, K contiguous
  CUtensorMap tmB;  // NT: N x K (K contiguous); NN: K x N (N contiguous)
  CUtensorMap tmC;  // C  M x N, N contiguous
  CUtensorMap tmB2;  // 256 x 480 pair tiles: B again, with the hi half's box height
  const float* row_scale;  // BF16_SCALED only: M floats
  const float* col_scale;  // BF16_SCALED only: N floats
  uint32_t M, N, K;
  uint32_t num_m_blk, num_n_blk, num_k_blk;
  uint32_t group_m;  // raster group height in M tiles (L2 reuse of B across a group)
  // Replicas of C (256 x 512 kernel, int32 out only): the epilogue also stores every tile to
  // these addresses (other GPUs' buffers mapped into this process), same row pitch as C.
  uint64_t peer_c[7];
  uint32_t npeers;
  uint32_t ldc;  // row pitch of C in elements (peer stores; the C tensor map carries its own)
  const uint32_t* c_base;  // C itself (replica copies read finished tiles back from it)
  // Kind::BF16 kernels with f16 operands: XORed into the instruction descriptor, it turns the
  // A and B formats from bf16 (1) to f16 (0); zero otherwise
  uint32_t idesc_xor;
};

template <Kind kKind, bool kBMajorMN, Out kOut, int kBN, int kStages>
struct GemmCfg {
  static constexpr int BM = 128;
  static constexpr int BN = kBN;
  static constexpr int ESZ = kKind == Kind::I8 ? 1 : 2;
  static constexpr int ROWB = 128;                 // bytes of K per operand row per stage
  static constexpr int BK = ROWB / ESZ;            // K elements per stage
  static constexpr int MMA_K = 32 / ESZ;           // K elements per tcgen05.mma
  static constexpr int KSTEPS = BK / MMA_K;        // MMAs per stage (4)
  static constexpr int A_BYTES = BM * ROWB;
  static constexpr int B_BYTES = BN * ROWB;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = kStages;
  static constexpr int OUT_ESZ = kOut == Out::BF16_SCALED ? 2 : 4;
  static constexpr int CHUNK_COLS = 128 / OUT_ESZ;  // output columns per 128-byte staging row
  static constexpr int NCHUNK = BN / CHUNK_COLS;
  static constexpr int EPI_WARPS = 4;
  static constexpr int EPI_BUF = 32 * 128;         // one warp's 32-row staging tile
  static constexpr int EPI_BYTES = EPI_WARPS * 2 * EPI_BUF;
  static constexpr uint32_t TMEM_COLS = 2 * BN;    // two accumulators of BN 32-bit columns
  static constexpr int THREADS = 32 * (2 + EPI_WARPS);
  // barriers: full[S], empty[S], tfull[2], tempty[2], drain; then tmem slot + abort flag
  static constexpr int BAR_BYTES = 8 * (2 * STAGES + 5) + 16;
  static constexpr int SMEM_BYTES = 1024 /*align slack*/ + STAGES * STAGE_BYTES + EPI_BYTES + BAR_BYTES;
  // B's MN-major stage layout: BN*ESZ/128 column blocks of [BK rows x 128 bytes].
  static constexpr int B_MN_BLOCKS = BN * ESZ / 128;
  static constexpr int B_MN_BLOCK_BYTES = BK * 128;
  static constexpr uint32_t IDESC =
      kKind == Kind::I8 ? idesc_make(/*s32*/ 2, /*s8*/ 1, /*s8*/ 1, 0, kBMajorMN ? 1 : 0, BM, BN)
                        : idesc_make(/*f32*/ 1, /*bf16*/ 1, /*bf16*/ 1, 0, kBMajorMN ? 1 : 0, BM, BN);
  static_assert(BN % 16 == 0 && BN >= 16 && BN <= 256, "tcgen05 M=128 needs N % 16 == 0, 16..256");
  static_assert(TMEM_COLS >= 32 && (TMEM_COLS & (TMEM_COLS - 1)) == 0 && TMEM_COLS <= 512,
                "TMEM allocation is a power of two in [32, 512]");
  static_assert(SMEM_BYTES <= 232448, "exceeds the 227 KB dynamic shared memory of one CTA");
};

__device__ __forceinline__ void tile_coords(uint32_t tile, const GemmParams& p, uint32_t& mb,
                                            uint32_t& nb) {
  const uint32_t group_tiles = p.group_m * p.num_n_blk;
  const uint32_t group = tile / group_tiles;
  const uint32_t first_m = group * p.group_m;
  const uint32_t gm = min(p.num_m_blk - first_m, p.group_m);
  const uint32_t in = tile - group * group_tiles;
  mb = first_m + in % gm;
  nb = in / gm;
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  const __nv_bfloat16 l = __float2bfloat16_rn(lo);
  const __nv_bfloat16 h = __float2bfloat16_rn(hi);
  return static_cast<uint32_t>(__bfloat16_as_ushort(l)) |
         (static_cast<uint32_t>(__bfloat16_as_ushort(h)) << 16);
}

template <Kind kKind, bool kBMajorMN, Out kOut, int kBN, int kStages>
__global__ void __launch_bounds__(192, 1)
    gemm_tc_kernel(const __grid_constant__ GemmParams p) {
  using C = GemmCfg<kKind, kBMajorMN, kOut, kBN, kStages>;
  extern __shared__ uint8_t smem_raw[];
  // the producer thread starts fetching its tensor maps at once, so the fetch overlaps the
  // barrier / TMEM set-up instead of delaying the first loads
  if (threadIdx.x == 0) {
    tma_prefetch_desc(&p.tmA);
    tma_prefetch_desc(&p.tmB);
    tma_prefetch_desc(&p.tmC);
  }
  // 1024-byte alignment: required by the 128B-swizzle atom (descriptor base offset 0).
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* const gbase = smem_raw + (base - raw);

  const uint32_t stage_base = base;
  const uint32_t epi_base = base + C::STAGES * C::STAGE_BYTES;
  const uint32_t bar_base = epi_base + C::EPI_BYTES;
  auto full_bar = [&](int s) { return bar_base + 8u * s; };
  auto empty_bar = [&](int s) { return bar_base + 8u * (C::STAGES + s); };
  auto tfull_bar = [&](int b) { return bar_base + 8u * (2 * C::STAGES + b); };
  auto tempty_bar = [&](int b) { return bar_base + 8u * (2 * C::STAGES + 2 + b); };
  const uint32_t drain_bar = bar_base + 8u * (2 * C::STAGES + 4);
  const uint32_t slot_off = 8u * (2 * C::STAGES + 5);
  volatile uint32_t* tmem_slot = reinterpret_cast<volatile uint32_t*>(gbase + (bar_base - base) + slot_off);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(gbase + (bar_base - base) + slot_off + 4);

  const uint32_t warp = threadIdx.x >> 5;
  const uint32_t lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(tfull_bar(b), 1);
      mbar_init(tempty_bar(b), C::EPI_WARPS);
    }
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    fence_mbar_init();
    fence_proxy_async_smem();
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(const_cast<uint32_t*>(tmem_slot)), C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const uint32_t num_tiles = p.num_m_blk * p.num_n_blk;

  if (warp == 0) {
    // ------------------------------------ TMA producer ------------------------------------
    if (lane == 0) {
      uint32_t stage = 0, phase = 0, issued = 0;
      bool ok = true;
      for (uint32_t tile = blockIdx.x; ok && tile < num_tiles; tile += gridDim.x) {
        uint32_t mb, nb;
        tile_coords(tile, p, mb, nb);
        const int32_t m0 = static_cast<int32_t>(mb * C::BM);
        const int32_t n0 = static_cast<int32_t>(nb * C::BN);
        for (uint32_t kb = 0; kb < p.num_k_blk; ++kb) {
          if (!mbar_wait(empty_bar(stage), phase ^ 1u, 0x01, abort_flag)) {
            *abort_flag = 1;
            ok = false;
            break;
          }
          const uint32_t sa = stage_base + stage * C::STAGE_BYTES;
          const uint32_t sb = sa + C::A_BYTES;
          const int32_t k0 = static_cast<int32_t>(kb * C::BK);
          if constexpr (!kBMajorMN) {
            mbar_arrive_expect_tx(full_bar(stage), C::STAGE_BYTES);
            tma_load_2d(sa, &p.tmA, full_bar(stage), k0, m0);
            tma_load_2d(sb, &p.tmB, full_bar(stage), k0, n0);
          } else {
            // Column blocks wholly past N are skipped: they only feed accumulator columns
            // that are never stored. Partially covered boxes are zero-filled by the TMA.
            int nblk = 0;
#pragma unroll
            for (int h = 0; h < C::B_MN_BLOCKS; ++h)
              nblk += (static_cast<uint32_t>(n0 + h * (128 / C::ESZ)) < p.N) ? 1 : 0;
            mbar_arrive_expect_tx(full_bar(stage), C::A_BYTES + nblk * C::B_MN_BLOCK_BYTES);
            tma_load_2d(sa, &p.tmA, full_bar(stage), k0, m0);
#pragma unroll
            for (int h = 0; h < C::B_MN_BLOCKS; ++h)
              if (h < nblk)
                tma_load_2d(sb + h * C::B_MN_BLOCK_BYTES, &p.tmB, full_bar(stage),
                            n0 + h * (128 / C::ESZ), k0);
          }
          ++issued;
          if (++stage == C::STAGES) { stage = 0; phase ^= 1u; }
        }
      }
      // Drain: the last load issued into each stage slot must have landed before this CTA's
      // shared memory can go away (normal path: already consumed, returns at once).
      const uint32_t tail = issued < (uint32_t)C::STAGES ? issued : (uint32_t)C::STAGES;
      for (uint32_t i = 0; i < tail; ++i) {
        // walk back from the slot before `stage`
        int s = static_cast<int>(stage) - 1 - static_cast<int>(i);
        uint32_t ph = phase;
        while (s < 0) { s += C::STAGES; ph ^= 1u; }
        mbar_wait(full_bar(s), ph, 0x02, nullptr);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // -------------------------------------- MMA issuer --------------------------------------
    if (lane == 0) {
      uint32_t stage = 0, phase = 0, local = 0;
      bool ok = true;
      for (uint32_t tile = blockIdx.x; ok && tile < num_tiles; tile += gridDim.x, ++local) {
        const uint32_t buf = local & 1u;
        const uint32_t use = local >> 1;
        if (!mbar_wait(tempty_bar(buf), (use & 1u) ^ 1u, 0x11, abort_flag)) {
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + buf * C::BN;
        for (uint32_t kb = 0; kb < p.num_k_blk; ++kb) {
          if (!mbar_wait(full_bar(stage), phase, 0x12, abort_flag)) {
            *abort_flag = 1;
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = stage_base + stage * C::STAGE_BYTES;
          const uint32_t sb = sa + C::A_BYTES;
#pragma unroll
          for (int kk = 0; kk < C::KSTEPS; ++kk) {
            const uint64_t adesc = smem_desc_sw128(sa + kk * 32, 16, 1024);
            uint64_t bdesc;
            if constexpr (!kBMajorMN)
              bdesc = smem_desc_sw128(sb + kk * 32, 16, 1024);
            else
              bdesc = smem_desc_sw128(sb + kk * C::MMA_K * 128, C::B_MN_BLOCK_BYTES, 1024);
            const uint32_t acc = (kb | static_cast<uint32_t>(kk)) != 0u;
            if constexpr (kKind == Kind::I8)
              mma_i8_ss(d_tmem, adesc, bdesc, C::IDESC, acc);
            else
              mma_f16_ss(d_tmem, adesc, bdesc, C::IDESC ^ p.idesc_xor, acc);
          }
          mma_commit(empty_bar(stage));
          if (++stage == C::STAGES) { stage = 0; phase ^= 1u; }
        }
        if (!ok) break;
        mma_commit(tfull_bar(buf));
      }
      // Drain every MMA this thread issued before TMEM can be released.
      mma_commit(drain_bar);
      mbar_wait(drain_bar, 0, 0x13, nullptr);
    }
    __syncwarp();
  } else {
    // --------------------------------------- epilogue ---------------------------------------
    const uint32_t q = warp & 3u;  // TMEM lane quarter this warp may access
    const uint32_t ew = warp - 2u;
    const uint32_t row_in_tile = q * 32u + lane;
    uint32_t local = 0;
    uint32_t chunk_ctr = 0;
    for (uint32_t tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++local) {
      uint32_t mb, nb;
      tile_coords(tile, p, mb, nb);
      const uint32_t m0 = mb * C::BM;
      const uint32_t n0 = nb * C::BN;
      const uint32_t buf = local & 1u;
      const uint32_t use = local >> 1;
      int ok = 1;
      if (lane == 0) ok = mbar_wait(tfull_bar(buf), use & 1u, 0x21, abort_flag) ? 1 : 0;
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) {
        if (lane == 0) *abort_flag = 1;
        break;
      }
      tc_fence_after();
      const uint32_t t_row = tmem_base + ((q * 32u) << 16) + buf * C::BN;
      float rs = 0.f;
      if constexpr (kOut == Out::BF16_SCALED) {
        const uint32_t gm = m0 + row_in_tile;
        rs = gm < p.M ? __ldg(p.row_scale + gm) : 0.f;
      }
#pragma unroll 1
      for (int j = 0; j < C::NCHUNK; ++j, ++chunk_ctr) {
        uint32_t w[32];  // 128 bytes of this thread's output row
        if constexpr (kOut == Out::BF16_SCALED) {
          uint32_t r0[32], r1[32];
          tmem_ld_32x32b_x32(t_row + j * 64, r0);
          tmem_ld_32x32b_x32(t_row + j * 64 + 32, r1);
          tmem_ld_wait();
          if (j == C::NCHUNK - 1) {
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(tempty_bar(buf));
          }
          const uint32_t nc = n0 + j * 64;
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            float cs[2];
#pragma unroll
            for (int e = 0; e < 2; ++e) {
              const uint32_t gn = nc + 2 * i + e;
              cs[e] = gn < p.N ? __ldg(p.col_scale + gn) : 0.f;
            }
            const float a0 = __fmul_rn(__fmul_rn(__int2float_rn(static_cast<int>(r0[2 * i])), rs), cs[0]);
            const float a1 = __fmul_rn(__fmul_rn(__int2float_rn(static_cast<int>(r0[2 * i + 1])), rs), cs[1]);
            w[i] = pack_bf16x2(a0, a1);
          }
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            float cs[2];
#pragma unroll
            for (int e = 0; e < 2; ++e) {
              const uint32_t gn = nc + 32 + 2 * i + e;
              cs[e] = gn < p.N ? __ldg(p.col_scale + gn) : 0.f;
            }
            const float a0 = __fmul_rn(__fmul_rn(__int2float_rn(static_cast<int>(r1[2 * i])), rs), cs[0]);
            const float a1 = __fmul_rn(__fmul_rn(__int2float_rn(static_cast<int>(r1[2 * i + 1])), rs), cs[1]);
            w[16 + i] = pack_bf16x2(a0, a1);
          }
        } else {
          tmem_ld_32x32b_x32(t_row + j * 32, w);
          tmem_ld_wait();
          if (j == C::NCHUNK - 1) {
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(tempty_bar(buf));
          }
        }
        // Staging tile: 32 rows x 128 B, 16-byte chunk c of row r at (c ^ (r & 7)) — the TMA
        // 128B swizzle pattern, which also makes these v4 stores bank-conflict free.
        const uint32_t sbuf = epi_base + (ew * 2u + (chunk_ctr & 1u)) * C::EPI_BUF;
        if (lane == 0) bulk_wait_read<1>();
        __syncwarp();
        const uint32_t row_addr = sbuf + lane * 128u;
#pragma unroll
        for (int c = 0; c < 8; ++c)
          st_shared_v4(row_addr + ((static_cast<uint32_t>(c) ^ (lane & 7u)) << 4), w[4 * c],
                       w[4 * c + 1], w[4 * c + 2], w[4 * c + 3]);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          const uint32_t xs = n0 + j * C::CHUNK_COLS, ys = m0 + q * 32u;
          if (xs < p.N && ys < p.M)  // boxes wholly outside C are not issued
            tma_store_2d(&p.tmC, sbuf, static_cast<int32_t>(xs), static_cast<int32_t>(ys));
          bulk_commit();
        }
      }
    }
    // the staging tiles must have been read before the CTA leaves; the global writes themselves
    // complete on their own and are visible to work ordered after the kernel
    if (lane == 0) bulk_wait_read<0>();
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
}

}  // namespace zx
