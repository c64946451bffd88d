// zx_gemm_sp2w.cuh — 2:4 structured-sparse int8 GEMM on CTA pairs with 256 x 480 tiles.
//
// Same operands and contract as zx_gemm_sp2.cuh (reference kernel imma_sp_s8,
// src/examples/imma_sp_s8.zig:144-187, metadata contract src/examples_abi.zig:71-81):
//   A_c M x K/2 int8, meta M x K/32 u32 (reference format, consumed as is), B N x K int8, C int32.
//
// Why a second sparse kernel. A sparse M=256 N=224 K=64 pair MMA issues in ~112 cycles (2x the
// dense rate), so the 256 x 224 pair tile needs 48 KB of operands per CTA per 256 dense k
// (A_c 16 KB + B 28 KB + metadata 4 KB) for 464 cycles of MMA work: ~100 B/clk, about twice what
// an SM takes in (~52 B/clk measured), and the tensor pipe idles half the time. Here one tile
// has two halves sharing the A_c rows: "lo" (256 columns, one N=256 MMA per 64 dense k) and "hi"
// (224 columns), so a CTA loads A_c 16 KB + B 32 + 28 KB + metadata 4 KB = 80 KB for 960 cycles
// of MMA work per stage: 25 % fewer bytes per multiply-add.
//
// The loop is bound by the bytes each SM keeps in flight, so the ring is deep and fine-grained:
// 5 stages of 128 dense k (40 KB each), and the epilogue stages its stores through 2 KB per warp
// (16-row boxes) to leave the shared memory to the ring.
// TMEM (512 columns): lo accumulator 0..255, hi accumulator 256..479, metadata of stage s at
// 480 + 4 s (4 columns = 128 dense k, one u32 per 32 dense k per row, the reference's words in
// order). Per stage slot: A_c 128 rows x 64 B (64B swizzle) | B lo 128 rows x 128 B | B hi
// 112 rows x 128 B (128B swizzle) | metadata 128 rows x 16 B (no swizzle).
// The accumulator hand-over follows the 256 x 512 dense kernel (zx_gemm_tc2w.cuh): the epilogue
// drains lo, releases it, then hi; the next tile's lo MMAs start once lo is free, its hi MMAs are
// held back stage by stage until hi is free. Metadata sits in a TMEM slot per stage, so a held
// stage's metadata is still in place when its hi MMAs are issued.
// Requires M % 128 == 0 and K % 256 == 0; NT only. Every wait is bounded.
// Measured on B200 at 8192^3: 274.9 us (4.0 POPS dense-equivalent) against 264.6 us for the
// 256 x 224 kernel and ~245 us for the 512 x 224 kernel (zx_gemm_sp4.cuh), so the automatic
// choice never picks it; zx_set_kernel_policy(4 or 5) selects it, and it is exact on every sparse
// test.
#pragma once
#include "zx_gemm_sp2.cuh"
#include "zx_gemm_tc2w.cuh"

namespace zx {

struct Sp2wCfg {
  static constexpr int BM = 256, BM_CTA = 128;
  static constexpr int BN_LO = 256, BN_HI = 224, BN = BN_LO + BN_HI;  // 480
  static constexpr int KD = 128;                            // dense k per stage
  static constexpr int A_BYTES = BM_CTA * 64;               // 64 compressed bytes per row
  static constexpr int BLO_BYTES = (BN_LO / 2) * 128;       // 128 rows x one 128-k swizzle atom
  static constexpr int BHI_BYTES = (BN_HI / 2) * 128;       // 112 rows x one atom
  static constexpr int E_BYTES = BM_CTA * 16;               // 128 rows x 16 B (4 words)
  static constexpr int OFF_BLO = A_BYTES, OFF_BHI = OFF_BLO + BLO_BYTES, OFF_E = OFF_BHI + BHI_BYTES;
  static constexpr int STAGE_BYTES = OFF_E + E_BYTES;       // 40 KB
  static constexpr int STAGES = 5;
  static constexpr int CHUNK_COLS = 32;                     // int32 out: 32 columns per 128 B
  static constexpr int EPI_WARPS = 8;
  static constexpr int EPI_ROWS = 16;                       // rows per staged store
  static constexpr int EPI_BUF = EPI_ROWS * 128;
  static constexpr int EPI_BYTES = EPI_WARPS * EPI_BUF;
  static constexpr uint32_t TMEM_COLS = 512;
  static constexpr uint32_t HI_COL = 256;
  static constexpr uint32_t E_COL = 480;                    // + 4 per stage slot
  static constexpr int THREADS = 32 * (2 + EPI_WARPS);
  static constexpr int NBARS = 2 * STAGES + 4;              // full, empty, tfull, tempty_lo, tempty_hi, drain
  static constexpr int BAR_BYTES = 8 * NBARS + 16;
  static constexpr int SMEM_BYTES = 1024 + STAGES * STAGE_BYTES + EPI_BYTES + BAR_BYTES;
  static constexpr uint32_t IDESC_LO = idesc_make(2, 1, 1, 0, 0, BM, BN_LO, /*sparse*/ 1);
  static constexpr uint32_t IDESC_HI = idesc_make(2, 1, 1, 0, 0, BM, BN_HI, /*sparse*/ 1);
  static_assert(STAGE_BYTES % 1024 == 0 && OFF_BLO % 1024 == 0 && OFF_BHI % 1024 == 0 && OFF_E % 16 == 0,
                "swizzle atom alignment (1024 B for 128B, 512 B for 64B)");
  static_assert(E_COL + 4 * STAGES <= TMEM_COLS && HI_COL + BN_HI <= E_COL, "TMEM layout");
  static_assert(SMEM_BYTES <= 232448, "exceeds the 227 KB dynamic shared memory of one CTA");
};

// Bytes CTA `rank` loads towards the leader's full barrier per stage of tile (mb, nb).
__device__ __forceinline__ uint32_t sp2w_stage_bytes(const GemmParams& p, uint32_t mb, uint32_t nb, uint32_t rank) {
  using C = Sp2wCfg;
  const uint32_t m_r = mb * C::BM + rank * C::BM_CTA;
  const uint32_t n_lo = nb * C::BN + rank * (C::BN_LO / 2u);
  const uint32_t n_hi = nb * C::BN + C::BN_LO + rank * (C::BN_HI / 2u);
  return (m_r < p.M ? uint32_t(C::A_BYTES + C::E_BYTES) : 0u) + (n_lo < p.N ? uint32_t(C::BLO_BYTES) : 0u) +
         (n_hi < p.N ? uint32_t(C::BHI_BYTES) : 0u);
}

// Shared-memory matrix descriptor, K-major with 64-byte swizzle (8-row groups 512 B apart).
__device__ __forceinline__ uint64_t smem_desc_sw64(uint32_t saddr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>(16u >> 4) << 16;
  d |= static_cast<uint64_t>(512u >> 4) << 32;
  d |= 1ull << 46;
  d |= 4ull << 61;
  return d;
}
// 128 lanes x 128 bits from shared memory (no-swizzle K-major: 16 B per row, 8-row groups 128 B
// apart) into TMEM of each CTA of the pair.
__device__ __forceinline__ void tmem_cp_128x128b_pair(uint32_t taddr, uint64_t sdesc) {
  asm volatile("tcgen05.cp.cta_group::2.128x128b [%0], %1;" ::"r"(taddr), "l"(sdesc) : "memory");
}

// The two sparse MMAs (64 dense k each) of one stage into one accumulator half.
__device__ __forceinline__ void sp2w_mma_half(uint32_t d_tmem, uint32_t sa, uint32_t sb, uint32_t e_tmem,
                                              uint32_t idesc, uint32_t first_kb) {
#pragma unroll
  for (int kk = 0; kk < 2; ++kk) {
    const uint64_t adesc = smem_desc_sw64(sa + kk * 32);
    const uint64_t bdesc = smem_desc_sw128(sb + kk * 64, 16, 1024);
    const uint32_t acc = (first_kb == 0u && kk == 0) ? 0u : 1u;
    mma_sp_i8_ss_pair(d_tmem, adesc, bdesc, e_tmem + 2 * kk, idesc, acc);
  }
}

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(Sp2wCfg::THREADS, 1)
    gemm_sp2w_kernel(const __grid_constant__ SpParams sp) {
  using C = Sp2wCfg;
  const GemmParams& p = sp.g;
  extern __shared__ uint8_t smem_raw[];
  // the producer thread starts fetching its tensor maps at once, so the fetch overlaps the
  // barrier / TMEM set-up instead of delaying the first loads
  if (threadIdx.x == 0) {
    tma_prefetch_desc(&p.tmA);
    tma_prefetch_desc(&p.tmB);
    tma_prefetch_desc(&p.tmB2);
    tma_prefetch_desc(&p.tmC);
    tma_prefetch_desc(&sp.tmE);
  }
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* const gbase = smem_raw + (base - raw);

  const uint32_t stage_base = base;
  const uint32_t epi_base = base + C::STAGES * C::STAGE_BYTES;
  const uint32_t bar_base = epi_base + C::EPI_BYTES;
  auto full_bar = [&](int s) { return bar_base + 8u * s; };
  auto empty_bar = [&](int s) { return bar_base + 8u * (C::STAGES + s); };
  const uint32_t tfull_bar = bar_base + 8u * (2 * C::STAGES);
  const uint32_t tempty_lo = tfull_bar + 8u;
  const uint32_t tempty_hi = tfull_bar + 16u;
  const uint32_t drain_bar = tfull_bar + 24u;
  const uint32_t slot_off = 8u * C::NBARS;
  volatile uint32_t* tmem_slot = reinterpret_cast<volatile uint32_t*>(gbase + (bar_base - base) + slot_off);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(gbase + (bar_base - base) + slot_off + 4);

  const uint32_t warp = threadIdx.x >> 5;
  const uint32_t lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const uint32_t pair = blockIdx.x >> 1;
  const uint32_t num_pairs = gridDim.x >> 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    mbar_init(tfull_bar, 1);
    mbar_init(tempty_lo, 2 * C::EPI_WARPS);
    mbar_init(tempty_hi, 2 * C::EPI_WARPS);
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    fence_mbar_init();
    fence_proxy_async_smem();
  }
  if (warp == 1) {
    tmem_alloc_pair(smem_u32(const_cast<uint32_t*>(tmem_slot)), C::TMEM_COLS);
    tmem_relinquish_pair();
  }
  if (warp >= 2) {
    // metadata slots start out well formed (every group keeps k 0 and 1); M % 128 == 0 keeps every
    // loaded half-tile wholly in range, so no slot feeds the tensor core uninitialised metadata
    for (uint32_t i = threadIdx.x - 64u; i < C::STAGES * C::E_BYTES / 16; i += 32u * C::EPI_WARPS) {
      const uint32_t st = i / (C::E_BYTES / 16), off = i % (C::E_BYTES / 16);
      st_shared_v4(stage_base + st * C::STAGE_BYTES + C::OFF_E + off * 16u, 0x44444444u, 0x44444444u,
                   0x44444444u, 0x44444444u);
    }
    fence_proxy_async_smem();
  }
  tc_fence_before();
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const uint32_t num_tiles = p.num_m_blk * p.num_n_blk;

  if (warp == 0) {
    // ------------------------------------ TMA producer ------------------------------------
    if (lane == 0) {
      uint32_t stage = 0, phase = 0, issued = 0;
      bool ok = true;
      for (uint32_t tile = pair; ok && tile < num_tiles; tile += num_pairs) {
        uint32_t mb, nb;
        tile_coords(tile, p, mb, nb);
        const uint32_t m_r = mb * C::BM + rank * C::BM_CTA;
        const uint32_t n_lo = nb * C::BN + rank * (C::BN_LO / 2u);
        const uint32_t n_hi = nb * C::BN + C::BN_LO + rank * (C::BN_HI / 2u);
        const uint32_t total = leader ? sp2w_stage_bytes(p, mb, nb, 0) + sp2w_stage_bytes(p, mb, nb, 1) : 0u;
        for (uint32_t kb = 0; kb < p.num_k_blk; ++kb) {
          if (!mbar_wait_cluster(empty_bar(stage), phase ^ 1u, 0x71, abort_flag)) {
            *abort_flag = 1;
            ok = false;
            break;
          }
          const uint32_t sa = stage_base + stage * C::STAGE_BYTES;
          const uint32_t bar = mapa_shared(full_bar(stage), 0);
          if (leader) mbar_arrive_expect_tx(full_bar(stage), total);
          const int32_t kc = static_cast<int32_t>(kb * 64);       // A_c byte column (64 per 128 dense k)
          const int32_t kd = static_cast<int32_t>(kb * C::KD);    // dense k of B
          const int32_t ke = static_cast<int32_t>(kb * 4);        // metadata word (4 per 128 dense k)
          if (m_r < p.M) {
            tma_load_2d_pair(sa, &p.tmA, bar, kc, static_cast<int32_t>(m_r));
            tma_load_2d_pair(sa + C::OFF_E, &sp.tmE, bar, ke, static_cast<int32_t>(m_r));
          }
          if (n_lo < p.N) tma_load_2d_pair(sa + C::OFF_BLO, &p.tmB, bar, kd, static_cast<int32_t>(n_lo));
          if (n_hi < p.N) tma_load_2d_pair(sa + C::OFF_BHI, &p.tmB2, bar, kd, static_cast<int32_t>(n_hi));
          ++issued;
          if (++stage == C::STAGES) { stage = 0; phase ^= 1u; }
        }
      }
      // the last load issued into each slot must land before the pair tears down
      if (leader) {
        const uint32_t tail = issued < (uint32_t)C::STAGES ? issued : (uint32_t)C::STAGES;
        for (uint32_t i = 0; i < tail; ++i) {
          int s = static_cast<int>(stage) - 1 - static_cast<int>(i);
          uint32_t ph = phase;
          while (s < 0) { s += C::STAGES; ph ^= 1u; }
          mbar_wait_cluster(full_bar(s), ph, 0x72, nullptr);
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---------------------------------- MMA issuer (leader) ----------------------------------
    if (leader && lane == 0) {
      uint32_t stage = 0, phase = 0, local = 0;
      bool ok = true;
      const uint32_t d_lo = tmem_base, d_hi = tmem_base + C::HI_COL;
      auto release = [&](uint32_t s) {
        mma_commit_pair(mapa_shared(empty_bar(s), 0));
        mma_commit_pair(mapa_shared(empty_bar(s), 1));
      };
      for (uint32_t tile = pair; ok && tile < num_tiles; tile += num_pairs, ++local) {
        const uint32_t tpar = (local & 1u) ^ 1u;  // previous tile's release phase
        if (!mbar_wait_cluster(tempty_lo, tpar, 0x81, abort_flag)) {
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        bool hi_on = false;
        uint32_t pend = 0;  // stages of this tile whose hi MMAs are still held back
        for (uint32_t kb = 0; kb < p.num_k_blk; ++kb) {
          if (!mbar_wait_cluster(full_bar(stage), phase, 0x82, abort_flag)) {
            *abort_flag = 1;
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = stage_base + stage * C::STAGE_BYTES;
          const uint32_t e_tmem = tmem_base + C::E_COL + 4u * stage;
          // this stage's metadata (128 rows x 32 B) into its own TMEM slot
          tmem_cp_128x128b_pair(e_tmem, smem_desc_noswz(sa + C::OFF_E, 128, 128));
          sp2w_mma_half(d_lo, sa, sa + C::OFF_BLO, e_tmem, C::IDESC_LO, kb);
          if (hi_on) {
            sp2w_mma_half(d_hi, sa, sa + C::OFF_BHI, e_tmem, C::IDESC_HI, kb);
            release(stage);
          } else {
            ++pend;
            bool ready = mbar_test_wait_cluster(tempty_hi, tpar);
            if (!ready && (pend == (uint32_t)C::STAGES || kb + 1 == p.num_k_blk)) {
              if (!mbar_wait_cluster(tempty_hi, tpar, 0x83, abort_flag)) {
                *abort_flag = 1;
                ok = false;
                break;
              }
              ready = true;
            }
            if (ready) {
              tc_fence_after();
              for (uint32_t i = 0; i < pend; ++i) {
                const uint32_t j = kb + 1 - pend + i;  // K block of the held stage
                const uint32_t s = (stage + C::STAGES + 1 - pend + i) % C::STAGES;
                const uint32_t sh = stage_base + s * C::STAGE_BYTES;
                sp2w_mma_half(d_hi, sh, sh + C::OFF_BHI, tmem_base + C::E_COL + 4u * s, C::IDESC_HI, j);
                release(s);
              }
              pend = 0;
              hi_on = true;
            }
          }
          if (++stage == C::STAGES) { stage = 0; phase ^= 1u; }
        }
        if (!ok) break;
        mma_commit_pair(mapa_shared(tfull_bar, 0));
        mma_commit_pair(mapa_shared(tfull_bar, 1));
      }
      mma_commit_pair(mapa_shared(drain_bar, 0));
      mbar_wait(drain_bar, 0, 0x84, nullptr);
    }
    __syncwarp();
  } else {
    // --------------------------------------- epilogue ---------------------------------------
    // Warp w reads TMEM lanes 32 (w % 4) .. +31; the two warps of a lane quadrant split each half:
    // set 0 its first 128 columns, set 1 the rest (128 of lo, 96 of hi). One tcgen05.ld of 128
    // columns per warp and half, release, then 16-row x 128-byte swizzled staging + TMA stores.
    const uint32_t q = warp & 3u;
    const uint32_t set = (warp - 2u) >> 2;
    const uint32_t sbuf = epi_base + (warp - 2u) * C::EPI_BUF;
    uint32_t local = 0;
    for (uint32_t tile = pair; tile < num_tiles; tile += num_pairs, ++local) {
      uint32_t mb, nb;
      tile_coords(tile, p, mb, nb);
      const uint32_t m0 = mb * C::BM + rank * C::BM_CTA;
      const uint32_t n0 = nb * C::BN;
      int ok = 1;
      if (lane == 0) ok = mbar_wait_cluster(tfull_bar, local & 1u, 0x91, abort_flag) ? 1 : 0;
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) {
        if (lane == 0) *abort_flag = 1;
        break;
      }
      tc_fence_after();
#pragma unroll 1
      for (uint32_t half = 0; half < 2; ++half) {
        const uint32_t col0 = half * C::HI_COL + set * 128u;  // TMEM column = tile column
        const uint32_t width = half == 0 ? uint32_t(C::BN_LO) : uint32_t(C::BN_HI);
        uint32_t r[128];
        tmem_ld_32x32b_x128_wait(tmem_base + ((q * 32u) << 16) + col0, r);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(mapa_shared(half == 0 ? tempty_lo : tempty_hi, 0));
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          if (set * 128u + j * C::CHUNK_COLS >= width) break;
          // the warp's 32 rows go out as two 16-row boxes through its 2 KB staging tile
#pragma unroll
          for (uint32_t sub = 0; sub < 2; ++sub) {
            if (lane == 0) bulk_wait_read<0>();  // the previous store has read the staging tile
            __syncwarp();
            if ((lane >> 4) == sub) {
              const uint32_t row_addr = sbuf + (lane & 15u) * 128u;
#pragma unroll
              for (int c = 0; c < 8; ++c)
                st_shared_v4(row_addr + ((static_cast<uint32_t>(c) ^ (lane & 7u)) << 4), r[32 * j + 4 * c],
                             r[32 * j + 4 * c + 1], r[32 * j + 4 * c + 2], r[32 * j + 4 * c + 3]);
              fence_proxy_async_smem();
            }
            __syncwarp();
            const uint32_t xs = n0 + col0 + j * C::CHUNK_COLS, ys = m0 + q * 32u + sub * 16u;
            if (lane == 0) {
              if (xs < p.N && ys < p.M) tma_store_2d(&p.tmC, sbuf, static_cast<int32_t>(xs), static_cast<int32_t>(ys));
              bulk_commit();
            }
          }
        }
      }
    }
    // the staging tiles must have been read before the CTA leaves; the global writes themselves
    // complete on their own and are visible to work ordered after the kernel
    if (lane == 0) bulk_wait_read<0>();
    __syncwarp();
  }

  tc_fence_before();
  cluster_sync();  // no CTA leaves while its peer may still touch its shared memory or TMEM
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, C::TMEM_COLS);
  }
}

}  // namespace zx
