// zx_gemm_sp4.cuh — 2:4 structured-sparse int8 GEMM on CTA pairs with 512 x 224 tiles.
//
// Same operands and contract as zx_gemm_sp2.cuh (reference kernel imma_sp_s8,
// src/examples/imma_sp_s8.zig:144-187, metadata contract src/examples_abi.zig:71-81):
//   A_c M x K/2 int8, meta M x K/32 u32 (reference format, consumed as is), B N x K int8, C int32.
//
// Why a third sparse kernel. The 256 x 224 pair kernel is bound by how fast its operands reach
// each SM (about 55 bytes per clock, set by the bytes a 227 KB ring keeps in flight against the L2
// latency under load), not by the tensor pipe: per 256 dense k each CTA takes in A_c 16 KB,
// B 28 KB and metadata 4 KB for 448 cycles of sparse MMA work. Here a pair tile is two 256-row
// blocks of A sharing one 224-column block of B: per 256 dense k a CTA takes in 2 x (A_c 16 KB +
// metadata 4 KB) + B 28 KB = 68 KB for 896 cycles of MMA work, 29 % fewer bytes per multiply-add,
// with the same bytes in flight (3 stages of 68 KB). 8192^3 is 16 x 37 = 592 tiles: exactly
// 8 waves of the 74 SM pairs.
//
// TMEM (512 columns): block 0's accumulator in columns 0..223, block 1's in 224..447, the
// metadata of the stage being issued at 448 (block 0) and 456 (block 1), 8 columns each (one u32
// per 32 dense k per row, the reference's words in order; tcgen05 ops of one thread execute in
// order, so one slot per block serves every stage). Both accumulators fill TMEM, so the
// hand-over follows the 256 x 512 dense kernel (zx_gemm_tc2w.cuh): the epilogue drains block 0,
// releases it, then block 1; the next tile's block-0 MMAs start as soon as block 0 is free and
// its block-1 MMAs (with their metadata copies) are held back stage by stage until block 1 is
// free. A held stage keeps its operands and metadata in the ring until then.
// Per stage slot (68 KB): A_c block 0 | A_c block 1 (128 rows x 128 B each, 128B swizzle) |
// metadata block 0 | block 1 (2 x [128 rows x 16 B] each, no swizzle) | B (2 x [112 rows x 128 B]).
// Requires M % 128 == 0 and K % 256 == 0; NT only. Every wait is bounded.
#pragma once
#include "zx_gemm_sp2w.cuh"

namespace zx {

struct Sp4Cfg {
  static constexpr int BM = 512, BM_BLK = 256, BM_CTA = 128;  // tile rows, rows per block, per CTA
  static constexpr int BN = 224, BN_CTA = 112;
  static constexpr int KD = 256;                             // dense k per stage
  static constexpr int A_BYTES = BM_CTA * 128;               // one block's A_c rows: 16 KB
  static constexpr int E_HALF = BM_CTA * 16;                 // 128 rows x 16 B (4 words)
  static constexpr int E_BYTES = 2 * E_HALF;                 // one block's metadata: 4 KB
  static constexpr int B_ATOM = BN_CTA * 128;                // one 128-k swizzle atom of B
  static constexpr int B_BYTES = 2 * B_ATOM;
  static constexpr int OFF_A1 = A_BYTES, OFF_E0 = 2 * A_BYTES, OFF_E1 = OFF_E0 + E_BYTES;
  static constexpr int OFF_B = OFF_E1 + E_BYTES;
  static constexpr int STAGE_BYTES = OFF_B + B_BYTES;        // 68 KB
  // Three stages of 256 dense k. Measured slower: six stages of 128 dense k (A_c rows of 64 B in
  // 64B swizzle), 281 us against 247 us at 8192^3.
  static constexpr int STAGES = 3;
  static constexpr int CHUNK_COLS = 32;                      // int32 out: 32 columns per 128 B
  static constexpr int EPI_WARPS = 8;
  static constexpr int EPI_ROWS = 16;                        // rows per staged store
  static constexpr int EPI_BUF = EPI_ROWS * 128;
  static constexpr int EPI_BYTES = EPI_WARPS * EPI_BUF;
  static constexpr uint32_t TMEM_COLS = 512;
  static constexpr uint32_t ACC1_COL = BN;                   // block 1's accumulator
  static constexpr uint32_t E_COL = 2 * BN;                  // + 8 per block
  static constexpr int THREADS = 32 * (2 + EPI_WARPS);
  static constexpr int NBARS = 2 * STAGES + 4;               // full, empty, tfull, tempty0, tempty1, drain
  static constexpr int BAR_BYTES = 8 * NBARS + 16;
  static constexpr int SMEM_BYTES = 1024 + STAGES * STAGE_BYTES + EPI_BYTES + BAR_BYTES;
  static constexpr uint32_t IDESC = idesc_make(2, 1, 1, 0, 0, BM_BLK, BN, /*sparse*/ 1);
  static_assert(STAGE_BYTES % 1024 == 0 && OFF_A1 % 1024 == 0 && OFF_B % 1024 == 0 && B_ATOM % 1024 == 0,
                "1024-byte swizzle alignment");
  static_assert(E_COL + 16 <= TMEM_COLS, "two accumulators and two metadata slots fit TMEM");
  static_assert(SMEM_BYTES <= 232448, "exceeds the 227 KB dynamic shared memory of one CTA");
};

// Bytes CTA `rank` loads towards the leader's full barrier per stage of tile (mb, nb).
__device__ __forceinline__ uint32_t sp4_stage_bytes(const GemmParams& p, uint32_t mb, uint32_t nb, uint32_t rank) {
  using C = Sp4Cfg;
  uint32_t bytes = 0;
  for (uint32_t b = 0; b < 2; ++b)
    if (mb * C::BM + b * C::BM_BLK + rank * C::BM_CTA < p.M) bytes += C::A_BYTES + C::E_BYTES;
  if (nb * C::BN + rank * C::BN_CTA < p.N) bytes += C::B_BYTES;
  return bytes;
}

// One stage's work for one block: its metadata into TMEM, then four M=256 N=224 K=64 sparse MMAs.
__device__ __forceinline__ void sp4_block_stage(uint32_t d_tmem, uint32_t e_tmem, uint32_t sa, uint32_t se,
                                                uint32_t sb, uint32_t first_kb) {
  using C = Sp4Cfg;
  tmem_cp_128x256b_pair(e_tmem, smem_desc_noswz(se, C::E_HALF, 128));
#pragma unroll
  for (int kk = 0; kk < 4; ++kk) {
    const uint64_t adesc = smem_desc_sw128(sa + kk * 32, 16, 1024);
    const uint64_t bdesc = smem_desc_sw128(sb + (kk >> 1) * C::B_ATOM + (kk & 1) * 64, 16, 1024);
    const uint32_t acc = (first_kb == 0u && kk == 0) ? 0u : 1u;
    mma_sp_i8_ss_pair(d_tmem, adesc, bdesc, e_tmem + 2 * kk, C::IDESC, acc);
  }
}

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(Sp4Cfg::THREADS, 1)
    gemm_sp4_kernel(const __grid_constant__ SpParams sp) {
  using C = Sp4Cfg;
  const GemmParams& p = sp.g;
  extern __shared__ uint8_t smem_raw[];
  if (threadIdx.x == 0) {
    tma_prefetch_desc(&p.tmA);
    tma_prefetch_desc(&p.tmB);
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
  const uint32_t tempty0 = tfull_bar + 8u;
  const uint32_t tempty1 = tfull_bar + 16u;
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
    mbar_init(tempty0, 2 * C::EPI_WARPS);
    mbar_init(tempty1, 2 * C::EPI_WARPS);
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
    // metadata regions start out well formed (every group keeps k 0 and 1): a block whose rows lie
    // past M is not loaded (M % 128 == 0 keeps every loaded block wholly in range), and its
    // MMAs then never see uninitialised metadata
    constexpr uint32_t per_stage = 2 * C::E_BYTES / 16;
    for (uint32_t i = threadIdx.x - 64u; i < C::STAGES * per_stage; i += 32u * C::EPI_WARPS)
      st_shared_v4(stage_base + (i / per_stage) * C::STAGE_BYTES + C::OFF_E0 + (i % per_stage) * 16u, 0x44444444u,
                   0x44444444u, 0x44444444u, 0x44444444u);
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
        const uint32_t n_r = nb * C::BN + rank * C::BN_CTA;
        const uint32_t total = leader ? sp4_stage_bytes(p, mb, nb, 0) + sp4_stage_bytes(p, mb, nb, 1) : 0u;
        for (uint32_t kb = 0; kb < p.num_k_blk; ++kb) {
          if (!mbar_wait_cluster(empty_bar(stage), phase ^ 1u, 0x71, abort_flag)) {
            *abort_flag = 1;
            ok = false;
            break;
          }
          const uint32_t sa = stage_base + stage * C::STAGE_BYTES;
          const uint32_t bar = mapa_shared(full_bar(stage), 0);
          if (leader) mbar_arrive_expect_tx(full_bar(stage), total);
#pragma unroll
          for (uint32_t b = 0; b < 2; ++b) {
            const uint32_t m_r = mb * C::BM + b * C::BM_BLK + rank * C::BM_CTA;
            if (m_r < p.M) {
              const uint32_t se = sa + C::OFF_E0 + b * C::E_BYTES;
              tma_load_2d_pair(sa + b * C::A_BYTES, &p.tmA, bar, static_cast<int32_t>(kb * 128),
                               static_cast<int32_t>(m_r));
              tma_load_2d_pair(se, &sp.tmE, bar, static_cast<int32_t>(kb * 8), static_cast<int32_t>(m_r));
              tma_load_2d_pair(se + C::E_HALF, &sp.tmE, bar, static_cast<int32_t>(kb * 8 + 4),
                               static_cast<int32_t>(m_r));
            }
          }
          if (n_r < p.N) {
            tma_load_2d_pair(sa + C::OFF_B, &p.tmB, bar, static_cast<int32_t>(kb * C::KD), static_cast<int32_t>(n_r));
            tma_load_2d_pair(sa + C::OFF_B + C::B_ATOM, &p.tmB, bar, static_cast<int32_t>(kb * C::KD + 128),
                             static_cast<int32_t>(n_r));
          }
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
      const uint32_t d0 = tmem_base, d1 = tmem_base + C::ACC1_COL;
      const uint32_t e0 = tmem_base + C::E_COL, e1 = e0 + 8u;
      auto release = [&](uint32_t s) {
        mma_commit_pair(mapa_shared(empty_bar(s), 0));
        mma_commit_pair(mapa_shared(empty_bar(s), 1));
      };
      auto block1 = [&](uint32_t s, uint32_t kb) {
        const uint32_t sa = stage_base + s * C::STAGE_BYTES;
        sp4_block_stage(d1, e1, sa + C::OFF_A1, sa + C::OFF_E1, sa + C::OFF_B, kb);
      };
      for (uint32_t tile = pair; ok && tile < num_tiles; tile += num_pairs, ++local) {
        const uint32_t tpar = (local & 1u) ^ 1u;  // previous tile's release phase
        if (!mbar_wait_cluster(tempty0, tpar, 0x81, abort_flag)) {
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        bool b1_on = false;
        uint32_t pend = 0;  // stages of this tile whose block-1 work is still held back
        for (uint32_t kb = 0; kb < p.num_k_blk; ++kb) {
          if (!mbar_wait_cluster(full_bar(stage), phase, 0x82, abort_flag)) {
            *abort_flag = 1;
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = stage_base + stage * C::STAGE_BYTES;
          sp4_block_stage(d0, e0, sa, sa + C::OFF_E0, sa + C::OFF_B, kb);
          if (b1_on) {
            block1(stage, kb);
            release(stage);
          } else {
            ++pend;
            bool ready = mbar_test_wait_cluster(tempty1, tpar);
            if (!ready && (pend == (uint32_t)C::STAGES || kb + 1 == p.num_k_blk)) {
              if (!mbar_wait_cluster(tempty1, tpar, 0x83, abort_flag)) {
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
                block1(s, j);
                release(s);
              }
              pend = 0;
              b1_on = true;
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
    // Warp w reads TMEM lanes 32 (w % 4) .. +31; the two warps of a lane quadrant split each
    // block's 224 columns: set 0 its first 128, set 1 the last 96. One tcgen05.ld of 128 columns
    // per warp and block, release, then 16-row x 128-byte swizzled staging + TMA stores.
    const uint32_t q = warp & 3u;
    const uint32_t set = (warp - 2u) >> 2;
    const uint32_t sbuf = epi_base + (warp - 2u) * C::EPI_BUF;
    uint32_t local = 0;
    for (uint32_t tile = pair; tile < num_tiles; tile += num_pairs, ++local) {
      uint32_t mb, nb;
      tile_coords(tile, p, mb, nb);
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
      for (uint32_t b = 0; b < 2; ++b) {
        const uint32_t m0 = mb * C::BM + b * C::BM_BLK + rank * C::BM_CTA;
        const uint32_t col0 = set * 128u;  // tile column of this warp's slice
        uint32_t r[128];
        tmem_ld_32x32b_x128_wait(tmem_base + ((q * 32u) << 16) + b * C::ACC1_COL + col0, r);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(mapa_shared(b == 0 ? tempty0 : tempty1, 0));
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          if (col0 + j * C::CHUNK_COLS >= uint32_t(C::BN)) break;
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
