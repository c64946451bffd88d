// zx_gemm_sp2.cuh — 2:4 structured-sparse int8 GEMM on CTA pairs (tcgen05.mma.sp kind::i8).
//
// BASELINE config 4; reference kernel imma_sp_s8 (src/examples/imma_sp_s8.zig:144-187) with the
// metadata contract of src/examples_abi.zig:71-81: one u32 per row per 32 dense k, nibble j =
// idx0 | idx1 << 2 for the group of 4 dense k at 4j..4j+3 (first kept index in the low 2 bits).
//
//   A_c  M x K/2 int8, kept values in k order (the compressed operand)
//   meta M x K/32 u32  (reference format, consumed as is)
//   B    N x K int8 (K contiguous, "column-major B")
//   C    M x N int32
//
// The tcgen05 int8 sparse metadata in TMEM is one lane per row with consecutive 32-bit columns
// covering consecutive dense k: 2 columns (64 dense k) per MMA, i.e. exactly the reference's u32
// words in order. Per stage (256 dense k) each CTA TMA-loads
//   A_c: 128 rows x 128 B (128B swizzle)   B: 2 x [112 rows x 128 B] (128B swizzle, one per 128 k)
//   E:   2 x [128 rows x 16 B] (row-major, no swizzle: the K-major no-swizzle core-matrix layout)
// and the leader copies E into TMEM with one tcgen05.cp.cta_group::2.128x256b (each CTA's shared
// memory -> its own TMEM) before the stage's four M=256 N=224 K=64 sparse MMAs; tcgen05 ops of
// one thread execute in order, so one TMEM metadata slot serves every stage.
// Pair tile 256 x 224 (TMEM: 2 x 224 accumulator columns + 8 metadata columns <= 512).
#pragma once
#include "zx_gemm_tc2.cuh"

namespace zx {

__device__ __forceinline__ void mma_sp_i8_ss_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                                  uint32_t e_tmem, uint32_t idesc,
                                                  uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %5, 0;\n\t"
      "tcgen05.mma.sp.cta_group::2.kind::i8 [%0], %1, %2, [%3], %4, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(e_tmem), "r"(idesc), "r"(accumulate)
      : "memory");
}
// 128 lanes x 256 bits from shared memory (no-swizzle K-major matrix descriptor: two 16-byte
// core-matrix columns per row, `lbo` bytes apart) into TMEM of each CTA of the pair.
__device__ __forceinline__ void tmem_cp_128x256b_pair(uint32_t taddr, uint64_t sdesc) {
  asm volatile("tcgen05.cp.cta_group::2.128x256b [%0], %1;" ::"r"(taddr), "l"(sdesc) : "memory");
}
// No-swizzle shared-memory matrix descriptor (layout type 0): 8-row x 16-byte core matrices,
// `sbo` bytes between 8-row groups, `lbo` bytes between 16-byte K chunks.
__device__ __forceinline__ uint64_t smem_desc_noswz(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32;
  d |= 1ull << 46;
  return d;
}

struct Sp2Cfg {
  static constexpr int BM = 256, BM_CTA = 128;
  static constexpr int BN = 224, BN_CTA = 112;
  static constexpr int KD = 256;                       // dense k per stage
  static constexpr int A_BYTES = BM_CTA * 128;         // 128 compressed bytes per row
  static constexpr int B_ATOM = BN_CTA * 128;          // one 128-k swizzle atom of B
  static constexpr int B_BYTES = 2 * B_ATOM;
  static constexpr int E_HALF = BM_CTA * 16;           // 128 rows x 16 B (4 words)
  static constexpr int E_BYTES = 2 * E_HALF;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES + E_BYTES;
  static constexpr int STAGES = 4;
  static constexpr int CHUNK_COLS = 32;                // int32 out: 32 columns per 128 B
  static constexpr int NCHUNK = BN / CHUNK_COLS;       // 7
  static constexpr int EPI_WARPS = 4;
  static constexpr int EPI_BUF = 32 * 128;
  static constexpr int EPI_BYTES = EPI_WARPS * 2 * EPI_BUF;
  static constexpr uint32_t TMEM_COLS = 512;
  static constexpr uint32_t E_COL = 2 * BN;            // metadata slot (8 columns)
  static constexpr int THREADS = 192;
  static constexpr int NBARS = 2 * STAGES + 5;
  static constexpr int BAR_BYTES = 8 * NBARS + 16;
  static constexpr int SMEM_BYTES = 1024 + STAGES * STAGE_BYTES + EPI_BYTES + BAR_BYTES;
  static constexpr uint32_t IDESC = idesc_make(2, 1, 1, 0, 0, BM, BN, /*sparse*/ 1);
  static_assert(STAGE_BYTES % 1024 == 0 && B_ATOM % 1024 == 0, "1024-byte swizzle alignment");
  static_assert(E_COL + 8 <= TMEM_COLS, "metadata slot fits beside two accumulators");
  static_assert(SMEM_BYTES <= 232448, "exceeds the 227 KB dynamic shared memory of one CTA");
};

// GemmParams reuse: tmA = A_c (K/2 x M bytes), tmB = B (K x N), tmC = C; tmE passed separately.
struct SpParams {
  GemmParams g;
  CUtensorMap tmE;  // meta: K/32 x M u32
};

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(192, 1)
    gemm_sp2_kernel(const __grid_constant__ SpParams sp) {
  using C = Sp2Cfg;
  const GemmParams& p = sp.g;
  extern __shared__ uint8_t smem_raw[];
  // the producer thread starts fetching its tensor maps at once, so the fetch overlaps the
  // barrier / TMEM set-up instead of delaying the first loads
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
  auto tfull_bar = [&](int b) { return bar_base + 8u * (2 * C::STAGES + b); };
  auto tempty_bar = [&](int b) { return bar_base + 8u * (2 * C::STAGES + 2 + b); };
  const uint32_t drain_bar = bar_base + 8u * (2 * C::STAGES + 4);
  const uint32_t slot_off = 8u * C::NBARS;
  volatile uint32_t* tmem_slot =
      reinterpret_cast<volatile uint32_t*>(gbase + (bar_base - base) + slot_off);
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
    for (int b = 0; b < 2; ++b) {
      mbar_init(tfull_bar(b), 1);
      mbar_init(tempty_bar(b), 2 * C::EPI_WARPS);
    }
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
    // Metadata slots start out holding a well-formed pattern (every group keeps k 0 and 1), so a
    // CTA whose half of the tile lies past M (its loads are skipped) never feeds the tensor core
    // uninitialised metadata. M % 128 == 0 keeps every loaded half wholly in range.
    for (uint32_t i = threadIdx.x - 64u; i < C::STAGES * C::E_BYTES / 16; i += 128u) {
      const uint32_t st = i / (C::E_BYTES / 16), off = i % (C::E_BYTES / 16);
      st_shared_v4(stage_base + st * C::STAGE_BYTES + C::A_BYTES + C::B_BYTES + off * 16u, 0x44444444u,
                   0x44444444u, 0x44444444u, 0x44444444u);
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
        const uint32_t n_r = nb * C::BN + rank * C::BN_CTA;
        auto bytes_of = [&](uint32_t r) {
          const uint32_t mm = mb * C::BM + r * C::BM_CTA, nn = nb * C::BN + r * C::BN_CTA;
          return (mm < p.M ? uint32_t(C::A_BYTES + C::E_BYTES) : 0u) + (nn < p.N ? uint32_t(C::B_BYTES) : 0u);
        };
        const uint32_t total = leader ? bytes_of(0) + bytes_of(1) : 0u;
        for (uint32_t kb = 0; kb < p.num_k_blk; ++kb) {
          if (!mbar_wait_cluster(empty_bar(stage), phase ^ 1u, 0x71, abort_flag)) {
            *abort_flag = 1;
            ok = false;
            break;
          }
          const uint32_t sa = stage_base + stage * C::STAGE_BYTES;
          const uint32_t sb = sa + C::A_BYTES;
          const uint32_t se = sb + C::B_BYTES;
          const uint32_t bar = mapa_shared(full_bar(stage), 0);
          if (leader) mbar_arrive_expect_tx(full_bar(stage), total);
          if (m_r < p.M) {
            tma_load_2d_pair(sa, &p.tmA, bar, static_cast<int32_t>(kb * 128), static_cast<int32_t>(m_r));
            tma_load_2d_pair(se, &sp.tmE, bar, static_cast<int32_t>(kb * 8), static_cast<int32_t>(m_r));
            tma_load_2d_pair(se + C::E_HALF, &sp.tmE, bar, static_cast<int32_t>(kb * 8 + 4),
                             static_cast<int32_t>(m_r));
          }
          if (n_r < p.N) {
            tma_load_2d_pair(sb, &p.tmB, bar, static_cast<int32_t>(kb * C::KD), static_cast<int32_t>(n_r));
            tma_load_2d_pair(sb + C::B_ATOM, &p.tmB, bar, static_cast<int32_t>(kb * C::KD + 128),
                             static_cast<int32_t>(n_r));
          }
          ++issued;
          if (++stage == C::STAGES) { stage = 0; phase ^= 1u; }
        }
      }
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
      const uint32_t e_tmem = tmem_base + C::E_COL;
      for (uint32_t tile = pair; ok && tile < num_tiles; tile += num_pairs, ++local) {
        const uint32_t buf = local & 1u;
        const uint32_t use = local >> 1;
        if (!mbar_wait_cluster(tempty_bar(buf), (use & 1u) ^ 1u, 0x81, abort_flag)) {
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + buf * C::BN;
        for (uint32_t kb = 0; kb < p.num_k_blk; ++kb) {
          if (!mbar_wait_cluster(full_bar(stage), phase, 0x82, abort_flag)) {
            *abort_flag = 1;
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = stage_base + stage * C::STAGE_BYTES;
          const uint32_t sb = sa + C::A_BYTES;
          const uint32_t se = sb + C::B_BYTES;
          // metadata: 128 rows x 32 B -> TMEM columns [E_COL, E_COL + 8) in one copy; the two
          // 16-byte halves of a row sit E_HALF apart (the descriptor's K-direction stride). One
          // 128x256b copy measured ~56 cycles per stage cheaper than two 128x128b copies.
          tmem_cp_128x256b_pair(e_tmem, smem_desc_noswz(se, C::E_HALF, 128));
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            const uint64_t adesc = smem_desc_sw128(sa + kk * 32, 16, 1024);
            const uint64_t bdesc = smem_desc_sw128(sb + (kk >> 1) * C::B_ATOM + (kk & 1) * 64, 16, 1024);
            const uint32_t acc = (kb | static_cast<uint32_t>(kk)) != 0u;
            mma_sp_i8_ss_pair(d_tmem, adesc, bdesc, e_tmem + 2 * kk, C::IDESC, acc);
          }
          mma_commit_pair(mapa_shared(empty_bar(stage), 0));
          mma_commit_pair(mapa_shared(empty_bar(stage), 1));
          if (++stage == C::STAGES) { stage = 0; phase ^= 1u; }
        }
        if (!ok) break;
        mma_commit_pair(mapa_shared(tfull_bar(buf), 0));
        mma_commit_pair(mapa_shared(tfull_bar(buf), 1));
      }
      mma_commit_pair(mapa_shared(drain_bar, 0));
      mbar_wait(drain_bar, 0, 0x83, nullptr);
    }
    __syncwarp();
  } else {
    // --------------------------------------- epilogue ---------------------------------------
    const uint32_t q = warp & 3u;
    const uint32_t ew = warp - 2u;
    uint32_t local = 0, chunk_ctr = 0;
    const uint64_t stream_out = l2_policy_evict_first();
    for (uint32_t tile = pair; tile < num_tiles; tile += num_pairs, ++local) {
      uint32_t mb, nb;
      tile_coords(tile, p, mb, nb);
      const uint32_t m0 = mb * C::BM + rank * C::BM_CTA;
      const uint32_t n0 = nb * C::BN;
      const uint32_t buf = local & 1u;
      const uint32_t use = local >> 1;
      int ok = 1;
      if (lane == 0) ok = mbar_wait_cluster(tfull_bar(buf), use & 1u, 0x91, abort_flag) ? 1 : 0;
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) {
        if (lane == 0) *abort_flag = 1;
        break;
      }
      tc_fence_after();
      const uint32_t t_row = tmem_base + ((q * 32u) << 16) + buf * C::BN;
#pragma unroll 1
      for (int j = 0; j < C::NCHUNK; ++j, ++chunk_ctr) {
        uint32_t w[32];
        tmem_ld_32x32b_x32(t_row + j * 32, w);
        tmem_ld_wait();
        if (j == C::NCHUNK - 1) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive_cluster(mapa_shared(tempty_bar(buf), 0));
        }
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
          if (xs < p.N && ys < p.M)
            tma_store_2d_hint(&p.tmC, sbuf, static_cast<int32_t>(xs), static_cast<int32_t>(ys), stream_out);
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
  cluster_sync();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, C::TMEM_COLS);
  }
}

}  // namespace zx
