// zx_gemm_tc2.cuh — 2-SM (cta_group::2) persistent tcgen05 GEMM for sm_100a.
//
// Same operator family and operand layouts as zx_gemm_tc.cuh, but each output tile is 256 x 256
// and is computed by a cluster of two CTAs on two SMs:
//   - CTA rank r of the pair TMA-loads A rows [m0 + 128 r, +128) and B rows (N) [n0 + 128 r, +128)
//     into its own shared memory; completion bytes of both CTAs are counted on the leader's
//     full[s] barrier (the cta_group::2 form of the load).
//   - the leader (rank 0) issues tcgen05.mma.cta_group::2 M=256 N=256, which reads A and B halves
//     from both CTAs and accumulates rows [128 r, +128) into CTA r's TMEM.
//   - the leader's MMA thread signals stage release (empty[s]) and accumulator-ready (tfull[b]) in
//     both CTAs with two plain tcgen05.commit's, one per CTA.
//   - each CTA's four epilogue warps drain their own TMEM half and arrive on the leader's
//     tempty[b] (count 8) through a cluster-scope remote arrive.
// Per SM this halves B's shared-memory footprint and L2->SM traffic relative to the one-SM
// 128 x 256 tile (32 KB instead of 48 KB per 128-byte K step).
//
// Kind::W4 (W4A8, BASELINE config 3; reference imma_s4, src/examples/imma_s4.zig:130-173): B is
// s4 weights packed along K. Each CTA TMA-loads its 128 x 64-byte packed tile into a staging
// slot (wfull[s], local), four transform warps unpack it to s8 in the 128B-swizzled B stage and
// fence the generic-proxy writes for the async proxy; after a named barrier one transform thread
// signals the leader with a 16-byte shared->cluster bulk copy whose complete_tx lands on the
// leader's full[s]. The leader's full[s] therefore completes on A's TMA bytes plus 2 x 16 signal
// bytes, all through the async proxy. (A cluster-scope mbarrier arrive per warp was measured at
// ~2700 cycles of blocking per call — five times the MMA time of a stage.)
// Every wait is bounded as in zx_gemm_tc.cuh.
#pragma once
#include "zx_gemm_tc.cuh"
#include "zx_unpack.cuh"

namespace zx {

// L2 policy of the pair kernel: operands are re-read by many tiles (keep them), C is written
// once (stream it out first). 0 disables the hints.
#ifndef ZX_L2_HINTS
#define ZX_L2_HINTS 1
#endif

// K bytes per operand row per stage = ZX_PAIR_KATOMS x 128 (one 128B-swizzle atom each).
#ifndef ZX_PAIR_KATOMS
#define ZX_PAIR_KATOMS 2
#endif

template <Kind kKind, bool kBMajorMN, Out kOut, int kStages, int kBN = 256>
struct Gemm2Cfg {
  static constexpr bool W4 = kKind == Kind::W4;
  static constexpr int BM = 256;  // rows per CTA pair
  static constexpr int BM_CTA = 128;
  static constexpr int BN = kBN;  // 256, or 224 to even out waves on some shapes
  static constexpr int BN_CTA = kBN / 2;  // B rows (N) loaded by each CTA
  static constexpr int ESZ = kKind == Kind::BF16 ? 2 : 1;
  static constexpr int KATOMS = W4 ? 1 : ZX_PAIR_KATOMS;
  static constexpr int ROWB = 128;                   // bytes per row of one swizzle atom
  static constexpr int BK = KATOMS * ROWB / ESZ;     // K elements per stage
  static constexpr int MMA_K = 32 / ESZ;
  static constexpr int KSTEPS = BK / MMA_K;
  static constexpr int A_ATOM = BM_CTA * ROWB;
  static constexpr int B_ATOM = BN_CTA * ROWB;
  static constexpr int A_BYTES = KATOMS * A_ATOM;
  static constexpr int B_BYTES = KATOMS * B_ATOM;
  static constexpr int W_BYTES = W4 ? BN_CTA * ROWB / 2 : 0;  // packed s4 staging
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES + W_BYTES;
  static constexpr int STAGES = kStages;
  static constexpr int OUT_ESZ = kOut == Out::BF16_SCALED ? 2 : 4;
  static constexpr int CHUNK_COLS = 128 / OUT_ESZ;
  static constexpr int NCHUNK = BN / CHUNK_COLS;
  static constexpr int EPI_WARPS = 4;
#ifndef ZX_TX_WARPS
#define ZX_TX_WARPS 4
#endif
  static constexpr int TX_WARPS = W4 ? ZX_TX_WARPS : 0;  // s4 -> s8 transform warps
  static constexpr int EPI_NBUF = W4 ? 1 : 2;  // staging tiles per epilogue warp
  static constexpr int EPI_BUF = 32 * 128;
  static constexpr int EPI_BYTES = EPI_WARPS * EPI_NBUF * EPI_BUF;
  static constexpr uint32_t TMEM_COLS = 512;
  static constexpr int THREADS = 32 * (2 + EPI_WARPS + TX_WARPS);
  static constexpr int NBARS = 3 * STAGES + 5;  // full, empty, wfull, tfull[2], tempty[2], drain
  static constexpr int BAR_BYTES = 8 * NBARS + 16 + (W4 ? 32 * STAGES + 16 : 0);  // + signal sinks
  static constexpr int SMEM_BYTES = 1024 + STAGES * STAGE_BYTES + EPI_BYTES + BAR_BYTES;
  static constexpr int B_MN_BLOCKS = BN_CTA * ESZ / 128;
  static constexpr int B_MN_BLOCK_BYTES = BK * 128;
  static constexpr uint32_t SIGNAL_BYTES = W4 ? 16 : 0;  // per CTA per stage (transform done)
  static constexpr uint32_t IDESC =
      kKind == Kind::BF16 ? idesc_make(1, 1, 1, 0, kBMajorMN ? 1 : 0, BM, BN)
                          : idesc_make(2, 1, 1, 0, kBMajorMN ? 1 : 0, BM, BN);
  static_assert(!(W4 && kBMajorMN), "W4A8 weights are K-major (packed along K)");
  static_assert(BN == 256 || (BN == 224 && !kBMajorMN && !W4 && CHUNK_COLS == 32),
                "224-column tiles: K-major B, 4-byte output");
  static_assert(2 * BN <= 512, "two accumulators fit in TMEM");
  static_assert(STAGE_BYTES % 1024 == 0, "stage slots keep the 1024-byte swizzle alignment");
  static_assert(SMEM_BYTES <= 232448, "exceeds the 227 KB dynamic shared memory of one CTA");
};

// Bytes CTA `rank` of the pair TMA-loads towards the leader's full[s] for one K step of tile
// (mb, nb). Boxes wholly outside the matrix are not issued: they only feed rows / columns that
// are never stored. W4 weights complete through transform arrivals, not bytes.
template <class C, bool kBMajorMN>
__device__ __forceinline__ uint32_t pair_stage_bytes(const GemmParams& p, uint32_t mb, uint32_t nb,
                                                     uint32_t rank) {
  const uint32_t m_r = mb * C::BM + rank * C::BM_CTA;
  const uint32_t n_r = nb * C::BN + rank * C::BN_CTA;
  uint32_t bytes = m_r < p.M ? C::A_BYTES : 0u;
  if constexpr (C::W4) {
    return bytes;
  } else if constexpr (!kBMajorMN) {
    bytes += n_r < p.N ? C::B_BYTES : 0u;
  } else {
#pragma unroll
    for (int h = 0; h < C::B_MN_BLOCKS; ++h)
      bytes += (n_r + h * (128 / C::ESZ) < p.N) ? C::B_MN_BLOCK_BYTES : 0u;
  }
  return bytes;
}

template <Kind kKind, bool kBMajorMN, Out kOut, int kStages, int kBN>
__global__ void __cluster_dims__(2, 1, 1)
    __launch_bounds__(Gemm2Cfg<kKind, kBMajorMN, kOut, kStages, kBN>::THREADS, 1)
    gemm_tc2_kernel(const __grid_constant__ GemmParams p) {
  using C = Gemm2Cfg<kKind, kBMajorMN, kOut, kStages, kBN>;
  extern __shared__ uint8_t smem_raw[];
  // the producer thread starts fetching its tensor maps at once, so the fetch overlaps the
  // barrier / TMEM set-up instead of delaying the first loads
  if (threadIdx.x == 0) {
    tma_prefetch_desc(&p.tmA);
    tma_prefetch_desc(&p.tmB);
    tma_prefetch_desc(&p.tmC);
  }
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* const gbase = smem_raw + (base - raw);

  const uint32_t stage_base = base;
  const uint32_t epi_base = base + C::STAGES * C::STAGE_BYTES;
  const uint32_t bar_base = epi_base + C::EPI_BYTES;
  auto full_bar = [&](int s) { return bar_base + 8u * s; };
  auto empty_bar = [&](int s) { return bar_base + 8u * (C::STAGES + s); };
  auto wfull_bar = [&](int s) { return bar_base + 8u * (2 * C::STAGES + s); };
  auto tfull_bar = [&](int b) { return bar_base + 8u * (3 * C::STAGES + b); };
  auto tempty_bar = [&](int b) { return bar_base + 8u * (3 * C::STAGES + 2 + b); };
  const uint32_t drain_bar = bar_base + 8u * (3 * C::STAGES + 4);
  const uint32_t slot_off = 8u * C::NBARS;
  volatile uint32_t* tmem_slot =
      reinterpret_cast<volatile uint32_t*>(gbase + (bar_base - base) + slot_off);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(gbase + (bar_base - base) + slot_off + 4);
  volatile int* tx_ok = reinterpret_cast<volatile int*>(gbase + (bar_base - base) + slot_off + 8);
  const uint32_t sink_base = (bar_base + slot_off + 16u + 15u) & ~15u;  // W4: 2 x 16 B per stage

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
      mbar_init(wfull_bar(s), 1);
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
  tc_fence_before();
  cluster_sync();  // barriers of both CTAs initialised, TMEM allocated in both
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const uint32_t num_tiles = p.num_m_blk * p.num_n_blk;

  if (warp == 0) {
    // ------------------------------------ TMA producer ------------------------------------
    if (lane == 0) {
      uint32_t stage = 0, phase = 0, issued = 0;
      bool ok = true;
      const uint64_t keep = l2_policy_evict_last();
      (void)keep;
      for (uint32_t tile = pair; ok && tile < num_tiles; tile += num_pairs) {
        uint32_t mb, nb;
        tile_coords(tile, p, mb, nb);
        const uint32_t m_r = mb * C::BM + rank * C::BM_CTA;
        const uint32_t n_r = nb * C::BN + rank * C::BN_CTA;
        const uint32_t my_bytes = pair_stage_bytes<C, kBMajorMN>(p, mb, nb, rank);
        const uint32_t total_bytes =
            leader ? my_bytes + pair_stage_bytes<C, kBMajorMN>(p, mb, nb, 1) + 2 * C::SIGNAL_BYTES : 0u;
        for (uint32_t kb = 0; kb < p.num_k_blk; ++kb) {
          if (!mbar_wait_cluster(empty_bar(stage), phase ^ 1u, 0x31, abort_flag)) {
            *abort_flag = 1;
            ok = false;
            break;
          }
          const uint32_t sa = stage_base + stage * C::STAGE_BYTES;
          const uint32_t sb = sa + C::A_BYTES;
          const int32_t k0 = static_cast<int32_t>(kb * C::BK);
          const uint32_t bar = mapa_shared(full_bar(stage), 0);
          if (leader) mbar_arrive_expect_tx(full_bar(stage), total_bytes);
#pragma unroll
          for (int a = 0; a < C::KATOMS; ++a) {
            const int32_t ka = k0 + a * (C::ROWB / C::ESZ);
#if ZX_L2_HINTS
            if (m_r < p.M) tma_load_2d_pair_hint(sa + a * C::A_ATOM, &p.tmA, bar, ka, static_cast<int32_t>(m_r), keep);
#else
            if (m_r < p.M) tma_load_2d_pair(sa + a * C::A_ATOM, &p.tmA, bar, ka, static_cast<int32_t>(m_r));
#endif
          }
          if constexpr (C::W4) {
            // packed weights into this CTA's staging slot; the transform warps take it from there
            const uint32_t sw = sb + C::B_BYTES;
            const bool in = n_r < p.N;
            mbar_arrive_expect_tx(wfull_bar(stage), in ? C::W_BYTES : 0u);
            if (in) tma_load_2d(sw, &p.tmB, wfull_bar(stage), k0 / 2, static_cast<int32_t>(n_r));
          } else if constexpr (!kBMajorMN) {
#pragma unroll
            for (int a = 0; a < C::KATOMS; ++a) {
              const int32_t ka = k0 + a * (C::ROWB / C::ESZ);
#if ZX_L2_HINTS
              if (n_r < p.N) tma_load_2d_pair_hint(sb + a * C::B_ATOM, &p.tmB, bar, ka, static_cast<int32_t>(n_r), keep);
#else
              if (n_r < p.N) tma_load_2d_pair(sb + a * C::B_ATOM, &p.tmB, bar, ka, static_cast<int32_t>(n_r));
#endif
            }
          } else {
#pragma unroll
            for (int h = 0; h < C::B_MN_BLOCKS; ++h) {
              const uint32_t x = n_r + h * (128 / C::ESZ);
              if (x < p.N) {
#if ZX_L2_HINTS
                tma_load_2d_pair_hint(sb + h * C::B_MN_BLOCK_BYTES, &p.tmB, bar, static_cast<int32_t>(x), k0, keep);
#else
                tma_load_2d_pair(sb + h * C::B_MN_BLOCK_BYTES, &p.tmB, bar, static_cast<int32_t>(x), k0);
#endif
              }
            }
          }
          ++issued;
          if (++stage == C::STAGES) { stage = 0; phase ^= 1u; }
        }
      }
      // Before the pair may tear down, the last load issued into each slot must have landed:
      // the leader's full barriers count both CTAs' operand bytes, each CTA's wfull barriers its
      // own packed weights (bounded waits; on the normal path they return at once).
      const uint32_t tail = issued < (uint32_t)C::STAGES ? issued : (uint32_t)C::STAGES;
      for (uint32_t i = 0; i < tail; ++i) {
        int s = static_cast<int>(stage) - 1 - static_cast<int>(i);
        uint32_t ph = phase;
        while (s < 0) { s += C::STAGES; ph ^= 1u; }
        if (leader) mbar_wait_cluster(full_bar(s), ph, 0x32, nullptr);
        if constexpr (C::W4) mbar_wait(wfull_bar(s), ph, 0x33, nullptr);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---------------------------------- MMA issuer (leader) ----------------------------------
    if (leader && lane == 0) {
      uint32_t stage = 0, phase = 0, local = 0;
      bool ok = true;
      for (uint32_t tile = pair; ok && tile < num_tiles; tile += num_pairs, ++local) {
        const uint32_t buf = local & 1u;
        const uint32_t use = local >> 1;
        if (!mbar_wait_cluster(tempty_bar(buf), (use & 1u) ^ 1u, 0x41, abort_flag)) {
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + buf * C::BN;
        for (uint32_t kb = 0; kb < p.num_k_blk; ++kb) {
          if (!mbar_wait_cluster(full_bar(stage), phase, 0x42, abort_flag)) {
            *abort_flag = 1;
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = stage_base + stage * C::STAGE_BYTES;
          const uint32_t sb = sa + C::A_BYTES;
#pragma unroll
          for (int kk = 0; kk < C::KSTEPS; ++kk) {
            const uint32_t atom = kk / 4, within = (kk % 4) * 32;
            const uint64_t adesc = smem_desc_sw128(sa + atom * C::A_ATOM + within, 16, 1024);
            uint64_t bdesc;
            if constexpr (!kBMajorMN)
              bdesc = smem_desc_sw128(sb + atom * C::B_ATOM + within, 16, 1024);
            else
              bdesc = smem_desc_sw128(sb + kk * C::MMA_K * 128, C::B_MN_BLOCK_BYTES, 1024);
            const uint32_t acc = (kb | static_cast<uint32_t>(kk)) != 0u;
            if constexpr (kKind == Kind::BF16)
              mma_f16_ss_pair(d_tmem, adesc, bdesc, C::IDESC ^ p.idesc_xor, acc);
            else
              mma_i8_ss_pair(d_tmem, adesc, bdesc, C::IDESC, acc);
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
      mbar_wait(drain_bar, 0, 0x43, nullptr);
    }
    __syncwarp();
  } else if (warp < 2 + C::EPI_WARPS) {
    // --------------------------------------- epilogue ---------------------------------------
    const uint32_t q = warp & 3u;
    const uint32_t ew = warp - 2u;
    const uint32_t row_in_cta = q * 32u + lane;
    uint32_t local = 0;
    uint32_t chunk_ctr = 0;
    const uint64_t stream_out = l2_policy_evict_first();
    (void)stream_out;
    for (uint32_t tile = pair; tile < num_tiles; tile += num_pairs, ++local) {
      uint32_t mb, nb;
      tile_coords(tile, p, mb, nb);
      const uint32_t m0 = mb * C::BM + rank * C::BM_CTA;
      const uint32_t n0 = nb * C::BN;
      const uint32_t buf = local & 1u;
      const uint32_t use = local >> 1;
      int ok = 1;
      if (lane == 0) ok = mbar_wait_cluster(tfull_bar(buf), use & 1u, 0x51, abort_flag) ? 1 : 0;
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) {
        if (lane == 0) *abort_flag = 1;
        break;
      }
      tc_fence_after();
      const uint32_t t_row = tmem_base + ((q * 32u) << 16) + buf * C::BN;
      float rs = 0.f;
      if constexpr (kOut == Out::BF16_SCALED) {
        const uint32_t gm = m0 + row_in_cta;
        rs = gm < p.M ? __ldg(p.row_scale + gm) : 0.f;
      }
#pragma unroll 1
      for (int j = 0; j < C::NCHUNK; ++j, ++chunk_ctr) {
        uint32_t w[32];
        if constexpr (kOut == Out::BF16_SCALED) {
          uint32_t r0[32], r1[32];
          tmem_ld_32x32b_x32(t_row + j * 64, r0);
          tmem_ld_32x32b_x32(t_row + j * 64 + 32, r1);
          tmem_ld_wait();
          if (j == C::NCHUNK - 1) {
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(mapa_shared(tempty_bar(buf), 0));
          }
          const uint32_t nc = n0 + j * 64;
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const uint32_t g0 = nc + 2 * i, g1 = g0 + 1;
            const float c0 = g0 < p.N ? __ldg(p.col_scale + g0) : 0.f;
            const float c1 = g1 < p.N ? __ldg(p.col_scale + g1) : 0.f;
            w[i] = pack_bf16x2(__fmul_rn(__fmul_rn(__int2float_rn(static_cast<int>(r0[2 * i])), rs), c0),
                               __fmul_rn(__fmul_rn(__int2float_rn(static_cast<int>(r0[2 * i + 1])), rs), c1));
          }
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const uint32_t g0 = nc + 32 + 2 * i, g1 = g0 + 1;
            const float c0 = g0 < p.N ? __ldg(p.col_scale + g0) : 0.f;
            const float c1 = g1 < p.N ? __ldg(p.col_scale + g1) : 0.f;
            w[16 + i] = pack_bf16x2(__fmul_rn(__fmul_rn(__int2float_rn(static_cast<int>(r1[2 * i])), rs), c0),
                                    __fmul_rn(__fmul_rn(__int2float_rn(static_cast<int>(r1[2 * i + 1])), rs), c1));
          }
        } else {
          tmem_ld_32x32b_x32(t_row + j * 32, w);
          tmem_ld_wait();
          if (j == C::NCHUNK - 1) {
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(mapa_shared(tempty_bar(buf), 0));
          }
        }
        const uint32_t sbuf =
            epi_base + (ew * C::EPI_NBUF + (C::EPI_NBUF == 2 ? (chunk_ctr & 1u) : 0u)) * C::EPI_BUF;
        if (lane == 0) {
          if constexpr (C::EPI_NBUF == 2)
            bulk_wait_read<1>();
          else
            bulk_wait_read<0>();
        }
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
          if (xs < p.N && ys < p.M) {
#if ZX_L2_HINTS
            tma_store_2d_hint(&p.tmC, sbuf, static_cast<int32_t>(xs), static_cast<int32_t>(ys), stream_out);
#else
            tma_store_2d(&p.tmC, sbuf, static_cast<int32_t>(xs), static_cast<int32_t>(ys));
#endif
          }
          bulk_commit();
        }
      }
    }
    // the staging tiles must have been read before the CTA leaves; the global writes themselves
    // complete on their own and are visible to work ordered after the kernel
    if (lane == 0) bulk_wait_read<0>();
    __syncwarp();
  } else {
    // ----------------------------- s4 -> s8 transform (W4 only) -----------------------------
    if constexpr (C::W4) {
      const uint32_t tid = threadIdx.x - 32u * (2 + C::EPI_WARPS);  // 0..127
      uint32_t stage = 0, phase = 0;
      bool ok = true;
      for (uint32_t tile = pair; ok && tile < num_tiles; tile += num_pairs) {
        uint32_t mb, nb;
        tile_coords(tile, p, mb, nb);
        const bool in = nb * C::BN + rank * C::BN_CTA < p.N;
        for (uint32_t kb = 0; kb < p.num_k_blk; ++kb) {
          // One thread waits and publishes the outcome; every transform warp reads it after the
          // named barrier, so all four take the same branch and the barriers below always fill.
          if (tid == 0) *tx_ok = mbar_wait(wfull_bar(stage), phase, 0x61, abort_flag) ? 1 : 0;
          named_bar_sync(1, 32 * C::TX_WARPS);
          if (!*tx_ok) {
            if (tid == 0) *abort_flag = 1;
            ok = false;
            break;
          }
          const uint32_t sb = stage_base + stage * C::STAGE_BYTES + C::A_BYTES;
          if (in) unpack_s4_stage<C::BN_CTA, 32 * C::TX_WARPS>(sb + C::B_BYTES, sb, tid);
          fence_proxy_async_smem();  // generic-proxy writes -> visible to the async proxy
          named_bar_sync(1, 32 * C::TX_WARPS);
          if (tid == 0)  // 16-byte signal: lands in this CTA's sink slot of the leader, counts on full[s]
            bulk_copy_s2cluster(mapa_shared(sink_base + (stage * 2u + rank) * 16u, 0), sb, C::SIGNAL_BYTES,
                                mapa_shared(full_bar(stage), 0));
          if (++stage == C::STAGES) { stage = 0; phase ^= 1u; }
        }
      }
    }
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
