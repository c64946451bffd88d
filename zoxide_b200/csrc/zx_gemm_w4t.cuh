// zx_gemm_w4t.cuh — W4A8 for large M on CTA pairs with the weights in tensor memory.
//
// C[M x N] int32 = A[M x K] int8 * W^T, W = N x K signed int4 packed two per byte along K (the
// reference's packS4 order along K; reference kernel imma_s4, src/examples/imma_s4.zig:130-173).
//
// Why. The 256 x 256 pair path (zx_gemm_tc2.cuh, Kind::W4) unpacks s4 -> s8 into shared memory,
// which costs ~170 bytes of shared-memory traffic per clock at the int8 tensor rate (TMA writes,
// unpack reads and writes, MMA reads) against a 128 B/clk port. Here the unpacked weights go to
// TENSOR MEMORY and are the MMA's A operand (tcgen05.mma.cta_group::2 ... [a_tmem], the 2-SM
// "TS" form): shared memory only sees the TMA writes, the unpack reads of packed weights and
// the MMA reads of the activations (~100 B/clk), and each SM takes in ~50 B/clk of operands.
//
// Pair tile: 256 weight rows (C columns n0 .. n0+255) x 256 activation rows (C rows m0 .. m0+255).
// CTA r holds weight rows [n0 + 128 r, +128) (its TMEM lanes: A rows and accumulator rows) and
// activation rows [m0 + 128 r, +128) (its half of the B operand). Per stage of 256 k, CTA r:
//   producer (warp 0)       TMA: packed W 128 rows x 128 B (128B swizzle, local wfull[s]) and
//                           activations 128 rows x 256 B (two 128B-swizzled atoms, counted on
//                           the leader's full[s], cta_group::2 form).
//   transform (warps 6..21) four sets of four warps; set t takes the stages g % 4 == t, which
//                           all land in ring slot t, and writes TMEM weight slot t (64 columns =
//                           256 k of s8): thread = weight row, 8 x 16 B shared loads, s4 -> s8 in
//                           registers, two tcgen05.st of 32 columns, tcgen05.wait::st; then one
//                           thread sends a 16-byte bulk copy to the leader whose completion
//                           counts on the leader's full[s]. With STAGES == SLOTS the producer's
//                           wait for empty[s] (MMAs of the slot's previous use done) already
//                           guarantees the slot is free when new weights arrive for it.
//   MMA (leader warp 1)     full[s] = both CTAs' activation bytes + both CTAs' transform
//                           signals; 8 x tcgen05.mma.cta_group::2.kind::i8 M=256 N=256 K=32 into
//                           the accumulator (TMEM columns 0..255), A = weight slot s; commit
//                           empty[s] in both CTAs; after the tile, commit tfull in both.
//   epilogue (warps 2..5)   warp q owns TMEM lanes 32 q .. +31 (32 weight rows = 32 C columns);
//                           per 32 accumulator columns (32 C rows) one tcgen05.ld.32x32b.x32:
//                           register i is C row m0 + 32 j + i, lanes are consecutive C
//                           columns, so each store instruction writes 128 contiguous bytes.
//                           Releases the accumulator (tempty, count 8) after its last load.
// TMEM: accumulator 256 columns + 4 weight slots x 64 columns = 512. Every wait is bounded; on a
// timeout every role leaves its loop and the pair still deallocates TMEM.
#pragma once
#include "zx_gemm_tc.cuh"
#include "zx_unpack.cuh"
#include "zx_gemm_w4s.cuh"

namespace zx {

struct W4tCfg {
  static constexpr int BW = 256, BW_CTA = 128;  // weight rows (C columns) per pair / per CTA
  static constexpr int BX = 256, BX_CTA = 128;  // activation rows (C rows) per pair / per CTA
  static constexpr int KSTEP = 256;             // k per stage
  static constexpr int W_BYTES = BW_CTA * 128;  // 128 rows x 128 packed bytes
  static constexpr int X_ATOM = BX_CTA * 128;   // 128 rows x 128 bytes (128 k)
  static constexpr int X_BYTES = 2 * X_ATOM;
  static constexpr int STAGE_BYTES = W_BYTES + X_BYTES;  // 48 KB
  static constexpr int STAGES = 4;
  static constexpr int SLOTS = 4;                // TMEM weight slots, slot t <-> ring stage t
  static constexpr int SLOT_COLS = 64;           // 256 k of s8 per TMEM lane
  static constexpr uint32_t ACC_COLS = 256;      // accumulator: one column per activation row
  static constexpr uint32_t TMEM_COLS = 512;
  static constexpr int TX_SETS = 4;
  static constexpr int EPI0 = 2, TX0 = 6;        // first epilogue / transform warp
  static constexpr int THREADS = 32 * (TX0 + 4 * TX_SETS);
  static constexpr uint32_t SIGNAL_BYTES = 16;   // transform-done signal per CTA per stage
  // full[S], empty[S], wfull[S], tfull, tempty, drain; then tmem slot, abort flag, per-set
  // transform outcome words; then 2 x 16-byte signal sinks per stage (leader)
  static constexpr int NBARS = 3 * STAGES + 3;
  static constexpr int BAR_BYTES = 8 * NBARS + 32 + 32 * STAGES + 16;
  static constexpr int SMEM_BYTES = 1024 + STAGES * STAGE_BYTES + BAR_BYTES;
  static constexpr uint32_t IDESC = idesc_make(2, 1, 1, 0, 0, BW, BX);  // s32 += s8 x s8, K-major
  static_assert(STAGES == SLOTS && SLOTS == TX_SETS, "stage t, TMEM slot t and transform set t coincide");
  static_assert(ACC_COLS + SLOTS * SLOT_COLS <= TMEM_COLS, "TMEM budget");
  static_assert(STAGE_BYTES % 1024 == 0, "stage slots keep the 1024-byte swizzle alignment");
  static_assert(SMEM_BYTES <= 232448, "shared memory budget");
};

// A from TMEM (weights), B from shared memory (activations), over the CTA pair.
__device__ __forceinline__ void mma_i8_ts_pair(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc,
                                               uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::i8 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Activation bytes CTA `rank` loads towards the leader's full[s] per stage of tile (xb, wb).
__device__ __forceinline__ uint32_t w4t_x_bytes(const GemmParams& p, uint32_t xb, uint32_t rank) {
  return xb * W4tCfg::BX + rank * W4tCfg::BX_CTA < p.M ? static_cast<uint32_t>(W4tCfg::X_BYTES) : 0u;
}


__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(W4tCfg::THREADS, 1)
    gemm_w4t_kernel(const __grid_constant__ GemmParams p, int32_t* __restrict__ Cout) {
  using C = W4tCfg;
  extern __shared__ uint8_t smem_raw[];
  // the producer thread starts fetching its tensor maps at once, so the fetch overlaps the
  // barrier / TMEM set-up instead of delaying the first loads
  if (threadIdx.x == 0) {
    tma_prefetch_desc(&p.tmA);
    tma_prefetch_desc(&p.tmB);
  }
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* const gbase = smem_raw + (base - raw);
  const uint32_t stage_base = base;
  const uint32_t bar_base = base + C::STAGES * C::STAGE_BYTES;
  auto full_bar = [&](uint32_t s) { return bar_base + 8u * s; };
  auto empty_bar = [&](uint32_t s) { return bar_base + 8u * (C::STAGES + s); };
  auto wfull_bar = [&](uint32_t s) { return bar_base + 8u * (2 * C::STAGES + s); };
  const uint32_t tfull_bar = bar_base + 8u * (3 * C::STAGES);
  const uint32_t tempty_bar = tfull_bar + 8u;
  const uint32_t drain_bar = tfull_bar + 16u;
  const uint32_t slot_off = 8u * C::NBARS;
  volatile uint32_t* tmem_slot = reinterpret_cast<volatile uint32_t*>(gbase + (bar_base - base) + slot_off);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(gbase + (bar_base - base) + slot_off + 4);
  volatile int* tx_ok = reinterpret_cast<volatile int*>(gbase + (bar_base - base) + slot_off + 8);  // [4]
  const uint32_t sink_base = (bar_base + slot_off + 32u + 15u) & ~15u;  // 2 x 16 B per stage

  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const uint32_t pair = blockIdx.x >> 1, num_pairs = gridDim.x >> 1;

  if (threadIdx.x == 0) {
    for (uint32_t s = 0; s < C::STAGES; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
      mbar_init(wfull_bar(s), 1);
    }
    mbar_init(tfull_bar, 1);
    mbar_init(tempty_bar, 2 * 4);
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
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t num_tiles = p.num_m_blk * p.num_n_blk;

  if (warp == 0) {
    // ------------------------------------ TMA producer ------------------------------------
    if (lane == 0) {
      const uint64_t keep = l2_policy_evict_last();  // activations are re-read by every weight tile
      uint32_t stage = 0, phase = 0, issued = 0;
      bool ok = true;
      for (uint32_t tile = pair; ok && tile < num_tiles; tile += num_pairs) {
        uint32_t xb, wb;
        tile_coords(tile, p, xb, wb);
        const uint32_t x_r = xb * C::BX + rank * C::BX_CTA, w_r = wb * C::BW + rank * C::BW_CTA;
        const uint32_t total = leader ? w4t_x_bytes(p, xb, 0) + w4t_x_bytes(p, xb, 1) + 2 * C::SIGNAL_BYTES : 0u;
        for (uint32_t kb = 0; kb < p.num_k_blk; ++kb) {
          if (!mbar_wait_cluster(empty_bar(stage), phase ^ 1u, 0xC1, abort_flag)) {
            *abort_flag = 1;
            ok = false;
            break;
          }
          const uint32_t sw = stage_base + stage * C::STAGE_BYTES, sx = sw + C::W_BYTES;
          const uint32_t bar = mapa_shared(full_bar(stage), 0);
          if (leader) mbar_arrive_expect_tx(full_bar(stage), total);
          if (x_r < p.M) {
            tma_load_2d_pair_hint(sx, &p.tmA, bar, static_cast<int32_t>(kb * 256), static_cast<int32_t>(x_r), keep);
            tma_load_2d_pair_hint(sx + C::X_ATOM, &p.tmA, bar, static_cast<int32_t>(kb * 256 + 128),
                                  static_cast<int32_t>(x_r), keep);
          }
          const bool w_in = w_r < p.N;
          mbar_arrive_expect_tx(wfull_bar(stage), w_in ? C::W_BYTES : 0u);
          if (w_in) tma_load_2d(sw, &p.tmB, wfull_bar(stage), static_cast<int32_t>(kb * 128), static_cast<int32_t>(w_r));
          ++issued;
          if (++stage == C::STAGES) { stage = 0; phase ^= 1u; }
        }
      }
      // the last load issued into each slot must land before the pair tears down
      const uint32_t tail = issued < (uint32_t)C::STAGES ? issued : (uint32_t)C::STAGES;
      for (uint32_t i = 0; i < tail; ++i) {
        int s = static_cast<int>(stage) - 1 - static_cast<int>(i);
        uint32_t ph = phase;
        while (s < 0) { s += C::STAGES; ph ^= 1u; }
        mbar_wait(wfull_bar(s), ph, 0xC2, nullptr);  // this CTA's weight loads
        if (leader) mbar_wait_cluster(full_bar(s), ph, 0xC8, nullptr);  // both CTAs' activation loads
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---------------------------------- MMA issuer (leader) ----------------------------------
    if (leader && lane == 0) {
      uint32_t stage = 0, phase = 0, local = 0;
      bool ok = true;
      for (uint32_t tile = pair; ok && tile < num_tiles; tile += num_pairs, ++local) {
        // one accumulator: the previous tile's epilogue must have read it
        if (!mbar_wait_cluster(tempty_bar, (local & 1u) ^ 1u, 0xC3, abort_flag)) {
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        for (uint32_t kb = 0; kb < p.num_k_blk; ++kb) {
          if (!mbar_wait_cluster(full_bar(stage), phase, 0xC4, abort_flag)) {
            *abort_flag = 1;
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sx = stage_base + stage * C::STAGE_BYTES + C::W_BYTES;
          const uint32_t a_slot = tmem + C::ACC_COLS + stage * C::SLOT_COLS;
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)
            mma_i8_ts_pair(tmem, a_slot + kk * 8u, smem_desc_sw128(sx + (kk / 4) * C::X_ATOM + (kk % 4) * 32, 16, 1024),
                           C::IDESC, (kb | static_cast<uint32_t>(kk)) != 0u ? 1u : 0u);
          mma_commit_pair(mapa_shared(empty_bar(stage), 0));
          mma_commit_pair(mapa_shared(empty_bar(stage), 1));
          if (++stage == C::STAGES) { stage = 0; phase ^= 1u; }
        }
        if (!ok) break;
        mma_commit_pair(mapa_shared(tfull_bar, 0));
        mma_commit_pair(mapa_shared(tfull_bar, 1));
      }
      mma_commit_pair(mapa_shared(drain_bar, 0));
      mbar_wait(drain_bar, 0, 0xC5, nullptr);
    }
    __syncwarp();
  } else if (warp < C::TX0) {
    // --------------------------------------- epilogue ---------------------------------------
    const uint32_t q = warp & 3u;
    uint32_t local = 0;
    for (uint32_t tile = pair; tile < num_tiles; tile += num_pairs, ++local) {
      uint32_t xb, wb;
      tile_coords(tile, p, xb, wb);
      const uint32_t m0 = xb * C::BX;
      const uint32_t n = wb * C::BW + rank * C::BW_CTA + q * 32u + lane;  // this lane's C column
      int ok = 1;
      if (lane == 0) ok = mbar_wait_cluster(tfull_bar, local & 1u, 0xC6, abort_flag) ? 1 : 0;
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) {
        if (lane == 0) *abort_flag = 1;
        break;
      }
      tc_fence_after();
#pragma unroll 1
      for (uint32_t j = 0; j < C::ACC_COLS / 32; ++j) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(tmem + ((q * 32u) << 16) + j * 32u, r);
        tmem_ld_wait();
        if (j == C::ACC_COLS / 32 - 1) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive_cluster(mapa_shared(tempty_bar, 0));
        }
        if (n < p.N) {
          const uint32_t mj = m0 + j * 32u;
#pragma unroll
          for (int i = 0; i < 32; ++i)  // lanes write 32 consecutive C columns of row mj + i
            if (mj + i < p.M) Cout[static_cast<size_t>(mj + i) * p.N + n] = static_cast<int32_t>(r[i]);
        }
      }
    }
    __syncwarp();
  } else {
    // ------------------------------- s4 -> s8 into TMEM A slots -------------------------------
    const uint32_t set = (warp - C::TX0) >> 2;   // 0..3: stages g % 4 == set, ring / TMEM slot set
    const uint32_t q = warp & 3u;                // TMEM lane quarter this warp may access
    const uint32_t tid = threadIdx.x - 32u * (C::TX0 + 4 * set);  // 0..127 within the set
    const uint32_t row = q * 32u + lane;         // weight row within the CTA == TMEM lane
    const uint32_t sw = stage_base + set * C::STAGE_BYTES;  // this set's ring slot (W at its start)
    uint32_t g = 0;
    bool ok = true;
    for (uint32_t tile = pair; ok && tile < num_tiles; tile += num_pairs) {
      for (uint32_t kb = 0; kb < p.num_k_blk; ++kb, ++g) {
        if (g % C::TX_SETS != set) continue;
        // One thread waits and publishes the outcome, so the set's four warps take the same branch
        // and every named barrier below fills.
        if (tid == 0) tx_ok[set] = mbar_wait(wfull_bar(set), (g / C::STAGES) & 1u, 0xC7, abort_flag) ? 1 : 0;
        named_bar_sync(1 + set, 128);
        if (!tx_ok[set]) {
          if (tid == 0) *abort_flag = 1;
          ok = false;
          break;
        }
        const uint32_t src = sw + row * 128u;
        const uint32_t phase = row & 7u;  // 128B swizzle phase of this row
#pragma unroll
        for (int h = 0; h < 2; ++h) {  // 128 k (64 packed bytes) per half
          uint32_t w[16];
#pragma unroll
          for (int c = 0; c < 4; ++c)
            ld_shared_v4(src + ((static_cast<uint32_t>(4 * h + c) ^ phase) << 4), w[4 * c], w[4 * c + 1],
                         w[4 * c + 2], w[4 * c + 3]);
          uint32_t o[32];
#pragma unroll
          for (int j = 0; j < 16; ++j) unpack8(w[j], o[2 * j], o[2 * j + 1]);
          tmem_st_32x32b_x32(tmem + ((q * 32u) << 16) + C::ACC_COLS + set * C::SLOT_COLS + h * 32u, o);
        }
        tmem_st_wait();
        tc_fence_before();
        named_bar_sync(1 + set, 128);  // all 128 weight rows of the slot are in TMEM
        if (tid == 0)  // 16-byte signal into this CTA's sink of the leader, counted on its full[set]
          bulk_copy_s2cluster(mapa_shared(sink_base + (set * 2u + rank) * 16u, 0), sw, C::SIGNAL_BYTES,
                              mapa_shared(full_bar(set), 0));
      }
    }
    __syncwarp();
  }

  tc_fence_before();
  cluster_sync();  // no CTA leaves while its peer may still touch its shared memory or TMEM
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, C::TMEM_COLS);
  }
}

}  // namespace zx
