// zx_gemm_tc2w.cuh — 2-SM (cta_group::2) persistent tcgen05 GEMM with 256 x 512 pair tiles.
//
// Why a second pair kernel. In the 256 x 256 pair kernel (zx_gemm_tc2.cuh) every SM takes in
// 128 A rows + 128 B rows per byte of K for 128 x 256 multiply-adds: 64 bytes per clock at the
// int8 (and bf16) tensor rate. Timestamped runs on B200 show an SM's operand intake saturating
// near 52 bytes per clock (the MMA thread then waits on data ~25 % of the time; with the operand
// reloads switched off the same MMA stream runs at the full tensor rate, and halving the number
// of active SMs does not help, so the limit is per SM, not L2). Here each CTA holds 128 A rows
// and 256 B rows per byte of K for 128 x 512 multiply-adds: 48 bytes per clock, below the intake
// limit, so the loop is tensor-bound.
//
// Layout of one pair tile (rows m0 .. m0+255, columns n0 .. n0+511):
//   - CTA r TMA-loads A rows [m0 + 128 r, +128), B rows [n0 + 128 r, +128) into its "lo" B slot
//     and B rows [n0 + 256 + 128 r, +128) into its "hi" B slot; one 128-byte swizzle atom of K per
//     stage (48 KB per CTA), 4 stages. All bytes of both CTAs complete on the leader's full[s].
//   - the leader issues, per 32-byte K step, tcgen05.mma.cta_group::2 M=256 N=256 into the lo
//     accumulator (TMEM columns 0..255, B from both CTAs' lo slots) and the same into the hi
//     accumulator (columns 256..511, hi slots). TMEM is fully used by one tile's accumulators.
//   - the epilogue drains lo first and releases it (tempty_lo), then hi (tempty_hi). The next
//     tile's lo MMAs start as soon as lo is free; its hi MMAs are held back, stage by stage, until
//     hi is free (the held stages stay in the ring and are released in order afterwards), so the
//     drain of hi overlaps the next tile's MMAs and only the lo drain is exposed.
//   - eight epilogue warps (two per TMEM lane quadrant, splitting the columns) each pull their
//     128 columns of a half into registers with one tcgen05.ld, release the half, and write the
//     values out through a swizzled 32-row staging tile and TMA stores. C is stored without an
//     L2 eviction hint: with one wave of tiles the whole of C is written at the end of the launch,
//     and letting it stay in L2 measured 1-2 % faster than an evict-first hint.
//   - replicas (GemmParams::npeers > 0, int32 out): two copy warps per CTA copy each finished
//     tile of C (this CTA's 128 rows, read back from L2 once its TMA stores have completed) to
//     the same offset of every peer buffer (the other GPUs' C, mapped into this process) with
//     coalesced 16-byte loads and stores: the GEMM and the all-gather of C in one kernel. The
//     epilogue only counts finished tiles, so the NVLink traffic never holds up the accumulator
//     drain, and the copies run behind the MMAs of the following tiles.
// C's row pitch is GemmParams::ldc elements (the C tensor map carries it for the TMA stores).
// K-major A and B only (B stored N x K, the BASELINE "column-major B"). Every wait is bounded as
// in zx_gemm_tc.cuh; on a timeout every role leaves its loop and the pair still deallocates TMEM.
#pragma once
#include "zx_gemm_tc.cuh"
#include "zx_unpack.cuh"

namespace zx {


// kHi = columns of the tile's "hi" half: 256, 224 (256 x 480 tiles) or 208 (256 x 464). Each
// MMA's time is proportional to its N, so where the tile count sets the waves a narrower tile
// shortens the launch: one eighth of 8192^3 (M = 1024, N = 8192) is 64 tiles of 512, or 72 of
// 480 or of 464, in one wave of 74 pairs; 464 is the narrowest width that keeps 72 tiles.
// With kHi = 208 the warps of the hi half's last 80 columns store 64 of them through the
// staging tile and TMA, and the last 16 (a 64-byte piece of each row) with plain stores.
template <Kind kKind, Out kOut, int kStages, int kHi = 256>
struct Gemm2wCfg {
  static constexpr int BM = 256;       // rows per CTA pair
  static constexpr int BM_CTA = 128;
  static constexpr int BNH = 256;      // columns of the lo half (one MMA); the hi half starts here
  static constexpr int BNH_HI = kHi;   // columns of the hi half (one MMA)
  static constexpr int BN = BNH + BNH_HI;  // columns per pair tile
  static constexpr int ESZ = kKind == Kind::BF16 ? 2 : 1;
  static constexpr int ROWB = 128;     // bytes of K per operand row per stage
  static constexpr int BK = ROWB / ESZ;
  static constexpr int MMA_K = 32 / ESZ;
  static constexpr int KSTEPS = BK / MMA_K;  // 4
  static constexpr int A_BYTES = BM_CTA * ROWB;     // 16 KB
  static constexpr int BH_BYTES = 128 * ROWB;       // one B half per CTA: 16 KB (slot size)
  static constexpr int BH_HI_BYTES = (BNH_HI / 2) * ROWB;  // bytes loaded into the hi slot
  static constexpr int STAGE_BYTES = A_BYTES + 2 * BH_BYTES;
  static constexpr int STAGES = kStages;
  static constexpr int OUT_ESZ = kOut == Out::BF16_SCALED ? 2 : 4;
  static constexpr int EPI_WARPS = 8;
  static constexpr int CHUNK_COLS = 128 / OUT_ESZ;  // output columns per 128-byte staging row
  static constexpr int EPI_BUF = 32 * 128;          // one warp's 32-row staging tile
  static constexpr int EPI_BYTES = EPI_WARPS * EPI_BUF;
  // replica copy warps (GemmParams::npeers > 0): 12 warps keep the 168-register budget of 10
  static constexpr int COPY_WARPS = 2;
  static constexpr int COPY0 = 2 + EPI_WARPS;  // first copy warp
  static constexpr int THREADS = 32 * (2 + EPI_WARPS + COPY_WARPS);
  static constexpr uint32_t TMEM_COLS = 512;
  static constexpr int NBARS = 2 * STAGES + 4;  // full, empty, tfull, tempty_lo, tempty_hi, drain
  static constexpr int BAR_BYTES = 8 * NBARS + 16;
  static constexpr int SMEM_BYTES = 1024 + STAGES * STAGE_BYTES + EPI_BYTES + BAR_BYTES;
  static constexpr uint32_t IDESC = kKind == Kind::BF16 ? idesc_make(1, 1, 1, 0, 0, BM, BNH)
                                                        : idesc_make(2, 1, 1, 0, 0, BM, BNH);
  static constexpr uint32_t IDESC_HI = kKind == Kind::BF16 ? idesc_make(1, 1, 1, 0, 0, BM, BNH_HI)
                                                           : idesc_make(2, 1, 1, 0, 0, BM, BNH_HI);
  static_assert(kHi == 256 || ((kHi == 224 || kHi == 208) && kOut != Out::BF16_SCALED),
                "a narrower hi half is stored as 32-column int32 / fp32 chunks (+ one 16-column piece)");
  // columns of the hi half's last store chunk that stay inside the tile (16 for kHi = 208)
  static constexpr int HI_TAIL = (kHi - 128) % CHUNK_COLS;
  static_assert(HI_TAIL == 0 || HI_TAIL == 16, "the hi half ends on a 32- or 16-column boundary");
  static_assert(kKind != Kind::W4, "W4A8 runs on the 256 x 256 pair kernel");
  static_assert(STAGE_BYTES % 1024 == 0, "stage slots keep the 1024-byte swizzle alignment");
  static_assert(SMEM_BYTES <= 232448, "exceeds the 227 KB dynamic shared memory of one CTA");
  static_assert(STAGES * STAGE_BYTES >= EPI_WARPS * 6 * EPI_BUF, "last-tile staging fits in the operand ring");
};

// Bytes CTA `rank` loads towards the leader's full[s] per stage of tile (mb, nb). Boxes wholly
// outside the matrix are not issued: they only feed rows / columns that are never stored.
template <class C>
__device__ __forceinline__ uint32_t wide_stage_bytes(const GemmParams& p, uint32_t mb, uint32_t nb,
                                                     uint32_t rank) {
  const uint32_t m_r = mb * C::BM + rank * C::BM_CTA;
  const uint32_t n_lo = nb * C::BN + rank * 128u;
  const uint32_t n_hi = nb * C::BN + C::BNH + rank * (C::BNH_HI / 2u);
  return (m_r < p.M ? C::A_BYTES : 0u) + (n_lo < p.N ? C::BH_BYTES : 0u) + (n_hi < p.N ? C::BH_HI_BYTES : 0u);
}

// Non-blocking probe of an mbarrier phase (acquire, cluster scope: arrivals come from both CTAs).
__device__ __forceinline__ bool mbar_test_wait_cluster(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.b32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}


// 16-byte load through L2 only (C just written by this CTA's TMA stores).
__device__ __forceinline__ void ld_global_cg_v4(const uint32_t* ptr, uint32_t& a, uint32_t& b, uint32_t& c, uint32_t& d) {
  asm volatile("ld.global.cg.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(a), "=r"(b), "=r"(c), "=r"(d) : "l"(ptr) : "memory");
}
// Orders this thread's completed bulk-async (TMA) writes to global memory before its later
// generic-proxy operations (here: the release of a shared counter that other warps read).
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}
// Bounded wait until a shared counter reaches `need` (wall-clock limit as for mbarrier waits;
// gives up early if the CTA's abort flag is raised, recording `site` on a timeout).
__device__ __forceinline__ bool wait_count_at_least(const volatile uint32_t* cnt, uint32_t need, uint32_t site,
                                                    const volatile int* abort_flag) {
  if (*cnt >= need) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t i = 1;; ++i) {
    if (*cnt >= need) return true;
    if ((i & 63u) == 0) {
      if (*abort_flag) return false;
      if (globaltimer_ns() - t0 > ZX_WAIT_LIMIT_NS) {
        atomicCAS(&g_status, 0u, 0x100u | site);
        return false;
      }
    }
    __nanosleep(64);
  }
}

// 16-byte store to a global address given as an integer (a peer GPU's buffer mapped into this
// process: plain stores travel over NVLink).
__device__ __forceinline__ void st_global_v4_u64(uint64_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.global.v4.b32 [%0], {%1, %2, %3, %4};" ::"l"(addr), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
}

#define ZX_R8(i) "=r"(r[i]), "=r"(r[i + 1]), "=r"(r[i + 2]), "=r"(r[i + 3]), "=r"(r[i + 4]), "=r"(r[i + 5]), \
                 "=r"(r[i + 6]), "=r"(r[i + 7])
// 32 TMEM lanes x 128 consecutive 32-bit columns into registers (thread i <- lane base + i), with
// the wait in the same statement so the registers are valid when it returns.
__device__ __forceinline__ void tmem_ld_32x32b_x128_wait(uint32_t taddr, uint32_t (&r)[128]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x128.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,"
      "%24,%25,%26,%27,%28,%29,%30,%31,%32,%33,%34,%35,%36,%37,%38,%39,%40,%41,%42,%43,%44,%45,%46,"
      "%47,%48,%49,%50,%51,%52,%53,%54,%55,%56,%57,%58,%59,%60,%61,%62,%63,%64,%65,%66,%67,%68,%69,"
      "%70,%71,%72,%73,%74,%75,%76,%77,%78,%79,%80,%81,%82,%83,%84,%85,%86,%87,%88,%89,%90,%91,%92,"
      "%93,%94,%95,%96,%97,%98,%99,%100,%101,%102,%103,%104,%105,%106,%107,%108,%109,%110,%111,%112,"
      "%113,%114,%115,%116,%117,%118,%119,%120,%121,%122,%123,%124,%125,%126,%127}, [%128];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : ZX_R8(0), ZX_R8(8), ZX_R8(16), ZX_R8(24), ZX_R8(32), ZX_R8(40), ZX_R8(48), ZX_R8(56),
        ZX_R8(64), ZX_R8(72), ZX_R8(80), ZX_R8(88), ZX_R8(96), ZX_R8(104), ZX_R8(112), ZX_R8(120)
      : "r"(taddr)
      : "memory");
}
#undef ZX_R8

template <class C, Kind kKind>
__device__ __forceinline__ void wide_mma_stage(uint32_t d_tmem, uint32_t sa, uint32_t sb_half,
                                               uint32_t first_kb, uint32_t idesc) {
#pragma unroll
  for (int kk = 0; kk < C::KSTEPS; ++kk) {
    const uint64_t adesc = smem_desc_sw128(sa + kk * 32, 16, 1024);
    const uint64_t bdesc = smem_desc_sw128(sb_half + kk * 32, 16, 1024);
    const uint32_t acc = (first_kb == 0u && kk == 0) ? 0u : 1u;
    if constexpr (kKind == Kind::BF16)
      mma_f16_ss_pair(d_tmem, adesc, bdesc, idesc, acc);
    else
      mma_i8_ss_pair(d_tmem, adesc, bdesc, idesc, acc);
  }
}

template <Kind kKind, Out kOut, int kStages, int kHi = 256>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(Gemm2wCfg<kKind, kOut, kStages, kHi>::THREADS, 1)
    gemm_tc2w_kernel(const __grid_constant__ GemmParams p) {
  using C = Gemm2wCfg<kKind, kOut, kStages, kHi>;
  extern __shared__ uint8_t smem_raw[];
  // the producer thread starts fetching its tensor maps at once, so the fetch overlaps the
  // barrier / TMEM set-up instead of delaying the first loads
  if (threadIdx.x == 0) {
    tma_prefetch_desc(&p.tmA);
    tma_prefetch_desc(&p.tmB);
    tma_prefetch_desc(&p.tmC);
    if (C::BNH_HI != C::BNH) tma_prefetch_desc(&p.tmB2);
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
  // tiles whose C stores have completed, counted once per epilogue warp (replica copies wait on it)
  volatile uint32_t* stored_cnt = reinterpret_cast<volatile uint32_t*>(gbase + (bar_base - base) + slot_off + 8);

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
    *stored_cnt = 0;
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
  const uint32_t tmem_base = *tmem_slot;
  const uint32_t num_tiles = p.num_m_blk * p.num_n_blk;

  if (warp == 0) {
    // ------------------------------------ TMA producer ------------------------------------
    if (lane == 0) {
      uint32_t stage = 0, phase = 0, issued = 0;
      bool ok = true;
      const uint64_t keep = l2_policy_evict_last();
      for (uint32_t tile = pair; ok && tile < num_tiles; tile += num_pairs) {
        uint32_t mb, nb;
        tile_coords(tile, p, mb, nb);
        const uint32_t m_r = mb * C::BM + rank * C::BM_CTA;
        const uint32_t n_lo = nb * C::BN + rank * 128u;
        const uint32_t n_hi = nb * C::BN + C::BNH + rank * (C::BNH_HI / 2u);
        const uint32_t total = leader ? wide_stage_bytes<C>(p, mb, nb, 0) + wide_stage_bytes<C>(p, mb, nb, 1) : 0u;
        for (uint32_t kb = 0; kb < p.num_k_blk; ++kb) {
          if (!mbar_wait_cluster(empty_bar(stage), phase ^ 1u, 0x71, abort_flag)) {
            *abort_flag = 1;
            ok = false;
            break;
          }
          const uint32_t sa = stage_base + stage * C::STAGE_BYTES;
          const uint32_t sb = sa + C::A_BYTES;
          const int32_t k0 = static_cast<int32_t>(kb * C::BK);
          const uint32_t bar = mapa_shared(full_bar(stage), 0);
          if (leader) mbar_arrive_expect_tx(full_bar(stage), total);
          if (m_r < p.M) tma_load_2d_pair_hint(sa, &p.tmA, bar, k0, static_cast<int32_t>(m_r), keep);
          if (n_lo < p.N) tma_load_2d_pair_hint(sb, &p.tmB, bar, k0, static_cast<int32_t>(n_lo), keep);
          if (n_hi < p.N)  // the hi half's rows come through the map whose box is BNH_HI / 2 rows
            tma_load_2d_pair_hint(sb + C::BH_BYTES, C::BNH_HI == C::BNH ? &p.tmB : &p.tmB2, bar, k0,
                                  static_cast<int32_t>(n_hi), keep);
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
      const uint32_t d_lo = tmem_base, d_hi = tmem_base + C::BNH;
      // Releases stage `s` in both CTAs once every MMA issued so far (hence both halves of s) is done.
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
          wide_mma_stage<C, kKind>(d_lo, sa, sa + C::A_BYTES, kb, C::IDESC ^ p.idesc_xor);
          if (hi_on) {
            wide_mma_stage<C, kKind>(d_hi, sa, sa + C::A_BYTES + C::BH_BYTES, kb, C::IDESC_HI ^ p.idesc_xor);
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
                wide_mma_stage<C, kKind>(d_hi, sh, sh + C::A_BYTES + C::BH_BYTES, j, C::IDESC_HI ^ p.idesc_xor);
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
  } else if (warp < static_cast<uint32_t>(C::COPY0)) {
    // --------------------------------------- epilogue ---------------------------------------
    // Warp w reads TMEM lanes 32 (w % 4) .. +31 (its quadrant); the two warps of a quadrant split
    // each accumulator half's 256 columns: set 0 the first 128, set 1 the last 128. Each warp
    // pulls its 128 columns into registers with one load, releases the half at once, then writes
    // them out through its 32-row x 128-byte staging tile (128B-swizzled) and TMA stores.
    const uint32_t q = warp & 3u;
    const uint32_t set = (warp - 2u) >> 2;
    const uint32_t row_in_cta = q * 32u + lane;
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
      // The pair's last tile: once its MMAs have completed the operand ring is idle, so each
      // epilogue warp also stages through its own 24 KB of the ring (7 buffers in rotation) and
      // its stores stay in flight instead of each waiting for the previous one to be read.
      // (int32 / fp32 out; the scaled-bf16 epilogue keeps one buffer: its registers are spent)
      const bool last = kOut != Out::BF16_SCALED && tile + num_pairs >= num_tiles;
      uint32_t chunk = 0;
      float rs = 0.f;
      if constexpr (kOut == Out::BF16_SCALED) {
        const uint32_t gm = m0 + row_in_cta;
        rs = gm < p.M ? __ldg(p.row_scale + gm) : 0.f;
      }
#pragma unroll 1
      for (uint32_t half = 0; half < 2; ++half) {
        const uint32_t col0 = half * C::BNH + set * 128u;  // accumulator (and tile) column of this slice
        const uint32_t half_end = half == 0 ? uint32_t(C::BNH) : uint32_t(C::BN);
        uint32_t r[128];
        tmem_ld_32x32b_x128_wait(tmem_base + ((q * 32u) << 16) + col0, r);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(mapa_shared(half == 0 ? tempty_lo : tempty_hi, 0));
        constexpr int NCH = 128 / C::CHUNK_COLS;  // 4 (int32 / fp32) or 2 (bf16)
#pragma unroll
        for (int j = 0; j < NCH; ++j) {
          uint32_t w[32];
          if constexpr (kOut == Out::BF16_SCALED) {
            const uint32_t nc = n0 + col0 + j * 64u;
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              const uint32_t g0 = nc + 2 * i, g1 = g0 + 1;
              const float c0 = g0 < p.N ? __ldg(p.col_scale + g0) : 0.f;
              const float c1 = g1 < p.N ? __ldg(p.col_scale + g1) : 0.f;
              w[i] = pack_bf16x2(__fmul_rn(__fmul_rn(__int2float_rn(static_cast<int>(r[64 * j + 2 * i])), rs), c0),
                                 __fmul_rn(__fmul_rn(__int2float_rn(static_cast<int>(r[64 * j + 2 * i + 1])), rs), c1));
            }
          } else {
#pragma unroll
            for (int i = 0; i < 32; ++i) w[i] = r[32 * j + i];
          }
          if constexpr (C::HI_TAIL != 0) {
            // the hi half's last piece: 16 columns (64 bytes of this lane's row) inside the tile;
            // a 32-column TMA box would overwrite the next tile's first 16 columns
            if (col0 + (j + 1) * C::CHUNK_COLS > half_end) {
              if (col0 + j * C::CHUNK_COLS < half_end) {
                const uint32_t gm = m0 + row_in_cta, gn = n0 + col0 + j * C::CHUNK_COLS;
                if (gm < p.M) {
                  uint32_t* const dst = const_cast<uint32_t*>(p.c_base) + static_cast<uint64_t>(gm) * p.ldc + gn;
#pragma unroll
                  for (int v = 0; v < 4; ++v) {
                    const uint32_t c = gn + 4u * v;
                    if (c + 3u < p.N) {
                      st_global_v4_u64(reinterpret_cast<uint64_t>(dst + 4 * v), w[4 * v], w[4 * v + 1],
                                       w[4 * v + 2], w[4 * v + 3]);
                    } else {
#pragma unroll
                      for (int e = 0; e < 4; ++e)
                        if (c + e < p.N) dst[4 * v + e] = w[4 * v + e];
                    }
                  }
                }
                if (p.npeers) {  // other warps read C back once the tile is counted as stored
                  __threadfence();
                  __syncwarp();
                }
              }
              continue;
            }
          }
          uint32_t buf = sbuf;
          if (last) {
            // buffer b was last used 7 stores ago (b = 0, the warp's own staging tile, at the
            // earliest 7 stores ago including the previous tile's): at most 6 may still be reading
            const uint32_t b = (chunk + 1u) % 7u;
            buf = b == 0 ? sbuf : stage_base + (warp - 2u) * (6u * C::EPI_BUF) + (b - 1u) * C::EPI_BUF;
            if (lane == 0) bulk_wait_read<6>();
          } else if (lane == 0) {
            bulk_wait_read<0>();  // the previous store has read the staging tile
          }
          ++chunk;
          __syncwarp();
          const uint32_t row_addr = buf + lane * 128u;
#pragma unroll
          for (int c = 0; c < 8; ++c)
            st_shared_v4(row_addr + ((static_cast<uint32_t>(c) ^ (lane & 7u)) << 4), w[4 * c], w[4 * c + 1],
                         w[4 * c + 2], w[4 * c + 3]);
          fence_proxy_async_smem();
          __syncwarp();
          const uint32_t xs = n0 + col0 + j * C::CHUNK_COLS, ys = m0 + q * 32u;
          if (lane == 0) {
            if (xs < p.N && ys < p.M && col0 + j * C::CHUNK_COLS < half_end)
              tma_store_2d(&p.tmC, buf, static_cast<int32_t>(xs), static_cast<int32_t>(ys));
            bulk_commit();
          }
        }
      }
      if (p.npeers) {  // count the tile once this warp's stores of it are complete and visible
        if (lane == 0) {
          bulk_wait<0>();
          fence_proxy_async_global();
          __threadfence_block();
          atomicAdd(const_cast<uint32_t*>(stored_cnt), 1u);
        }
        __syncwarp();
      }
    }
    // the staging tiles must have been read before the CTA leaves; the global writes themselves
    // complete on their own and are visible to work ordered after the kernel
    if (lane == 0) bulk_wait_read<0>();
    __syncwarp();
  } else {
    // ----------------------------- replica copies (npeers > 0) -----------------------------
    // Tile by tile, once all eight epilogue warps have counted the tile's C stores complete,
    // copy this CTA's rows of it from C (still in L2) to every peer buffer at the same offset:
    // warp c of the two takes row groups c, c + 2, ... of CROWS rows; a group's 4 CROWS loads of
    // 16 bytes per lane (each load instruction a coalesced 512-byte read) are in flight before its
    // stores.
    if (kOut != Out::BF16_SCALED && p.npeers) {  // replicas are int32 / fp32 only
      constexpr uint32_t CROWS = 8;
      const uint32_t cw = warp - C::COPY0;
      uint32_t local = 0;
      for (uint32_t tile = pair; tile < num_tiles; tile += num_pairs, ++local) {
        uint32_t mb, nb;
        tile_coords(tile, p, mb, nb);
        const uint32_t m0 = mb * C::BM + rank * C::BM_CTA;
        const uint32_t n0 = nb * C::BN;
        const uint32_t need = static_cast<uint32_t>(C::EPI_WARPS) * (local + 1u);
        int ok = 1;
        if (lane == 0) ok = wait_count_at_least(stored_cnt, need, 0x95, abort_flag) ? 1 : 0;
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (!ok) break;
        __threadfence_block();
        const uint32_t rows = m0 < p.M ? (p.M - m0 < 128u ? p.M - m0 : 128u) : 0u;
        const uint32_t cols = n0 < p.N ? (p.N - n0 < uint32_t(C::BN) ? p.N - n0 : uint32_t(C::BN)) : 0u;
        for (uint32_t r0 = cw * CROWS; r0 < rows; r0 += CROWS * C::COPY_WARPS) {
          uint32_t v[CROWS][4][4];
#pragma unroll
          for (int rr = 0; rr < static_cast<int>(CROWS); ++rr)
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              const uint32_t row = r0 + rr, col = 4u * (lane + 32u * k);
              if (row < rows && col < cols)
                ld_global_cg_v4(p.c_base + (static_cast<uint64_t>(m0 + row) * p.ldc + n0 + col), v[rr][k][0],
                                v[rr][k][1], v[rr][k][2], v[rr][k][3]);
            }
#pragma unroll
          for (int rr = 0; rr < static_cast<int>(CROWS); ++rr)
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              const uint32_t row = r0 + rr, col = 4u * (lane + 32u * k);
              if (row < rows && col < cols) {
                const uint64_t off = (static_cast<uint64_t>(m0 + row) * p.ldc + n0 + col) * 4u;
                for (uint32_t pi = 0; pi < p.npeers; ++pi)
                  st_global_v4_u64(p.peer_c[pi] + off, v[rr][k][0], v[rr][k][1], v[rr][k][2], v[rr][k][3]);
              }
            }
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
