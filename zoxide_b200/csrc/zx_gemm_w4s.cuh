// zx_gemm_w4s.cuh — W4A8 for few activation rows (M <= 64, the decode-like BASELINE config 3'):
// HBM-bound on the packed int4 weights, so the kernel is built to stream W once at full rate.
//
// Roles are swapped relative to the large-M path: the weights are the MMA's A operand (M = 128
// weight rows per CTA) and live in TENSOR MEMORY, the activations are the B operand (N = NX,
// 16..64 rows) in shared memory. Per K step of 256:
//   producer (warp 0)        TMA: packed W tile 128 rows x 128 B (128B swizzle) + X tile NX x 256 B
//                            (two 128B-swizzled atoms) into stage s; full[s] counts both. 128-byte
//                            row pieces: a read-bandwidth probe over this matrix on B200 measured
//                            2.49 TB/s with 64-byte row pieces and 3.70 TB/s with 128-byte ones.
//   transform (warps ...)    four sets of four warps, set t for steps g % 4 == t (TMEM slot t);
//                            thread = one weight row: 8 x 16 B shared loads (conflict-free under
//                            the 128B swizzle), s4 -> s8 in registers, two tcgen05.st of 32 columns
//                            into TMEM slot g % 4; afull[slot] after tcgen05.wait::st.
//   MMA issuers (1 thread)   8 x tcgen05.mma kind::i8 [acc], [A slot + 8 kk], X desc; commit
//                            empty[s] (frees the smem stage and, four steps later, the TMEM slot).
//   epilogue (warps 18..21)  tcgen05.ld of NX accumulator columns per weight row; exact int32
//                            red.global.add into C (zeroed by the launcher).
// Work: the (weight tile, K step) space split into equal contiguous ranges, one per CTA (see
// W4sRange), so every SM streams the same share of W.
// Unpacked weights never touch shared memory: shared traffic per step is the TMA writes plus
// 8 KB of transform reads plus the small X reads.
#pragma once
#include "zx_gemm_tc.cuh"
#include "zx_unpack.cuh"

namespace zx {

// Loads are issued in groups of ZX_W4S_BURST stages; 1 (each stage as soon as it is free) measured
// fastest on B200 (M = 16: 40.0 us vs 42.0 us with groups of 4).
#ifndef ZX_W4S_BURST
#define ZX_W4S_BURST 1
#endif

struct W4sParams {
  CUtensorMap tmW;  // packed W: N rows x K/2 bytes
  CUtensorMap tmX;  // activations: M rows x K bytes
  int32_t* C;       // M x N int32
  // Split-tile partial sums. Null: C is zeroed by the launcher and every unit adds its partial
  // sums into C with exact int32 atomics. Non-null (a caller workspace, zero on first use): a
  // unit that covers a whole weight tile stores C directly; the units of a tile split between
  // CTAs write their partials to ws_part and count themselves in ws_cnt[tile]; the last one to
  // count adds the others' partials to its own, stores C and resets the counter to zero.
  int32_t* ws_part;   // [2 x gridDim.x slots][NX rows][128 columns] int32
  uint32_t* ws_cnt;   // [n_tiles] arrival counters
  uint32_t M, N, K;
  uint32_t n_tiles, nk;  // 128-row weight tiles, K steps of 256
};

// Workspace bytes of the split-tile protocol for NX activation columns and `ctas` CTAs.
__host__ __device__ constexpr uint64_t w4s_ws_part_bytes(uint32_t nx, uint32_t ctas) {
  return 2ull * ctas * nx * 128u * 4u;
}

// CTA whose step range contains global step l (ranges: [total*b/G, total*(b+1)/G)).
__device__ __forceinline__ uint32_t w4s_cta_of(uint64_t l, uint64_t total, uint32_t G) {
  return static_cast<uint32_t>(((l + 1) * G - 1) / total);
}

// Work split: the (weight tile, K step) space, n_tiles x nk steps in tile-major order, is cut
// into gridDim.x contiguous ranges of equal length (+-1 step); a CTA's range is a few "units"
// (maximal runs within one weight tile), each flushed into C (see W4sParams::ws_part).
struct W4sUnit {
  uint32_t nt, kb0, kb1;
};
struct W4sRange {
  uint32_t l, l1, nk;
  __device__ W4sRange(const W4sParams& p) : nk(p.nk) {
    const uint64_t total = uint64_t(p.n_tiles) * p.nk;
    l = static_cast<uint32_t>(total * blockIdx.x / gridDim.x);
    l1 = static_cast<uint32_t>(total * (blockIdx.x + 1) / gridDim.x);
  }
  __device__ bool next(W4sUnit& u) {
    if (l >= l1) return false;
    u.nt = l / nk;
    u.kb0 = l % nk;
    u.kb1 = min(nk, u.kb0 + (l1 - l));
    l += u.kb1 - u.kb0;
    return true;
  }
};

template <int NX>
struct W4sCfg {
  static constexpr int KSTEP = 256;             // k per step
  static constexpr int W_BYTES = 128 * 128;     // 128 weight rows x 128 packed bytes (256 k)
  static constexpr int X_ATOM = NX * 128;       // NX activation rows x 128 bytes (128 k)
  static constexpr int X_BYTES = 2 * X_ATOM;
  static constexpr int STAGE_BYTES = W_BYTES + X_BYTES;
  // deep ring: the kernel is bound by how many weight bytes each SM keeps in flight
  static constexpr int STAGES = NX <= 32 ? 8 : 4;
  static constexpr int SLOTS = 4;               // TMEM A slots of 64 columns (256 k of s8)
  static constexpr int SLOT_COLS = 64;
  static constexpr uint32_t ACC_COL = SLOTS * SLOT_COLS;  // accumulators: [buffer][issuer] x NX columns
  static constexpr uint32_t TMEM_COLS = 512;
  static constexpr int TX_SETS = 4;              // transform warp sets; set t owns steps g % 4 == t
  static constexpr int TX_WARPS = 4 * TX_SETS;
  // MMA issuers take steps round-robin into their own accumulators (as many as TMEM holds)
  static constexpr int MMA_WARPS = NX <= 32 ? 4 : 2;
  static constexpr int TX0 = 1 + MMA_WARPS;      // first transform warp
  static constexpr int EPI0 = TX0 + TX_WARPS;    // first epilogue warp
  static constexpr int THREADS = 32 * (EPI0 + 4);
  static constexpr int NBARS = 2 * STAGES + SLOTS + 5;  // full, empty, afull, tfull[2], tempty[2], drain
  static constexpr int SMEM_BYTES = 1024 + STAGES * STAGE_BYTES + 8 * NBARS + 16;
  static constexpr uint32_t IDESC = idesc_make(2, 1, 1, 0, 0, 128, NX);
  static_assert(NX % 16 == 0 && NX >= 16 && NX <= 64, "NX in {16, 32, 48, 64}");
  static_assert(STAGE_BYTES % 1024 == 0, "stage slots keep 1024-byte swizzle alignment");
  static_assert(ACC_COL + 2 * MMA_WARPS * NX <= TMEM_COLS, "TMEM budget");
  // The transform of step g waits for empty[(g - SLOTS) % STAGES] at the phase of step g - SLOTS.
  // The next step that commits that barrier is g - SLOTS + STAGES; it must belong to the same
  // transform set as g (which runs its steps in order), or that later commit could flip the
  // phase before the wait is made.
  static_assert(STAGES >= SLOTS && (STAGES - SLOTS) % TX_SETS == 0, "slot-reuse wait is phase-safe");
  static_assert(SLOTS == TX_SETS, "set t owns TMEM slot t");
  // Issuer j takes the steps g with g % MMA_WARPS == j. With MMA_WARPS dividing SLOTS, every fill
  // of a TMEM slot (steps s, s + SLOTS, ...) is consumed by one issuer, in order, so its parity
  // wait on afull[slot] always refers to the next fill (a fill cannot run two ahead: the slot
  // is refilled only after the MMAs of its previous fill have completed).
  static_assert(SLOTS % MMA_WARPS == 0, "each slot's fills are consumed in order by one issuer");
  static_assert(SMEM_BYTES <= 232448, "shared memory budget");
};

__device__ __forceinline__ void mma_i8_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc,
                                          uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void tmem_st_32x32b_x32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]),
      "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]),
      "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
__device__ __forceinline__ void tmem_ld_32x32b_x16(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
__device__ __forceinline__ void red_add_s32(int32_t* p, int32_t v) {
  asm volatile("red.global.add.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

template <int NX>
__global__ void __launch_bounds__(W4sCfg<NX>::THREADS, 1) gemm_w4s_kernel(const __grid_constant__ W4sParams p) {
  using C = W4sCfg<NX>;
  extern __shared__ uint8_t smem_raw[];
  // the producer thread starts fetching its tensor maps at once, so the fetch overlaps the
  // barrier / TMEM set-up instead of delaying the first loads
  if (threadIdx.x == 0) {
    tma_prefetch_desc(&p.tmW);
    tma_prefetch_desc(&p.tmX);
  }
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* const gbase = smem_raw + (base - raw);
  const uint32_t bar_base = base + C::STAGES * C::STAGE_BYTES;
  auto full_bar = [&](uint32_t s) { return bar_base + 8u * s; };
  auto empty_bar = [&](uint32_t s) { return bar_base + 8u * (C::STAGES + s); };
  auto afull_bar = [&](uint32_t a) { return bar_base + 8u * (2 * C::STAGES + a); };
  auto tfull_bar = [&](uint32_t b) { return bar_base + 8u * (2 * C::STAGES + C::SLOTS + b); };
  auto tempty_bar = [&](uint32_t b) { return bar_base + 8u * (2 * C::STAGES + C::SLOTS + 2 + b); };
  const uint32_t drain_bar = bar_base + 8u * (2 * C::STAGES + C::SLOTS + 4);
  volatile uint32_t* tmem_slot = reinterpret_cast<volatile uint32_t*>(gbase + (bar_base - base) + 8u * C::NBARS);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(gbase + (bar_base - base) + 8u * C::NBARS + 4);
  volatile int* last_flag = reinterpret_cast<volatile int*>(gbase + (bar_base - base) + 8u * C::NBARS + 8);

  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (uint32_t s = 0; s < C::STAGES; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    for (uint32_t a = 0; a < C::SLOTS; ++a) mbar_init(afull_bar(a), 4);
    for (uint32_t b = 0; b < 2; ++b) {
      mbar_init(tfull_bar(b), C::MMA_WARPS);
      mbar_init(tempty_bar(b), 4);
    }
    mbar_init(drain_bar, C::MMA_WARPS);
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
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------ TMA producer ------------------------------------
    if (lane == 0) {
      const uint64_t stream_w = l2_policy_evict_first();  // W is read exactly once
      uint32_t g = 0;
      bool ok = true;
      W4sRange range(p);
      W4sUnit un;
      while (ok && range.next(un)) {
        const uint32_t steps = un.kb1 - un.kb0;
        // Loads go out in groups of ZX_W4S_BURST consecutive K steps, issued back to back once
        // that many stages are free.
        for (uint32_t i0 = 0; ok && i0 < steps; i0 += ZX_W4S_BURST) {
          const uint32_t nb = min(static_cast<uint32_t>(ZX_W4S_BURST), steps - i0);
          for (uint32_t j = 0; j < nb; ++j) {
            const uint32_t gj = g + j;
            if (!mbar_wait(empty_bar(gj % C::STAGES), ((gj / C::STAGES) & 1u) ^ 1u, 0xB1, abort_flag)) {
              *abort_flag = 1;
              ok = false;
              break;
            }
          }
          if (!ok) break;
          for (uint32_t j = 0; j < nb; ++j, ++g) {
            const uint32_t s = g % C::STAGES;
            const uint32_t kb = un.kb0 + i0 + j;
            const uint32_t sw = base + s * C::STAGE_BYTES, sx = sw + C::W_BYTES;
            mbar_arrive_expect_tx(full_bar(s), C::STAGE_BYTES);
            tma_load_2d_hint(sw, &p.tmW, full_bar(s), static_cast<int32_t>(kb * 128), static_cast<int32_t>(un.nt * 128), stream_w);
            tma_load_2d(sx, &p.tmX, full_bar(s), static_cast<int32_t>(kb * 256), 0);
            tma_load_2d(sx + C::X_ATOM, &p.tmX, full_bar(s), static_cast<int32_t>(kb * 256 + 128), 0);
          }
        }
      }
      // drain: the last load issued into each slot must have landed
      const uint32_t tail = g < (uint32_t)C::STAGES ? g : (uint32_t)C::STAGES;
      for (uint32_t i = 1; i <= tail; ++i) {
        const uint32_t gg = g - i;
        mbar_wait(full_bar(gg % C::STAGES), (gg / C::STAGES) & 1u, 0xB2, nullptr);
      }
    }
    __syncwarp();
  } else if (warp < C::TX0) {
    // ----------------------------- MMA issuers (one thread each) -----------------------------
    // Issuer j takes the steps g with g % MMA_WARPS == j (g counts this CTA's steps across its
    // units) into its own accumulator of the unit: an A-from-TMEM MMA was measured at ~100 cycles
    // of issue each, so several issuers keep more in flight. The epilogue adds the accumulators.
    const uint32_t j = warp - 1u;
    if (lane == 0) {
      uint32_t g = 0, local = 0;
      bool ok = true;
      W4sRange range(p);
      W4sUnit un;
      for (; ok && range.next(un); ++local) {
        const uint32_t buf = local & 1u, use = local >> 1;
        if (!mbar_wait(tempty_bar(buf), (use & 1u) ^ 1u, 0xB3, abort_flag)) { *abort_flag = 1; break; }
        tc_fence_after();
        const uint32_t d = tmem + C::ACC_COL + (buf * C::MMA_WARPS + j) * NX;
        bool first = true;
        for (uint32_t i = 0; i < un.kb1 - un.kb0; ++i, ++g) {
          if (g % C::MMA_WARPS != j) continue;
          const uint32_t s = g % C::STAGES, slot = g % C::SLOTS;
          if (!mbar_wait(afull_bar(slot), (g / C::SLOTS) & 1u, 0xB4, abort_flag)) { *abort_flag = 1; ok = false; break; }
          tc_fence_after();
          const uint32_t sx = base + s * C::STAGE_BYTES + C::W_BYTES;
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)
            mma_i8_ts(d, tmem + slot * C::SLOT_COLS + kk * 8u,
                      smem_desc_sw128(sx + (kk / 4) * C::X_ATOM + (kk % 4) * 32, 16, 1024), C::IDESC,
                      (!first || kk != 0) ? 1u : 0u);
          first = false;
          mma_commit(empty_bar(s));
        }
        if (!ok) break;
        mma_commit(tfull_bar(buf));
      }
      mma_commit(drain_bar);
      mbar_wait(drain_bar, 0, 0xB5, nullptr);
    }
    __syncwarp();
  } else if (warp < C::EPI0) {
    // ------------------------------- s4 -> s8 into TMEM A slots -------------------------------
    // Four sets of four warps; set t handles the steps g with g % 4 == t (TMEM slot t), so four
    // steps' unpack / tcgen05.st / wait chains run at once; a slot is refilled once the MMAs of
    // step g - 4 have completed. Within a set, warp w covers TMEM lane quarter w % 4 (the quarter
    // a warp may access).
    const uint32_t q = warp & 3u;
    const uint32_t set = (warp - C::TX0) >> 2;
    const uint32_t row = q * 32u + lane;  // weight row within the tile == TMEM lane
    uint32_t g = 0;
    bool ok = true;
    W4sRange range(p);
    W4sUnit un;
    while (ok && range.next(un)) {
      for (uint32_t i = 0; i < un.kb1 - un.kb0; ++i, ++g) {
        const uint32_t s = g % C::STAGES, slot = g % C::SLOTS;
        if (g % C::TX_SETS != set) continue;
        int w_ok = 1;
        if (lane == 0) {
          w_ok = mbar_wait(full_bar(s), (g / C::STAGES) & 1u, 0xB6, abort_flag);
          // TMEM slot reuse: the MMAs of step g - SLOTS (same slot) must have completed
          if (w_ok && g >= C::SLOTS) {
            const uint32_t gp = g - C::SLOTS;
            w_ok = mbar_wait(empty_bar(gp % C::STAGES), (gp / C::STAGES) & 1u, 0xB7, abort_flag);
          }
        }
        w_ok = __shfl_sync(0xffffffffu, w_ok, 0);
        if (!w_ok) { if (lane == 0) *abort_flag = 1; ok = false; break; }
        tc_fence_after();
        const uint32_t src = base + s * C::STAGE_BYTES + row * 128u;
        const uint32_t sw = row & 7u;  // 128B swizzle phase of this row
#pragma unroll
        for (int h = 0; h < 2; ++h) {  // 128 k (64 packed bytes) per half
          uint32_t w[16];
#pragma unroll
          for (int c = 0; c < 4; ++c)
            ld_shared_v4(src + ((static_cast<uint32_t>(4 * h + c) ^ sw) << 4), w[4 * c], w[4 * c + 1], w[4 * c + 2],
                         w[4 * c + 3]);
          uint32_t o[32];
#pragma unroll
          for (int j = 0; j < 16; ++j) unpack8(w[j], o[2 * j], o[2 * j + 1]);
          tmem_st_32x32b_x32(tmem + ((q * 32u) << 16) + slot * C::SLOT_COLS + h * 32u, o);
        }
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(afull_bar(slot));
      }
    }
    __syncwarp();
  } else {
    // --------------------------------------- epilogue ---------------------------------------
    const uint32_t q = warp & 3u;
    uint32_t local = 0, g0 = 0;  // g0: this CTA's step count before the unit
    W4sRange range(p);
    W4sUnit un;
    for (; range.next(un); ++local) {
      const uint32_t nt = un.nt;
      const uint32_t len = un.kb1 - un.kb0;
      const uint32_t buf = local & 1u, use = local >> 1;
      int ok = 1;
      if (lane == 0) ok = mbar_wait(tfull_bar(buf), use & 1u, 0xB8, abort_flag);
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) { if (lane == 0) *abort_flag = 1; break; }
      tc_fence_after();
      uint32_t v[NX];
#pragma unroll
      for (int m = 0; m < NX; ++m) v[m] = 0u;
      const uint32_t acc0 = tmem + ((q * 32u) << 16) + C::ACC_COL + buf * C::MMA_WARPS * NX;
      // issuer jj wrote its accumulator iff the unit has a step g with g % MMA_WARPS == jj
#pragma unroll 1
      for (uint32_t jj = 0; jj < static_cast<uint32_t>(C::MMA_WARPS); ++jj) {
        const uint32_t first_i = (jj + C::MMA_WARPS - g0 % C::MMA_WARPS) % C::MMA_WARPS;
        if (first_i >= len) continue;
        uint32_t v1[NX];
#pragma unroll
        for (int c = 0; c < NX / 16; ++c) tmem_ld_32x32b_x16(acc0 + jj * NX + c * 16, v1 + 16 * c);
        tmem_ld_wait();
#pragma unroll
        for (int m = 0; m < NX; ++m) v[m] += v1[m];
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(tempty_bar(buf));
      g0 += len;
      const uint32_t col = q * 32u + lane;  // column of the tile == TMEM lane
      const uint32_t n = nt * 128u + col;
      if (!p.ws_cnt) {
        if (n < p.N) {
#pragma unroll
          for (int m = 0; m < NX; ++m)
            if (static_cast<uint32_t>(m) < p.M) red_add_s32(p.C + static_cast<size_t>(m) * p.N + n, static_cast<int32_t>(v[m]));
        }
      } else if (un.kb0 == 0 && un.kb1 == p.nk) {  // the whole tile in this unit: store C
        if (n < p.N) {
#pragma unroll
          for (int m = 0; m < NX; ++m)
            if (static_cast<uint32_t>(m) < p.M) p.C[static_cast<size_t>(m) * p.N + n] = static_cast<int32_t>(v[m]);
        }
      } else {
        // split tile: publish the partial, count in; the last contributor finishes the tile
        const uint64_t total = uint64_t(p.n_tiles) * p.nk;
        const uint32_t G = gridDim.x;
        const uint32_t c0 = w4s_cta_of(uint64_t(nt) * p.nk, total, G);
        const uint32_t c1 = w4s_cta_of(uint64_t(nt + 1) * p.nk - 1, total, G);
        auto slot_of = [&](uint32_t c) {  // a CTA's first unit uses slot 2c, any later one 2c + 1
          const uint32_t first_tile = static_cast<uint32_t>(total * c / G / p.nk);
          return 2u * c + (first_tile == nt ? 0u : 1u);
        };
        int32_t* mine = p.ws_part + static_cast<size_t>(slot_of(blockIdx.x)) * NX * 128u;
#pragma unroll
        for (int m = 0; m < NX; ++m) mine[m * 128 + col] = static_cast<int32_t>(v[m]);
        __threadfence();
        named_bar_sync(2, 128);
        if (warp == C::EPI0 && lane == 0) {
          const uint32_t arrived = atomicAdd(p.ws_cnt + nt, 1u) + 1u;
          *last_flag = arrived == c1 - c0 + 1u;
        }
        named_bar_sync(2, 128);
        if (*last_flag) {
          __threadfence();
          for (uint32_t c = c0; c <= c1; ++c) {
            if (c == blockIdx.x) continue;
            const int32_t* other = p.ws_part + static_cast<size_t>(slot_of(c)) * NX * 128u;
#pragma unroll
            for (int m = 0; m < NX; ++m)
              if (static_cast<uint32_t>(m) < p.M) v[m] += static_cast<uint32_t>(__ldcg(other + m * 128 + col));
          }
          if (n < p.N) {
#pragma unroll
            for (int m = 0; m < NX; ++m)
              if (static_cast<uint32_t>(m) < p.M) p.C[static_cast<size_t>(m) * p.N + n] = static_cast<int32_t>(v[m]);
          }
          if (warp == C::EPI0 && lane == 0) p.ws_cnt[nt] = 0u;  // ready for the next launch
        }
        named_bar_sync(2, 128);  // last_flag is rewritten for the next split unit
      }
    }
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

}  // namespace zx
