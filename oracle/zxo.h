/* zxo.h — CPU oracle for the quantised-GEMM path. TEST INFRASTRUCTURE ONLY.
 *
 * A plain-C restatement of the reference's host-side data generation and CPU GEMM check
 * (zig-ecosystem/zoxide, src/bench.zig and src/examples_abi.zig). The reference is Zig 0.16
 * and no Zig toolchain exists on these machines, so it cannot be compiled or run; parity is
 * pinned by (a) Marsaglia's published xorshift32 output, (b) hand-computed known answers and
 * (c) fixtures written by an independent pure-Python restatement (tests/golden/).
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference arm may load
 * this library. The product (libzoxide_b200.so) never links or calls it.
 */
#ifndef ZXO_H
#define ZXO_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- generators --------------------------------------------------------------------- */
/* xorshift32, shifts 13/17/5 (src/bench.zig:26-33). */
uint32_t zxo_xorshift32(uint32_t* state);
/* BASELINE "seed" -> non-zero xorshift state (splitmix64 finaliser; state 0 is a fixed point). */
uint32_t zxo_state_from_seed(uint64_t seed);
/* n int8 values, each the low byte of one draw (src/bench.zig:653-655). */
void zxo_fill_s8(int8_t* dst, size_t n, uint32_t* state);
/* two's-complement s4 pack, even index in the low nibble (src/examples_abi.zig:54-56). */
uint8_t zxo_pack_s4(int8_t even, int8_t odd);
/* sign-extended s4 at logical index idx of a packed buffer (src/bench.zig:753-759). */
int8_t zxo_s4_at(const uint8_t* bytes, size_t idx);
/* nbytes packed s4 bytes; per byte a low-nibble draw then a high-nibble draw, each the
 * sign-extended low nibble of one xorshift output (src/bench.zig:774-786). */
void zxo_fill_s4_packed(uint8_t* dst, size_t nbytes, uint32_t* state);
/* 2:4 prune of a rows x k int8 A (k % 32 == 0), src/bench.zig:1027-1058: per group of 4 along
 * k, combos[draw % 6] picks the kept pair, then one value draw per kept element (k order);
 * dropped elements are 0 in a_dense. a_comp is rows x k/2 (kept values in k order), meta is
 * rows x k/32 u32 words with nibble j = idx0 | idx1 << 2. a_dense may be NULL. */
void zxo_prune24_s8(size_t rows, size_t k, uint32_t* state, int8_t* a_dense, int8_t* a_comp,
                    uint32_t* meta);
/* n floats uniform in [lo, hi): lo + (hi - lo) * (draw >> 8) / 2^24 (24-bit mantissa draw, the
 * reference's fillRandom construction, src/bench.zig:35-41). */
/* 4:8 pair-clustered s4 prune of runImmaSpS4 (src/bench.zig:1178-1213); a_dense may be NULL. */
void zxo_prune48_s4(size_t rows, size_t k, uint32_t* state, int8_t* a_dense, uint8_t* a_comp,
                    uint32_t* meta);
void zxo_decompress48_s4(const uint8_t* a_comp, const uint32_t* meta, int8_t* a_dense, size_t M,
                         size_t K);
/* n logical packed-s4 values -> int8 (s4At order). */
void zxo_unpack_s4(const uint8_t* packed, int8_t* out, size_t n);
void zxo_fill_uniform_f32(float* dst, size_t n, float lo, float hi, uint32_t* state);
/* n bf16 values N(0,1) * scale (Box-Muller over two 24-bit draws, computed in double, rounded
 * to float then to bf16 round-to-nearest-even). */
void zxo_fill_normal_bf16(uint16_t* dst, size_t n, double scale, uint32_t* state);
uint16_t zxo_f32_to_bf16_rne(float x);
float zxo_bf16_to_f32(uint16_t b);

/* ---- reference CPU check, restated (src/bench.zig:712-740) ----------------------------- */
/* layout 0 = NT (B is N x K, K contiguous), 1 = NN (B is K x N, the reference's layout). */
int64_t zxo_dot_s8(const int8_t* A, const int8_t* B, size_t N, size_t K, int layout, size_t row,
                   size_t col);
/* Draw `samples` indices idx = xorshift(vstate) % (M*N) and compare C[idx] with the i64 dot
 * product. Returns the number of mismatches; the first one is reported through the outputs. */
size_t zxo_check_samples_s8(const int8_t* A, const int8_t* B, const int32_t* C, size_t M,
                            size_t N, size_t K, int layout, size_t samples, uint32_t vstate,
                            size_t* first_bad, int64_t* want, int32_t* got);
/* The reference check loop itself (i64 accumulate, B read in its stored layout) over rows
 * [r0, r1) and every column, written to out (i64, (r1-r0) x N). threads = 0: all cores.
 * This is the timed CPU baseline; it is deliberately not blocked or hand-vectorised. */
void zxo_ref_loop_s8(const int8_t* A, const int8_t* B, int64_t* out, size_t N, size_t K,
                     int layout, size_t r0, size_t r1, int threads);

/* ---- exact / reference GEMMs used as checkers ------------------------------------------ */
/* C (int32, M x N) = A * op(B), exact (int32 accumulate; exact for K < 131072). */
void zxo_gemm_s8(const int8_t* A, const int8_t* B, int32_t* C, size_t M, size_t N, size_t K,
                 int layout, int threads);
/* bf16 C = bf16_rne(((float)acc * rs[m]) * cs[n]) over rows [r0, r1) (out is (r1-r0) x N). */
void zxo_gemm_s8_scaled_bf16(const int8_t* A, const int8_t* B, const float* rs, const float* cs,
                             uint16_t* out, size_t N, size_t K, int layout, size_t r0, size_t r1,
                             int threads);
/* Epilogue alone: bf16_rne(((float)acc * rs) * cs). */
uint16_t zxo_scale_to_bf16(int32_t acc, float rs, float cs);
/* W4A8: A int8 M x K, W s4 N x K packed along K (K/2 bytes per row, low nibble = even k). */
void zxo_gemm_w4a8(const int8_t* A, const uint8_t* W, int32_t* C, size_t M, size_t N, size_t K,
                   int threads);
/* 2:4 sparse: C = decompress(a_comp, meta) * op(B); a_comp rows x K/2, meta rows x K/32. */
void zxo_gemm_sp_s8(const int8_t* a_comp, const uint32_t* meta, const int8_t* B, int32_t* C,
                    size_t M, size_t N, size_t K, int layout, int threads);
/* Decompress 2:4 A to dense (M x K). */
void zxo_decompress24_s8(const int8_t* a_comp, const uint32_t* meta, int8_t* a_dense, size_t M,
                         size_t K);
/* bf16 x bf16 -> f64 rows [r0, r1) of A * op(B) (out (r1-r0) x N). */
void zxo_gemm_bf16_f64(const uint16_t* A, const uint16_t* B, double* out, size_t N, size_t K,
                       int layout, size_t r0, size_t r1, int threads);

/* ---- size-independent checks ----------------------------------------------------------- */
/* y = C x (int32 C M x N, int64 x, y), exact. */
void zxo_matvec_s32(const int32_t* C, const int64_t* x, int64_t* y, size_t M, size_t N,
                    int threads);
/* y = A (op(B) x) exactly in int64: the Freivalds right-hand side for C = A op(B). */
void zxo_gemv_chain_s8(const int8_t* A, const int8_t* B, const int64_t* x, int64_t* y, size_t M,
                       size_t N, size_t K, int layout, int threads);

int zxo_num_threads(int requested);

#ifdef __cplusplus
}
#endif
#endif
