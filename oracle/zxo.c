/* zxo.c — CPU oracle (test infrastructure only; see zxo.h for scope and pinning).
 *
 * Every function names the reference lines it restates. Arithmetic contracts:
 *   - integer products accumulate exactly (int64 in the reference loop, int32 in the fast
 *     checkers where |sum| <= K * 128 * 128 < 2^31 for K < 131072);
 *   - float work is compiled with -ffp-contract=off so a*b*c is two rounded multiplies.
 */
#define _GNU_SOURCE
#include "zxo.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

/* ------------------------------------------------------------------------------------------ */
/* generators                                                                                 */
/* ------------------------------------------------------------------------------------------ */

/* src/bench.zig:26-33 */
uint32_t zxo_xorshift32(uint32_t* state) {
  uint32_t x = *state;
  x ^= x << 13;
  x ^= x >> 17;
  x ^= x << 5;
  *state = x;
  return x;
}

uint32_t zxo_state_from_seed(uint64_t seed) {
  uint64_t z = seed + 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  z ^= z >> 31;
  uint32_t s = (uint32_t)(z ^ (z >> 32));
  return s ? s : 0x13579bdfu;
}

/* src/bench.zig:653-655: @bitCast(@as(u8, @truncate(xorshift(&rng)))) */
void zxo_fill_s8(int8_t* dst, size_t n, uint32_t* state) {
  for (size_t i = 0; i < n; ++i) dst[i] = (int8_t)(uint8_t)zxo_xorshift32(state);
}

/* src/examples_abi.zig:54-56 */
uint8_t zxo_pack_s4(int8_t even, int8_t odd) {
  return (uint8_t)(((uint8_t)even & 0xF) | (((uint8_t)odd & 0xF) << 4));
}

/* src/bench.zig:753-759 */
int8_t zxo_s4_at(const uint8_t* bytes, size_t idx) {
  const uint8_t byte = bytes[idx / 2];
  const uint8_t nib = (idx % 2 == 0) ? (byte & 0xF) : (byte >> 4);
  return (int8_t)((int8_t)(uint8_t)(nib << 4) >> 4);
}

static int8_t s4_from_draw(uint32_t d) { return (int8_t)((int8_t)(uint8_t)((d & 0xF) << 4) >> 4); }

/* src/bench.zig:774-786: per byte, lo = draw & 0xF sign-extended, hi = next draw likewise. */
void zxo_fill_s4_packed(uint8_t* dst, size_t nbytes, uint32_t* state) {
  for (size_t i = 0; i < nbytes; ++i) {
    const int8_t lo = s4_from_draw(zxo_xorshift32(state));
    const int8_t hi = s4_from_draw(zxo_xorshift32(state));
    dst[i] = zxo_pack_s4(lo, hi);
  }
}

/* src/bench.zig:1027-1058 (A part of runImmaSpS8). */
void zxo_prune24_s8(size_t rows, size_t k, uint32_t* state, int8_t* a_dense, int8_t* a_comp,
                    uint32_t* meta) {
  static const uint8_t combos[6][2] = {{0, 1}, {0, 2}, {0, 3}, {1, 2}, {1, 3}, {2, 3}};
  for (size_t row = 0; row < rows; ++row) {
    for (size_t kb = 0; kb < k / 32; ++kb) {
      uint32_t word = 0;
      for (int j = 0; j < 8; ++j) {
        const size_t group_base = row * k + kb * 32 + 4 * (size_t)j;
        const uint8_t* combo = combos[zxo_xorshift32(state) % 6];
        if (a_dense) memset(a_dense + group_base, 0, 4);
        for (int e = 0; e < 2; ++e) {
          const int8_t val = (int8_t)(uint8_t)zxo_xorshift32(state);
          if (a_dense) a_dense[group_base + combo[e]] = val;
          a_comp[row * (k / 2) + kb * 16 + 2 * (size_t)j + (size_t)e] = val;
        }
        word |= ((uint32_t)combo[0] | ((uint32_t)combo[1] << 2)) << (4 * j);
      }
      meta[row * (k / 32) + kb] = word;
    }
  }
}

/* src/bench.zig:1178-1213 (A part of runImmaSpS4): 4:8 pair-clustered prune of s4 A. Per row,
 * per 64 dense k one metadata word; per 8-wide chunk j: a combo draw (xorshift % 6 picks the two
 * surviving 2-wide sub-chunks, first < second), then two s4 draws for each of the four
 * sub-chunks; the surviving sub-chunks become one packS4 byte each (a_comp, k/4 bytes per row)
 * and nibble j of the word is first | second << 2. a_dense (optional) receives the logical pruned
 * row (dropped sub-chunks 0). */
void zxo_prune48_s4(size_t rows, size_t k, uint32_t* state, int8_t* a_dense, uint8_t* a_comp,
                    uint32_t* meta) {
  static const uint8_t combos[6][2] = {{0, 1}, {0, 2}, {0, 3}, {1, 2}, {1, 3}, {2, 3}};
  for (size_t row = 0; row < rows; ++row) {
    for (size_t kb = 0; kb < k / 64; ++kb) {
      uint32_t word = 0;
      for (int j = 0; j < 8; ++j) {
        const size_t chunk = row * k + kb * 64 + 8 * (size_t)j;
        const uint8_t* combo = combos[zxo_xorshift32(state) % 6];
        int8_t pr[4][2];
        for (int q = 0; q < 4; ++q) {
          pr[q][0] = s4_from_draw(zxo_xorshift32(state));
          pr[q][1] = s4_from_draw(zxo_xorshift32(state));
        }
        for (int e = 0; e < 2; ++e)
          a_comp[row * (k / 4) + kb * 16 + 2 * (size_t)j + (size_t)e] =
              zxo_pack_s4(pr[combo[e]][0], pr[combo[e]][1]);
        if (a_dense)
          for (int q = 0; q < 4; ++q) {
            const int keep = q == combo[0] || q == combo[1];
            a_dense[chunk + 2 * (size_t)q] = keep ? pr[q][0] : 0;
            a_dense[chunk + 2 * (size_t)q + 1] = keep ? pr[q][1] : 0;
          }
        word |= ((uint32_t)combo[0] | ((uint32_t)combo[1] << 2)) << (4 * j);
      }
      meta[row * (k / 64) + kb] = word;
    }
  }
}

/* Inverse of zxo_prune48_s4's packing (contract src/examples_abi.zig:83-96). */
void zxo_decompress48_s4(const uint8_t* a_comp, const uint32_t* meta, int8_t* a_dense, size_t M,
                         size_t K) {
  memset(a_dense, 0, M * K);
  for (size_t m = 0; m < M; ++m)
    for (size_t kb = 0; kb < K / 64; ++kb) {
      const uint32_t w = meta[m * (K / 64) + kb];
      for (int j = 0; j < 8; ++j) {
        const uint32_t nib = (w >> (4 * j)) & 0xF;
        const size_t chunk = m * K + kb * 64 + 8 * (size_t)j;
        const uint8_t* c = a_comp + m * (K / 4) + kb * 16 + 2 * (size_t)j;
        const uint32_t q0 = nib & 3, q1 = nib >> 2;
        a_dense[chunk + 2 * q0] = zxo_s4_at(c, 0);
        a_dense[chunk + 2 * q0 + 1] = zxo_s4_at(c, 1);
        a_dense[chunk + 2 * q1] = zxo_s4_at(c + 1, 0);
        a_dense[chunk + 2 * q1 + 1] = zxo_s4_at(c + 1, 1);
      }
    }
}

/* n logical s4 values (two per byte, even index in the low nibble) -> int8, via s4At
 * (src/bench.zig:753-759). */
void zxo_unpack_s4(const uint8_t* packed, int8_t* out, size_t n) {
  for (size_t i = 0; i < n; ++i) out[i] = zxo_s4_at(packed, i);
}

/* 24-bit draw as in fillRandom (src/bench.zig:35-41), mapped to [lo, hi). */
void zxo_fill_uniform_f32(float* dst, size_t n, float lo, float hi, uint32_t* state) {
  for (size_t i = 0; i < n; ++i) {
    const double u = (double)(zxo_xorshift32(state) >> 8) / 16777216.0;
    float v = (float)((double)lo + ((double)hi - (double)lo) * u);
    if (v >= hi) v = nextafterf(hi, lo);
    dst[i] = v;
  }
}

uint16_t zxo_f32_to_bf16_rne(float x) {
  uint32_t u;
  memcpy(&u, &x, 4);
  if ((u & 0x7F800000u) == 0x7F800000u && (u & 0x007FFFFFu)) return (uint16_t)((u >> 16) | 0x40);
  const uint32_t lsb = (u >> 16) & 1u;
  u += 0x7FFFu + lsb;
  return (uint16_t)(u >> 16);
}

float zxo_bf16_to_f32(uint16_t b) {
  const uint32_t u = (uint32_t)b << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

void zxo_fill_normal_bf16(uint16_t* dst, size_t n, double scale, uint32_t* state) {
  const double two_pi = 6.283185307179586476925286766559;
  size_t i = 0;
  while (i < n) {
    const double u1 = ((double)(zxo_xorshift32(state) >> 8) + 1.0) / 16777216.0; /* (0, 1] */
    const double u2 = (double)(zxo_xorshift32(state) >> 8) / 16777216.0;         /* [0, 1) */
    const double r = sqrt(-2.0 * log(u1));
    dst[i++] = zxo_f32_to_bf16_rne((float)(r * cos(two_pi * u2) * scale));
    if (i < n) dst[i++] = zxo_f32_to_bf16_rne((float)(r * sin(two_pi * u2) * scale));
  }
}

/* ------------------------------------------------------------------------------------------ */
/* threading                                                                                  */
/* ------------------------------------------------------------------------------------------ */

int zxo_num_threads(int requested) {
  if (requested > 0) return requested;
  long n = sysconf(_SC_NPROCESSORS_ONLN);
  return n > 0 ? (int)n : 1;
}

typedef void (*row_fn)(void* ctx, size_t r0, size_t r1);
typedef struct {
  row_fn fn;
  void* ctx;
  size_t r0, r1;
} task_t;

static void* task_run(void* p) {
  task_t* t = (task_t*)p;
  t->fn(t->ctx, t->r0, t->r1);
  return NULL;
}

/* Split rows [r0, r1) into contiguous blocks over `threads` POSIX threads. */
static void parallel_rows(row_fn fn, void* ctx, size_t r0, size_t r1, int threads) {
  threads = zxo_num_threads(threads);
  const size_t rows = r1 - r0;
  if ((size_t)threads > rows) threads = (int)(rows ? rows : 1);
  if (threads <= 1) {
    fn(ctx, r0, r1);
    return;
  }
  pthread_t* th = (pthread_t*)malloc(sizeof(pthread_t) * (size_t)threads);
  task_t* ts = (task_t*)malloc(sizeof(task_t) * (size_t)threads);
  for (int i = 0; i < threads; ++i) {
    ts[i].fn = fn;
    ts[i].ctx = ctx;
    ts[i].r0 = r0 + rows * (size_t)i / (size_t)threads;
    ts[i].r1 = r0 + rows * (size_t)(i + 1) / (size_t)threads;
    pthread_create(&th[i], NULL, task_run, &ts[i]);
  }
  for (int i = 0; i < threads; ++i) pthread_join(th[i], NULL);
  free(th);
  free(ts);
}

/* ------------------------------------------------------------------------------------------ */
/* the reference check, restated                                                              */
/* ------------------------------------------------------------------------------------------ */

/* src/bench.zig:723-727: want += i64(A[row*n+k]) * i64(B[k*n+col]) (NN); NT reads B[col*K+k]. */
int64_t zxo_dot_s8(const int8_t* A, const int8_t* B, size_t N, size_t K, int layout, size_t row,
                   size_t col) {
  int64_t want = 0;
  for (size_t k = 0; k < K; ++k) {
    const int64_t b = layout == 1 ? (int64_t)B[k * N + col] : (int64_t)B[col * K + k];
    want += (int64_t)A[row * K + k] * b;
  }
  return want;
}

/* src/bench.zig:712-740 (sample draw from xorshift(0xdeadbeef), exact equality). */
size_t zxo_check_samples_s8(const int8_t* A, const int8_t* B, const int32_t* C, size_t M,
                            size_t N, size_t K, int layout, size_t samples, uint32_t vstate,
                            size_t* first_bad, int64_t* want, int32_t* got) {
  size_t bad = 0;
  const size_t elems = M * N;
  for (size_t si = 0; si < samples; ++si) {
    const size_t idx = (size_t)zxo_xorshift32(&vstate) % elems;
    const size_t row = idx / N, col = idx % N;
    const int64_t w = zxo_dot_s8(A, B, N, K, layout, row, col);
    if (w != (int64_t)C[idx]) {
      if (bad == 0) {
        if (first_bad) *first_bad = idx;
        if (want) *want = w;
        if (got) *got = C[idx];
      }
      ++bad;
    }
  }
  return bad;
}

typedef struct {
  const int8_t *A, *B;
  int64_t* out;
  size_t N, K, base;
  int layout;
} refloop_ctx;

static void refloop_rows(void* p, size_t r0, size_t r1) {
  const refloop_ctx* c = (const refloop_ctx*)p;
  for (size_t row = r0; row < r1; ++row)
    for (size_t col = 0; col < c->N; ++col)
      c->out[(row - c->base) * c->N + col] = zxo_dot_s8(c->A, c->B, c->N, c->K, c->layout, row, col);
}

void zxo_ref_loop_s8(const int8_t* A, const int8_t* B, int64_t* out, size_t N, size_t K,
                     int layout, size_t r0, size_t r1, int threads) {
  refloop_ctx c = {A, B, out, N, K, r0, layout};
  parallel_rows(refloop_rows, &c, r0, r1, threads);
}

/* ------------------------------------------------------------------------------------------ */
/* fast exact checkers                                                                        */
/* ------------------------------------------------------------------------------------------ */

/* Contiguous int8 dot product with int32 accumulation; gcc vectorises it (pmaddwd / vpmaddwd).
 * target_clones picks an AVX2 body at load time where the host supports it. */
__attribute__((target_clones("avx2", "default"), optimize("O3"))) static int32_t dot_i8(const int8_t* a,
                                                                      const int8_t* b, size_t k) {
  int32_t s = 0;
  for (size_t i = 0; i < k; ++i) s += (int32_t)a[i] * (int32_t)b[i];
  return s;
}

typedef struct {
  const int8_t *A, *Bt; /* Bt is N x K */
  int32_t* C;
  size_t N, K, base;
} gemm_ctx;

static void gemm_rows(void* p, size_t r0, size_t r1) {
  const gemm_ctx* c = (const gemm_ctx*)p;
  const size_t NB = 64; /* column block: 64 rows of Bt stay in L2 while a row block streams */
  for (size_t n0 = 0; n0 < c->N; n0 += NB) {
    const size_t n1 = n0 + NB < c->N ? n0 + NB : c->N;
    for (size_t m = r0; m < r1; ++m) {
      const int8_t* a = c->A + m * c->K;
      int32_t* crow = c->C + (m - c->base) * c->N;
      for (size_t n = n0; n < n1; ++n) crow[n] = dot_i8(a, c->Bt + n * c->K, c->K);
    }
  }
}

static int8_t* transpose_s8(const int8_t* B, size_t K, size_t N) {
  int8_t* t = (int8_t*)malloc(K * N);
  for (size_t k = 0; k < K; ++k)
    for (size_t n = 0; n < N; ++n) t[n * K + k] = B[k * N + n];
  return t;
}

void zxo_gemm_s8(const int8_t* A, const int8_t* B, int32_t* C, size_t M, size_t N, size_t K,
                 int layout, int threads) {
  int8_t* bt = layout == 1 ? transpose_s8(B, K, N) : NULL;
  gemm_ctx c = {A, bt ? bt : B, C, N, K, 0};
  parallel_rows(gemm_rows, &c, 0, M, threads);
  free(bt);
}

/* The scaled epilogue: (float)acc RNE, then two RNE multiplies, then bf16 RNE. */
uint16_t zxo_scale_to_bf16(int32_t acc, float rs, float cs) {
  volatile float f = (float)acc;
  volatile float t = f * rs;
  volatile float u = t * cs;
  return zxo_f32_to_bf16_rne(u);
}

typedef struct {
  const int8_t *A, *Bt;
  const float *rs, *cs;
  uint16_t* out;
  size_t N, K, base;
} sgemm_ctx;

static void scaled_rows(void* p, size_t r0, size_t r1) {
  const sgemm_ctx* c = (const sgemm_ctx*)p;
  for (size_t m = r0; m < r1; ++m)
    for (size_t n = 0; n < c->N; ++n)
      c->out[(m - c->base) * c->N + n] =
          zxo_scale_to_bf16(dot_i8(c->A + m * c->K, c->Bt + n * c->K, c->K), c->rs[m], c->cs[n]);
}

void zxo_gemm_s8_scaled_bf16(const int8_t* A, const int8_t* B, const float* rs, const float* cs,
                             uint16_t* out, size_t N, size_t K, int layout, size_t r0, size_t r1,
                             int threads) {
  int8_t* bt = layout == 1 ? transpose_s8(B, K, N) : NULL;
  sgemm_ctx c = {A, bt ? bt : B, rs, cs, out, N, K, r0};
  parallel_rows(scaled_rows, &c, r0, r1, threads);
  free(bt);
}

/* W4A8: unpack W with the s4At convention along K, then an int8 GEMM. */
void zxo_gemm_w4a8(const int8_t* A, const uint8_t* W, int32_t* C, size_t M, size_t N, size_t K,
                   int threads) {
  int8_t* w8 = (int8_t*)malloc(N * K);
  for (size_t n = 0; n < N; ++n)
    for (size_t k = 0; k < K; ++k) w8[n * K + k] = zxo_s4_at(W + n * (K / 2), k);
  gemm_ctx c = {A, w8, C, N, K, 0};
  parallel_rows(gemm_rows, &c, 0, M, threads);
  free(w8);
}

/* Inverse of zxo_prune24_s8's packing (metadata contract src/examples_abi.zig:71-81). */
void zxo_decompress24_s8(const int8_t* a_comp, const uint32_t* meta, int8_t* a_dense, size_t M,
                         size_t K) {
  memset(a_dense, 0, M * K);
  for (size_t m = 0; m < M; ++m)
    for (size_t kb = 0; kb < K / 32; ++kb) {
      const uint32_t w = meta[m * (K / 32) + kb];
      for (int j = 0; j < 8; ++j) {
        const uint32_t nib = (w >> (4 * j)) & 0xF;
        const size_t gb = m * K + kb * 32 + 4 * (size_t)j;
        const size_t cb = m * (K / 2) + kb * 16 + 2 * (size_t)j;
        a_dense[gb + (nib & 3)] = a_comp[cb];
        a_dense[gb + (nib >> 2)] = a_comp[cb + 1];
      }
    }
}

void zxo_gemm_sp_s8(const int8_t* a_comp, const uint32_t* meta, const int8_t* B, int32_t* C,
                    size_t M, size_t N, size_t K, int layout, int threads) {
  int8_t* ad = (int8_t*)malloc(M * K);
  zxo_decompress24_s8(a_comp, meta, ad, M, K);
  zxo_gemm_s8(ad, B, C, M, N, K, layout, threads);
  free(ad);
}

typedef struct {
  const uint16_t *A, *B;
  double* out;
  size_t N, K, base;
  int layout;
} bgemm_ctx;

static void bf16_rows(void* p, size_t r0, size_t r1) {
  const bgemm_ctx* c = (const bgemm_ctx*)p;
  double* arow = (double*)malloc(sizeof(double) * c->K);
  for (size_t m = r0; m < r1; ++m) {
    for (size_t k = 0; k < c->K; ++k) arow[k] = zxo_bf16_to_f32(c->A[m * c->K + k]);
    for (size_t n = 0; n < c->N; ++n) {
      double s = 0.0;
      for (size_t k = 0; k < c->K; ++k) {
        const uint16_t b = c->layout == 1 ? c->B[k * c->N + n] : c->B[n * c->K + k];
        s += arow[k] * (double)zxo_bf16_to_f32(b);
      }
      c->out[(m - c->base) * c->N + n] = s;
    }
  }
  free(arow);
}

void zxo_gemm_bf16_f64(const uint16_t* A, const uint16_t* B, double* out, size_t N, size_t K,
                       int layout, size_t r0, size_t r1, int threads) {
  bgemm_ctx c = {A, B, out, N, K, r0, layout};
  parallel_rows(bf16_rows, &c, r0, r1, threads);
}

/* ------------------------------------------------------------------------------------------ */
/* size-independent checks                                                                    */
/* ------------------------------------------------------------------------------------------ */

typedef struct {
  const int32_t* C;
  const int64_t* x;
  int64_t* y;
  size_t N;
} mv_ctx;

static void mv_rows(void* p, size_t r0, size_t r1) {
  const mv_ctx* c = (const mv_ctx*)p;
  for (size_t m = r0; m < r1; ++m) {
    int64_t s = 0;
    const int32_t* row = c->C + m * c->N;
    for (size_t n = 0; n < c->N; ++n) s += (int64_t)row[n] * c->x[n];
    c->y[m] = s;
  }
}

void zxo_matvec_s32(const int32_t* C, const int64_t* x, int64_t* y, size_t M, size_t N,
                    int threads) {
  mv_ctx c = {C, x, y, N};
  parallel_rows(mv_rows, &c, 0, M, threads);
}

typedef struct {
  const int8_t* A;
  const int64_t* v;
  int64_t* y;
  size_t K;
} av_ctx;

static void av_rows(void* p, size_t r0, size_t r1) {
  const av_ctx* c = (const av_ctx*)p;
  for (size_t m = r0; m < r1; ++m) {
    int64_t s = 0;
    const int8_t* row = c->A + m * c->K;
    for (size_t k = 0; k < c->K; ++k) s += (int64_t)row[k] * c->v[k];
    c->y[m] = s;
  }
}

void zxo_gemv_chain_s8(const int8_t* A, const int8_t* B, const int64_t* x, int64_t* y, size_t M,
                       size_t N, size_t K, int layout, int threads) {
  /* v = op(B) x : v[k] = sum_n B(k, n) x[n] */
  int64_t* v = (int64_t*)calloc(K, sizeof(int64_t));
  if (layout == 1) {
    for (size_t k = 0; k < K; ++k) {
      int64_t s = 0;
      for (size_t n = 0; n < N; ++n) s += (int64_t)B[k * N + n] * x[n];
      v[k] = s;
    }
  } else {
    for (size_t n = 0; n < N; ++n) {
      const int8_t* brow = B + n * K;
      const int64_t xn = x[n];
      for (size_t k = 0; k < K; ++k) v[k] += (int64_t)brow[k] * xn;
    }
  }
  av_ctx c = {A, v, y, K};
  parallel_rows(av_rows, &c, 0, M, threads);
  free(v);
}
