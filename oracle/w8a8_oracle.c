/*
 * w8a8_oracle.c — CPU restatement of the W8A8 operator contract.
 *
 * TEST INFRASTRUCTURE ONLY: the parity checker for the CUDA kernels in
 * lema_b200/csrc. Only tests/, __graft_entry__.smoke() and bench.py's CPU
 * baseline leg load this library; the product path never does.
 *
 * Parity status: the reference (Pomilon/LEMA) has no quantised linear
 * (README.md:143-145 lists quantisation as planned work), so no reference
 * golden vectors exist for these functions — their parity is UNPINNED against
 * the reference. The functions restate the contract written in
 * include/lema_b200.h and are cross-checked in tests against an independent
 * numpy restatement (oracle/oracle.py) and hand-derived known answers. The
 * unquantised surroundings they plug into are the reference's nn.Linear call
 * sites (adapters/_llama.py:245-250 via _lora.py:23-26).
 *
 * Built with -O2 -ffp-contract=off (no FMA contraction, IEEE fp32 division on
 * SSE); the GEMM loops run on POSIX threads.
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <string.h>
#include <unistd.h>

/* Row-parallel loop over [0, n) on up to `oracle_threads` POSIX threads. */
static int oracle_threads = 0;
void oracle_set_threads(int n) { oracle_threads = n; }

typedef void (*row_fn)(int64_t lo, int64_t hi, void* ctx);
typedef struct {
  row_fn fn;
  void* ctx;
  int64_t lo, hi;
} span_t;

static void* run_span(void* p) {
  span_t* s = (span_t*)p;
  s->fn(s->lo, s->hi, s->ctx);
  return NULL;
}

static void parallel_rows(int64_t n, row_fn fn, void* ctx) {
  int t = oracle_threads > 0 ? oracle_threads : (int)sysconf(_SC_NPROCESSORS_ONLN);
  if (t < 1) t = 1;
  if (t > 256) t = 256;
  if (n < t) t = (int)(n > 0 ? n : 1);
  pthread_t th[256];
  span_t sp[256];
  for (int i = 0; i < t; ++i) {
    sp[i].fn = fn;
    sp[i].ctx = ctx;
    sp[i].lo = n * i / t;
    sp[i].hi = n * (i + 1) / t;
  }
  for (int i = 1; i < t; ++i)
    if (pthread_create(&th[i], NULL, run_span, &sp[i]) != 0) run_span(&sp[i]), th[i] = 0;
  run_span(&sp[0]);
  for (int i = 1; i < t; ++i)
    if (th[i]) pthread_join(th[i], NULL);
}

static float bf16_to_f32(uint16_t h) {
  uint32_t u = (uint32_t)h << 16;
  float f;
  memcpy(&f, &u, sizeof f);
  return f;
}

/* Round-to-nearest-even fp32 -> bf16 (NaN kept quiet). */
static uint16_t f32_to_bf16(float f) {
  uint32_t u;
  memcpy(&u, &f, sizeof u);
  if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u);
  u += 0x7fffu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}

static float row_scale(float amax) { return amax > 0.0f ? amax / 127.0f : 1.0f; }

static int8_t quant1(float x, float s) {
  float r = nearbyintf(x / s); /* default rounding mode: nearest, ties to even */
  if (r > 127.0f) r = 127.0f;
  if (r < -127.0f) r = -127.0f;
  return (int8_t)r;
}

/* A1/A2 quantiser on bf16 rows (activations per token, weights per channel). */
void oracle_quantize_rows_bf16(const uint16_t* x, int64_t rows, int64_t cols, int64_t ldx,
                               int8_t* q, int64_t ldq, float* scale) {
  for (int64_t r = 0; r < rows; ++r) {
    const uint16_t* xr = x + r * ldx;
    float amax = 0.0f;
    for (int64_t c = 0; c < cols; ++c) {
      float a = fabsf(bf16_to_f32(xr[c]));
      if (a > amax) amax = a;
    }
    const float s = row_scale(amax);
    for (int64_t c = 0; c < cols; ++c) q[r * ldq + c] = quant1(bf16_to_f32(xr[c]), s);
    scale[r] = s;
  }
}

/* Same rule on fp32 rows (true weights of trainable projections). */
void oracle_quantize_rows_f32(const float* x, int64_t rows, int64_t cols, int64_t ldx, int8_t* q,
                              int64_t ldq, float* scale) {
  for (int64_t r = 0; r < rows; ++r) {
    const float* xr = x + r * ldx;
    float amax = 0.0f;
    for (int64_t c = 0; c < cols; ++c) {
      float a = fabsf(xr[c]);
      if (a > amax) amax = a;
    }
    const float s = row_scale(amax);
    for (int64_t c = 0; c < cols; ++c) q[r * ldq + c] = quant1(xr[c], s);
    scale[r] = s;
  }
}

/* A2 GEMM: acc[m,n] = sum_k a[m,k] * b[n,k], exact in int32. */
typedef struct {
  const int8_t *a, *b;
  int64_t lda, ldb, N, K, ldacc;
  int32_t* acc;
} i8gemm_t;

static void i8gemm_rows(int64_t lo, int64_t hi, void* p) {
  const i8gemm_t* g = (const i8gemm_t*)p;
  for (int64_t m = lo; m < hi; ++m) {
    const int8_t* ar = g->a + m * g->lda;
    for (int64_t n = 0; n < g->N; ++n) {
      const int8_t* br = g->b + n * g->ldb;
      int32_t s = 0;
      for (int64_t k = 0; k < g->K; ++k) s += (int32_t)ar[k] * (int32_t)br[k];
      g->acc[m * g->ldacc + n] = s;
    }
  }
}

void oracle_int8_gemm(const int8_t* a, int64_t lda, const int8_t* b, int64_t ldb, int64_t M,
                      int64_t N, int64_t K, int32_t* acc, int64_t ldacc) {
  i8gemm_t g = {a, b, lda, ldb, N, K, ldacc, acc};
  parallel_rows(M, i8gemm_rows, &g);
}

/* A3 epilogue: y = bf16((float(acc) * sx[m]) * sw[n] + bias[n]); bias may be NULL (no add). */
void oracle_epilogue(const int32_t* acc, int64_t ldacc, const float* sx, const float* sw,
                     const uint16_t* bias, int64_t M, int64_t N, uint16_t* y, int64_t ldy) {
  for (int64_t m = 0; m < M; ++m)
    for (int64_t n = 0; n < N; ++n) {
      float f = ((float)acc[m * ldacc + n] * sx[m]) * sw[n];
      if (bias) f = f + bf16_to_f32(bias[n]);
      y[m * ldy + n] = f32_to_bf16(f);
    }
}

/* A4 dequant: wdT[k, n] = bf16(float(wq[n, k]) * sw[n]). */
void oracle_dequant_transpose(const int8_t* wq, int64_t ldw, const float* sw, int64_t N, int64_t K,
                              uint16_t* wdT, int64_t ldt) {
  for (int64_t n = 0; n < N; ++n)
    for (int64_t k = 0; k < K; ++k) wdT[k * ldt + n] = f32_to_bf16((float)wq[n * ldw + k] * sw[n]);
}

/* bf16 GEMM reference: y[m,n] = bf16(sum_k a[m,k] * b[n,k]), accumulated in
 * double so the comparison tolerance covers only the device's fp32 ordering. */
typedef struct {
  const uint16_t *a, *b;
  int64_t lda, ldb, N, K, ldy;
  uint16_t* y;
  float* y_f32;
} bfgemm_t;

static void bfgemm_rows(int64_t lo, int64_t hi, void* p) {
  const bfgemm_t* g = (const bfgemm_t*)p;
  for (int64_t m = lo; m < hi; ++m)
    for (int64_t n = 0; n < g->N; ++n) {
      double s = 0.0;
      for (int64_t k = 0; k < g->K; ++k)
        s += (double)bf16_to_f32(g->a[m * g->lda + k]) * (double)bf16_to_f32(g->b[n * g->ldb + k]);
      if (g->y) g->y[m * g->ldy + n] = f32_to_bf16((float)s);
      if (g->y_f32) g->y_f32[m * g->N + n] = (float)s;
    }
}

void oracle_bf16_gemm_tn(const uint16_t* a, int64_t lda, const uint16_t* b, int64_t ldb, int64_t M,
                         int64_t N, int64_t K, uint16_t* y, int64_t ldy, float* y_f32) {
  bfgemm_t g = {a, b, lda, ldb, N, K, ldy, y, y_f32};
  parallel_rows(M, bfgemm_rows, &g);
}

/* Exact checksums of an int8 GEMM without forming it: row sums
 * r[m] = sum_n acc[m,n] = sum_k a[m,k] * (sum_n b[n,k]) and column sums
 * c[n] = sum_k b[n,k] * (sum_m a[m,k]), in int64. */
void oracle_int8_gemm_checksums(const int8_t* a, int64_t lda, const int8_t* b, int64_t ldb,
                                int64_t M, int64_t N, int64_t K, int64_t* row_sums,
                                int64_t* col_sums) {
  for (int64_t m = 0; m < M; ++m) row_sums[m] = 0;
  for (int64_t n = 0; n < N; ++n) col_sums[n] = 0;
  /* sum_n b[n,k] and sum_m a[m,k] per k, streamed in blocks of 4096 k. */
  enum { KB = 4096 };
  int64_t bs[KB], as[KB];
  for (int64_t k0 = 0; k0 < K; k0 += KB) {
    const int64_t kn = (K - k0) < KB ? (K - k0) : KB;
    for (int64_t j = 0; j < kn; ++j) bs[j] = as[j] = 0;
    for (int64_t n = 0; n < N; ++n)
      for (int64_t j = 0; j < kn; ++j) bs[j] += b[n * ldb + k0 + j];
    for (int64_t m = 0; m < M; ++m)
      for (int64_t j = 0; j < kn; ++j) as[j] += a[m * lda + k0 + j];
    for (int64_t m = 0; m < M; ++m) {
      int64_t s = 0;
      for (int64_t j = 0; j < kn; ++j) s += (int64_t)a[m * lda + k0 + j] * bs[j];
      row_sums[m] += s;
    }
    for (int64_t n = 0; n < N; ++n) {
      int64_t s = 0;
      for (int64_t j = 0; j < kn; ++j) s += (int64_t)b[n * ldb + k0 + j] * as[j];
      col_sums[n] += s;
    }
  }
}
