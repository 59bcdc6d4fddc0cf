/*
 * xvram_oracle.c -- CPU FP64 oracle for the out-of-core SGEMM path.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the product library links, loads or calls
 * this file.  It is used by tests/, by __graft_entry__.smoke() and by bench.py's
 * cpu_baseline / --impl reference legs, and only as the checker or the timed CPU
 * baseline, never as the thing measured or shipped.
 *
 * Parity is pinned two ways (see tests/test_oracle_cpu.py):
 *   1. against the reference's own pattern and FP64 reference code, compiled from
 *      its sources into oracle/_ref/ by oracle/Makefile (container only), and
 *   2. against the committed fixtures under tests/golden/, which were generated
 *      from that compiled reference code by tests/golden/make_golden.py.
 *
 * What is restated (reference file:line):
 *   - FP64 reference GEMM: FP64 sum of (double)a*(double)b over k in ascending
 *     order, then alpha*dot + beta*c in double
 *       examples/preview-gemm/main.cpp:109-118, src/compat_bench/pattern.cpp:102-124
 *   - compat-bench analytic operand patterns
 *       src/compat_bench/pattern.cpp:56-69 (pattern_a/pattern_b/pattern_c)
 *   - gemm-bench exact integer closed form
 *       src/gemm_bench/pattern.cpp:207-237
 *   - preview-gemm operand values
 *       examples/preview-gemm/main.cpp:53-58
 *   - the reference's acceptance criterion |err| <= 1e-4 + 2e-5*|ref|
 *       src/compat_bench/executor.cpp:93-96
 *
 * A float product a*b is exact in double (24+24 bit significands), so any loop order
 * that keeps k ascending for each output gives bit-identical FP64 sums.  The oracle
 * uses that freedom to stream column-major operands with unit stride.
 *
 * Synthetic inputs: uniform[-1,1) from a counter-based generator (SplitMix64 finaliser,
 * Steele/Lea/Flood 2014) so that any element can be recomputed from (seed, index)
 * and large operands fill in parallel.  The product library carries its own copy of
 * the same generator; tests check the two agree bit for bit.
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define XO_EXPORT __attribute__((visibility("default")))

/* ------------------------------------------------------------------ generator */

static inline uint64_t xo_mix64(uint64_t z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

/* Element `index` of the stream `seed`: (q - 2^23) * 2^-23 with q a 24-bit draw.
 * The value is exact in binary32 and lies in [-1, 1 - 2^-23]. */
XO_EXPORT float xo_uniform_at(uint64_t seed, uint64_t index) {
  const uint64_t u = xo_mix64(xo_mix64(seed) ^ index);
  const int32_t q = (int32_t)(u >> 40);
  return (float)(q - 8388608) * (1.0f / 8388608.0f);
}

XO_EXPORT void xo_fill_uniform(float* dst, uint64_t count, uint64_t seed, uint64_t first_index) {
  const uint64_t s = xo_mix64(seed);
  for (uint64_t i = 0; i < count; ++i) {
    const uint64_t u = xo_mix64(s ^ (first_index + i));
    dst[i] = (float)((int32_t)(u >> 40) - 8388608) * (1.0f / 8388608.0f);
  }
}

/* ------------------------------------------------------------------ FP64 GEMM */

typedef struct {
  int op_a, op_b;
  int64_t m, n, k;
  double alpha, beta;
  const float* a;
  int64_t lda;
  const float* b;
  int64_t ldb;
  const float* c;   /* may be NULL when beta == 0 */
  int64_t ldc;
  double* out;      /* m x n, column-major, leading dimension ldo */
  int64_t ldo;
  int64_t col_begin, col_end;
} xo_job;

static inline double xo_b_at(const xo_job* j, int64_t p, int64_t col) {
  return (double)(j->op_b == 0 ? j->b[p + col * j->ldb] : j->b[col + p * j->ldb]);
}

static void* xo_gemm_worker(void* arg) {
  const xo_job* j = (const xo_job*)arg;
  double* acc = NULL;
  if (j->op_a == 0) {
    acc = (double*)malloc((size_t)j->m * sizeof(double));
    if (!acc) return (void*)1;
  }
  for (int64_t col = j->col_begin; col < j->col_end; ++col) {
    double* o = j->out + col * j->ldo;
    if (j->op_a == 0) {
      /* op(A)(i,p) = A[i + p*lda]: stream A column p, k ascending per output. */
      memset(acc, 0, (size_t)j->m * sizeof(double));
      for (int64_t p = 0; p < j->k; ++p) {
        const double bv = xo_b_at(j, p, col);
        const float* ap = j->a + p * j->lda;
        for (int64_t i = 0; i < j->m; ++i) acc[i] += (double)ap[i] * bv;
      }
      for (int64_t i = 0; i < j->m; ++i) {
        const double cv = j->c ? (double)j->c[i + col * j->ldc] : 0.0;
        o[i] = j->alpha * acc[i] + j->beta * cv;
      }
    } else {
      /* op(A)(i,p) = A[p + i*lda]: contiguous in p. */
      for (int64_t i = 0; i < j->m; ++i) {
        const float* ai = j->a + i * j->lda;
        double dot = 0.0;
        if (j->op_b == 0) {
          const float* bj = j->b + col * j->ldb;
          for (int64_t p = 0; p < j->k; ++p) dot += (double)ai[p] * (double)bj[p];
        } else {
          for (int64_t p = 0; p < j->k; ++p) dot += (double)ai[p] * (double)j->b[col + p * j->ldb];
        }
        const double cv = j->c ? (double)j->c[i + col * j->ldc] : 0.0;
        o[i] = j->alpha * dot + j->beta * cv;
      }
    }
  }
  free(acc);
  return NULL;
}

/* out(i,j) = alpha * sum_p op(A)(i,p) op(B)(p,j) + beta * C(i,j), all in FP64.
 * Column-major; op 0 = N, 1 = T.  `threads` host threads split the n columns.
 * Returns 0 on success. */
XO_EXPORT int xo_gemm_f64(int op_a, int op_b, int64_t m, int64_t n, int64_t k, double alpha,
                          const float* a, int64_t lda, const float* b, int64_t ldb, double beta,
                          const float* c, int64_t ldc, double* out, int64_t ldo, int threads) {
  if (m <= 0 || n <= 0 || k <= 0 || (op_a != 0 && op_a != 1) || (op_b != 0 && op_b != 1))
    return 1;
  if (threads < 1) threads = 1;
  if (threads > n) threads = (int)n;
  xo_job* jobs = (xo_job*)calloc((size_t)threads, sizeof(xo_job));
  pthread_t* tids = (pthread_t*)calloc((size_t)threads, sizeof(pthread_t));
  if (!jobs || !tids) {
    free(jobs);
    free(tids);
    return 2;
  }
  int rc = 0;
  for (int t = 0; t < threads; ++t) {
    xo_job* j = &jobs[t];
    j->op_a = op_a; j->op_b = op_b; j->m = m; j->n = n; j->k = k;
    j->alpha = alpha; j->beta = beta;
    j->a = a; j->lda = lda; j->b = b; j->ldb = ldb; j->c = c; j->ldc = ldc;
    j->out = out; j->ldo = ldo;
    j->col_begin = n * t / threads;
    j->col_end = n * (t + 1) / threads;
  }
  int started = 0;
  for (int t = 1; t < threads; ++t) {
    if (pthread_create(&tids[t], NULL, xo_gemm_worker, &jobs[t]) != 0) { rc = 3; break; }
    ++started;
  }
  if (xo_gemm_worker(&jobs[0]) != NULL) rc = 4;
  for (int t = 1; t <= started; ++t) {
    void* r = NULL;
    pthread_join(tids[t], &r);
    if (r) rc = 4;
  }
  free(jobs);
  free(tids);
  return rc;
}

/* FP64-input GEMM for the FP64 arithmetic mode (the reference hands FP64 tiles to
 * cublasDgemm, src/platform/cublas/cublas_api.cpp:673-676, under the type rule of
 * src/gemm/planner.cpp:836-839): out = alpha * op(A) op(B) + beta * C with every product
 * and sum in long double (64-bit significand on x86-64), so the FP64 kernel's rounding
 * error is measured against a reference that carries 11 more bits.  Column-major,
 * single-threaded (test sizes).  Returns 0 on success. */
XO_EXPORT int xo_gemm_f64_inputs(int op_a, int op_b, int64_t m, int64_t n, int64_t k,
                                 double alpha, const double* a, int64_t lda, const double* b,
                                 int64_t ldb, double beta, const double* c, int64_t ldc,
                                 double* out, int64_t ldo) {
  if (m <= 0 || n <= 0 || k < 0 || (op_a != 0 && op_a != 1) || (op_b != 0 && op_b != 1))
    return 1;
  for (int64_t col = 0; col < n; ++col)
    for (int64_t i = 0; i < m; ++i) {
      long double dot = 0.0L;
      for (int64_t p = 0; p < k; ++p) {
        const long double x = op_a == 0 ? a[i + p * lda] : a[p + i * lda];
        const long double y = op_b == 0 ? b[p + col * ldb] : b[col + p * ldb];
        dot += x * y;
      }
      const long double cv = c ? (long double)c[i + col * ldc] : 0.0L;
      out[i + col * ldo] = (double)((long double)alpha * dot + (long double)beta * cv);
    }
  return 0;
}

typedef struct {
  int op_a, op_b;
  int64_t k;
  double alpha, beta;
  const float *a, *b, *c;
  int64_t lda, ldb, ldc;
  const int64_t *rows, *cols;
  double* out;
  int64_t begin, end;
} xo_sample_job;

static void* xo_sample_worker(void* arg) {
  const xo_sample_job* s = (const xo_sample_job*)arg;
  for (int64_t t = s->begin; t < s->end; ++t) {
    const int64_t i = s->rows[t], j = s->cols[t];
    double dot = 0.0;
    for (int64_t p = 0; p < s->k; ++p) {
      const double av = s->op_a == 0 ? s->a[i + p * s->lda] : s->a[p + i * s->lda];
      const double bv = s->op_b == 0 ? s->b[p + j * s->ldb] : s->b[j + p * s->ldb];
      dot += av * bv;
    }
    const double cv = s->c ? (double)s->c[i + j * s->ldc] : 0.0;
    s->out[t] = s->alpha * dot + s->beta * cv;
  }
  return NULL;
}

/* Same arithmetic as xo_gemm_f64 for a list of (row, col) outputs; used for the large
 * configurations where a full FP64 product is impractical. */
XO_EXPORT int xo_gemm_f64_sampled(int op_a, int op_b, int64_t k, double alpha, const float* a,
                                  int64_t lda, const float* b, int64_t ldb, double beta,
                                  const float* c, int64_t ldc, const int64_t* rows,
                                  const int64_t* cols, int64_t count, double* out, int threads) {
  if (count <= 0) return 0;
  if (threads < 1) threads = 1;
  if (threads > count) threads = (int)count;
  xo_sample_job* jobs = (xo_sample_job*)calloc((size_t)threads, sizeof(xo_sample_job));
  pthread_t* tids = (pthread_t*)calloc((size_t)threads, sizeof(pthread_t));
  if (!jobs || !tids) {
    free(jobs);
    free(tids);
    return 2;
  }
  for (int t = 0; t < threads; ++t) {
    xo_sample_job* s = &jobs[t];
    s->op_a = op_a; s->op_b = op_b; s->k = k; s->alpha = alpha; s->beta = beta;
    s->a = a; s->b = b; s->c = c; s->lda = lda; s->ldb = ldb; s->ldc = ldc;
    s->rows = rows; s->cols = cols; s->out = out;
    s->begin = count * t / threads;
    s->end = count * (t + 1) / threads;
  }
  int rc = 0, started = 0;
  for (int t = 1; t < threads; ++t) {
    if (pthread_create(&tids[t], NULL, xo_sample_worker, &jobs[t]) != 0) { rc = 3; break; }
    ++started;
  }
  xo_sample_worker(&jobs[0]);
  for (int t = 1; t <= started; ++t) pthread_join(tids[t], NULL);
  free(jobs);
  free(tids);
  return rc;
}

/* ------------------------------------------------------- reference patterns */

/* src/compat_bench/pattern.cpp:56-59 */
XO_EXPORT float xo_cb_pattern_a(uint64_t row, uint64_t k, uint64_t seed) {
  static const float cycle[4] = {1.0f, -1.0f, 0.5f, 0.5f};
  return (float)(1u + (row + seed % 3u) % 3u) * cycle[k % 4u];
}
/* src/compat_bench/pattern.cpp:60-64 */
XO_EXPORT float xo_cb_pattern_b(uint64_t k, uint64_t column, uint64_t seed) {
  static const float cycle[4] = {1.0f, 1.0f, 0.5f, 0.5f};
  return (float)(1u + (column + (seed >> 8u) % 3u) % 3u) * cycle[k % 4u];
}
/* src/compat_bench/pattern.cpp:65-67 */
XO_EXPORT float xo_cb_pattern_c(uint64_t row, uint64_t column) {
  return (float)(1u + (row + column) % 7u) * 0.25f;
}
/* src/compat_bench/pattern.cpp:68-83, full (k-loop) and periodic closed form. */
XO_EXPORT double xo_cb_reference_dot(uint64_t row, uint64_t column, uint64_t k, uint64_t seed,
                                     int full) {
  double total = 0.0;
  if (full) {
    for (uint64_t p = 0; p < k; ++p)
      total += (double)xo_cb_pattern_a(row, p, seed) * (double)xo_cb_pattern_b(p, column, seed);
    return total;
  }
  /* The operand cycles multiply to {1, -1, 0.25, 0.25} * scale, so every whole period of
   * four k steps adds 0.5 * scale; the ragged tail is summed term by term. */
  const double scale = (double)xo_cb_pattern_a(row, 0, seed) * (double)xo_cb_pattern_b(0, column, seed);
  total = (double)(k / 4u) * 0.5 * scale;
  for (uint64_t p = 0; p < k % 4u; ++p)
    total += (double)xo_cb_pattern_a(row, p, seed) * (double)xo_cb_pattern_b(p, column, seed);
  return total;
}
/* src/compat_bench/pattern.cpp:84-92: `passes` repeated C = alpha*AB + beta*C updates. */
XO_EXPORT double xo_cb_reference_result(uint64_t row, uint64_t column, uint64_t k, uint64_t seed,
                                        float alpha, float beta, uint32_t passes, int full) {
  const double dot = xo_cb_reference_dot(row, column, k, seed, full);
  double result = (double)xo_cb_pattern_c(row, column);
  for (uint32_t p = 0; p < passes; ++p) result = (double)alpha * dot + (double)beta * result;
  return result;
}

/* src/gemm_bench/pattern.cpp:207-213 */
XO_EXPORT uint64_t xo_gb_a(uint64_t row, uint64_t k) { return 1u + row % 3u + k % 2u; }
XO_EXPORT uint64_t xo_gb_b(uint64_t k, uint64_t column) { return 1u + column % 5u + k % 3u; }
/* src/gemm_bench/pattern.cpp:215-237: sum_p (a0 + p%2)(b0 + p%3) in closed form. */
XO_EXPORT uint64_t xo_gb_expected(uint64_t row, uint64_t column, uint64_t k) {
  static const uint64_t q_rem[3] = {0, 0, 1};
  static const uint64_t pq_rem[6] = {0, 0, 1, 1, 1, 1};
  const uint64_t a = 1u + row % 3u, b = 1u + column % 5u;
  const uint64_t sum_p = k / 2u;                              /* sum of p%2 */
  const uint64_t sum_q = 3u * (k / 3u) + q_rem[k % 3u];       /* sum of p%3 */
  const uint64_t sum_pq = 3u * (k / 6u) + pq_rem[k % 6u];     /* sum of (p%2)(p%3) */
  return k * a * b + a * sum_q + b * sum_p + sum_pq;
}

/* examples/preview-gemm/main.cpp:53-58 */
XO_EXPORT float xo_pv_a(int row, int column) { return (float)((row + 3 * column) % 17 - 8) / 16.0f; }
XO_EXPORT float xo_pv_b(int row, int column) { return (float)((2 * row + column) % 13 - 6) / 16.0f; }

/* src/compat_bench/executor.cpp:93-96 */
XO_EXPORT int xo_close_enough(double actual, double expected) {
  return isfinite(actual) && isfinite(expected) &&
         fabs(actual - expected) <= 1e-4 + 2e-5 * fabs(expected);
}
