/* sdk_consumer.c -- a plain C program that uses the SDK v1 table (xvram_get_api) through
 * the public header, linked against the SDK drop-in library (libxvram.so, which exports
 * xvram_get_api alone).
 *
 * TEST INFRASTRUCTURE: built and run by tests/test_c_consumer_gpu.py.
 *
 * Flow: one session with a 16 MiB device budget and 2 MiB chunks; then
 *   1. an FP32 row-major GEMM (1536 x 1280 x 1024, op(B) = T, strict FP32) whose 20 MiB of
 *      operands exceed the budget, so the plan streams panels (tile_count > 1), run with
 *      gemm_execute;
 *   2. an FP64 column-major GEMM (96 x 80 x 70) submitted as an operation and waited for;
 * each result checked element by element against a double (or long double) sum.  Exit
 * status 0 means both passed.
 */
#include "xvram/xvram.h"

#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#define CHECK(call)                                                                          \
  do {                                                                                       \
    xvram_status st_ = (call);                                                               \
    if (st_ != XVRAM_STATUS_SUCCESS) {                                                       \
      fprintf(stderr, "%s failed with status %d\n", #call, (int)st_);                        \
      return 1;                                                                              \
    }                                                                                        \
  } while (0)

static double val(unsigned r, unsigned c, unsigned salt) {
  /* exactly representable values in [-0.5, 0.5) */
  return (double)((int)((r * 7u + c * 13u + salt * 5u) % 32u) - 16) / 32.0;
}

static xvram_status new_allocation(const xvram_api_v1* api, xvram_session s, uint64_t bytes,
                                   xvram_allocation* out) {
  xvram_allocation_desc_v1 d = XVRAM_ALLOCATION_DESC_V1_INIT;
  d.size_bytes = bytes;
  return api->allocation_create(s, &d, out);
}

int main(void) {
  xvram_api_v1 api;
  memset(&api, 0, sizeof api);
  CHECK(xvram_get_api(XVRAM_ABI_VERSION_1, (uint32_t)sizeof api, &api));
  xvram_session_config_v1 cfg = XVRAM_SESSION_CONFIG_V1_INIT;
  cfg.cache_target_bytes = 16u << 20;
  cfg.chunk_size_bytes = 2u << 20;
  xvram_session s = NULL;
  CHECK(api.session_create(&cfg, &s));
  int failures = 0;

  { /* 1. FP32, row-major, op(B) = T (B stored n x k), out of core */
    const unsigned m = 1536, n = 1280, k = 1024;
    float* a = (float*)malloc(sizeof(float) * m * k);
    float* b = (float*)malloc(sizeof(float) * n * k);
    float* c = (float*)malloc(sizeof(float) * m * n);
    float* out = (float*)malloc(sizeof(float) * m * n);
    if (!a || !b || !c || !out)
      return 1;
    for (unsigned i = 0; i < m; ++i)
      for (unsigned p = 0; p < k; ++p)
        a[i * k + p] = (float)val(i, p, 1);
    for (unsigned j = 0; j < n; ++j)
      for (unsigned p = 0; p < k; ++p)
        b[j * k + p] = (float)val(p, j, 2);
    for (unsigned i = 0; i < m; ++i)
      for (unsigned j = 0; j < n; ++j)
        c[i * n + j] = (float)val(i, j, 3);
    xvram_allocation A = NULL, B = NULL, C = NULL;
    CHECK(new_allocation(&api, s, sizeof(float) * m * k, &A));
    CHECK(new_allocation(&api, s, sizeof(float) * n * k, &B));
    CHECK(new_allocation(&api, s, sizeof(float) * m * n, &C));
    CHECK(api.allocation_write(A, 0, a, sizeof(float) * m * k));
    CHECK(api.allocation_write(B, 0, b, sizeof(float) * n * k));
    CHECK(api.allocation_write(C, 0, c, sizeof(float) * m * n));
    xvram_gemm_desc_v1 g = XVRAM_GEMM_DESC_V1_INIT;
    g.a.allocation = A;
    g.a.rows = m;
    g.a.columns = k;
    g.a.leading_dimension = k;
    g.b.allocation = B;
    g.b.rows = n;
    g.b.columns = k;
    g.b.leading_dimension = k;
    g.c.allocation = C;
    g.c.rows = m;
    g.c.columns = n;
    g.c.leading_dimension = n;
    g.operation_b = XVRAM_MATRIX_OP_T;
    g.compute_mode = XVRAM_COMPUTE_FP32_STRICT;
    g.alpha = 0.5;
    g.beta = 1.5;
    xvram_gemm_plan plan = NULL;
    CHECK(api.gemm_plan_create(s, &g, &plan));
    xvram_gemm_plan_info_v1 info = XVRAM_GEMM_PLAN_INFO_V1_INIT;
    CHECK(api.gemm_plan_get_info(plan, &info));
    CHECK(api.gemm_execute(plan, XVRAM_TIMEOUT_INFINITE));
    api.gemm_plan_release(plan);
    CHECK(api.allocation_read(C, 0, out, sizeof(float) * m * n));
    int bad = 0;
    double worst = 0.0;
    for (unsigned i = 0; i < m; ++i)
      for (unsigned j = 0; j < n; ++j) {
        double dot = 0.0;
        for (unsigned p = 0; p < k; ++p)
          dot += (double)a[i * k + p] * (double)b[j * k + p];
        const double ref = 0.5 * dot + 1.5 * (double)c[i * n + j];
        const double err = fabs((double)out[i * n + j] - ref) / (double)k; /* |a|,|b| <= 1/2 */
        if (err > worst)
          worst = err;
        if (!(err <= 1e-6))
          ++bad;
      }
    printf("fp32 row-major streamed: tiles %llu, max err/K %.3g, %d mismatches\n",
           (unsigned long long)info.tile_count, worst, bad);
    if (info.tile_count <= 1)
      ++bad;
    failures += bad;
    CHECK(api.allocation_release(A));
    CHECK(api.allocation_release(B));
    CHECK(api.allocation_release(C));
    free(a);
    free(b);
    free(c);
    free(out);
  }

  { /* 2. FP64, column-major, submitted and waited for */
    const unsigned m = 96, n = 80, k = 70;
    double* a = (double*)malloc(sizeof(double) * m * k);
    double* b = (double*)malloc(sizeof(double) * k * n);
    double* out = (double*)malloc(sizeof(double) * m * n);
    if (!a || !b || !out)
      return 1;
    for (unsigned p = 0; p < k; ++p)
      for (unsigned i = 0; i < m; ++i)
        a[i + p * m] = val(i, p, 4) + val(p, i, 5) / 4096.0; /* more than 24 bits */
    for (unsigned j = 0; j < n; ++j)
      for (unsigned p = 0; p < k; ++p)
        b[p + j * k] = val(p, j, 6) + val(j, p, 7) / 4096.0;
    xvram_allocation A = NULL, B = NULL, C = NULL;
    CHECK(new_allocation(&api, s, sizeof(double) * m * k, &A));
    CHECK(new_allocation(&api, s, sizeof(double) * k * n, &B));
    CHECK(new_allocation(&api, s, sizeof(double) * m * n, &C));
    CHECK(api.allocation_write(A, 0, a, sizeof(double) * m * k));
    CHECK(api.allocation_write(B, 0, b, sizeof(double) * k * n));
    xvram_gemm_desc_v1 g = XVRAM_GEMM_DESC_V1_INIT;
    g.a.allocation = A;
    g.a.data_type = XVRAM_DATA_FP64;
    g.a.rows = m;
    g.a.columns = k;
    g.a.leading_dimension = m;
    g.a.layout = XVRAM_MATRIX_COLUMN_MAJOR;
    g.b.allocation = B;
    g.b.data_type = XVRAM_DATA_FP64;
    g.b.rows = k;
    g.b.columns = n;
    g.b.leading_dimension = k;
    g.b.layout = XVRAM_MATRIX_COLUMN_MAJOR;
    g.c.allocation = C;
    g.c.data_type = XVRAM_DATA_FP64;
    g.c.rows = m;
    g.c.columns = n;
    g.c.leading_dimension = m;
    g.c.layout = XVRAM_MATRIX_COLUMN_MAJOR;
    g.compute_mode = XVRAM_COMPUTE_AUTO; /* FP64 data: FP64 arithmetic */
    xvram_gemm_plan plan = NULL;
    CHECK(api.gemm_plan_create(s, &g, &plan));
    xvram_operation op = NULL;
    CHECK(api.gemm_submit(plan, &op));
    xvram_operation_info_v1 oi = XVRAM_OPERATION_INFO_V1_INIT;
    CHECK(api.operation_wait(op, XVRAM_TIMEOUT_INFINITE, &oi));
    api.operation_release(op);
    api.gemm_plan_release(plan);
    CHECK(api.allocation_read(C, 0, out, sizeof(double) * m * n));
    int bad = 0;
    for (unsigned j = 0; j < n; ++j)
      for (unsigned i = 0; i < m; ++i) {
        long double dot = 0.0L;
        for (unsigned p = 0; p < k; ++p)
          dot += (long double)a[i + p * m] * (long double)b[p + j * k];
        if (!(fabsl((long double)out[i + j * m] - dot) <= 1e-13L * k))
          ++bad;
      }
    printf("fp64 column-major submitted: state %u, %d mismatches\n", (unsigned)oi.state, bad);
    if (oi.state != XVRAM_OPERATION_COMPLETED || oi.result != XVRAM_STATUS_SUCCESS)
      ++bad;
    failures += bad;
    CHECK(api.allocation_release(A));
    CHECK(api.allocation_release(B));
    CHECK(api.allocation_release(C));
    free(a);
    free(b);
    free(out);
  }

  CHECK(api.session_close(s, XVRAM_TIMEOUT_INFINITE));
  api.session_release(s);
  return failures == 0 ? 0 : 2;
}
