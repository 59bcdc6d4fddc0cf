/* compat_consumer.c -- a plain C program that uses the compat table the way a CUDA/cuBLAS
 * program uses cudaMalloc / cudaMemcpy / cublasSgemm, linked against this library with
 * only the public header (the reference's own consumers bind the same table; see
 * include/xvram/cuda_compat.h:103-139 in the reference).
 *
 * TEST INFRASTRUCTURE: built and run by tests/test_c_consumer_gpu.py.
 *
 * Flow: get the table, initialize, allocate A, B and C, copy them in, create a handle,
 * C = alpha op(A) op(B) + beta C for each of NN / NT / TN / TT on a ragged 37 x 19 x 67
 * problem with padded leading dimensions, copy C out, check every element against a
 * double-precision sum (|err| <= 1e-4 + 2e-5 |ref|), check that the padding rows of C
 * were not touched, then free everything and shut down.  Exit status 0 means all passed.
 */
#include "xvram/cuda_compat.h"

#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#define M 37
#define N 19
#define K 67
#define PAD 5
#define PAD_VALUE (-1234.5f)

/* Small exactly representable values (multiples of 1/16 in [-0.5, 0.5]). */
static float a_val(int r, int c) { return (float)(((r + 3 * c) % 17) - 8) / 16.0f; }
static float b_val(int r, int c) { return (float)(((2 * r + c) % 13) - 6) / 16.0f; }
static float c_val(int r, int c) { return (float)(((5 * r + 7 * c) % 11) - 5) / 8.0f; }

#define CHECK(call)                                                                          \
  do {                                                                                       \
    xvram_status st_ = (call);                                                               \
    if (st_ != XVRAM_STATUS_SUCCESS) {                                                       \
      fprintf(stderr, "%s failed with status %d\n", #call, (int)st_);                        \
      return 1;                                                                              \
    }                                                                                        \
  } while (0)

int main(void) {
  xvram_cuda_compat_api_v1 api;
  memset(&api, 0, sizeof api);
  CHECK(xvram_cuda_compat_get_api(XVRAM_CUDA_COMPAT_ABI_VERSION_1, (uint32_t)sizeof api, &api));
  xvram_cuda_compat_config_v1 cfg = XVRAM_CUDA_COMPAT_CONFIG_V1_INIT;
  CHECK(api.initialize(&cfg));
  /* The table's copy entry is named memcpy; calling it through a separate pointer keeps
     any memcpy macro of <string.h> out of the way. */
  xvram_status(XVRAM_CALL * copy)(void*, const void*, uint64_t, uint32_t) = api.memcpy;
  void* handle = NULL;
  CHECK(api.blas_create(&handle));
  int failures = 0;
  for (int op_a = 0; op_a < 2; ++op_a) {
    for (int op_b = 0; op_b < 2; ++op_b) {
      /* stored shapes (column-major) with padded leading dimensions */
      const int ar = op_a ? K : M, ac = op_a ? M : K;
      const int br = op_b ? N : K, bc = op_b ? K : N;
      const int lda = ar + PAD, ldb = br + PAD, ldc = M + PAD;
      const size_t na = (size_t)lda * ac, nb = (size_t)ldb * bc, nc = (size_t)ldc * N;
      float* ha = (float*)malloc(na * sizeof(float));
      float* hb = (float*)malloc(nb * sizeof(float));
      float* hc = (float*)malloc(nc * sizeof(float));
      float* out = (float*)malloc(nc * sizeof(float));
      if (!ha || !hb || !hc || !out)
        return 1;
      for (size_t i = 0; i < na; ++i)
        ha[i] = PAD_VALUE;
      for (size_t i = 0; i < nb; ++i)
        hb[i] = PAD_VALUE;
      for (size_t i = 0; i < nc; ++i)
        hc[i] = PAD_VALUE;
      /* op(A)(i, p) and op(B)(p, j) are the logical values a_val / b_val */
      for (int i = 0; i < M; ++i)
        for (int p = 0; p < K; ++p)
          ha[op_a ? (size_t)p + (size_t)i * lda : (size_t)i + (size_t)p * lda] = a_val(i, p);
      for (int p = 0; p < K; ++p)
        for (int j = 0; j < N; ++j)
          hb[op_b ? (size_t)j + (size_t)p * ldb : (size_t)p + (size_t)j * ldb] = b_val(p, j);
      for (int j = 0; j < N; ++j)
        for (int i = 0; i < M; ++i)
          hc[(size_t)i + (size_t)j * ldc] = c_val(i, j);
      void *da = NULL, *db = NULL, *dc = NULL;
      CHECK(api.malloc_device(&da, na * sizeof(float)));
      CHECK(api.malloc_device(&db, nb * sizeof(float)));
      CHECK(api.malloc_device(&dc, nc * sizeof(float)));
      CHECK(copy(da, ha, na * sizeof(float), XVRAM_CUDA_COMPAT_H2D));
      CHECK(copy(db, hb, nb * sizeof(float), XVRAM_CUDA_COMPAT_H2D));
      CHECK(copy(dc, hc, nc * sizeof(float), XVRAM_CUDA_COMPAT_H2D));
      const float alpha = 0.75f, beta = -0.5f;
      CHECK(api.blas_sgemm(handle, (uint32_t)op_a, (uint32_t)op_b, M, N, K, &alpha,
                           (const float*)da, lda, (const float*)db, ldb, &beta, (float*)dc,
                           ldc));
      CHECK(copy(out, dc, nc * sizeof(float), XVRAM_CUDA_COMPAT_D2H));
      int bad = 0;
      for (int j = 0; j < N; ++j) {
        for (int i = 0; i < ldc; ++i) {
          const float got = out[(size_t)i + (size_t)j * ldc];
          if (i >= M) { /* padding rows below m: never written */
            if (memcmp(&got, &hc[(size_t)i + (size_t)j * ldc], sizeof got) != 0)
              ++bad;
            continue;
          }
          double dot = 0.0;
          for (int p = 0; p < K; ++p)
            dot += (double)a_val(i, p) * (double)b_val(p, j);
          const double ref = (double)alpha * dot + (double)beta * (double)c_val(i, j);
          if (!(fabs((double)got - ref) <= 1e-4 + 2e-5 * fabs(ref)))
            ++bad;
        }
      }
      printf("op %c%c: %d mismatches\n", op_a ? 'T' : 'N', op_b ? 'T' : 'N', bad);
      failures += bad;
      CHECK(api.free_device(da));
      CHECK(api.free_device(db));
      CHECK(api.free_device(dc));
      free(ha);
      free(hb);
      free(hc);
      free(out);
    }
  }
  CHECK(api.blas_destroy(handle));
  CHECK(api.synchronize());
  CHECK(api.shutdown());
  return failures == 0 ? 0 : 2;
}
