// facade_consumer.cpp -- a cuBLAS-style C++ program (cudaMalloc / cudaMemcpy /
// cublasCreate / cublasSgemm / cudaFree, as written against the CUDA toolkit) compiled
// against <xvram/cuda_compat.hpp> with XVRAM_CUDA_COMPAT_REMAP_NAMES, and linked against
// libxvram_cuda_compat.so only: no libcudart, no libcublas.
//
// TEST INFRASTRUCTURE: built and run by tests/test_c_consumer_gpu.py.
//
// The adapter is initialised through the C table (the facade has no spelling for that),
// then C = alpha op(A) op(B) + beta C runs for op(A) = T, op(B) = N on a 300 x 200 x 128
// problem with padded leading dimensions; every element is checked against a double sum
// (|err| <= 1e-4 + 2e-5 |ref|), the error-state calls are exercised, and everything is
// released.  Exit status 0 means all passed.
#define XVRAM_CUDA_COMPAT_REMAP_NAMES 1
#include <xvram/cuda_compat.hpp>

#include <cmath>
#include <cstdio>
#include <vector>

namespace {
constexpr int kM = 300, kN = 200, kK = 128, kPad = 3;

float value(int r, int c, int salt) {
  return static_cast<float>(((r * 7 + c * 13 + salt) % 23) - 11) / 16.0F;
}

#define REQUIRE(cond)                                                                        \
  do {                                                                                       \
    if (!(cond)) {                                                                           \
      std::fprintf(stderr, "line %d: %s\n", __LINE__, #cond);                                \
      return 1;                                                                              \
    }                                                                                        \
  } while (0)
} // namespace

int main() {
  xvram_cuda_compat_api_v1 api{};
  REQUIRE(xvram_cuda_compat_get_api(XVRAM_CUDA_COMPAT_ABI_VERSION_1, sizeof(api), &api) ==
          XVRAM_STATUS_SUCCESS);
  // Before initialisation every call is refused as cudaErrorInitializationError.
  float* early = nullptr;
  REQUIRE(cudaMalloc(&early, 16) == cudaErrorInitializationError && early == nullptr);
  REQUIRE(cudaGetLastError() == cudaErrorInitializationError);
  REQUIRE(cudaPeekAtLastError() == cudaSuccess);

  const xvram_cuda_compat_config_v1 config = XVRAM_CUDA_COMPAT_CONFIG_V1_INIT;
  REQUIRE(api.initialize(&config) == XVRAM_STATUS_SUCCESS);
  int count = 0, device = -1;
  REQUIRE(cudaGetDeviceCount(&count) == cudaSuccess && count >= 1);
  REQUIRE(cudaGetDevice(&device) == cudaSuccess && device == 0);

  const int lda = kK + kPad, ldb = kK + kPad, ldc = kM + kPad;  // A is k x m (op T)
  std::vector<float> a(static_cast<size_t>(lda) * kM), b(static_cast<size_t>(ldb) * kN),
      c(static_cast<size_t>(ldc) * kN);
  for (int col = 0; col < kM; ++col)
    for (int row = 0; row < lda; ++row) a[row + static_cast<size_t>(col) * lda] = value(row, col, 1);
  for (int col = 0; col < kN; ++col)
    for (int row = 0; row < ldb; ++row) b[row + static_cast<size_t>(col) * ldb] = value(row, col, 2);
  for (int col = 0; col < kN; ++col)
    for (int row = 0; row < ldc; ++row) c[row + static_cast<size_t>(col) * ldc] = value(row, col, 3);
  const std::vector<float> c0 = c;

  float *da = nullptr, *db = nullptr, *dc = nullptr;
  REQUIRE(cudaMalloc(&da, a.size() * sizeof(float)) == cudaSuccess);
  REQUIRE(cudaMalloc(&db, b.size() * sizeof(float)) == cudaSuccess);
  REQUIRE(cudaMalloc(reinterpret_cast<void**>(&dc), c.size() * sizeof(float)) == cudaSuccess);
  REQUIRE(cudaMemcpy(da, a.data(), a.size() * sizeof(float), cudaMemcpyHostToDevice) == cudaSuccess);
  REQUIRE(cudaMemcpy(db, b.data(), b.size() * sizeof(float), cudaMemcpyHostToDevice) == cudaSuccess);
  REQUIRE(cudaMemcpy(dc, c.data(), c.size() * sizeof(float), cudaMemcpyHostToDevice) == cudaSuccess);

  cublasHandle_t handle = nullptr;
  REQUIRE(cublasCreate(&handle) == CUBLAS_STATUS_SUCCESS && handle != nullptr);
  cublasPointerMode_t mode = CUBLAS_POINTER_MODE_DEVICE;
  REQUIRE(cublasGetPointerMode(handle, &mode) == CUBLAS_STATUS_SUCCESS &&
          mode == CUBLAS_POINTER_MODE_HOST);
  const float alpha = 0.5F, beta = 1.5F;
  REQUIRE(cublasSgemm(handle, CUBLAS_OP_T, CUBLAS_OP_N, kM, kN, kK, &alpha, da, lda, db, ldb,
                      &beta, dc, ldc) == CUBLAS_STATUS_SUCCESS);
  // An invalid leading dimension maps to CUBLAS_STATUS_INVALID_VALUE and changes nothing.
  REQUIRE(cublasSgemm(handle, CUBLAS_OP_T, CUBLAS_OP_N, kM, kN, kK, &alpha, da, kK - 1, db, ldb,
                      &beta, dc, ldc) == CUBLAS_STATUS_INVALID_VALUE);
  REQUIRE(cudaDeviceSynchronize() == cudaSuccess);
  REQUIRE(cudaMemcpy(c.data(), dc, c.size() * sizeof(float), cudaMemcpyDeviceToHost) == cudaSuccess);

  long bad = 0;
  for (int col = 0; col < kN; ++col) {
    for (int row = 0; row < ldc; ++row) {
      const size_t at = row + static_cast<size_t>(col) * ldc;
      if (row >= kM) {  // padding rows are not part of C
        bad += c[at] != c0[at];
        continue;
      }
      double dot = 0;
      for (int i = 0; i < kK; ++i)
        dot += static_cast<double>(a[i + static_cast<size_t>(row) * lda]) *
               b[i + static_cast<size_t>(col) * ldb];
      const double want = alpha * dot + static_cast<double>(beta) * c0[at];
      bad += !(std::fabs(c[at] - want) <= 1e-4 + 2e-5 * std::fabs(want));
    }
  }
  std::printf("facade TN %dx%dx%d: %ld mismatches\n", kM, kN, kK, bad);
  REQUIRE(bad == 0);

  REQUIRE(cublasDestroy(handle) == CUBLAS_STATUS_SUCCESS);
  REQUIRE(cudaFree(da) == cudaSuccess && cudaFree(db) == cudaSuccess && cudaFree(dc) == cudaSuccess);
  REQUIRE(cudaFree(dc) == cudaErrorInvalidValue);  // double free is refused
  REQUIRE(cudaGetLastError() == cudaErrorInvalidValue);
  REQUIRE(api.shutdown() == XVRAM_STATUS_SUCCESS);
  std::printf("facade consumer passed\n");
  return 0;
}
