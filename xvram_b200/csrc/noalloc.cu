// noalloc.cu -- SGEMM on device pointers without allocating any device memory.
//
// Some callers cannot allocate device memory at the moment they need a GEMM: an
// application that has already given all of the GPU's memory to its own allocator (an
// inference server or framework running from a fixed arena), code that runs inside such an
// allocator's callbacks, where a cudaMalloc would fail or re-enter the allocator, and
// plugins whose host only lets them touch memory it hands in.  xvram_b200_sgemm_device
// takes its scratch from a memory pool, so it is unusable there; the entry point in this
// file takes it from a fixed array compiled into the library instead.
//
// The array lives in the library's device image: it occupies its
// XVRAM_B200_NOALLOC_SCRATCH_BYTES on every GPU where the library's device code is loaded,
// until the process exits.  Host code cannot use the name `noalloc_scratch` as an address
// (on the host it only names a stand-in object); the device address is looked up with
// cudaGetSymbolAddress, once per device, with that device current.
#include "xvram_b200.h"

#include "kernels.hpp"

#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>

namespace {

static __device__ __align__(256) unsigned char noalloc_scratch[XVRAM_B200_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mu;
void* g_scratch_addr[kMaxDevices] = {};

// Device address of noalloc_scratch on the current device; the first call per device looks
// it up (this may load the library's device code on that device).  The address is cached
// for the life of the process, so a cudaDeviceReset of that device afterwards is not
// supported (the next call would use the old context's address).
cudaError_t scratch_address(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess)
    return e;
  if (dev < 0 || dev >= kMaxDevices)
    return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (!g_scratch_addr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, noalloc_scratch);
    if (e != cudaSuccess)
      return e;
    g_scratch_addr[dev] = p;
  }
  *out = g_scratch_addr[dev];
  return cudaSuccess;
}

xvram_status status_of(cudaError_t e) {
  switch (e) {
  case cudaSuccess:
    return XVRAM_STATUS_SUCCESS;
  case cudaErrorInvalidValue:
  case cudaErrorInvalidConfiguration:
    return XVRAM_STATUS_INVALID_ARGUMENT;
  case cudaErrorNoDevice:
  case cudaErrorInvalidDevice:
  case cudaErrorInsufficientDriver:
    return XVRAM_STATUS_UNAVAILABLE;
  case cudaErrorMemoryAllocation: // loading the device code (and the array) found no room
    return XVRAM_STATUS_DEVICE_OUT_OF_MEMORY;
  default:
    return XVRAM_STATUS_CUDA_ERROR;
  }
}

} // namespace

extern "C" XVRAM_B200_API xvram_status XVRAM_CALL xvram_b200_sgemm_device_noalloc(
    uint32_t op_a, uint32_t op_b, int64_t m, int64_t n, int64_t k, float alpha, const float* a,
    int64_t lda, const float* b, int64_t ldb, float beta, float* c, int64_t ldc, uint64_t stream,
    uint32_t path) {
  if (op_a > 1 || op_b > 1 || m < 0 || n < 0 || k < 0 || m > INT32_MAX || n > INT32_MAX ||
      k > INT32_MAX || path > XVRAM_B200_PATH_GENERIC)
    return XVRAM_STATUS_INVALID_ARGUMENT;
  if (m == 0 || n == 0)
    return XVRAM_STATUS_SUCCESS;
  if (!c || ldc < m ||
      (k > 0 && (!a || !b || lda < (op_a == 0 ? m : k) || ldb < (op_b == 0 ? k : n))))
    return XVRAM_STATUS_INVALID_ARGUMENT;
  const int oa = static_cast<int>(op_a), ob = static_cast<int>(op_b);
  const int mi = static_cast<int>(m), ni = static_cast<int>(n), ki = static_cast<int>(k);
  const xvram::SgemmPath p = path == XVRAM_B200_PATH_TMA       ? xvram::SgemmPath::tma
                             : path == XVRAM_B200_PATH_GENERIC ? xvram::SgemmPath::generic
                                                               : xvram::SgemmPath::automatic;
  // Scratch is needed only when K-major operands will be transposed for the TMA kernel.
  const bool transposes =
      path != XVRAM_B200_PATH_GENERIC && xvram::sgemm_tma_eligible(oa, ob, a, lda, b, ldb);
  const uint64_t need = transposes ? xvram::sgemm_workspace_bytes(oa, ob, mi, ni, ki) : 0;
  if (need > XVRAM_B200_NOALLOC_SCRATCH_BYTES)
    return XVRAM_STATUS_BUDGET_PRESSURE; // more scratch than the fixed array holds
  void* ws = nullptr;
  if (need) {
    const cudaError_t e = scratch_address(&ws);
    if (e != cudaSuccess)
      return status_of(e);
  }
  // The transposes write every scratch byte the kernel then reads, so leftovers from
  // an earlier call never reach a result and nothing has to be cleared first.
  return status_of(xvram::sgemm_ffma_ws(oa, ob, mi, ni, ki, alpha, a, lda, b, ldb, beta, c, ldc,
                                        ws, need ? XVRAM_B200_NOALLOC_SCRATCH_BYTES : 0,
                                        reinterpret_cast<cudaStream_t>(stream), p));
}
