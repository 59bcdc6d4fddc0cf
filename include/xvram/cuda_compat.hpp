/*
 * xvram/cuda_compat.hpp -- header-only C++ facade that spells the compat table as the
 * CUDA runtime / cuBLAS calls it replaces (B200 implementation).
 *
 * Source-compatible with the reference's include/xvram/cuda_compat.hpp: the same
 * functions in namespace xvram::cuda_compat, the same xvram_status -> cudaError_t and
 * xvram_status -> cublasStatus_t mapping (callers branch on those codes), a thread-local
 * last error behind cudaGetLastError / cudaPeekAtLastError, and the same opt-in
 * XVRAM_CUDA_COMPAT_REMAP_NAMES spelling macros.  Everything goes through the one
 * exported symbol, xvram_cuda_compat_get_api; nothing links against libcudart or
 * libcublas.  The table is negotiated once per process; a failed negotiation, a table
 * of another ABI version or an empty member makes the affected calls answer
 * cudaErrorNotSupported / CUBLAS_STATUS_NOT_SUPPORTED instead of calling through a null
 * pointer.
 *
 *   reference include/xvram/cuda_compat.hpp:3-5     host compiler only
 *   reference include/xvram/cuda_compat.hpp:22-58   table negotiation, missing members
 *   reference include/xvram/cuda_compat.hpp:59-140  status mappings, thread-local error
 *   reference include/xvram/cuda_compat.hpp:141-232 the runtime and cuBLAS spellings
 *   reference include/xvram/cuda_compat.hpp:234-258 XVRAM_CUDA_COMPAT_REMAP_NAMES
 */
#ifndef XVRAM_CUDA_COMPAT_HPP
#define XVRAM_CUDA_COMPAT_HPP

#if defined(__CUDACC__) || defined(__CUDA_ARCH__)
#error "XVRAM_CUDA_COMPAT_HOST_ONLY: this facade is host code; build it with the host C++ compiler, not nvcc"
#endif

#include "cuda_compat.h"

#include <cublas_v2.h>
#include <cuda_runtime_api.h>

#include <cstddef>
#include <cstdint>

/* cublas_v2.h maps these spellings onto versioned symbols (cublasCreate_v2, ...).  The
 * facade defines its own functions under the plain names, so only these maps go; every
 * other CUDA and cuBLAS name keeps its native declaration (and, unlinked, fails to link). */
#undef cublasCreate
#undef cublasDestroy
#undef cublasGetVersion
#undef cublasSetStream
#undef cublasGetStream
#undef cublasSetPointerMode
#undef cublasGetPointerMode
#undef cublasSgemm

namespace xvram::cuda_compat {
namespace detail {

/* A stand-in for a table member that is absent or unusable: same signature, refuses. */
template <class Member> struct Refuse;
template <class... Args> struct Refuse<xvram_status(XVRAM_CALL*)(Args...)> {
  static xvram_status XVRAM_CALL call(Args...) noexcept { return XVRAM_STATUS_INCOMPATIBLE_ABI; }
};

template <class Member> inline void keep_or_refuse(Member& slot, bool usable) noexcept {
  if (!usable || slot == nullptr)
    slot = &Refuse<Member>::call;
}

inline xvram_cuda_compat_api_v1 negotiate() noexcept {
  xvram_cuda_compat_api_v1 t{};
  const xvram_status st = xvram_cuda_compat_get_api(XVRAM_CUDA_COMPAT_ABI_VERSION_1,
                                                    static_cast<uint32_t>(sizeof(t)), &t);
  const bool usable = st == XVRAM_STATUS_SUCCESS && t.struct_size >= sizeof(t) &&
                      t.abi_version == XVRAM_CUDA_COMPAT_ABI_VERSION_1;
  keep_or_refuse(t.initialize, usable);
  keep_or_refuse(t.shutdown, usable);
  keep_or_refuse(t.get_error, usable);
  keep_or_refuse(t.get_telemetry, usable);
  keep_or_refuse(t.malloc_device, usable);
  keep_or_refuse(t.free_device, usable);
  keep_or_refuse(t.memcpy, usable);
  keep_or_refuse(t.get_device, usable);
  keep_or_refuse(t.get_device_count, usable);
  keep_or_refuse(t.set_device, usable);
  keep_or_refuse(t.synchronize, usable);
  keep_or_refuse(t.mem_get_info, usable);
  keep_or_refuse(t.blas_create, usable);
  keep_or_refuse(t.blas_destroy, usable);
  keep_or_refuse(t.blas_get_version, usable);
  keep_or_refuse(t.blas_set_stream, usable);
  keep_or_refuse(t.blas_get_stream, usable);
  keep_or_refuse(t.blas_set_pointer_mode, usable);
  keep_or_refuse(t.blas_get_pointer_mode, usable);
  keep_or_refuse(t.blas_set_math_mode, usable);
  keep_or_refuse(t.blas_get_math_mode, usable);
  keep_or_refuse(t.blas_sgemm, usable);
  return t;
}

/* Negotiated on first use (thread-safe static initialisation), once per process. */
inline const xvram_cuda_compat_api_v1& table() noexcept {
  static const xvram_cuda_compat_api_v1 negotiated = negotiate();
  return negotiated;
}

/* Indexed by xvram_status (0 .. XVRAM_STATUS_INTERNAL). */
inline constexpr cudaError_t kRuntimeError[] = {
    cudaSuccess,                  /* SUCCESS */
    cudaErrorInvalidValue,        /* INVALID_ARGUMENT */
    cudaErrorNotSupported,        /* INCOMPATIBLE_ABI */
    cudaErrorNotSupported,        /* UNSUPPORTED */
    cudaErrorNoDevice,            /* UNAVAILABLE */
    cudaErrorMemoryAllocation,    /* HOST_OUT_OF_MEMORY */
    cudaErrorMemoryAllocation,    /* DEVICE_OUT_OF_MEMORY */
    cudaErrorMemoryAllocation,    /* BUDGET_PRESSURE */
    cudaErrorUnknown,             /* BUSY */
    cudaErrorInitializationError, /* NOT_READY */
    cudaErrorLaunchTimeout,       /* TIMEOUT */
    cudaErrorLaunchFailure,       /* CORRUPTION */
    cudaErrorUnknown,             /* CALLBACK_FAILED */
    cudaErrorLaunchFailure,       /* CUDA_ERROR */
    cudaErrorUnknown,             /* CUBLAS_ERROR */
    cudaErrorLaunchFailure,       /* POISONED */
    cudaErrorLaunchFailure,       /* CLEANUP_FAILED */
    cudaErrorInitializationError, /* CLOSED */
    cudaErrorUnknown,             /* CANCELLED */
    cudaErrorUnknown,             /* INTERNAL */
};
inline constexpr cublasStatus_t kBlasStatus[] = {
    CUBLAS_STATUS_SUCCESS,          /* SUCCESS */
    CUBLAS_STATUS_INVALID_VALUE,    /* INVALID_ARGUMENT */
    CUBLAS_STATUS_NOT_SUPPORTED,    /* INCOMPATIBLE_ABI */
    CUBLAS_STATUS_NOT_SUPPORTED,    /* UNSUPPORTED */
    CUBLAS_STATUS_NOT_INITIALIZED,  /* UNAVAILABLE */
    CUBLAS_STATUS_ALLOC_FAILED,     /* HOST_OUT_OF_MEMORY */
    CUBLAS_STATUS_ALLOC_FAILED,     /* DEVICE_OUT_OF_MEMORY */
    CUBLAS_STATUS_ALLOC_FAILED,     /* BUDGET_PRESSURE */
    CUBLAS_STATUS_INTERNAL_ERROR,   /* BUSY */
    CUBLAS_STATUS_NOT_INITIALIZED,  /* NOT_READY */
    CUBLAS_STATUS_EXECUTION_FAILED, /* TIMEOUT */
    CUBLAS_STATUS_EXECUTION_FAILED, /* CORRUPTION */
    CUBLAS_STATUS_INTERNAL_ERROR,   /* CALLBACK_FAILED */
    CUBLAS_STATUS_EXECUTION_FAILED, /* CUDA_ERROR */
    CUBLAS_STATUS_EXECUTION_FAILED, /* CUBLAS_ERROR */
    CUBLAS_STATUS_EXECUTION_FAILED, /* POISONED */
    CUBLAS_STATUS_INTERNAL_ERROR,   /* CLEANUP_FAILED */
    CUBLAS_STATUS_NOT_INITIALIZED,  /* CLOSED */
    CUBLAS_STATUS_INTERNAL_ERROR,   /* CANCELLED */
    CUBLAS_STATUS_INTERNAL_ERROR,   /* INTERNAL */
};
inline constexpr std::size_t kStatusCount = sizeof(kRuntimeError) / sizeof(kRuntimeError[0]);
static_assert(kStatusCount == XVRAM_STATUS_INTERNAL + 1, "one entry per xvram_status");
static_assert(sizeof(kBlasStatus) / sizeof(kBlasStatus[0]) == kStatusCount,
              "one entry per xvram_status");

/* The facade's cudaGetLastError state: per thread, set by every failing runtime call. */
inline thread_local cudaError_t t_last_error = cudaSuccess;

inline cudaError_t runtime_result(xvram_status st) noexcept {
  const cudaError_t e = st < kStatusCount ? kRuntimeError[st] : cudaErrorUnknown;
  if (e != cudaSuccess)
    t_last_error = e;
  return e;
}
inline cublasStatus_t blas_result(xvram_status st) noexcept {
  return st < kStatusCount ? kBlasStatus[st] : CUBLAS_STATUS_INTERNAL_ERROR;
}

} // namespace detail

/* ---- CUDA runtime spellings ---------------------------------------------------------- */
inline cudaError_t cudaMalloc(void** ptr, std::size_t bytes) noexcept {
  return detail::runtime_result(detail::table().malloc_device(ptr, bytes));
}
template <class T> inline cudaError_t cudaMalloc(T** ptr, std::size_t bytes) noexcept {
  return detail::runtime_result(
      detail::table().malloc_device(reinterpret_cast<void**>(ptr), bytes));
}
inline cudaError_t cudaFree(void* ptr) noexcept {
  return detail::runtime_result(detail::table().free_device(ptr));
}
inline cudaError_t cudaMemcpy(void* dst, const void* src, std::size_t bytes,
                              cudaMemcpyKind kind) noexcept {
  return detail::runtime_result(
      detail::table().memcpy(dst, src, bytes, static_cast<uint32_t>(kind)));
}
inline cudaError_t cudaGetDevice(int* device) noexcept {
  return detail::runtime_result(detail::table().get_device(device));
}
inline cudaError_t cudaGetDeviceCount(int* count) noexcept {
  return detail::runtime_result(detail::table().get_device_count(count));
}
inline cudaError_t cudaSetDevice(int device) noexcept {
  return detail::runtime_result(detail::table().set_device(device));
}
inline cudaError_t cudaDeviceSynchronize() noexcept {
  return detail::runtime_result(detail::table().synchronize());
}
inline cudaError_t cudaPeekAtLastError() noexcept { return detail::t_last_error; }
inline cudaError_t cudaGetLastError() noexcept {
  const cudaError_t e = detail::t_last_error;
  detail::t_last_error = cudaSuccess;
  return e;
}
/* Names for the codes this facade can return; anything else reads as cudaErrorUnknown. */
inline const char* cudaGetErrorName(cudaError_t error) noexcept {
  struct Named {
    cudaError_t code;
    const char* name;
  };
  static constexpr Named kNames[] = {
      {cudaSuccess, "cudaSuccess"},
      {cudaErrorInvalidValue, "cudaErrorInvalidValue"},
      {cudaErrorMemoryAllocation, "cudaErrorMemoryAllocation"},
      {cudaErrorInitializationError, "cudaErrorInitializationError"},
      {cudaErrorNoDevice, "cudaErrorNoDevice"},
      {cudaErrorNotSupported, "cudaErrorNotSupported"},
      {cudaErrorLaunchTimeout, "cudaErrorLaunchTimeout"},
      {cudaErrorLaunchFailure, "cudaErrorLaunchFailure"},
  };
  for (const Named& n : kNames)
    if (n.code == error)
      return n.name;
  return "cudaErrorUnknown";
}
inline const char* cudaGetErrorString(cudaError_t error) noexcept {
  return xvram::cuda_compat::cudaGetErrorName(error);
}

/* ---- cuBLAS spellings ---------------------------------------------------------------- */
inline cublasStatus_t cublasCreate(cublasHandle_t* handle) noexcept {
  return detail::blas_result(detail::table().blas_create(reinterpret_cast<void**>(handle)));
}
inline cublasStatus_t cublasDestroy(cublasHandle_t handle) noexcept {
  return detail::blas_result(detail::table().blas_destroy(handle));
}
inline cublasStatus_t cublasGetVersion(cublasHandle_t handle, int* version) noexcept {
  return detail::blas_result(detail::table().blas_get_version(handle, version));
}
inline cublasStatus_t cublasSetStream(cublasHandle_t handle, cudaStream_t stream) noexcept {
  return detail::blas_result(
      detail::table().blas_set_stream(handle, reinterpret_cast<uintptr_t>(stream)));
}
inline cublasStatus_t cublasGetStream(cublasHandle_t handle, cudaStream_t* stream) noexcept {
  return detail::blas_result(
      detail::table().blas_get_stream(handle, reinterpret_cast<uint64_t*>(stream)));
}
inline cublasStatus_t cublasSetPointerMode(cublasHandle_t handle,
                                           cublasPointerMode_t mode) noexcept {
  return detail::blas_result(
      detail::table().blas_set_pointer_mode(handle, static_cast<uint32_t>(mode)));
}
inline cublasStatus_t cublasGetPointerMode(cublasHandle_t handle,
                                           cublasPointerMode_t* mode) noexcept {
  static_assert(sizeof(cublasPointerMode_t) == sizeof(uint32_t), "enum read as uint32_t");
  return detail::blas_result(
      detail::table().blas_get_pointer_mode(handle, reinterpret_cast<uint32_t*>(mode)));
}
inline cublasStatus_t cublasSetMathMode(cublasHandle_t handle, cublasMath_t mode) noexcept {
  return detail::blas_result(
      detail::table().blas_set_math_mode(handle, static_cast<uint32_t>(mode)));
}
inline cublasStatus_t cublasGetMathMode(cublasHandle_t handle, cublasMath_t* mode) noexcept {
  static_assert(sizeof(cublasMath_t) == sizeof(uint32_t), "enum read as uint32_t");
  return detail::blas_result(
      detail::table().blas_get_math_mode(handle, reinterpret_cast<uint32_t*>(mode)));
}
inline cublasStatus_t cublasSgemm(cublasHandle_t handle, cublasOperation_t op_a,
                                  cublasOperation_t op_b, int m, int n, int k, const float* alpha,
                                  const float* a, int lda, const float* b, int ldb,
                                  const float* beta, float* c, int ldc) noexcept {
  return detail::blas_result(detail::table().blas_sgemm(
      handle, static_cast<uint32_t>(op_a), static_cast<uint32_t>(op_b), m, n, k, alpha, a, lda,
      b, ldb, beta, c, ldc));
}

} // namespace xvram::cuda_compat

/* Opt-in: with XVRAM_CUDA_COMPAT_REMAP_NAMES defined non-zero before this header, the
 * listed CUDA / cuBLAS spellings (bare or ::-qualified) resolve to the facade.  Without it,
 * call xvram::cuda_compat::cudaMalloc and so on explicitly. */
#if defined(XVRAM_CUDA_COMPAT_REMAP_NAMES) && XVRAM_CUDA_COMPAT_REMAP_NAMES
#define cudaMalloc xvram::cuda_compat::cudaMalloc
#define cudaFree xvram::cuda_compat::cudaFree
#define cudaMemcpy xvram::cuda_compat::cudaMemcpy
#define cudaGetDevice xvram::cuda_compat::cudaGetDevice
#define cudaGetDeviceCount xvram::cuda_compat::cudaGetDeviceCount
#define cudaSetDevice xvram::cuda_compat::cudaSetDevice
#define cudaDeviceSynchronize xvram::cuda_compat::cudaDeviceSynchronize
#define cudaPeekAtLastError xvram::cuda_compat::cudaPeekAtLastError
#define cudaGetLastError xvram::cuda_compat::cudaGetLastError
#define cudaGetErrorName xvram::cuda_compat::cudaGetErrorName
#define cudaGetErrorString xvram::cuda_compat::cudaGetErrorString
#define cublasCreate xvram::cuda_compat::cublasCreate
#define cublasDestroy xvram::cuda_compat::cublasDestroy
#define cublasGetVersion xvram::cuda_compat::cublasGetVersion
#define cublasSetStream xvram::cuda_compat::cublasSetStream
#define cublasGetStream xvram::cuda_compat::cublasGetStream
#define cublasSetPointerMode xvram::cuda_compat::cublasSetPointerMode
#define cublasGetPointerMode xvram::cuda_compat::cublasGetPointerMode
#define cublasSetMathMode xvram::cuda_compat::cublasSetMathMode
#define cublasGetMathMode xvram::cuda_compat::cublasGetMathMode
#define cublasSgemm xvram::cuda_compat::cublasSgemm
#endif

#endif /* XVRAM_CUDA_COMPAT_HPP */
