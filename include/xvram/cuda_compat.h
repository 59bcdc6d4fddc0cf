/*
 * xvram/cuda_compat.h -- the cudaMalloc/cudaMemcpy/cublasSgemm-style C table
 * (B200 implementation).
 *
 * This is the drop-in boundary.  It is binary-compatible with the reference's
 * include/xvram/cuda_compat.h:
 *   reference include/xvram/cuda_compat.h:20-28   ABI version, lifecycle states, copy kinds
 *   reference include/xvram/cuda_compat.h:30-54   xvram_cuda_compat_config_v1 + defaults
 *   reference include/xvram/cuda_compat.h:56-101  xvram_cuda_compat_telemetry_v1
 *   reference include/xvram/cuda_compat.h:103-136 xvram_cuda_compat_api_v1 (function table)
 *   reference include/xvram/cuda_compat.h:138-139 xvram_cuda_compat_get_api (the one export)
 *
 * Semantics kept from the reference: device pointers handed out by malloc_device
 * are opaque stable addresses owned by the library; memcpy(H2D) stores into the
 * host-resident backing of the allocation (operands are streamed to HBM only when a
 * GEMM needs them); blas_sgemm is blocking, positive-dimension, column-major FP32 with
 * N/T operations, host-pointer alpha/beta and strict FP32 arithmetic; every call is
 * serialised; a failure after device work was submitted poisons the adapter; one
 * initialisation per process.
 *
 * What is different inside: the GEMM runs on the library's own sm_100a kernels (no
 * cuBLAS), operands stream from pinned host memory through a CUDA VMM frame pool in
 * HBM with copy/compute overlap, and the panel schedule is planned against the
 * device budget (session.cache_target_bytes).  The cublas_library paths of the
 * configuration are accepted and ignored.
 */
#ifndef XVRAM_CUDA_COMPAT_H
#define XVRAM_CUDA_COMPAT_H

#include "xvram.h"

#if defined(__GNUC__) && defined(XVRAM_BUILDING_CUDA_COMPAT)
#define XVRAM_CUDA_COMPAT_API __attribute__((visibility("default")))
#else
#define XVRAM_CUDA_COMPAT_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define XVRAM_CUDA_COMPAT_ABI_VERSION_1 UINT32_C(1)

/* Adapter lifecycle, reported in telemetry.state. */
enum {
  XVRAM_CUDA_COMPAT_UNINITIALIZED = 0,
  XVRAM_CUDA_COMPAT_INITIALIZING = 1,
  XVRAM_CUDA_COMPAT_READY = 2,
  XVRAM_CUDA_COMPAT_POISONED = 3,
  XVRAM_CUDA_COMPAT_CLOSED = 4
};

/* memcpy kinds (same values as cudaMemcpyHostToDevice / DeviceToHost). */
enum { XVRAM_CUDA_COMPAT_H2D = 1, XVRAM_CUDA_COMPAT_D2H = 2 };

/* Adapter configuration.  flags and reserved must be zero; session.context_mode must
 * be ISOLATED; the two library paths are either both empty or both absolute. */
typedef struct xvram_cuda_compat_config_v1 {
  uint32_t struct_size;
  uint32_t flags;
  xvram_session_config_v1 session;
  uint64_t stall_timeout_ms;
  char cublas_library[1024];
  char cublas_lt_library[1024];
  uint64_t reserved[4];
} xvram_cuda_compat_config_v1;

#define XVRAM_CUDA_COMPAT_CONFIG_V1_INIT                                                         \
  {(uint32_t)sizeof(xvram_cuda_compat_config_v1), 0U, XVRAM_SESSION_CONFIG_V1_INIT,              \
   UINT64_C(5000), {0}, {0}, {0, 0, 0, 0}}

/* Snapshot of the adapter: lifecycle, device, call accounting, allocation and copy
 * volume, GEMM tile progress and the residency counters in `runtime`. */
typedef struct xvram_cuda_compat_telemetry_v1 {
  uint32_t struct_size;
  uint32_t state;
  xvram_session_telemetry_v1 runtime;
  int32_t device_ordinal;
  uint32_t device_count;
  char device_name[128];
  uint64_t total_vram_bytes;
  uint64_t host_physical_bytes;
  uint64_t host_available_bytes;
  uint64_t host_store_cap_bytes;
  uint64_t host_headroom_bytes;
  uint64_t effective_chunk_bytes;
  uint64_t calls_attempted;
  uint64_t calls_submitted;
  uint64_t calls_completed;
  uint64_t calls_rejected;
  uint64_t allocations_created;
  uint64_t allocations_released;
  uint64_t live_allocations;
  uint64_t logical_bytes;
  uint64_t logical_bytes_peak;
  uint64_t handles_created;
  uint64_t handles_destroyed;
  uint64_t live_handles;
  uint64_t h2d_bytes;
  uint64_t d2h_bytes;
  uint64_t gemm_calls;
  uint64_t tiles_submitted;
  uint64_t tiles_retired;
  uint64_t progress_sequence;
  uint64_t retired_va_reservations;
  uint64_t retired_va_reservations_freed;
  uint64_t retired_va_bytes;
  uint64_t retired_va_bytes_freed;
  uint64_t host_backing_bytes;
  uint64_t host_backing_peak_bytes;
  uint64_t host_budget_bytes;
  uint32_t cleanup_operations_drained;
  uint32_t cleanup_events_drained;
  uint32_t cleanup_completed;
  uint32_t quarantined;
  uint64_t reserved[4];
} xvram_cuda_compat_telemetry_v1;

/* The function table.  Member order is the ABI. */
typedef struct xvram_cuda_compat_api_v1 {
  uint32_t struct_size;
  uint32_t abi_version;
  xvram_status(XVRAM_CALL* initialize)(const xvram_cuda_compat_config_v1* config);
  xvram_status(XVRAM_CALL* shutdown)(void);
  xvram_status(XVRAM_CALL* get_error)(xvram_error_info_v1* output);
  xvram_status(XVRAM_CALL* get_telemetry)(xvram_cuda_compat_telemetry_v1* output);
  xvram_status(XVRAM_CALL* malloc_device)(void** output, uint64_t bytes);
  xvram_status(XVRAM_CALL* free_device)(void* pointer);
  xvram_status(XVRAM_CALL* memcpy)(void* destination, const void* source, uint64_t bytes,
                                   uint32_t kind);
  xvram_status(XVRAM_CALL* get_device)(int32_t* output);
  xvram_status(XVRAM_CALL* get_device_count)(int32_t* output);
  xvram_status(XVRAM_CALL* set_device)(int32_t device);
  xvram_status(XVRAM_CALL* synchronize)(void);
  xvram_status(XVRAM_CALL* mem_get_info)(uint64_t* free_bytes, uint64_t* total_bytes);
  xvram_status(XVRAM_CALL* blas_create)(void** output);
  xvram_status(XVRAM_CALL* blas_destroy)(void* handle);
  xvram_status(XVRAM_CALL* blas_get_version)(void* handle, int32_t* output);
  xvram_status(XVRAM_CALL* blas_set_stream)(void* handle, uint64_t stream);
  xvram_status(XVRAM_CALL* blas_get_stream)(void* handle, uint64_t* output);
  xvram_status(XVRAM_CALL* blas_set_pointer_mode)(void* handle, uint32_t mode);
  xvram_status(XVRAM_CALL* blas_get_pointer_mode)(void* handle, uint32_t* output);
  xvram_status(XVRAM_CALL* blas_set_math_mode)(void* handle, uint32_t mode);
  xvram_status(XVRAM_CALL* blas_get_math_mode)(void* handle, uint32_t* output);
  /* C = alpha * op(A) * op(B) + beta * C, column-major FP32, op in {N, T}. */
  xvram_status(XVRAM_CALL* blas_sgemm)(void* handle, uint32_t op_a, uint32_t op_b, int32_t m,
                                       int32_t n, int32_t k, const float* alpha, const float* a,
                                       int32_t lda, const float* b, int32_t ldb, const float* beta,
                                       float* c, int32_t ldc);
  uint64_t reserved[8];
} xvram_cuda_compat_api_v1;

/* Copies the v1 table into `output` (caller_api_size writable bytes).
 * INVALID_ARGUMENT if output is NULL; INCOMPATIBLE_ABI if the version is not 1 or the
 * caller's table is smaller than v1.  Replaces reference src/cuda_compat/api.cpp:56-64. */
XVRAM_CUDA_COMPAT_API xvram_status XVRAM_CALL
xvram_cuda_compat_get_api(uint32_t requested_abi_version, uint32_t caller_api_size, void* output);

#ifdef __cplusplus
}
#endif
#endif /* XVRAM_CUDA_COMPAT_H */
