/* Prints the binary layout of the v1 compat ABI as JSON: sizeof and offsetof of every
 * field, enumerator values, and the bytes of the *_INIT default initialisers.
 * Compiled against the reference headers (XVRAM_DUMP_REFERENCE, by make_abi_layout.py)
 * and against include/ (by tests/test_abi_layout.py); the two outputs must match. */
#include <stddef.h>
#include <stdio.h>
#include <string.h>
#ifdef XVRAM_DUMP_REFERENCE
#include <xvram/cuda_compat.h>
#else
#include "xvram_cuda_compat.h"
#endif

static int first = 1;
static void sep(void) { printf(first ? "\n" : ",\n"); first = 0; }
/* Two levels so a struct name given through a macro (T below) is expanded first. */
#define SZ2(T) do { sep(); printf("  \"sizeof %s\": %zu", #T, sizeof(T)); } while (0)
#define OF2(T, f) do { sep(); printf("  \"%s.%s\": [%zu, %zu]", #T, #f, offsetof(T, f), sizeof(((T*)0)->f)); } while (0)
#define SZ(T) SZ2(T)
#define OF(T, f) OF2(T, f)
#define EN(e) do { sep(); printf("  \"%s\": %lld", #e, (long long)(e)); } while (0)
static void bytes(const char* name, const void* p, size_t n) {
  sep();
  printf("  \"init %s\": \"", name);
  for (size_t i = 0; i < n; ++i) printf("%02x", ((const unsigned char*)p)[i]);
  printf("\"");
}

int main(void) {
  printf("{");
  SZ(xvram_error_info_v1);
  OF(xvram_error_info_v1, struct_size); OF(xvram_error_info_v1, status);
  OF(xvram_error_info_v1, native_domain); OF(xvram_error_info_v1, reserved0);
  OF(xvram_error_info_v1, native_code); OF(xvram_error_info_v1, stage);
  OF(xvram_error_info_v1, operation); OF(xvram_error_info_v1, native_name);
  OF(xvram_error_info_v1, message);

  SZ(xvram_session_config_v1);
  OF(xvram_session_config_v1, struct_size); OF(xvram_session_config_v1, flags);
  OF(xvram_session_config_v1, device_ordinal); OF(xvram_session_config_v1, context_mode);
  OF(xvram_session_config_v1, chunk_size_bytes); OF(xvram_session_config_v1, cache_target_bytes);
  OF(xvram_session_config_v1, device_headroom_bytes); OF(xvram_session_config_v1, workspace_cap_bytes);
  OF(xvram_session_config_v1, budget_poll_ms); OF(xvram_session_config_v1, max_transaction_ms);
  OF(xvram_session_config_v1, staging_slots); OF(xvram_session_config_v1, cache_policy);
  OF(xvram_session_config_v1, prefetch_distance); OF(xvram_session_config_v1, reserved0);
  OF(xvram_session_config_v1, reserved);

  SZ(xvram_session_telemetry_v1);
#define T xvram_session_telemetry_v1
  OF(T, struct_size); OF(T, flags); OF(T, cache_target_bytes); OF(T, cache_target_minimum_bytes);
  OF(T, cache_target_maximum_bytes); OF(T, resident_bytes); OF(T, resident_bytes_peak);
  OF(T, workspace_bytes); OF(T, bytes_h2d); OF(T, bytes_d2h); OF(T, cache_hits); OF(T, cache_misses);
  OF(T, clean_evictions); OF(T, dirty_evictions); OF(T, writebacks_completed); OF(T, mappings);
  OF(T, unmaps); OF(T, set_access_calls); OF(T, handle_reuses); OF(T, unsafe_remaps);
  OF(T, unsafe_transitions); OF(T, budget_shrinks); OF(T, budget_grows); OF(T, cuda_driver_version);
  OF(T, cublas_version); OF(T, cublas_lt_available); OF(T, poisoned); OF(T, physical_handles_created);
  OF(T, physical_handles_released); OF(T, event_boundaries); OF(T, pinned_staging_bytes);
  OF(T, transactions_completed); OF(T, algorithm_selections); OF(T, algorithm_cache_hits);
  OF(T, last_transaction_ms); OF(T, budget_sample_count); OF(T, cuda_free_bytes_minimum);
  OF(T, cuda_free_bytes_end); OF(T, cublas_lt_version); OF(T, cublas_library_source);
  OF(T, wddm_available_bytes_minimum); OF(T, wddm_available_bytes_end); OF(T, wddm_budget_observed);
  OF(T, watchdog_rejections); OF(T, target_oom_retries);
#undef T

  SZ(xvram_cuda_compat_config_v1);
#define T xvram_cuda_compat_config_v1
  OF(T, struct_size); OF(T, flags); OF(T, session); OF(T, stall_timeout_ms);
  OF(T, cublas_library); OF(T, cublas_lt_library); OF(T, reserved);
#undef T

  SZ(xvram_cuda_compat_telemetry_v1);
#define T xvram_cuda_compat_telemetry_v1
  OF(T, struct_size); OF(T, state); OF(T, runtime); OF(T, device_ordinal); OF(T, device_count);
  OF(T, device_name); OF(T, total_vram_bytes); OF(T, host_physical_bytes); OF(T, host_available_bytes);
  OF(T, host_store_cap_bytes); OF(T, host_headroom_bytes); OF(T, effective_chunk_bytes);
  OF(T, calls_attempted); OF(T, calls_submitted); OF(T, calls_completed); OF(T, calls_rejected);
  OF(T, allocations_created); OF(T, allocations_released); OF(T, live_allocations); OF(T, logical_bytes);
  OF(T, logical_bytes_peak); OF(T, handles_created); OF(T, handles_destroyed); OF(T, live_handles);
  OF(T, h2d_bytes); OF(T, d2h_bytes); OF(T, gemm_calls); OF(T, tiles_submitted); OF(T, tiles_retired);
  OF(T, progress_sequence); OF(T, retired_va_reservations); OF(T, retired_va_reservations_freed);
  OF(T, retired_va_bytes); OF(T, retired_va_bytes_freed); OF(T, host_backing_bytes);
  OF(T, host_backing_peak_bytes); OF(T, host_budget_bytes); OF(T, cleanup_operations_drained);
  OF(T, cleanup_events_drained); OF(T, cleanup_completed); OF(T, quarantined); OF(T, reserved);
#undef T

  SZ(xvram_cuda_compat_api_v1);
#define T xvram_cuda_compat_api_v1
  OF(T, struct_size); OF(T, abi_version); OF(T, initialize); OF(T, shutdown); OF(T, get_error);
  OF(T, get_telemetry); OF(T, malloc_device); OF(T, free_device); OF(T, memcpy); OF(T, get_device);
  OF(T, get_device_count); OF(T, set_device); OF(T, synchronize); OF(T, mem_get_info);
  OF(T, blas_create); OF(T, blas_destroy); OF(T, blas_get_version); OF(T, blas_set_stream);
  OF(T, blas_get_stream); OF(T, blas_set_pointer_mode); OF(T, blas_get_pointer_mode);
  OF(T, blas_set_math_mode); OF(T, blas_get_math_mode); OF(T, blas_sgemm); OF(T, reserved);
#undef T

  EN(XVRAM_ABI_VERSION_1); EN(XVRAM_ABI_VERSION_CURRENT); EN(XVRAM_TIMEOUT_INFINITE);
  EN(XVRAM_STATUS_SUCCESS); EN(XVRAM_STATUS_INVALID_ARGUMENT); EN(XVRAM_STATUS_INCOMPATIBLE_ABI);
  EN(XVRAM_STATUS_UNSUPPORTED); EN(XVRAM_STATUS_UNAVAILABLE); EN(XVRAM_STATUS_HOST_OUT_OF_MEMORY);
  EN(XVRAM_STATUS_DEVICE_OUT_OF_MEMORY); EN(XVRAM_STATUS_BUDGET_PRESSURE); EN(XVRAM_STATUS_BUSY);
  EN(XVRAM_STATUS_NOT_READY); EN(XVRAM_STATUS_TIMEOUT); EN(XVRAM_STATUS_CORRUPTION);
  EN(XVRAM_STATUS_CALLBACK_FAILED); EN(XVRAM_STATUS_CUDA_ERROR); EN(XVRAM_STATUS_CUBLAS_ERROR);
  EN(XVRAM_STATUS_POISONED); EN(XVRAM_STATUS_CLEANUP_FAILED); EN(XVRAM_STATUS_CLOSED);
  EN(XVRAM_STATUS_CANCELLED); EN(XVRAM_STATUS_INTERNAL);
  EN(XVRAM_NATIVE_ERROR_NONE); EN(XVRAM_NATIVE_ERROR_CUDA); EN(XVRAM_NATIVE_ERROR_CUBLAS);
  EN(XVRAM_NATIVE_ERROR_PLATFORM); EN(XVRAM_NATIVE_ERROR_CALLBACK); EN(XVRAM_NATIVE_ERROR_INTERNAL);
  EN(XVRAM_CONTEXT_ISOLATED); EN(XVRAM_CONTEXT_ATTACH_CURRENT);
  EN(XVRAM_CACHE_POLICY_CLOCK); EN(XVRAM_CACHE_POLICY_LRU);
  EN(XVRAM_MATRIX_OP_N); EN(XVRAM_MATRIX_OP_T);
  EN(XVRAM_TELEMETRY_STABLE_VIRTUAL_ADDRESSES); EN(XVRAM_TELEMETRY_NO_PHYSICAL_ALIASES);
  EN(XVRAM_CUDA_COMPAT_ABI_VERSION_1);
  EN(XVRAM_CUDA_COMPAT_UNINITIALIZED); EN(XVRAM_CUDA_COMPAT_INITIALIZING);
  EN(XVRAM_CUDA_COMPAT_READY); EN(XVRAM_CUDA_COMPAT_POISONED); EN(XVRAM_CUDA_COMPAT_CLOSED);
  EN(XVRAM_CUDA_COMPAT_H2D); EN(XVRAM_CUDA_COMPAT_D2H);

  {
    xvram_error_info_v1 e = XVRAM_ERROR_INFO_V1_INIT;
    xvram_session_config_v1 s;
    xvram_cuda_compat_config_v1 c;
    memset(&s, 0, sizeof s);
    memset(&c, 0, sizeof c);
    { xvram_session_config_v1 t = XVRAM_SESSION_CONFIG_V1_INIT; memcpy(&s, &t, sizeof s); }
    { xvram_cuda_compat_config_v1 t = XVRAM_CUDA_COMPAT_CONFIG_V1_INIT; memcpy(&c, &t, sizeof c); }
    bytes("xvram_error_info_v1", &e, sizeof e);
    bytes("xvram_session_config_v1", &s, sizeof s);
    /* The compat config is 2 KiB of mostly zero path buffers; its head and tail suffice. */
    bytes("xvram_cuda_compat_config_v1[head]", &c, offsetof(xvram_cuda_compat_config_v1, cublas_library));
    bytes("xvram_cuda_compat_config_v1[tail]", c.reserved, sizeof c.reserved);
  }
  printf("\n}\n");
  return 0;
}
