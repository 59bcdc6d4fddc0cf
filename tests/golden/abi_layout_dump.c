/* Prints the binary layout of the v1 compat and SDK ABIs as JSON: sizeof and offsetof of every
 * field, enumerator values, and the bytes of the *_INIT default initialisers.
 * Compiled against the reference headers (XVRAM_DUMP_REFERENCE, by make_abi_layout.py)
 * and against include/ (by tests/test_abi_layout.py); the two outputs must match. */
#include <stddef.h>
#include <stdio.h>
#include <string.h>
/* Both header sets are found as <xvram/...> through -I. */
#include <xvram/cuda_compat.h>

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

  /* SDK v1 (xvram_get_api) */
  SZ(xvram_allocation_desc_v1);
#define T xvram_allocation_desc_v1
  OF(T, struct_size); OF(T, flags); OF(T, size_bytes); OF(T, alignment_bytes); OF(T, priority);
  OF(T, reserved0); OF(T, reserved);
#undef T
  SZ(xvram_allocation_info_v1);
#define T xvram_allocation_info_v1
  OF(T, struct_size); OF(T, flags); OF(T, allocation_id); OF(T, size_bytes); OF(T, alignment_bytes);
  OF(T, priority); OF(T, stable_virtual_address); OF(T, reserved);
#undef T
  SZ(xvram_access_range_v1);
#define T xvram_access_range_v1
  OF(T, allocation); OF(T, offset_bytes); OF(T, length_bytes); OF(T, mode); OF(T, reserved0);
#undef T
  SZ(xvram_prefetch_desc_v1);
#define T xvram_prefetch_desc_v1
  OF(T, struct_size); OF(T, flags); OF(T, ranges); OF(T, range_count); OF(T, deadline_ms);
  OF(T, reserved);
#undef T
  SZ(xvram_resolved_range_v1);
#define T xvram_resolved_range_v1
  OF(T, allocation_id); OF(T, offset_bytes); OF(T, length_bytes); OF(T, device_address);
  OF(T, mode); OF(T, reserved0);
#undef T
  SZ(xvram_transaction_context_v1);
#define T xvram_transaction_context_v1
  OF(T, struct_size); OF(T, flags); OF(T, operation_id); OF(T, transaction_id); OF(T, ranges);
  OF(T, range_count); OF(T, workspace_device_address); OF(T, workspace_bytes);
  OF(T, native_stream); OF(T, reserved);
#undef T
  SZ(xvram_transaction_desc_v1);
#define T xvram_transaction_desc_v1
  OF(T, struct_size); OF(T, flags); OF(T, ranges); OF(T, range_count); OF(T, workspace_bytes);
  OF(T, deadline_ms); OF(T, callback); OF(T, user_data); OF(T, reserved);
#undef T
  SZ(xvram_operation_info_v1);
#define T xvram_operation_info_v1
  OF(T, struct_size); OF(T, state); OF(T, result); OF(T, reserved0); OF(T, operation_id);
  OF(T, units_completed); OF(T, units_total); OF(T, elapsed_ms); OF(T, bytes_h2d); OF(T, bytes_d2h);
  OF(T, cache_hits); OF(T, cache_misses); OF(T, reserved);
#undef T
  SZ(xvram_matrix_v1);
#define T xvram_matrix_v1
  OF(T, struct_size); OF(T, data_type); OF(T, allocation); OF(T, offset_bytes); OF(T, rows);
  OF(T, columns); OF(T, leading_dimension); OF(T, layout); OF(T, reserved0); OF(T, reserved);
#undef T
  SZ(xvram_gemm_desc_v1);
#define T xvram_gemm_desc_v1
  OF(T, struct_size); OF(T, flags); OF(T, a); OF(T, b); OF(T, c); OF(T, operation_a);
  OF(T, operation_b); OF(T, compute_mode); OF(T, reserved0); OF(T, alpha); OF(T, beta);
  OF(T, workspace_cap_bytes); OF(T, deadline_ms); OF(T, tile_m_hint); OF(T, tile_n_hint);
  OF(T, tile_k_hint); OF(T, reserved);
#undef T
  SZ(xvram_gemm_plan_info_v1);
#define T xvram_gemm_plan_info_v1
  OF(T, struct_size); OF(T, flags); OF(T, m); OF(T, n); OF(T, k); OF(T, tile_m); OF(T, tile_n);
  OF(T, tile_k); OF(T, maximum_working_set_bytes); OF(T, workspace_bytes); OF(T, tile_count);
  OF(T, effective_compute_mode); OF(T, uses_cublas_lt); OF(T, reserved);
#undef T
  SZ(xvram_api_v1);
#define T xvram_api_v1
  OF(T, struct_size); OF(T, abi_version); OF(T, status_name); OF(T, session_create);
  OF(T, session_get_error); OF(T, session_get_telemetry); OF(T, session_drain);
  OF(T, session_close); OF(T, session_release); OF(T, allocation_create);
  OF(T, allocation_get_info); OF(T, allocation_write); OF(T, allocation_read);
  OF(T, allocation_release); OF(T, prefetch_submit); OF(T, transaction_submit);
  OF(T, transaction_execute); OF(T, gemm_plan_create); OF(T, gemm_plan_get_info);
  OF(T, gemm_submit); OF(T, gemm_execute); OF(T, gemm_plan_release); OF(T, operation_poll);
  OF(T, operation_wait); OF(T, operation_cancel); OF(T, operation_get_error);
  OF(T, operation_release); OF(T, reserved);
#undef T
  EN(XVRAM_ALLOCATION_NORMAL); EN(XVRAM_ALLOCATION_HOT); EN(XVRAM_ALLOCATION_STREAMING);
  EN(XVRAM_ALLOCATION_FLAG_ZERO_INITIALIZE);
  EN(XVRAM_ACCESS_READ); EN(XVRAM_ACCESS_READ_WRITE); EN(XVRAM_ACCESS_WRITE_ONLY);
  EN(XVRAM_OPERATION_QUEUED); EN(XVRAM_OPERATION_RUNNING); EN(XVRAM_OPERATION_COMPLETED);
  EN(XVRAM_OPERATION_CANCELLED); EN(XVRAM_OPERATION_FAILED);
  EN(XVRAM_DATA_FP16); EN(XVRAM_DATA_BF16); EN(XVRAM_DATA_FP32); EN(XVRAM_DATA_FP64);
  EN(XVRAM_COMPUTE_AUTO); EN(XVRAM_COMPUTE_FP32_STRICT); EN(XVRAM_COMPUTE_FP32_TF32);
  EN(XVRAM_COMPUTE_FP64); EN(XVRAM_MATRIX_ROW_MAJOR); EN(XVRAM_MATRIX_COLUMN_MAJOR);
  EN(XVRAM_CUBLAS_SOURCE_UNKNOWN); EN(XVRAM_CUBLAS_SOURCE_SYSTEM);
  EN(XVRAM_CUBLAS_SOURCE_APP_LOCAL); EN(XVRAM_CUBLAS_SOURCE_EXPLICIT);
  {
    /* none of these structures has padding, so their initialisers' bytes are defined */
    xvram_allocation_desc_v1 ad = XVRAM_ALLOCATION_DESC_V1_INIT;
    xvram_operation_info_v1 oi = XVRAM_OPERATION_INFO_V1_INIT;
    xvram_matrix_v1 mx = XVRAM_MATRIX_V1_INIT;
    xvram_gemm_desc_v1 gd = XVRAM_GEMM_DESC_V1_INIT;
    xvram_gemm_plan_info_v1 pi = XVRAM_GEMM_PLAN_INFO_V1_INIT;
    bytes("xvram_allocation_desc_v1", &ad, sizeof ad);
    bytes("xvram_operation_info_v1", &oi, sizeof oi);
    bytes("xvram_matrix_v1", &mx, sizeof mx);
    bytes("xvram_gemm_desc_v1", &gd, sizeof gd);
    bytes("xvram_gemm_plan_info_v1", &pi, sizeof pi);
  }

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
