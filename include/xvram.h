/*
 * xvram.h -- shared v1 ABI types of the xVRAM C interfaces (B200 implementation).
 *
 * Binary-compatible with the reference's include/xvram/xvram.h: every structure,
 * enumerator and macro below has the same name, value, field order and size as the
 * reference declares, so callers compiled against the reference headers link
 * against this library unchanged.  tests/test_abi_layout.py pins sizeof/offsetof of
 * every field against tests/golden/abi_layout.json, which was produced from the
 * reference headers.
 *
 *   reference include/xvram/xvram.h:7-9    64-bit only
 *   reference include/xvram/xvram.h:11-26  XVRAM_CALL / XVRAM_API
 *   reference include/xvram/xvram.h:44-75  ABI version, handles, status codes
 *   reference include/xvram/xvram.h:77-109 native error domains and error record
 *   reference include/xvram/xvram.h:111-150 session configuration and its defaults
 *   reference include/xvram/xvram.h:314-318 matrix operation constants
 *   reference include/xvram/xvram.h:411-457 session telemetry
 *
 * Convention: every public structure begins with struct_size, which the caller
 * sets to sizeof() of the structure it was compiled against; the library rejects
 * anything smaller than the v1 prefix.  Reserved fields must be zero.
 */
#ifndef XVRAM_XVRAM_H
#define XVRAM_XVRAM_H

#include <stddef.h>
#include <stdint.h>

#if UINTPTR_MAX != UINT64_MAX
#error "the xVRAM v1 ABI is defined for 64-bit targets only"
#endif

#if defined(_WIN32)
#define XVRAM_CALL __cdecl
#else
#define XVRAM_CALL
#endif
#if defined(__GNUC__) && defined(XVRAM_BUILDING_LIBRARY)
#define XVRAM_API __attribute__((visibility("default")))
#else
#define XVRAM_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define XVRAM_ABI_VERSION_1 UINT32_C(1)
#define XVRAM_ABI_VERSION_CURRENT XVRAM_ABI_VERSION_1
#define XVRAM_TIMEOUT_INFINITE UINT64_MAX

/* Status codes returned by every entry point. */
typedef uint32_t xvram_status;
enum {
  XVRAM_STATUS_SUCCESS = 0,
  XVRAM_STATUS_INVALID_ARGUMENT = 1,
  XVRAM_STATUS_INCOMPATIBLE_ABI = 2,
  XVRAM_STATUS_UNSUPPORTED = 3,
  XVRAM_STATUS_UNAVAILABLE = 4,
  XVRAM_STATUS_HOST_OUT_OF_MEMORY = 5,
  XVRAM_STATUS_DEVICE_OUT_OF_MEMORY = 6,
  XVRAM_STATUS_BUDGET_PRESSURE = 7,
  XVRAM_STATUS_BUSY = 8,
  XVRAM_STATUS_NOT_READY = 9,
  XVRAM_STATUS_TIMEOUT = 10,
  XVRAM_STATUS_CORRUPTION = 11,
  XVRAM_STATUS_CALLBACK_FAILED = 12,
  XVRAM_STATUS_CUDA_ERROR = 13,
  XVRAM_STATUS_CUBLAS_ERROR = 14,
  XVRAM_STATUS_POISONED = 15,
  XVRAM_STATUS_CLEANUP_FAILED = 16,
  XVRAM_STATUS_CLOSED = 17,
  XVRAM_STATUS_CANCELLED = 18,
  XVRAM_STATUS_INTERNAL = 19
};

/* Which native layer produced native_code in an error record. */
typedef uint32_t xvram_native_error_domain;
enum {
  XVRAM_NATIVE_ERROR_NONE = 0,
  XVRAM_NATIVE_ERROR_CUDA = 1,
  XVRAM_NATIVE_ERROR_CUBLAS = 2,
  XVRAM_NATIVE_ERROR_PLATFORM = 3,
  XVRAM_NATIVE_ERROR_CALLBACK = 4,
  XVRAM_NATIVE_ERROR_INTERNAL = 5
};

/* Detail of the most recent failure: where it happened and what the native layer said.
 * The character fields are NUL-terminated and truncated to fit. */
typedef struct xvram_error_info_v1 {
  uint32_t struct_size;
  xvram_status status;
  xvram_native_error_domain native_domain;
  uint32_t reserved0;
  int64_t native_code;
  char stage[32];
  char operation[64];
  char native_name[64];
  char message[256];
} xvram_error_info_v1;

#define XVRAM_ERROR_INFO_V1_INIT                                                                 \
  {(uint32_t)sizeof(xvram_error_info_v1), XVRAM_STATUS_SUCCESS, XVRAM_NATIVE_ERROR_NONE, 0U,     \
   INT64_C(0), {0}, {0}, {0}, {0}}

typedef uint32_t xvram_context_mode;
enum { XVRAM_CONTEXT_ISOLATED = 0, XVRAM_CONTEXT_ATTACH_CURRENT = 1 };

/* Victim selection of the device frame cache.  CLOCK and LRU are accepted for
 * compatibility; the B200 scheduler additionally knows each frame's next use from
 * the panel plan and prefers the frame used furthest in the future. */
typedef uint32_t xvram_cache_policy;
enum { XVRAM_CACHE_POLICY_CLOCK = 0, XVRAM_CACHE_POLICY_LRU = 1 };

/* Session configuration.  cache_target_bytes is the device memory budget for operand
 * frames (0 = automatic: device free memory minus device_headroom_bytes);
 * max_transaction_ms 0 = automatic. */
typedef struct xvram_session_config_v1 {
  uint32_t struct_size;
  uint32_t flags;
  int32_t device_ordinal;
  xvram_context_mode context_mode;
  uint64_t chunk_size_bytes;
  uint64_t cache_target_bytes;
  uint64_t device_headroom_bytes;
  uint64_t workspace_cap_bytes;
  uint64_t budget_poll_ms;
  uint64_t max_transaction_ms;
  uint32_t staging_slots;
  xvram_cache_policy cache_policy;
  uint32_t prefetch_distance;
  uint32_t reserved0;
  uint64_t reserved[4];
} xvram_session_config_v1;

/* Defaults: 64 MiB chunks, automatic target, 512 MiB headroom, 4 MiB workspace,
 * 100 ms budget poll, 4 staging slots, CLOCK, prefetch distance 2. */
#define XVRAM_SESSION_CONFIG_V1_INIT                                                             \
  {(uint32_t)sizeof(xvram_session_config_v1), 0U, 0, XVRAM_CONTEXT_ISOLATED,                     \
   UINT64_C(67108864), UINT64_C(0), UINT64_C(536870912), UINT64_C(4194304), UINT64_C(100),       \
   UINT64_C(0), 4U, XVRAM_CACHE_POLICY_CLOCK, 2U, 0U, {0, 0, 0, 0}}

/* Operation applied to a stored column-major matrix before the product. */
typedef uint32_t xvram_matrix_operation;
enum { XVRAM_MATRIX_OP_N = 0, XVRAM_MATRIX_OP_T = 1 };

/* Cumulative counters of the residency layer.  The B200 implementation fills the
 * fields it has an equivalent for and leaves the rest zero: cublas_* (no cuBLAS on
 * the path) and wddm_* (Windows only). */
typedef struct xvram_session_telemetry_v1 {
  uint32_t struct_size;
  uint32_t flags;
  uint64_t cache_target_bytes;
  uint64_t cache_target_minimum_bytes;
  uint64_t cache_target_maximum_bytes;
  uint64_t resident_bytes;
  uint64_t resident_bytes_peak;
  uint64_t workspace_bytes;
  uint64_t bytes_h2d;
  uint64_t bytes_d2h;
  uint64_t cache_hits;
  uint64_t cache_misses;
  uint64_t clean_evictions;
  uint64_t dirty_evictions;
  uint64_t writebacks_completed;
  uint64_t mappings;
  uint64_t unmaps;
  uint64_t set_access_calls;
  uint64_t handle_reuses;
  uint64_t unsafe_remaps;
  uint64_t unsafe_transitions;
  uint64_t budget_shrinks;
  uint64_t budget_grows;
  uint32_t cuda_driver_version;
  uint32_t cublas_version;
  uint32_t cublas_lt_available;
  uint32_t poisoned;
  uint64_t physical_handles_created;
  uint64_t physical_handles_released;
  uint64_t event_boundaries;
  uint64_t pinned_staging_bytes;
  uint64_t transactions_completed;
  uint64_t algorithm_selections;
  uint64_t algorithm_cache_hits;
  double last_transaction_ms;
  uint64_t budget_sample_count;
  uint64_t cuda_free_bytes_minimum;
  uint64_t cuda_free_bytes_end;
  uint32_t cublas_lt_version;
  uint32_t cublas_library_source;
  uint64_t wddm_available_bytes_minimum;
  uint64_t wddm_available_bytes_end;
  uint32_t wddm_budget_observed;
  uint32_t watchdog_rejections;
  uint64_t target_oom_retries;
} xvram_session_telemetry_v1;

enum {
  XVRAM_TELEMETRY_STABLE_VIRTUAL_ADDRESSES = 1U << 0U,
  XVRAM_TELEMETRY_NO_PHYSICAL_ALIASES = 1U << 1U
};

#ifdef __cplusplus
} /* extern "C" */
#endif

#endif /* XVRAM_XVRAM_H */
