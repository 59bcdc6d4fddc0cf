/*
 * xvram_b200.h -- native entry points of the B200 implementation.
 *
 * The drop-in boundary is xvram/cuda_compat.h.  The functions here expose the pieces
 * underneath it to callers that already manage device memory (the tile contraction on
 * raw device pointers) and to measurement and test harnesses (planner inspection,
 * validation, synthetic inputs, the FFMA peak probe).  All functions are plain C:
 * integer sizes, raw pointers, CUDA streams passed as uint64_t (0 = legacy default
 * stream).  Each notes the reference interface it stands in for, if any.
 */
#ifndef XVRAM_B200_H
#define XVRAM_B200_H

#include "xvram/xvram.h"

#if defined(__GNUC__) && defined(XVRAM_BUILDING_CUDA_COMPAT)
#define XVRAM_B200_API __attribute__((visibility("default")))
#else
#define XVRAM_B200_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define XVRAM_B200_VERSION_NUMBER 100 /* 0.1.0 */

/* Path selection for xvram_b200_sgemm_device. */
enum {
  XVRAM_B200_PATH_AUTO = 0,    /* TMA kernel when aligned, else the generic kernel */
  XVRAM_B200_PATH_TMA = 1,     /* TMA kernel or INVALID_ARGUMENT */
  XVRAM_B200_PATH_GENERIC = 2, /* generic kernel (any alignment) */
  /* Three-term TF32 on the tensor cores (tcgen05/TMEM): FP32-accurate within
   * max|err| / (K max|a| max|b|) <= 1e-6 but not bit-identical to the FFMA kernels.
   * Needs xvram_b200_sgemm_workspace_bytes(...) with this path, k > 0. */
  XVRAM_B200_PATH_TF32X3 = 3
};

/*
 * C = alpha * op(A) * op(B) + beta * C on device-resident column-major FP32 matrices,
 * enqueued on `stream` and not synchronised.  op 0 = N, 1 = T.  m, n, k >= 0 (k == 0
 * scales C by beta); beta == 0 does not read C.  Strict FP32: every multiply-add is an
 * FFMA.  K-major operands are transposed into stream-ordered scratch taken from a private
 * per-device memory pool (see xvram_b200_sgemm_device_ws to supply the scratch instead).  Stands in for the per-tile library call of the reference's executor
 * (src/gemm/executor.cpp:147-329 -> cublasLtMatmul, src/platform/cublas/cublas_api.cpp:751-918).
 */
XVRAM_B200_API xvram_status XVRAM_CALL xvram_b200_sgemm_device(
    uint32_t op_a, uint32_t op_b, int64_t m, int64_t n, int64_t k, float alpha, const float* a,
    int64_t lda, const float* b, int64_t ldb, float beta, float* c, int64_t ldc, uint64_t stream,
    uint32_t path);

/* Bytes of device workspace the K-major operand canonicalisation needs for this problem:
 * transposed copies of op(A) when op_a = T and of op(B) when op_b = N (0 for op_a = N,
 * op_b = T).  Pass op_a | XVRAM_B200_WORKSPACE_TF32X3 for the tensor-core path's split
 * operands instead.  No reference counterpart. */
#define XVRAM_B200_WORKSPACE_TF32X3 0x100u
XVRAM_B200_API uint64_t XVRAM_CALL xvram_b200_sgemm_workspace_bytes(uint32_t op_a, uint32_t op_b,
                                                                    int64_t m, int64_t n,
                                                                    int64_t k);

/* The C tile (rows x columns) the TMA-fed FFMA kernel uses for an m x n problem whose
 * operands are M-major / N-major (as they are after the K-major ones are transposed into
 * workspace) on the current device: 192 x 192 (12 warps), 128 x 256 or 128 x 128 (8 warps),
 * whichever takes fewer tile-waves on the device's SM count.  Every tiling computes each
 * output as the same FFMA chain in k order, so results do not depend on it.
 * INVALID_ARGUMENT for m or n outside [1, INT32_MAX] or a null output.  No reference
 * counterpart. */
XVRAM_B200_API xvram_status XVRAM_CALL xvram_b200_sgemm_tile_shape(int64_t m, int64_t n,
                                                                 int32_t* tile_m,
                                                                 int32_t* tile_n);

/*
 * xvram_b200_sgemm_device with caller-provided device workspace (256-byte aligned).  With
 * at least xvram_b200_sgemm_workspace_bytes, K-major operands are transposed into it and
 * the faster M-major/N-major kernel runs; with less, the call behaves exactly like
 * xvram_b200_sgemm_device without allocating.  Results are bit-identical either way.
 * Calls that share one workspace must be ordered on the device (same stream or events).
 */
XVRAM_B200_API xvram_status XVRAM_CALL xvram_b200_sgemm_device_ws(
    uint32_t op_a, uint32_t op_b, int64_t m, int64_t n, int64_t k, float alpha, const float* a,
    int64_t lda, const float* b, int64_t ldb, float beta, float* c, int64_t ldc, void* workspace,
    uint64_t workspace_bytes, uint64_t stream, uint32_t path);

/* Size of the fixed scratch array behind xvram_b200_sgemm_device_noalloc (32 MiB). */
#define XVRAM_B200_NOALLOC_SCRATCH_BYTES (32u << 20)

/*
 * xvram_b200_sgemm_device for callers that must not allocate device memory.  No
 * counterpart in the reference.
 *
 * Who needs it: an application that has already handed the GPU's memory to its own
 * allocator (a fixed arena in a serving process or framework), code running inside such
 * an allocator's callbacks, and plugins whose host only lets them use memory it passes in.
 * For them a cudaMalloc -- or a pool allocation, which xvram_b200_sgemm_device makes for
 * its scratch -- fails or re-enters their allocator.
 *
 * What it does instead: the scratch for transposing K-major operands comes from one
 * array compiled into the library, XVRAM_B200_NOALLOC_SCRATCH_BYTES large, which sits in
 * device memory on every GPU where the library's device code is loaded until the process
 * exits.  The call makes no cudaMalloc, cudaFree or other allocating call.  The caller
 * still provides A, B and C.  Arguments and results are those of xvram_b200_sgemm_device
 * (bit-identical results), except that path XVRAM_B200_PATH_TF32X3 is not offered here
 * and returns XVRAM_STATUS_INVALID_ARGUMENT; the device is the caller's current device.
 *
 * Limits: a problem that needs more scratch than the array
 * (xvram_b200_sgemm_workspace_bytes > XVRAM_B200_NOALLOC_SCRATCH_BYTES, for example a TN
 * product with (M + N) x K above 8 Mi floats) is refused with
 * XVRAM_STATUS_BUDGET_PRESSURE before anything is launched.  Every call uses the same array
 * and it keeps whatever the last call left there; each call overwrites all the scratch it
 * reads, so nothing needs clearing, but calls that overlap on the GPU (different streams
 * without ordering, or different host threads) race on it and must be serialised by the
 * caller.
 *
 * First call on a device: it looks up the array's device address (cudaGetSymbolAddress),
 * which loads this library's device code, the array included, on that device.  Under
 * CUDA's lazy module loading (the default) each kernel's code is also loaded at its first
 * launch.  Those loads need device memory, so make the first call on each device -- with
 * the shapes and operations you will use, since an empty problem returns before loading
 * anything -- before your allocator takes the GPU's memory (or start the process with
 * CUDA_MODULE_LOADING=EAGER); a load that finds no room fails the call with
 * XVRAM_STATUS_DEVICE_OUT_OF_MEMORY.  Make that first call before any stream capture, and
 * do not reset the device (cudaDeviceReset) afterwards: the address is kept for the life
 * of the process.
 */
XVRAM_B200_API xvram_status XVRAM_CALL xvram_b200_sgemm_device_noalloc(
    uint32_t op_a, uint32_t op_b, int64_t m, int64_t n, int64_t k, float alpha, const float* a,
    int64_t lda, const float* b, int64_t ldb, float beta, float* c, int64_t ldc, uint64_t stream,
    uint32_t path);

/* Synchronises `stream`, then returns and clears the device's sticky kernel error word
 * (nonzero: a pipeline wait inside a kernel ran out of time and the kernel returned
 * without finishing).  No reference counterpart (the reference has no kernels). */
XVRAM_B200_API xvram_status XVRAM_CALL xvram_b200_kernel_status(uint64_t stream,
                                                                uint32_t* word);

/* dst[i] = uniform[-1, 1) draw (seed, first_index + i) on `threads` host threads
 * (0 = all).  Counter-based: any element can be recomputed independently. */
XVRAM_B200_API void XVRAM_CALL xvram_b200_fill_uniform(float* dst, uint64_t count,
                                                       uint64_t seed, uint64_t first_index,
                                                       int32_t threads);

/* Panel plan summary for an out-of-core problem under a device budget.  Stands in for
 * the reference's gemm::make_plan inspection (src/gemm/planner.cpp:1005-1153). */
typedef struct xvram_b200_plan_info_v1 {
  uint32_t struct_size;
  uint32_t status; /* 0 ok, 1 invalid, 2 budget too small */
  int64_t block_m, block_n, panel_k;
  int32_t n_outer; /* 1: n blocks outer loop */
  int32_t panel_slots;
  int32_t c_slots;
  int32_t reserved0;
  uint64_t slot_bytes, c_slot_bytes;
  uint64_t steps, panel_loads, panel_hits, panel_evictions;
  uint64_t h2d_bytes, d2h_bytes;
  double est_seconds;
} xvram_b200_plan_info_v1;

XVRAM_B200_API xvram_status XVRAM_CALL xvram_b200_plan_panels(
    uint32_t op_a, uint32_t op_b, int64_t m, int64_t n, int64_t k, int32_t beta_nonzero,
    uint64_t budget_bytes, uint64_t quantum_bytes, double flops_per_s, double h2d_bytes_per_s,
    double d2h_bytes_per_s, int64_t force_mb, int64_t force_nb, int64_t force_kb,
    xvram_b200_plan_info_v1* out);

/* Writes the plan's step list: for step i, out[5*i .. 5*i+4] = bm, bn, bk, slot_a, slot_b.
 * `capacity` is the number of steps `out` can hold; returns INVALID_ARGUMENT if smaller. */
XVRAM_B200_API xvram_status XVRAM_CALL xvram_b200_plan_steps(
    uint32_t op_a, uint32_t op_b, int64_t m, int64_t n, int64_t k, int32_t beta_nonzero,
    uint64_t budget_bytes, uint64_t quantum_bytes, int64_t force_mb, int64_t force_nb,
    int64_t force_kb, int32_t* out, uint64_t capacity);

/* Column-major FP32 GEMM problem validation.  Returns the problem-error enumerator of the
 * reference's gemm::validate_problem (src/gemm/planner.cpp:785-859) and its operand
 * letter.  Arrays are indexed A, B, C. */
XVRAM_B200_API int32_t XVRAM_CALL xvram_b200_validate_gemm(
    uint64_t m, uint64_t n, uint64_t k, uint32_t op_a, uint32_t op_b,
    const uint64_t allocation_ids[3], const uint64_t allocation_bytes[3],
    const uint64_t offsets[3], const uint64_t rows[3], const uint64_t columns[3],
    const uint64_t lds[3], char* operand);

/* The reference benches' report digests, for reports in their formats.  Hex form of a
 * state: 16 hex digits of state[1], then 16 of state[0].
 *   GEMM bench (src/gemm_bench/executor.cpp:42-65): bytes with their absolute offsets.
 *   Compat bench (src/compat_bench/pattern.cpp, pattern.hpp:29-30): FP32 values. */
#define XVRAM_B200_BENCH_DIGEST_INIT {UINT64_C(1469598103934665603), \
                                      UINT64_C(1099511628211) ^ UINT64_C(0x9E3779B97F4A7C15)}
#define XVRAM_B200_COMPAT_DIGEST_INIT {UINT64_C(1469598103934665603), UINT64_C(0x9e3779b97f4a7c15)}
XVRAM_B200_API void XVRAM_CALL xvram_b200_digest_bench(const void* data, uint64_t len,
                                                       uint64_t absolute_offset, uint64_t state[2]);
XVRAM_B200_API void XVRAM_CALL xvram_b200_digest_compat(const float* values, uint64_t count,
                                                        uint64_t state[2]);

/* What the library's device layer reports for one device (the GEMM bench report's device
 * and build sections).  struct_size = sizeof before the call. */
typedef struct xvram_b200_device_info_v1 {
  uint32_t struct_size;
  int32_t ordinal;
  int32_t device_count;
  char name[128];
  uint64_t total_bytes;
  uint64_t free_bytes;
  int32_t sm_count;
  int32_t compute_capability_major;
  int32_t compute_capability_minor;
  int32_t driver_version;           /* cudaDriverGetVersion */
  uint64_t vmm_granularity;         /* recommended physical allocation granularity */
  int32_t runtime_headers_version;  /* CUDART_VERSION the library was built with */
  int32_t reserved0;
} xvram_b200_device_info_v1;

XVRAM_B200_API xvram_status XVRAM_CALL xvram_b200_device_query(int32_t ordinal,
                                                               xvram_b200_device_info_v1* out);

/* xvram_b200_validate_gemm with element types (A, B, C; XVRAM_DATA_* numbering) and an
 * arithmetic (0 strict FP32, 1 TF32, 2 FP64: the reference's gemm::ComputeMode,
 * src/gemm/planner.hpp:25-36), following the whole of gemm::validate_problem
 * (src/gemm/planner.cpp:785-859) including its type rule. */
XVRAM_B200_API int32_t XVRAM_CALL xvram_b200_validate_gemm_typed(
    uint64_t m, uint64_t n, uint64_t k, uint32_t op_a, uint32_t op_b,
    const uint64_t allocation_ids[3], const uint64_t allocation_bytes[3],
    const uint64_t offsets[3], const uint64_t rows[3], const uint64_t columns[3],
    const uint64_t lds[3], const uint32_t data_types[3], int32_t compute, char* operand);

/* Device GEMM of the reference's other type combinations (the per-tile contraction the
 * reference hands to cuBLASLt / cublasDgemm, src/platform/cublas/cublas_api.cpp:634-918):
 * FP16 or BF16 A and B with strict FP32 arithmetic and C of the same type or FP32, FP32
 * (strict or three-term TF32), FP64.  Column-major device pointers aligned to their
 * element size; alpha and beta in FP64 for FP64 arithmetic, else rounded to FP32.  The
 * workspace (256-byte aligned, xvram_b200_gemm_typed_workspace_bytes) holds widened or
 * canonicalised operands.  INVALID_ARGUMENT for an unsupported combination. */
XVRAM_B200_API uint64_t XVRAM_CALL xvram_b200_gemm_typed_workspace_bytes(
    uint32_t ab_type, uint32_t c_type, int32_t compute, uint32_t op_a, uint32_t op_b, int64_t m,
    int64_t n, int64_t k);
XVRAM_B200_API xvram_status XVRAM_CALL xvram_b200_gemm_device_typed(
    uint32_t ab_type, uint32_t c_type, int32_t compute, uint32_t op_a, uint32_t op_b, int64_t m,
    int64_t n, int64_t k, double alpha, const void* a, int64_t lda, const void* b, int64_t ldb,
    double beta, void* c, int64_t ldc, void* workspace, uint64_t workspace_bytes,
    uint64_t stream);

/* Launches `blocks` x 256 threads of dependent FFMA chains (`iterations` x 512 FFMA per
 * thread) on `stream`; the measured FP32 pipe peak is 2 * blocks * 256 * iterations * 512
 * FLOP over the launch time.  `sink` (device, >= 1 float) defeats dead-code elimination. */
XVRAM_B200_API xvram_status XVRAM_CALL xvram_b200_ffma_probe(int32_t blocks, int32_t iterations,
                                                             float* sink, uint64_t stream);

/* The same probe with packed FP32 FMAs (two per lane per instruction, 8 float2 chains per
 * thread, the same 512 FMAs per thread per iteration, so the same FLOP formula). */
XVRAM_B200_API xvram_status XVRAM_CALL xvram_b200_ffma2_probe(int32_t blocks, int32_t iterations,
                                                              float* sink, uint64_t stream);

/*
 * Multi-GPU partitioned SGEMM (no reference counterpart: the reference is single-GPU,
 * src/cuda_compat/adapter.cpp:595-600).  One process or thread per GPU:
 *   rank 0: xvram_b200_shard_unique_id(id, 128) and share the 128 bytes with the others;
 *   every rank, with its GPU current: xvram_b200_shard_group_create(id, 128, rank, world, &g);
 *   every rank, collectively: xvram_b200_sgemm_sharded(g, ...) on its own rows.
 * Group creation waits at most 120 s for the other ranks (UNAVAILABLE after that).
 */
XVRAM_B200_API xvram_status XVRAM_CALL xvram_b200_shard_unique_id(void* out, uint64_t bytes);
XVRAM_B200_API xvram_status XVRAM_CALL xvram_b200_shard_group_create(const void* unique_id,
                                                                   uint64_t bytes, int32_t rank,
                                                                   int32_t world,
                                                                   uint64_t* out_group);
XVRAM_B200_API xvram_status XVRAM_CALL xvram_b200_shard_group_destroy(uint64_t group);

/*
 * Collectives supplied by the caller, for a group that should not (or cannot) use NCCL:
 * an application with its own communicator, or a host-memory test device.  Both functions
 * are called by every rank in the same order and must act as the collective of that name
 * over the group's ranks, enqueued on `stream` (the group's native collective stream, a
 * cudaStream_t of the group's device) or completed before returning:
 *   all_reduce_max_u64: buffer[0..count) = elementwise maximum over the ranks, in place;
 *   all_gather_f32:     recv[q count .. (q+1) count) = rank q's send, for every q; send
 *                       may be recv + rank * count (in place).
 * Pointers are device addresses of the group's device.  A non-SUCCESS return fails the
 * call that issued it and leaves the group unusable (POISONED).
 */
typedef struct xvram_b200_shard_collectives_v1 {
  uint32_t struct_size; /* sizeof(xvram_b200_shard_collectives_v1) */
  uint32_t reserved0;
  void* context; /* passed back as the first argument */
  xvram_status(XVRAM_CALL* all_reduce_max_u64)(void* context, uint64_t* buffer, uint64_t count,
                                               uint64_t stream);
  xvram_status(XVRAM_CALL* all_gather_f32)(void* context, const float* send, float* recv,
                                           uint64_t count, uint64_t stream);
} xvram_b200_shard_collectives_v1;

/* Creates this rank's group with the caller's collectives instead of NCCL, on the calling
 * thread's current device.  No reference counterpart. */
XVRAM_B200_API xvram_status XVRAM_CALL xvram_b200_shard_group_create_custom(
    const xvram_b200_shard_collectives_v1* ops, int32_t rank, int32_t world, uint64_t* out_group);

/* The rows of an m-row C that `rank` of `world` owns in the partition this library uses:
 * whole 128-row tiles dealt out as evenly as possible (rank r gets tiles
 * [r T / world, (r + 1) T / world) of T = ceil(m / 128)), the last tile cut at m.  Ranks
 * past the tile count get *row_count = 0.  Pass those rows of A and C to
 * xvram_b200_sgemm_sharded.  No reference counterpart. */
XVRAM_B200_API xvram_status XVRAM_CALL xvram_b200_shard_rows(int64_t m, int32_t world,
                                                           int32_t rank, int64_t* row_begin,
                                                           int64_t* row_count);

/* The plan the group's ranks agreed on for the last xvram_b200_sgemm_sharded call, and
 * what this rank moved.  Every rank of a group reports the same fields down to
 * device_bytes; rank, h2d_bytes and d2h_bytes are this rank's. */
typedef struct xvram_b200_shard_plan_v1 {
  uint32_t struct_size; /* set by the caller to sizeof(xvram_b200_shard_plan_v1) */
  int32_t world;
  uint64_t m_max;         /* largest m_local over the ranks */
  uint64_t avail_min;     /* smallest device memory the ranks offered (bytes) */
  uint64_t row_groups;    /* row groups of A kept resident in turn */
  uint64_t group_rows;    /* rows per group (a multiple of 128) */
  uint64_t block_n;       /* C column block width */
  uint64_t panel_k;       /* K panel depth of A's first arrival */
  uint64_t b_slice_cols;  /* op(B) = N: block columns each rank copies (0 for op T) */
  uint64_t b_slice_k;     /* op(B) = T: k rows each rank copies (0 for op N) */
  uint64_t slice_elems;   /* floats each rank contributes to one B all-gather */
  uint64_t device_bytes;  /* device memory the plan's buffers take on each rank */
  int32_t rank;
  uint32_t reserved0;
  uint64_t gathers;       /* B all-gathers issued */
  uint64_t h2d_bytes;     /* host -> device bytes this rank copied */
  uint64_t d2h_bytes;     /* device -> host bytes this rank copied */
} xvram_b200_shard_plan_v1;

XVRAM_B200_API xvram_status XVRAM_CALL xvram_b200_shard_last_plan(uint64_t group,
                                                                xvram_b200_shard_plan_v1* out);

/* All-gather of row blocks, collectively on every rank of the group, enqueued on `stream`
 * (a cudaStream_t of the group's device): rank q's block (rows x cols, column-major,
 * ld_block) becomes rows [q rows, (q + 1) rows) of every rank's dst (world rows x cols,
 * ld_dst).  `staging` is device scratch of world x rows x cols floats.  This is the
 * activation exchange of a Linear layer split by output features (each rank computes its
 * rows of Y = W X; the next layer needs all of them).  One ncclAllGather over NVLink plus
 * device copies; POISONED after the group was aborted. */
XVRAM_B200_API xvram_status XVRAM_CALL xvram_b200_shard_allgather_rows(
    uint64_t group, const float* block, int64_t rows, int64_t cols, int64_t ld_block, float* dst,
    int64_t ld_dst, void* staging, uint64_t staging_bytes, uint64_t stream);

/*
 * C_local = alpha * op(A_local) * op(B) + beta * C_local for this rank's m_local rows of C,
 * all operands in (preferably page-locked) host memory, column-major.  A_local holds this
 * rank's rows of op(A) (m_local x k for op N, k x m_local for op T); B is the whole
 * matrix on every rank, but each rank copies only a 1/world slice of each block of B to
 * its GPU and the slices are all-gathered over NVLink.  A_local is kept resident in HBM
 * (in row groups when it does not fit next to the other buffers), arriving in K panels of
 * `panel_k` (0 = 1024) so the first kernel starts after the first panel; C is processed in
 * column blocks whose copies in and out overlap the neighbouring blocks' kernels.  Ranks
 * may pass different m_local (0 included); the call agrees on one plan first.  Blocking;
 * every wait is bounded (TIMEOUT after 60 s without progress, after which the group is
 * unusable and returns POISONED).  Tuning (environment, read per call; the same on every
 * rank): XVRAM_B200_SHARD_BLOCK_N = C block width (default 576),
 * XVRAM_B200_SHARD_BUDGET_BYTES = cap on the device memory the call may use.
 */
XVRAM_B200_API xvram_status XVRAM_CALL xvram_b200_sgemm_sharded(
    uint64_t group, uint32_t op_a, uint32_t op_b, int64_t m_local, int64_t n, int64_t k,
    float alpha, const float* a, int64_t lda, const float* b, int64_t ldb, float beta, float* c,
    int64_t ldc, int64_t panel_k);

/*
 * Y = act(Y + bias) over a column-major rows x cols FP32 block on the device (bias: rows
 * floats, or 0 for none), enqueued on `stream` (a cudaStream_t; 0 = the legacy default
 * stream).  No reference counterpart: the reference's tiled GEMM takes no bias and its
 * torch route rejects biased linear layers (reference python/xvram/torch_native.py:
 * 1913-1921).  Meant for SDK transaction callbacks, which receive the resident addresses
 * and the stream (xvram_transaction_context_v1), so a caller can run Linear + bias + ReLU
 * as gemm_execute followed by transaction_execute on the output.
 */
enum { XVRAM_B200_ACTIVATION_NONE = 0, XVRAM_B200_ACTIVATION_RELU = 1 };
XVRAM_B200_API xvram_status XVRAM_CALL xvram_b200_bias_activation(uint64_t y, int64_t ldy,
                                                                 int64_t rows, int64_t cols,
                                                                 uint64_t bias,
                                                                 uint32_t activation,
                                                                 uint64_t stream);

/* Extra state of the compat adapter's runtime (not in the reference telemetry). */
typedef struct xvram_b200_runtime_info_v1 {
  uint32_t struct_size;
  uint32_t reserved0;
  uint64_t frame_bytes;
  uint64_t frame_capacity;
  uint64_t gemm_in_place;
  uint64_t gemm_streamed;
  uint64_t last_block_m, last_block_n, last_panel_k;
  uint64_t last_steps;
  uint64_t last_panel_slots;
  double last_gemm_ms;
  /* blas_sgemm calls that returned before their kernels finished (the default; the
     environment variable XVRAM_B200_SYNC_GEMM=1 waits for them), and the C column blocks
     those kernels ran as. */
  uint64_t gemm_deferred;
  uint64_t gemm_column_blocks;
  /* Streamed GEMMs: panel loads into a slot that held another panel (the slot's frames stay
     mapped, so the reference-format counters -- evictions and handle reuses, which count
     VMM unmaps and remaps -- do not include them). */
  uint64_t panel_slot_refills;
} xvram_b200_runtime_info_v1;

XVRAM_B200_API xvram_status XVRAM_CALL
xvram_b200_compat_runtime_info(xvram_b200_runtime_info_v1* out);

#ifdef __cplusplus
}
#endif
#endif /* XVRAM_B200_H */
