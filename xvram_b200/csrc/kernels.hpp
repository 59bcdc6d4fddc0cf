// kernels.hpp -- host-side launch interface of the library's CUDA kernels.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

namespace xvram {

enum class SgemmPath { automatic = 0, tma = 1, generic = 2 };

// C = alpha * op(A) * op(B) + beta * C on device-resident column-major FP32 data, on
// `stream`.  op 0 = N, 1 = T.  beta == 0 never reads C.  `automatic` selects the TMA
// kernel when the operands satisfy its alignment (16-byte bases, ld % 4 == 0).
cudaError_t sgemm_ffma(int op_a, int op_b, int m, int n, int k, float alpha, const float* a,
                       long long lda, const float* b, long long ldb, float beta, float* c,
                       long long ldc, cudaStream_t stream, SgemmPath path = SgemmPath::automatic);

// Workspace that sgemm_ffma_ws uses to canonicalise K-major operands (0 when op(A) = N
// and op(B) = T, which the kernel already reads in its fastest form).
uint64_t sgemm_workspace_bytes(int op_a, int op_b, int m, int n, int k);
// The C tile the TMA kernel uses for an M-/N-major (canonicalised) m x n problem on the
// current device: 192 x 192, 128 x 256 or 128 x 128.
void sgemm_tile_shape(int m, int n, int* tile_m, int* tile_n);

// sgemm_ffma with a workspace: when the workspace is at least sgemm_workspace_bytes and
// 256-byte aligned, K-major operands are transposed into it first and the M-major /
// N-major kernel runs; otherwise identical to sgemm_ffma.  Same result either way
// (the transposes move values, they do not round).
cudaError_t sgemm_ffma_ws(int op_a, int op_b, int m, int n, int k, float alpha, const float* a,
                          long long lda, const float* b, long long ldb, float beta, float* c,
                          long long ldc, void* workspace, uint64_t workspace_bytes,
                          cudaStream_t stream, SgemmPath path = SgemmPath::automatic);

bool sgemm_tma_eligible(int op_a, int op_b, const float* a, long long lda, const float* b,
                        long long ldb);

// One FP32 GEMM in two parts, so C's column blocks can be launched separately (and on
// different streams) after a single preparation of the operands:
//   sgemm_prepare  brings op(A) and op(B) into the form the kernel reads (the FFMA path's
//                  transposes into the workspace, the TF32 path's hi/lo splits);
//   sgemm_block    computes C's columns [n0, n0 + nj) from the prepared operands; c points
//                  at column n0.
// Each output is computed exactly as by one sgemm_ffma_ws / sgemm_tf32x3 call over all of
// C, provided n0 is a multiple of 256 (whole tile columns): block results are
// bit-identical to the unsplit call.  The prepared operands live in the workspace, so it
// must not be reused until every block has run.
struct SgemmPrepared {
  bool tf32 = false;
  // FFMA: the operands as the kernel reads them (canonical op N / op T when transposed)
  const float* a = nullptr;
  const float* b = nullptr;
  long long lda = 0, ldb = 0;
  int op_a = 0, op_b = 0;
  // TF32: K-major hi/lo parts, leading dimension kp
  const float *a_hi = nullptr, *a_lo = nullptr, *b_hi = nullptr, *b_lo = nullptr;
  long long kp = 0;
};
cudaError_t sgemm_prepare(bool tf32, int op_a, int op_b, int m, int n, int k, const float* a,
                          long long lda, const float* b, long long ldb, void* workspace,
                          uint64_t workspace_bytes, cudaStream_t stream, SgemmPrepared* out);
cudaError_t sgemm_block(const SgemmPrepared& p, int m, int n0, int nj, int k, float alpha,
                        float beta, float* c, long long ldc, cudaStream_t stream);

// dst (cols x rows, column-major, ldd) = src^T (src: rows x cols, column-major, lds), on
// `stream`.  Moves values only; used to bring K-major operands into the M/N-major form
// the kernel reads fastest.
cudaError_t transpose_f32_async(const float* src, long long lds, float* dst, long long ldd,
                                int rows, int cols, cudaStream_t stream);

// Three-term TF32 tensor-core GEMM (tcgen05 + TMEM), FP32-accurate within the path's
// tolerance but not bit-identical to the FFMA kernel.  Needs sgemm_tf32x3_workspace_bytes
// of 256-byte-aligned scratch for the split hi/lo operands; k must be positive.
uint64_t sgemm_tf32x3_workspace_bytes(int m, int n, int k);
cudaError_t sgemm_tf32x3(int op_a, int op_b, int m, int n, int k, float alpha, const float* a,
                         long long lda, const float* b, long long ldb, float beta, float* c,
                         long long ldc, void* workspace, uint64_t workspace_bytes,
                         cudaStream_t stream);
// The TF32 halves of sgemm_prepare / sgemm_block: the hi/lo splits into the workspace, and
// the kernel's K chunks over C's columns [n0, n0 + nj).
cudaError_t sgemm_tf32x3_prepare(int op_a, int op_b, int m, int n, int k, const float* a,
                                 long long lda, const float* b, long long ldb, void* workspace,
                                 uint64_t workspace_bytes, cudaStream_t stream,
                                 SgemmPrepared* out);
cudaError_t sgemm_tf32x3_block(const SgemmPrepared& p, int m, int n0, int nj, int k, float alpha,
                               float beta, float* c, long long ldc, cudaStream_t stream);

// GEMM of any supported element-type combination (types and arithmetic numbered as
// validate.hpp's DataType and ComputeKind): FP32 runs sgemm_ffma_ws or sgemm_tf32x3;
// FP16 / BF16 inputs are widened into the workspace and run on the FFMA kernel (strict
// FP32 arithmetic, C FP32 or rounded to the input type once at the end); FP64 runs the
// FP64 tensor-core kernel.  Needs gemm_typed_workspace_bytes of 256-byte-aligned scratch;
// pointers must be aligned to their element size (cudaErrorInvalidValue otherwise).
uint64_t gemm_typed_workspace_bytes(uint32_t ab_type, uint32_t c_type, int compute, int op_a,
                                    int op_b, int m, int n, int k);
cudaError_t gemm_typed(uint32_t ab_type, uint32_t c_type, int compute, int op_a, int op_b, int m,
                       int n, int k, double alpha, const void* a, long long lda, const void* b,
                       long long ldb, double beta, void* c, long long ldc, void* workspace,
                       uint64_t workspace_bytes, cudaStream_t stream);
// dst (rows x cols, ldd) = src converted between FP16 / BF16 and FP32 (round to nearest
// even when narrowing).
cudaError_t convert_matrix(uint32_t src_type, const void* src, long long lds, uint32_t dst_type,
                           void* dst, long long ldd, int rows, int cols, cudaStream_t stream);

// Reads (synchronising `stream`) and clears the device's sticky kernel error word.
cudaError_t read_and_clear_kernel_error(unsigned int* out, cudaStream_t stream);
cudaError_t read_and_clear_kernel_error_tc(unsigned int* out, cudaStream_t stream);

unsigned long long kernel_wait_limit_ns();

// Host-side probes used by bench.py for its roofline denominators.
cudaError_t ffma_peak_probe(int blocks, int iterations, float* sink, cudaStream_t stream,
                            bool packed = false);

} // namespace xvram
