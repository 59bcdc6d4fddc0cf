// gemm_typed.cu -- GEMMs of the reference's other element types, and type conversion.
//
// The reference accepts, besides FP32 (reference src/gemm/planner.cpp:819-842):
//   * FP16 / BF16 A and B with strict FP32 arithmetic and an FP16 / BF16 (same type) or
//     FP32 C -- cuBLASLt with CUBLAS_COMPUTE_32F_PEDANTIC in the reference
//     (src/platform/cublas/cublas_api.cpp:751-918);
//   * FP64 A, B and C with FP64 arithmetic (cublasDgemm, cublas_api.cpp:673-676).
//
// FP16 / BF16: every FP16 or BF16 value is exactly representable in FP32 and the product
// of two of them is exact in FP32 (at most 11 x 11 significant bits), so "strict FP32
// arithmetic on half inputs" is exactly the FP32 FFMA kernel run on the widened values.
// The operands are widened once into workspace, in the M-major / N-major layout the FFMA
// kernel reads fastest (one pass that also transposes K-major operands); a half C is
// widened to an FP32 copy (only when beta != 0), the kernel updates that copy, and it is
// rounded to the C type once at the end (round to nearest even).
//
// FP64: the 5th-generation tensor cores (tcgen05) have no FP64 form, so the FP64 kernel
// uses the FP64 MMA of the warp-level tensor path, mma.sync m16n8k8 .f64 (each
// multiply-add an FP64 operation, no reduced precision), fed by a 3-stage cp.async ring:
//   * 128 x 128 C tile per CTA, 8 warps as 2 (M) x 4 (N), each warp 64 x 32 = 4 x 4
//     blocks of 16 x 8, accumulators in registers (64 doubles per thread);
//   * K in stages of 32; stage tiles [32 k][128 + 8] doubles -- the 8-double pad puts
//     consecutive k rows 16 banks apart, so a fragment load (4 k rows x 8 consecutive
//     doubles across the warp) takes the minimum two wavefronts;
//   * operands canonicalised first, as for FP32: op(A) M-major and op(B) N-major
//     (K-major operands are transposed into workspace); 16-byte cp.async (8-byte when a
//     base or leading dimension is not 16-byte aligned) with zero fill covers ragged
//     edges.
// There are no spin-waits in these kernels (cp.async groups and block barriers only).
#include "kernels.hpp"
#include "validate.hpp"

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <type_traits>

namespace xvram {
namespace {

// ------------------------------------------------------------------ conversions
template <class T> struct Elem;
template <> struct Elem<float> {
  __device__ static float to_f(float x) { return x; }
  __device__ static float from_f(float x) { return x; }
};
template <> struct Elem<__half> {
  __device__ static float to_f(__half x) { return __half2float(x); }
  __device__ static __half from_f(float x) { return __float2half_rn(x); }
};
template <> struct Elem<__nv_bfloat16> {
  __device__ static float to_f(__nv_bfloat16 x) { return __bfloat162float(x); }
  __device__ static __nv_bfloat16 from_f(float x) { return __float2bfloat16_rn(x); }
};

template <class S, class D> __device__ __forceinline__ D convert_elem(S x) {
  if constexpr (std::is_same_v<S, D>)
    return x;
  else
    return Elem<D>::from_f(Elem<S>::to_f(x));
}

// dst = convert(src) (TRANSPOSE false: dst is rows x cols) or convert(src)^T (TRANSPOSE
// true: dst is cols x rows); src is rows x cols column-major with leading dimension lds.
// 32 x 32 tiles through shared memory, so both the reads and the writes are coalesced.
template <class S, class D, bool TRANSPOSE>
__global__ void __launch_bounds__(256)
    relayout_kernel(const S* __restrict__ src, long long lds, D* __restrict__ dst, long long ldd,
                    int rows, int cols, int tiles_r) {
  __shared__ D tile[32][33];
  const int tr = blockIdx.x % tiles_r;
  const int tc = blockIdx.x / tiles_r;
  const int r0 = tr * 32, c0 = tc * 32;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  if constexpr (!TRANSPOSE) {
#pragma unroll
    for (int j = ty; j < 32; j += 8) {
      const int r = r0 + tx, c = c0 + j;
      if (r < rows && c < cols)
        dst[r + static_cast<long long>(c) * ldd] =
            convert_elem<S, D>(src[r + static_cast<long long>(c) * lds]);
    }
  } else {
#pragma unroll
    for (int j = ty; j < 32; j += 8) {
      const int r = r0 + tx, c = c0 + j;
      if (r < rows && c < cols)
        tile[j][tx] = convert_elem<S, D>(src[r + static_cast<long long>(c) * lds]);
    }
    __syncthreads();
#pragma unroll
    for (int j = ty; j < 32; j += 8) {
      const int c = c0 + tx, r = r0 + j;
      if (r < rows && c < cols)
        dst[c + static_cast<long long>(r) * ldd] = tile[tx][j];
    }
  }
}

template <class S, class D>
cudaError_t relayout(const void* src, long long lds, void* dst, long long ldd, int rows, int cols,
                     bool transpose, cudaStream_t stream) {
  if (rows <= 0 || cols <= 0)
    return cudaSuccess;
  const long long tiles_r = (rows + 31) / 32, tiles_c = (cols + 31) / 32;
  if (tiles_r * tiles_c > 0x7fffffffll)
    return cudaErrorInvalidConfiguration;
  const unsigned grid = static_cast<unsigned>(tiles_r * tiles_c);
  if (transpose)
    relayout_kernel<S, D, true><<<grid, 256, 0, stream>>>(
        static_cast<const S*>(src), lds, static_cast<D*>(dst), ldd, rows, cols,
        static_cast<int>(tiles_r));
  else
    relayout_kernel<S, D, false><<<grid, 256, 0, stream>>>(
        static_cast<const S*>(src), lds, static_cast<D*>(dst), ldd, rows, cols,
        static_cast<int>(tiles_r));
  return cudaGetLastError();
}

// ------------------------------------------------------------------ FP64 kernel
// K per stage and ring depth: C2 FP64 NT, (16, 3) 29.6, (16, 4) 29.9, (32, 2) 30.9, (32, 3)
// 30.9 TFLOP/s -- fewer block barriers per k.
#ifndef XVRAM_DGEMM_BK
#define XVRAM_DGEMM_BK 32
#endif
#ifndef XVRAM_DGEMM_STAGES
#define XVRAM_DGEMM_STAGES 3
#endif
constexpr int kDBM = 128, kDBN = 128, kDBK = XVRAM_DGEMM_BK, kDStages = XVRAM_DGEMM_STAGES;
constexpr int kDPad = 8;
constexpr int kDRow = kDBM + kDPad;            // doubles per k row of a stage tile
constexpr int kDStageDoubles = kDBK * kDRow;   // one operand's stage tile
constexpr int kDSmemBytes = kDStages * 2 * kDStageDoubles * 8;
constexpr int kDThreads = 256;

__device__ __forceinline__ void cp_async8(double* dst, const double* src, bool valid) {
  const uint32_t d = static_cast<uint32_t>(__cvta_generic_to_shared(dst));
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8, %2;" ::"r"(d), "l"(src),
               "r"(valid ? 8 : 0)
               : "memory");
}
// 16 bytes (two doubles); `bytes` (0, 8 or 16) are read, the rest of the 16 zero-filled.
__device__ __forceinline__ void cp_async16(double* dst, const double* src, int bytes) {
  const uint32_t d = static_cast<uint32_t>(__cvta_generic_to_shared(dst));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(d), "l"(src), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N> __device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

#ifndef XVRAM_DGEMM_MMA_K
#define XVRAM_DGEMM_MMA_K 8
#endif
#if XVRAM_DGEMM_MMA_K == 4
// d (8 x 8) += a (8 x 4, row) * b (4 x 8, col); lane l (g = l/4, t = l%4) holds a[g][t],
// b[t][g] and d[g][2t], d[g][2t+1].
__device__ __forceinline__ void dmma_8x8x4(double (&d)[2], double a, double b) {
  asm volatile("mma.sync.aligned.m8n8k4.row.col.f64.f64.f64.f64 {%0,%1}, {%2}, {%3}, {%0,%1};"
               : "+d"(d[0]), "+d"(d[1])
               : "d"(a), "d"(b));
}
#else
// d (16 x 8) += a (16 x 8, row) * b (8 x 8, col); lane l (g = l/4, t = l%4) holds
// a = {a[g][t], a[g+8][t], a[g][t+4], a[g+8][t+4]}, b = {b[t][g], b[t+4][g]} and
// d = {d[g][2t], d[g][2t+1], d[g+8][2t], d[g+8][2t+1]}.
__device__ __forceinline__ void dmma_16x8x8(double (&d)[4], const double (&a)[4],
                                            const double (&b)[2]) {
  asm volatile("mma.sync.aligned.m16n8k8.row.col.f64.f64.f64.f64 {%0,%1,%2,%3}, "
               "{%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
               : "+d"(d[0]), "+d"(d[1]), "+d"(d[2]), "+d"(d[3])
               : "d"(a[0]), "d"(a[1]), "d"(a[2]), "d"(a[3]), "d"(b[0]), "d"(b[1]));
}
#endif

// Stage kt of op(A) (M-major, element (i, k) at a[i + k lda]) and op(B) (N-major, element
// (k, j) at b[j + k ldb]) into shared stage s: 2048 doubles each, threads consecutive
// along M / N so each warp reads contiguous bytes of a column.  VEC16: 16-byte copies
// (bases 16-byte aligned, even leading dimensions), 4 per thread per operand; else
// 8-byte copies, 8 per thread.
template <bool VEC16>
__device__ __forceinline__ void dgemm_load_stage(double* As, double* Bs, const double* a,
                                                 long long lda, const double* b, long long ldb,
                                                 int m, int n, int k, int m0, int n0, int kt,
                                                 int s, int tid) {
  if constexpr (VEC16) {
#pragma unroll
    for (int i = 0; i < (kDBK * kDBM) / (2 * kDThreads); ++i) {
      const int idx = tid + kDThreads * i;
      const int kk = idx / (kDBM / 2), rr = (idx % (kDBM / 2)) * 2;
      const int gk = kt * kDBK + kk;
      const int gm = m0 + rr, gn = n0 + rr;
      const int ba = gk < k ? (gm + 1 < m ? 16 : gm < m ? 8 : 0) : 0;
      const int bb = gk < k ? (gn + 1 < n ? 16 : gn < n ? 8 : 0) : 0;
      cp_async16(As + s * kDStageDoubles + kk * kDRow + rr,
                 ba ? a + gm + static_cast<long long>(gk) * lda : a, ba);
      cp_async16(Bs + s * kDStageDoubles + kk * kDRow + rr,
                 bb ? b + gn + static_cast<long long>(gk) * ldb : b, bb);
    }
  } else {
#pragma unroll
    for (int i = 0; i < (kDBK * kDBM) / kDThreads; ++i) {
      const int idx = tid + kDThreads * i;
      const int kk = idx / kDBM, rr = idx % kDBM;
      const int gk = kt * kDBK + kk;
      const int gm = m0 + rr, gn = n0 + rr;
      const bool va = gk < k && gm < m, vb = gk < k && gn < n;
      cp_async8(As + s * kDStageDoubles + kk * kDRow + rr,
                va ? a + gm + static_cast<long long>(gk) * lda : a, va);
      cp_async8(Bs + s * kDStageDoubles + kk * kDRow + rr,
                vb ? b + gn + static_cast<long long>(gk) * ldb : b, vb);
    }
  }
}

template <bool VEC16>
__global__ void __launch_bounds__(kDThreads, 1)
    dgemm_dmma(int m, int n, int k, double alpha, const double* __restrict__ a, long long lda,
               const double* __restrict__ b, long long ldb, double beta, double* __restrict__ c,
               long long ldc, int tiles_m) {
  extern __shared__ __align__(16) double dsm[];
  double* As = dsm;
  double* Bs = dsm + kDStages * kDStageDoubles;
  const int m0 = (blockIdx.x % tiles_m) * kDBM;
  const int n0 = (blockIdx.x / tiles_m) * kDBN;
  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int wm = warp & 1, wn = warp >> 1; // warp tile: rows wm*64.., columns wn*32..
  const int g = lane >> 2, t = lane & 3;

#if XVRAM_DGEMM_MMA_K == 4
  double acc[8][4][2]; // 8 x 4 blocks of 8 x 8
#else
  double acc[4][4][4]; // 4 x 4 blocks of 16 x 8
#endif
#pragma unroll
  for (int i = 0; i < int(sizeof(acc) / sizeof(double)); ++i)
    (&acc[0][0][0])[i] = 0.0;

  const int k_tiles = (k + kDBK - 1) / kDBK;
#pragma unroll
  for (int s = 0; s < kDStages - 1; ++s) {
    if (s < k_tiles)
      dgemm_load_stage<VEC16>(As, Bs, a, lda, b, ldb, m, n, k, m0, n0, s, s, tid);
    cp_async_commit(); // empty groups keep the group count uniform
  }
  for (int kt = 0; kt < k_tiles; ++kt) {
    cp_async_wait<kDStages - 2>(); // stage kt has landed (this thread's copies)
    __syncthreads();               // ... everyone's; and stage kt - 1 is free
    const int nk = kt + kDStages - 1;
    if (nk < k_tiles)
      dgemm_load_stage<VEC16>(As, Bs, a, lda, b, ldb, m, n, k, m0, n0, nk, nk % kDStages, tid);
    cp_async_commit();
    const double* as = As + (kt % kDStages) * kDStageDoubles + wm * 64 + g;
    const double* bs = Bs + (kt % kDStages) * kDStageDoubles + wn * 32 + g;
#if XVRAM_DGEMM_MMA_K == 4
#pragma unroll
    for (int k4 = 0; k4 < kDBK / 4; ++k4) {
      const int kr = (4 * k4 + t) * kDRow;
      double af[8], bf[4];
#pragma unroll
      for (int i = 0; i < 8; ++i)
        af[i] = as[kr + 8 * i];
#pragma unroll
      for (int j = 0; j < 4; ++j)
        bf[j] = bs[kr + 8 * j];
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j)
          dmma_8x8x4(acc[i][j], af[i], bf[j]);
    }
#else
#pragma unroll
    for (int k8 = 0; k8 < kDBK / 8; ++k8) {
      const int r0 = (8 * k8 + t) * kDRow, r4 = r0 + 4 * kDRow;
      double af[4][4], bf[4][2];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        af[i][0] = as[r0 + 16 * i];
        af[i][1] = as[r0 + 16 * i + 8];
        af[i][2] = as[r4 + 16 * i];
        af[i][3] = as[r4 + 16 * i + 8];
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        bf[j][0] = bs[r0 + 8 * j];
        bf[j][1] = bs[r4 + 8 * j];
      }
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j)
          dmma_16x8x8(acc[i][j], af[i], bf[j]);
    }
#endif
  }
  cp_async_wait<0>();

  // Epilogue: alpha * acc + beta * C in FP64; C is not read when beta == 0.
  const auto put = [&](int row, int col, double v) {
    if (row < m && col < n) {
      double* p = c + row + static_cast<long long>(col) * ldc;
      const double x = alpha * v;
      *p = beta == 0.0 ? x : fma(beta, *p, x);
    }
  };
#if XVRAM_DGEMM_MMA_K == 4
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
      for (int v = 0; v < 2; ++v)
        put(m0 + wm * 64 + 8 * i + g, n0 + wn * 32 + 8 * j + 2 * t + v, acc[i][j][v]);
#else
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
      for (int v = 0; v < 4; ++v)
        put(m0 + wm * 64 + 16 * i + g + 8 * (v >> 1), n0 + wn * 32 + 8 * j + 2 * t + (v & 1),
            acc[i][j][v]);
#endif
}

uint64_t up(uint64_t v, uint64_t q) { return (v + q - 1) / q * q; }

bool aligned(const void* p, uint64_t esize) {
  return (reinterpret_cast<uintptr_t>(p) % esize) == 0;
}

template <class H>
cudaError_t gemm_half(int op_a, int op_b, int m, int n, int k, float alpha, const void* a,
                      long long lda, const void* b, long long ldb, float beta, void* c,
                      long long ldc, bool c_half, void* ws, cudaStream_t stream) {
  const long long lda2 = static_cast<long long>(up(static_cast<uint64_t>(m), 4));
  const long long ldb2 = static_cast<long long>(up(static_cast<uint64_t>(n), 4));
  char* w = static_cast<char*>(ws);
  float* a32 = reinterpret_cast<float*>(w);
  w += up(static_cast<uint64_t>(lda2) * static_cast<uint64_t>(k) * 4, 256);
  float* b32 = reinterpret_cast<float*>(w);
  w += up(static_cast<uint64_t>(ldb2) * static_cast<uint64_t>(k) * 4, 256);
  if (k > 0) {
    // op(A) M-major: op N is stored m x k (widen), op T is stored k x m (widen + transpose).
    cudaError_t e = op_a == 0 ? relayout<H, float>(a, lda, a32, lda2, m, k, false, stream)
                              : relayout<H, float>(a, lda, a32, lda2, k, m, true, stream);
    if (e != cudaSuccess)
      return e;
    // op(B) N-major (element (k, j) at j + k ldb2): op T is stored n x k (widen), op N is
    // stored k x n (widen + transpose).
    e = op_b != 0 ? relayout<H, float>(b, ldb, b32, ldb2, n, k, false, stream)
                  : relayout<H, float>(b, ldb, b32, ldb2, k, n, true, stream);
    if (e != cudaSuccess)
      return e;
  }
  float* c32 = static_cast<float*>(c);
  long long ldc32 = ldc;
  if (c_half) {
    c32 = reinterpret_cast<float*>(w);
    ldc32 = lda2;
    if (beta != 0.0f)
      if (cudaError_t e = relayout<H, float>(c, ldc, c32, ldc32, m, n, false, stream);
          e != cudaSuccess)
        return e;
  }
  if (cudaError_t e = sgemm_ffma(0, 1, m, n, k, alpha, a32, lda2, b32, ldb2, beta, c32, ldc32,
                                 stream);
      e != cudaSuccess)
    return e;
  if (c_half)
    return relayout<float, H>(c32, ldc32, c, ldc, m, n, false, stream);
  return cudaSuccess;
}

cudaError_t gemm_fp64(int op_a, int op_b, int m, int n, int k, double alpha, const double* a,
                      long long lda, const double* b, long long ldb, double beta, double* c,
                      long long ldc, void* ws, cudaStream_t stream) {
  char* w = static_cast<char*>(ws);
  const double* a2 = a;
  const double* b2 = b;
  long long lda2 = lda, ldb2 = ldb;
  if (op_a != 0 && k > 0) { // stored k x m -> m x k
    lda2 = static_cast<long long>(up(static_cast<uint64_t>(m), 4));
    double* at = reinterpret_cast<double*>(w);
    w += up(static_cast<uint64_t>(lda2) * static_cast<uint64_t>(k) * 8, 256);
    if (cudaError_t e = relayout<double, double>(a, lda, at, lda2, k, m, true, stream);
        e != cudaSuccess)
      return e;
    a2 = at;
  }
  if (op_b == 0 && k > 0) { // stored k x n -> n x k (element (k, j) at j + k ldb2)
    ldb2 = static_cast<long long>(up(static_cast<uint64_t>(n), 4));
    double* bt = reinterpret_cast<double*>(w);
    if (cudaError_t e = relayout<double, double>(b, ldb, bt, ldb2, k, n, true, stream);
        e != cudaSuccess)
      return e;
    b2 = bt;
  }
  const long long tiles_m = (m + kDBM - 1) / kDBM, tiles_n = (n + kDBN - 1) / kDBN;
  if (tiles_m * tiles_n > 0x7fffffffll)
    return cudaErrorInvalidConfiguration;
  const bool vec16 = aligned(a2, 16) && aligned(b2, 16) && lda2 % 2 == 0 && ldb2 % 2 == 0;
  const auto kernel = vec16 ? dgemm_dmma<true> : dgemm_dmma<false>;
  // Per call: the attribute belongs to the current device.
  if (cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           kDSmemBytes);
      e != cudaSuccess)
    return e;
  kernel<<<static_cast<unsigned>(tiles_m * tiles_n), kDThreads, kDSmemBytes, stream>>>(
      m, n, k, alpha, a2, lda2, b2, ldb2, beta, c, ldc, static_cast<int>(tiles_m));
  return cudaGetLastError();
}

} // namespace

uint64_t gemm_typed_workspace_bytes(uint32_t ab, uint32_t ct, int compute, int op_a, int op_b,
                                    int m, int n, int k) {
  if (m <= 0 || n <= 0 || k < 0)
    return 0;
  const uint64_t um = static_cast<uint64_t>(m), un = static_cast<uint64_t>(n),
                 uk = static_cast<uint64_t>(k);
  switch (ab) {
  case kFp32:
    if (k == 0)
      return 0;
    return compute == kTf32 ? sgemm_tf32x3_workspace_bytes(m, n, k)
                                   : sgemm_workspace_bytes(op_a, op_b, m, n, k);
  case kFp16:
  case kBf16:
    return up(up(um, 4) * uk * 4, 256) + up(up(un, 4) * uk * 4, 256) +
           (ct != kFp32 ? up(up(um, 4) * un * 4, 256) : 0);
  case kFp64:
    return (op_a != 0 ? up(up(um, 4) * uk * 8, 256) : 0) +
           (op_b == 0 ? up(up(un, 4) * uk * 8, 256) : 0);
  default:
    return 0;
  }
}

cudaError_t gemm_typed(uint32_t ab, uint32_t ct, int compute, int op_a, int op_b, int m, int n,
                       int k, double alpha, const void* a, long long lda, const void* b,
                       long long ldb, double beta, void* c, long long ldc, void* workspace,
                       uint64_t workspace_bytes, cudaStream_t stream) {
  if (m <= 0 || n <= 0)
    return cudaSuccess;
  const uint64_t need = gemm_typed_workspace_bytes(ab, ct, compute, op_a, op_b, m, n, k);
  const uint64_t esize = ab == kFp64 ? 8 : ab == kFp32 ? 4 : 2;
  const uint64_t csize = ct == kFp64 ? 8 : ct == kFp32 ? 4 : 2;
  if (k < 0 || !aligned(a, esize) || !aligned(b, esize) || !aligned(c, csize) ||
      (need > 0 && (!workspace || workspace_bytes < need ||
                    (reinterpret_cast<uintptr_t>(workspace) & 255u))))
    return cudaErrorInvalidValue;
  switch (ab) {
  case kFp32:
    if (ct != kFp32)
      return cudaErrorInvalidValue;
    if (compute == kTf32 && k > 0)
      return sgemm_tf32x3(op_a, op_b, m, n, k, static_cast<float>(alpha),
                          static_cast<const float*>(a), lda, static_cast<const float*>(b), ldb,
                          static_cast<float>(beta), static_cast<float*>(c), ldc, workspace,
                          workspace_bytes, stream);
    return sgemm_ffma_ws(op_a, op_b, m, n, k, static_cast<float>(alpha),
                         static_cast<const float*>(a), lda, static_cast<const float*>(b), ldb,
                         static_cast<float>(beta), static_cast<float*>(c), ldc, workspace,
                         workspace_bytes, stream);
  case kFp16:
  case kBf16:
    if ((ct != ab && ct != kFp32) || compute != kStrictFp32)
      return cudaErrorInvalidValue;
    return ab == kFp16
               ? gemm_half<__half>(op_a, op_b, m, n, k, static_cast<float>(alpha), a, lda, b,
                                   ldb, static_cast<float>(beta), c, ldc, ct != kFp32,
                                   workspace, stream)
               : gemm_half<__nv_bfloat16>(op_a, op_b, m, n, k, static_cast<float>(alpha), a,
                                          lda, b, ldb, static_cast<float>(beta), c, ldc,
                                          ct != kFp32, workspace, stream);
  case kFp64:
    if (ct != kFp64 || compute != kComputeFp64)
      return cudaErrorInvalidValue;
    return gemm_fp64(op_a, op_b, m, n, k, alpha, static_cast<const double*>(a), lda,
                     static_cast<const double*>(b), ldb, beta, static_cast<double*>(c), ldc,
                     workspace, stream);
  default:
    return cudaErrorInvalidValue;
  }
}

cudaError_t convert_matrix(uint32_t src_type, const void* src, long long lds, uint32_t dst_type,
                           void* dst, long long ldd, int rows, int cols, cudaStream_t stream) {
  if (rows <= 0 || cols <= 0)
    return cudaSuccess;
  if (src_type == kFp16 && dst_type == kFp32)
    return relayout<__half, float>(src, lds, dst, ldd, rows, cols, false, stream);
  if (src_type == kBf16 && dst_type == kFp32)
    return relayout<__nv_bfloat16, float>(src, lds, dst, ldd, rows, cols, false, stream);
  if (src_type == kFp32 && dst_type == kFp16)
    return relayout<float, __half>(src, lds, dst, ldd, rows, cols, false, stream);
  if (src_type == kFp32 && dst_type == kBf16)
    return relayout<float, __nv_bfloat16>(src, lds, dst, ldd, rows, cols, false, stream);
  return cudaErrorInvalidValue;
}

} // namespace xvram
