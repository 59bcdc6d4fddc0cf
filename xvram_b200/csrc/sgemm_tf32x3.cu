// sgemm_tf32x3.cu -- FP32 GEMM on the 5th-generation tensor cores (tcgen05, TMEM) by
// three-term TF32 splitting ("3xTF32").
//
//   x = hi(x) + lo(x),  hi = TF32(x),  lo = TF32(x - hi)          (round to nearest)
//   a*b ~ hi(a)*hi(b) + hi(a)*lo(b) + lo(a)*hi(b)                   (lo*lo dropped)
//
// Each representation error is below 2^-21 |x|, so a product carries a relative error of
// a few 2^-21.  The larger error source is the tensor core's FP32 accumulation, which
// does not round to nearest: every MMA can lose up to about one unit in the last place of
// the accumulator, and these losses do not cancel.  Two measures bound it:
//   * the small cross terms hi*lo + lo*hi accumulate in their own TMEM accumulator, so the
//     large accumulator takes K/8 MMAs instead of 3K/8; the epilogue adds the two in FP32
//     (round to nearest);
//   * K is processed in launches of at most kChunkK, each ending in an FP32 round-to-
//     nearest update of C (beta on the first launch, 1 after), so no accumulator chain is
//     longer than kChunkK.
// The result meets the path's stated tolerance max|err| / (K max|a| max|b|) <= 1e-6; it
// is not bit-identical to the FFMA kernels.
//
// Pipeline:
//   split pass : operands -> hi/lo arrays in K-major layout [rows][K] (one HBM pass, also
//                transposing M-/N-major operands), in caller-provided scratch.
//   GEMM kernel: CTA tile 128 x 256, K in stages of 16 (64-byte rows, 64-byte swizzle);
//     warp 0      one lane: 2D TMA loads of A_hi, A_lo, B_hi, B_lo into a 4-deep ring;
//     warp 1      allocates 256 TMEM columns; one lane issues, per k8 step,
//                 tcgen05.mma.kind::tf32 lo*hi, hi*lo, hi*hi (M=128, N=256) into the TMEM
//                 accumulator and commits each stage back to the producer;
//     warps 2..5  epilogue: tcgen05.ld 32 lanes x 16 columns at a time, alpha/beta, stores
//                 coalesced along M.
// All waits are bounded; a timeout sets a bit in the kernel error word, the CTA drains
// what it issued, frees its TMEM and returns.
#include "device_common.cuh"
#include "kernels.hpp"

#include <cuda_runtime.h>
#include <cudaTypedefs.h>

namespace xvram {

// Sticky error word of the tensor-core kernel (bits as in the FFMA kernel's word, plus
// bit 3: the epilogue gave up waiting for the accumulator).
__device__ unsigned int xvram_kernel_error_tc = 0;

namespace {

constexpr int kBM = 128;
constexpr int kBN = 256;
constexpr int kBK = 16;                 // tf32 elements per stage row (64 bytes)
constexpr int kStages = 4;
constexpr int kThreads = 192;           // 6 warps
constexpr uint32_t kTileA = kBM * kBK * 4; // 8 KB
constexpr uint32_t kTileB = kBN * kBK * 4; // 16 KB
constexpr uint32_t kStageBytes = 2 * kTileA + 2 * kTileB;
constexpr int kSmemBytes = kStages * kStageBytes + 1024 + 256;
constexpr uint32_t kTmemCols = 512;    // two 128 x 256 FP32 accumulators
constexpr uint32_t kSmallCol = 256;     // column of the cross-term accumulator
constexpr int kChunkK = 2048;           // longest tensor-core accumulation chain

// Instruction descriptor: D F32, A/B TF32, both K-major, N = 256, M = 128.
constexpr uint32_t kIdesc = (1u << 4) | (2u << 7) | (2u << 10) | ((kBN >> 3) << 17) |
                            ((kBM >> 4) << 24);

// Shared-memory matrix descriptor for a K-major tile with 64-byte swizzle: core matrices
// of 8 rows x 64 bytes, 512 bytes apart (stride byte offset); leading byte offset unused.
__device__ __forceinline__ uint64_t smem_desc_sw64(uint32_t saddr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr & 0x3FFFF) >> 4);
  d |= static_cast<uint64_t>(1) << 16;              // LBO (ignored for swizzled K-major)
  d |= static_cast<uint64_t>(512 >> 4) << 32;       // SBO
  d |= static_cast<uint64_t>(1) << 46;              // descriptor version (sm_100)
  d |= static_cast<uint64_t>(4) << 61;              // SWIZZLE_64B
  return d;
}

__device__ __forceinline__ void mma_tf32(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n"
      "  .reg .pred p;\n"
      "  setp.ne.b32 p, %4, 0;\n"
      "  tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n"
      "}\n" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(kIdesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i)
    v[i] = __uint_as_float(r[i]);
}

struct Tf32Params {
  int m, n, k;
  int k_begin; // first K tile of this launch
  int k_tiles, tiles_m, tiles_n;
  float alpha, beta;
  float* c;
  long long ldc;
  unsigned long long timeout_ns;
};

__global__ void __launch_bounds__(kThreads, 1)
    sgemm_tf32x3_kernel(const __grid_constant__ CUtensorMap tm_ahi,
                        const __grid_constant__ CUtensorMap tm_alo,
                        const __grid_constant__ CUtensorMap tm_bhi,
                        const __grid_constant__ CUtensorMap tm_blo, const Tf32Params p) {
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kStages * kStageBytes);
  uint64_t* empty = full + kStages;
  uint64_t* acc_full = empty + kStages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_full + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int bid = blockIdx.x;
  const int group_span = 8 * p.tiles_n;
  const int first_m = (bid / group_span) * 8;
  const int group_m = min(8, p.tiles_m - first_m);
  const int m0 = (first_m + (bid % group_span) % group_m) * kBM;
  const int n0 = ((bid % group_span) / group_m) * kBN;

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;

  if (tid == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(acc_full, 1);
    *abort_flag = 0;
    fence_mbarrier_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  auto stage_ptr = [&](int s, int which) -> unsigned char* {
    // which: 0 A_hi, 1 A_lo, 2 B_hi, 3 B_lo
    unsigned char* base = smem + s * kStageBytes;
    return base + (which < 2 ? which * kTileA : 2 * kTileA + (which - 2) * kTileB);
  };

  if (warp == 0) {
    // ---------------------------------------------------------------- producer
    if (lane == 0) {
      prefetch_tensormap(&tm_ahi);
      prefetch_tensormap(&tm_alo);
      prefetch_tensormap(&tm_bhi);
      prefetch_tensormap(&tm_blo);
      int issued = 0;
      for (int kt = 0; kt < p.k_tiles; ++kt) {
        const int s = kt % kStages;
        const int fill = kt / kStages;
        if (*abort_flag)
          break;
        if (fill > 0 && !mbar_wait_bounded(&empty[s], (fill - 1) & 1, p.timeout_ns)) {
          atomicOr(&xvram_kernel_error_tc, 2u);
          *abort_flag = 1;
          break;
        }
        mbar_arrive_expect_tx(&full[s], kStageBytes);
        const int k0 = (p.k_begin + kt) * kBK;
        tma_load_2d(stage_ptr(s, 0), &tm_ahi, &full[s], k0, m0);
        tma_load_2d(stage_ptr(s, 1), &tm_alo, &full[s], k0, m0);
        tma_load_2d(stage_ptr(s, 2), &tm_bhi, &full[s], k0, n0);
        tma_load_2d(stage_ptr(s, 3), &tm_blo, &full[s], k0, n0);
        ++issued;
      }
      // Drain: every armed fill has landed before this CTA may exit.
      for (int kt = (issued > kStages ? issued - kStages : 0); kt < issued; ++kt)
        if (!mbar_wait_bounded(&full[kt % kStages], (kt / kStages) & 1, p.timeout_ns)) {
          atomicOr(&xvram_kernel_error_tc, 4u);
          break;
        }
    }
  } else if (warp == 1) {
    // -------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      for (int kt = 0; kt < p.k_tiles; ++kt) {
        const int s = kt % kStages;
        if (*abort_flag)
          break;
        if (!mbar_wait_bounded(&full[s], (kt / kStages) & 1, p.timeout_ns)) {
          atomicOr(&xvram_kernel_error_tc, 1u);
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        const uint32_t a_hi = smem_u32(stage_ptr(s, 0)), a_lo = smem_u32(stage_ptr(s, 1));
        const uint32_t b_hi = smem_u32(stage_ptr(s, 2)), b_lo = smem_u32(stage_ptr(s, 3));
#pragma unroll
        for (int kk = 0; kk < kBK / 8; ++kk) {
          const uint32_t off = kk * 32; // 8 tf32 = 32 bytes along K inside the swizzle atom
          const uint32_t acc = (kt == 0 && kk == 0) ? 0u : 1u; // first MMA overwrites
          mma_tf32(tmem + kSmallCol, smem_desc_sw64(a_lo + off), smem_desc_sw64(b_hi + off), acc);
          mma_tf32(tmem + kSmallCol, smem_desc_sw64(a_hi + off), smem_desc_sw64(b_lo + off), 1u);
          mma_tf32(tmem, smem_desc_sw64(a_hi + off), smem_desc_sw64(b_hi + off), acc);
        }
        mma_commit(&empty[s]); // stage free once these MMAs have read it
      }
      mma_commit(acc_full); // accumulator complete (or everything issued has drained)
    }
    __syncwarp();
  } else {
    // ---------------------------------------------------------------- epilogue
    const bool ok = mbar_wait_bounded(acc_full, 0, p.timeout_ns * 4);
    if (!ok) {
      atomicOr(&xvram_kernel_error_tc, 8u);
      *abort_flag = 1;
    }
    tc_fence_after();
    const int quad = warp & 3; // TMEM lanes 32*quad .. 32*quad+31 belong to this warp
    const int row = m0 + 32 * quad + lane;
    // tcgen05.ld is warp-collective: decide for the whole warp at once.
    if (__all_sync(0xffffffffu, ok && !*abort_flag)) {
      const uint32_t t_row = tmem + (static_cast<uint32_t>(32 * quad) << 16);
      for (int c0 = 0; c0 < kBN; c0 += 16) {
        float v[16], w[16];
        tmem_ld16(t_row + c0, v);
        tmem_ld16(t_row + kSmallCol + c0, w);
#pragma unroll
        for (int j = 0; j < 16; ++j)
          v[j] += w[j];
        if (row < p.m) {
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int col = n0 + c0 + j;
            if (col < p.n) {
              float* cp = p.c + row + static_cast<long long>(col) * p.ldc;
              const float r = p.alpha * v[j];
              *cp = (p.beta == 0.0f) ? r : fmaf(p.beta, *cp, r);
            }
          }
        }
      }
    }
    tc_fence_before();
  }

  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(kTmemCols)
                 : "memory");
  }
}

// ------------------------------------------------------------------------ split pass
__device__ __forceinline__ float to_tf32(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
}

// hi/lo of X(r, k) into K-major [rows][ldo]: X(r, k) = src[k + r*lds] when k_contig,
// else src[r + k*lds].  32 x 32 tiles through shared memory.
__global__ void __launch_bounds__(256)
    split_tf32_kernel(const float* __restrict__ src, long long lds, bool k_contig, int rows,
                      int kdim, float* __restrict__ hi, float* __restrict__ lo, long long ldo,
                      int tiles_r) {
  __shared__ float tile[32][33];
  const int tr = blockIdx.x % tiles_r, tk = blockIdx.x / tiles_r;
  const int r0 = tr * 32, k0 = tk * 32;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
#pragma unroll
  for (int j = ty; j < 32; j += 8) {
    // tile[rr][kk] = X(r0 + rr, k0 + kk)
    if (k_contig) {
      const int r = r0 + j, k = k0 + tx;
      tile[j][tx] = (r < rows && k < kdim) ? src[k + static_cast<long long>(r) * lds] : 0.0f;
    } else {
      const int r = r0 + tx, k = k0 + j;
      tile[tx][j] = (r < rows && k < kdim) ? src[r + static_cast<long long>(k) * lds] : 0.0f;
    }
  }
  __syncthreads();
#pragma unroll
  for (int j = ty; j < 32; j += 8) {
    const int r = r0 + j, k = k0 + tx;
    if (r < rows && k < kdim) {
      const float x = tile[j][tx];
      const float h = to_tf32(x);
      const long long o = k + static_cast<long long>(r) * ldo;
      hi[o] = h;
      lo[o] = to_tf32(x - h);
    }
  }
}

bool encode_kmajor(CUtensorMap* map, const float* base, uint64_t kdim, uint64_t rows, uint64_t ld,
                   uint32_t box_rows) {
  static PFN_cuTensorMapEncodeTiled_v12000 encode = [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) !=
            cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      f = nullptr;
    return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
  }();
  if (!encode)
    return false;
  const cuuint64_t dims[2] = {kdim, rows};
  const cuuint64_t strides[1] = {ld * sizeof(float)};
  const cuuint32_t box[2] = {static_cast<cuuint32_t>(kBK), box_rows};
  const cuuint32_t es[2] = {1, 1};
  return encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(base), dims, strides,
                box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B,
                CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

uint64_t up(uint64_t v, uint64_t q) { return (v + q - 1) / q * q; }

} // namespace

uint64_t sgemm_tf32x3_workspace_bytes(int m, int n, int k) {
  if (m <= 0 || n <= 0 || k <= 0)
    return 0;
  const uint64_t kp = up(static_cast<uint64_t>(k), 4);
  return 2 * up(static_cast<uint64_t>(m) * kp * 4, 256) + 2 * up(static_cast<uint64_t>(n) * kp * 4, 256);
}

cudaError_t sgemm_tf32x3(int op_a, int op_b, int m, int n, int k, float alpha, const float* a,
                         long long lda, const float* b, long long ldb, float beta, float* c,
                         long long ldc, void* workspace, uint64_t workspace_bytes,
                         cudaStream_t stream) {
  if (m <= 0 || n <= 0)
    return cudaSuccess;
  if (k <= 0 || !workspace || (reinterpret_cast<uintptr_t>(workspace) & 255u) ||
      workspace_bytes < sgemm_tf32x3_workspace_bytes(m, n, k))
    return cudaErrorInvalidValue;
  const uint64_t kp = up(static_cast<uint64_t>(k), 4);
  char* ws = static_cast<char*>(workspace);
  float* a_hi = reinterpret_cast<float*>(ws);
  ws += up(static_cast<uint64_t>(m) * kp * 4, 256);
  float* a_lo = reinterpret_cast<float*>(ws);
  ws += up(static_cast<uint64_t>(m) * kp * 4, 256);
  float* b_hi = reinterpret_cast<float*>(ws);
  ws += up(static_cast<uint64_t>(n) * kp * 4, 256);
  float* b_lo = reinterpret_cast<float*>(ws);

  // Split (and canonicalise to K-major): A(m,k) is K-contiguous for op T; op(B)^T(n,k) is
  // K-contiguous for op N.
  const auto split = [&](const float* src, long long ld, bool k_contig, int rows, float* hi,
                         float* lo) {
    const long long tiles_r = (rows + 31) / 32, tiles_k = (k + 31) / 32;
    if (tiles_r * tiles_k > 0x7fffffffll)
      return cudaErrorInvalidConfiguration;
    split_tf32_kernel<<<static_cast<unsigned>(tiles_r * tiles_k), 256, 0, stream>>>(
        src, ld, k_contig, rows, k, hi, lo, static_cast<long long>(kp), static_cast<int>(tiles_r));
    return cudaGetLastError();
  };
  if (cudaError_t e = split(a, lda, op_a != 0, m, a_hi, a_lo); e != cudaSuccess)
    return e;
  if (cudaError_t e = split(b, ldb, op_b == 0, n, b_hi, b_lo); e != cudaSuccess)
    return e;

  CUtensorMap t_ahi, t_alo, t_bhi, t_blo;
  if (!encode_kmajor(&t_ahi, a_hi, k, m, kp, kBM) || !encode_kmajor(&t_alo, a_lo, k, m, kp, kBM) ||
      !encode_kmajor(&t_bhi, b_hi, k, n, kp, kBN) || !encode_kmajor(&t_blo, b_lo, k, n, kp, kBN))
    return cudaErrorInvalidValue;
  static cudaError_t attr = cudaFuncSetAttribute(
      sgemm_tf32x3_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
  if (attr != cudaSuccess)
    return attr;
  Tf32Params p;
  p.m = m;
  p.n = n;
  p.k = k;
  p.tiles_m = (m + kBM - 1) / kBM;
  p.tiles_n = (n + kBN - 1) / kBN;
  p.alpha = alpha;
  p.c = c;
  p.ldc = ldc;
  p.timeout_ns = kernel_wait_limit_ns();
  const long long grid = static_cast<long long>(p.tiles_m) * p.tiles_n;
  if (grid > 0x7fffffffll)
    return cudaErrorInvalidConfiguration;
  const int total_tiles = (k + kBK - 1) / kBK;
  constexpr int kChunkTiles = kChunkK / kBK;
  for (int t0 = 0; t0 < total_tiles; t0 += kChunkTiles) {
    p.k_begin = t0;
    p.k_tiles = total_tiles - t0 < kChunkTiles ? total_tiles - t0 : kChunkTiles;
    p.beta = t0 == 0 ? beta : 1.0f; // later chunks accumulate into C
    sgemm_tf32x3_kernel<<<static_cast<unsigned>(grid), kThreads, kSmemBytes, stream>>>(
        t_ahi, t_alo, t_bhi, t_blo, p);
    if (cudaError_t e = cudaGetLastError(); e != cudaSuccess)
      return e;
  }
  return cudaSuccess;
}

cudaError_t read_and_clear_kernel_error_tc(unsigned int* out, cudaStream_t stream) {
  unsigned int zero = 0;
  cudaError_t e = cudaMemcpyFromSymbolAsync(out, xvram_kernel_error_tc, sizeof(unsigned int), 0,
                                            cudaMemcpyDeviceToHost, stream);
  if (e != cudaSuccess)
    return e;
  e = cudaStreamSynchronize(stream);
  if (e != cudaSuccess || *out == 0)
    return e;
  e = cudaMemcpyToSymbolAsync(xvram_kernel_error_tc, &zero, sizeof(zero), 0,
                              cudaMemcpyHostToDevice, stream);
  if (e != cudaSuccess)
    return e;
  return cudaStreamSynchronize(stream);
}

} // namespace xvram
