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
//   GEMM kernel: a CTA pair (cluster of 2, one per SM) computes a 256 x 256 tile of C;
//     each CTA stages its 128 rows of A and its 128-row half of B, K in stages of 32
//     (128-byte rows, 128-byte swizzle) through a 3-deep ring of 64 KB stages.  Rows of
//     128 bytes halve the TMA row requests per MMA against 64-byte rows, and the pair
//     halves each SM's B bytes against a single-CTA 128 x 256 tile;
//     warp 0      one lane per CTA: 2D TMA loads (cta_group::2 form) of A_hi, A_lo, B_hi,
//                 B_lo, completion counted on the leader's barrier;
//     warp 1      allocates 512 TMEM columns in each CTA; on the leader one lane issues,
//                 per k8 step, tcgen05.mma.cta_group::2.kind::tf32 lo*hi, hi*lo (cross-term
//                 accumulator) and hi*hi (M=256, N=256), and commits each stage back to
//                 both CTAs' producers;
//     warps 2..9  epilogue per CTA, two warps per TMEM lane quarter splitting the columns:
//                 tcgen05.ld 32 lanes x 16 columns of both accumulators, sum, alpha/beta,
//                 stores coalesced along M (the epilogue is not overlapped with MMAs --
//                 both accumulators fill TMEM -- so its length counts directly).
// All waits are bounded; a timeout sets a bit in the kernel error word, the CTA drains
// what it issued, frees its TMEM and returns.
#include "device_common.cuh"
#include "kernels.hpp"

#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <algorithm>

namespace xvram {

// Sticky error word of the tensor-core kernel (bits as in the FFMA kernel's word, plus
// bit 3: the epilogue gave up waiting for the accumulator).
__device__ unsigned int xvram_kernel_error_tc = 0;

namespace {

// A CTA pair (cluster of 2) computes one 256 x 256 tile of C: CTA rank r holds rows
// [128 r, 128 r + 128) of the A tile and rows [128 r, 128 r + 128) of the B tile (N half),
// and its TMEM holds its 128 rows x 256 columns of the accumulators.  Only the pair's
// leader (rank 0) issues the MMAs (cta_group::2, M = 256, N = 256); the hardware reads
// the A and B halves from both CTAs' shared memory at the same offsets.
constexpr int kPairM = 256;
constexpr int kPairN = 256;
constexpr int kRows = 128;              // rows of A and of B each CTA stages
constexpr int kBK = 32;                 // tf32 elements per stage row (128 bytes)
constexpr int kStages = 3;
constexpr int kThreads = 320;           // 10 warps: producer, MMA, 8 epilogue
constexpr uint32_t kTile = kRows * kBK * 4;          // 16 KB: one of A_hi, A_lo, B_hi, B_lo
constexpr uint32_t kStageBytes = 4 * kTile;          // 64 KB per CTA per stage
constexpr int kSmemBytes = kStages * kStageBytes + 1024 + 256;
constexpr uint32_t kTmemCols = 512;    // two 128 x 256 FP32 accumulators per CTA
constexpr uint32_t kSmallCol = 256;     // column of the cross-term accumulator
constexpr int kChunkK = 2048;           // longest tensor-core accumulation chain

// Instruction descriptor: D F32, A/B TF32, both K-major, N = 256, M = 256 (CTA pair).
constexpr uint32_t kIdesc = (1u << 4) | (2u << 7) | (2u << 10) | ((kPairN >> 3) << 17) |
                            ((kPairM >> 4) << 24);

// Shared-memory matrix descriptor for a K-major tile with 128-byte swizzle: core matrices
// of 8 rows x 128 bytes, 1024 bytes apart (stride byte offset); leading byte offset unused.
// A K step of 8 tf32 inside the 128-byte row advances the start address by 32 bytes.
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t saddr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr & 0x3FFFF) >> 4);
  d |= static_cast<uint64_t>(1) << 16;              // LBO (ignored for swizzled K-major)
  d |= static_cast<uint64_t>(1024 >> 4) << 32;      // SBO
  d |= static_cast<uint64_t>(1) << 46;              // descriptor version (sm_100)
  d |= static_cast<uint64_t>(2) << 61;              // SWIZZLE_128B
  return d;
}

__device__ __forceinline__ void mma_tf32_pair(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc,
                                              uint32_t accumulate) {
  asm volatile(
      "{\n"
      "  .reg .pred p;\n"
      "  setp.ne.b32 p, %4, 0;\n"
      "  tcgen05.mma.cta_group::2.kind::tf32 [%0], %1, %2, %3, p;\n"
      "}\n" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(kIdesc), "r"(accumulate)
      : "memory");
}

// Arrives on the mbarrier at shared::cluster address `bar` (this CTA's or the peer's) once
// every tensor-core operation issued so far by this thread has completed.
__device__ __forceinline__ void mma_commit_pair(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   bar)
               : "memory");
}

// shared::cluster address of the same shared::cta offset in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t cluster_addr(const void* p, uint32_t rank) {
  uint32_t out;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(out) : "r"(smem_u32(p)), "r"(rank));
  return out;
}

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n"
               "barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// 2D TMA load into this CTA's shared memory whose completion bytes are counted on the
// mbarrier at shared::cluster address `bar` (the pair leader's barrier).
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* map, uint32_t bar,
                                                 int32_t x, int32_t y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(x), "r"(y)
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

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
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

  const uint32_t rank = cluster_rank();
  const bool leader = rank == 0;
  const int pair = blockIdx.x >> 1;
  const int group_span = 8 * p.tiles_n;
  const int first_m = (pair / group_span) * 8;
  const int group_m = min(8, p.tiles_m - first_m);
  const int pm0 = (first_m + (pair % group_span) % group_m) * kPairM;
  const int pn0 = ((pair % group_span) / group_m) * kPairN;
  const int m0 = pm0 + kRows * static_cast<int>(rank); // this CTA's A rows (and C rows)
  const int nb0 = pn0 + kRows * static_cast<int>(rank); // this CTA's B rows (N half)

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;

  if (tid == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1); // used on the leader: its producer's expect_tx arrival
      mbar_init(&empty[s], 1);
    }
    mbar_init(acc_full, 1);
    *abort_flag = 0;
    fence_mbarrier_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  cluster_sync(); // both CTAs' barriers exist before any cross-CTA arrival
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  auto stage_ptr = [&](int s, int which) -> unsigned char* {
    return smem + s * kStageBytes + which * kTile; // 0 A_hi, 1 A_lo, 2 B_hi, 3 B_lo
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
        const uint32_t bar = cluster_addr(&full[s], 0);
        if (leader)
          mbar_arrive_expect_tx(&full[s], 2 * kStageBytes); // both CTAs' copies
        const int k0 = (p.k_begin + kt) * kBK;
        tma_load_2d_pair(stage_ptr(s, 0), &tm_ahi, bar, k0, m0);
        tma_load_2d_pair(stage_ptr(s, 1), &tm_alo, bar, k0, m0);
        tma_load_2d_pair(stage_ptr(s, 2), &tm_bhi, bar, k0, nb0);
        tma_load_2d_pair(stage_ptr(s, 3), &tm_blo, bar, k0, nb0);
        ++issued;
      }
      // Drain: every stage this CTA filled has been consumed (or times out) before exit.
      for (int kt = (issued > kStages ? issued - kStages : 0); kt < issued; ++kt) {
        if (!mbar_wait_bounded(&empty[kt % kStages], (kt / kStages) & 1, p.timeout_ns)) {
          atomicOr(&xvram_kernel_error_tc, 4u);
          break;
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------- MMA issuer (pair leader)
    if (leader && lane == 0) {
      const uint32_t empty_peer0 = cluster_addr(&empty[0], 1);
      const uint32_t empty_self0 = cluster_addr(&empty[0], 0);
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
          mma_tf32_pair(tmem + kSmallCol, smem_desc_sw128(a_lo + off), smem_desc_sw128(b_hi + off),
                        acc);
          mma_tf32_pair(tmem + kSmallCol, smem_desc_sw128(a_hi + off), smem_desc_sw128(b_lo + off),
                        1u);
          mma_tf32_pair(tmem, smem_desc_sw128(a_hi + off), smem_desc_sw128(b_hi + off), acc);
        }
        // Stage s is free in both CTAs once these MMAs have read it.
        const uint32_t soff = static_cast<uint32_t>(s) * sizeof(uint64_t);
        mma_commit_pair(empty_self0 + soff);
        mma_commit_pair(empty_peer0 + soff);
      }
      mma_commit_pair(cluster_addr(acc_full, 0));
      mma_commit_pair(cluster_addr(acc_full, 1));
    }
    __syncwarp();
  } else {
    // ---------------------------------------------------------------- epilogue
    // Two epilogue warps per TMEM lane quarter (a warp may only read lanes 32 * (warp % 4)
    // onwards), each taking half of the 256 columns.
    const int quad = warp & 3; // TMEM lanes 32*quad .. 32*quad+31 belong to this warp
    const int col_begin = ((warp - 2) >> 2) * (kPairN / 2);
    const int col_end = col_begin + kPairN / 2;
    const int row = m0 + 32 * quad + lane;
    // While the MMAs run, pull this thread's row of the C tile into L2: a warp's 32 rows of
    // one column are one 128-byte line, so the epilogue's reads below hit L2.
    if (p.beta != 0.0f && row < p.m) {
      for (int c = col_begin; c < col_end; ++c) {
        const int col = pn0 + c;
        if (col < p.n)
          asm volatile("prefetch.global.L2 [%0];" ::"l"(p.c + row + static_cast<long long>(col) * p.ldc));
      }
    }
    const bool ok = mbar_wait_bounded(acc_full, 0, p.timeout_ns * 4);
    if (!ok) {
      atomicOr(&xvram_kernel_error_tc, 8u);
      *abort_flag = 1;
    }
    tc_fence_after();
    // tcgen05.ld is warp-collective: decide for the whole warp at once.
    if (__all_sync(0xffffffffu, ok && !*abort_flag)) {
      const uint32_t t_row = tmem + (static_cast<uint32_t>(32 * quad) << 16);
      for (int c0 = col_begin; c0 < col_end; c0 += 16) {
        float v[16], w[16];
        tmem_ld16(t_row + c0, v);
        tmem_ld16(t_row + kSmallCol + c0, w);
#pragma unroll
        for (int j = 0; j < 16; ++j)
          v[j] += w[j];
        if (row < p.m) {
          // All sixteen C reads are issued before any store: read-then-write per column
          // would make each read wait for the previous column's store (the columns' addresses
          // are not provably distinct), one memory round trip per column.
          float cv[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int col = pn0 + c0 + j;
            cv[j] = (p.beta != 0.0f && col < p.n)
                        ? p.c[row + static_cast<long long>(col) * p.ldc]
                        : 0.0f;
          }
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int col = pn0 + c0 + j;
            if (col < p.n) {
              const float r = p.alpha * v[j];
              p.c[row + static_cast<long long>(col) * p.ldc] =
                  (p.beta == 0.0f) ? r : fmaf(p.beta, cv[j], r);
            }
          }
        }
      }
    }
    tc_fence_before();
  }

  // Neither CTA leaves (or frees TMEM) while its partner may still use its shared memory
  // or TMEM: every wait above is bounded, so both CTAs reach this point.
  __syncthreads();
  cluster_sync();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem),
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

// hi/lo of an operand that is already K-contiguous with K and its leading dimension
// multiples of 4: a streaming elementwise pass, 16 bytes in and 2 x 16 bytes out per
// thread and step (no transpose, no shared memory).
__global__ void __launch_bounds__(256)
    split_tf32_vec4(const float4* __restrict__ src, long long lds4, int rows, int k4,
                    float4* __restrict__ hi, float4* __restrict__ lo, long long ldo4) {
  const long long total = static_cast<long long>(rows) * k4;
  for (long long i = blockIdx.x * 256ll + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * 256) {
    const long long r = i / k4, q = i - r * k4;
    const float4 x = src[q + r * lds4];
    float4 h, l;
    h.x = to_tf32(x.x);
    h.y = to_tf32(x.y);
    h.z = to_tf32(x.z);
    h.w = to_tf32(x.w);
    l.x = to_tf32(x.x - h.x);
    l.y = to_tf32(x.y - h.y);
    l.z = to_tf32(x.z - h.z);
    l.w = to_tf32(x.w - h.w);
    hi[q + r * ldo4] = h;
    lo[q + r * ldo4] = l;
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
                box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
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
  SgemmPrepared p;
  if (cudaError_t e = sgemm_tf32x3_prepare(op_a, op_b, m, n, k, a, lda, b, ldb, workspace,
                                           workspace_bytes, stream, &p);
      e != cudaSuccess)
    return e;
  return sgemm_tf32x3_block(p, m, 0, n, k, alpha, beta, c, ldc, stream);
}

cudaError_t sgemm_tf32x3_prepare(int op_a, int op_b, int m, int n, int k, const float* a,
                                 long long lda, const float* b, long long ldb, void* workspace,
                                 uint64_t workspace_bytes, cudaStream_t stream,
                                 SgemmPrepared* out) {
  if (m <= 0 || n <= 0 || k <= 0 || !workspace ||
      (reinterpret_cast<uintptr_t>(workspace) & 255u) ||
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
    if (k_contig && k % 4 == 0 && ld % 4 == 0 && (reinterpret_cast<uintptr_t>(src) & 15u) == 0) {
      int dev = 0, sms = 148;
      if (cudaGetDevice(&dev) == cudaSuccess)
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
      const long long work = static_cast<long long>(rows) * (k / 4);
      const long long blocks = std::min<long long>((work + 255) / 256, 16ll * sms);
      split_tf32_vec4<<<static_cast<unsigned>(blocks), 256, 0, stream>>>(
          reinterpret_cast<const float4*>(src), ld / 4, rows, k / 4,
          reinterpret_cast<float4*>(hi), reinterpret_cast<float4*>(lo),
          static_cast<long long>(kp) / 4);
      return cudaGetLastError();
    }
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
  *out = SgemmPrepared{};
  out->tf32 = true;
  out->a_hi = a_hi;
  out->a_lo = a_lo;
  out->b_hi = b_hi;
  out->b_lo = b_lo;
  out->kp = static_cast<long long>(kp);
  return cudaSuccess;
}

cudaError_t sgemm_tf32x3_block(const SgemmPrepared& o, int m, int n0, int nj, int k, float alpha,
                               float beta, float* c, long long ldc, cudaStream_t stream) {
  if (m <= 0 || nj <= 0)
    return cudaSuccess;
  if (k <= 0 || !o.tf32 || n0 < 0)
    return cudaErrorInvalidValue;
  const uint64_t kp = static_cast<uint64_t>(o.kp);
  const int n = nj;
  // op(B)'s columns n0.. are rows n0.. of the K-major splits.
  const float* b_hi = o.b_hi + static_cast<uint64_t>(n0) * kp;
  const float* b_lo = o.b_lo + static_cast<uint64_t>(n0) * kp;
  CUtensorMap t_ahi, t_alo, t_bhi, t_blo;
  if (!encode_kmajor(&t_ahi, o.a_hi, k, m, kp, kRows) ||
      !encode_kmajor(&t_alo, o.a_lo, k, m, kp, kRows) ||
      !encode_kmajor(&t_bhi, b_hi, k, n, kp, kRows) ||
      !encode_kmajor(&t_blo, b_lo, k, n, kp, kRows))
    return cudaErrorInvalidValue;
  static cudaError_t attr = cudaFuncSetAttribute(
      sgemm_tf32x3_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
  if (attr != cudaSuccess)
    return attr;
  Tf32Params p;
  p.m = m;
  p.n = n;
  p.k = k;
  p.tiles_m = (m + kPairM - 1) / kPairM;
  p.tiles_n = (n + kPairN - 1) / kPairN;
  p.alpha = alpha;
  p.c = c;
  p.ldc = ldc;
  p.timeout_ns = kernel_wait_limit_ns();
  const long long grid = 2ll * p.tiles_m * p.tiles_n; // two CTAs per tile (cluster pairs)
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
