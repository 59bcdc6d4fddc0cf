// sgemm_ffma.cu -- strict-FP32 tile contraction for sm_100a.
//
//   C[m0.., n0..] = alpha * op(A) * op(B) + beta * C      (column-major, op in {N, T})
//
// This is the arithmetic the reference delegates to cublasLtMatmul with
// CUBLAS_COMPUTE_32F_PEDANTIC for every tile of its tiled executor
// (reference src/gemm/executor.cpp:147-329, src/platform/cublas/cublas_api.cpp:751-918).
// Every product and sum is an FP32 FFMA; there is no TF32 or reduced-precision step.
//
// Two tilings of one TMA-fed design (which one runs: tiling.hpp):
//   * sgemm_ffma_tma_192 (M-/N-major operands): 192 x 192 C tiles, 12 warps, 12 x 8 per
//     thread -- see its own comment further down;
//   * sgemm_ffma_tma (every layout): described here.
// sgemm_ffma_tma: 128 x BN C tile per CTA (BN = 256 by default, 128 for narrow N), K in
// stages of 32.
//   * 8 warps (256 threads) each own an 8 x (BN/16) block of C per thread in registers;
//     a warp releases a stage on its "empty" mbarrier when it has consumed it;
//   * thread 0 also drives the 4-deep ring of 2D TMA loads: it fills every stage up
//     front and refills a stage with the tile 4 ahead once all eight warps have
//     released it; completion is signalled on the stage's "full" mbarrier.
//   There is no separate producer warp: a 9-warp block would cap every thread at 224
//   registers, too few for 8x16 (240-254).
// Why 8x16 per thread: an LDS.128 costs four shared-memory wavefronts whatever the
// broadcast, so shared-memory bandwidth per FFMA falls only with the register tile.  An
// 8x8 tile needs one wavefront per SM-clock at full FFMA rate (all of it); 8x16 needs
// 0.75.  The 16 B values are streamed one column (K-major B) or one k row (N-major B)
// at a time so the 128 accumulators fit in the register budget.
// Shared-memory stage layouts follow the stored layout of each operand so that TMA
// writes them without transposition:
//   op(A)=N : A stored M-major -> tile [32 k][128 m], no swizzle.  A thread's rows are
//             4 consecutive m at tm*4 and 4 more at 64+tm*4 (two LDS.128 per k).
//   op(A)=T : A stored K-major -> tile [128 m][32 k], 128-byte swizzle.  A thread's rows
//             are tm + 16*i; one LDS.128 fetches 4 consecutive k of one row.
//   op(B)=N : B stored K-major -> tile [128 n][32 k], 128-byte swizzle (as op(A)=T).
//   op(B)=T : B stored N-major -> tile [32 k][128 n], no swizzle (as op(A)=N).
// Out-of-range rows, columns and k are zero-filled by TMA, so ragged edges need no
// special path in the main loop; the epilogue predicates its stores.
//
// TMA needs 16-byte aligned bases and leading dimensions that are multiples of 4
// floats.  The out-of-core executor always packs panels that way; the generic
// kernel below covers every other device-pointer call.
#include "device_common.cuh"
#include "kernels.hpp"
#include "tiling.hpp"

#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <atomic>
#include <cstdio>
#include <mutex>

namespace xvram {

// Sticky per-device error word written by kernels whose bounded waits ran out.
// Bit 0: a consumer gave up on a full barrier; bit 1: the producer gave up on an
// empty barrier; bit 2: the producer gave up draining its own copies.
__device__ unsigned int xvram_kernel_error = 0;

// Test hook: nonzero makes every later FFMA TMA launch stall on a barrier nothing completes
// for this many ns and then abort through the error word.  Only the test suite's link of the
// library exports the setter (xvram_b200_test_set_kernel_stall, at the end of this file).
std::atomic<unsigned long long> g_test_stall_ns{0};

namespace {

#ifndef XVRAM_FFMA_STAGES
#define XVRAM_FFMA_STAGES 4
#endif
// Groups of 4 k unrolled per loop iteration of the K-major kernels.  With one FFMA per
// FMA, 2 keeps the loop body (~1,100 instructions) small enough for the instruction cache;
// the fully unrolled 32-k stage (8) stalls on instruction fetch (ncu: no_instruction 0.61
// per issue) and runs ~2 % slower.  The packed M-/N-major stage has half the FMA
// instructions and runs fully unrolled (C2: 1, 2, 4, 8 groups -> 56.9, 55.5, 61.1, 61.5
// TFLOP/s).
#ifndef XVRAM_FFMA_GROUP_UNROLL
#define XVRAM_FFMA_GROUP_UNROLL 2
#endif
constexpr int kBM = 128;
constexpr int kBK = 32;
constexpr int kStages = XVRAM_FFMA_STAGES;
constexpr int kGroupUnroll = XVRAM_FFMA_GROUP_UNROLL;
constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kTnCount = kThreads / 16;     // threads sharing an A fragment: 16 B fragments
constexpr int kCtasPerSm = 1;               // the ring takes ~193 KB of shared memory
constexpr int kAStageFloats = kBM * kBK;

// Thread tile 8 x TN (TN = 8 or 16): CTA tile 128 x (16 * TN).
template <int TN> struct TileCfg {
  static constexpr int BN = kTnCount * TN;
  static constexpr int BStageFloats = BN * kBK;
  static constexpr uint32_t StageBytes = (kAStageFloats + BStageFloats) * sizeof(float);
  static constexpr int SmemBytes =
      kStages * (kAStageFloats + BStageFloats) * sizeof(float) + 1024 /*align*/ + 256;
};

struct FfmaParams {
  int m, n, k;
  int k_tiles;
  int tiles_m, tiles_n;
  // Work units [0, full_tiles) are whole tiles; every later pair of units splits one of
  // the remaining tiles into two half-width tiles (see launch_tma).  Unit u runs as block u.
  int full_tiles;
  float alpha, beta;
  float* c;
  long long ldc;
  unsigned long long timeout_ns;
  // Test hook (0 in production): every CTA first waits this long on a barrier that nothing
  // completes, so its bounded wait runs out and the kernel takes its abort path.
  unsigned long long stall_ns;
};

// Fragment loads for one group of 4 consecutive k (g = 0..7 inside a 32-wide stage).
// frag[kk][i] = op(X)(row_i, 4g + kk).
template <bool KMAJOR>
__device__ __forceinline__ void load_frag(const float* tile, int g, int t, float (&frag)[4][8]) {
  if constexpr (KMAJOR) {
    // [128 rows][32 k], 128-byte swizzle: 16-byte chunk c of row r sits at c ^ (r & 7).
    const int chunk = (g ^ (t & 7)) * 4;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float4 v = *reinterpret_cast<const float4*>(tile + (t + 16 * i) * kBK + chunk);
      frag[0][i] = v.x;
      frag[1][i] = v.y;
      frag[2][i] = v.z;
      frag[3][i] = v.w;
    }
  } else {
    // [32 k][128 rows], unswizzled.
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      const float* row = tile + (4 * g + kk) * kBM;
      const float4 lo = *reinterpret_cast<const float4*>(row + 4 * t);
      const float4 hi = *reinterpret_cast<const float4*>(row + 64 + 4 * t);
      frag[kk][0] = lo.x;
      frag[kk][1] = lo.y;
      frag[kk][2] = lo.z;
      frag[kk][3] = lo.w;
      frag[kk][4] = hi.x;
      frag[kk][5] = hi.y;
      frag[kk][6] = hi.z;
      frag[kk][7] = hi.w;
    }
  }
}

// Tile-local row (or column) of a thread's i-th fragment entry: 16-strided rows for
// K-major tiles, groups of four consecutive rows every 64 for M/N-major tiles.
template <bool KMAJOR, int S = 16> __device__ __forceinline__ int frag_index(int t, int i) {
  if constexpr (KMAJOR)
    return t + S * i;
  else
    return 4 * S * (i >> 2) + 4 * t + (i & 3);
}

// Accumulators: acc[i][j / 2] holds columns j (x) and j + 1 (y) of row i.
__device__ __forceinline__ float& acc_at(float2& pair, int odd) { return odd ? pair.y : pair.x; }

// One k-group (4 consecutive k) of a K-major B tile, streamed one column j at a time
// (b = 4 k of column j).  NJ <= TN: a half-width tile computes only the thread's first NJ
// columns.
template <int TN, int NJ>
__device__ __forceinline__ void ffma_group_bk(const float (&a)[4][8], const float* bs, int g,
                                              int tn, float2 (&acc)[8][NJ / 2]) {
  const int chunk = (g ^ (tn & 7)) * 4;
#pragma unroll
  for (int j = 0; j < NJ; ++j) {
    const float4 v = *reinterpret_cast<const float4*>(bs + (tn + kTnCount * j) * kBK + chunk);
    const float b[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int kk = 0; kk < 4; ++kk)
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        float& c = acc_at(acc[i][j >> 1], j & 1);
        c = fmaf(a[kk][i], b[kk], c);
      }
  }
}

// N-major B tile [32 k][BN]: one k row of the thread's TN columns at a time.
// Columns j and j + 1 (j even) of a thread's fragment are adjacent in an N-major row, so
// one float4 load gives two column pairs.
template <int TN, int NJ>
__device__ __forceinline__ void ffma_group_bn(const float (&a)[4][8], const float* bs, int g,
                                              int tn, float2 (&acc)[8][NJ / 2]) {
  constexpr int BN = kTnCount * TN;
#pragma unroll
  for (int kk = 0; kk < 4; ++kk) {
    const float* row = bs + (4 * g + kk) * BN + 4 * tn;
    float2 b[NJ / 2];
#pragma unroll
    for (int q = 0; q < NJ / 4; ++q) {
      const float4 v = *reinterpret_cast<const float4*>(row + 4 * kTnCount * q);
      b[2 * q + 0] = make_float2(v.x, v.y);
      b[2 * q + 1] = make_float2(v.z, v.w);
    }
    // Scalar FMAs: with all four k of A held (K-major A), the packed form's duplicated A
    // values do not fit the register budget.
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
      for (int j2 = 0; j2 < NJ / 2; ++j2) {
        acc[i][j2].x = fmaf(a[kk][i], b[j2].x, acc[i][j2].x);
        acc[i][j2].y = fmaf(a[kk][i], b[j2].y, acc[i][j2].y);
      }
  }
}

// One 32-k stage of M-major A and N-major B (the layout the canonicalising transposes
// produce).  Per k a thread loads its 8 A values (two 16-byte loads) and NJ B values, and
// issues 8 x NJ / 2 packed FP32 FMAs (FFMA2, sm_100: one instruction updates two adjacent
// accumulator columns with the same round-to-nearest FMA per component as fmaf, so the
// bits equal the scalar form's).  The next k's fragments are loaded into a second register
// set before the current k's FMAs (CUDA events, C2: 6.692 against 6.699 ms with the loads
// issued just before their own FMAs).
template <int TN, int NJ>
__device__ __forceinline__ void ffma_stage_mn(const float* as, const float* bs, int tm, int tn,
                                              float2 (&acc)[8][NJ / 2]) {
  constexpr int BN = kTnCount * TN;
  float4 al[2], ah[2], bv[2][NJ / 4];
  auto load = [&](int kk, int slot) {
    const float* arow = as + kk * kBM + 4 * tm;
    al[slot] = *reinterpret_cast<const float4*>(arow);
    ah[slot] = *reinterpret_cast<const float4*>(arow + 64);
    const float* brow = bs + kk * BN + 4 * tn;
#pragma unroll
    for (int q = 0; q < NJ / 4; ++q)
      bv[slot][q] = *reinterpret_cast<const float4*>(brow + 4 * kTnCount * q);
  };
  load(0, 0);
#pragma unroll
  for (int kk = 0; kk < kBK; ++kk) {
    const int cur = kk & 1;
    if (kk + 1 < kBK)
      load(kk + 1, cur ^ 1);
    const float a[8] = {al[cur].x, al[cur].y, al[cur].z, al[cur].w,
                        ah[cur].x, ah[cur].y, ah[cur].z, ah[cur].w};
    float2 b[NJ / 2];
#pragma unroll
    for (int q = 0; q < NJ / 4; ++q) {
      b[2 * q + 0] = make_float2(bv[cur][q].x, bv[cur][q].y);
      b[2 * q + 1] = make_float2(bv[cur][q].z, bv[cur][q].w);
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float2 ai = make_float2(a[i], a[i]);
#pragma unroll
      for (int j2 = 0; j2 < NJ / 2; ++j2)
        acc[i][j2] = __ffma2_rn(ai, b[j2], acc[i][j2]);
    }
  }
}

// Arms stage s of the ring with K tile kt: expected bytes, then the A and B TMA loads.
template <bool A_KMAJOR, bool B_KMAJOR, int TN>
__device__ __forceinline__ void issue_stage(const CUtensorMap* tmap_a, const CUtensorMap* tmap_b,
                                            float* smem_a, float* smem_b, uint64_t* full, int kt,
                                            int m0, int n0) {
  using Cfg = TileCfg<TN>;
  const int s = kt % kStages;
  mbar_arrive_expect_tx(&full[s], Cfg::StageBytes);
  const int k0 = kt * kBK;
  float* sa = smem_a + s * kAStageFloats;
  float* sb = smem_b + s * Cfg::BStageFloats;
  if constexpr (A_KMAJOR)
    tma_load_2d(sa, tmap_a, &full[s], k0, m0);
  else
    tma_load_2d(sa, tmap_a, &full[s], m0, k0);
  if constexpr (B_KMAJOR)
    tma_load_2d(sb, tmap_b, &full[s], k0, n0);
  else
    tma_load_2d(sb, tmap_b, &full[s], n0, k0);
}

// After a wait ran out: never leave the CTA with copies still landing in its shared
// memory.  Thread 0 waits for the last fill of every slot it armed (loads
// [issued - kStages, issued) of its running count), with a bound ten times the pipeline
// wait's, since only a copy the hardware never completes can reach it; past that bound
// bit 2 of the error word is set and the CTA returns anyway.
__device__ __forceinline__ void drain_loads(uint64_t* full, int issued,
                                            unsigned long long timeout_ns) {
  for (int L = issued > kStages ? issued - kStages : 0; L < issued; ++L)
    if (!mbar_wait_bounded(&full[L % kStages], (L / kStages) & 1, 10ull * timeout_ns)) {
      atomicOr(&xvram_kernel_error, 4u);
      return;
    }
}

// Where work unit u sits in C.  Grouped rasterisation: 8 consecutive M tiles sweep the N
// tiles together so the B stage tiles they share stay in L2.  A half unit's TMA box starts
// at its own first column; the box's second half (columns of the partner, or past N where
// TMA fills zeros) is loaded and not used.
struct UnitCoords {
  int m0, n0;
  bool half;
};
template <int BN, int BM = kBM>
__device__ __forceinline__ UnitCoords unit_coords(const FfmaParams& p, int u) {
  const bool half = u >= p.full_tiles;
  const int tile_lin = half ? p.full_tiles + ((u - p.full_tiles) >> 1) : u;
  const int half_index = half ? ((u - p.full_tiles) & 1) : 0;
  const int group_span = 8 * p.tiles_n;
  const int first_m = (tile_lin / group_span) * 8;
  const int group_m = min(8, p.tiles_m - first_m);
  const int tile_m = first_m + (tile_lin % group_span) % group_m;
  const int tile_n = (tile_lin % group_span) / group_m;
  return {tile_m * BM, tile_n * BN + half_index * (BN / 2), half};
}

// The epilogue reads this thread's C entries; ask L2 for their lines before the K loop,
// so those reads hit L2 afterwards instead of waiting on DRAM.
template <bool A_KMAJOR, bool B_KMAJOR, int NJ>
__device__ __forceinline__ void prefetch_c(const FfmaParams& p, int m0, int n0) {
  if (p.beta == 0.0f)
    return;
  const int tm = threadIdx.x & 15;
  const int tn = threadIdx.x >> 4;
#pragma unroll
  for (int j = 0; j < NJ; ++j) {
    const int col = n0 + frag_index<B_KMAJOR, kTnCount>(tn, j);
    if (col < p.n) {
      const float* cc = p.c + static_cast<long long>(col) * p.ldc;
#pragma unroll
      for (int i = 0; i < 8; i += (A_KMAJOR ? 1 : 4)) { // M-major rows come in fours
        const int row = m0 + frag_index<A_KMAJOR>(tm, i);
        if (row < p.m)
          asm volatile("prefetch.global.L2 [%0];" ::"l"(cc + row));
      }
    }
  }
}

// C = alpha * acc + beta * C for the thread's 8 x NJ entries, two columns at a time: their
// 16 C reads are issued before any store (a read after a store to another column would
// wait for it -- the addresses are not provably distinct).
template <bool A_KMAJOR, bool B_KMAJOR, int NJ>
__device__ __forceinline__ void epilogue(const FfmaParams& p, int m0, int n0,
                                         float2 (&acc)[8][NJ / 2]) {
  const int tm = threadIdx.x & 15;
  const int tn = threadIdx.x >> 4;
  const float alpha = p.alpha, beta = p.beta;
#pragma unroll
  for (int j0 = 0; j0 < NJ; j0 += 2) {
    float cv[2][8];
#pragma unroll
    for (int jj = 0; jj < 2; ++jj) {
      const int col = n0 + frag_index<B_KMAJOR, kTnCount>(tn, j0 + jj);
      const float* cc = p.c + static_cast<long long>(col) * p.ldc;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int row = m0 + frag_index<A_KMAJOR>(tm, i);
        cv[jj][i] = (beta != 0.0f && col < p.n && row < p.m) ? cc[row] : 0.0f;
      }
    }
#pragma unroll
    for (int jj = 0; jj < 2; ++jj) {
      const int col = n0 + frag_index<B_KMAJOR, kTnCount>(tn, j0 + jj);
      if (col >= p.n)
        continue;
      float* cc = p.c + static_cast<long long>(col) * p.ldc;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int row = m0 + frag_index<A_KMAJOR>(tm, i);
        if (row < p.m) {
          const float v = alpha * acc_at(acc[i][(j0 + jj) >> 1], jj & 1);
          cc[row] = (beta == 0.0f) ? v : fmaf(beta, cv[jj][i], v);
        }
      }
    }
  }
}

// The K loop and epilogue of one CTA tile computing the thread's first NJ columns (NJ = TN
// for a whole tile, TN / 2 for a half-width tile).  Every output element is one FFMA chain
// in k order whichever NJ computes it, so whole and half tiles give identical bits.
template <bool A_KMAJOR, bool B_KMAJOR, int TN, int NJ>
__device__ __forceinline__ void tile_main(const CUtensorMap* tmap_a, const CUtensorMap* tmap_b,
                                          float* smem_a, float* smem_b, uint64_t* full,
                                          uint64_t* empty, const FfmaParams& p, int m0, int n0,
                                          int issued) {
  using Cfg = TileCfg<TN>;
  const int tid = threadIdx.x;
  const int tm = tid & 15;
  const int tn = tid >> 4;
  prefetch_c<A_KMAJOR, B_KMAJOR, NJ>(p, m0, n0);
  float2 acc[8][NJ / 2];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < NJ / 2; ++j)
      acc[i][j] = make_float2(0.0f, 0.0f);

  bool aborted = false;
  if (p.stall_ns && !mbar_wait_bounded(empty + kStages, 0, p.stall_ns)) {
    atomicOr(&xvram_kernel_error, 1u);
    aborted = true;
  }
  for (int kt = 0; kt < p.k_tiles && !aborted; ++kt) {
    const int s = kt % kStages;
    const uint32_t phase = (kt / kStages) & 1;
    if (!mbar_wait_bounded(&full[s], phase, p.timeout_ns)) {
      atomicOr(&xvram_kernel_error, 1u);
      aborted = true;
      break;
    }
    const float* as = smem_a + s * kAStageFloats;
    const float* bs = smem_b + s * Cfg::BStageFloats;
    if constexpr (!A_KMAJOR && !B_KMAJOR) {
      ffma_stage_mn<TN, NJ>(as, bs, tm, tn, acc);
    } else {
#pragma unroll kGroupUnroll
      for (int g = 0; g < kBK / 4; ++g) {
        float a[4][8];
        load_frag<A_KMAJOR>(as, g, tm, a);
        if constexpr (B_KMAJOR)
          ffma_group_bk<TN, NJ>(a, bs, g, tn, acc);
        else
          ffma_group_bn<TN, NJ>(a, bs, g, tn, acc);
      }
    }
    __syncwarp();
    if ((tid & 31) == 0)
      mbar_arrive(&empty[s]);
    // Refill this stage with tile kt + 4 once every warp has released tile kt.
    if (tid == 0 && issued < p.k_tiles) {
      if (!mbar_wait_bounded(&empty[s], phase, p.timeout_ns)) {
        atomicOr(&xvram_kernel_error, 2u);
        aborted = true;
        break;
      }
      issue_stage<A_KMAJOR, B_KMAJOR, TN>(tmap_a, tmap_b, smem_a, smem_b, full, issued++, m0, n0);
    }
  }
  if (aborted) {
    if (tid == 0)
      drain_loads(full, issued, p.timeout_ns);
    return;
  }

  epilogue<A_KMAJOR, B_KMAJOR, NJ>(p, m0, n0, acc);
}

template <bool A_KMAJOR, bool B_KMAJOR, int TN>
__global__ void __launch_bounds__(kThreads, kCtasPerSm)
    sgemm_ffma_tma(const __grid_constant__ CUtensorMap tmap_a,
                   const __grid_constant__ CUtensorMap tmap_b, const FfmaParams p) {
  using Cfg = TileCfg<TN>;
  constexpr int BN = Cfg::BN;
  extern __shared__ unsigned char smem_raw[];
  // The 128-byte swizzle pattern repeats every 1024 bytes and is computed from the
  // absolute shared address, so stage buffers start on a 1024-byte boundary.
  float* smem = reinterpret_cast<float*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  float* smem_a = smem;
  float* smem_b = smem + kStages * kAStageFloats;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem_b + kStages * Cfg::BStageFloats);
  uint64_t* empty = full + kStages;

  // Blocks past full_tiles come in pairs that share one tile, each taking half of its
  // columns: the last, partial wave then lasts about half a tile.
  const UnitCoords uc = unit_coords<BN>(p, blockIdx.x);
  const bool half = uc.half;
  const int m0 = uc.m0, n0 = uc.n0;

  const int tid = threadIdx.x;
  if (tid == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kWarps);
    }
    mbar_init(&empty[kStages], 1); // the stall hook's barrier: nothing arrives on it
    fence_mbarrier_init();
  }
  __syncthreads();

  int issued = 0; // meaningful in thread 0 only
  if (tid == 0) {
    prefetch_tensormap(&tmap_a);
    prefetch_tensormap(&tmap_b);
    for (; issued < kStages && issued < p.k_tiles; ++issued)
      issue_stage<A_KMAJOR, B_KMAJOR, TN>(&tmap_a, &tmap_b, smem_a, smem_b, full, issued, m0, n0);
  }
  if (half)
    tile_main<A_KMAJOR, B_KMAJOR, TN, TN / 2>(&tmap_a, &tmap_b, smem_a, smem_b, full, empty, p,
                                              m0, n0, issued);
  else
    tile_main<A_KMAJOR, B_KMAJOR, TN, TN>(&tmap_a, &tmap_b, smem_a, smem_b, full, empty, p, m0,
                                          n0, issued);
}

// ---------------------------------------------------------------------------------
// The 192 x 192 tiling of the M-/N-major kernel: 12 warps (384 threads, three warps on
// each SM sub-partition instead of two), each thread a 12 x 8 block of C (96 accumulators,
// 168 registers: 65,536 / 384).  Per k a thread loads 12 A values (three 16-byte loads)
// and 8 B values (two) and issues 48 packed FMAs; shared-memory traffic per FMA is 11 %
// above the 8 x 16 form's, but the third warp per sub-partition keeps the FMA pipe fed
// while the others wait (9216 x 9216 x 4096 NT, CUDA events: 10.867 against 11.391 ms).
// Same ring (4 stages of 32 k, one 2D TMA load per operand, full/empty mbarriers, thread 0
// producing), same bounded waits and abort path, same tail split into half-width (96
// column) units, and each output is the same FFMA chain in k order, so the bits equal the
// 128 x 256 form's and the generic kernel's.  Used where its waves cost less (t192_fits).
constexpr int kT192Threads = 384;
constexpr int kT192Warps = kT192Threads / 32;
constexpr int kT192 = 192;
constexpr int kT192StageFloats = kT192 * kBK; // per operand
constexpr uint32_t kT192StageBytes = 2u * kT192StageFloats * sizeof(float);
constexpr int kT192Smem = kStages * 2 * kT192StageFloats * sizeof(float) + 1024 + 256;

// Tile-local row of a thread's i-th accumulator row (three runs of four, 64 apart) and
// column of its j-th column (two runs of four, 96 apart).
__device__ __forceinline__ int t192_row(int tm, int i) { return 64 * (i >> 2) + 4 * tm + (i & 3); }
__device__ __forceinline__ int t192_col(int tn, int j) { return 96 * (j >> 2) + 4 * tn + (j & 3); }

// One 32-k stage: A tile [32 k][192 m], B tile [32 k][192 n], both unswizzled; the next
// k's fragments are loaded before the current k's packed FMAs.
template <int NJ>
__device__ __forceinline__ void t192_stage(const float* as, const float* bs, int tm, int tn,
                                           float2 (&acc)[12][NJ / 2]) {
  float4 a4[2][3], b4[2][NJ / 4];
  auto load = [&](int kk, int slot) {
    const float* ar = as + kk * kT192 + 4 * tm;
#pragma unroll
    for (int r = 0; r < 3; ++r)
      a4[slot][r] = *reinterpret_cast<const float4*>(ar + 64 * r);
    const float* br = bs + kk * kT192 + 4 * tn;
#pragma unroll
    for (int q = 0; q < NJ / 4; ++q)
      b4[slot][q] = *reinterpret_cast<const float4*>(br + 96 * q);
  };
  load(0, 0);
#pragma unroll
  for (int kk = 0; kk < kBK; ++kk) {
    const int cur = kk & 1;
    if (kk + 1 < kBK)
      load(kk + 1, cur ^ 1);
    float a[12];
#pragma unroll
    for (int r = 0; r < 3; ++r) {
      a[4 * r + 0] = a4[cur][r].x;
      a[4 * r + 1] = a4[cur][r].y;
      a[4 * r + 2] = a4[cur][r].z;
      a[4 * r + 3] = a4[cur][r].w;
    }
    float2 b[NJ / 2];
#pragma unroll
    for (int q = 0; q < NJ / 4; ++q) {
      b[2 * q + 0] = make_float2(b4[cur][q].x, b4[cur][q].y);
      b[2 * q + 1] = make_float2(b4[cur][q].z, b4[cur][q].w);
    }
#pragma unroll
    for (int i = 0; i < 12; ++i) {
      const float2 ai = make_float2(a[i], a[i]);
#pragma unroll
      for (int j2 = 0; j2 < NJ / 2; ++j2)
        acc[i][j2] = __ffma2_rn(ai, b[j2], acc[i][j2]);
    }
  }
}

__device__ __forceinline__ void t192_issue(const CUtensorMap* tmap_a, const CUtensorMap* tmap_b,
                                           float* smem_a, float* smem_b, uint64_t* full, int kt,
                                           int m0, int n0) {
  const int s = kt % kStages;
  mbar_arrive_expect_tx(&full[s], kT192StageBytes);
  tma_load_2d(smem_a + s * kT192StageFloats, tmap_a, &full[s], m0, kt * kBK);
  tma_load_2d(smem_b + s * kT192StageFloats, tmap_b, &full[s], n0, kt * kBK);
}

// K loop and epilogue of one 192 x 192 tile (NJ = 8) or of its half-width unit (NJ = 4:
// the thread's first run of four columns, 96 of the tile's 192).
template <int NJ>
__device__ __forceinline__ void t192_tile(const CUtensorMap* tmap_a, const CUtensorMap* tmap_b,
                                          float* smem_a, float* smem_b, uint64_t* full,
                                          uint64_t* empty, const FfmaParams& p, int m0, int n0,
                                          int issued) {
  const int tid = threadIdx.x;
  const int tm = tid & 15, tn = tid >> 4;
  if (p.beta != 0.0f) { // C's lines into L2 before the K loop (one prefetch per run of four)
#pragma unroll
    for (int j = 0; j < NJ; ++j) {
      const int col = n0 + t192_col(tn, j);
      if (col < p.n) {
        const float* cc = p.c + static_cast<long long>(col) * p.ldc;
#pragma unroll
        for (int i = 0; i < 12; i += 4) {
          const int row = m0 + t192_row(tm, i);
          if (row < p.m)
            asm volatile("prefetch.global.L2 [%0];" ::"l"(cc + row));
        }
      }
    }
  }
  float2 acc[12][NJ / 2];
#pragma unroll
  for (int i = 0; i < 12; ++i)
#pragma unroll
    for (int j = 0; j < NJ / 2; ++j)
      acc[i][j] = make_float2(0.0f, 0.0f);
  bool aborted = false;
  if (p.stall_ns && !mbar_wait_bounded(empty + kStages, 0, p.stall_ns)) {
    atomicOr(&xvram_kernel_error, 1u);
    aborted = true;
  }
  for (int kt = 0; kt < p.k_tiles && !aborted; ++kt) {
    const int s = kt % kStages;
    const uint32_t phase = (kt / kStages) & 1;
    if (!mbar_wait_bounded(&full[s], phase, p.timeout_ns)) {
      atomicOr(&xvram_kernel_error, 1u);
      aborted = true;
      break;
    }
    t192_stage<NJ>(smem_a + s * kT192StageFloats, smem_b + s * kT192StageFloats, tm, tn, acc);
    __syncwarp();
    if ((tid & 31) == 0)
      mbar_arrive(&empty[s]);
    // Refill this stage with tile kt + 4 once every warp has released tile kt.
    if (tid == 0 && issued < p.k_tiles) {
      if (!mbar_wait_bounded(&empty[s], phase, p.timeout_ns)) {
        atomicOr(&xvram_kernel_error, 2u);
        aborted = true;
        break;
      }
      t192_issue(tmap_a, tmap_b, smem_a, smem_b, full, issued++, m0, n0);
    }
  }
  if (aborted) {
    if (tid == 0)
      drain_loads(full, issued, p.timeout_ns);
    return;
  }
  // C = alpha * acc + beta * C, a column at a time: its 12 C reads before its stores.
  const float alpha = p.alpha, beta = p.beta;
#pragma unroll
  for (int j = 0; j < NJ; ++j) {
    const int col = n0 + t192_col(tn, j);
    if (col >= p.n)
      continue;
    float* cc = p.c + static_cast<long long>(col) * p.ldc;
    float cv[12];
#pragma unroll
    for (int i = 0; i < 12; ++i) {
      const int row = m0 + t192_row(tm, i);
      cv[i] = (beta != 0.0f && row < p.m) ? cc[row] : 0.0f;
    }
#pragma unroll
    for (int i = 0; i < 12; ++i) {
      const int row = m0 + t192_row(tm, i);
      if (row < p.m) {
        const float v = alpha * acc_at(acc[i][j >> 1], j & 1);
        cc[row] = (beta == 0.0f) ? v : fmaf(beta, cv[i], v);
      }
    }
  }
}

__global__ void __launch_bounds__(kT192Threads, 1)
    sgemm_ffma_tma_192(const __grid_constant__ CUtensorMap tmap_a,
                       const __grid_constant__ CUtensorMap tmap_b, const FfmaParams p) {
  extern __shared__ unsigned char smem_raw[];
  float* smem = reinterpret_cast<float*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  float* smem_a = smem;
  float* smem_b = smem + kStages * kT192StageFloats;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem_b + kStages * kT192StageFloats);
  uint64_t* empty = full + kStages;
  const UnitCoords uc = unit_coords<kT192, kT192>(p, blockIdx.x);
  const int m0 = uc.m0, n0 = uc.n0;
  const int tid = threadIdx.x;
  if (tid == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kT192Warps);
    }
    mbar_init(&empty[kStages], 1); // the stall hook's barrier: nothing arrives on it
    fence_mbarrier_init();
  }
  __syncthreads();
  int issued = 0; // meaningful in thread 0 only
  if (tid == 0) {
    prefetch_tensormap(&tmap_a);
    prefetch_tensormap(&tmap_b);
    for (; issued < kStages && issued < p.k_tiles; ++issued)
      t192_issue(&tmap_a, &tmap_b, smem_a, smem_b, full, issued, m0, n0);
  }
  if (uc.half)
    t192_tile<4>(&tmap_a, &tmap_b, smem_a, smem_b, full, empty, p, m0, n0, issued);
  else
    t192_tile<8>(&tmap_a, &tmap_b, smem_a, smem_b, full, empty, p, m0, n0, issued);
}

// ---------------------------------------------------------------------------------
// Layout canonicalisation.  K-major operand tiles (op(A)=T, op(B)=N) cost the FFMA
// kernel 15-25 % against M/N-major tiles (the 4-k fragment loads keep the whole A or B
// fragment live and the register budget is exhausted), so the workspace path first
// transposes such operands in HBM -- a bandwidth-bound pass of 2 x the operand bytes,
// about 1-2 % of the GEMM time -- and then runs the M-major / N-major kernel.
//
// dst (cols x rows, column-major, ldd) = src^T (src rows x cols, column-major, lds).
__global__ void __launch_bounds__(256)
    transpose_f32(const float* __restrict__ src, long long lds, float* __restrict__ dst,
                  long long ldd, int rows, int cols, int tiles_r) {
  __shared__ float tile[32][33];
  const int tr = blockIdx.x % tiles_r;
  const int tc = blockIdx.x / tiles_r;
  const int r0 = tr * 32, c0 = tc * 32;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
#pragma unroll
  for (int j = ty; j < 32; j += 8) {
    const int r = r0 + tx, c = c0 + j;
    if (r < rows && c < cols)
      tile[j][tx] = src[r + static_cast<long long>(c) * lds];
  }
  __syncthreads();
#pragma unroll
  for (int j = ty; j < 32; j += 8) {
    const int c = c0 + tx, r = r0 + j;
    if (r < rows && c < cols)
      dst[c + static_cast<long long>(r) * ldd] = tile[tx][j];
  }
}

// The same transpose with 64 x 64 tiles and 16-byte global loads and stores on both sides
// (four 16-byte accesses in flight per thread, eight blocks per SM), for 16-byte aligned
// bases and leading dimensions that are multiples of 4 floats; a tile's ragged edge falls
// back to 4-byte accesses.
__global__ void __launch_bounds__(256)
    transpose_f32_vec4(const float* __restrict__ src, long long lds, float* __restrict__ dst,
                       long long ldd, int rows, int cols, int tiles_r) {
  __shared__ float tile[64][65]; // [column of src][row of src]
  const int tr = blockIdx.x % tiles_r;
  const int tc = blockIdx.x / tiles_r;
  const int r0 = tr * 64, c0 = tc * 64;
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  const int r = r0 + 4 * tx;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int cl = ty + 16 * j, c = c0 + cl;
    if (c >= cols)
      continue;
    const float* s = src + static_cast<long long>(c) * lds + r;
    float v[4];
    if (r + 3 < rows) {
      const float4 q = *reinterpret_cast<const float4*>(s);
      v[0] = q.x;
      v[1] = q.y;
      v[2] = q.z;
      v[3] = q.w;
    } else {
#pragma unroll
      for (int e = 0; e < 4; ++e)
        v[e] = r + e < rows ? s[e] : 0.0f;
    }
#pragma unroll
    for (int e = 0; e < 4; ++e)
      tile[cl][4 * tx + e] = v[e];
  }
  __syncthreads();
  const int c = c0 + 4 * tx;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int rl = ty + 16 * j, rr = r0 + rl;
    if (rr >= rows)
      continue;
    float* d = dst + static_cast<long long>(rr) * ldd + c;
    const float v[4] = {tile[4 * tx][rl], tile[4 * tx + 1][rl], tile[4 * tx + 2][rl],
                        tile[4 * tx + 3][rl]};
    if (c + 3 < cols) {
      *reinterpret_cast<float4*>(d) = make_float4(v[0], v[1], v[2], v[3]);
    } else {
#pragma unroll
      for (int e = 0; e < 4; ++e)
        if (c + e < cols)
          d[e] = v[e];
    }
  }
}

cudaError_t launch_transpose(const float* src, long long lds, float* dst, long long ldd, int rows,
                             int cols, cudaStream_t stream) {
  const bool vec4 = (reinterpret_cast<uintptr_t>(src) & 15u) == 0 &&
                    (reinterpret_cast<uintptr_t>(dst) & 15u) == 0 && lds % 4 == 0 &&
                    ldd % 4 == 0;
  if (vec4) {
    const long long tr = (rows + 63) / 64, tc = (cols + 63) / 64;
    if (tr * tc > 0x7fffffffll)
      return cudaErrorInvalidConfiguration;
    transpose_f32_vec4<<<static_cast<unsigned>(tr * tc), 256, 0, stream>>>(
        src, lds, dst, ldd, rows, cols, static_cast<int>(tr));
    return cudaGetLastError();
  }
  const long long tiles_r = (rows + 31) / 32, tiles_c = (cols + 31) / 32;
  if (tiles_r * tiles_c > 0x7fffffffll)
    return cudaErrorInvalidConfiguration;
  transpose_f32<<<static_cast<unsigned>(tiles_r * tiles_c), 256, 0, stream>>>(
      src, lds, dst, ldd, rows, cols, static_cast<int>(tiles_r));
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------------
// Generic kernel: any alignment and leading dimension.  64x64 C tile, 256 threads,
// 4x4 per thread, k in steps of 16 through plain shared memory.
__global__ void __launch_bounds__(256)
    sgemm_ffma_generic(int op_a, int op_b, int m, int n, int k, float alpha, const float* a,
                       long long lda, const float* b, long long ldb, float beta, float* c,
                       long long ldc) {
  __shared__ float as[16][64 + 4];
  __shared__ float bs[16][64 + 4];
  const int m0 = blockIdx.x * 64, n0 = blockIdx.y * 64;
  const int tid = threadIdx.x;
  const int tx = tid & 15, ty = tid >> 4;
  float acc[4][4] = {};
  for (int k0 = 0; k0 < k; k0 += 16) {
    for (int e = tid; e < 16 * 64; e += 256) {
      const int kk = e >> 6, r = e & 63;
      const int gi = m0 + r, gk = k0 + kk;
      float av = 0.0f;
      if (gi < m && gk < k)
        av = op_a == 0 ? a[gi + gk * lda] : a[gk + gi * lda];
      as[kk][r] = av;
      const int gj = n0 + r;
      float bv = 0.0f;
      if (gj < n && gk < k)
        bv = op_b == 0 ? b[gk + gj * ldb] : b[gj + gk * ldb];
      bs[kk][r] = bv;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < 16; ++kk) {
      float ar[4], br[4];
#pragma unroll
      for (int i = 0; i < 4; ++i)
        ar[i] = as[kk][tx + 16 * i];
#pragma unroll
      for (int j = 0; j < 4; ++j)
        br[j] = bs[kk][ty + 16 * j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j)
          acc[i][j] = fmaf(ar[i], br[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int col = n0 + ty + 16 * j;
    if (col >= n)
      continue;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int row = m0 + tx + 16 * i;
      if (row < m) {
        float* cp = c + row + static_cast<long long>(col) * ldc;
        const float v = alpha * acc[i][j];
        *cp = (beta == 0.0f) ? v : fmaf(beta, *cp, v);
      }
    }
  }
}

// ---------------------------------------------------------------------------------
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) !=
            cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      p = nullptr;
    return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }();
  return fn;
}

// 2D FP32 tensor map over a column-major matrix stored as `inner` x `outer` with
// leading dimension `ld` (elements), box = box_inner x box_outer.
bool encode_2d(CUtensorMap* map, const float* base, uint64_t inner, uint64_t outer, uint64_t ld,
               uint32_t box_inner, uint32_t box_outer, bool swizzle128) {
  auto encode = tensor_map_encoder();
  if (!encode)
    return false;
  const cuuint64_t dims[2] = {inner, outer};
  const cuuint64_t strides[1] = {ld * sizeof(float)};
  const cuuint32_t box[2] = {box_inner, box_outer};
  const cuuint32_t elem_strides[2] = {1, 1};
  const CUresult r =
      encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(base), dims, strides, box,
             elem_strides, CU_TENSOR_MAP_INTERLEAVE_NONE,
             swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

template <bool AK, bool BK, int TN> cudaError_t configure_once() {
  static cudaError_t status =
      cudaFuncSetAttribute(sgemm_ffma_tma<AK, BK, TN>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           TileCfg<TN>::SmemBytes);
  return status;
}

int sm_count() {
  static int cached[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64)
    return 148;
  if (!cached[dev]) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = 148;
    cached[dev] = n;
  }
  return cached[dev];
}

// One CTA per SM (the ring takes ~193 KB of shared memory), so tiles run in waves of the
// SM count.  When the last wave would be at most half full, its tiles are launched as
// two half-width blocks each: the same work on twice the SMs, half the tail time.
template <bool AK, bool BK, int TN>
cudaError_t launch_tma(const CUtensorMap& ta, const CUtensorMap& tb, FfmaParams p,
                       cudaStream_t stream) {
  if (cudaError_t e = configure_once<AK, BK, TN>(); e != cudaSuccess)
    return e;
  const long long tiles = static_cast<long long>(p.tiles_m) * p.tiles_n;
  const long long sms = static_cast<long long>(sm_count()) * kCtasPerSm;
  const long long tail = tiles % sms;
  long long grid = tiles;
  p.full_tiles = static_cast<int>(tiles);
  if (tail > 0 && 2 * tail <= sms) {
    p.full_tiles = static_cast<int>(tiles - tail);
    grid = tiles + tail;
  }
  if (grid > 0x7fffffffll)
    return cudaErrorInvalidConfiguration;
  sgemm_ffma_tma<AK, BK, TN>
      <<<static_cast<unsigned>(grid), kThreads, TileCfg<TN>::SmemBytes, stream>>>(ta, tb, p);
  return cudaGetLastError();
}

// Whether an M-/N-major problem runs as 192 x 192 tiles on this device (tiling.hpp).
bool t192_fits(int m, int n) { return choose_tiling(m, n, sm_count()).tile_m == kT192; }

cudaError_t launch_t192(const CUtensorMap& ta, const CUtensorMap& tb, FfmaParams p,
                        cudaStream_t stream) {
  static const cudaError_t configured = cudaFuncSetAttribute(
      sgemm_ffma_tma_192, cudaFuncAttributeMaxDynamicSharedMemorySize, kT192Smem);
  if (configured != cudaSuccess)
    return configured;
  const long long tiles = static_cast<long long>(p.tiles_m) * p.tiles_n;
  const long long sms = sm_count();
  const long long tail = tiles % sms;
  long long grid = tiles;
  p.full_tiles = static_cast<int>(tiles);
  if (tail > 0 && 2 * tail <= sms) {
    p.full_tiles = static_cast<int>(tiles - tail);
    grid = tiles + tail;
  }
  if (grid > 0x7fffffffll)
    return cudaErrorInvalidConfiguration;
  sgemm_ffma_tma_192<<<static_cast<unsigned>(grid), kT192Threads, kT192Smem, stream>>>(ta, tb,
                                                                                      p);
  return cudaGetLastError();
}

template <int TN>
cudaError_t launch_tn(bool a_kmajor, bool b_kmajor, const CUtensorMap& ta, const CUtensorMap& tb,
                      const FfmaParams& p, cudaStream_t stream) {
  if (a_kmajor && b_kmajor)
    return launch_tma<true, true, TN>(ta, tb, p, stream);
  if (a_kmajor)
    return launch_tma<true, false, TN>(ta, tb, p, stream);
  if (b_kmajor)
    return launch_tma<false, true, TN>(ta, tb, p, stream);
  return launch_tma<false, false, TN>(ta, tb, p, stream);
}

} // namespace

void sgemm_tile_shape(int m, int n, int* tile_m, int* tile_n) {
  const Tiling t = choose_tiling(m, n, sm_count());
  *tile_m = t.tile_m;
  *tile_n = t.tile_n;
}

bool sgemm_tma_eligible(int op_a, int op_b, const float* a, long long lda, const float* b,
                        long long ldb) {
  (void)op_a;
  (void)op_b;
  const auto aligned16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  return aligned16(a) && aligned16(b) && lda % 4 == 0 && ldb % 4 == 0 && lda > 0 && ldb > 0 &&
         lda < (1ll << 37) && ldb < (1ll << 37) && tensor_map_encoder() != nullptr;
}

uint64_t sgemm_workspace_bytes(int op_a, int op_b, int m, int n, int k) {
  if (m <= 0 || n <= 0 || k <= 0)
    return 0;
  const auto up = [](uint64_t v, uint64_t q) { return (v + q - 1) / q * q; };
  uint64_t bytes = 0;
  if (op_a != 0)
    bytes += up(up(static_cast<uint64_t>(m), 4) * static_cast<uint64_t>(k) * 4, 256);
  if (op_b == 0)
    bytes += up(up(static_cast<uint64_t>(n), 4) * static_cast<uint64_t>(k) * 4, 256);
  return bytes;
}

namespace {

// The FFMA half of sgemm_prepare; `tma` says whether the canonical operands go to the TMA
// kernel (they always qualify) or the operands stay as given.
cudaError_t ffma_prepare(int op_a, int op_b, int m, int n, int k, const float* a, long long lda,
                         const float* b, long long ldb, void* workspace, uint64_t workspace_bytes,
                         SgemmPath path, cudaStream_t stream, SgemmPrepared* out, bool* tma) {
  *out = SgemmPrepared{};
  out->a = a;
  out->b = b;
  out->lda = lda;
  out->ldb = ldb;
  out->op_a = op_a;
  out->op_b = op_b;
  *tma = false;
  const uint64_t need = sgemm_workspace_bytes(op_a, op_b, m, n, k);
  if (need == 0 || !workspace || workspace_bytes < need || path == SgemmPath::generic ||
      (reinterpret_cast<uintptr_t>(workspace) & 255u) != 0 ||
      !sgemm_tma_eligible(op_a, op_b, a, lda, b, ldb))
    return cudaSuccess;
  // Canonicalise K-major operands into the workspace for the M/N-major kernel.
  const auto up4 = [](long long v) { return (v + 3) / 4 * 4; };
  char* ws = static_cast<char*>(workspace);
  if (op_a != 0) {
    float* at = reinterpret_cast<float*>(ws);
    out->lda = up4(m);
    if (cudaError_t e = launch_transpose(a, lda, at, out->lda, k, m, stream); e != cudaSuccess)
      return e;
    out->a = at;
    out->op_a = 0;
    ws += (static_cast<uint64_t>(out->lda) * k * 4 + 255) / 256 * 256;
  }
  if (op_b == 0) {
    float* bt = reinterpret_cast<float*>(ws);
    out->ldb = up4(n);
    if (cudaError_t e = launch_transpose(b, ldb, bt, out->ldb, k, n, stream); e != cudaSuccess)
      return e;
    out->b = bt;
    out->op_b = 1;
  }
  *tma = true;
  return cudaSuccess;
}

// C's columns [n0, n0 + nj): op(B)'s columns n0.. are B's columns (op N) or rows (op T).
cudaError_t ffma_block(const SgemmPrepared& p, int m, int n0, int nj, int k, float alpha,
                       float beta, float* c, long long ldc, cudaStream_t stream, SgemmPath path) {
  const float* b = p.op_b == 0 ? p.b + static_cast<long long>(n0) * p.ldb : p.b + n0;
  return sgemm_ffma(p.op_a, p.op_b, m, nj, k, alpha, p.a, p.lda, b, p.ldb, beta, c, ldc, stream,
                    path);
}

} // namespace

cudaError_t sgemm_ffma_ws(int op_a, int op_b, int m, int n, int k, float alpha, const float* a,
                          long long lda, const float* b, long long ldb, float beta, float* c,
                          long long ldc, void* workspace, uint64_t workspace_bytes,
                          cudaStream_t stream, SgemmPath path) {
  if (m <= 0 || n <= 0)
    return cudaSuccess;
  SgemmPrepared p;
  bool tma = false;
  if (cudaError_t e = ffma_prepare(op_a, op_b, m, n, k, a, lda, b, ldb, workspace,
                                   workspace_bytes, path, stream, &p, &tma);
      e != cudaSuccess)
    return e;
  return ffma_block(p, m, 0, n, k, alpha, beta, c, ldc, stream, tma ? SgemmPath::tma : path);
}

cudaError_t sgemm_prepare(bool tf32, int op_a, int op_b, int m, int n, int k, const float* a,
                          long long lda, const float* b, long long ldb, void* workspace,
                          uint64_t workspace_bytes, cudaStream_t stream, SgemmPrepared* out) {
  if (tf32)
    return sgemm_tf32x3_prepare(op_a, op_b, m, n, k, a, lda, b, ldb, workspace,
                                workspace_bytes, stream, out);
  bool tma = false;
  return ffma_prepare(op_a, op_b, m, n, k, a, lda, b, ldb, workspace, workspace_bytes,
                      SgemmPath::automatic, stream, out, &tma);
}

cudaError_t sgemm_block(const SgemmPrepared& p, int m, int n0, int nj, int k, float alpha,
                        float beta, float* c, long long ldc, cudaStream_t stream) {
  if (m <= 0 || nj <= 0)
    return cudaSuccess;
  if (p.tf32)
    return sgemm_tf32x3_block(p, m, n0, nj, k, alpha, beta, c, ldc, stream);
  return ffma_block(p, m, n0, nj, k, alpha, beta, c, ldc, stream, SgemmPath::automatic);
}

cudaError_t sgemm_ffma(int op_a, int op_b, int m, int n, int k, float alpha, const float* a,
                       long long lda, const float* b, long long ldb, float beta, float* c,
                       long long ldc, cudaStream_t stream, SgemmPath path) {
  if (m <= 0 || n <= 0)
    return cudaSuccess;
  if (k <= 0) {
    // C = beta * C: the generic kernel with k = 0 runs the epilogue only.
    path = SgemmPath::generic;
  }
  const bool tma_ok = k > 0 && sgemm_tma_eligible(op_a, op_b, a, lda, b, ldb);
  if (path == SgemmPath::tma && !tma_ok)
    return cudaErrorInvalidValue;
  if (path == SgemmPath::automatic)
    path = tma_ok ? SgemmPath::tma : SgemmPath::generic;

  if (path == SgemmPath::generic) {
    dim3 grid((m + 63) / 64, (n + 63) / 64);
    if (grid.y > 65535)
      return cudaErrorInvalidConfiguration;
    sgemm_ffma_generic<<<grid, 256, 0, stream>>>(op_a, op_b, m, n, k, alpha, a, lda, b, ldb, beta,
                                                 c, ldc);
    return cudaGetLastError();
  }

  const bool a_kmajor = op_a != 0;
  const bool b_kmajor = op_b == 0;
  FfmaParams p;
  p.m = m;
  p.n = n;
  p.k = k;
  p.k_tiles = (k + kBK - 1) / kBK;
  p.alpha = alpha;
  p.beta = beta;
  p.c = c;
  p.ldc = ldc;
  p.timeout_ns = kernel_wait_limit_ns();
  p.stall_ns = g_test_stall_ns.load(std::memory_order_relaxed);
  if (!a_kmajor && !b_kmajor && t192_fits(m, n)) {
    CUtensorMap ta, tb;
    if (!encode_2d(&ta, a, m, k, lda, kT192, kBK, false) ||
        !encode_2d(&tb, b, n, k, ldb, kT192, kBK, false))
      return cudaErrorInvalidValue;
    p.tiles_m = (m + kT192 - 1) / kT192;
    p.tiles_n = (n + kT192 - 1) / kT192;
    return launch_t192(ta, tb, p, stream);
  }
  // Wide tiles halve shared-memory traffic per FFMA; narrow N keeps 128-wide tiles so
  // fewer columns are wasted on padding.
  const int tn = n > 128 ? 16 : 8;
  const int bn = kTnCount * tn;
  CUtensorMap ta, tb;
  bool ok = a_kmajor ? encode_2d(&ta, a, k, m, lda, kBK, kBM, true)
                     : encode_2d(&ta, a, m, k, lda, kBM, kBK, false);
  ok = ok && (b_kmajor ? encode_2d(&tb, b, k, n, ldb, kBK, bn, true)
                       : encode_2d(&tb, b, n, k, ldb, bn, kBK, false));
  if (!ok)
    return cudaErrorInvalidValue;
  p.tiles_m = (m + kBM - 1) / kBM;
  p.tiles_n = (n + bn - 1) / bn;
  if (static_cast<long long>(p.tiles_m) * p.tiles_n > 0x7fffffffll)
    return cudaErrorInvalidConfiguration;
  return tn == 16 ? launch_tn<16>(a_kmajor, b_kmajor, ta, tb, p, stream)
                  : launch_tn<8>(a_kmajor, b_kmajor, ta, tb, p, stream);
}

cudaError_t transpose_f32_async(const float* src, long long lds, float* dst, long long ldd,
                                int rows, int cols, cudaStream_t stream) {
  if (rows <= 0 || cols <= 0)
    return cudaSuccess;
  return launch_transpose(src, lds, dst, ldd, rows, cols, stream);
}

cudaError_t read_and_clear_kernel_error(unsigned int* out, cudaStream_t stream) {
  unsigned int zero = 0;
  cudaError_t e = cudaMemcpyFromSymbolAsync(out, xvram_kernel_error, sizeof(unsigned int), 0,
                                            cudaMemcpyDeviceToHost, stream);
  if (e != cudaSuccess)
    return e;
  e = cudaStreamSynchronize(stream);
  if (e != cudaSuccess || *out == 0)
    return e;
  e = cudaMemcpyToSymbolAsync(xvram_kernel_error, &zero, sizeof(zero), 0, cudaMemcpyHostToDevice,
                              stream);
  if (e != cudaSuccess)
    return e;
  return cudaStreamSynchronize(stream);
}

unsigned long long kernel_wait_limit_ns() {
  // One second of wall clock for any single mbarrier wait; a stage tile lands in
  // microseconds, so only a broken pipeline ever reaches it.
  return 1000ull * 1000ull * 1000ull;
}

} // namespace xvram

// Testing seam (not exported by the product libraries; tests/fake_device/testing.exports.map
// adds it to the test suite's link): the kernel-stall hook above, in nanoseconds (0: off).
extern "C" __attribute__((visibility("default"))) void
xvram_b200_test_set_kernel_stall(unsigned long long ns) {
  xvram::g_test_stall_ns.store(ns, std::memory_order_relaxed);
}
