// native_api.cpp -- implementations of include/xvram_b200.h.
#include "xvram_b200.h"

#include "host_util.hpp"
#include "kernels.hpp"
#include "planner.hpp"
#include "validate.hpp"

#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <mutex>

namespace xvram {
xvram_status compat_runtime_info(xvram_b200_runtime_info_v1* out);
}

using namespace xvram;

namespace {

cudaStream_t as_stream(uint64_t s) { return reinterpret_cast<cudaStream_t>(s); }

xvram_status from_cuda(cudaError_t e) {
  switch (e) {
  case cudaSuccess:
    return XVRAM_STATUS_SUCCESS;
  case cudaErrorInvalidValue:
  case cudaErrorInvalidConfiguration:
    return XVRAM_STATUS_INVALID_ARGUMENT;
  case cudaErrorMemoryAllocation:
    return XVRAM_STATUS_DEVICE_OUT_OF_MEMORY;
  case cudaErrorNoDevice:
  case cudaErrorInsufficientDriver:
    return XVRAM_STATUS_UNAVAILABLE;
  default:
    return XVRAM_STATUS_CUDA_ERROR;
  }
}

// Private stream-ordered pool per device for the scratch of xvram_b200_sgemm_device.
// Its release threshold is unlimited so steady-state calls reuse pooled memory.
cudaMemPool_t scratch_pool(int device) {
  static std::mutex mu;
  static cudaMemPool_t pools[64] = {};
  std::lock_guard<std::mutex> lock(mu);
  if (device < 0 || device >= 64)
    return nullptr;
  if (!pools[device]) {
    cudaMemPoolProps props{};
    props.allocType = cudaMemAllocationTypePinned;
    props.location.type = cudaMemLocationTypeDevice;
    props.location.id = device;
    cudaMemPool_t pool = nullptr;
    if (cudaMemPoolCreate(&pool, &props) != cudaSuccess) {
      cudaGetLastError();
      return nullptr;
    }
    uint64_t threshold = UINT64_MAX;
    cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &threshold);
    pools[device] = pool;
  }
  return pools[device];
}

bool valid_args(uint32_t op_a, uint32_t op_b, int64_t m, int64_t n, int64_t k, const float* a,
                int64_t lda, const float* b, int64_t ldb, float* c, int64_t ldc, uint32_t path) {
  if (op_a > 1 || op_b > 1 || m < 0 || n < 0 || k < 0 || m > INT32_MAX || n > INT32_MAX ||
      k > INT32_MAX || path > XVRAM_B200_PATH_TF32X3)
    return false;
  if (m == 0 || n == 0)
    return true;
  return c && ldc >= m &&
         (k == 0 || (a && b && lda >= (op_a == 0 ? m : k) && ldb >= (op_b == 0 ? k : n)));
}

SgemmPath to_path(uint32_t path) {
  // (XVRAM_B200_PATH_TF32X3 is dispatched before this mapping is used.)
  return path == XVRAM_B200_PATH_TMA       ? SgemmPath::tma
         : path == XVRAM_B200_PATH_GENERIC ? SgemmPath::generic
                                           : SgemmPath::automatic;
}

PlanStatus plan_for(uint32_t op_a, uint32_t op_b, int64_t m, int64_t n, int64_t k,
                    int32_t beta_nonzero, uint64_t budget, uint64_t quantum, double fps,
                    double h2d, double d2h, int64_t fm, int64_t fn, int64_t fk, Plan* plan) {
  PlanProblem p;
  p.op_a = static_cast<int>(op_a);
  p.op_b = static_cast<int>(op_b);
  p.m = m;
  p.n = n;
  p.k = k;
  p.beta_nonzero = beta_nonzero != 0;
  PlanLimits lim;
  lim.budget_bytes = budget;
  lim.quantum_bytes = quantum;
  if (fps > 0)
    lim.flops_per_s = fps;
  if (h2d > 0)
    lim.h2d_bytes_per_s = h2d;
  if (d2h > 0)
    lim.d2h_bytes_per_s = d2h;
  lim.force_mb = fm;
  lim.force_nb = fn;
  lim.force_kb = fk;
  return make_panel_plan(p, lim, plan);
}

} // namespace

extern "C" {

XVRAM_B200_API xvram_status XVRAM_CALL xvram_b200_sgemm_device(
    uint32_t op_a, uint32_t op_b, int64_t m, int64_t n, int64_t k, float alpha, const float* a,
    int64_t lda, const float* b, int64_t ldb, float beta, float* c, int64_t ldc, uint64_t stream,
    uint32_t path) {
  if (!valid_args(op_a, op_b, m, n, k, a, lda, b, ldb, c, ldc, path))
    return XVRAM_STATUS_INVALID_ARGUMENT;
  if (m == 0 || n == 0)
    return XVRAM_STATUS_SUCCESS;
  const int oa = static_cast<int>(op_a), ob = static_cast<int>(op_b);
  const int mi = static_cast<int>(m), ni = static_cast<int>(n), ki = static_cast<int>(k);
  cudaStream_t s = as_stream(stream);
  if (path == XVRAM_B200_PATH_TF32X3 && k > 0) {
    const uint64_t tneed = sgemm_tf32x3_workspace_bytes(mi, ni, ki);
    int dev = 0;
    cudaMemPool_t pool = cudaGetDevice(&dev) == cudaSuccess ? scratch_pool(dev) : nullptr;
    void* ws = nullptr;
    if (!pool || cudaMallocFromPoolAsync(&ws, tneed, pool, s) != cudaSuccess) {
      cudaGetLastError();
      return XVRAM_STATUS_DEVICE_OUT_OF_MEMORY;
    }
    const cudaError_t e =
        sgemm_tf32x3(oa, ob, mi, ni, ki, alpha, a, lda, b, ldb, beta, c, ldc, ws, tneed, s);
    const cudaError_t f = cudaFreeAsync(ws, s);
    return from_cuda(e != cudaSuccess ? e : f);
  }
  const uint64_t need = sgemm_workspace_bytes(oa, ob, mi, ni, ki);
  if (need && path != XVRAM_B200_PATH_GENERIC && sgemm_tma_eligible(oa, ob, a, lda, b, ldb)) {
    int dev = 0;
    cudaMemPool_t pool = cudaGetDevice(&dev) == cudaSuccess ? scratch_pool(dev) : nullptr;
    void* ws = nullptr;
    if (pool && cudaMallocFromPoolAsync(&ws, need, pool, s) == cudaSuccess) {
      const cudaError_t e = sgemm_ffma_ws(oa, ob, mi, ni, ki, alpha, a, lda, b, ldb, beta, c, ldc,
                                          ws, need, s, to_path(path));
      const cudaError_t f = cudaFreeAsync(ws, s);
      return from_cuda(e != cudaSuccess ? e : f);
    }
    cudaGetLastError(); // no scratch: run the K-major kernel directly
  }
  return from_cuda(sgemm_ffma(oa, ob, mi, ni, ki, alpha, a, lda, b, ldb, beta, c, ldc, s,
                              to_path(path)));
}

XVRAM_B200_API uint64_t XVRAM_CALL xvram_b200_sgemm_workspace_bytes(uint32_t op_a, uint32_t op_b,
                                                                    int64_t m, int64_t n,
                                                                    int64_t k) {
  const bool tf32x3 = (op_a & XVRAM_B200_WORKSPACE_TF32X3) != 0;
  op_a &= ~XVRAM_B200_WORKSPACE_TF32X3;
  if (op_a > 1 || op_b > 1 || m <= 0 || n <= 0 || k <= 0 || m > INT32_MAX || n > INT32_MAX ||
      k > INT32_MAX)
    return 0;
  if (tf32x3)
    return sgemm_tf32x3_workspace_bytes(static_cast<int>(m), static_cast<int>(n),
                                        static_cast<int>(k));
  return sgemm_workspace_bytes(static_cast<int>(op_a), static_cast<int>(op_b),
                               static_cast<int>(m), static_cast<int>(n), static_cast<int>(k));
}

XVRAM_B200_API xvram_status XVRAM_CALL xvram_b200_sgemm_tile_shape(int64_t m, int64_t n,
                                                                 int32_t* tile_m,
                                                                 int32_t* tile_n) {
  if (m <= 0 || n <= 0 || m > INT32_MAX || n > INT32_MAX || !tile_m || !tile_n)
    return XVRAM_STATUS_INVALID_ARGUMENT;
  int tm = 0, tn = 0;
  sgemm_tile_shape(static_cast<int>(m), static_cast<int>(n), &tm, &tn);
  *tile_m = tm;
  *tile_n = tn;
  return XVRAM_STATUS_SUCCESS;
}

XVRAM_B200_API xvram_status XVRAM_CALL xvram_b200_sgemm_device_ws(
    uint32_t op_a, uint32_t op_b, int64_t m, int64_t n, int64_t k, float alpha, const float* a,
    int64_t lda, const float* b, int64_t ldb, float beta, float* c, int64_t ldc, void* workspace,
    uint64_t workspace_bytes, uint64_t stream, uint32_t path) {
  if (!valid_args(op_a, op_b, m, n, k, a, lda, b, ldb, c, ldc, path))
    return XVRAM_STATUS_INVALID_ARGUMENT;
  if (m == 0 || n == 0)
    return XVRAM_STATUS_SUCCESS;
  if (path == XVRAM_B200_PATH_TF32X3 && k > 0)
    return from_cuda(sgemm_tf32x3(static_cast<int>(op_a), static_cast<int>(op_b),
                                  static_cast<int>(m), static_cast<int>(n), static_cast<int>(k),
                                  alpha, a, lda, b, ldb, beta, c, ldc, workspace, workspace_bytes,
                                  as_stream(stream)));
  return from_cuda(sgemm_ffma_ws(static_cast<int>(op_a), static_cast<int>(op_b),
                                 static_cast<int>(m), static_cast<int>(n), static_cast<int>(k),
                                 alpha, a, lda, b, ldb, beta, c, ldc, workspace, workspace_bytes,
                                 as_stream(stream), to_path(path)));
}

XVRAM_B200_API xvram_status XVRAM_CALL xvram_b200_kernel_status(uint64_t stream, uint32_t* word) {
  if (!word)
    return XVRAM_STATUS_INVALID_ARGUMENT;
  unsigned int w = 0, wt = 0;
  cudaError_t e = read_and_clear_kernel_error(&w, as_stream(stream));
  if (e == cudaSuccess)
    e = read_and_clear_kernel_error_tc(&wt, as_stream(stream));
  *word = w | (wt << 8); // tensor-core kernel bits in the second byte
  return from_cuda(e);
}

XVRAM_B200_API void XVRAM_CALL xvram_b200_fill_uniform(float* dst, uint64_t count, uint64_t seed,
                                                       uint64_t first_index, int32_t threads) {
  if (dst && count)
    fill_uniform(dst, count, seed, first_index, threads);
}

// The reference GEMM bench's 128-bit digest (src/gemm_bench/executor.cpp:42-65): two 64-bit
// lanes over the bytes, each mixed with its absolute offset.  The digest is part of the
// report format (expected and output digests are compared across tools), so its steps are
// the reference's.  state = {low, high}; start from XVRAM_B200_BENCH_DIGEST_INIT.
XVRAM_B200_API void XVRAM_CALL xvram_b200_digest_bench(const void* data, uint64_t len,
                                                       uint64_t absolute_offset,
                                                       uint64_t state[2]) {
  if (!data || !state)
    return;
  const unsigned char* p = static_cast<const unsigned char*>(data);
  uint64_t low = state[0], high = state[1], index = absolute_offset;
  for (uint64_t i = 0; i < len; ++i, ++index) {
    const uint64_t v = p[i];
    low ^= v + (index & 0xFFull);
    low *= 1099511628211ull;
    high ^= v + 0x9Eull + (index >> 8);
    high *= 0x100000001B3ull;
    high ^= high >> 29;
  }
  state[0] = low;
  state[1] = high;
}

// The reference compat bench's digest (src/compat_bench/pattern.cpp Digest::add, state
// pattern.hpp:29-30): per float, its four bytes from the least significant.
// state = {a, b}; start from XVRAM_B200_COMPAT_DIGEST_INIT.
XVRAM_B200_API void XVRAM_CALL xvram_b200_digest_compat(const float* values, uint64_t count,
                                                        uint64_t state[2]) {
  if (!values || !state)
    return;
  uint64_t a = state[0], b = state[1];
  for (uint64_t i = 0; i < count; ++i) {
    uint32_t bits;
    std::memcpy(&bits, values + i, 4);
    for (unsigned shift = 0; shift < 32; shift += 8) {
      const uint64_t byte = (bits >> shift) & 255u;
      a = (a ^ byte) * 1099511628211ull;
      b = (b ^ (byte + 0x9eu)) * 0x100000001b3ull;
      b ^= b >> 29;
    }
  }
  state[0] = a;
  state[1] = b;
}

XVRAM_B200_API xvram_status XVRAM_CALL xvram_b200_plan_panels(
    uint32_t op_a, uint32_t op_b, int64_t m, int64_t n, int64_t k, int32_t beta_nonzero,
    uint64_t budget_bytes, uint64_t quantum_bytes, double flops_per_s, double h2d_bytes_per_s,
    double d2h_bytes_per_s, int64_t force_mb, int64_t force_nb, int64_t force_kb,
    xvram_b200_plan_info_v1* out) {
  if (!out || out->struct_size < sizeof(*out))
    return XVRAM_STATUS_INVALID_ARGUMENT;
  Plan plan;
  const PlanStatus st = plan_for(op_a, op_b, m, n, k, beta_nonzero, budget_bytes, quantum_bytes,
                                 flops_per_s, h2d_bytes_per_s, d2h_bytes_per_s, force_mb,
                                 force_nb, force_kb, &plan);
  const uint32_t size = out->struct_size;
  *out = xvram_b200_plan_info_v1{};
  out->struct_size = size;
  out->status = static_cast<uint32_t>(st);
  if (st != PlanStatus::ok)
    return st == PlanStatus::invalid ? XVRAM_STATUS_INVALID_ARGUMENT : XVRAM_STATUS_BUDGET_PRESSURE;
  out->block_m = plan.mb;
  out->block_n = plan.nb;
  out->panel_k = plan.kb;
  out->n_outer = plan.n_outer ? 1 : 0;
  out->panel_slots = plan.panel_slots;
  out->c_slots = plan.c_slots;
  out->slot_bytes = plan.slot_bytes;
  out->c_slot_bytes = plan.c_slot_bytes;
  out->steps = plan.steps.size();
  out->panel_loads = plan.panel_loads;
  out->panel_hits = plan.panel_hits;
  out->panel_evictions = plan.panel_evictions;
  out->h2d_bytes = plan.h2d_bytes;
  out->d2h_bytes = plan.d2h_bytes;
  out->est_seconds = plan.est_seconds;
  return XVRAM_STATUS_SUCCESS;
}

XVRAM_B200_API xvram_status XVRAM_CALL xvram_b200_plan_steps(
    uint32_t op_a, uint32_t op_b, int64_t m, int64_t n, int64_t k, int32_t beta_nonzero,
    uint64_t budget_bytes, uint64_t quantum_bytes, int64_t force_mb, int64_t force_nb,
    int64_t force_kb, int32_t* out, uint64_t capacity) {
  Plan plan;
  const PlanStatus st = plan_for(op_a, op_b, m, n, k, beta_nonzero, budget_bytes, quantum_bytes,
                                 0, 0, 0, force_mb, force_nb, force_kb, &plan);
  if (st != PlanStatus::ok)
    return st == PlanStatus::invalid ? XVRAM_STATUS_INVALID_ARGUMENT : XVRAM_STATUS_BUDGET_PRESSURE;
  if (!out || capacity < plan.steps.size())
    return XVRAM_STATUS_INVALID_ARGUMENT;
  for (size_t i = 0; i < plan.steps.size(); ++i) {
    const PlanStep& s = plan.steps[i];
    out[5 * i + 0] = s.bm;
    out[5 * i + 1] = s.bn;
    out[5 * i + 2] = s.bk;
    out[5 * i + 3] = s.slot_a;
    out[5 * i + 4] = s.slot_b;
  }
  return XVRAM_STATUS_SUCCESS;
}

XVRAM_B200_API int32_t XVRAM_CALL xvram_b200_validate_gemm(
    uint64_t m, uint64_t n, uint64_t k, uint32_t op_a, uint32_t op_b,
    const uint64_t allocation_ids[3], const uint64_t allocation_bytes[3],
    const uint64_t offsets[3], const uint64_t rows[3], const uint64_t columns[3],
    const uint64_t lds[3], char* operand) {
  GemmShape s;
  s.m = m;
  s.n = n;
  s.k = k;
  s.op_a = static_cast<int>(op_a);
  s.op_b = static_cast<int>(op_b);
  MatrixRef* mats[3] = {&s.a, &s.b, &s.c};
  for (int i = 0; i < 3; ++i) {
    mats[i]->allocation_id = allocation_ids[i];
    mats[i]->allocation_bytes = allocation_bytes[i];
    mats[i]->offset_bytes = offsets[i];
    mats[i]->rows = rows[i];
    mats[i]->columns = columns[i];
    mats[i]->ld = lds[i];
  }
  const Validation v = validate_gemm(s);
  if (operand)
    *operand = v.operand;
  return static_cast<int32_t>(v.error);
}

XVRAM_B200_API int32_t XVRAM_CALL xvram_b200_validate_gemm_typed(
    uint64_t m, uint64_t n, uint64_t k, uint32_t op_a, uint32_t op_b,
    const uint64_t allocation_ids[3], const uint64_t allocation_bytes[3],
    const uint64_t offsets[3], const uint64_t rows[3], const uint64_t columns[3],
    const uint64_t lds[3], const uint32_t data_types[3], int32_t compute, char* operand) {
  GemmShape s;
  s.m = m;
  s.n = n;
  s.k = k;
  s.op_a = static_cast<int>(op_a);
  s.op_b = static_cast<int>(op_b);
  s.compute = compute;
  MatrixRef* mats[3] = {&s.a, &s.b, &s.c};
  for (int i = 0; i < 3; ++i) {
    mats[i]->allocation_id = allocation_ids[i];
    mats[i]->allocation_bytes = allocation_bytes[i];
    mats[i]->offset_bytes = offsets[i];
    mats[i]->rows = rows[i];
    mats[i]->columns = columns[i];
    mats[i]->ld = lds[i];
    mats[i]->dtype = data_types[i];
  }
  const Validation v = validate_gemm(s);
  if (operand)
    *operand = v.operand;
  return static_cast<int32_t>(v.error);
}

XVRAM_B200_API uint64_t XVRAM_CALL xvram_b200_gemm_typed_workspace_bytes(
    uint32_t ab_type, uint32_t c_type, int32_t compute, uint32_t op_a, uint32_t op_b, int64_t m,
    int64_t n, int64_t k) {
  if (op_a > 1 || op_b > 1 || m <= 0 || n <= 0 || k < 0 || m > INT32_MAX || n > INT32_MAX ||
      k > INT32_MAX || !supported_types(ab_type, c_type, compute))
    return 0;
  return gemm_typed_workspace_bytes(ab_type, c_type, compute, static_cast<int>(op_a),
                                    static_cast<int>(op_b), static_cast<int>(m),
                                    static_cast<int>(n), static_cast<int>(k));
}

XVRAM_B200_API xvram_status XVRAM_CALL xvram_b200_gemm_device_typed(
    uint32_t ab_type, uint32_t c_type, int32_t compute, uint32_t op_a, uint32_t op_b, int64_t m,
    int64_t n, int64_t k, double alpha, const void* a, int64_t lda, const void* b, int64_t ldb,
    double beta, void* c, int64_t ldc, void* workspace, uint64_t workspace_bytes,
    uint64_t stream) {
  if (op_a > 1 || op_b > 1 || m < 0 || n < 0 || k < 0 || m > INT32_MAX || n > INT32_MAX ||
      k > INT32_MAX || !supported_types(ab_type, c_type, compute))
    return XVRAM_STATUS_INVALID_ARGUMENT;
  if (m == 0 || n == 0)
    return XVRAM_STATUS_SUCCESS;
  const int64_t a_rows = op_a == 0 ? m : k, b_rows = op_b == 0 ? k : n;
  if (!a || !b || !c || lda < std::max<int64_t>(1, a_rows) || ldb < std::max<int64_t>(1, b_rows) ||
      ldc < m)
    return XVRAM_STATUS_INVALID_ARGUMENT;
  return from_cuda(gemm_typed(ab_type, c_type, compute, static_cast<int>(op_a),
                              static_cast<int>(op_b), static_cast<int>(m), static_cast<int>(n),
                              static_cast<int>(k), alpha, a, lda, b, ldb, beta, c, ldc, workspace,
                              workspace_bytes, as_stream(stream)));
}

XVRAM_B200_API xvram_status XVRAM_CALL xvram_b200_ffma_probe(int32_t blocks, int32_t iterations,
                                                             float* sink, uint64_t stream) {
  if (blocks <= 0 || iterations <= 0 || !sink)
    return XVRAM_STATUS_INVALID_ARGUMENT;
  return from_cuda(ffma_peak_probe(blocks, iterations, sink, as_stream(stream)));
}

XVRAM_B200_API xvram_status XVRAM_CALL xvram_b200_ffma2_probe(int32_t blocks, int32_t iterations,
                                                              float* sink, uint64_t stream) {
  if (blocks <= 0 || iterations <= 0 || !sink)
    return XVRAM_STATUS_INVALID_ARGUMENT;
  return from_cuda(ffma_peak_probe(blocks, iterations, sink, as_stream(stream), true));
}

XVRAM_B200_API xvram_status XVRAM_CALL
xvram_b200_compat_runtime_info(xvram_b200_runtime_info_v1* out) {
  return compat_runtime_info(out);
}

} // extern "C"
