// sharded.cpp -- multi-GPU partitioned SGEMM: C rows split over the GPUs of a group,
// B panels read from the host once per group and all-gathered over NVLink.
//
// The reference is single-GPU (reference src/cuda_compat/adapter.cpp:595-600 rejects any
// other device); this is new capability.  One process (or thread) per GPU calls
// xvram_b200_sgemm_sharded collectively with its own rows of A and C and the whole B in
// host memory.  Per K panel each rank
//   1. copies its A panel and a 1/P slice of the B panel from pinned host memory
//      (pitched 2D copies on the H2D stream, double-buffered),
//   2. completes the B panel with an in-place NCCL all-gather on the collective stream
//      (each rank's slice is one contiguous block of the packed panel),
//   3. runs the sm_100a kernel on the compute stream, beta applied on the first panel,
// so the copies and the all-gather of panel p+1 overlap the kernel of panel p.  C is
// copied in once (beta != 0) and out once.  Kernels only read local HBM; nothing loads
// from a peer's memory, and every TMA load targets only the issuing CTA.
//
// NCCL is loaded at run time (dlopen of libnccl.so.2, whichever the process already has),
// so the library keeps no link-time NCCL dependency.  Communicator creation is
// non-blocking with a deadline, and every host wait on a collective is bounded: a peer
// that never arrives produces TIMEOUT and an aborted communicator, not a hang.
#include "xvram_b200.h"

#include "kernels.hpp"

#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <chrono>
#include <cstring>
#include <mutex>
#include <thread>

namespace {

struct NcclApi {
  decltype(&ncclGetUniqueId) get_unique_id = nullptr;
  decltype(&ncclCommInitRankConfig) init_rank_config = nullptr;
  decltype(&ncclCommGetAsyncError) async_error = nullptr;
  decltype(&ncclCommAbort) abort = nullptr;
  decltype(&ncclCommDestroy) destroy = nullptr;
  decltype(&ncclAllGather) all_gather = nullptr;
  bool ok = false;
};

const NcclApi& nccl() {
  static const NcclApi api = [] {
    NcclApi a;
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h)
      return a;
    auto sym = [h](const char* n) { return dlsym(h, n); };
    a.get_unique_id = reinterpret_cast<decltype(a.get_unique_id)>(sym("ncclGetUniqueId"));
    a.init_rank_config =
        reinterpret_cast<decltype(a.init_rank_config)>(sym("ncclCommInitRankConfig"));
    a.async_error = reinterpret_cast<decltype(a.async_error)>(sym("ncclCommGetAsyncError"));
    a.abort = reinterpret_cast<decltype(a.abort)>(sym("ncclCommAbort"));
    a.destroy = reinterpret_cast<decltype(a.destroy)>(sym("ncclCommDestroy"));
    a.all_gather = reinterpret_cast<decltype(a.all_gather)>(sym("ncclAllGather"));
    a.ok = a.get_unique_id && a.init_rank_config && a.async_error && a.abort && a.destroy &&
           a.all_gather;
    return a;
  }();
  return api;
}

constexpr double kInitTimeoutS = 120.0;
constexpr double kWaitTimeoutS = 60.0;

struct Buffer {
  void* p = nullptr;
  size_t bytes = 0;
  cudaError_t ensure(size_t want) {
    if (bytes >= want)
      return cudaSuccess;
    if (p)
      cudaFree(p);
    p = nullptr;
    bytes = 0;
    const cudaError_t e = cudaMalloc(&p, want);
    if (e == cudaSuccess)
      bytes = want;
    return e;
  }
  void release() {
    if (p)
      cudaFree(p);
    p = nullptr;
    bytes = 0;
  }
};

struct ShardGroup {
  ncclComm_t comm = nullptr;
  int rank = 0, world = 1, device = 0;
  cudaStream_t h2d = nullptr, coll = nullptr, comp = nullptr, d2h = nullptr;
  cudaEvent_t loaded[2] = {}, gathered[2] = {}, consumed[2] = {}, c_in = nullptr, done = nullptr,
              out = nullptr;
  Buffer a_slot[2], b_slot[2], c_buf, ws;
  bool aborted = false;
  std::mutex mu;
};

uint64_t up(uint64_t v, uint64_t q) { return (v + q - 1) / q * q; }

xvram_status cuda_status(cudaError_t e) {
  if (e == cudaSuccess)
    return XVRAM_STATUS_SUCCESS;
  return e == cudaErrorMemoryAllocation ? XVRAM_STATUS_DEVICE_OUT_OF_MEMORY
                                        : XVRAM_STATUS_CUDA_ERROR;
}

// Waits for `e` with a deadline, watching the communicator for asynchronous errors.
xvram_status bounded_wait(ShardGroup& g, cudaEvent_t e) {
  const auto start = std::chrono::steady_clock::now();
  for (;;) {
    const cudaError_t q = cudaEventQuery(e);
    if (q == cudaSuccess)
      return XVRAM_STATUS_SUCCESS;
    if (q != cudaErrorNotReady)
      return XVRAM_STATUS_CUDA_ERROR;
    ncclResult_t ar = ncclSuccess;
    if (g.comm && nccl().async_error(g.comm, &ar) == ncclSuccess && ar != ncclSuccess &&
        ar != ncclInProgress) {
      nccl().abort(g.comm);
      g.comm = nullptr;
      g.aborted = true;
      return XVRAM_STATUS_CUDA_ERROR;
    }
    if (std::chrono::duration<double>(std::chrono::steady_clock::now() - start).count() >
        kWaitTimeoutS) {
      if (g.comm)
        nccl().abort(g.comm);
      g.comm = nullptr;
      g.aborted = true;
      return XVRAM_STATUS_TIMEOUT;
    }
    std::this_thread::sleep_for(std::chrono::microseconds(50));
  }
}

void destroy_group(ShardGroup* g) {
  if (!g)
    return;
  int saved = 0;
  cudaGetDevice(&saved);
  cudaSetDevice(g->device);
  for (auto* s : {g->h2d, g->coll, g->comp, g->d2h})
    if (s) {
      cudaStreamSynchronize(s);
      cudaStreamDestroy(s);
    }
  for (auto* arr : {g->loaded, g->gathered, g->consumed})
    for (int i = 0; i < 2; ++i)
      if (arr[i])
        cudaEventDestroy(arr[i]);
  for (auto* e : {g->c_in, g->done, g->out})
    if (e)
      cudaEventDestroy(e);
  for (int i = 0; i < 2; ++i) {
    g->a_slot[i].release();
    g->b_slot[i].release();
  }
  g->c_buf.release();
  g->ws.release();
  if (g->comm)
    nccl().destroy(g->comm);
  cudaSetDevice(saved);
  delete g;
}

} // namespace

extern "C" {

XVRAM_B200_API xvram_status XVRAM_CALL xvram_b200_shard_unique_id(void* out, uint64_t bytes) {
  if (!out || bytes < NCCL_UNIQUE_ID_BYTES)
    return XVRAM_STATUS_INVALID_ARGUMENT;
  if (!nccl().ok)
    return XVRAM_STATUS_UNAVAILABLE;
  ncclUniqueId id;
  if (nccl().get_unique_id(&id) != ncclSuccess)
    return XVRAM_STATUS_UNAVAILABLE;
  std::memcpy(out, &id, NCCL_UNIQUE_ID_BYTES);
  return XVRAM_STATUS_SUCCESS;
}

XVRAM_B200_API xvram_status XVRAM_CALL xvram_b200_shard_group_create(const void* unique_id,
                                                                   uint64_t bytes, int32_t rank,
                                                                   int32_t world,
                                                                   uint64_t* out_group) {
  if (!unique_id || bytes < NCCL_UNIQUE_ID_BYTES || !out_group || world < 1 || rank < 0 ||
      rank >= world)
    return XVRAM_STATUS_INVALID_ARGUMENT;
  if (!nccl().ok)
    return XVRAM_STATUS_UNAVAILABLE;
  auto* g = new ShardGroup;
  g->rank = rank;
  g->world = world;
  if (cudaGetDevice(&g->device) != cudaSuccess) {
    delete g;
    return XVRAM_STATUS_CUDA_ERROR;
  }
  cudaError_t e = cudaSuccess;
  for (auto* s : {&g->h2d, &g->coll, &g->comp, &g->d2h})
    if (e == cudaSuccess)
      e = cudaStreamCreateWithFlags(s, cudaStreamNonBlocking);
  for (auto* arr : {g->loaded, g->gathered, g->consumed})
    for (int i = 0; i < 2; ++i)
      if (e == cudaSuccess)
        e = cudaEventCreateWithFlags(&arr[i], cudaEventDisableTiming);
  for (auto* ev : {&g->c_in, &g->done, &g->out})
    if (e == cudaSuccess)
      e = cudaEventCreateWithFlags(ev, cudaEventDisableTiming);
  if (e != cudaSuccess) {
    destroy_group(g);
    return XVRAM_STATUS_CUDA_ERROR;
  }
  ncclUniqueId id;
  std::memcpy(&id, unique_id, NCCL_UNIQUE_ID_BYTES);
  ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
  cfg.blocking = 0;
  ncclResult_t r = nccl().init_rank_config(&g->comm, world, id, rank, &cfg);
  const auto start = std::chrono::steady_clock::now();
  while (r == ncclInProgress || r == ncclSuccess) {
    ncclResult_t state = ncclSuccess;
    if (nccl().async_error(g->comm, &state) != ncclSuccess) {
      r = ncclInternalError;
      break;
    }
    if (state != ncclInProgress) {
      r = state;
      break;
    }
    if (std::chrono::duration<double>(std::chrono::steady_clock::now() - start).count() >
        kInitTimeoutS) {
      r = ncclInternalError;
      break;
    }
    std::this_thread::sleep_for(std::chrono::milliseconds(1));
  }
  if (r != ncclSuccess) {
    if (g->comm)
      nccl().abort(g->comm);
    g->comm = nullptr;
    destroy_group(g);
    return XVRAM_STATUS_UNAVAILABLE;
  }
  *out_group = reinterpret_cast<uint64_t>(g);
  return XVRAM_STATUS_SUCCESS;
}

XVRAM_B200_API xvram_status XVRAM_CALL xvram_b200_shard_group_destroy(uint64_t group) {
  destroy_group(reinterpret_cast<ShardGroup*>(group));
  return XVRAM_STATUS_SUCCESS;
}

XVRAM_B200_API xvram_status XVRAM_CALL xvram_b200_sgemm_sharded(
    uint64_t group, uint32_t op_a, uint32_t op_b, int64_t m_local, int64_t n, int64_t k,
    float alpha, const float* a, int64_t lda, const float* b, int64_t ldb, float beta, float* c,
    int64_t ldc, int64_t panel_k) {
  auto* g = reinterpret_cast<ShardGroup*>(group);
  if (!g || op_a > 1 || op_b > 1 || m_local < 0 || n <= 0 || k <= 0 || m_local > INT32_MAX ||
      n > INT32_MAX || k > INT32_MAX || !b || ldb < (op_b == 0 ? k : n) ||
      (m_local > 0 && (!a || !c || lda < (op_a == 0 ? m_local : k) || ldc < m_local)))
    return XVRAM_STATUS_INVALID_ARGUMENT;
  std::lock_guard<std::mutex> lock(g->mu);
  if (g->aborted || !g->comm)
    return XVRAM_STATUS_POISONED;
  int saved = 0;
  cudaGetDevice(&saved);
  cudaSetDevice(g->device);
  struct Restore {
    int d;
    ~Restore() { cudaSetDevice(d); }
  } restore{saved};

  const int P = g->world, r = g->rank;
  const uint64_t M = static_cast<uint64_t>(m_local), Nn = static_cast<uint64_t>(n),
                 K = static_cast<uint64_t>(k);
  const uint64_t kb = panel_k > 0 ? up(static_cast<uint64_t>(panel_k), 32) : std::min<uint64_t>(up(K, 32), 1024);
  const uint64_t panels = (K + kb - 1) / kb;
  // Packed panel layouts (all leading dimensions multiples of 4 floats for TMA).
  const uint64_t lda_p = op_a == 0 ? up(std::max<uint64_t>(M, 1), 4) : kb;  // A: M x kb or kb x M
  const uint64_t a_bytes = (op_a == 0 ? lda_p * kb : kb * std::max<uint64_t>(M, 1)) * 4;
  // B op N: kb x n, ld kb, sliced by columns; B op T: n x kb, ld up4(n), sliced by k.
  const uint64_t w_cols = (Nn + P - 1) / P;               // columns per rank (op N)
  const uint64_t w_k = (kb + P - 1) / P;                  // panel k per rank (op T)
  const uint64_t ldb_p = op_b == 0 ? kb : up(Nn, 4);
  const uint64_t slice_elems = op_b == 0 ? w_cols * kb : w_k * ldb_p;
  const uint64_t b_bytes = slice_elems * static_cast<uint64_t>(P) * 4;
  const uint64_t ldc_p = up(std::max<uint64_t>(M, 1), 4);
  const uint64_t ws_need = xvram::sgemm_workspace_bytes(static_cast<int>(op_a),
                                                        static_cast<int>(op_b),
                                                        static_cast<int>(std::max<uint64_t>(M, 1)),
                                                        static_cast<int>(Nn), static_cast<int>(kb));
  cudaError_t e = cudaSuccess;
  for (int i = 0; i < 2 && e == cudaSuccess; ++i) {
    e = g->a_slot[i].ensure(a_bytes);
    if (e == cudaSuccess)
      e = g->b_slot[i].ensure(b_bytes);
  }
  if (e == cudaSuccess)
    e = g->c_buf.ensure(ldc_p * Nn * 4);
  if (e == cudaSuccess && ws_need)
    e = g->ws.ensure(ws_need);
  if (e != cudaSuccess)
    return cuda_status(e);

  const char* ah = reinterpret_cast<const char*>(a);
  const char* bh = reinterpret_cast<const char*>(b);
  char* ch = reinterpret_cast<char*>(c);
  float* cdev = static_cast<float*>(g->c_buf.p);
  if (M > 0 && beta != 0.0f) {
    e = cudaMemcpy2DAsync(cdev, ldc_p * 4, ch, static_cast<size_t>(ldc) * 4, M * 4, Nn,
                          cudaMemcpyHostToDevice, g->h2d);
    if (e == cudaSuccess)
      e = cudaEventRecord(g->c_in, g->h2d);
    if (e == cudaSuccess)
      e = cudaStreamWaitEvent(g->comp, g->c_in, 0);
  }
  for (uint64_t p = 0; p < panels && e == cudaSuccess; ++p) {
    const int s = static_cast<int>(p & 1);
    const uint64_t k0 = p * kb, kr = std::min<uint64_t>(kb, K - k0);
    if (p >= 2)
      e = cudaStreamWaitEvent(g->h2d, g->consumed[s], 0);
    // 1a. this rank's A panel
    char* ad = static_cast<char*>(g->a_slot[s].p);
    if (e == cudaSuccess && M > 0) {
      if (op_a == 0) // A_local is M x k: kr columns of M floats
        e = cudaMemcpy2DAsync(ad, lda_p * 4, ah + k0 * static_cast<uint64_t>(lda) * 4,
                              static_cast<size_t>(lda) * 4, M * 4, kr, cudaMemcpyHostToDevice,
                              g->h2d);
      else // A_local is k x M: M columns of kr floats
        e = cudaMemcpy2DAsync(ad, kb * 4, ah + k0 * 4, static_cast<size_t>(lda) * 4, kr * 4, M,
                              cudaMemcpyHostToDevice, g->h2d);
    }
    // 1b. this rank's slice of the B panel, straight into its place in the packed panel
    char* bd = static_cast<char*>(g->b_slot[s].p);
    if (e == cudaSuccess) {
      if (op_b == 0) {
        const uint64_t c0 = static_cast<uint64_t>(r) * w_cols;
        const uint64_t cols = c0 < Nn ? std::min<uint64_t>(w_cols, Nn - c0) : 0;
        if (cols)
          e = cudaMemcpy2DAsync(bd + c0 * kb * 4, kb * 4,
                                bh + (k0 + c0 * static_cast<uint64_t>(ldb)) * 4,
                                static_cast<size_t>(ldb) * 4, kr * 4, cols,
                                cudaMemcpyHostToDevice, g->h2d);
      } else {
        const uint64_t q0 = static_cast<uint64_t>(r) * w_k;
        const uint64_t ks = q0 < kr ? std::min<uint64_t>(w_k, kr - q0) : 0;
        if (ks)
          e = cudaMemcpy2DAsync(bd + q0 * ldb_p * 4, ldb_p * 4,
                                bh + (k0 + q0) * static_cast<uint64_t>(ldb) * 4,
                                static_cast<size_t>(ldb) * 4, Nn * 4, ks, cudaMemcpyHostToDevice,
                                g->h2d);
      }
    }
    if (e == cudaSuccess)
      e = cudaEventRecord(g->loaded[s], g->h2d);
    // 2. complete the panel over NVLink: in-place all-gather of the P slices
    if (e == cudaSuccess)
      e = cudaStreamWaitEvent(g->coll, g->loaded[s], 0);
    if (e == cudaSuccess && P > 1) {
      const ncclResult_t nr = nccl().all_gather(bd + static_cast<uint64_t>(r) * slice_elems * 4,
                                                bd, slice_elems, ncclFloat, g->comm, g->coll);
      if (nr != ncclSuccess && nr != ncclInProgress) {
        g->aborted = true;
        return XVRAM_STATUS_CUDA_ERROR;
      }
      // A non-blocking communicator may still be enqueueing the call: wait (bounded)
      // until it has been issued before the next NCCL call.
      if (nr == ncclInProgress) {
        const auto t0 = std::chrono::steady_clock::now();
        ncclResult_t st = ncclInProgress;
        while (st == ncclInProgress) {
          if (nccl().async_error(g->comm, &st) != ncclSuccess ||
              std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count() >
                  kWaitTimeoutS) {
            st = ncclInternalError;
            break;
          }
        }
        if (st != ncclSuccess) {
          nccl().abort(g->comm);
          g->comm = nullptr;
          g->aborted = true;
          return XVRAM_STATUS_TIMEOUT;
        }
      }
    }
    if (e == cudaSuccess)
      e = cudaEventRecord(g->gathered[s], g->coll);
    // 3. contract
    if (e == cudaSuccess)
      e = cudaStreamWaitEvent(g->comp, g->gathered[s], 0);
    if (e == cudaSuccess && M > 0)
      e = xvram::sgemm_ffma_ws(static_cast<int>(op_a), static_cast<int>(op_b),
                               static_cast<int>(M), static_cast<int>(Nn), static_cast<int>(kr),
                               alpha, reinterpret_cast<const float*>(ad),
                               static_cast<long long>(op_a == 0 ? lda_p : kb),
                               reinterpret_cast<const float*>(bd), static_cast<long long>(ldb_p),
                               p == 0 ? beta : 1.0f, cdev, static_cast<long long>(ldc_p),
                               g->ws.p, g->ws.bytes, g->comp);
    if (e == cudaSuccess)
      e = cudaEventRecord(g->consumed[s], g->comp);
  }
  if (e == cudaSuccess)
    e = cudaEventRecord(g->done, g->comp);
  if (e == cudaSuccess && M > 0) {
    e = cudaStreamWaitEvent(g->d2h, g->done, 0);
    if (e == cudaSuccess)
      e = cudaMemcpy2DAsync(ch, static_cast<size_t>(ldc) * 4, cdev, ldc_p * 4, M * 4, Nn,
                            cudaMemcpyDeviceToHost, g->d2h);
  }
  if (e == cudaSuccess)
    e = cudaEventRecord(g->out, g->d2h);
  if (e != cudaSuccess) {
    g->aborted = true;
    return cuda_status(e);
  }
  xvram_status st = bounded_wait(*g, g->out);
  if (st == XVRAM_STATUS_SUCCESS) {
    unsigned int word = 0;
    if (xvram::read_and_clear_kernel_error(&word, g->comp) != cudaSuccess)
      st = XVRAM_STATUS_CUDA_ERROR;
    else if (word)
      st = XVRAM_STATUS_TIMEOUT;
  }
  if (st != XVRAM_STATUS_SUCCESS)
    g->aborted = true;
  return st;
}

} // extern "C"
