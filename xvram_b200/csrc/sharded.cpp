// sharded.cpp -- multi-GPU partitioned SGEMM: C rows split over the GPUs of a group,
// B read from the host once per group and all-gathered over NVLink.
//
// The reference is single-GPU (reference src/cuda_compat/adapter.cpp:595-600 rejects any
// other device); this is new capability.  One process (or thread) per GPU calls
// xvram_b200_sgemm_sharded collectively with its own rows of A and C and the whole B in
// host memory.  Per call:
//   * the ranks agree on one plan with a tiny NCCL all-reduce (largest row count, smallest
//     free device memory), so every rank issues the same collectives even when their row
//     counts or free memory differ;
//   * this rank's rows of A are made resident in HBM in row groups that fit the agreed
//     budget (normally one group), arriving in K panels so the first kernel starts after
//     the first panel; K-major A is transposed once, on arrival, into the M-major form;
//   * C is processed in column blocks (double-buffered): for block j each rank copies a
//     1/P slice of B's block from pinned host memory, the slices are all-gathered in place
//     on a collective stream (K-major B is then transposed to N-major once), C's block
//     comes in on the H2D stream (beta != 0), one kernel contracts the full K, and the
//     block goes back on the D2H stream -- so the copies of block j+1, the write-back of
//     block j-1 and the all-gather overlap block j's kernel;
//   * blocks alternate between two compute streams so the last wave of one block's
//     kernel overlaps the first wave of the next.
// Kernels only read local HBM; nothing loads from a peer's memory, and every TMA load
// targets only the issuing CTA.
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

#include <algorithm>
#include <chrono>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <thread>
#include <vector>

namespace {

struct NcclApi {
  decltype(&ncclGetUniqueId) get_unique_id = nullptr;
  decltype(&ncclCommInitRankConfig) init_rank_config = nullptr;
  decltype(&ncclCommGetAsyncError) async_error = nullptr;
  decltype(&ncclCommAbort) abort = nullptr;
  decltype(&ncclCommDestroy) destroy = nullptr;
  decltype(&ncclAllGather) all_gather = nullptr;
  decltype(&ncclAllReduce) all_reduce = nullptr;
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
    a.all_reduce = reinterpret_cast<decltype(a.all_reduce)>(sym("ncclAllReduce"));
    a.ok = a.get_unique_id && a.init_rank_config && a.async_error && a.abort && a.destroy &&
           a.all_gather && a.all_reduce;
    return a;
  }();
  return api;
}

constexpr double kInitTimeoutS = 120.0;
constexpr double kWaitTimeoutS = 60.0;
constexpr uint64_t kHeadroomBytes = 1ull << 30; // left free on the device for everything else
constexpr uint64_t kDefaultBlockN = 1024;       // C block width (columns)
constexpr uint64_t kTileM = 128;                // row granularity of a row group
// B and C block buffers in flight: block j+2's copies may start while block j's
// write-back is still running.
constexpr int kSlots = 3;

struct Buffer {
  void* p = nullptr;
  size_t bytes = 0;
  cudaError_t ensure(size_t want) {
    if (bytes >= want)
      return cudaSuccess;
    release();
    const cudaError_t e = cudaMalloc(&p, want);
    if (e == cudaSuccess)
      bytes = want;
    else
      p = nullptr;
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
  cudaStream_t h2d = nullptr, coll = nullptr, comp[2] = {}, d2h = nullptr;
  // Per double-buffer slot: B block copied / gathered (and canonical) / no longer read;
  // C block copied in / computed / copied out.
  cudaEvent_t b_loaded[kSlots] = {}, b_ready[kSlots] = {}, b_free[kSlots] = {};
  cudaEvent_t c_loaded[kSlots] = {}, c_done[kSlots] = {}, c_free[kSlots] = {};
  // A raw panel slot reusable (K-major A), all of A canonical, end of a row group per
  // compute stream, end of the call, plan exchange done.
  cudaEvent_t a_free[2] = {}, a_all = nullptr, group_end[2] = {}, out = nullptr,
              plan_ev = nullptr;
  std::vector<cudaEvent_t> a_ev; // one per A panel: panel p resident (and canonical)
  Buffer a_canon, a_raw[2], b_raw[kSlots], b_canon[kSlots], c_blk[kSlots], plan_dev;
  uint64_t* plan_host = nullptr; // 2 x u64, page-locked
  bool aborted = false;
  std::mutex mu;
  // Device memory this group may use (free + its own buffers), as sampled for the last
  // call, with that call's shape: a repeat of the same shape within a second reuses it
  // instead of calling cudaMemGetInfo, whose latency now and then reaches milliseconds.
  uint64_t avail_sampled = 0;
  uint64_t shape_sampled[6] = {};
  std::chrono::steady_clock::time_point when_sampled{};

  static constexpr int kBuffers = 3 + 3 * kSlots + 1;
  Buffer* buffers[kBuffers] = {&a_canon,    &a_raw[0],   &a_raw[1],   &b_raw[0], &b_raw[1],
                               &b_raw[2],   &b_canon[0], &b_canon[1], &b_canon[2],
                               &c_blk[0],   &c_blk[1],   &c_blk[2],   &plan_dev};
  uint64_t held_bytes() const {
    uint64_t n = 0;
    for (const Buffer* b : buffers)
      n += b->bytes;
    return n;
  }
};

uint64_t up(uint64_t v, uint64_t q) { return (v + q - 1) / q * q; }
uint64_t up4(uint64_t v) { return up(v, 4); }

uint64_t env_u64(const char* name, uint64_t fallback) {
  const char* v = std::getenv(name);
  if (!v || !*v)
    return fallback;
  char* end = nullptr;
  const unsigned long long x = std::strtoull(v, &end, 10);
  return (end && *end == '\0' && x > 0) ? static_cast<uint64_t>(x) : fallback;
}

xvram_status cuda_status(cudaError_t e) {
  if (e == cudaSuccess)
    return XVRAM_STATUS_SUCCESS;
  return e == cudaErrorMemoryAllocation ? XVRAM_STATUS_DEVICE_OUT_OF_MEMORY
                                        : XVRAM_STATUS_CUDA_ERROR;
}

void abort_group(ShardGroup& g) {
  if (g.comm)
    nccl().abort(g.comm);
  g.comm = nullptr;
  g.aborted = true;
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
      abort_group(g);
      return XVRAM_STATUS_CUDA_ERROR;
    }
    if (std::chrono::duration<double>(std::chrono::steady_clock::now() - start).count() >
        kWaitTimeoutS) {
      abort_group(g);
      return XVRAM_STATUS_TIMEOUT;
    }
    std::this_thread::sleep_for(std::chrono::microseconds(50));
  }
}

// A non-blocking communicator may return ncclInProgress while it is still enqueueing a
// call: wait (bounded) until the call has been issued before the next NCCL call.
xvram_status nccl_issued(ShardGroup& g, ncclResult_t nr) {
  if (nr == ncclSuccess)
    return XVRAM_STATUS_SUCCESS;
  if (nr != ncclInProgress) {
    abort_group(g);
    return XVRAM_STATUS_CUDA_ERROR;
  }
  const auto t0 = std::chrono::steady_clock::now();
  ncclResult_t st = ncclInProgress;
  while (st == ncclInProgress) {
    if (nccl().async_error(g.comm, &st) != ncclSuccess ||
        std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count() >
            kWaitTimeoutS) {
      st = ncclInternalError;
      break;
    }
  }
  if (st != ncclSuccess) {
    abort_group(g);
    return XVRAM_STATUS_TIMEOUT;
  }
  return XVRAM_STATUS_SUCCESS;
}

void destroy_group(ShardGroup* g) {
  if (!g)
    return;
  int saved = 0;
  cudaGetDevice(&saved);
  cudaSetDevice(g->device);
  for (auto* s : {g->h2d, g->coll, g->comp[0], g->comp[1], g->d2h})
    if (s) {
      cudaStreamSynchronize(s);
      cudaStreamDestroy(s);
    }
  for (auto* arr : {g->b_loaded, g->b_ready, g->b_free, g->c_loaded, g->c_done, g->c_free})
    for (int i = 0; i < kSlots; ++i)
      if (arr[i])
        cudaEventDestroy(arr[i]);
  for (auto* arr : {g->a_free, g->group_end})
    for (int i = 0; i < 2; ++i)
      if (arr[i])
        cudaEventDestroy(arr[i]);
  for (auto* e : {g->a_all, g->out, g->plan_ev})
    if (e)
      cudaEventDestroy(e);
  for (cudaEvent_t e : g->a_ev)
    cudaEventDestroy(e);
  for (Buffer* b : g->buffers)
    b->release();
  if (g->plan_host)
    cudaFreeHost(g->plan_host);
  if (g->comm)
    nccl().destroy(g->comm);
  cudaSetDevice(saved);
  delete g;
}

// The geometry every rank derives from the same agreed numbers.
struct Plan {
  uint64_t groups = 0; // row groups (0: nothing to do on any rank)
  uint64_t mg = 0;     // rows per group
  uint64_t nb = 0;     // C block width
  uint64_t kb = 0;     // A panel depth
  uint64_t ldk = 0, ldn = 0, ldm = 0; // packed leading dimensions (K-major B raw, N, M)
  uint64_t wc = 0, wk = 0;            // per-rank B slice: columns (op N) or k (op T)
  uint64_t slice_elems = 0;
  uint64_t bytes_a_canon = 0, bytes_a_raw = 0, bytes_b_raw = 0, bytes_b_canon = 0,
           bytes_c = 0;
};

// Sizes the buffers for `mg` rows per group.
void size_plan(Plan& pl, uint32_t op_a, uint32_t op_b, uint64_t n, uint64_t k, int P) {
  pl.ldm = up4(std::max<uint64_t>(pl.mg, 1));
  pl.bytes_a_canon = pl.ldm * k * 4;
  pl.bytes_a_raw = op_a != 0 ? up4(pl.kb) * std::max<uint64_t>(pl.mg, 1) * 4 : 0;
  pl.bytes_c = pl.ldm * pl.nb * 4;
  if (op_b == 0) {
    pl.wc = (pl.nb + P - 1) / P;
    pl.slice_elems = pl.wc * pl.ldk;
    pl.bytes_b_raw = pl.slice_elems * static_cast<uint64_t>(P) * 4;
    pl.bytes_b_canon = pl.ldn * k * 4;
  } else {
    pl.wk = (k + P - 1) / P;
    pl.slice_elems = pl.wk * pl.ldn;
    pl.bytes_b_raw = 0;
    pl.bytes_b_canon = pl.slice_elems * static_cast<uint64_t>(P) * 4;
  }
  (void)n;
}

uint64_t plan_bytes(const Plan& pl) {
  return pl.bytes_a_canon + 2 * pl.bytes_a_raw +
         kSlots * (pl.bytes_b_raw + pl.bytes_b_canon + pl.bytes_c);
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
  for (auto* s : {&g->h2d, &g->coll, &g->comp[0], &g->comp[1], &g->d2h})
    if (e == cudaSuccess)
      e = cudaStreamCreateWithFlags(s, cudaStreamNonBlocking);
  for (auto* arr : {g->b_loaded, g->b_ready, g->b_free, g->c_loaded, g->c_done, g->c_free})
    for (int i = 0; i < kSlots; ++i)
      if (e == cudaSuccess)
        e = cudaEventCreateWithFlags(&arr[i], cudaEventDisableTiming);
  for (auto* arr : {g->a_free, g->group_end})
    for (int i = 0; i < 2; ++i)
      if (e == cudaSuccess)
        e = cudaEventCreateWithFlags(&arr[i], cudaEventDisableTiming);
  for (auto* ev : {&g->a_all, &g->out, &g->plan_ev})
    if (e == cudaSuccess)
      e = cudaEventCreateWithFlags(ev, cudaEventDisableTiming);
  if (e == cudaSuccess)
    e = cudaHostAlloc(reinterpret_cast<void**>(&g->plan_host), 2 * sizeof(uint64_t),
                      cudaHostAllocDefault);
  if (e == cudaSuccess)
    e = g->plan_dev.ensure(256);
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

XVRAM_B200_API xvram_status XVRAM_CALL xvram_b200_shard_allgather_rows(
    uint64_t group, const float* block, int64_t rows, int64_t cols, int64_t ld_block, float* dst,
    int64_t ld_dst, void* staging, uint64_t staging_bytes, uint64_t stream) {
  auto* g = reinterpret_cast<ShardGroup*>(group);
  if (!g || !block || !dst || !staging || rows <= 0 || cols <= 0 || ld_block < rows ||
      ld_dst < rows * g->world)
    return XVRAM_STATUS_INVALID_ARGUMENT;
  const uint64_t per_rank = static_cast<uint64_t>(rows) * static_cast<uint64_t>(cols);
  if (staging_bytes < per_rank * 4 * static_cast<uint64_t>(g->world))
    return XVRAM_STATUS_INVALID_ARGUMENT;
  if (g->aborted)
    return XVRAM_STATUS_POISONED;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  float* stage = static_cast<float*>(staging);
  float* mine = stage + per_rank * static_cast<uint64_t>(g->rank);
  // 1. this rank's block, packed (ld = rows) into its slot of the staging buffer
  cudaError_t e = cudaMemcpy2DAsync(mine, static_cast<size_t>(rows) * 4, block,
                                    static_cast<size_t>(ld_block) * 4,
                                    static_cast<size_t>(rows) * 4, static_cast<size_t>(cols),
                                    cudaMemcpyDeviceToDevice, s);
  if (e != cudaSuccess)
    return XVRAM_STATUS_CUDA_ERROR;
  // 2. every rank's block into every rank's staging buffer (in place)
  if (g->world > 1)
    if (xvram_status st = nccl_issued(*g, nccl().all_gather(mine, stage, per_rank, ncclFloat,
                                                            g->comm, s));
        st != XVRAM_STATUS_SUCCESS)
      return st;
  // 3. block q becomes rows [q rows, (q + 1) rows) of dst
  for (int q = 0; q < g->world; ++q) {
    e = cudaMemcpy2DAsync(dst + static_cast<uint64_t>(q) * static_cast<uint64_t>(rows),
                          static_cast<size_t>(ld_dst) * 4, stage + per_rank * q,
                          static_cast<size_t>(rows) * 4, static_cast<size_t>(rows) * 4,
                          static_cast<size_t>(cols), cudaMemcpyDeviceToDevice, s);
    if (e != cudaSuccess)
      return XVRAM_STATUS_CUDA_ERROR;
  }
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
      n > INT32_MAX || k > INT32_MAX || panel_k < 0 || !b || ldb < (op_b == 0 ? k : n) ||
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
  const uint64_t M = static_cast<uint64_t>(m_local), N = static_cast<uint64_t>(n),
                 K = static_cast<uint64_t>(k);

  // ---- 1. agree on the plan: max rows over ranks, min device memory available.
  const uint64_t shape[6] = {M, N, K, op_a, op_b, static_cast<uint64_t>(panel_k)};
  const auto now = std::chrono::steady_clock::now();
  uint64_t avail = g->avail_sampled;
  if (std::memcmp(shape, g->shape_sampled, sizeof shape) != 0 ||
      now - g->when_sampled > std::chrono::seconds(1) || avail == 0) {
    uint64_t free_b = 0, total_b = 0;
    if (cudaError_t e = cudaMemGetInfo(&free_b, &total_b); e != cudaSuccess)
      return cuda_status(e);
    avail = free_b + g->held_bytes() - g->plan_dev.bytes;
    g->avail_sampled = avail;
    std::memcpy(g->shape_sampled, shape, sizeof shape);
    g->when_sampled = now;
  }
  avail = avail > kHeadroomBytes ? avail - kHeadroomBytes : 0;
  avail = std::min(avail, env_u64("XVRAM_B200_SHARD_BUDGET_BYTES", UINT64_MAX));
  g->plan_host[0] = M;
  g->plan_host[1] = UINT64_MAX - avail;
  {
    cudaError_t e = cudaMemcpyAsync(g->plan_dev.p, g->plan_host, 2 * sizeof(uint64_t),
                                    cudaMemcpyHostToDevice, g->coll);
    if (e != cudaSuccess) {
      g->aborted = true;
      return cuda_status(e);
    }
    if (P > 1) {
      if (xvram_status st = nccl_issued(
              *g, nccl().all_reduce(g->plan_dev.p, g->plan_dev.p, 2, ncclUint64, ncclMax, g->comm,
                                    g->coll));
          st != XVRAM_STATUS_SUCCESS)
        return st;
    }
    e = cudaMemcpyAsync(g->plan_host, g->plan_dev.p, 2 * sizeof(uint64_t), cudaMemcpyDeviceToHost,
                        g->coll);
    if (e == cudaSuccess)
      e = cudaEventRecord(g->plan_ev, g->coll);
    if (e != cudaSuccess) {
      g->aborted = true;
      return cuda_status(e);
    }
    if (xvram_status st = bounded_wait(*g, g->plan_ev); st != XVRAM_STATUS_SUCCESS)
      return st;
  }
  const uint64_t m_max = g->plan_host[0];
  const uint64_t avail_min = UINT64_MAX - g->plan_host[1];
  if (m_max == 0)
    return XVRAM_STATUS_SUCCESS; // no rank has rows: nothing to compute or gather

  Plan pl;
  pl.kb = std::min<uint64_t>(up(panel_k > 0 ? static_cast<uint64_t>(panel_k) : 1024, 32), up(K, 32));
  pl.nb = std::min<uint64_t>(N, up(env_u64("XVRAM_B200_SHARD_BLOCK_N", kDefaultBlockN), 32));
  pl.ldk = up4(K);
  pl.ldn = up4(pl.nb);
  // Largest row group (multiple of 128 rows, at most all rows) whose buffers fit.
  pl.mg = up(m_max, kTileM);
  size_plan(pl, op_a, op_b, N, K, P);
  while (plan_bytes(pl) > avail_min && pl.mg > kTileM) {
    pl.mg = std::max<uint64_t>(kTileM, up(pl.mg / 2, kTileM));
    size_plan(pl, op_a, op_b, N, K, P);
  }
  if (plan_bytes(pl) > avail_min)
    return XVRAM_STATUS_DEVICE_OUT_OF_MEMORY; // same verdict on every rank
  pl.groups = (m_max + pl.mg - 1) / pl.mg;

  // ---- 2. buffers (all released first when any must grow, so the old ones never
  // coexist with the new ones).
  {
    constexpr int kData = ShardGroup::kBuffers - 1; // all but plan_dev
    const uint64_t want[kData] = {pl.bytes_a_canon, pl.bytes_a_raw,   pl.bytes_a_raw,
                                  pl.bytes_b_raw,   pl.bytes_b_raw,   pl.bytes_b_raw,
                                  pl.bytes_b_canon, pl.bytes_b_canon, pl.bytes_b_canon,
                                  pl.bytes_c,       pl.bytes_c,       pl.bytes_c};
    bool grow = false;
    for (int i = 0; i < kData; ++i)
      grow = grow || g->buffers[i]->bytes < want[i];
    cudaError_t e = cudaSuccess;
    if (grow) {
      for (int i = 0; i < kData; ++i)
        g->buffers[i]->release();
      for (int i = 0; i < kData && e == cudaSuccess; ++i)
        if (want[i])
          e = g->buffers[i]->ensure(want[i]);
    }
    if (e != cudaSuccess) {
      // The other ranks planned with the same numbers; this rank failing leaves them to
      // time out in the next all-gather, so the group is not reusable.
      abort_group(*g);
      return cuda_status(e);
    }
    const uint64_t panels = (K + pl.kb - 1) / pl.kb;
    while (g->a_ev.size() < panels) {
      cudaEvent_t ev = nullptr;
      if ((e = cudaEventCreateWithFlags(&ev, cudaEventDisableTiming)) != cudaSuccess)
        return cuda_status(e);
      g->a_ev.push_back(ev);
    }
  }

  // ---- 3. enqueue
  const char* ah = reinterpret_cast<const char*>(a);
  const char* bh = reinterpret_cast<const char*>(b);
  char* ch = reinterpret_cast<char*>(c);
  float* a_canon = static_cast<float*>(g->a_canon.p);
  const uint64_t blocks = (N + pl.nb - 1) / pl.nb;
  const uint64_t panels = (K + pl.kb - 1) / pl.kb;
  const long long ldm = static_cast<long long>(pl.ldm), ldn = static_cast<long long>(pl.ldn);
  uint64_t q = 0; // global block counter: slot q % kSlots, compute stream q & 1
  cudaError_t e = cudaSuccess;
  for (uint64_t grp = 0; grp < pl.groups && e == cudaSuccess; ++grp) {
    const uint64_t r0 = grp * pl.mg;
    const uint64_t mr = r0 < M ? std::min(pl.mg, M - r0) : 0;
    if (grp > 0) {
      // a_canon is rewritten: every kernel of the previous group must be done.
      for (int i = 0; i < 2 && e == cudaSuccess; ++i)
        e = cudaStreamWaitEvent(g->h2d, g->group_end[i], 0);
      if (e == cudaSuccess)
        e = cudaStreamWaitEvent(g->comp[0], g->group_end[1], 0);
      if (e == cudaSuccess)
        e = cudaStreamWaitEvent(g->comp[1], g->group_end[0], 0);
    }
    for (uint64_t j = 0; j < blocks && e == cudaSuccess; ++j, ++q) {
      const int s = static_cast<int>(q % kSlots);
      cudaStream_t cs = g->comp[q & 1];
      const uint64_t n0 = j * pl.nb, nbj = std::min(pl.nb, N - n0);
      char* braw = static_cast<char*>(g->b_raw[s].p);
      char* bcan = static_cast<char*>(g->b_canon[s].p);
      const float* bcanf = reinterpret_cast<const float*>(bcan);
      float* cblk = static_cast<float*>(g->c_blk[s].p);

      // (a) this rank's slice of B's block j, then the in-place all-gather
      e = cudaStreamWaitEvent(g->h2d, g->b_free[s], 0);
      if (e == cudaSuccess) {
        if (op_b == 0) { // B stored K x N: slice = columns [c0, c0 + wc) of the block
          const uint64_t c0 = static_cast<uint64_t>(r) * pl.wc;
          const uint64_t cols = c0 < nbj ? std::min(pl.wc, nbj - c0) : 0;
          if (cols)
            e = cudaMemcpy2DAsync(braw + c0 * pl.ldk * 4, pl.ldk * 4,
                                  bh + (n0 + c0) * static_cast<uint64_t>(ldb) * 4,
                                  static_cast<size_t>(ldb) * 4, K * 4, cols,
                                  cudaMemcpyHostToDevice, g->h2d);
        } else { // B stored N x K: slice = k range [q0, q0 + wk) of rows [n0, n0 + nbj)
          const uint64_t q0 = static_cast<uint64_t>(r) * pl.wk;
          const uint64_t ks = q0 < K ? std::min(pl.wk, K - q0) : 0;
          if (ks)
            e = cudaMemcpy2DAsync(bcan + q0 * pl.ldn * 4, pl.ldn * 4,
                                  bh + (n0 + q0 * static_cast<uint64_t>(ldb)) * 4,
                                  static_cast<size_t>(ldb) * 4, nbj * 4, ks,
                                  cudaMemcpyHostToDevice, g->h2d);
        }
      }
      if (e == cudaSuccess)
        e = cudaEventRecord(g->b_loaded[s], g->h2d);
      if (e == cudaSuccess)
        e = cudaStreamWaitEvent(g->coll, g->b_loaded[s], 0);
      if (e == cudaSuccess && P > 1) {
        char* base = op_b == 0 ? braw : bcan;
        if (xvram_status st = nccl_issued(
                *g, nccl().all_gather(base + static_cast<uint64_t>(r) * pl.slice_elems * 4, base,
                                      pl.slice_elems, ncclFloat, g->comm, g->coll));
            st != XVRAM_STATUS_SUCCESS)
          return st;
      }
      if (e == cudaSuccess && op_b == 0) // K-major block -> N-major (nbj x K, ld ldn)
        e = xvram::transpose_f32_async(reinterpret_cast<const float*>(braw),
                                       static_cast<long long>(pl.ldk),
                                       reinterpret_cast<float*>(bcan), ldn, static_cast<int>(K),
                                       static_cast<int>(nbj), g->coll);
      if (e == cudaSuccess)
        e = cudaEventRecord(g->b_ready[s], g->coll);

      // (b) C's block j (rows [r0, r0 + mr) of this rank)
      if (e == cudaSuccess && mr > 0 && beta != 0.0f) {
        e = cudaStreamWaitEvent(g->h2d, g->c_free[s], 0);
        if (e == cudaSuccess)
          e = cudaMemcpy2DAsync(cblk, pl.ldm * 4,
                                ch + (r0 + n0 * static_cast<uint64_t>(ldc)) * 4,
                                static_cast<size_t>(ldc) * 4, mr * 4, nbj, cudaMemcpyHostToDevice,
                                g->h2d);
        if (e == cudaSuccess)
          e = cudaEventRecord(g->c_loaded[s], g->h2d);
      }

      // (c) the kernel(s)
      if (e == cudaSuccess)
        e = cudaStreamWaitEvent(cs, g->b_ready[s], 0);
      if (e == cudaSuccess && mr > 0)
        e = cudaStreamWaitEvent(cs, beta != 0.0f ? g->c_loaded[s] : g->c_free[s], 0);
      if (e == cudaSuccess && mr > 0 && j == 0) {
        // First block of the group: A arrives panel by panel and each panel's kernel
        // starts as soon as it is resident (beta on the first, 1 afterwards).
        for (uint64_t p = 0; p < panels && e == cudaSuccess; ++p) {
          const uint64_t k0 = p * pl.kb, kr = std::min(pl.kb, K - k0);
          const int as = static_cast<int>(p & 1);
          if (op_a == 0) { // A stored M x K: kr columns of mr floats
            e = cudaMemcpy2DAsync(a_canon + k0 * pl.ldm, pl.ldm * 4,
                                  ah + (r0 + k0 * static_cast<uint64_t>(lda)) * 4,
                                  static_cast<size_t>(lda) * 4, mr * 4, kr, cudaMemcpyHostToDevice,
                                  g->h2d);
            if (e == cudaSuccess)
              e = cudaEventRecord(g->a_ev[p], g->h2d);
            if (e == cudaSuccess)
              e = cudaStreamWaitEvent(cs, g->a_ev[p], 0);
          } else { // A stored K x M: mr columns of kr floats, then transposed on arrival
            float* raw = static_cast<float*>(g->a_raw[as].p);
            e = cudaStreamWaitEvent(g->h2d, g->a_free[as], 0);
            if (e == cudaSuccess)
              e = cudaMemcpy2DAsync(raw, up4(pl.kb) * 4,
                                    ah + (k0 + r0 * static_cast<uint64_t>(lda)) * 4,
                                    static_cast<size_t>(lda) * 4, kr * 4, mr,
                                    cudaMemcpyHostToDevice, g->h2d);
            if (e == cudaSuccess)
              e = cudaEventRecord(g->a_ev[p], g->h2d);
            if (e == cudaSuccess)
              e = cudaStreamWaitEvent(cs, g->a_ev[p], 0);
            if (e == cudaSuccess)
              e = xvram::transpose_f32_async(raw, static_cast<long long>(up4(pl.kb)),
                                             a_canon + k0 * pl.ldm, ldm, static_cast<int>(kr),
                                             static_cast<int>(mr), cs);
            if (e == cudaSuccess)
              e = cudaEventRecord(g->a_free[as], cs);
          }
          if (e == cudaSuccess && p + 1 == panels)
            e = cudaEventRecord(g->a_all, cs);
          if (e == cudaSuccess)
            e = xvram::sgemm_ffma(0, 1, static_cast<int>(mr), static_cast<int>(nbj),
                                  static_cast<int>(kr), alpha, a_canon + k0 * pl.ldm, ldm,
                                  bcanf + k0 * pl.ldn, ldn, p == 0 ? beta : 1.0f, cblk, ldm, cs);
        }
      } else if (e == cudaSuccess && mr > 0) {
        e = cudaStreamWaitEvent(cs, g->a_all, 0);
        if (e == cudaSuccess)
          e = xvram::sgemm_ffma(0, 1, static_cast<int>(mr), static_cast<int>(nbj),
                                static_cast<int>(K), alpha, a_canon, ldm, bcanf, ldn, beta, cblk,
                                ldm, cs);
      }
      if (e == cudaSuccess)
        e = cudaEventRecord(g->b_free[s], cs);

      // (d) C's block j back to the host
      if (e == cudaSuccess && mr > 0) {
        e = cudaEventRecord(g->c_done[s], cs);
        if (e == cudaSuccess)
          e = cudaStreamWaitEvent(g->d2h, g->c_done[s], 0);
        if (e == cudaSuccess)
          e = cudaMemcpy2DAsync(ch + (r0 + n0 * static_cast<uint64_t>(ldc)) * 4,
                                static_cast<size_t>(ldc) * 4, cblk, pl.ldm * 4, mr * 4, nbj,
                                cudaMemcpyDeviceToHost, g->d2h);
        if (e == cudaSuccess)
          e = cudaEventRecord(g->c_free[s], g->d2h);
      }
    }
    for (int i = 0; i < 2 && e == cudaSuccess; ++i)
      e = cudaEventRecord(g->group_end[i], g->comp[i]);
  }
  // The call is over when both compute streams (which waited for every gather) and the
  // last write-back are done.
  for (int i = 0; i < 2 && e == cudaSuccess; ++i)
    e = cudaStreamWaitEvent(g->d2h, g->group_end[i], 0);
  if (e == cudaSuccess)
    e = cudaEventRecord(g->out, g->d2h);
  if (e != cudaSuccess) {
    g->aborted = true;
    return cuda_status(e);
  }
  xvram_status st = bounded_wait(*g, g->out);
  if (st == XVRAM_STATUS_SUCCESS) {
    unsigned int word = 0;
    if (xvram::read_and_clear_kernel_error(&word, g->d2h) != cudaSuccess)
      st = XVRAM_STATUS_CUDA_ERROR;
    else if (word)
      st = XVRAM_STATUS_TIMEOUT;
  }
  if (st != XVRAM_STATUS_SUCCESS)
    g->aborted = true;
  return st;
}

} // extern "C"
