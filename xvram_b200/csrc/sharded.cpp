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
// The executor reaches the GPU only through the runtime's Device interface (device.hpp)
// and its peers only through a ShardComm (below): NCCL for groups made from a unique id,
// or caller-supplied collectives (xvram_b200_shard_group_create_custom).  The same
// schedule therefore also runs on the host-memory fake device with host collectives,
// which is how the CPU test suite checks the partition, the B slices and the plan
// agreement across ranks.
//
// NCCL is loaded at run time (dlopen of libnccl.so.2, whichever the process already has),
// so the library keeps no link-time NCCL dependency.  Communicator creation is
// non-blocking with a deadline, and every host wait on a collective is bounded: a peer
// that never arrives produces TIMEOUT and an aborted communicator, not a hang.
#include "xvram_b200.h"

#include "device.hpp"

#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <algorithm>
#include <chrono>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <mutex>
#include <thread>
#include <vector>

namespace {

using xvram::Device;
using xvram::EventId;
using xvram::StreamId;

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
constexpr double kWaitTimeoutS = 60.0;   // per host wait (per stretch of blocks at the end)
constexpr uint64_t kProgressMarks = 256;   // progress events per call at most
constexpr uint64_t kHeadroomBytes = 1ull << 30; // left free on the device for everything else
// C block width (columns).  Measured on C2 TN at one GPU (median of 8 calls): 512 -> 10.76
// ms, 1024 -> 11.18 ms, 2048 -> 12.21 ms: narrower blocks start the first kernel and end
// the last write-back sooner.  576 = 3 x 192 lets the 192 x 192 kernel tiling run whole
// tiles (65536 x 65536 x 16384 on one GPU: 512 -> 63.0, 576 -> 64.6, 768 -> 64.5 TFLOP/s).
constexpr uint64_t kDefaultBlockN = 576;
constexpr uint64_t kTileM = 128;                // row granularity of partitions and row groups
// B and C block buffers in flight: block j+2's copies may start while block j's
// write-back is still running.
constexpr int kSlots = 3;

double seconds_since(std::chrono::steady_clock::time_point t0) {
  return std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
}

// The collectives a shard group needs, enqueued on the group's collective stream (its
// native handle).  Buffers are device addresses of the group's device.
class ShardComm {
public:
  virtual ~ShardComm() = default;
  // In place: buf[0..count) = elementwise maximum over the ranks.
  virtual xvram_status all_reduce_max_u64(uint64_t* buf, uint64_t count, uint64_t stream) = 0;
  // recv = the ranks' `count`-float sends, in rank order; send may be recv + rank * count.
  virtual xvram_status all_gather_f32(const float* send, float* recv, uint64_t count,
                                      uint64_t stream) = 0;
  // Polled while the host waits on the device: non-SUCCESS once the collectives failed.
  virtual xvram_status health() = 0;
  virtual void abort() = 0;
};

class NcclComm final : public ShardComm {
public:
  explicit NcclComm(ncclComm_t c) : comm_(c) {}
  ~NcclComm() override {
    if (comm_)
      nccl().destroy(comm_);
  }
  xvram_status all_reduce_max_u64(uint64_t* buf, uint64_t count, uint64_t stream) override {
    return issued(nccl().all_reduce(buf, buf, count, ncclUint64, ncclMax, comm_,
                                    reinterpret_cast<cudaStream_t>(stream)));
  }
  xvram_status all_gather_f32(const float* send, float* recv, uint64_t count,
                              uint64_t stream) override {
    return issued(nccl().all_gather(send, recv, count, ncclFloat, comm_,
                                    reinterpret_cast<cudaStream_t>(stream)));
  }
  xvram_status health() override {
    ncclResult_t ar = ncclSuccess;
    if (!comm_)
      return XVRAM_STATUS_POISONED;
    if (nccl().async_error(comm_, &ar) == ncclSuccess && ar != ncclSuccess &&
        ar != ncclInProgress)
      return XVRAM_STATUS_CUDA_ERROR;
    return XVRAM_STATUS_SUCCESS;
  }
  void abort() override {
    if (comm_)
      nccl().abort(comm_);
    comm_ = nullptr;
  }

private:
  // A non-blocking communicator may return ncclInProgress while it is still enqueueing a
  // call: wait (bounded) until the call has been issued before the next NCCL call.
  xvram_status issued(ncclResult_t nr) {
    if (nr == ncclSuccess)
      return XVRAM_STATUS_SUCCESS;
    if (nr != ncclInProgress)
      return XVRAM_STATUS_CUDA_ERROR;
    const auto t0 = std::chrono::steady_clock::now();
    ncclResult_t st = ncclInProgress;
    while (st == ncclInProgress) {
      if (nccl().async_error(comm_, &st) != ncclSuccess || seconds_since(t0) > kWaitTimeoutS)
        return XVRAM_STATUS_TIMEOUT;
    }
    return st == ncclSuccess ? XVRAM_STATUS_SUCCESS : XVRAM_STATUS_CUDA_ERROR;
  }
  ncclComm_t comm_ = nullptr;
};

// Collectives the caller supplies (xvram_b200_shard_collectives_v1).
class CallbackComm final : public ShardComm {
public:
  explicit CallbackComm(const xvram_b200_shard_collectives_v1& ops) : ops_(ops) {}
  xvram_status all_reduce_max_u64(uint64_t* buf, uint64_t count, uint64_t stream) override {
    return ops_.all_reduce_max_u64(ops_.context, buf, count, stream);
  }
  xvram_status all_gather_f32(const float* send, float* recv, uint64_t count,
                              uint64_t stream) override {
    return ops_.all_gather_f32(ops_.context, send, recv, count, stream);
  }
  xvram_status health() override { return XVRAM_STATUS_SUCCESS; }
  void abort() override {}

private:
  xvram_b200_shard_collectives_v1 ops_;
};

struct Buffer {
  uint64_t p = 0;
  uint64_t bytes = 0;
};

struct ShardGroup {
  std::unique_ptr<Device> dev;
  std::unique_ptr<ShardComm> comm;
  int rank = 0, world = 1, device = 0;
  StreamId h2d = 0, coll = 0, comp[2] = {}, d2h = 0;
  // Per buffer slot: B block copied / gathered (and canonical) / no longer read;
  // C block copied in / computed / copied out.
  EventId b_loaded[kSlots] = {}, b_ready[kSlots] = {}, b_free[kSlots] = {};
  EventId c_loaded[kSlots] = {}, c_done[kSlots] = {}, c_free[kSlots] = {};
  // A raw panel slot reusable (K-major A), all of A canonical, end of a row group per
  // compute stream, end of the call, plan exchange done.
  EventId a_free[2] = {}, a_all = 0, group_end[2] = {}, out = 0, plan_ev = 0;
  std::vector<EventId> a_ev; // one per A panel: panel p resident (and canonical)
  // Progress marks: recorded on the compute stream after every `stride`-th block's kernel,
  // so the end-of-call wait allows kWaitTimeoutS per stretch of blocks, not for the whole
  // call (a full-size call runs for minutes).
  std::vector<EventId> progress_ev;
  Buffer a_canon, a_raw[2], b_raw[kSlots], b_canon[kSlots], c_blk[kSlots], plan_dev;
  uint64_t* plan_host = nullptr; // 2 x u64, page-locked
  bool aborted = false;
  std::mutex mu;
  // Device memory this group may use (free + its own buffers), as sampled for the last
  // call, with that call's shape: a repeat of the same shape within a second reuses it
  // instead of asking the device again, whose latency now and then reaches milliseconds.
  uint64_t avail_sampled = 0;
  uint64_t shape_sampled[6] = {};
  std::chrono::steady_clock::time_point when_sampled{};
  xvram_b200_shard_plan_v1 last{};

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
  bool ensure(Buffer& b, uint64_t want) {
    if (b.bytes >= want)
      return true;
    release(b);
    if (dev->mem_alloc(want, &b.p))
      return false;
    b.bytes = want;
    return true;
  }
  void release(Buffer& b) {
    if (b.p)
      dev->mem_free(b.p);
    b.p = 0;
    b.bytes = 0;
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

void abort_group(ShardGroup& g) {
  if (g.comm)
    g.comm->abort();
  g.aborted = true;
}

// Waits for `e` with a deadline, watching the collectives for asynchronous errors.
xvram_status bounded_wait(ShardGroup& g, EventId e) {
  const auto start = std::chrono::steady_clock::now();
  for (;;) {
    bool done = false;
    if (g.dev->event_query(e, &done))
      return XVRAM_STATUS_CUDA_ERROR;
    if (done)
      return XVRAM_STATUS_SUCCESS;
    if (xvram_status h = g.comm->health(); h != XVRAM_STATUS_SUCCESS) {
      abort_group(g);
      return h;
    }
    if (seconds_since(start) > kWaitTimeoutS) {
      abort_group(g);
      return XVRAM_STATUS_TIMEOUT;
    }
    std::this_thread::sleep_for(std::chrono::microseconds(50));
  }
}

void destroy_group(ShardGroup* g) {
  if (!g)
    return;
  if (g->dev) {
    int prev = 0;
    const bool switched = !g->dev->make_current(&prev);
    for (StreamId s : {g->h2d, g->coll, g->comp[0], g->comp[1], g->d2h})
      if (s)
        g->dev->stream_sync(s);
    for (Buffer* b : g->buffers)
      g->release(*b);
    if (g->plan_host)
      g->dev->host_free(g->plan_host);
    g->comm.reset();
    g->dev->close(); // streams and events
    if (switched)
      g->dev->restore_current(prev);
  }
  delete g;
}

// Opens the group's device (the current CUDA device, or the installed test device) and
// creates its streams, events and plan-exchange buffers.
xvram_status setup_group(ShardGroup& g) {
  g.dev = xvram::device_factory()();
  int ordinal = 0;
  if (cudaGetDevice(&ordinal) != cudaSuccess) { // no CUDA here: only a test device opens
    cudaGetLastError();
    ordinal = 0;
  }
  xvram::DeviceInfo info;
  if (xvram::Error e = g.dev->open(ordinal, &info))
    return e.status;
  g.device = ordinal;
  Device& d = *g.dev;
  for (StreamId* s : {&g.h2d, &g.coll, &g.comp[0], &g.comp[1], &g.d2h})
    if (d.stream_create(s))
      return XVRAM_STATUS_CUDA_ERROR;
  for (EventId* arr : {g.b_loaded, g.b_ready, g.b_free, g.c_loaded, g.c_done, g.c_free})
    for (int i = 0; i < kSlots; ++i)
      if (d.event_create(&arr[i]))
        return XVRAM_STATUS_CUDA_ERROR;
  for (EventId* arr : {g.a_free, g.group_end})
    for (int i = 0; i < 2; ++i)
      if (d.event_create(&arr[i]))
        return XVRAM_STATUS_CUDA_ERROR;
  for (EventId* e : {&g.a_all, &g.out, &g.plan_ev})
    if (d.event_create(e))
      return XVRAM_STATUS_CUDA_ERROR;
  void* ph = nullptr;
  if (d.host_alloc(2 * sizeof(uint64_t), &ph))
    return XVRAM_STATUS_HOST_OUT_OF_MEMORY;
  g.plan_host = static_cast<uint64_t*>(ph);
  if (!g.ensure(g.plan_dev, 256))
    return XVRAM_STATUS_DEVICE_OUT_OF_MEMORY;
  return XVRAM_STATUS_SUCCESS;
}

} // namespace

namespace xvram {

// Rows [*begin, *begin + *count) of an m-row C that rank `rank` of `world` owns: whole
// 128-row tiles dealt out as evenly as possible (rank r takes tiles [r T / P, (r+1) T / P)),
// the last tile cut at m.  Ranks beyond the tile count get no rows.
void shard_rows(uint64_t m, int world, int rank, uint64_t* begin, uint64_t* count) {
  const uint64_t tiles = (m + kTileM - 1) / kTileM;
  const uint64_t t0 = tiles * static_cast<uint64_t>(rank) / static_cast<uint64_t>(world);
  const uint64_t t1 = tiles * static_cast<uint64_t>(rank + 1) / static_cast<uint64_t>(world);
  const uint64_t r0 = std::min(m, t0 * kTileM), r1 = std::min(m, t1 * kTileM);
  *begin = r0;
  *count = r1 - r0;
}

// The geometry every rank derives from the same agreed numbers (largest row count over the
// ranks, smallest device memory available), so every rank issues the same collectives.
struct ShardPlan {
  uint64_t groups = 0; // row groups (0: nothing to do on any rank)
  uint64_t mg = 0;     // rows per group
  uint64_t nb = 0;     // C block width
  uint64_t kb = 0;     // A panel depth
  uint64_t ldk = 0, ldn = 0, ldm = 0; // packed leading dimensions (K-major B raw, N, M)
  uint64_t wc = 0, wk = 0;            // per-rank B slice: columns (op N) or k (op T)
  uint64_t slice_elems = 0;
  uint64_t bytes_a_canon = 0, bytes_a_raw = 0, bytes_b_raw = 0, bytes_b_canon = 0,
           bytes_c = 0;
  uint64_t device_bytes() const {
    return bytes_a_canon + 2 * bytes_a_raw + kSlots * (bytes_b_raw + bytes_b_canon + bytes_c);
  }
};

namespace {
void size_plan(ShardPlan& pl, uint32_t op_a, uint32_t op_b, uint64_t k, int P) {
  pl.ldm = up4(std::max<uint64_t>(pl.mg, 1));
  pl.bytes_a_canon = pl.ldm * k * 4;
  pl.bytes_a_raw = op_a != 0 ? up4(pl.kb) * std::max<uint64_t>(pl.mg, 1) * 4 : 0;
  pl.bytes_c = pl.ldm * pl.nb * 4;
  if (op_b == 0) {
    pl.wc = (pl.nb + P - 1) / P;
    pl.wk = 0;
    pl.slice_elems = pl.wc * pl.ldk;
    pl.bytes_b_raw = pl.slice_elems * static_cast<uint64_t>(P) * 4;
    pl.bytes_b_canon = pl.ldn * k * 4;
  } else {
    pl.wk = (k + P - 1) / P;
    pl.wc = 0;
    pl.slice_elems = pl.wk * pl.ldn;
    pl.bytes_b_raw = 0;
    pl.bytes_b_canon = pl.slice_elems * static_cast<uint64_t>(P) * 4;
  }
}
} // namespace

// Plans the call from the agreed numbers; false when not even one 128-row group fits.
bool make_shard_plan(uint32_t op_a, uint32_t op_b, uint64_t m_max, uint64_t avail_min,
                     uint64_t n, uint64_t k, int world, uint64_t panel_k, uint64_t block_n,
                     ShardPlan* out) {
  ShardPlan pl;
  pl.kb = std::min<uint64_t>(up(panel_k > 0 ? panel_k : 1024, 32), up(k, 32));
  pl.nb = std::min<uint64_t>(n, up(block_n, 32));
  pl.ldk = up4(k);
  pl.ldn = up4(pl.nb);
  // Largest row group (multiple of 128 rows, at most all rows) whose buffers fit.
  pl.mg = up(std::max<uint64_t>(m_max, 1), kTileM);
  size_plan(pl, op_a, op_b, k, world);
  while (pl.device_bytes() > avail_min && pl.mg > kTileM) {
    pl.mg = std::max<uint64_t>(kTileM, up(pl.mg / 2, kTileM));
    size_plan(pl, op_a, op_b, k, world);
  }
  pl.groups = m_max == 0 ? 0 : (m_max + pl.mg - 1) / pl.mg;
  *out = pl;
  return pl.device_bytes() <= avail_min;
}

// Rank `rank`'s slice of C block [n0, n0 + nbj) of B: for op(B) = N (B stored K x N) the
// block columns [*first, *first + *count) relative to n0; for op(B) = T (B stored N x K)
// the k range [*first, *first + *count).
void shard_b_slice(const ShardPlan& pl, uint32_t op_b, uint64_t nbj, uint64_t k, int rank,
                   uint64_t* first, uint64_t* count) {
  if (op_b == 0) {
    const uint64_t c0 = static_cast<uint64_t>(rank) * pl.wc;
    *first = c0;
    *count = c0 < nbj ? std::min(pl.wc, nbj - c0) : 0;
  } else {
    const uint64_t q0 = static_cast<uint64_t>(rank) * pl.wk;
    *first = q0;
    *count = q0 < k ? std::min(pl.wk, k - q0) : 0;
  }
}

} // namespace xvram

namespace {

xvram_status status_of(const xvram::Error& e) {
  return e ? (e.status ? e.status : XVRAM_STATUS_CUDA_ERROR) : XVRAM_STATUS_SUCCESS;
}

// The body of xvram_b200_sgemm_sharded, with g's device current and g.mu held.
xvram_status run_sharded(ShardGroup& g, uint32_t op_a, uint32_t op_b, uint64_t M, uint64_t N,
                         uint64_t K, float alpha, const float* a, uint64_t lda, const float* b,
                         uint64_t ldb, float beta, float* c, uint64_t ldc, int64_t panel_k) {
  Device& d = *g.dev;
  const int P = g.world, r = g.rank;
  using xvram::CopyDir;
  xvram_b200_shard_plan_v1 info{};
  info.struct_size = sizeof info;
  info.world = P;
  info.rank = r;

  // ---- 1. agree on the plan: max rows over ranks, min device memory available.
  const uint64_t shape[6] = {M, N, K, op_a, op_b, static_cast<uint64_t>(panel_k)};
  const auto now = std::chrono::steady_clock::now();
  uint64_t avail = g.avail_sampled;
  if (std::memcmp(shape, g.shape_sampled, sizeof shape) != 0 ||
      now - g.when_sampled > std::chrono::seconds(1) || avail == 0) {
    uint64_t free_b = 0, total_b = 0;
    if (xvram::Error e = d.mem_get_info(&free_b, &total_b))
      return status_of(e);
    avail = free_b + g.held_bytes() - g.plan_dev.bytes;
    g.avail_sampled = avail;
    std::memcpy(g.shape_sampled, shape, sizeof shape);
    g.when_sampled = now;
  }
  avail = avail > kHeadroomBytes ? avail - kHeadroomBytes : 0;
  avail = std::min(avail, env_u64("XVRAM_B200_SHARD_BUDGET_BYTES", UINT64_MAX));
  g.plan_host[0] = M;
  g.plan_host[1] = UINT64_MAX - avail;
  {
    const uint64_t ph = reinterpret_cast<uint64_t>(g.plan_host);
    xvram::Error e = d.copy_2d(g.plan_dev.p, 16, ph, 16, 16, 1, CopyDir::h2d, g.coll);
    if (e) {
      g.aborted = true;
      return status_of(e);
    }
    if (P > 1) {
      const xvram_status st = g.comm->all_reduce_max_u64(
          reinterpret_cast<uint64_t*>(g.plan_dev.p), 2, d.native_stream(g.coll));
      if (st != XVRAM_STATUS_SUCCESS) {
        abort_group(g);
        return st;
      }
    }
    e = d.copy_2d(ph, 16, g.plan_dev.p, 16, 16, 1, CopyDir::d2h, g.coll);
    if (!e)
      e = d.event_record(g.plan_ev, g.coll);
    if (e) {
      g.aborted = true;
      return status_of(e);
    }
    if (xvram_status st = bounded_wait(g, g.plan_ev); st != XVRAM_STATUS_SUCCESS)
      return st;
  }
  const uint64_t m_max = g.plan_host[0];
  const uint64_t avail_min = UINT64_MAX - g.plan_host[1];
  info.m_max = m_max;
  info.avail_min = avail_min;
  if (m_max == 0) {
    g.last = info;
    return XVRAM_STATUS_SUCCESS; // no rank has rows: nothing to compute or gather
  }

  xvram::ShardPlan pl;
  if (!xvram::make_shard_plan(op_a, op_b, m_max, avail_min, N, K, P,
                              static_cast<uint64_t>(panel_k),
                              env_u64("XVRAM_B200_SHARD_BLOCK_N", kDefaultBlockN), &pl))
    return XVRAM_STATUS_DEVICE_OUT_OF_MEMORY; // same verdict on every rank
  info.row_groups = pl.groups;
  info.group_rows = pl.mg;
  info.block_n = pl.nb;
  info.panel_k = pl.kb;
  info.b_slice_cols = pl.wc;
  info.b_slice_k = pl.wk;
  info.slice_elems = pl.slice_elems;
  info.device_bytes = pl.device_bytes();

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
      grow = grow || g.buffers[i]->bytes < want[i];
    bool ok = true;
    if (grow) {
      for (int i = 0; i < kData; ++i)
        g.release(*g.buffers[i]);
      for (int i = 0; i < kData && ok; ++i)
        if (want[i])
          ok = g.ensure(*g.buffers[i], want[i]);
    }
    if (!ok) {
      // The other ranks planned with the same numbers; this rank failing leaves them to
      // time out in the next all-gather, so the group is not reusable.
      abort_group(g);
      return XVRAM_STATUS_DEVICE_OUT_OF_MEMORY;
    }
    const uint64_t panels = (K + pl.kb - 1) / pl.kb;
    while (g.a_ev.size() < panels) {
      EventId ev = 0;
      if (xvram::Error e = d.event_create(&ev))
        return status_of(e);
      g.a_ev.push_back(ev);
    }
    const uint64_t marks = std::min<uint64_t>(kProgressMarks, pl.groups * ((N + pl.nb - 1) / pl.nb));
    while (g.progress_ev.size() < marks) {
      EventId ev = 0;
      if (xvram::Error e = d.event_create(&ev))
        return status_of(e);
      g.progress_ev.push_back(ev);
    }
  }

  // ---- 3. enqueue
  const uint64_t ah = reinterpret_cast<uint64_t>(a), bh = reinterpret_cast<uint64_t>(b),
                 ch = reinterpret_cast<uint64_t>(c);
  const uint64_t a_canon = g.a_canon.p;
  const uint64_t blocks = (N + pl.nb - 1) / pl.nb;
  const uint64_t panels = (K + pl.kb - 1) / pl.kb;
  const int64_t ldm = static_cast<int64_t>(pl.ldm), ldn = static_cast<int64_t>(pl.ldn);
  const xvram::GemmTypes fp32{};
  uint64_t q = 0; // global block counter: slot q % kSlots, compute stream q & 1
  const uint64_t total_blocks = pl.groups * blocks;
  const uint64_t marks = std::min<uint64_t>(kProgressMarks, total_blocks);
  const uint64_t stride = (total_blocks + marks - 1) / marks; // blocks per progress mark
  uint64_t marked = 0;
  xvram::Error e;
  auto h2d = [&](uint64_t dst, uint64_t dp, uint64_t src, uint64_t sp, uint64_t w, uint64_t h) {
    info.h2d_bytes += w * h;
    return d.copy_2d(dst, dp, src, sp, w, h, CopyDir::h2d, g.h2d);
  };
  for (uint64_t grp = 0; grp < pl.groups && !e; ++grp) {
    const uint64_t r0 = grp * pl.mg;
    const uint64_t mr = r0 < M ? std::min(pl.mg, M - r0) : 0;
    if (grp > 0) {
      // a_canon is rewritten: every kernel of the previous group must be done.
      for (int i = 0; i < 2 && !e; ++i)
        e = d.stream_wait_event(g.h2d, g.group_end[i]);
      if (!e)
        e = d.stream_wait_event(g.comp[0], g.group_end[1]);
      if (!e)
        e = d.stream_wait_event(g.comp[1], g.group_end[0]);
    }
    for (uint64_t j = 0; j < blocks && !e; ++j, ++q) {
      const int s = static_cast<int>(q % kSlots);
      const StreamId cs = g.comp[q & 1];
      const uint64_t n0 = j * pl.nb, nbj = std::min(pl.nb, N - n0);
      const uint64_t braw = g.b_raw[s].p, bcan = g.b_canon[s].p, cblk = g.c_blk[s].p;

      // (a) this rank's slice of B's block j, then the in-place all-gather
      uint64_t first = 0, count = 0;
      xvram::shard_b_slice(pl, op_b, nbj, K, r, &first, &count);
      e = d.stream_wait_event(g.h2d, g.b_free[s]);
      if (!e && count) {
        if (op_b == 0) // B stored K x N: block columns [first, first + count)
          e = h2d(braw + first * pl.ldk * 4, pl.ldk * 4, bh + (n0 + first) * ldb * 4, ldb * 4,
                  K * 4, count);
        else // B stored N x K: k range [first, first + count) of rows [n0, n0 + nbj)
          e = h2d(bcan + first * pl.ldn * 4, pl.ldn * 4, bh + (n0 + first * ldb) * 4, ldb * 4,
                  nbj * 4, count);
      }
      if (!e)
        e = d.event_record(g.b_loaded[s], g.h2d);
      if (!e)
        e = d.stream_wait_event(g.coll, g.b_loaded[s]);
      if (!e && P > 1) {
        float* base = reinterpret_cast<float*>(op_b == 0 ? braw : bcan);
        const xvram_status st = g.comm->all_gather_f32(
            base + static_cast<uint64_t>(r) * pl.slice_elems, base, pl.slice_elems,
            d.native_stream(g.coll));
        if (st != XVRAM_STATUS_SUCCESS) {
          abort_group(g);
          return st;
        }
        ++info.gathers;
      }
      if (!e && op_b == 0) // K-major block -> N-major (nbj x K, ld ldn)
        e = d.transpose_f32(braw, static_cast<int64_t>(pl.ldk), bcan, ldn,
                            static_cast<int64_t>(K), static_cast<int64_t>(nbj), g.coll);
      if (!e)
        e = d.event_record(g.b_ready[s], g.coll);

      // (b) C's block j (rows [r0, r0 + mr) of this rank)
      if (!e && mr > 0 && beta != 0.0f) {
        e = d.stream_wait_event(g.h2d, g.c_free[s]);
        if (!e)
          e = h2d(cblk, pl.ldm * 4, ch + (r0 + n0 * ldc) * 4, ldc * 4, mr * 4, nbj);
        if (!e)
          e = d.event_record(g.c_loaded[s], g.h2d);
      }

      // (c) the kernel(s)
      if (!e)
        e = d.stream_wait_event(cs, g.b_ready[s]);
      if (!e && mr > 0)
        e = d.stream_wait_event(cs, beta != 0.0f ? g.c_loaded[s] : g.c_free[s]);
      if (!e && mr > 0 && j == 0) {
        // First block of the group: A arrives panel by panel and each panel's kernel
        // starts as soon as it is resident (beta on the first, 1 afterwards).
        for (uint64_t p = 0; p < panels && !e; ++p) {
          const uint64_t k0 = p * pl.kb, kr = std::min(pl.kb, K - k0);
          const int as = static_cast<int>(p & 1);
          if (op_a == 0) { // A stored M x K: kr columns of mr floats
            e = h2d(a_canon + k0 * pl.ldm * 4, pl.ldm * 4, ah + (r0 + k0 * lda) * 4, lda * 4,
                    mr * 4, kr);
            if (!e)
              e = d.event_record(g.a_ev[p], g.h2d);
            if (!e)
              e = d.stream_wait_event(cs, g.a_ev[p]);
          } else { // A stored K x M: mr columns of kr floats, then transposed on arrival
            const uint64_t raw = g.a_raw[as].p;
            e = d.stream_wait_event(g.h2d, g.a_free[as]);
            if (!e)
              e = h2d(raw, up4(pl.kb) * 4, ah + (k0 + r0 * lda) * 4, lda * 4, kr * 4, mr);
            if (!e)
              e = d.event_record(g.a_ev[p], g.h2d);
            if (!e)
              e = d.stream_wait_event(cs, g.a_ev[p]);
            if (!e)
              e = d.transpose_f32(raw, static_cast<int64_t>(up4(pl.kb)), a_canon + k0 * pl.ldm * 4,
                                  ldm, static_cast<int64_t>(kr), static_cast<int64_t>(mr), cs);
            if (!e)
              e = d.event_record(g.a_free[as], cs);
          }
          if (!e && p + 1 == panels)
            e = d.event_record(g.a_all, cs);
          if (!e)
            e = d.gemm(fp32, 0, 1, static_cast<int64_t>(mr), static_cast<int64_t>(nbj),
                       static_cast<int64_t>(kr), alpha, a_canon + k0 * pl.ldm * 4, ldm,
                       bcan + k0 * pl.ldn * 4, ldn, p == 0 ? beta : 1.0f, cblk, ldm, 0, 0, cs);
        }
      } else if (!e && mr > 0) {
        e = d.stream_wait_event(cs, g.a_all);
        if (!e)
          e = d.gemm(fp32, 0, 1, static_cast<int64_t>(mr), static_cast<int64_t>(nbj),
                     static_cast<int64_t>(K), alpha, a_canon, ldm, bcan, ldn, beta, cblk, ldm, 0,
                     0, cs);
      }
      if (!e)
        e = d.event_record(g.b_free[s], cs);
      if (!e && (q + 1) % stride == 0 && marked < marks)
        e = d.event_record(g.progress_ev[marked++], cs);

      // (d) C's block j back to the host
      if (!e && mr > 0) {
        e = d.event_record(g.c_done[s], cs);
        if (!e)
          e = d.stream_wait_event(g.d2h, g.c_done[s]);
        if (!e) {
          info.d2h_bytes += mr * 4 * nbj;
          e = d.copy_2d(ch + (r0 + n0 * ldc) * 4, ldc * 4, cblk, pl.ldm * 4, mr * 4, nbj,
                        CopyDir::d2h, g.d2h);
        }
        if (!e)
          e = d.event_record(g.c_free[s], g.d2h);
      }
    }
    for (int i = 0; i < 2 && !e; ++i)
      e = d.event_record(g.group_end[i], g.comp[i]);
  }
  // The call is over when both compute streams (which waited for every gather) and the
  // last write-back are done.
  for (int i = 0; i < 2 && !e; ++i)
    e = d.stream_wait_event(g.d2h, g.group_end[i]);
  if (!e)
    e = d.event_record(g.out, g.d2h);
  if (e) {
    g.aborted = true;
    return status_of(e);
  }
  // Every stretch of blocks must finish within kWaitTimeoutS of the one before; then the
  // last write-back.
  xvram_status st = XVRAM_STATUS_SUCCESS;
  for (uint64_t i = 0; i < marked && st == XVRAM_STATUS_SUCCESS; ++i)
    st = bounded_wait(g, g.progress_ev[i]);
  if (st == XVRAM_STATUS_SUCCESS)
    st = bounded_wait(g, g.out);
  if (st == XVRAM_STATUS_SUCCESS) {
    uint32_t word = 0;
    if (d.kernel_status(g.d2h, &word))
      st = XVRAM_STATUS_CUDA_ERROR;
    else if (word)
      st = XVRAM_STATUS_TIMEOUT;
  }
  if (st != XVRAM_STATUS_SUCCESS)
    g.aborted = true;
  g.last = info;
  return st;
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
  if (xvram_status st = setup_group(*g); st != XVRAM_STATUS_SUCCESS) {
    destroy_group(g);
    return st;
  }
  ncclUniqueId id;
  std::memcpy(&id, unique_id, NCCL_UNIQUE_ID_BYTES);
  ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
  cfg.blocking = 0;
  ncclComm_t comm = nullptr;
  ncclResult_t r = nccl().init_rank_config(&comm, world, id, rank, &cfg);
  const auto start = std::chrono::steady_clock::now();
  while (r == ncclInProgress || r == ncclSuccess) {
    ncclResult_t state = ncclSuccess;
    if (nccl().async_error(comm, &state) != ncclSuccess) {
      r = ncclInternalError;
      break;
    }
    if (state != ncclInProgress) {
      r = state;
      break;
    }
    if (seconds_since(start) > kInitTimeoutS) {
      r = ncclInternalError;
      break;
    }
    std::this_thread::sleep_for(std::chrono::milliseconds(1));
  }
  if (r != ncclSuccess) {
    if (comm)
      nccl().abort(comm);
    destroy_group(g);
    return XVRAM_STATUS_UNAVAILABLE;
  }
  g->comm = std::make_unique<NcclComm>(comm);
  *out_group = reinterpret_cast<uint64_t>(g);
  return XVRAM_STATUS_SUCCESS;
}

XVRAM_B200_API xvram_status XVRAM_CALL xvram_b200_shard_group_create_custom(
    const xvram_b200_shard_collectives_v1* ops, int32_t rank, int32_t world,
    uint64_t* out_group) {
  if (!ops || ops->struct_size < sizeof(xvram_b200_shard_collectives_v1) || !out_group ||
      world < 1 || rank < 0 || rank >= world || !ops->all_reduce_max_u64 || !ops->all_gather_f32)
    return XVRAM_STATUS_INVALID_ARGUMENT;
  auto* g = new ShardGroup;
  g->rank = rank;
  g->world = world;
  if (xvram_status st = setup_group(*g); st != XVRAM_STATUS_SUCCESS) {
    destroy_group(g);
    return st;
  }
  g->comm = std::make_unique<CallbackComm>(*ops);
  *out_group = reinterpret_cast<uint64_t>(g);
  return XVRAM_STATUS_SUCCESS;
}

XVRAM_B200_API xvram_status XVRAM_CALL xvram_b200_shard_rows(int64_t m, int32_t world,
                                                           int32_t rank, int64_t* row_begin,
                                                           int64_t* row_count) {
  if (m < 0 || world < 1 || rank < 0 || rank >= world || !row_begin || !row_count)
    return XVRAM_STATUS_INVALID_ARGUMENT;
  uint64_t b0 = 0, n = 0;
  xvram::shard_rows(static_cast<uint64_t>(m), world, rank, &b0, &n);
  *row_begin = static_cast<int64_t>(b0);
  *row_count = static_cast<int64_t>(n);
  return XVRAM_STATUS_SUCCESS;
}

XVRAM_B200_API xvram_status XVRAM_CALL xvram_b200_shard_last_plan(uint64_t group,
                                                                xvram_b200_shard_plan_v1* out) {
  auto* g = reinterpret_cast<ShardGroup*>(group);
  if (!g || !out || out->struct_size < sizeof(xvram_b200_shard_plan_v1))
    return XVRAM_STATUS_INVALID_ARGUMENT;
  std::lock_guard<std::mutex> lock(g->mu);
  *out = g->last;
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
  // Device pointers and a native stream of the caller: CUDA devices only.
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
  if (g->world > 1) {
    const xvram_status st = g->comm->all_gather_f32(mine, stage, per_rank, stream);
    if (st != XVRAM_STATUS_SUCCESS) {
      abort_group(*g);
      return st;
    }
  }
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
  int previous = 0;
  if (xvram::Error e = g->dev->make_current(&previous))
    return status_of(e);
  const xvram_status st =
      run_sharded(*g, op_a, op_b, static_cast<uint64_t>(m_local), static_cast<uint64_t>(n),
                  static_cast<uint64_t>(k), alpha, a, static_cast<uint64_t>(lda), b,
                  static_cast<uint64_t>(ldb), beta, c, static_cast<uint64_t>(ldc), panel_k);
  g->dev->restore_current(previous);
  return st;
}

} // extern "C"
