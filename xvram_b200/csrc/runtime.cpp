// runtime.cpp -- see runtime.hpp.
#include "runtime.hpp"
#include "host_util.hpp"

#include <algorithm>
#include <chrono>
#include <climits>
#include <condition_variable>
#include <cstdlib>
#include <cstring>
#include <functional>
#include <map>
#include <mutex>
#include <set>
#include <thread>
#include <utility>

namespace xvram {
namespace {

constexpr uint64_t kArenaOwner = UINT64_MAX;
// Internal allocation that holds the kernels' canonicalisation workspace for in-place
// GEMMs.  Its chunks are never "written", so evicting them is free (no write-back).
constexpr uint64_t kScratchId = UINT64_MAX - 1;

// The device GEMM of a whole problem: the types as declared.
GemmTypes gemm_types(const GemmShape& s) { return {s.a.dtype, s.c.dtype, s.compute}; }
// The device GEMM of one out-of-core step: an FP16 / BF16 C accumulates across K panels in
// FP32 in its slot and is rounded to its type once, when the block is written back.
GemmTypes step_types(const GemmShape& s) {
  GemmTypes t = gemm_types(s);
  if ((s.c.dtype == kFp16 || s.c.dtype == kBf16) && s.compute == kStrictFp32)
    t.c = kFp32;
  return t;
}

struct Chunk {
  int32_t frame = -1;         // frame index while resident
  bool written = false;       // holds caller data (else contents are undefined)
  bool backing_valid = false; // host backing holds the current data
  bool dev_valid = false;     // the resident frame holds the current data
};

struct Alloc {
  uint64_t id = 0;
  uint64_t bytes = 0;
  uint64_t va = 0;
  uint64_t reserved = 0;
  void* host = nullptr;
  std::vector<Chunk> chunks;
  bool live = true;
  bool zero_fill = false; // never-written bytes read as zero (host and device)
};

// Budget sampler threads of open runtimes.  At process exit the CUDA runtime tears its
// state down from an exit handler; a sampler of a runtime its owner never closed (a
// session left open until exit) must not query the device after that.  The first sampler
// registers stop_all_samplers with std::atexit -- after the CUDA runtime has registered
// its own teardown, so it runs before it -- and it stops and joins every live sampler.
std::mutex g_samplers_mu;
std::set<std::function<void()>*> g_samplers; // each entry stops one sampler
std::once_flag g_samplers_hook;

void stop_all_samplers() {
  std::vector<std::function<void()>*> live;
  {
    std::lock_guard<std::mutex> lk(g_samplers_mu);
    live.assign(g_samplers.begin(), g_samplers.end());
  }
  for (auto* stop : live)
    (*stop)();
}

struct Frame {
  uint64_t handle = 0;
  uint64_t owner = 0; // allocation id, kArenaOwner, or 0 when free
  uint32_t chunk = 0;
  uint64_t touch = 0;
  EventId last_use = 0;
  EventId ready = 0;      // recorded on the H2D stream after the frame's last upload
  bool used = false;      // has held data before (the next owner is a handle reuse)
  bool pending = false;   // last_use has been recorded
  bool uploading = false; // ready has been recorded and not yet observed complete
  bool prefetched = false; // made resident by a prefetch and not yet used by an operation
  bool referenced = false; // CLOCK's reference bit: used since the hand last passed
};

} // namespace

struct Runtime::Impl {
  RuntimeConfig cfg;
  std::unique_ptr<Device> dev;
  DeviceInfo info;
  xvram_session_telemetry_v1 t{};
  RuntimeExtra x;
  uint64_t cb = 0;       // chunk bytes
  uint64_t capacity = 0; // frames the budget allows now
  uint64_t max_capacity = 0; // frames of the budget at open (the scratch range is this big)
  // Free device memory sampled every budget_poll_ms by a thread of its own (see
  // apply_budget): the latest figure and how many samples have been taken.
  std::thread sampler;
  std::mutex sample_mu;
  std::condition_variable sample_cv;
  bool sampler_stop = false;
  uint64_t sampled_free = 0;
  uint64_t sample_seq = 0;  // samples taken by the sampler thread
  uint64_t applied_seq = 0; // the last of them apply_budget used

  void sampler_loop() {
    std::unique_lock<std::mutex> lk(sample_mu);
    while (!sampler_stop) {
      lk.unlock();
      uint64_t f = 0, total = 0;
      const bool ok = !dev->mem_get_info(&f, &total);
      lk.lock();
      if (ok) {
        sampled_free = f;
        ++sample_seq;
      }
      sample_cv.wait_for(lk, std::chrono::milliseconds(cfg.budget_poll_ms),
                         [this] { return sampler_stop; });
    }
  }
  ~Impl() { stop_sampler(); }
  // Registered in g_samplers while the sampler runs (see stop_all_samplers).
  std::function<void()> stop_hook = [this] { stop_sampler(); };
  std::mutex stop_mu; // serialises stop_sampler between the owner and the exit handler
  void start_sampler() {
    std::call_once(g_samplers_hook, [] { std::atexit(stop_all_samplers); });
    sampler = std::thread([this] { sampler_loop(); });
    std::lock_guard<std::mutex> lk(g_samplers_mu);
    g_samplers.insert(&stop_hook);
  }
  void stop_sampler() {
    std::lock_guard<std::mutex> stop_lk(stop_mu);
    if (!sampler.joinable())
      return;
    {
      std::lock_guard<std::mutex> lk(sample_mu);
      sampler_stop = true;
    }
    sample_cv.notify_all();
    sampler.join();
    std::lock_guard<std::mutex> lk(g_samplers_mu);
    g_samplers.erase(&stop_hook);
  }
  uint32_t growth_samples = 0;
  size_t clock_hand = 0; // CLOCK: where the next victim search starts
  std::vector<Frame> frames;
  std::map<uint64_t, Alloc> allocs;
  uint64_t next_id = 1;
  uint64_t clock = 0;
  StreamId s_h2d = 0, s_d2h = 0, s_compute = 0;
  StreamId s_compute2 = 0; // column blocks of a deferred GEMM alternate between the two
  EventId e_a = 0, e_b = 0;
  std::vector<EventId> event_pool;
  bool opened = false;

  // The C column blocks of the last deferred GEMM: byte ranges of one allocation and the
  // event after which each holds its final values.  Valid until the next operation that
  // launches device work or touches that allocation.
  struct BlockRange {
    uint64_t begin = 0, end = 0;
    EventId done = 0;
  };
  uint64_t staged_alloc = 0;
  std::vector<BlockRange> staged;
  bool status_unchecked = false; // a deferred GEMM's error word has not been read yet

  void clear_staged() {
    for (const BlockRange& r : staged)
      put_event(r.done);
    staged.clear();
    staged_alloc = 0;
  }
  // Reads the kernels' error word once a deferred GEMM's kernels have been waited for.
  Error check_deferred() {
    if (!status_unchecked)
      return {};
    status_unchecked = false;
    uint32_t word = 0;
    if (Error e = dev->kernel_status(s_compute, &word))
      return e;
    if (word)
      return make_error(XVRAM_STATUS_TIMEOUT, "executor", "sgemm",
                        "a kernel pipeline wait exceeded its limit");
    return {};
  }

  uint64_t chunk_len(const Alloc& a, uint64_t c) const {
    return std::min<uint64_t>(cb, a.bytes - c * cb);
  }

  Error get_event(EventId* e) {
    if (!event_pool.empty()) {
      *e = event_pool.back();
      event_pool.pop_back();
      return {};
    }
    return dev->event_create(e);
  }
  void put_event(EventId e) {
    if (e)
      event_pool.push_back(e);
  }

  void update_resident() {
    uint64_t owned = 0;
    for (const auto& f : frames)
      if (f.owner)
        ++owned;
    t.resident_bytes = owned * cb;
    t.resident_bytes_peak = std::max(t.resident_bytes_peak, t.resident_bytes);
  }

  Error ensure_backing(Alloc& a) {
    if (a.host)
      return {};
    if (cfg.host_store_cap_bytes && a.bytes > cfg.host_store_cap_bytes - std::min(
                                                  cfg.host_store_cap_bytes, x.host_backing_bytes))
      return make_error(XVRAM_STATUS_HOST_OUT_OF_MEMORY, "runtime", "host_backing",
                        "the allocation's host backing would exceed the host store cap");
    void* p = nullptr;
    if (Error e = dev->host_alloc(a.bytes, &p))
      return e;
    if (a.zero_fill)
      std::memset(p, 0, a.bytes);
    a.host = p;
    x.host_backing_bytes += a.bytes;
    x.host_backing_peak_bytes = std::max(x.host_backing_peak_bytes, x.host_backing_bytes);
    t.pinned_staging_bytes = x.host_backing_bytes;
    return {};
  }

  // Waits until the device is done with frame f: its last kernel use and its last upload.
  Error wait_idle(Frame& f) {
    if (f.pending) {
      if (Error e = dev->event_sync(f.last_use))
        return e;
      f.pending = false;
    }
    if (f.uploading) {
      if (Error e = dev->event_sync(f.ready))
        return e;
      f.uploading = false;
    }
    return {};
  }

  Error new_frame(Frame* f) {
    if (Error e = dev->handle_create(cb, &f->handle))
      return e;
    if (Error e = dev->event_create(&f->last_use)) {
      dev->handle_release(f->handle);
      return e;
    }
    if (Error e = dev->event_create(&f->ready)) {
      dev->event_destroy(f->last_use);
      dev->handle_release(f->handle);
      return e;
    }
    ++t.physical_handles_created;
    return {};
  }

  // Makes stream s wait for every upload still in flight into the chunks of `keep`.
  Error await_uploads(const std::set<std::pair<uint64_t, uint32_t>>& keep, StreamId s) {
    for (const auto& [id, c] : keep) {
      const int32_t fi = allocs.at(id).chunks[c].frame;
      if (fi >= 0 && frames[static_cast<size_t>(fi)].uploading)
        if (Error e = dev->stream_wait_event(s, frames[static_cast<size_t>(fi)].ready))
          return e;
    }
    return {};
  }

  // Takes frame `fi` away from its chunk: waits for the chunk's last device use, writes
  // it back to the host when the device copy is newer, and unmaps it.
  Error evict_frame(size_t fi) { return evict_frames({fi}); }

  // Takes the frames `fis` away from their chunks together: every dirty chunk's D2H copy is
  // issued first, then one wait covers them all, then the frames are unmapped.  Evicting
  // many frames (a streamed GEMM taking the whole pool, a budget shrink) thus costs one
  // round trip instead of one per dirty chunk, and the copies queue back to back on the
  // copy engine.  Frames that are free or hold the arena are skipped.
  Error evict_frames(const std::vector<size_t>& fis) {
    std::vector<size_t> owned, dirty;
    for (size_t fi : fis) {
      Frame& f = frames[fi];
      if (!f.owner || f.owner == kArenaOwner)
        continue;
      if (Error e = wait_idle(f))
        return e;
      owned.push_back(fi);
      Alloc& a = allocs.at(f.owner);
      Chunk& ch = a.chunks[f.chunk];
      if (ch.written && ch.dev_valid && !ch.backing_valid) {
        if (Error e = ensure_backing(a))
          return e;
        const uint64_t off = static_cast<uint64_t>(f.chunk) * cb;
        const uint64_t len = chunk_len(a, f.chunk);
        if (Error e = dev->copy_2d(reinterpret_cast<uint64_t>(a.host) + off, len, a.va + off,
                                   len, len, 1, CopyDir::d2h, s_d2h))
          return e;
        dirty.push_back(fi);
        t.bytes_d2h += len;
      }
    }
    if (!dirty.empty())
      if (Error e = dev->stream_sync(s_d2h))
        return e;
    for (size_t fi : dirty) {
      Frame& f = frames[fi];
      allocs.at(f.owner).chunks[f.chunk].backing_valid = true;
      ++t.dirty_evictions;
      ++t.writebacks_completed;
    }
    t.clean_evictions += owned.size() - dirty.size();
    for (size_t fi : owned) {
      Frame& f = frames[fi];
      Alloc& a = allocs.at(f.owner);
      Chunk& ch = a.chunks[f.chunk];
      if (Error e = dev->unmap(a.va + static_cast<uint64_t>(f.chunk) * cb, cb))
        return e;
      ++t.unmaps;
      ++t.event_boundaries; // a safe unmap: after the frame's completion events (wait_idle)
      ch.frame = -1;
      ch.dev_valid = false;
      f.owner = 0;
    }
    update_resident();
    return {};
  }

  // A free frame for a new owner; creates one while under capacity, else evicts the
  // least recently used frame whose chunk is not in `keep`.
  Error acquire_frame(const std::set<std::pair<uint64_t, uint32_t>>& keep, size_t* out) {
    for (size_t i = 0; i < frames.size(); ++i) {
      if (!frames[i].owner) {
        *out = i;
        if (frames[i].used)
          ++t.handle_reuses;
        return {};
      }
    }
    if (frames.size() < capacity) {
      Frame f;
      if (Error e = new_frame(&f))
        return e;
      frames.push_back(f);
      *out = frames.size() - 1;
      return {};
    }
    size_t victim = cfg.cache_policy == XVRAM_CACHE_POLICY_LRU ? lru_victim(keep)
                                                                 : clock_victim(keep);
    if (victim == frames.size())
      return make_error(XVRAM_STATUS_BUDGET_PRESSURE, "residency", "acquire_frame",
                        "every frame is pinned by the current operation");
    if (Error e = evict_frame(victim))
      return e;
    ++t.handle_reuses;
    *out = victim;
    return {};
  }

  bool evictable(const Frame& f, const std::set<std::pair<uint64_t, uint32_t>>& keep) const {
    return f.owner && f.owner != kArenaOwner && !keep.count({f.owner, f.chunk});
  }

  // CLOCK, as the reference's default policy (reference src/residency/policy.cpp:17-28,
  // 88-): frames fall into cost classes -- clean before dirty, a frame a prefetch filled
  // and nothing used yet before one in use -- and within the cheapest class the hand
  // sweeps from where it stopped, clearing reference bits, and takes the first frame whose
  // bit is already clear (second chance).  frames.size() if none is evictable.
  size_t clock_victim(const std::set<std::pair<uint64_t, uint32_t>>& keep) {
    const size_t n = frames.size();
    auto cost = [this](const Frame& f) {
      const Chunk& ch = allocs.at(f.owner).chunks[f.chunk];
      const bool dirty = ch.written && ch.dev_valid && !ch.backing_valid;
      return (dirty ? 3u : 0u) + (f.prefetched ? 1u : 2u);
    };
    unsigned cheapest = UINT_MAX;
    for (const Frame& f : frames)
      if (evictable(f, keep))
        cheapest = std::min(cheapest, cost(f));
    if (cheapest == UINT_MAX)
      return n;
    for (int pass = 0; pass < 2; ++pass)
      for (size_t scanned = 0; scanned < n; ++scanned) {
        const size_t i = (clock_hand + scanned) % n;
        Frame& f = frames[i];
        if (!evictable(f, keep) || cost(f) != cheapest)
          continue;
        if (f.referenced) {
          f.referenced = false;
          continue;
        }
        clock_hand = (i + 1) % n;
        return i;
      }
    return n;
  }

  // LRU: least recently used first, but a frame that a prefetch filled for an operation
  // that has not run yet goes only when nothing else can: evicting it would make that
  // operation upload it again.
  size_t lru_victim(const std::set<std::pair<uint64_t, uint32_t>>& keep) const {
    size_t victim = frames.size();
    for (int pass = 0; pass < 2 && victim == frames.size(); ++pass) {
      uint64_t oldest = UINT64_MAX;
      for (size_t i = 0; i < frames.size(); ++i) {
        const Frame& f = frames[i];
        if (f.owner == kArenaOwner || keep.count({f.owner, f.chunk}) ||
            (pass == 0 && f.prefetched))
          continue;
        if (f.touch < oldest) {
          oldest = f.touch;
          victim = i;
        }
      }
    }
    return victim;
  }

  // Maps chunk c of `a` if needed; uploads its host data when `upload` and the host copy
  // is the current one.  Uploads go on s_h2d.
  Error make_resident(Alloc& a, uint32_t c, bool upload,
                      const std::set<std::pair<uint64_t, uint32_t>>& keep, bool* uploaded) {
    Chunk& ch = a.chunks[c];
    if (ch.frame >= 0) {
      ++t.cache_hits;
      frames[static_cast<size_t>(ch.frame)].touch = ++clock;
      frames[static_cast<size_t>(ch.frame)].referenced = true;
      return {};
    }
    ++t.cache_misses;
    size_t fi = 0;
    if (Error e = acquire_frame(keep, &fi))
      return e;
    Frame& f = frames[fi];
    f.prefetched = false;
    const uint64_t off = static_cast<uint64_t>(c) * cb;
    if (Error e = dev->map(a.va + off, cb, f.handle))
      return e;
    ++t.mappings;
    ++t.set_access_calls;
    f.owner = a.id;
    f.chunk = c;
    f.used = true;
    f.touch = ++clock;
    f.referenced = true;
    ch.frame = static_cast<int32_t>(fi);
    ch.dev_valid = !ch.written; // undefined contents are valid anywhere
    if (upload && ch.written && ch.backing_valid && a.host) {
      const uint64_t len = chunk_len(a, c);
      if (Error e = dev->copy_2d(a.va + off, len, reinterpret_cast<uint64_t>(a.host) + off, len,
                                 len, 1, CopyDir::h2d, s_h2d))
        return e;
      t.bytes_h2d += len;
      ch.dev_valid = true;
      *uploaded = true;
      if (Error e = dev->event_record(f.ready, s_h2d))
        return e;
      f.uploading = true;
    } else if (!ch.written && a.zero_fill) {
      // A reused frame holds someone else's bytes: zero it (on the H2D stream, so a
      // partial write that follows lands on top).
      if (Error e = dev->memset_d32(a.va + off, 0, cb / 4, s_h2d))
        return e;
      *uploaded = true;
      if (Error e = dev->event_record(f.ready, s_h2d))
        return e;
      f.uploading = true;
    }
    update_resident();
    return {};
  }

  uint64_t free_frames() const {
    uint64_t n = capacity - frames.size();
    for (const auto& f : frames)
      if (!f.owner)
        ++n;
    return n;
  }

  Error evict_all() {
    std::vector<size_t> all(frames.size());
    for (size_t i = 0; i < all.size(); ++i)
      all[i] = i;
    return evict_frames(all);
  }

  // Live budget (reference src/residency/runtime.cpp:3213-3468): between operations, the
  // pool may hold at most (free device memory + its own frames - headroom), capped by the
  // budget it opened with.  A lower figure releases frames at once (free ones first, then
  // least recently used ones, written back when dirty); a higher one is taken only after
  // three consecutive samples agree.
  //
  // With budget_poll_ms > 0 the samples come from a thread of their own, every
  // budget_poll_ms, and an operation applies the newest one it has not applied yet:
  // cudaMemGetInfo usually returns in tens of microseconds but now and then takes tens of
  // milliseconds, which would otherwise stall the operation (and its kernels' launch).
  // With 0, every operation samples inline; refresh_budget (force) always does.
  Error apply_budget(bool force) {
    uint64_t free_b = 0, total_b = 0;
    if (!force && cfg.budget_poll_ms > 0) {
      std::lock_guard<std::mutex> lk(sample_mu);
      if (sample_seq == applied_seq)
        return {};
      t.budget_sample_count += sample_seq - applied_seq;
      applied_seq = sample_seq;
      free_b = sampled_free;
    } else {
      if (Error e = dev->mem_get_info(&free_b, &total_b))
        return e;
      ++t.budget_sample_count;
    }
    t.cuda_free_bytes_end = free_b;
    t.cuda_free_bytes_minimum = std::min(t.cuda_free_bytes_minimum, free_b);
    const uint64_t reclaimable = free_b + static_cast<uint64_t>(frames.size()) * cb;
    const uint64_t after = reclaimable > cfg.headroom_bytes ? reclaimable - cfg.headroom_bytes : 0;
    const uint64_t target = std::max<uint64_t>(2, std::min(after / cb, max_capacity));
    if (target < capacity) {
      growth_samples = 0;
      if (frames.size() > target) {
        // The frames to release, free ones first, then least recently used; their dirty
        // chunks are written back together.
        std::vector<size_t> order;
        for (size_t i = 0; i < frames.size(); ++i)
          if (frames[i].owner != kArenaOwner)
            order.push_back(i);
        std::stable_sort(order.begin(), order.end(), [this](size_t x, size_t y) {
          const uint64_t kx = frames[x].owner ? frames[x].touch + 1 : 0;
          const uint64_t ky = frames[y].owner ? frames[y].touch + 1 : 0;
          return kx < ky;
        });
        order.resize(std::min<size_t>(order.size(), frames.size() - target));
        if (Error e = evict_frames(order))
          return e;
      }
      while (frames.size() > target) {
        size_t victim = frames.size();
        for (size_t i = 0; i < frames.size() && victim == frames.size(); ++i)
          if (!frames[i].owner)
            victim = i;
        if (victim == frames.size())
          return make_error(XVRAM_STATUS_BUDGET_PRESSURE, "budget", "shrink",
                            "no frame can be released");
        if (Error e = wait_idle(frames[victim]))
          return e;
        Frame gone = frames[victim];
        if (Error e = dev->handle_release(gone.handle))
          return e;
        dev->event_destroy(gone.last_use);
        dev->event_destroy(gone.ready);
        ++t.physical_handles_released;
        // Keep the vector dense: the last frame takes the victim's index.
        if (victim + 1 != frames.size()) {
          frames[victim] = frames.back();
          const Frame& moved = frames[victim];
          if (moved.owner && moved.owner != kArenaOwner)
            allocs.at(moved.owner).chunks[moved.chunk].frame = static_cast<int32_t>(victim);
        }
        frames.pop_back();
      }
      capacity = target;
      ++t.budget_shrinks;
      t.cache_target_bytes = capacity * cb;
      t.cache_target_minimum_bytes = std::min(t.cache_target_minimum_bytes, capacity * cb);
      update_resident();
    } else if (target > capacity) {
      if (++growth_samples >= 3) {
        growth_samples = 0;
        capacity = target;
        ++t.budget_grows;
        t.cache_target_bytes = capacity * cb;
        t.cache_target_maximum_bytes = std::max(t.cache_target_maximum_bytes, capacity * cb);
      }
    } else {
      growth_samples = 0;
    }
    return {};
  }

  Error gemm_in_place(const GemmCall& call, Alloc& A, Alloc& B, Alloc& C,
                      const std::set<std::pair<uint64_t, uint32_t>>& keep, uint64_t ws);
  Error gemm_streamed(const GemmCall& call, Alloc& A, Alloc& B, Alloc& C);
  std::vector<int64_t> column_block_edges(const GemmCall& call) const;
  Error gemm_column_blocks(const GemmCall& call, const Alloc& A, const Alloc& B, const Alloc& C,
                           uint64_t ws_va, uint64_t ws, const std::vector<int64_t>& edges);
  void gemm_chunks(const GemmCall& call, std::set<std::pair<uint64_t, uint32_t>>* keep,
                   uint64_t* ws, bool* in_place);
  PlanLimits streamed_limits(const GemmCall& call) const;
  static PlanProblem plan_problem(const GemmCall& call);

  // The chunks [offset, offset + length) of allocation `a` covers.
  void range_chunks(const Alloc& a, uint64_t offset, uint64_t length,
                    std::set<std::pair<uint64_t, uint32_t>>* keep) const {
    for (uint64_t c = offset / cb; c <= (offset + length - 1) / cb; ++c)
      keep->insert({a.id, static_cast<uint32_t>(c)});
  }
  Error check_ranges(const std::vector<AccessRange>& ranges, const char* op) const {
    for (const AccessRange& r : ranges) {
      auto it = allocs.find(r.allocation_id);
      if (it == allocs.end() || !it->second.live || r.allocation_id == kScratchId)
        return make_error(XVRAM_STATUS_INVALID_ARGUMENT, "residency", op, "unknown allocation");
      if (r.length_bytes == 0 || r.offset_bytes > it->second.bytes ||
          r.length_bytes > it->second.bytes - r.offset_bytes || r.mode < 0 || r.mode > 2)
        return make_error(XVRAM_STATUS_INVALID_ARGUMENT, "residency", op,
                          "access range lies outside its allocation");
    }
    return {};
  }
  // Whether chunk c needs its current contents on the device for `ranges`: anything but
  // write-only ranges that cover the whole chunk.
  bool chunk_needs_upload(const Alloc& a, uint32_t c, const std::vector<AccessRange>& ranges) const {
    const uint64_t cbeg = static_cast<uint64_t>(c) * cb, cend = cbeg + chunk_len(a, c);
    for (const AccessRange& r : ranges) {
      if (r.allocation_id != a.id || r.offset_bytes >= cend ||
          r.offset_bytes + r.length_bytes <= cbeg)
        continue;
      if (r.mode != 2)
        return true;
    }
    uint64_t covered_to = cbeg; // write-only ranges: is the chunk covered completely?
    bool progress = true;
    while (progress && covered_to < cend) {
      progress = false;
      for (const AccessRange& r : ranges)
        if (r.allocation_id == a.id && r.offset_bytes <= covered_to &&
            r.offset_bytes + r.length_bytes > covered_to) {
          covered_to = r.offset_bytes + r.length_bytes;
          progress = true;
        }
    }
    return covered_to < cend;
  }
};

Runtime::Runtime() : impl_(std::make_unique<Impl>()) {}
Runtime::~Runtime() {
  if (impl_ && impl_->opened)
    (void)close();
}

const DeviceInfo& Runtime::info() const { return impl_->info; }
const xvram_session_telemetry_v1& Runtime::counters() const { return impl_->t; }
const RuntimeExtra& Runtime::extra() const { return impl_->x; }
uint64_t Runtime::chunk_bytes() const { return impl_->cb; }
uint64_t Runtime::frame_capacity() const { return impl_->capacity; }

Error Runtime::open(const RuntimeConfig& cfg, std::unique_ptr<Device> device) {
  Impl& m = *impl_;
  m.cfg = cfg;
  m.dev = std::move(device);
  m.t = xvram_session_telemetry_v1{};
  m.t.struct_size = sizeof(m.t);
  if (Error e = m.dev->open(cfg.device_ordinal, &m.info))
    return e;
  if (cfg.chunk_bytes == 0 || (cfg.chunk_bytes & (cfg.chunk_bytes - 1)) != 0 ||
      (m.info.vmm_granularity && cfg.chunk_bytes % m.info.vmm_granularity != 0))
    return make_error(XVRAM_STATUS_INVALID_ARGUMENT, "runtime", "open",
                      "chunk size must be a power of two multiple of the VMM granularity");
  m.cb = cfg.chunk_bytes;
  uint64_t free_b = 0, total_b = 0;
  if (Error e = m.dev->mem_get_info(&free_b, &total_b))
    return e;
  const uint64_t usable = free_b > cfg.headroom_bytes ? free_b - cfg.headroom_bytes : 0;
  const uint64_t budget = cfg.cache_target_bytes ? std::min(cfg.cache_target_bytes, usable) : usable;
  m.capacity = budget / m.cb;
  if (m.capacity < 2)
    return make_error(XVRAM_STATUS_DEVICE_OUT_OF_MEMORY, "runtime", "open",
                      "device budget is smaller than two frames");
  m.max_capacity = m.capacity;
  m.t.cache_target_bytes = m.capacity * m.cb;
  // Lowest and highest targets seen so far (reference src/residency/runtime.cpp:321,
  // :3415-3460).
  m.t.cache_target_minimum_bytes = m.capacity * m.cb;
  m.t.cache_target_maximum_bytes = m.capacity * m.cb;
  m.t.cuda_driver_version = static_cast<uint32_t>(m.info.driver_version);
  m.t.cuda_free_bytes_minimum = free_b;
  m.t.cuda_free_bytes_end = free_b;
  m.t.budget_sample_count = 1;
  m.t.flags = XVRAM_TELEMETRY_STABLE_VIRTUAL_ADDRESSES | XVRAM_TELEMETRY_NO_PHYSICAL_ALIASES;
  if (Error e = m.dev->stream_create(&m.s_h2d))
    return e;
  if (Error e = m.dev->stream_create(&m.s_d2h))
    return e;
  if (Error e = m.dev->stream_create(&m.s_compute))
    return e;
  if (Error e = m.dev->stream_create(&m.s_compute2))
    return e;
  if (Error e = m.dev->event_create(&m.e_a))
    return e;
  if (Error e = m.dev->event_create(&m.e_b))
    return e;
  {
    Alloc scratch;
    scratch.id = kScratchId;
    scratch.bytes = m.capacity * m.cb;
    scratch.reserved = scratch.bytes;
    if (Error e = m.dev->va_reserve(scratch.reserved, &scratch.va))
      return e;
    scratch.chunks.resize(static_cast<size_t>(m.capacity));
    m.allocs.emplace(kScratchId, std::move(scratch));
  }
  m.opened = true;
  if (cfg.budget_poll_ms > 0)
    m.start_sampler();
  return {};
}

Error Runtime::close() {
  Impl& m = *impl_;
  if (!m.opened)
    return {};
  Error first;
  auto keep = [&first](Error e) {
    if (e && !first)
      first = e;
  };
  m.stop_sampler();
  keep(m.dev->stream_sync(m.s_h2d));
  keep(m.dev->stream_sync(m.s_compute2));
  keep(m.dev->stream_sync(m.s_compute));
  keep(m.dev->stream_sync(m.s_d2h));
  keep(m.check_deferred());
  m.clear_staged();
  for (auto& [id, a] : m.allocs) {
    for (size_t c = 0; c < a.chunks.size(); ++c) {
      if (a.chunks[c].frame >= 0) {
        keep(m.dev->unmap(a.va + c * m.cb, m.cb));
        ++m.t.unmaps;
        ++m.t.event_boundaries; // after the stream drains above
        m.frames[static_cast<size_t>(a.chunks[c].frame)].owner = 0;
        a.chunks[c].frame = -1;
      }
    }
    if (a.host) {
      keep(m.dev->host_free(a.host));
      a.host = nullptr;
    }
    keep(m.dev->va_free(a.va, a.reserved));
    if (!a.live) { // a tombstoned range of a released allocation: current -> freed
      --m.x.retired_va_reservations;
      m.x.retired_va_bytes -= a.reserved;
      ++m.x.retired_va_reservations_freed;
      m.x.retired_va_bytes_freed += a.reserved;
    }
  }
  m.allocs.clear();
  for (auto& f : m.frames) {
    keep(m.dev->handle_release(f.handle));
    ++m.t.physical_handles_released;
    keep(m.dev->event_destroy(f.last_use));
    keep(m.dev->event_destroy(f.ready));
  }
  m.frames.clear();
  for (EventId e : m.event_pool)
    keep(m.dev->event_destroy(e));
  m.event_pool.clear();
  keep(m.dev->close());
  m.opened = false;
  m.t.resident_bytes = 0;
  return first;
}

Error Runtime::allocate(uint64_t bytes, uint64_t* id, uint64_t* va, bool zero_fill) {
  Impl& m = *impl_;
  if (bytes == 0 || bytes > UINT64_MAX - m.cb)
    return make_error(XVRAM_STATUS_INVALID_ARGUMENT, "runtime", "allocate", "invalid size");
  Alloc a;
  a.id = m.next_id++;
  a.bytes = bytes;
  a.zero_fill = zero_fill;
  a.reserved = round_up(bytes, m.cb);
  if (Error e = m.dev->va_reserve(a.reserved, &a.va))
    return e;
  a.chunks.resize(static_cast<size_t>(a.reserved / m.cb));
  *id = a.id;
  *va = a.va;
  m.allocs.emplace(a.id, std::move(a));
  return {};
}

Error Runtime::release(uint64_t id) {
  Impl& m = *impl_;
  auto it = m.allocs.find(id);
  if (it == m.allocs.end() || !it->second.live)
    return make_error(XVRAM_STATUS_INVALID_ARGUMENT, "runtime", "release", "unknown allocation");
  Alloc& a = it->second;
  if (m.staged_alloc == id)
    m.clear_staged();
  for (size_t c = 0; c < a.chunks.size(); ++c) {
    Chunk& ch = a.chunks[c];
    if (ch.frame < 0)
      continue;
    Frame& f = m.frames[static_cast<size_t>(ch.frame)];
    if (Error e = m.wait_idle(f))
      return e;
    if (Error e = m.dev->unmap(a.va + c * m.cb, m.cb))
      return e;
    ++m.t.unmaps;
    ++m.t.event_boundaries; // after wait_idle
    f.owner = 0;
    ch.frame = -1;
  }
  if (a.host) {
    if (Error e = m.dev->host_free(a.host))
      return e;
    m.x.host_backing_bytes -= a.bytes;
    m.t.pinned_staging_bytes = m.x.host_backing_bytes;
    a.host = nullptr;
  }
  // The address range stays reserved (tombstoned) until close so a freed pointer can
  // never alias a later allocation.
  a.live = false;
  a.chunks.clear();
  a.chunks.shrink_to_fit();
  ++m.x.retired_va_reservations;
  m.x.retired_va_bytes += a.reserved;
  m.update_resident();
  return {};
}

Error Runtime::write(uint64_t id, uint64_t offset, const void* src, uint64_t bytes) {
  Impl& m = *impl_;
  Alloc& a = m.allocs.at(id);
  if (bytes == 0)
    return {};
  if (m.staged_alloc == id)
    m.clear_staged();
  const uint32_t c0 = static_cast<uint32_t>(offset / m.cb);
  const uint32_t c1 = static_cast<uint32_t>((offset + bytes - 1) / m.cb);
  bool all_resident = true;
  uint64_t missing = 0;
  for (size_t c = 0; c < a.chunks.size(); ++c)
    if (a.chunks[c].frame < 0) {
      ++missing;
      if (c >= c0 && c <= c1)
        all_resident = false;
    }
  const bool to_device = all_resident || missing <= m.free_frames();
  if (to_device) {
    // Write-allocate: the data goes straight to HBM and the chunks become dirty.
    std::set<std::pair<uint64_t, uint32_t>> keep;
    for (uint32_t c = c0; c <= c1; ++c)
      keep.insert({a.id, c});
    bool uploaded = false;
    for (uint32_t c = c0; c <= c1; ++c) {
      const uint64_t cbeg = static_cast<uint64_t>(c) * m.cb;
      const uint64_t cend = cbeg + m.chunk_len(a, c);
      const bool covers = offset <= cbeg && offset + bytes >= cend;
      if (Error e = m.make_resident(a, c, !covers, keep, &uploaded))
        return e;
    }
    // The copy must follow any earlier device work on these frames and any upload.
    if (Error e = m.dev->event_record(m.e_a, m.s_compute))
      return e;
    if (Error e = m.dev->stream_wait_event(m.s_h2d, m.e_a))
      return e;
    if (Error e = m.dev->copy_2d(a.va + offset, bytes, reinterpret_cast<uint64_t>(src), bytes,
                                 bytes, 1, CopyDir::h2d, m.s_h2d))
      return e;
    if (Error e = m.dev->stream_sync(m.s_h2d))
      return e;
    m.t.bytes_h2d += bytes;
    for (uint32_t c = c0; c <= c1; ++c) {
      Chunk& ch = a.chunks[c];
      ch.written = true;
      ch.dev_valid = true;
      ch.backing_valid = false;
    }
    return {};
  }
  // Host path: bring any newer device data home first, then update the backing.
  for (uint32_t c = c0; c <= c1; ++c)
    if (a.chunks[c].frame >= 0)
      if (Error e = m.evict_frame(static_cast<size_t>(a.chunks[c].frame)))
        return e;
  if (Error e = m.ensure_backing(a))
    return e;
  // Chunks written for the first time but only partly: their other bytes are undefined,
  // which the backing already represents.
  parallel_memcpy(static_cast<char*>(a.host) + offset, src, bytes);
  for (uint32_t c = c0; c <= c1; ++c) {
    Chunk& ch = a.chunks[c];
    ch.written = true;
    ch.backing_valid = true;
    ch.dev_valid = false;
  }
  return {};
}

Error Runtime::read(uint64_t id, uint64_t offset, void* dst, uint64_t bytes) {
  Impl& m = *impl_;
  Alloc& a = m.allocs.at(id);
  if (bytes == 0)
    return {};
  const uint64_t end = offset + bytes;
  bool any_dma = false;
  // e_a follows all device work so far (a deferred GEMM's blocks are joined into s_compute).
  // A read of the C of the last deferred GEMM waits for each column block's own kernel
  // instead, so the first blocks come home while the last ones compute.
  if (Error e = m.dev->event_record(m.e_a, m.s_compute))
    return e;
  const bool by_block = m.staged_alloc == id && !m.staged.empty();
  if (!by_block)
    if (Error e = m.dev->stream_wait_event(m.s_d2h, m.e_a))
      return e;
  EventId waited = by_block ? 0 : m.e_a;
  // Chunks still being uploaded (a prefetch) are read after their upload.
  for (uint64_t c = offset / m.cb; c <= (end - 1) / m.cb; ++c) {
    const int32_t fi = a.chunks[static_cast<size_t>(c)].frame;
    if (fi >= 0 && m.frames[static_cast<size_t>(fi)].uploading)
      if (Error e = m.dev->stream_wait_event(m.s_d2h, m.frames[static_cast<size_t>(fi)].ready))
        return e;
  }
  uint64_t pos = offset;
  while (pos < end) {
    const uint32_t c = static_cast<uint32_t>(pos / m.cb);
    const uint64_t cend = std::min(end, static_cast<uint64_t>(c + 1) * m.cb);
    // Merge consecutive chunks with the same source into one copy.
    const Chunk& ch = a.chunks[c];
    const bool from_dev = ch.frame >= 0 && ch.dev_valid && ch.written;
    uint64_t run_end = cend;
    while (run_end < end) {
      const Chunk& nx = a.chunks[static_cast<size_t>(run_end / m.cb)];
      const bool nx_dev = nx.frame >= 0 && nx.dev_valid && nx.written;
      if (nx_dev != from_dev || nx.written != ch.written)
        break;
      run_end = std::min(end, (run_end / m.cb + 1) * m.cb);
    }
    EventId need = m.e_a;
    if (by_block) { // the piece ends at the edge of its column block
      for (const Impl::BlockRange& r : m.staged) {
        if (pos >= r.end)
          continue;
        if (pos >= r.begin) {
          run_end = std::min(run_end, r.end);
          need = r.done;
        } else {
          run_end = std::min(run_end, r.begin);
        }
        break;
      }
    }
    char* out = static_cast<char*>(dst) + (pos - offset);
    const uint64_t len = run_end - pos;
    if (from_dev) {
      if (waited != m.e_a && need != waited) {
        if (Error e = m.dev->stream_wait_event(m.s_d2h, need))
          return e;
        waited = need;
      }
      if (Error e = m.dev->copy_2d(reinterpret_cast<uint64_t>(out), len, a.va + pos, len, len, 1,
                                   CopyDir::d2h, m.s_d2h))
        return e;
      m.t.bytes_d2h += len;
      any_dma = true;
    } else if (ch.written && a.host) {
      parallel_memcpy(out, static_cast<const char*>(a.host) + pos, len);
    } else {
      std::memset(out, 0, len); // never written: contents are undefined, report zeros
    }
    pos = run_end;
  }
  if (any_dma)
    if (Error e = m.dev->stream_sync(m.s_d2h))
      return e;
  return m.check_deferred();
}

Error Runtime::synchronize() {
  Impl& m = *impl_;
  if (Error e = m.dev->stream_sync(m.s_h2d))
    return e;
  if (Error e = m.dev->stream_sync(m.s_compute2))
    return e;
  if (Error e = m.dev->stream_sync(m.s_compute))
    return e;
  if (Error e = m.dev->stream_sync(m.s_d2h))
    return e;
  return m.check_deferred();
}

Error Runtime::mem_get_info(uint64_t* free_bytes, uint64_t* total_bytes) {
  Impl& m = *impl_;
  if (Error e = m.dev->mem_get_info(free_bytes, total_bytes))
    return e;
  m.t.cuda_free_bytes_end = *free_bytes;
  m.t.cuda_free_bytes_minimum = std::min(m.t.cuda_free_bytes_minimum, *free_bytes);
  ++m.t.budget_sample_count;
  return {};
}

// The chunks an in-place GEMM pins (operands, then kernel workspace from the scratch
// pseudo-allocation) and the workspace bytes; in_place says whether they fit the pool.
void Runtime::Impl::gemm_chunks(const GemmCall& call, std::set<std::pair<uint64_t, uint32_t>>* keep,
                                uint64_t* ws, bool* in_place) {
  const MatrixRef* mats[3] = {&call.shape.a, &call.shape.b, &call.shape.c};
  for (int i = 0; i < 3; ++i) {
    uint64_t b = 0, e = 0;
    matrix_byte_span(*mats[i], &b, &e);
    for (uint64_t c = b / cb; c <= (e - 1) / cb; ++c)
      keep->insert({mats[i]->allocation_id, static_cast<uint32_t>(c)});
  }
  // The kernel's canonicalisation workspace comes out of the same frame budget.
  const GemmShape& sh = call.shape;
  *ws = dev->gemm_workspace(gemm_types(sh), sh.op_a, sh.op_b, static_cast<int64_t>(sh.m),
                            static_cast<int64_t>(sh.n), static_cast<int64_t>(sh.k));
  const uint64_t ws_chunks = (*ws + cb - 1) / cb;
  const size_t data_chunks = keep->size();
  for (uint64_t c = 0; c < ws_chunks && c < capacity; ++c)
    keep->insert({kScratchId, static_cast<uint32_t>(c)});
  *in_place = data_chunks + ws_chunks <= capacity;
}

PlanLimits Runtime::Impl::streamed_limits(const GemmCall& call) const {
  const GemmShape& s = call.shape;
  PlanLimits lim;
  lim.budget_bytes = capacity * cb;
  lim.quantum_bytes = cb;
  lim.flops_per_s = call.flops_per_s > 0 ? call.flops_per_s : cfg.flops_per_s;
  lim.h2d_bytes_per_s = cfg.h2d_bytes_per_s;
  lim.d2h_bytes_per_s = cfg.d2h_bytes_per_s;
  // Workspace per step is whatever the device's kernel asks for: transposes of K-major
  // panels (FFMA, FP64), the hi/lo split (tensor cores), widened FP16 / BF16 panels.
  const GemmTypes st = step_types(s);
  Device* d = dev.get();
  const int op_a = s.op_a, op_b = s.op_b;
  lim.step_workspace = [d, st, op_a, op_b](int64_t mb, int64_t nb, int64_t kb) {
    return d->gemm_workspace(st, op_a, op_b, mb, nb, kb);
  };
  lim.ab_bytes = static_cast<uint32_t>(element_bytes(s.a.dtype));
  lim.c_host_bytes = static_cast<uint32_t>(element_bytes(s.c.dtype));
  lim.c_acc_bytes = static_cast<uint32_t>(element_bytes(st.c));
  return lim;
}

PlanProblem Runtime::Impl::plan_problem(const GemmCall& call) {
  const GemmShape& s = call.shape;
  PlanProblem pp;
  pp.op_a = s.op_a;
  pp.op_b = s.op_b;
  pp.m = static_cast<int64_t>(s.m);
  pp.n = static_cast<int64_t>(s.n);
  pp.k = static_cast<int64_t>(s.k);
  pp.beta_nonzero = call.beta != 0.0;
  return pp;
}

Error Runtime::describe_gemm(const GemmCall& call, GemmLayout* out) {
  Impl& m = *impl_;
  std::set<std::pair<uint64_t, uint32_t>> keep;
  uint64_t ws = 0;
  bool in_place = false;
  m.gemm_chunks(call, &keep, &ws, &in_place);
  *out = GemmLayout{};
  if (in_place) {
    out->in_place = true;
    out->tile_m = call.shape.m;
    out->tile_n = call.shape.n;
    out->tile_k = call.shape.k;
    out->tiles = 1;
    out->working_set_bytes = keep.size() * m.cb;
    out->workspace_bytes = ws;
    return {};
  }
  Plan plan;
  const PlanStatus ps = make_panel_plan(Impl::plan_problem(call), m.streamed_limits(call), &plan);
  if (ps != PlanStatus::ok)
    return make_error(ps == PlanStatus::budget_too_small ? XVRAM_STATUS_BUDGET_PRESSURE
                                                         : XVRAM_STATUS_INVALID_ARGUMENT,
                      "planner", "make_panel_plan", "no panel geometry fits the device budget");
  out->tile_m = static_cast<uint64_t>(plan.mb);
  out->tile_n = static_cast<uint64_t>(plan.nb);
  out->tile_k = static_cast<uint64_t>(plan.kb);
  out->tiles = plan.steps.size();
  out->working_set_bytes = plan.slot_bytes * static_cast<uint64_t>(plan.panel_slots) +
                           plan.c_slot_bytes * static_cast<uint64_t>(plan.c_slots) +
                           plan.workspace_bytes;
  out->workspace_bytes = plan.workspace_bytes;
  return {};
}

Error Runtime::refresh_budget() { return impl_->apply_budget(true); }

Error Runtime::gemm(const GemmCall& call) {
  Impl& m = *impl_;
  const auto t0 = std::chrono::steady_clock::now();
  // Kernels address elements with their natural alignment (allocations start on frame
  // boundaries, so the offsets decide it).
  for (const MatrixRef* r : {&call.shape.a, &call.shape.b, &call.shape.c}) {
    const uint64_t es = element_bytes(r->dtype);
    if (es == 0 || r->offset_bytes % es != 0)
      return make_error(XVRAM_STATUS_INVALID_ARGUMENT, "executor", "gemm",
                        "a matrix offset is not a multiple of its element size");
  }
  m.clear_staged();
  if (Error e = m.apply_budget(false))
    return e;
  Alloc& A = m.allocs.at(call.shape.a.allocation_id);
  Alloc& B = m.allocs.at(call.shape.b.allocation_id);
  Alloc& C = m.allocs.at(call.shape.c.allocation_id);
  std::set<std::pair<uint64_t, uint32_t>> keep;
  uint64_t ws = 0;
  bool in_place = false;
  m.gemm_chunks(call, &keep, &ws, &in_place);
  const uint64_t retired_before = m.x.tiles_retired;
  Error err = in_place ? m.gemm_in_place(call, A, B, C, keep, ws) : m.gemm_streamed(call, A, B, C);
  m.x.last_gemm_ms =
      std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
  m.t.last_transaction_ms = m.x.last_gemm_ms;
  // One residency transaction per retired tile, as the reference counts them: at
  // quiescence transactions_completed equals tiles_retired (docs/cuda-compat.md:159).
  if (!err)
    m.t.transactions_completed += m.x.tiles_retired - retired_before;
  return err;
}

Error Runtime::Impl::gemm_in_place(const GemmCall& call, Alloc& A, Alloc& B, Alloc& C,
                                   const std::set<std::pair<uint64_t, uint32_t>>& keep,
                                   uint64_t ws) {
  bool uploaded = false;
  for (const auto& [id, c] : keep)
    if (Error e = make_resident(allocs.at(id), c, true, keep, &uploaded))
      return e;
  // Wait only for this GEMM's own chunks: uploads for later operations (prefetches) stay
  // in flight behind the kernel.
  if (Error e = await_uploads(keep, s_compute))
    return e;
  for (const auto& [id, c] : keep)
    frames[static_cast<size_t>(allocs.at(id).chunks[c].frame)].prefetched = false;
  const GemmShape& s = call.shape;
  ++x.tiles_submitted;
  ++x.gemm_in_place;
  const uint64_t ws_va = ws ? allocs.at(kScratchId).va : 0;
  const std::vector<int64_t> edges =
      call.defer_completion ? column_block_edges(call) : std::vector<int64_t>{};
  if (!edges.empty()) {
    if (Error e = gemm_column_blocks(call, A, B, C, ws_va, ws, edges))
      return e;
  } else if (Error e = dev->gemm(gemm_types(s), s.op_a, s.op_b, static_cast<int64_t>(s.m),
                                 static_cast<int64_t>(s.n), static_cast<int64_t>(s.k),
                                 call.alpha, A.va + s.a.offset_bytes,
                                 static_cast<int64_t>(s.a.ld), B.va + s.b.offset_bytes,
                                 static_cast<int64_t>(s.b.ld), call.beta,
                                 C.va + s.c.offset_bytes, static_cast<int64_t>(s.c.ld), ws_va, ws,
                                 s_compute)) {
    return e;
  }
  for (const auto& [id, c] : keep) {
    Frame& f = frames[static_cast<size_t>(allocs.at(id).chunks[c].frame)];
    if (Error e = dev->event_record(f.last_use, s_compute))
      return e;
    f.pending = true;
  }
  if (call.defer_completion) {
    // The frames stay pending (evicting or releasing them waits for last_use); C's
    // chunks hold the result from here on in stream order.
    for (const auto& [id, c] : keep)
      if (id == C.id) {
        Chunk& ch = C.chunks[c];
        ch.written = true;
        ch.dev_valid = true;
        ch.backing_valid = false;
      }
    status_unchecked = true;
    ++x.gemm_deferred;
    ++x.tiles_retired;
    return {};
  }
  uint32_t word = 0;
  if (Error e = dev->kernel_status(s_compute, &word))
    return e;
  if (word)
    return make_error(XVRAM_STATUS_TIMEOUT, "executor", "sgemm",
                      "a kernel pipeline wait exceeded its limit");
  for (const auto& [id, c] : keep) {
    if (id != C.id)
      continue;
    Chunk& ch = C.chunks[c];
    ch.written = true;
    ch.dev_valid = true;
    ch.backing_valid = false;
    frames[static_cast<size_t>(ch.frame)].pending = false;
  }
  for (const auto& [id, c] : keep)
    frames[static_cast<size_t>(allocs.at(id).chunks[c].frame)].pending = false;
  ++x.tiles_retired;
  return {};
}

// Column blocks for a deferred in-place GEMM, as the column edges [0, e1, ..., n]: whole
// 256-column tile columns, about one wave of tiles per block (128 x 256 tiles, one per SM,
// for FFMA; 256 x 256 tiles, one per SM pair, for TF32) and at most 8 blocks, so a block's
// D2H copy takes less time than the next block's kernels.  With 4 or more blocks the first
// and last are one tile column wide: the copies start sooner (the TF32 path, whose D2H
// outlasts its kernels) and the copy left after the last kernel is short (the FFMA path).
// Empty = launch it whole: FP16 / BF16 / FP64, or fewer than two waves of tiles.
std::vector<int64_t> Runtime::Impl::column_block_edges(const GemmCall& call) const {
  const GemmShape& s = call.shape;
  const GemmTypes t = gemm_types(s);
  if (t.ab != kFp32 || t.c != kFp32 || (t.compute != kStrictFp32 && t.compute != kTf32) ||
      s.k == 0)
    return {};
  const uint64_t tile_m = t.compute == kTf32 ? 256 : 128;
  const uint64_t tiles_m = (s.m + tile_m - 1) / tile_m, tiles_n = (s.n + 255) / 256;
  const uint64_t sms = static_cast<uint64_t>(std::max(1, info.sm_count));
  const uint64_t wave = t.compute == kTf32 ? std::max<uint64_t>(1, sms / 2) : sms;
  const uint64_t blocks = std::min<uint64_t>({8, tiles_n, tiles_m * tiles_n / wave});
  if (blocks < 2)
    return {};
  // Tile columns per block.
  std::vector<uint64_t> widths;
  const bool narrow_ends = blocks >= 4 && tiles_n >= blocks + 2;
  const uint64_t inner = narrow_ends ? blocks - 2 : blocks;
  const uint64_t inner_tiles = narrow_ends ? tiles_n - 2 : tiles_n;
  if (narrow_ends)
    widths.push_back(1);
  for (uint64_t i = 0; i < inner; ++i) // near-equal, wider ones first
    widths.push_back(inner_tiles / inner + (i < inner_tiles % inner ? 1 : 0));
  if (narrow_ends)
    widths.push_back(1);
  std::vector<int64_t> edges{0};
  for (uint64_t w : widths)
    edges.push_back(std::min<int64_t>(static_cast<int64_t>(s.n), edges.back() +
                                                                   static_cast<int64_t>(w * 256)));
  return edges;
}

// The deferred in-place GEMM as column blocks: the operands are prepared once in the
// workspace (the FFMA path's transposes, the TF32 path's hi/lo splits), then block j
// computes C's columns [edges[j], edges[j + 1]) on one of two streams, so a block's last
// wave overlaps the next block's first.  Every output is computed as in the unsplit launch, so
// the results are bit-identical.
Error Runtime::Impl::gemm_column_blocks(const GemmCall& call, const Alloc& A, const Alloc& B,
                                        const Alloc& C, uint64_t ws_va, uint64_t ws,
                                        const std::vector<int64_t>& edges) {
  const GemmShape& s = call.shape;
  const int64_t m = static_cast<int64_t>(s.m), n = static_cast<int64_t>(s.n),
                k = static_cast<int64_t>(s.k), ldc = static_cast<int64_t>(s.c.ld);
  PreparedGemm prep;
  if (Error e = dev->gemm_prepare(gemm_types(s), s.op_a, s.op_b, m, n, k, A.va + s.a.offset_bytes,
                                  static_cast<int64_t>(s.a.ld), B.va + s.b.offset_bytes,
                                  static_cast<int64_t>(s.b.ld), ws_va, ws, s_compute, &prep))
    return e;
  // The second stream starts after the uploads and the preparation.
  if (Error e = dev->event_record(e_b, s_compute))
    return e;
  if (Error e = dev->stream_wait_event(s_compute2, e_b))
    return e;
  clear_staged();
  staged_alloc = C.id;
  EventId last2 = 0;
  int64_t j = 0;
  for (; j + 1 < static_cast<int64_t>(edges.size()); ++j) {
    const int64_t j0 = edges[static_cast<size_t>(j)];
    const int64_t nj = edges[static_cast<size_t>(j) + 1] - j0;
    const StreamId st = (j & 1) ? s_compute2 : s_compute;
    const uint64_t col = s.c.offset_bytes + static_cast<uint64_t>(j0 * ldc) * 4;
    if (Error e = dev->gemm_block(prep, m, j0, nj, k, call.alpha, call.beta, C.va + col, ldc, st))
      return e;
    EventId done = 0;
    if (Error e = get_event(&done))
      return e;
    // Block ranges tile C's span without gaps: the rows below m of a block's last column
    // (ldc > m) belong to it, so a read of the whole span never waits for all blocks.
    const int64_t end_elem = j0 + nj < n ? (j0 + nj) * ldc : (n - 1) * ldc + m;
    staged.push_back({col, s.c.offset_bytes + static_cast<uint64_t>(end_elem) * 4, done});
    if (Error e = dev->event_record(done, st))
      return e;
    if (st == s_compute2)
      last2 = done;
  }
  // Later work on s_compute (and events recorded there) follows every block.
  if (last2)
    if (Error e = dev->stream_wait_event(s_compute, last2))
      return e;
  x.gemm_column_blocks += static_cast<uint64_t>(j);
  return {};
}

Error Runtime::Impl::gemm_streamed(const GemmCall& call, Alloc& A, Alloc& B, Alloc& C) {
  const GemmShape& s = call.shape;
  // 1. Every frame goes to the slot arena: write back and unmap all resident chunks.
  if (Error e = evict_all())
    return e;
  for (Alloc* a : {&A, &B, &C})
    if (Error e = ensure_backing(*a))
      return e;
  // 2. Plan against the whole pool.
  Plan plan;
  const PlanStatus ps = make_panel_plan(plan_problem(call), streamed_limits(call), &plan);
  if (ps != PlanStatus::ok)
    return make_error(ps == PlanStatus::budget_too_small ? XVRAM_STATUS_BUDGET_PRESSURE
                                                         : XVRAM_STATUS_INTERNAL,
                      "planner", "make_panel_plan", "no panel geometry fits the device budget");
  x.last_mb = plan.mb;
  x.last_nb = plan.nb;
  x.last_kb = plan.kb;
  x.last_steps = static_cast<int64_t>(plan.steps.size());
  x.last_panel_slots = plan.panel_slots;
  ++x.gemm_streamed;

  // 3. Slot arena: panel slots then C slots, each a run of whole frames.
  const uint64_t fps = plan.slot_bytes / cb;
  const uint64_t fpc = plan.c_slot_bytes / cb;
  const uint64_t nframes = fps * static_cast<uint64_t>(plan.panel_slots) +
                           fpc * static_cast<uint64_t>(plan.c_slots) + plan.workspace_bytes / cb;
  while (frames.size() < nframes) {
    Frame f;
    if (Error e = new_frame(&f))
      return e;
    frames.push_back(f);
  }
  uint64_t arena = 0;
  if (Error e = dev->va_reserve(nframes * cb, &arena))
    return e;
  std::vector<size_t> arena_frames;
  Error err;
  for (size_t i = 0; i < frames.size() && arena_frames.size() < nframes; ++i) {
    if (frames[i].owner)
      continue;
    if ((err = dev->map(arena + arena_frames.size() * cb, cb, frames[i].handle)))
      break;
    ++t.mappings;
    ++t.set_access_calls;
    if (frames[i].used)
      ++t.handle_reuses;
    frames[i].owner = kArenaOwner;
    frames[i].prefetched = false;
    frames[i].used = true;
    arena_frames.push_back(i);
  }
  update_resident();
  const uint64_t c_base = arena + fps * cb * static_cast<uint64_t>(plan.panel_slots);
  const uint64_t ws_base = c_base + fpc * cb * static_cast<uint64_t>(plan.c_slots);

  std::vector<EventId> ready(static_cast<size_t>(plan.panel_slots)),
      used(static_cast<size_t>(plan.panel_slots)), c_ready(static_cast<size_t>(plan.c_slots)),
      c_done(static_cast<size_t>(plan.c_slots)), c_wb(static_cast<size_t>(plan.c_slots));
  std::vector<char> used_rec(static_cast<size_t>(plan.panel_slots), 0),
      wb_rec(static_cast<size_t>(plan.c_slots), 0);
  for (auto* v : {&ready, &used, &c_ready, &c_done, &c_wb})
    for (auto& e : *v)
      if (!err)
        err = get_event(&e);

  const uint64_t ha = reinterpret_cast<uint64_t>(A.host) + s.a.offset_bytes;
  const uint64_t hb = reinterpret_cast<uint64_t>(B.host) + s.b.offset_bytes;
  const uint64_t hc = reinterpret_cast<uint64_t>(C.host) + s.c.offset_bytes;
  const int64_t M = static_cast<int64_t>(s.m), N = static_cast<int64_t>(s.n),
                K = static_cast<int64_t>(s.k);
  const uint64_t lda = s.a.ld, ldb = s.b.ld, ldc = s.c.ld;
  const int64_t mb = plan.mb, nb = plan.nb, kb = plan.kb;
  // Element bytes of A / B and of C as stored; the C slot accumulates in step.c's type,
  // with a staging copy in the stored type at c_stage_offset when that is narrower.
  const uint64_t ea = element_bytes(s.a.dtype), ec = element_bytes(s.c.dtype);
  const GemmTypes step = step_types(s);
  const bool c_staged = plan.c_stage_offset != 0;
  const auto slot_va = [&](int32_t slot) {
    return arena + static_cast<uint64_t>(slot) * fps * cb;
  };

  // 4. Replay the plan.
  for (size_t si = 0; si < plan.steps.size() && !err; ++si) {
    const PlanStep& st = plan.steps[si];
    const int64_t m0 = static_cast<int64_t>(st.bm) * mb, n0 = static_cast<int64_t>(st.bn) * nb,
                  k0 = static_cast<int64_t>(st.bk) * kb;
    const int64_t mr = std::min(mb, M - m0), nr = std::min(nb, N - n0), kr = std::min(kb, K - k0);
    for (uint32_t li = st.load_begin; li < st.load_begin + st.load_count && !err; ++li) {
      const PanelLoad& ld = plan.loads[li];
      const size_t sl = static_cast<size_t>(ld.slot);
      // A slot is refilled only after the event of its last GEMM (device-side ordering;
      // the slot's frames stay mapped).
      if (used_rec[sl]) {
        if ((err = dev->stream_wait_event(s_h2d, used[sl])))
          break;
      }
      const int64_t lk0 = static_cast<int64_t>(ld.kpanel) * kb;
      const int64_t lkr = std::min(kb, K - lk0);
      uint64_t src = 0, spitch = 0, width = 0, height = 0, dpitch = 0;
      if (ld.operand == 0) {
        const int64_t lm0 = static_cast<int64_t>(ld.block) * mb, lmr = std::min(mb, M - lm0);
        if (s.op_a == 0) { // A is m x k: kr columns of mr floats
          src = ha + (static_cast<uint64_t>(lm0) + static_cast<uint64_t>(lk0) * lda) * ea;
          width = static_cast<uint64_t>(lmr) * ea;
          height = static_cast<uint64_t>(lkr);
          dpitch = static_cast<uint64_t>(mb) * ea;
        } else { // A is k x m: mr columns of kr floats
          src = ha + (static_cast<uint64_t>(lk0) + static_cast<uint64_t>(lm0) * lda) * ea;
          width = static_cast<uint64_t>(lkr) * ea;
          height = static_cast<uint64_t>(lmr);
          dpitch = static_cast<uint64_t>(kb) * ea;
        }
        spitch = lda * ea;
      } else {
        const int64_t ln0 = static_cast<int64_t>(ld.block) * nb, lnr = std::min(nb, N - ln0);
        if (s.op_b == 0) { // B is k x n: nr columns of kr floats
          src = hb + (static_cast<uint64_t>(lk0) + static_cast<uint64_t>(ln0) * ldb) * ea;
          width = static_cast<uint64_t>(lkr) * ea;
          height = static_cast<uint64_t>(lnr);
          dpitch = static_cast<uint64_t>(kb) * ea;
        } else { // B is n x k: kr columns of nr floats
          src = hb + (static_cast<uint64_t>(ln0) + static_cast<uint64_t>(lk0) * ldb) * ea;
          width = static_cast<uint64_t>(lnr) * ea;
          height = static_cast<uint64_t>(lkr);
          dpitch = static_cast<uint64_t>(nb) * ea;
        }
        spitch = ldb * ea;
      }
      if ((err = dev->copy_2d(slot_va(ld.slot), dpitch, src, spitch, width, height, CopyDir::h2d,
                              s_h2d)))
        break;
      if ((err = dev->event_record(ready[sl], s_h2d)))
        break;
      t.bytes_h2d += width * height;
      ++t.cache_misses;
      if (ld.evicts)
        ++x.panel_slot_refills;
    }
    if (err)
      break;
    t.cache_hits += 2 - st.load_count;
    const size_t cs = static_cast<size_t>(st.c_slot);
    const uint64_t cva = c_base + static_cast<uint64_t>(cs) * fpc * cb;
    const uint64_t cstage = cva + plan.c_stage_offset;
    const uint64_t c_host = hc + (static_cast<uint64_t>(m0) + static_cast<uint64_t>(n0) * ldc) * ec;
    double beta_eff = 1.0;
    if (st.first_k) {
      beta_eff = call.beta;
      if (call.beta != 0.0) {
        if (wb_rec[cs] && (err = dev->stream_wait_event(s_h2d, c_wb[cs])))
          break;
        if ((err = dev->copy_2d(c_staged ? cstage : cva, static_cast<uint64_t>(mb) * ec, c_host,
                                ldc * ec, static_cast<uint64_t>(mr) * ec,
                                static_cast<uint64_t>(nr), CopyDir::h2d, s_h2d)))
          break;
        t.bytes_h2d += static_cast<uint64_t>(mr) * static_cast<uint64_t>(nr) * ec;
        if ((err = dev->event_record(c_ready[cs], s_h2d)) ||
            (err = dev->stream_wait_event(s_compute, c_ready[cs])))
          break;
        if (c_staged && (err = dev->convert(s.c.dtype, cstage, mb, step.c, cva, mb, mr, nr,
                                            s_compute)))
          break;
      } else if (wb_rec[cs] && (err = dev->stream_wait_event(s_compute, c_wb[cs]))) {
        break;
      }
    }
    if ((err = dev->stream_wait_event(s_compute, ready[static_cast<size_t>(st.slot_a)])) ||
        (err = dev->stream_wait_event(s_compute, ready[static_cast<size_t>(st.slot_b)])))
      break;
    const int64_t lda_s = s.op_a == 0 ? mb : kb;
    const int64_t ldb_s = s.op_b == 0 ? kb : nb;
    if ((err = dev->gemm(step, s.op_a, s.op_b, mr, nr, kr, call.alpha, slot_va(st.slot_a),
                         lda_s, slot_va(st.slot_b), ldb_s, beta_eff, cva, mb,
                         plan.workspace_bytes ? ws_base : 0, plan.workspace_bytes, s_compute)))
      break;
    ++x.tiles_submitted;
    for (int32_t sl : {st.slot_a, st.slot_b}) {
      if ((err = dev->event_record(used[static_cast<size_t>(sl)], s_compute)))
        break;
      used_rec[static_cast<size_t>(sl)] = 1;
    }
    if (err)
      break;
    if (st.last_k) {
      if (c_staged &&
          (err = dev->convert(step.c, cva, mb, s.c.dtype, cstage, mb, mr, nr, s_compute)))
        break;
      if ((err = dev->event_record(c_done[cs], s_compute)) ||
          (err = dev->stream_wait_event(s_d2h, c_done[cs])) ||
          (err = dev->copy_2d(c_host, ldc * ec, c_staged ? cstage : cva,
                              static_cast<uint64_t>(mb) * ec, static_cast<uint64_t>(mr) * ec,
                              static_cast<uint64_t>(nr), CopyDir::d2h, s_d2h)) ||
          (err = dev->event_record(c_wb[cs], s_d2h)))
        break;
      wb_rec[cs] = 1;
      t.bytes_d2h += static_cast<uint64_t>(mr) * static_cast<uint64_t>(nr) * ec;
      // A finished C tile leaves its slot dirty-for-home: one dirty eviction written back,
      // so dirty_evictions == writebacks_completed as in the reference's accounting.
      ++t.dirty_evictions;
      ++t.writebacks_completed;
    }
  }

  // 5. Drain, check the kernels' error word, dissolve the arena.
  Error drain;
  if (!(drain = dev->stream_sync(s_h2d)) && !(drain = dev->stream_sync(s_compute)))
    drain = dev->stream_sync(s_d2h);
  if (!err && drain)
    err = drain;
  if (!err) {
    uint32_t word = 0;
    err = dev->kernel_status(s_compute, &word);
    if (!err && word)
      err = make_error(XVRAM_STATUS_TIMEOUT, "executor", "sgemm",
                       "a kernel pipeline wait exceeded its limit");
  }
  if (!err)
    x.tiles_retired += plan.steps.size();
  for (size_t i = 0; i < arena_frames.size(); ++i) {
    Error e = dev->unmap(arena + i * cb, cb);
    if (e && !err)
      err = e;
    ++t.unmaps;
    ++t.event_boundaries; // unmapped after the drain above
    frames[arena_frames[i]].owner = 0;
  }
  if (Error e = dev->va_free(arena, nframes * cb); e && !err)
    err = e;
  for (auto* v : {&ready, &used, &c_ready, &c_done, &c_wb})
    for (auto& e : *v)
      put_event(e);
  update_resident();
  if (err)
    return err;
  // C's rows/columns inside the matrix are now current in the host backing.
  uint64_t cb0 = 0, ce0 = 0;
  matrix_byte_span(s.c, &cb0, &ce0);
  for (uint64_t c = cb0 / cb; c <= (ce0 - 1) / cb; ++c) {
    Chunk& ch = C.chunks[static_cast<size_t>(c)];
    ch.written = true;
    ch.backing_valid = true;
    ch.dev_valid = false;
  }
  return {};
}

} // namespace xvram

namespace xvram {

bool Runtime::live(uint64_t id) const {
  auto it = impl_->allocs.find(id);
  return it != impl_->allocs.end() && it->second.live && id != kScratchId;
}

uint64_t Runtime::allocation_bytes(uint64_t id) const {
  auto it = impl_->allocs.find(id);
  return it == impl_->allocs.end() ? 0 : it->second.bytes;
}

Error Runtime::prefetch(const std::vector<AccessRange>& ranges) {
  Impl& m = *impl_;
  if (Error e = m.check_ranges(ranges, "prefetch"))
    return e;
  if (Error e = m.apply_budget(false))
    return e;
  std::set<std::pair<uint64_t, uint32_t>> keep;
  for (const AccessRange& r : ranges)
    m.range_chunks(m.allocs.at(r.allocation_id), r.offset_bytes, r.length_bytes, &keep);
  if (keep.size() > m.capacity)
    return make_error(XVRAM_STATUS_BUDGET_PRESSURE, "residency", "prefetch",
                      "the ranges exceed the device budget");
  bool uploaded = false;
  for (const auto& [id, c] : keep) {
    Alloc& a = m.allocs.at(id);
    if (Error e = m.make_resident(a, c, m.chunk_needs_upload(a, c, ranges), keep, &uploaded))
      return e;
    m.frames[static_cast<size_t>(a.chunks[c].frame)].prefetched = true;
  }
  return {};
}

Error Runtime::transaction(const std::vector<AccessRange>& ranges, uint64_t workspace_bytes,
                           const TransactionBody& body) {
  Impl& m = *impl_;
  const auto t0 = std::chrono::steady_clock::now();
  if (Error e = m.check_ranges(ranges, "transaction"))
    return e;
  m.clear_staged();
  if (Error e = m.apply_budget(false))
    return e;
  std::set<std::pair<uint64_t, uint32_t>> keep;
  for (const AccessRange& r : ranges)
    m.range_chunks(m.allocs.at(r.allocation_id), r.offset_bytes, r.length_bytes, &keep);
  const uint64_t ws_chunks = (workspace_bytes + m.cb - 1) / m.cb;
  if (keep.size() + ws_chunks > m.capacity)
    return make_error(XVRAM_STATUS_BUDGET_PRESSURE, "residency", "transaction",
                      "the ranges and workspace exceed the device budget");
  for (uint64_t c = 0; c < ws_chunks; ++c)
    keep.insert({kScratchId, static_cast<uint32_t>(c)});
  bool uploaded = false;
  for (const auto& [id, c] : keep) {
    Alloc& a = m.allocs.at(id);
    const bool upload = id != kScratchId && m.chunk_needs_upload(a, c, ranges);
    if (Error e = m.make_resident(a, c, upload, keep, &uploaded))
      return e;
  }
  if (Error e = m.await_uploads(keep, m.s_compute))
    return e;
  for (const auto& [id, c] : keep)
    m.frames[static_cast<size_t>(m.allocs.at(id).chunks[c].frame)].prefetched = false;
  std::vector<ResolvedRange> resolved;
  resolved.reserve(ranges.size());
  for (const AccessRange& r : ranges)
    resolved.push_back(ResolvedRange{r.allocation_id, r.offset_bytes, r.length_bytes,
                                     m.allocs.at(r.allocation_id).va + r.offset_bytes, r.mode});
  const uint64_t ws_addr = ws_chunks ? m.allocs.at(kScratchId).va : 0;
  Error body_error = body(resolved, ws_addr, workspace_bytes, m.dev->native_stream(m.s_compute));
  // Whatever the body enqueued may have written its read-write and write-only ranges.
  for (const auto& [id, c] : keep) {
    Frame& f = m.frames[static_cast<size_t>(m.allocs.at(id).chunks[c].frame)];
    if (Error e = m.dev->event_record(f.last_use, m.s_compute))
      return e;
    f.pending = true;
  }
  for (const AccessRange& r : ranges) {
    if (r.mode == 0)
      continue;
    Alloc& a = m.allocs.at(r.allocation_id);
    for (uint64_t c = r.offset_bytes / m.cb; c <= (r.offset_bytes + r.length_bytes - 1) / m.cb;
         ++c) {
      Chunk& ch = a.chunks[static_cast<size_t>(c)];
      ch.written = true;
      ch.dev_valid = true;
      ch.backing_valid = false;
    }
  }
  if (Error e = m.dev->stream_sync(m.s_compute))
    return body_error ? body_error : e;
  for (const auto& [id, c] : keep)
    m.frames[static_cast<size_t>(m.allocs.at(id).chunks[c].frame)].pending = false;
  m.t.last_transaction_ms =
      std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
  if (body_error)
    return body_error;
  ++m.t.transactions_completed;
  return {};
}

} // namespace xvram
