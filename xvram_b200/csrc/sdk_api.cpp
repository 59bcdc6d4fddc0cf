// sdk_api.cpp -- xvram_get_api: the SDK v1 function table over the residency runtime.
//
// Behaviour follows the reference SDK (reference src/sdk/api.cpp:100-1035 argument
// checks and handle lifetimes, src/sdk/runtime.cpp:144-280 operations, :395-500
// prefetch and transactions, :1175-1364 GEMM plans):
//   * every public structure is checked for its v1 size (INCOMPATIBLE_ABI when smaller)
//     and for zero flags / reserved fields (INVALID_ARGUMENT);
//   * a session owns one worker thread that opens the runtime (so the session's device is
//     current there) and runs every operation in submission order; synchronous calls
//     (allocation_*, gemm_plan_create, telemetry) are queued behind earlier operations;
//   * an operation can be cancelled while queued; once running, cancel answers BUSY;
//   * deadlines count from submission and are checked before the operation starts and
//     again before a transaction's callback runs (TIMEOUT);
//   * a failure that may leave device state undefined (CUDA errors, kernel wait limits,
//     internal errors) poisons the session: later operations fail with POISONED.
// What differs, by design of this implementation:
//   * GEMMs run on this library's sm_100a kernels, for the reference's type combinations
//     (FP32, FP16 / BF16 inputs with strict FP32 arithmetic, FP64).  Row-major matrices
//     are handled as the transposed column-major view (the operation flips; a row-major C
//     swaps the operands).  FP32_TF32 (and AUTO on FP32 data, as in the reference) runs
//     the three-term TF32 tensor-core kernel, which is FP32-accurate where the
//     reference's single-pass TF32 is not.
//   * Tile hints are ignored: the panel planner picks the geometry from the budget.
#include "xvram/xvram.h"

#include "device.hpp"
#include "runtime.hpp"
#include "status.hpp"
#include "validate.hpp"

#include <algorithm>
#include <atomic>
#include <chrono>
#include <cmath>
#include <condition_variable>
#include <cstring>
#include <deque>
#include <functional>
#include <limits>
#include <memory>
#include <mutex>
#include <new>
#include <thread>
#include <vector>

namespace xvram {
namespace sdk {
namespace {

using Clock = std::chrono::steady_clock;

Error invalid(const char* op, const char* msg) {
  return make_error(XVRAM_STATUS_INVALID_ARGUMENT, "sdk", op, msg);
}
Error incompatible(const char* op, const char* msg) {
  return make_error(XVRAM_STATUS_INCOMPATIBLE_ABI, "sdk", op, msg);
}

template <class T> bool has_v1_size(const T* v) { return v && v->struct_size >= sizeof(T); }
template <class T, size_t N> bool all_zero(const T (&v)[N]) {
  return std::all_of(std::begin(v), std::end(v), [](T x) { return x == 0; });
}

bool poisons(const Error& e) {
  switch (e.status) {
  case XVRAM_STATUS_CUDA_ERROR:
  case XVRAM_STATUS_INTERNAL:
  case XVRAM_STATUS_CORRUPTION:
  case XVRAM_STATUS_CLEANUP_FAILED:
    return true;
  default:
    return false;
  }
}

// Deadlines are milliseconds after submission; they must be representable on the clock.
bool deadline_ok(uint64_t deadline_ms) {
  if (deadline_ms == 0)
    return true;
  const auto left = std::chrono::duration_cast<std::chrono::milliseconds>(
                        Clock::time_point::max() - Clock::now())
                        .count();
  return left > 0 && deadline_ms <= static_cast<uint64_t>(left);
}

// ------------------------------------------------------------------------ operation
class Op {
public:
  Op(uint64_t id, uint64_t units, uint64_t deadline_ms) : submitted_(Clock::now()) {
    info_ = XVRAM_OPERATION_INFO_V1_INIT;
    info_.operation_id = id;
    info_.units_total = units;
    if (deadline_ms) {
      has_deadline_ = true;
      deadline_ = submitted_ + std::chrono::milliseconds(deadline_ms);
    }
  }

  std::function<Error(Op&)> body;
  bool closes_session = false; // runs even on a poisoned session
  bool read_only = false;      // diagnostics (telemetry): also run on a poisoned session

  bool expired() const { return has_deadline_ && Clock::now() >= deadline_; }
  Error deadline_error(const char* stage, const char* op) const {
    return expired() ? make_error(XVRAM_STATUS_TIMEOUT, stage, op,
                                  "the operation's deadline passed before a safe launch point")
                     : Error{};
  }
  uint64_t id() const { return info_.operation_id; }

  // Queued -> running, unless it was cancelled or its deadline passed in the queue.
  bool begin() {
    std::lock_guard<std::mutex> lk(mu_);
    if (cancel_requested_) {
      info_.state = XVRAM_OPERATION_CANCELLED;
      info_.result = XVRAM_STATUS_CANCELLED;
      error_ = make_error(XVRAM_STATUS_CANCELLED, "operation", "cancel", "operation cancelled");
      cv_.notify_all();
      return false;
    }
    if (expired()) {
      info_.state = XVRAM_OPERATION_FAILED;
      info_.result = XVRAM_STATUS_TIMEOUT;
      error_ = make_error(XVRAM_STATUS_TIMEOUT, "operation", "queue_deadline",
                          "the operation's deadline passed while it was queued");
      info_.elapsed_ms =
          std::chrono::duration<double, std::milli>(Clock::now() - submitted_).count();
      cv_.notify_all();
      return false;
    }
    info_.state = XVRAM_OPERATION_RUNNING;
    started_ = Clock::now();
    return true;
  }

  void finish(const Error& e, const xvram_session_telemetry_v1& before,
              const xvram_session_telemetry_v1& after) {
    std::lock_guard<std::mutex> lk(mu_);
    error_ = e;
    info_.result = e.status;
    info_.state = e ? XVRAM_OPERATION_FAILED : XVRAM_OPERATION_COMPLETED;
    if (!e)
      info_.units_completed = info_.units_total;
    info_.elapsed_ms = std::chrono::duration<double, std::milli>(Clock::now() - started_).count();
    info_.bytes_h2d = after.bytes_h2d - before.bytes_h2d;
    info_.bytes_d2h = after.bytes_d2h - before.bytes_d2h;
    info_.cache_hits = after.cache_hits - before.cache_hits;
    info_.cache_misses = after.cache_misses - before.cache_misses;
    cv_.notify_all();
  }

  void poll(xvram_operation_info_v1* out) {
    std::lock_guard<std::mutex> lk(mu_);
    *out = info_;
  }

  Error wait(uint64_t timeout_ms, xvram_operation_info_v1* out) {
    std::unique_lock<std::mutex> lk(mu_);
    const auto done = [this] {
      return info_.state == XVRAM_OPERATION_COMPLETED ||
             info_.state == XVRAM_OPERATION_CANCELLED || info_.state == XVRAM_OPERATION_FAILED;
    };
    bool ok = true;
    if (timeout_ms == XVRAM_TIMEOUT_INFINITE)
      cv_.wait(lk, done);
    else
      ok = cv_.wait_for(lk, std::chrono::milliseconds(timeout_ms), done);
    if (out)
      *out = info_;
    return ok ? Error{}
              : make_error(XVRAM_STATUS_TIMEOUT, "operation", "wait",
                           "the operation did not finish before the timeout");
  }

  Error cancel() {
    std::lock_guard<std::mutex> lk(mu_);
    if (info_.state == XVRAM_OPERATION_QUEUED) {
      cancel_requested_ = true;
      return {};
    }
    if (info_.state == XVRAM_OPERATION_RUNNING)
      return make_error(XVRAM_STATUS_BUSY, "operation", "cancel",
                        "a running device operation cannot be cancelled safely");
    return {};
  }

  Error error() {
    std::lock_guard<std::mutex> lk(mu_);
    return error_;
  }

private:
  std::mutex mu_;
  std::condition_variable cv_;
  xvram_operation_info_v1 info_{};
  Error error_;
  bool cancel_requested_ = false;
  bool has_deadline_ = false;
  Clock::time_point submitted_, started_, deadline_;
};

// -------------------------------------------------------------------------- session
class Session {
public:
  explicit Session(const xvram_session_config_v1& cfg) : cfg_(cfg) {
    telemetry_.struct_size = sizeof(telemetry_);
  }
  ~Session() { stop_worker(); }
  Session(const Session&) = delete;
  Session& operator=(const Session&) = delete;

  const xvram_session_config_v1& config() const { return cfg_; }
  Runtime& runtime() { return rt_; }
  uint64_t chunk_bytes() const { return chunk_bytes_; }
  std::atomic<bool> closed{false};

  Error start() {
    worker_ = std::thread([this] { loop(); });
    Error e = invoke_sync([this]() -> Error {
      RuntimeConfig rc;
      rc.device_ordinal = cfg_.device_ordinal;
      rc.chunk_bytes = cfg_.chunk_size_bytes;
      rc.cache_target_bytes = cfg_.cache_target_bytes;
      rc.headroom_bytes = cfg_.device_headroom_bytes;
      rc.budget_poll_ms = cfg_.budget_poll_ms;
      rc.cache_policy = cfg_.cache_policy;
      DeviceFactory factory = device_factory();
      std::unique_ptr<Device> dev = factory ? factory() : nullptr;
      if (!dev)
        return make_error(XVRAM_STATUS_UNAVAILABLE, "session", "open", "no device backend");
      if (Error oe = rt_.open(rc, std::move(dev)))
        return oe;
      opened_ = true;
      chunk_bytes_ = rt_.chunk_bytes();
      return {};
    });
    if (e)
      stop_worker();
    return e;
  }

  Error enqueue(std::function<Error(Op&)> body, uint64_t units, uint64_t deadline_ms,
                std::shared_ptr<Op>* out, bool read_only = false) {
    std::lock_guard<std::mutex> lk(qmu_);
    if (closing_)
      return make_error(XVRAM_STATUS_CLOSED, "session", "submit", "the session is closed");
    auto op = std::make_shared<Op>(next_op_++, units, deadline_ms);
    op->body = std::move(body);
    op->read_only = read_only; // before the worker can see it
    queue_.push_back(op);
    qcv_.notify_all();
    *out = std::move(op);
    return {};
  }

  // True on the session's worker thread, i.e. inside a transaction callback.
  bool on_worker() const { return worker_.get_id() == std::this_thread::get_id(); }

  Error invoke_sync(std::function<Error()> fn, bool read_only = false) {
    if (on_worker()) // queued behind the running callback, it could never run
      return make_error(XVRAM_STATUS_BUSY, "session", "reentrant_call",
                        "synchronous SDK calls are not allowed from a transaction callback");
    std::shared_ptr<Op> op;
    if (Error e = enqueue([fn = std::move(fn)](Op&) { return fn(); }, 1, 0, &op, read_only))
      return e;
    (void)op->wait(XVRAM_TIMEOUT_INFINITE, nullptr);
    return op->error();
  }

  Error drain(uint64_t timeout_ms) {
    if (on_worker())
      return make_error(XVRAM_STATUS_BUSY, "session", "reentrant_call",
                        "session_drain is not allowed from a transaction callback");
    std::unique_lock<std::mutex> lk(qmu_);
    const auto idle = [this] { return queue_.empty() && !active_; };
    if (timeout_ms == XVRAM_TIMEOUT_INFINITE) {
      qcv_.wait(lk, idle);
      return {};
    }
    if (!qcv_.wait_for(lk, std::chrono::milliseconds(timeout_ms), idle))
      return make_error(XVRAM_STATUS_TIMEOUT, "session", "drain",
                        "operations were still running at the timeout");
    return {};
  }

  // Runs the queued operations, closes the runtime and stops the worker.
  Error close(uint64_t timeout_ms) {
    if (closed.load())
      return {};
    if (on_worker())
      return make_error(XVRAM_STATUS_BUSY, "session", "reentrant_call",
                        "session_close is not allowed from a transaction callback");
    std::shared_ptr<Op> op;
    {
      std::lock_guard<std::mutex> lk(qmu_);
      if (!closing_) {
        auto cop = std::make_shared<Op>(next_op_++, 1, 0);
        cop->closes_session = true;
        cop->body = [this](Op&) -> Error {
          Error e = opened_ ? rt_.close() : Error{};
          snapshot();
          opened_ = false;
          return e;
        };
        queue_.push_back(cop);
        close_op_ = cop;
        closing_ = true;
        qcv_.notify_all();
      }
      op = close_op_;
    }
    if (!op) { // the worker never started
      stop_worker();
      closed.store(true);
      return {};
    }
    if (Error we = op->wait(timeout_ms, nullptr))
      return make_error(XVRAM_STATUS_TIMEOUT, "session", "close",
                        "queued operations did not finish before the timeout");
    stop_worker();
    closed.store(true);
    return op->error();
  }

  void record(const Error& e) {
    if (!e)
      return;
    std::lock_guard<std::mutex> lk(emu_);
    last_error_ = e;
  }
  Error last_error() {
    std::lock_guard<std::mutex> lk(emu_);
    return last_error_;
  }

  Error telemetry(xvram_session_telemetry_v1* out) {
    if (!closed.load()) {
      if (Error e = invoke_sync(
              [this]() -> Error {
                snapshot();
                return {};
              },
              true))
        if (e.status != XVRAM_STATUS_CLOSED)
          return e;
    }
    std::lock_guard<std::mutex> lk(tmu_);
    *out = telemetry_;
    return {};
  }

private:
  void snapshot() {
    std::lock_guard<std::mutex> lk(tmu_);
    if (opened_)
      telemetry_ = rt_.counters();
    telemetry_.struct_size = sizeof(telemetry_);
    telemetry_.poisoned = poisoned_ ? 1u : 0u;
  }

  void loop() {
    for (;;) {
      std::shared_ptr<Op> op;
      {
        std::unique_lock<std::mutex> lk(qmu_);
        qcv_.wait(lk, [this] { return stop_ || !queue_.empty(); });
        if (queue_.empty())
          return;
        op = queue_.front();
        queue_.pop_front();
        active_ = true;
      }
      if (op->begin()) {
        const xvram_session_telemetry_v1 before =
            opened_ ? rt_.counters() : xvram_session_telemetry_v1{};
        Error e;
        if (poisoned_ && !op->closes_session && !op->read_only) {
          e = make_error(XVRAM_STATUS_POISONED, "session", "execute",
                         "an earlier failure left the device state undefined");
        } else {
          try {
            e = op->body(*op);
          } catch (const std::bad_alloc&) {
            e = make_error(XVRAM_STATUS_HOST_OUT_OF_MEMORY, "sdk", "execute",
                           "host allocation failed");
          } catch (...) {
            e = make_error(XVRAM_STATUS_INTERNAL, "sdk", "execute", "unexpected exception");
          }
          if (e && poisons(e))
            poisoned_ = true;
        }
        const xvram_session_telemetry_v1 after =
            opened_ ? rt_.counters() : xvram_session_telemetry_v1{};
        if (e)
          record(e);
        op->finish(e, before, after);
      }
      {
        std::lock_guard<std::mutex> lk(qmu_);
        active_ = false;
        qcv_.notify_all();
      }
    }
  }

  void stop_worker() {
    {
      std::lock_guard<std::mutex> lk(qmu_);
      stop_ = true;
      closing_ = true;
      qcv_.notify_all();
    }
    if (worker_.joinable() && worker_.get_id() != std::this_thread::get_id())
      worker_.join();
  }

  xvram_session_config_v1 cfg_;
  Runtime rt_;
  bool opened_ = false;
  bool poisoned_ = false; // worker thread only
  uint64_t chunk_bytes_ = 0;
  std::thread worker_;
  std::mutex qmu_;
  std::condition_variable qcv_;
  std::deque<std::shared_ptr<Op>> queue_;
  std::shared_ptr<Op> close_op_;
  bool active_ = false, stop_ = false, closing_ = false;
  uint64_t next_op_ = 1;
  std::mutex emu_;
  Error last_error_;
  std::mutex tmu_;
  xvram_session_telemetry_v1 telemetry_{};

public:
  std::atomic<uint64_t> next_transaction{1};
};

} // namespace
} // namespace sdk
} // namespace xvram

// Handle types (opaque in the header).
struct xvram_session_t {
  std::shared_ptr<xvram::sdk::Session> s;
};
struct xvram_allocation_t {
  std::shared_ptr<xvram::sdk::Session> owner;
  uint64_t id = 0;
  uint64_t size = 0;
  uint64_t alignment = 0;
  uint32_t flags = 0;
  xvram_allocation_priority priority = XVRAM_ALLOCATION_NORMAL;
};
struct xvram_operation_t {
  std::shared_ptr<xvram::sdk::Session> owner;
  std::shared_ptr<xvram::sdk::Op> op;
};
struct xvram_gemm_plan_t {
  std::shared_ptr<xvram::sdk::Session> owner;
  xvram::GemmCall call;
  xvram::GemmLayout layout;
  xvram_compute_mode effective = XVRAM_COMPUTE_FP32_STRICT;
  uint64_t deadline_ms = 0;
};

namespace xvram {
namespace sdk {
namespace {

using SessionPtr = std::shared_ptr<Session>;

// Publishes a failure as the session's last error and returns its status.
template <class F> xvram_status boundary(const SessionPtr& s, const char* op, F&& f) noexcept {
  try {
    Error e = f();
    if (e && s)
      s->record(e);
    return e.status;
  } catch (const std::bad_alloc&) {
    if (s)
      s->record(make_error(XVRAM_STATUS_HOST_OUT_OF_MEMORY, "sdk", op, "host allocation failed"));
    return XVRAM_STATUS_HOST_OUT_OF_MEMORY;
  } catch (...) {
    if (s)
      s->record(make_error(XVRAM_STATUS_INTERNAL, "sdk", op, "unexpected exception"));
    return XVRAM_STATUS_INTERNAL;
  }
}

Error validate_session_config(const xvram_session_config_v1* c) {
  if (!has_v1_size(c))
    return incompatible("session_create", "session config is null or smaller than v1");
  if (c->flags != 0 || c->reserved0 != 0 || !all_zero(c->reserved))
    return invalid("session_create", "unknown flags or non-zero reserved field");
  if (c->context_mode != XVRAM_CONTEXT_ISOLATED && c->context_mode != XVRAM_CONTEXT_ATTACH_CURRENT)
    return invalid("session_create", "invalid context mode");
  if (c->cache_policy != XVRAM_CACHE_POLICY_CLOCK && c->cache_policy != XVRAM_CACHE_POLICY_LRU)
    return invalid("session_create", "invalid cache policy");
  if (c->device_ordinal < 0)
    return invalid("session_create", "device ordinal must be non-negative");
  if (c->chunk_size_bytes == 0)
    return invalid("session_create", "chunk size must be non-zero");
  if (c->staging_slots < 2 || c->staging_slots > 8)
    return invalid("session_create", "staging slot count must be in [2, 8]");
  if (c->prefetch_distance > 8)
    return invalid("session_create", "prefetch distance must be in [0, 8]");
  const uint64_t max64 = static_cast<uint64_t>(std::numeric_limits<int64_t>::max());
  if (c->budget_poll_ms == 0 || c->budget_poll_ms > max64 || c->max_transaction_ms > max64)
    return invalid("session_create", "budget and transaction durations are out of range");
  return {};
}

Error collect_ranges(const SessionPtr& s, const xvram_access_range_v1* ranges, uint64_t count,
                     std::vector<AccessRange>* out, const char* op) {
  if (count == 0)
    return invalid(op, "at least one access range is required");
  if (!ranges)
    return invalid(op, "range array is null");
  if (count > (1ull << 32))
    return invalid(op, "range count is too large");
  out->reserve(static_cast<size_t>(count));
  for (uint64_t i = 0; i < count; ++i) {
    const xvram_access_range_v1& r = ranges[i];
    if (!r.allocation)
      return invalid(op, "access range contains a null allocation");
    if (r.allocation->owner.get() != s.get())
      return invalid(op, "all access ranges must belong to the session");
    if (r.mode > XVRAM_ACCESS_WRITE_ONLY || r.reserved0 != 0)
      return invalid(op, "access range has an invalid mode or reserved field");
    if (r.length_bytes == 0)
      return invalid(op, "access range length must be non-zero");
    if (r.offset_bytes > UINT64_MAX - r.length_bytes)
      return invalid(op, "access range overflows uint64");
    out->push_back(AccessRange{r.allocation->id, r.offset_bytes, r.length_bytes,
                               static_cast<int>(r.mode)});
  }
  return {};
}

// Requested mode -> arithmetic, as reference src/sdk/runtime.cpp:119-142: AUTO is FP64 on
// FP64 data, strict FP32 on FP16 / BF16 data and TF32 on FP32 data.
int compute_kind(xvram_compute_mode mode, xvram_data_type a_type) {
  if (mode == XVRAM_COMPUTE_AUTO)
    return a_type == XVRAM_DATA_FP64                                ? kComputeFp64
           : a_type == XVRAM_DATA_FP16 || a_type == XVRAM_DATA_BF16 ? kStrictFp32
                                                                    : kTf32;
  if (mode == XVRAM_COMPUTE_FP64)
    return kComputeFp64;
  return mode == XVRAM_COMPUTE_FP32_STRICT ? kStrictFp32 : kTf32;
}

// The column-major view of a matrix descriptor and the operation it then needs: a
// row-major rows x columns matrix is the column-major columns x rows matrix, transposed.
struct View {
  MatrixRef ref;
  int op = 0;
};

Error make_view(const SessionPtr& s, const xvram_matrix_v1& m, xvram_matrix_operation op,
                View* out) {
  if (m.struct_size < sizeof(xvram_matrix_v1))
    return incompatible("gemm_plan_create", "matrix descriptor is smaller than v1");
  if (!m.allocation)
    return invalid("gemm_plan_create", "matrix allocation is null");
  if (m.allocation->owner.get() != s.get())
    return invalid("gemm_plan_create", "matrix allocation belongs to another session");
  if (m.data_type > XVRAM_DATA_FP64 || m.layout > XVRAM_MATRIX_COLUMN_MAJOR || m.reserved0 != 0 ||
      !all_zero(m.reserved))
    return invalid("gemm_plan_create", "matrix descriptor has invalid enum or reserved fields");
  if (m.rows == 0 || m.columns == 0 || m.leading_dimension == 0)
    return invalid("gemm_plan_create", "matrix dimensions and leading dimension must be non-zero");
  const bool row = m.layout == XVRAM_MATRIX_ROW_MAJOR;
  out->ref.allocation_id = m.allocation->id;
  out->ref.allocation_bytes = m.allocation->size;
  out->ref.offset_bytes = m.offset_bytes;
  out->ref.rows = row ? m.columns : m.rows;
  out->ref.columns = row ? m.rows : m.columns;
  out->ref.ld = m.leading_dimension;
  out->ref.dtype = m.data_type;
  out->op = row ? 1 - static_cast<int>(op) : static_cast<int>(op);
  return {};
}

Error build_plan(const SessionPtr& s, const xvram_gemm_desc_v1* d, xvram_gemm_plan_t* plan) {
  if (!has_v1_size(d))
    return incompatible("gemm_plan_create", "GEMM descriptor is null or smaller than v1");
  if (d->flags != 0 || d->reserved0 != 0 || !all_zero(d->reserved))
    return invalid("gemm_plan_create", "unknown GEMM flags or non-zero reserved field");
  if (d->operation_a > XVRAM_MATRIX_OP_T || d->operation_b > XVRAM_MATRIX_OP_T ||
      d->compute_mode > XVRAM_COMPUTE_FP64)
    return invalid("gemm_plan_create", "invalid GEMM operation or compute mode");
  if (!deadline_ok(d->deadline_ms))
    return make_error(XVRAM_STATUS_INVALID_ARGUMENT, "deadline", "gemm_plan_create",
                      "deadline_ms cannot be represented by the monotonic clock");
  View a, b, c;
  if (Error e = make_view(s, d->a, d->operation_a, &a))
    return e;
  if (Error e = make_view(s, d->b, d->operation_b, &b))
    return e;
  if (Error e = make_view(s, d->c, XVRAM_MATRIX_OP_N, &c))
    return e;
  if (!std::isfinite(d->alpha) || !std::isfinite(d->beta))
    return invalid("gemm_plan_create", "alpha and beta must be finite");
  // Logical sizes from the descriptors (reference src/sdk/runtime.cpp:1303-1308).
  const uint64_t m = d->operation_a == XVRAM_MATRIX_OP_N ? d->a.rows : d->a.columns;
  const uint64_t k = d->operation_a == XVRAM_MATRIX_OP_N ? d->a.columns : d->a.rows;
  const uint64_t n = d->operation_b == XVRAM_MATRIX_OP_N ? d->b.columns : d->b.rows;
  GemmCall call;
  call.alpha = d->alpha;
  call.beta = d->beta;
  GemmShape& sh = call.shape;
  sh.compute = compute_kind(d->compute_mode, d->a.data_type);
  if (sh.compute == kTf32)
    call.flops_per_s = 150e12; // plan for the tensor-core rate
  else if (sh.compute == kComputeFp64)
    call.flops_per_s = 35e12;
  if (d->c.layout == XVRAM_MATRIX_COLUMN_MAJOR) {
    sh.m = m;
    sh.n = n;
    sh.k = k;
    sh.op_a = a.op;
    sh.op_b = b.op;
    sh.a = a.ref;
    sh.b = b.ref;
  } else { // C^T = op(B)^T op(A)^T in the column-major view of C
    sh.m = n;
    sh.n = m;
    sh.k = k;
    sh.op_a = 1 - b.op;
    sh.op_b = 1 - a.op;
    sh.a = b.ref;
    sh.b = a.ref;
  }
  sh.c = c.ref;
  const Validation v = validate_gemm(sh);
  if (v)
    for (const MatrixRef* r : {&sh.a, &sh.b, &sh.c})
      if (r->offset_bytes % element_bytes(r->dtype) != 0)
        return invalid("gemm_plan_create",
                       "a matrix offset is not a multiple of its element size");
  if (!v) {
    std::string msg = std::string(problem_error_name(v.error));
    if (v.operand)
      msg += std::string(" (operand ") + v.operand + ")";
    return make_error(XVRAM_STATUS_INVALID_ARGUMENT, "gemm", "validate", msg);
  }
  plan->owner = s;
  plan->call = call;
  plan->effective = sh.compute == kComputeFp64 ? XVRAM_COMPUTE_FP64
                    : sh.compute == kTf32      ? XVRAM_COMPUTE_FP32_TF32
                                               : XVRAM_COMPUTE_FP32_STRICT;
  plan->deadline_ms = d->deadline_ms;
  // (Operation bodies hold the session by raw pointer: the handles own it, and the last
  // owner must never be released on the worker thread itself.)
  Session* raw = s.get();
  return s->invoke_sync([raw, plan]() -> Error {
    for (uint64_t id : {plan->call.shape.a.allocation_id, plan->call.shape.b.allocation_id,
                        plan->call.shape.c.allocation_id})
      if (!raw->runtime().live(id))
        return invalid("gemm_plan_create", "a GEMM allocation was released");
    return raw->runtime().describe_gemm(plan->call, &plan->layout);
  });
}

Error wrap(const SessionPtr& s, std::shared_ptr<Op> op, xvram_operation* out) {
  auto* h = new (std::nothrow) xvram_operation_t{s, op};
  if (!h) {
    (void)op->cancel();
    return make_error(XVRAM_STATUS_HOST_OUT_OF_MEMORY, "sdk", "operation_create",
                      "failed to allocate operation handle");
  }
  *out = h;
  return {};
}

// ------------------------------------------------------------------- entry points
const char* XVRAM_CALL status_name_entry(xvram_status st) {
  switch (st) {
  case XVRAM_STATUS_SUCCESS: return "success";
  case XVRAM_STATUS_INVALID_ARGUMENT: return "invalid_argument";
  case XVRAM_STATUS_INCOMPATIBLE_ABI: return "incompatible_abi";
  case XVRAM_STATUS_UNSUPPORTED: return "unsupported";
  case XVRAM_STATUS_UNAVAILABLE: return "unavailable";
  case XVRAM_STATUS_HOST_OUT_OF_MEMORY: return "host_out_of_memory";
  case XVRAM_STATUS_DEVICE_OUT_OF_MEMORY: return "device_out_of_memory";
  case XVRAM_STATUS_BUDGET_PRESSURE: return "budget_pressure";
  case XVRAM_STATUS_BUSY: return "busy";
  case XVRAM_STATUS_NOT_READY: return "not_ready";
  case XVRAM_STATUS_TIMEOUT: return "timeout";
  case XVRAM_STATUS_CORRUPTION: return "corruption";
  case XVRAM_STATUS_CALLBACK_FAILED: return "callback_failed";
  case XVRAM_STATUS_CUDA_ERROR: return "cuda_error";
  case XVRAM_STATUS_CUBLAS_ERROR: return "cublas_error";
  case XVRAM_STATUS_POISONED: return "poisoned";
  case XVRAM_STATUS_CLEANUP_FAILED: return "cleanup_failed";
  case XVRAM_STATUS_CLOSED: return "closed";
  case XVRAM_STATUS_CANCELLED: return "cancelled";
  case XVRAM_STATUS_INTERNAL: return "internal";
  default: return "unknown";
  }
}

xvram_status XVRAM_CALL session_create_entry(const xvram_session_config_v1* config,
                                             xvram_session* out) {
  if (!out)
    return XVRAM_STATUS_INVALID_ARGUMENT;
  *out = nullptr;
  return boundary(nullptr, "session_create", [&]() -> Error {
    if (Error e = validate_session_config(config))
      return e;
    if (config->context_mode == XVRAM_CONTEXT_ATTACH_CURRENT)
      return make_error(XVRAM_STATUS_UNSUPPORTED, "session", "create",
                        "sessions own their worker thread and device selection; use ISOLATED");
    auto s = std::make_shared<Session>(*config);
    if (Error e = s->start())
      return e;
    auto* h = new (std::nothrow) xvram_session_t{s};
    if (!h) {
      (void)s->close(XVRAM_TIMEOUT_INFINITE);
      return make_error(XVRAM_STATUS_HOST_OUT_OF_MEMORY, "sdk", "session_create",
                        "failed to allocate session handle");
    }
    *out = h;
    return {};
  });
}

xvram_status XVRAM_CALL session_get_error_entry(xvram_session session, xvram_error_info_v1* out) {
  if (!session || !session->s || !has_v1_size(out))
    return XVRAM_STATUS_INVALID_ARGUMENT;
  write_error_info(session->s->last_error(), *out);
  return XVRAM_STATUS_SUCCESS;
}

xvram_status XVRAM_CALL session_get_telemetry_entry(xvram_session session,
                                                    xvram_session_telemetry_v1* out) {
  if (!session || !session->s || !has_v1_size(out))
    return XVRAM_STATUS_INVALID_ARGUMENT;
  return boundary(session->s, "session_get_telemetry", [&]() -> Error {
    const uint32_t size = out->struct_size;
    xvram_session_telemetry_v1 t{};
    if (Error e = session->s->telemetry(&t))
      return e;
    *out = t;
    out->struct_size = size;
    return {};
  });
}

xvram_status XVRAM_CALL session_drain_entry(xvram_session session, uint64_t timeout_ms) {
  if (!session || !session->s)
    return XVRAM_STATUS_INVALID_ARGUMENT;
  return boundary(session->s, "session_drain", [&] { return session->s->drain(timeout_ms); });
}

xvram_status XVRAM_CALL session_close_entry(xvram_session session, uint64_t timeout_ms) {
  if (!session || !session->s)
    return XVRAM_STATUS_INVALID_ARGUMENT;
  return boundary(session->s, "session_close", [&] { return session->s->close(timeout_ms); });
}

void XVRAM_CALL session_release_entry(xvram_session session) {
  if (!session)
    return;
  if (session->s && session->s->on_worker()) {
    // From a transaction callback the session cannot be closed (its worker is running the
    // callback); the handle stays valid and must be released from another thread.
    session->s->record(make_error(XVRAM_STATUS_BUSY, "session", "reentrant_call",
                                  "session_release is not allowed from a transaction callback"));
    return;
  }
  try {
    if (session->s && !session->s->closed.load())
      session->s->record(session->s->close(XVRAM_TIMEOUT_INFINITE));
  } catch (...) {
  }
  delete session;
}

xvram_status XVRAM_CALL allocation_create_entry(xvram_session session,
                                                const xvram_allocation_desc_v1* desc,
                                                xvram_allocation* out) {
  if (!out)
    return XVRAM_STATUS_INVALID_ARGUMENT;
  *out = nullptr;
  if (!session || !session->s)
    return XVRAM_STATUS_INVALID_ARGUMENT;
  const SessionPtr& s = session->s;
  return boundary(s, "allocation_create", [&]() -> Error {
    if (!has_v1_size(desc))
      return incompatible("allocation_create", "allocation descriptor is null or smaller than v1");
    if (desc->size_bytes == 0)
      return invalid("allocation_create", "allocation size must be non-zero");
    if ((desc->flags & ~static_cast<uint32_t>(XVRAM_ALLOCATION_FLAG_ZERO_INITIALIZE)) != 0 ||
        desc->reserved0 != 0 || !all_zero(desc->reserved))
      return invalid("allocation_create", "unknown flags or non-zero reserved field");
    if (desc->priority > XVRAM_ALLOCATION_STREAMING)
      return invalid("allocation_create", "invalid allocation priority");
    const uint64_t al = desc->alignment_bytes;
    if (al != 0 && (al & (al - 1)) != 0)
      return invalid("allocation_create", "alignment must be zero or a power of two");
    if (al > s->chunk_bytes() || (al != 0 && s->chunk_bytes() % al != 0))
      return invalid("allocation_create", "alignment must divide the effective runtime chunk size");
    auto* h = new (std::nothrow) xvram_allocation_t;
    if (!h)
      return make_error(XVRAM_STATUS_HOST_OUT_OF_MEMORY, "sdk", "allocation_create",
                        "failed to allocate handle");
    const bool zero = (desc->flags & XVRAM_ALLOCATION_FLAG_ZERO_INITIALIZE) != 0;
    uint64_t id = 0;
    Error e = s->invoke_sync([&]() -> Error {
      uint64_t va = 0;
      return s->runtime().allocate(desc->size_bytes, &id, &va, zero);
    });
    if (e) {
      delete h;
      return e;
    }
    h->owner = s;
    h->id = id;
    h->size = desc->size_bytes;
    h->alignment = al;
    h->flags = desc->flags;
    h->priority = desc->priority;
    *out = h;
    return {};
  });
}

xvram_status XVRAM_CALL allocation_get_info_entry(xvram_allocation a,
                                                  xvram_allocation_info_v1* out) {
  if (!a || !a->owner || !has_v1_size(out))
    return XVRAM_STATUS_INVALID_ARGUMENT;
  const uint32_t size = out->struct_size;
  std::memset(out, 0, sizeof(*out));
  out->struct_size = size;
  out->flags = a->flags;
  out->allocation_id = a->id;
  out->size_bytes = a->size;
  out->alignment_bytes = a->alignment;
  out->priority = a->priority;
  out->stable_virtual_address = 1;
  return XVRAM_STATUS_SUCCESS;
}

Error bounds(const xvram_allocation_t* a, uint64_t offset, uint64_t bytes, const char* op) {
  if (offset > a->size || bytes > a->size - offset)
    return invalid(op, "the byte range lies outside the allocation");
  return {};
}

xvram_status XVRAM_CALL allocation_write_entry(xvram_allocation a, uint64_t offset,
                                               const void* src, uint64_t bytes) {
  if (!a || !a->owner || (bytes != 0 && !src))
    return XVRAM_STATUS_INVALID_ARGUMENT;
  return boundary(a->owner, "allocation_write", [&]() -> Error {
    if (Error e = bounds(a, offset, bytes, "allocation_write"))
      return e;
    if (bytes == 0)
      return {};
    return a->owner->invoke_sync(
        [&]() { return a->owner->runtime().write(a->id, offset, src, bytes); });
  });
}

xvram_status XVRAM_CALL allocation_read_entry(xvram_allocation a, uint64_t offset, void* dst,
                                              uint64_t bytes) {
  if (!a || !a->owner || (bytes != 0 && !dst))
    return XVRAM_STATUS_INVALID_ARGUMENT;
  return boundary(a->owner, "allocation_read", [&]() -> Error {
    if (Error e = bounds(a, offset, bytes, "allocation_read"))
      return e;
    if (bytes == 0)
      return {};
    return a->owner->invoke_sync(
        [&]() { return a->owner->runtime().read(a->id, offset, dst, bytes); });
  });
}

xvram_status XVRAM_CALL allocation_release_entry(xvram_allocation a) {
  if (!a || !a->owner)
    return XVRAM_STATUS_INVALID_ARGUMENT;
  // After a successful close every allocation is gone; releasing the handle is local.
  if (a->owner->closed.load()) {
    delete a;
    return XVRAM_STATUS_SUCCESS;
  }
  const xvram_status st = boundary(a->owner, "allocation_release", [&]() -> Error {
    return a->owner->invoke_sync([&]() { return a->owner->runtime().release(a->id); });
  });
  if (st == XVRAM_STATUS_SUCCESS)
    delete a;
  return st;
}

xvram_status XVRAM_CALL prefetch_submit_entry(xvram_session session,
                                              const xvram_prefetch_desc_v1* desc,
                                              xvram_operation* out) {
  if (!out)
    return XVRAM_STATUS_INVALID_ARGUMENT;
  *out = nullptr;
  if (!session || !session->s)
    return XVRAM_STATUS_INVALID_ARGUMENT;
  const SessionPtr& s = session->s;
  return boundary(s, "prefetch_submit", [&]() -> Error {
    if (!has_v1_size(desc))
      return incompatible("prefetch_submit", "prefetch descriptor is null or smaller than v1");
    if (desc->flags != 0 || !all_zero(desc->reserved))
      return invalid("prefetch_submit", "unknown flags or non-zero reserved field");
    if (!deadline_ok(desc->deadline_ms))
      return make_error(XVRAM_STATUS_INVALID_ARGUMENT, "deadline", "prefetch_submit",
                        "deadline_ms cannot be represented by the monotonic clock");
    std::vector<AccessRange> ranges;
    if (Error e = collect_ranges(s, desc->ranges, desc->range_count, &ranges, "prefetch_submit"))
      return e;
    std::shared_ptr<Op> op;
    Session* raw = s.get();
    if (Error e = s->enqueue(
            [raw, ranges = std::move(ranges)](Op&) { return raw->runtime().prefetch(ranges); }, 1,
            desc->deadline_ms, &op))
      return e;
    return wrap(s, std::move(op), out);
  });
}

xvram_status XVRAM_CALL transaction_submit_entry(xvram_session session,
                                                 const xvram_transaction_desc_v1* desc,
                                                 xvram_operation* out) {
  if (!out)
    return XVRAM_STATUS_INVALID_ARGUMENT;
  *out = nullptr;
  if (!session || !session->s)
    return XVRAM_STATUS_INVALID_ARGUMENT;
  const SessionPtr& s = session->s;
  return boundary(s, "transaction_submit", [&]() -> Error {
    if (!has_v1_size(desc))
      return incompatible("transaction_submit",
                          "transaction descriptor is null or smaller than v1");
    if (desc->flags != 0 || !all_zero(desc->reserved))
      return invalid("transaction_submit", "unknown flags or non-zero reserved field");
    if (!desc->callback)
      return invalid("transaction_submit", "transaction callback is null");
    if (desc->workspace_bytes > s->config().workspace_cap_bytes)
      return invalid("transaction_submit", "transaction workspace exceeds the session cap");
    if (!deadline_ok(desc->deadline_ms))
      return make_error(XVRAM_STATUS_INVALID_ARGUMENT, "deadline", "transaction_submit",
                        "deadline_ms cannot be represented by the monotonic clock");
    std::vector<AccessRange> ranges;
    if (Error e =
            collect_ranges(s, desc->ranges, desc->range_count, &ranges, "transaction_submit"))
      return e;
    const uint64_t txn = s->next_transaction.fetch_add(1);
    const xvram_transaction_callback_v1 cb = desc->callback;
    void* const user = desc->user_data;
    const uint64_t ws = desc->workspace_bytes;
    Session* raw = s.get();
    std::shared_ptr<Op> op;
    if (Error e = s->enqueue(
            [raw, ranges = std::move(ranges), cb, user, ws, txn](Op& self) -> Error {
              if (Error de = self.deadline_error("operation", "pre_launch_deadline"))
                return de;
              Error cb_error;
              Error e = raw->runtime().transaction(
                  ranges, ws,
                  [&](const std::vector<ResolvedRange>& res, uint64_t ws_addr, uint64_t ws_bytes,
                      uint64_t stream) -> Error {
                    if (Error de = self.deadline_error("operation", "post_residency_deadline"))
                      return cb_error = de;
                    std::vector<xvram_resolved_range_v1> pub;
                    pub.reserve(res.size());
                    for (const ResolvedRange& r : res)
                      pub.push_back(xvram_resolved_range_v1{
                          r.allocation_id, r.offset_bytes, r.length_bytes, r.device_address,
                          static_cast<xvram_access_mode>(r.mode), 0u});
                    xvram_transaction_context_v1 ctx{};
                    ctx.struct_size = sizeof(ctx);
                    ctx.operation_id = self.id();
                    ctx.transaction_id = txn;
                    ctx.ranges = pub.data();
                    ctx.range_count = pub.size();
                    ctx.workspace_device_address = ws_addr;
                    ctx.workspace_bytes = ws_bytes;
                    ctx.native_stream = stream;
                    xvram_error_info_v1 native = XVRAM_ERROR_INFO_V1_INIT;
                    const xvram_status st = cb(&ctx, user, &native);
                    if (st != XVRAM_STATUS_SUCCESS) {
                      native.message[sizeof(native.message) - 1] = '\0';
                      native.stage[sizeof(native.stage) - 1] = '\0';
                      native.operation[sizeof(native.operation) - 1] = '\0';
                      native.native_name[sizeof(native.native_name) - 1] = '\0';
                      cb_error.status = st;
                      cb_error.domain = XVRAM_NATIVE_ERROR_CALLBACK;
                      cb_error.native_code = native.native_code;
                      cb_error.stage = native.stage;
                      cb_error.operation = native.operation;
                      cb_error.native_name = native.native_name;
                      cb_error.message =
                          native.message[0] ? native.message : "transaction callback failed";
                      return cb_error;
                    }
                    return Error{};
                  });
              return cb_error ? cb_error : e;
            },
            1, desc->deadline_ms, &op))
      return e;
    return wrap(s, std::move(op), out);
  });
}

xvram_status XVRAM_CALL operation_wait_entry(xvram_operation op, uint64_t timeout_ms,
                                             xvram_operation_info_v1* out);
void XVRAM_CALL operation_release_entry(xvram_operation op);

// Submit, wait, and report the operation's own error (reference src/sdk/api.cpp:762-791).
template <class Submit>
xvram_status execute(const SessionPtr& s, Submit&& submit, uint64_t timeout_ms, const char* what) {
  xvram_operation op = nullptr;
  const xvram_status st = submit(&op);
  if (st != XVRAM_STATUS_SUCCESS)
    return st;
  xvram_operation_info_v1 info = XVRAM_OPERATION_INFO_V1_INIT;
  const xvram_status wst = operation_wait_entry(op, timeout_ms, &info);
  if (wst != XVRAM_STATUS_SUCCESS) {
    operation_release_entry(op);
    return wst;
  }
  xvram_status result = info.result;
  if (result != XVRAM_STATUS_SUCCESS) {
    Error e = op->op->error();
    if (!e)
      e = make_error(info.result, what, "execute", "the operation failed");
    s->record(e);
    result = e.status;
  }
  operation_release_entry(op);
  return result;
}

xvram_status XVRAM_CALL transaction_execute_entry(xvram_session session,
                                                  const xvram_transaction_desc_v1* desc,
                                                  uint64_t timeout_ms) {
  if (!session || !session->s)
    return XVRAM_STATUS_INVALID_ARGUMENT;
  return execute(
      session->s,
      [&](xvram_operation* op) { return transaction_submit_entry(session, desc, op); },
      timeout_ms, "transaction");
}

xvram_status XVRAM_CALL gemm_plan_create_entry(xvram_session session,
                                               const xvram_gemm_desc_v1* desc,
                                               xvram_gemm_plan* out) {
  if (!out)
    return XVRAM_STATUS_INVALID_ARGUMENT;
  *out = nullptr;
  if (!session || !session->s)
    return XVRAM_STATUS_INVALID_ARGUMENT;
  const SessionPtr& s = session->s;
  return boundary(s, "gemm_plan_create", [&]() -> Error {
    auto plan = std::make_unique<xvram_gemm_plan_t>();
    if (Error e = build_plan(s, desc, plan.get()))
      return e;
    *out = plan.release();
    return {};
  });
}

xvram_status XVRAM_CALL gemm_plan_get_info_entry(xvram_gemm_plan plan,
                                                 xvram_gemm_plan_info_v1* out) {
  if (!plan || !plan->owner || !has_v1_size(out))
    return XVRAM_STATUS_INVALID_ARGUMENT;
  const uint32_t size = out->struct_size;
  xvram_gemm_plan_info_v1 info = XVRAM_GEMM_PLAN_INFO_V1_INIT;
  const GemmShape& sh = plan->call.shape;
  info.m = sh.m;
  info.n = sh.n;
  info.k = sh.k;
  info.tile_m = plan->layout.tile_m;
  info.tile_n = plan->layout.tile_n;
  info.tile_k = plan->layout.tile_k;
  info.maximum_working_set_bytes = plan->layout.working_set_bytes;
  info.workspace_bytes = plan->layout.workspace_bytes;
  info.tile_count = plan->layout.tiles;
  info.effective_compute_mode = plan->effective;
  info.uses_cublas_lt = 0;
  *out = info;
  out->struct_size = size;
  return XVRAM_STATUS_SUCCESS;
}

xvram_status XVRAM_CALL gemm_submit_entry(xvram_gemm_plan plan, xvram_operation* out) {
  if (!out)
    return XVRAM_STATUS_INVALID_ARGUMENT;
  *out = nullptr;
  if (!plan || !plan->owner)
    return XVRAM_STATUS_INVALID_ARGUMENT;
  const SessionPtr& s = plan->owner;
  return boundary(s, "gemm_submit", [&]() -> Error {
    Session* raw = s.get();
    const GemmCall call = plan->call;
    std::shared_ptr<Op> op;
    if (Error e = s->enqueue(
            [raw, call](Op& self) -> Error {
              if (Error de = self.deadline_error("gemm", "pre_launch_deadline"))
                return de;
              for (uint64_t id : {call.shape.a.allocation_id, call.shape.b.allocation_id,
                                  call.shape.c.allocation_id})
                if (!raw->runtime().live(id))
                  return invalid("gemm_submit", "a GEMM allocation was released");
              return raw->runtime().gemm(call);
            },
            plan->layout.tiles ? plan->layout.tiles : 1, plan->deadline_ms, &op))
      return e;
    return wrap(s, std::move(op), out);
  });
}

xvram_status XVRAM_CALL gemm_execute_entry(xvram_gemm_plan plan, uint64_t timeout_ms) {
  if (!plan || !plan->owner)
    return XVRAM_STATUS_INVALID_ARGUMENT;
  return execute(
      plan->owner, [&](xvram_operation* op) { return gemm_submit_entry(plan, op); }, timeout_ms,
      "gemm");
}

void XVRAM_CALL gemm_plan_release_entry(xvram_gemm_plan plan) { delete plan; }

xvram_status XVRAM_CALL operation_poll_entry(xvram_operation op, xvram_operation_info_v1* out) {
  if (!op || !op->op || !has_v1_size(out))
    return XVRAM_STATUS_INVALID_ARGUMENT;
  const uint32_t size = out->struct_size;
  op->op->poll(out);
  out->struct_size = size;
  return XVRAM_STATUS_SUCCESS;
}

xvram_status XVRAM_CALL operation_wait_entry(xvram_operation op, uint64_t timeout_ms,
                                             xvram_operation_info_v1* out) {
  if (!op || !op->op || !has_v1_size(out))
    return XVRAM_STATUS_INVALID_ARGUMENT;
  return boundary(op->owner, "operation_wait", [&]() -> Error {
    const uint32_t size = out->struct_size;
    if (op->owner && op->owner->on_worker()) {
      // Inside a transaction callback every other operation is queued behind it.
      op->op->poll(out);
      out->struct_size = size;
      const bool done = out->state == XVRAM_OPERATION_COMPLETED ||
                        out->state == XVRAM_OPERATION_CANCELLED ||
                        out->state == XVRAM_OPERATION_FAILED;
      return done ? Error{}
                  : make_error(XVRAM_STATUS_BUSY, "operation", "reentrant_wait",
                               "waiting from a transaction callback would never finish");
    }
    Error e = op->op->wait(timeout_ms, out);
    out->struct_size = size;
    return e;
  });
}

xvram_status XVRAM_CALL operation_cancel_entry(xvram_operation op) {
  if (!op || !op->op)
    return XVRAM_STATUS_INVALID_ARGUMENT;
  return boundary(op->owner, "operation_cancel", [&] { return op->op->cancel(); });
}

xvram_status XVRAM_CALL operation_get_error_entry(xvram_operation op, xvram_error_info_v1* out) {
  if (!op || !op->op || !has_v1_size(out))
    return XVRAM_STATUS_INVALID_ARGUMENT;
  write_error_info(op->op->error(), *out);
  return XVRAM_STATUS_SUCCESS;
}

void XVRAM_CALL operation_release_entry(xvram_operation op) { delete op; }

const xvram_api_v1& api_v1() {
  static const xvram_api_v1 api = [] {
    xvram_api_v1 v{};
    v.struct_size = sizeof(v);
    v.abi_version = XVRAM_ABI_VERSION_1;
    v.status_name = &status_name_entry;
    v.session_create = &session_create_entry;
    v.session_get_error = &session_get_error_entry;
    v.session_get_telemetry = &session_get_telemetry_entry;
    v.session_drain = &session_drain_entry;
    v.session_close = &session_close_entry;
    v.session_release = &session_release_entry;
    v.allocation_create = &allocation_create_entry;
    v.allocation_get_info = &allocation_get_info_entry;
    v.allocation_write = &allocation_write_entry;
    v.allocation_read = &allocation_read_entry;
    v.allocation_release = &allocation_release_entry;
    v.prefetch_submit = &prefetch_submit_entry;
    v.transaction_submit = &transaction_submit_entry;
    v.transaction_execute = &transaction_execute_entry;
    v.gemm_plan_create = &gemm_plan_create_entry;
    v.gemm_plan_get_info = &gemm_plan_get_info_entry;
    v.gemm_submit = &gemm_submit_entry;
    v.gemm_execute = &gemm_execute_entry;
    v.gemm_plan_release = &gemm_plan_release_entry;
    v.operation_poll = &operation_poll_entry;
    v.operation_wait = &operation_wait_entry;
    v.operation_cancel = &operation_cancel_entry;
    v.operation_get_error = &operation_get_error_entry;
    v.operation_release = &operation_release_entry;
    return v;
  }();
  return api;
}

} // namespace
} // namespace sdk
} // namespace xvram

// The SDK's only export (reference include/xvram/xvram.h:529-531, src/sdk/api.cpp:1017-1035).
extern "C" XVRAM_API xvram_status XVRAM_CALL xvram_get_api(uint32_t requested_abi_version,
                                                           uint32_t caller_api_size,
                                                           void* out_api) {
  if (requested_abi_version != XVRAM_ABI_VERSION_1)
    return XVRAM_STATUS_INCOMPATIBLE_ABI;
  if (!out_api || caller_api_size < sizeof(xvram_api_v1))
    return XVRAM_STATUS_INVALID_ARGUMENT;
  std::memcpy(out_api, &xvram::sdk::api_v1(), sizeof(xvram_api_v1));
  return XVRAM_STATUS_SUCCESS;
}
