// compat_api.cpp -- xvram_cuda_compat_get_api and the adapter behind it.
//
// Behaviour follows the reference adapter (reference src/cuda_compat/adapter.cpp,
// api.cpp:16-64) call for call:
//   * one initialisation attempt per process; calls before it return NOT_READY, calls
//     after shutdown CLOSED, data calls on a poisoned adapter POISONED (adapter.cpp:127-192);
//   * configuration checks (adapter.cpp:31-46, 361-379);
//   * host pointers must not touch managed ranges; device ranges must lie inside one
//     live allocation; cudaFree needs the exact base (adapter.cpp:269-317, 475-577);
//   * blas_sgemm preflight order: initialised, live handle, N/T and positive sizes
//     (UNSUPPORTED), host scalars, leading dimensions, live allocations, float
//     alignment, finite scalars, then problem validation (adapter.cpp:719-793);
//   * a failure after device work may have been submitted poisons the adapter.
// Calls are serialised by a mutex and run on the calling thread; the caller's current
// CUDA device is restored on return.
#include "xvram_b200.h"
#include "xvram/cuda_compat.h"

#include "device.hpp"
#include "runtime.hpp"
#include "status.hpp"
#include "validate.hpp"

#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <map>
#include <memory>
#include <mutex>
#include <new>
#include <vector>

#include <fstream>
#include <string>
#include <unistd.h>

namespace {
// Physical and currently available host RAM: /proc/meminfo's MemTotal and MemAvailable,
// else the page counts sysconf reports.
bool host_memory(uint64_t* physical, uint64_t* available) {
  std::ifstream f("/proc/meminfo");
  std::string key;
  uint64_t kib = 0, total = 0, avail = 0;
  std::string unit;
  while (f >> key >> kib) {
    std::getline(f, unit);
    if (key == "MemTotal:")
      total = kib << 10;
    else if (key == "MemAvailable:")
      avail = kib << 10;
  }
  if (!total || !avail) {
    const long page = sysconf(_SC_PAGESIZE), pages = sysconf(_SC_PHYS_PAGES),
               free_pages = sysconf(_SC_AVPHYS_PAGES);
    if (page > 0 && pages > 0 && free_pages > 0) {
      total = static_cast<uint64_t>(page) * static_cast<uint64_t>(pages);
      avail = static_cast<uint64_t>(page) * static_cast<uint64_t>(free_pages);
    }
  }
  *physical = total;
  *available = avail;
  return total != 0 && avail != 0;
}
} // namespace

namespace xvram {
namespace {

Error invalid(const char* op, const char* msg) {
  Error e = make_error(XVRAM_STATUS_INVALID_ARGUMENT, "compat_preflight", op, msg);
  return e;
}
Error unsupported(const char* op, const char* msg) {
  return make_error(XVRAM_STATUS_UNSUPPORTED, "compat_preflight", op, msg);
}

template <class T> bool has_size(const T* v) { return v && v->struct_size >= sizeof(T); }
template <class T, size_t N> bool all_zero(const T (&v)[N]) {
  return std::all_of(std::begin(v), std::end(v), [](T x) { return x == 0; });
}

bool valid_config(const xvram_cuda_compat_config_v1& c) {
  const auto& s = c.session;
  return c.flags == 0 && all_zero(c.reserved) && s.struct_size >= sizeof(s) && s.flags == 0 &&
         s.device_ordinal >= 0 && s.context_mode == XVRAM_CONTEXT_ISOLATED &&
         s.chunk_size_bytes > 0 && (s.chunk_size_bytes & (s.chunk_size_bytes - 1)) == 0 &&
         s.staging_slots >= 2 && s.staging_slots <= 8 && s.prefetch_distance <= 8 &&
         s.budget_poll_ms > 0 && s.cache_policy <= XVRAM_CACHE_POLICY_LRU && s.reserved0 == 0 &&
         all_zero(s.reserved) && s.budget_poll_ms <= static_cast<uint64_t>(INT64_MAX) &&
         s.max_transaction_ms <= 250 && c.stall_timeout_ms > 0 &&
         c.stall_timeout_ms <= static_cast<uint64_t>(INT64_MAX);
}

bool terminated(const char* v, size_t n) { return std::memchr(v, 0, n) != nullptr; }

bool poisons(const Error& e) {
  switch (e.status) {
  case XVRAM_STATUS_CUDA_ERROR:
  case XVRAM_STATUS_TIMEOUT:
  case XVRAM_STATUS_INTERNAL:
  case XVRAM_STATUS_CORRUPTION:
  case XVRAM_STATUS_CLEANUP_FAILED:
    return true;
  default:
    return false;
  }
}

class DeviceScope {
public:
  explicit DeviceScope(int ordinal) {
    if (cudaGetDevice(&saved_) != cudaSuccess)
      saved_ = -1;
    cudaGetLastError();
    if (ordinal >= 0 && ordinal != saved_)
      cudaSetDevice(ordinal);
  }
  ~DeviceScope() {
    int now = -1;
    if (saved_ >= 0 && cudaGetDevice(&now) == cudaSuccess && now != saved_)
      cudaSetDevice(saved_);
    cudaGetLastError();
  }

private:
  int saved_ = -1;
};

class Adapter {
public:
  Adapter() {
    tel_.struct_size = sizeof(tel_);
    tel_.runtime.struct_size = sizeof(tel_.runtime);
    tel_.state = XVRAM_CUDA_COMPAT_UNINITIALIZED;
  }
  ~Adapter() { (void)shutdown(); }

  // ----------------------------------------------------------------- lifecycle
  xvram_status initialize(const xvram_cuda_compat_config_v1* config) {
    std::lock_guard call(call_mu_);
    count_attempt();
    if (!has_size(config))
      return reject(invalid("initialize", "configuration prefix is missing"));
    if (!valid_config(*config))
      return reject(invalid("initialize", "unsupported configuration or nonzero reserved fields"));
    if (!terminated(config->cublas_library, sizeof(config->cublas_library)) ||
        !terminated(config->cublas_lt_library, sizeof(config->cublas_lt_library)))
      return reject(invalid("initialize", "library paths must be NUL terminated"));
    const bool core = config->cublas_library[0] != 0, lt = config->cublas_lt_library[0] != 0;
    if (core != lt || (core && (config->cublas_library[0] != '/' || config->cublas_lt_library[0] != '/')))
      return reject(invalid("initialize", "library paths must be an absolute core/Lt pair"));
    if (attempted_)
      return reject(make_error(XVRAM_STATUS_CLOSED, "compat", "initialize",
                               "only one initialization attempt is permitted"));
    attempted_ = true;
    config_ = *config;
    {
      const char* v = std::getenv("XVRAM_B200_SYNC_GEMM");
      sync_gemm_ = v && v[0] == '1';
    }
    set_state(XVRAM_CUDA_COMPAT_INITIALIZING);
    count_submitted();
    RuntimeConfig rc;
    rc.device_ordinal = config->session.device_ordinal;
    rc.chunk_bytes = config->session.chunk_size_bytes;
    rc.cache_target_bytes = config->session.cache_target_bytes;
    rc.headroom_bytes = config->session.device_headroom_bytes;
    rc.budget_poll_ms = config->session.budget_poll_ms;
    rc.cache_policy = config->session.cache_policy;
    Error err;
    // Host-memory admission (reference src/cuda_compat/runtime_backend.cpp:103-139): keep
    // max(4 GiB, physical / 4) of RAM free and cap the runtime's host ledger -- the pinned
    // host backing of allocations -- at the rest of what is available now.
    uint64_t physical = 0, available = 0;
    if (!host_memory(&physical, &available))
      err = make_error(XVRAM_STATUS_UNAVAILABLE, "cuda_compat", "host_budget",
                       "host memory telemetry is required for raw backing admission");
    const uint64_t host_headroom = std::max<uint64_t>(4ull << 30, physical / 4);
    {
      std::lock_guard lock(snap_mu_);
      tel_.host_physical_bytes = physical;
      tel_.host_available_bytes = available;
    }
    if (!err && available <= host_headroom)
      err = make_error(XVRAM_STATUS_HOST_OUT_OF_MEMORY, "cuda_compat", "host_budget",
                       "available RAM does not leave the automatic host headroom");
    if (!err) {
      rc.host_store_cap_bytes = available - host_headroom;
      std::lock_guard lock(snap_mu_);
      tel_.host_headroom_bytes = host_headroom;
      tel_.host_store_cap_bytes = rc.host_store_cap_bytes;
    }
    if (!err) try {
      DeviceScope scope(rc.device_ordinal);
      auto factory = device_factory();
      std::unique_ptr<Device> dev = factory ? factory() : nullptr;
      if (!dev) {
        err = make_error(XVRAM_STATUS_INTERNAL, "compat", "initialize", "no device backend");
      } else {
        runtime_ = std::make_unique<Runtime>();
        err = runtime_->open(rc, std::move(dev));
      }
    } catch (const std::bad_alloc&) {
      err = make_error(XVRAM_STATUS_HOST_OUT_OF_MEMORY, "compat", "initialize", "out of memory");
    }
    if (err) {
      if (runtime_) {
        (void)runtime_->close();
        runtime_.reset();
      }
      set_state(XVRAM_CUDA_COMPAT_CLOSED);
      return reject(err);
    }
    {
      std::lock_guard lock(snap_mu_);
      const DeviceInfo& di = runtime_->info();
      tel_.device_ordinal = di.ordinal;
      tel_.device_count = static_cast<uint32_t>(di.device_count);
      copy_field(tel_.device_name, sizeof(tel_.device_name), di.name);
      tel_.total_vram_bytes = di.total_bytes;
      tel_.effective_chunk_bytes = runtime_->chunk_bytes();
    }
    publish();
    set_state(XVRAM_CUDA_COMPAT_READY);
    return complete();
  }

  xvram_status shutdown() {
    std::lock_guard call(call_mu_);
    if (state() != XVRAM_CUDA_COMPAT_READY && state() != XVRAM_CUDA_COMPAT_POISONED)
      return XVRAM_STATUS_SUCCESS;
    count_attempt();
    count_submitted();
    Error err;
    {
      DeviceScope scope(config_.session.device_ordinal);
      err = runtime_->close();
    }
    publish();
    runtime_.reset();
    {
      std::lock_guard lock(snap_mu_);
      if (!err) {
        tel_.allocations_released = tel_.allocations_created;
        tel_.handles_destroyed = tel_.handles_created;
        tel_.live_allocations = 0;
        tel_.live_handles = 0;
        tel_.logical_bytes = 0;
        // The worker had no call in flight (calls are serialised) and the runtime's close
        // synchronised its streams and destroyed every event.
        tel_.cleanup_operations_drained = 1;
        tel_.cleanup_events_drained = 1;
        tel_.cleanup_completed = 1;
      }
    }
    for (auto& [base, e] : allocs_)
      e.live = false;
    handles_.clear();
    set_state(XVRAM_CUDA_COMPAT_CLOSED);
    if (err)
      return reject(err);
    return complete();
  }

  xvram_status get_error(xvram_error_info_v1* out) const {
    if (!has_size(out))
      return XVRAM_STATUS_INVALID_ARGUMENT;
    std::lock_guard lock(snap_mu_);
    write_error_info(error_, *out);
    return XVRAM_STATUS_SUCCESS;
  }

  xvram_status get_telemetry(xvram_cuda_compat_telemetry_v1* out) const {
    if (!has_size(out))
      return XVRAM_STATUS_INVALID_ARGUMENT;
    std::lock_guard lock(snap_mu_);
    const uint32_t size = out->struct_size;
    *out = tel_;
    out->struct_size = size;
    return XVRAM_STATUS_SUCCESS;
  }

  // -------------------------------------------------------------------- memory
  xvram_status malloc_device(void** out, uint64_t bytes) {
    return run("cudaMalloc", [&]() -> Error {
      if (!host_ok(out, sizeof(*out)) || bytes == 0 ||
          bytes > UINT64_MAX - (config_.session.chunk_size_bytes - 1))
        return invalid("cudaMalloc", "a host output pointer and positive representable size are required");
      uint64_t id = 0, va = 0;
      if (Error e = runtime_->allocate(bytes, &id, &va))
        return e;
      Entry entry;
      entry.id = id;
      entry.base = va;
      entry.bytes = bytes;
      entry.reserved = (bytes + runtime_->chunk_bytes() - 1) / runtime_->chunk_bytes() *
                       runtime_->chunk_bytes();
      allocs_[va] = entry;
      {
        std::lock_guard lock(snap_mu_);
        ++tel_.allocations_created;
        ++tel_.live_allocations;
        tel_.logical_bytes += bytes;
        tel_.logical_bytes_peak = std::max(tel_.logical_bytes_peak, tel_.logical_bytes);
      }
      void* p = reinterpret_cast<void*>(static_cast<uintptr_t>(va));
      std::memcpy(out, &p, sizeof(p));
      return {};
    });
  }

  xvram_status free_device(void* pointer) {
    return run("cudaFree", [&]() -> Error {
      if (!pointer)
        return {};
      Entry* e = lookup(pointer, 1);
      if (!e || e->base != reinterpret_cast<uintptr_t>(pointer))
        return invalid("cudaFree", "pointer is not a live allocation base");
      if (Error err = runtime_->release(e->id))
        return err;
      e->live = false;
      std::lock_guard lock(snap_mu_);
      ++tel_.allocations_released;
      --tel_.live_allocations;
      tel_.logical_bytes -= e->bytes;
      return {};
    });
  }

  xvram_status memcpy_(void* dst, const void* src, uint64_t bytes, uint32_t kind) {
    return run("cudaMemcpy", [&]() -> Error {
      if (kind != XVRAM_CUDA_COMPAT_H2D && kind != XVRAM_CUDA_COMPAT_D2H)
        return unsupported("cudaMemcpy",
                           "only explicit host-to-device and device-to-host copies are supported");
      if (bytes == 0)
        return {};
      const void* device = kind == XVRAM_CUDA_COMPAT_H2D ? dst : src;
      const void* host = kind == XVRAM_CUDA_COMPAT_H2D ? src : dst;
      Entry* e = lookup(device, bytes);
      if (!e || !host_ok(host, bytes))
        return invalid("cudaMemcpy", "copy must pair one live managed range with a host range");
      const uint64_t off = reinterpret_cast<uintptr_t>(device) - e->base;
      Error err = kind == XVRAM_CUDA_COMPAT_H2D ? runtime_->write(e->id, off, src, bytes)
                                                : runtime_->read(e->id, off, dst, bytes);
      if (err)
        return err;
      std::lock_guard lock(snap_mu_);
      (kind == XVRAM_CUDA_COMPAT_H2D ? tel_.h2d_bytes : tel_.d2h_bytes) += bytes;
      return {};
    });
  }

  // -------------------------------------------------------------------- device
  xvram_status get_device(int32_t* out) {
    return run("cudaGetDevice", [&]() -> Error {
      if (!host_ok(out, sizeof(*out)))
        return invalid("cudaGetDevice", "host output required");
      *out = config_.session.device_ordinal;
      return {};
    });
  }
  xvram_status get_device_count(int32_t* out) {
    return run("cudaGetDeviceCount", [&]() -> Error {
      if (!host_ok(out, sizeof(*out)))
        return invalid("cudaGetDeviceCount", "host output required");
      std::lock_guard lock(snap_mu_);
      *out = static_cast<int32_t>(tel_.device_count);
      return {};
    });
  }
  xvram_status set_device(int32_t d) {
    return run("cudaSetDevice", [&]() -> Error {
      return d == config_.session.device_ordinal
                 ? Error{}
                 : unsupported("cudaSetDevice", "only the initialized device may be selected");
    });
  }
  xvram_status synchronize() {
    return run("cudaDeviceSynchronize", [&]() -> Error { return runtime_->synchronize(); });
  }
  xvram_status mem_get_info(uint64_t* free_b, uint64_t* total_b) {
    return run("cudaMemGetInfo", [&]() -> Error {
      if (!host_ok(free_b, sizeof(*free_b)) || !host_ok(total_b, sizeof(*total_b)) ||
          free_b == total_b)
        return invalid("cudaMemGetInfo", "distinct host outputs required");
      uint64_t f = 0, t = 0;
      if (Error e = runtime_->mem_get_info(&f, &t))
        return e;
      *free_b = f;
      *total_b = t;
      return {};
    });
  }

  // ---------------------------------------------------------------------- blas
  xvram_status blas_create(void** out) {
    return run("cublasCreate", [&]() -> Error {
      if (!host_ok(out, sizeof(*out)))
        return invalid("cublasCreate", "host output required");
      auto h = std::make_unique<Handle>();
      void* p = h.get();
      handles_.push_back(std::move(h));
      {
        std::lock_guard lock(snap_mu_);
        ++tel_.handles_created;
        ++tel_.live_handles;
      }
      std::memcpy(out, &p, sizeof(p));
      return {};
    });
  }
  xvram_status blas_destroy(void* h) {
    return run("cublasDestroy", [&]() -> Error {
      Handle* hd = handle(h);
      if (!hd)
        return invalid("cublasDestroy", "unknown or destroyed handle");
      hd->live = false;
      std::lock_guard lock(snap_mu_);
      ++tel_.handles_destroyed;
      --tel_.live_handles;
      return {};
    });
  }
  xvram_status blas_get_version(void* h, int32_t* out) {
    return run("cublasGetVersion", [&]() -> Error {
      if (!handle(h) || !host_ok(out, sizeof(*out)))
        return invalid("cublasGetVersion", "live handle and host output required");
      *out = XVRAM_B200_VERSION_NUMBER;
      return {};
    });
  }
  xvram_status blas_set_stream(void* h, uint64_t s) {
    return run("cublasSetStream", [&]() -> Error {
      if (!handle(h))
        return invalid("cublasSetStream", "live handle required");
      return s == 0 ? Error{} : unsupported("cublasSetStream", "only the default stream is supported");
    });
  }
  xvram_status blas_get_stream(void* h, uint64_t* out) {
    return run("cublasGetStream", [&]() -> Error {
      if (!handle(h) || !host_ok(out, sizeof(*out)))
        return invalid("cublasGetStream", "live handle and host output required");
      *out = 0;
      return {};
    });
  }
  xvram_status blas_set_pointer_mode(void* h, uint32_t mode) {
    return run("cublasSetPointerMode", [&]() -> Error {
      if (!handle(h))
        return invalid("cublasSetPointerMode", "live handle required");
      return mode == 0 ? Error{} : unsupported("cublasSetPointerMode", "only host pointer mode is supported");
    });
  }
  xvram_status blas_get_pointer_mode(void* h, uint32_t* out) {
    return run("cublasGetPointerMode", [&]() -> Error {
      if (!handle(h) || !host_ok(out, sizeof(*out)))
        return invalid("cublasGetPointerMode", "live handle and host output required");
      *out = 0;
      return {};
    });
  }
  xvram_status blas_set_math_mode(void* h, uint32_t mode) {
    return run("cublasSetMathMode", [&]() -> Error {
      Handle* hd = handle(h);
      if (!hd)
        return invalid("cublasSetMathMode", "live handle required");
      // 0 default and 2 pedantic: strict FP32 (FFMA), as in the reference.  3 (TF32 tensor-op
      // math) selects the three-term TF32 tensor-core path, which is more accurate than the
      // single-TF32 products that mode permits.
      if (mode != 0 && mode != 2 && mode != 3)
        return unsupported("cublasSetMathMode", "math modes 0, 2 (strict FP32) and 3 (tensor cores) are supported");
      hd->math_mode = mode;
      return {};
    });
  }
  xvram_status blas_get_math_mode(void* h, uint32_t* out) {
    return run("cublasGetMathMode", [&]() -> Error {
      Handle* hd = handle(h);
      if (!hd || !host_ok(out, sizeof(*out)))
        return invalid("cublasGetMathMode", "live handle and host output required");
      *out = hd->math_mode;
      return {};
    });
  }

  xvram_status blas_sgemm(void* h, uint32_t op_a, uint32_t op_b, int32_t m, int32_t n, int32_t k,
                          const float* alpha, const float* a, int32_t lda, const float* b,
                          int32_t ldb, const float* beta, float* c, int32_t ldc) {
    // Host pointer mode: the scalars are read on the calling thread before the call is
    // admitted, as the reference does.
    return run("cublasSgemm", [&]() -> Error {
      if (!handle(h))
        return invalid("cublasSgemm", "live adapter handle required");
      if (op_a > 1 || op_b > 1 || m <= 0 || n <= 0 || k <= 0)
        return unsupported("cublasSgemm", "positive dimensions and N/T operations are required");
      if (!host_ok(alpha, sizeof(float)) || !host_ok(beta, sizeof(float)))
        return invalid("cublasSgemm", "alpha and beta must be host pointers");
      float alpha_v = 0, beta_v = 0;
      std::memcpy(&alpha_v, alpha, sizeof(float));
      std::memcpy(&beta_v, beta, sizeof(float));
      if (lda < (op_a == 0 ? m : k) || ldb < (op_b == 0 ? k : n) || ldc < m)
        return invalid("cublasSgemm", "leading dimension is too small");
      Entry* ae = lookup(a, sizeof(float));
      Entry* be = lookup(b, sizeof(float));
      Entry* ce = lookup(c, sizeof(float));
      if (!ae || !be || !ce)
        return invalid("cublasSgemm", "all matrices must be live adapter allocations");
      if ((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(b) |
           reinterpret_cast<uintptr_t>(c)) % alignof(float) != 0)
        return invalid("cublasSgemm", "FP32 matrices must be aligned");
      if (!std::isfinite(alpha_v) || !std::isfinite(beta_v))
        return unsupported("cublasSgemm", "finite host scalars are required");
      GemmCall call;
      GemmShape& s = call.shape;
      s.m = static_cast<uint64_t>(m);
      s.n = static_cast<uint64_t>(n);
      s.k = static_cast<uint64_t>(k);
      s.op_a = static_cast<int>(op_a);
      s.op_b = static_cast<int>(op_b);
      auto view = [](const Entry& e, const void* p, uint64_t rows, uint64_t cols, int32_t ld) {
        MatrixRef r;
        r.allocation_id = e.id;
        r.allocation_bytes = e.bytes;
        r.offset_bytes = reinterpret_cast<uintptr_t>(p) - e.base;
        r.rows = rows;
        r.columns = cols;
        r.ld = static_cast<uint64_t>(ld);
        return r;
      };
      s.a = view(*ae, a, op_a == 0 ? s.m : s.k, op_a == 0 ? s.k : s.m, lda);
      s.b = view(*be, b, op_b == 0 ? s.k : s.n, op_b == 0 ? s.n : s.k, ldb);
      s.c = view(*ce, c, s.m, s.n, ldc);
      // Math mode 3 (CUBLAS_TF32_TENSOR_OP_MATH) selects the three-term TF32 kernel.
      s.compute = handle(h)->math_mode == 3 ? kTf32 : kStrictFp32;
      const Validation v = validate_gemm(s);
      if (!v)
        return make_error(XVRAM_STATUS_INVALID_ARGUMENT, "compat_preflight", "cublasSgemm",
                          problem_error_name(v.error));
      call.alpha = alpha_v;
      call.beta = beta_v;
      if (s.compute == kTf32)
        call.flops_per_s = 150e12; // plan for the tensor-core rate
      // cuBLAS semantics: the call returns once the kernels are queued and the next
      // cudaMemcpy of C (or cudaDeviceSynchronize) waits for them and reports a failed
      // kernel.  XVRAM_B200_SYNC_GEMM=1 keeps the reference's synchronous completion.
      call.defer_completion = !sync_gemm_;
      if (Error e = runtime_->gemm(call))
        return e;
      std::lock_guard lock(snap_mu_);
      ++tel_.gemm_calls;
      return {};
    });
  }

  xvram_status extra(xvram_b200_runtime_info_v1* out) const {
    if (!has_size(out))
      return XVRAM_STATUS_INVALID_ARGUMENT;
    std::lock_guard lock(snap_mu_);
    const uint32_t size = out->struct_size;
    *out = info_;
    out->struct_size = size;
    return XVRAM_STATUS_SUCCESS;
  }

private:
  struct Entry {
    uint64_t id = 0, base = 0, bytes = 0, reserved = 0;
    bool live = true;
  };
  struct Handle {
    uint32_t math_mode = 0;
    bool live = true;
  };

  uint32_t state() const {
    std::lock_guard lock(snap_mu_);
    return tel_.state;
  }
  void set_state(uint32_t s) {
    std::lock_guard lock(snap_mu_);
    tel_.state = s;
    tel_.runtime.poisoned = s == XVRAM_CUDA_COMPAT_POISONED ? 1u : 0u;
  }
  void count_attempt() {
    std::lock_guard lock(snap_mu_);
    ++tel_.calls_attempted;
  }
  void count_submitted() {
    std::lock_guard lock(snap_mu_);
    ++tel_.calls_submitted;
  }
  xvram_status reject(const Error& e) {
    std::lock_guard lock(snap_mu_);
    error_ = e;
    ++tel_.calls_rejected;
    return e.status;
  }
  xvram_status complete() {
    std::lock_guard lock(snap_mu_);
    ++tel_.calls_completed;
    return XVRAM_STATUS_SUCCESS;
  }

  // Copies the runtime's counters into the published snapshot.
  void publish() {
    if (!runtime_)
      return;
    std::lock_guard lock(snap_mu_);
    const uint32_t size = tel_.runtime.struct_size;
    const uint32_t poisoned = tel_.runtime.poisoned;
    tel_.runtime = runtime_->counters();
    tel_.runtime.struct_size = size;
    tel_.runtime.poisoned = poisoned;
    const RuntimeExtra& x = runtime_->extra();
    tel_.tiles_submitted = x.tiles_submitted;
    tel_.tiles_retired = x.tiles_retired;
    tel_.host_backing_bytes = x.host_backing_bytes;
    tel_.host_backing_peak_bytes = x.host_backing_peak_bytes;
    tel_.host_budget_bytes = x.host_backing_bytes; // the host ledger now (current state)
    tel_.retired_va_reservations = x.retired_va_reservations;
    tel_.retired_va_bytes = x.retired_va_bytes;
    tel_.retired_va_reservations_freed = x.retired_va_reservations_freed;
    tel_.retired_va_bytes_freed = x.retired_va_bytes_freed;
    ++tel_.progress_sequence;
    info_.struct_size = sizeof(info_);
    info_.frame_bytes = runtime_->chunk_bytes();
    info_.frame_capacity = runtime_->frame_capacity();
    info_.gemm_in_place = x.gemm_in_place;
    info_.gemm_streamed = x.gemm_streamed;
    info_.last_block_m = static_cast<uint64_t>(x.last_mb);
    info_.last_block_n = static_cast<uint64_t>(x.last_nb);
    info_.last_panel_k = static_cast<uint64_t>(x.last_kb);
    info_.last_steps = static_cast<uint64_t>(x.last_steps);
    info_.last_panel_slots = static_cast<uint64_t>(x.last_panel_slots);
    info_.last_gemm_ms = x.last_gemm_ms;
    info_.gemm_deferred = x.gemm_deferred;
    info_.gemm_column_blocks = x.gemm_column_blocks;
    info_.panel_slot_refills = x.panel_slot_refills;
  }

  template <class F> xvram_status run(const char* op, F&& fn) {
    std::lock_guard call(call_mu_);
    count_attempt();
    const uint32_t st = state();
    if (st == XVRAM_CUDA_COMPAT_UNINITIALIZED || st == XVRAM_CUDA_COMPAT_INITIALIZING)
      return reject(make_error(XVRAM_STATUS_NOT_READY, "compat", op,
                               "explicit initialization is required and a closed adapter cannot reopen"));
    if (st == XVRAM_CUDA_COMPAT_CLOSED)
      return reject(make_error(XVRAM_STATUS_CLOSED, "compat", op,
                               "explicit initialization is required and a closed adapter cannot reopen"));
    if (st == XVRAM_CUDA_COMPAT_POISONED)
      return reject(make_error(XVRAM_STATUS_POISONED, "compat", op,
                               "adapter does not admit data operations in this lifecycle state"));
    count_submitted();
    Error err;
    try {
      DeviceScope scope(config_.session.device_ordinal);
      err = fn();
    } catch (const std::bad_alloc&) {
      err = make_error(XVRAM_STATUS_HOST_OUT_OF_MEMORY, "compat", op, "host allocation failed");
    } catch (const std::exception& ex) {
      err = make_error(XVRAM_STATUS_INTERNAL, "compat", op, ex.what());
    }
    publish();
    if (err) {
      if (poisons(err))
        set_state(XVRAM_CUDA_COMPAT_POISONED);
      return reject(err);
    }
    return complete();
  }

  // Live allocation containing [p, p + len).
  Entry* lookup(const void* p, uint64_t len) {
    const uint64_t addr = reinterpret_cast<uintptr_t>(p);
    auto it = allocs_.upper_bound(addr);
    if (it == allocs_.begin())
      return nullptr;
    --it;
    Entry& e = it->second;
    const uint64_t off = addr - e.base;
    return e.live && off <= e.bytes && len <= e.bytes - off ? &e : nullptr;
  }
  // True when [p, p + len) is a host range: non-null and touching no managed
  // (live or retired) reservation and no adapter handle.
  bool host_ok(const void* p, uint64_t len) const {
    if (!p)
      return false;
    const uint64_t addr = reinterpret_cast<uintptr_t>(p);
    const uint64_t extent = std::max<uint64_t>(len, 1);
    if (extent > UINT64_MAX - addr)
      return false;
    const uint64_t end = addr + extent;
    for (const auto& [base, e] : allocs_) {
      if (base >= end)
        break;
      if (base + e.reserved > addr)
        return false;
    }
    for (const auto& h : handles_) {
      const uint64_t v = reinterpret_cast<uintptr_t>(h.get());
      if (addr < v + sizeof(Handle) && v < end)
        return false;
    }
    return true;
  }
  Handle* handle(void* p) const {
    for (const auto& h : handles_)
      if (h.get() == p)
        return h->live ? h.get() : nullptr;
    return nullptr;
  }

  std::mutex call_mu_;
  mutable std::mutex snap_mu_;
  xvram_cuda_compat_telemetry_v1 tel_{};
  xvram_b200_runtime_info_v1 info_{};
  Error error_;
  xvram_cuda_compat_config_v1 config_{};
  bool attempted_ = false;
  bool sync_gemm_ = false; // blas_sgemm waits for its kernels (XVRAM_B200_SYNC_GEMM=1)
  std::unique_ptr<Runtime> runtime_;
  std::map<uint64_t, Entry> allocs_;
  std::vector<std::unique_ptr<Handle>> handles_;
};

Adapter& adapter() {
  static Adapter a;
  return a;
}

template <class F> xvram_status boundary(F&& f) noexcept {
  try {
    return f();
  } catch (...) {
    return XVRAM_STATUS_HOST_OUT_OF_MEMORY;
  }
}

const xvram_cuda_compat_api_v1& table() {
  static const xvram_cuda_compat_api_v1 t = [] {
    xvram_cuda_compat_api_v1 a{};
    a.struct_size = sizeof(a);
    a.abi_version = XVRAM_CUDA_COMPAT_ABI_VERSION_1;
    a.initialize = [](const xvram_cuda_compat_config_v1* c) {
      return boundary([&] { return adapter().initialize(c); });
    };
    a.shutdown = [] { return boundary([] { return adapter().shutdown(); }); };
    a.get_error = [](xvram_error_info_v1* o) { return boundary([&] { return adapter().get_error(o); }); };
    a.get_telemetry = [](xvram_cuda_compat_telemetry_v1* o) {
      return boundary([&] { return adapter().get_telemetry(o); });
    };
    a.malloc_device = [](void** o, uint64_t n) {
      return boundary([&] { return adapter().malloc_device(o, n); });
    };
    a.free_device = [](void* p) { return boundary([&] { return adapter().free_device(p); }); };
    a.memcpy = [](void* d, const void* s, uint64_t n, uint32_t k) {
      return boundary([&] { return adapter().memcpy_(d, s, n, k); });
    };
    a.get_device = [](int32_t* o) { return boundary([&] { return adapter().get_device(o); }); };
    a.get_device_count = [](int32_t* o) {
      return boundary([&] { return adapter().get_device_count(o); });
    };
    a.set_device = [](int32_t d) { return boundary([&] { return adapter().set_device(d); }); };
    a.synchronize = [] { return boundary([] { return adapter().synchronize(); }); };
    a.mem_get_info = [](uint64_t* f, uint64_t* t) {
      return boundary([&] { return adapter().mem_get_info(f, t); });
    };
    a.blas_create = [](void** o) { return boundary([&] { return adapter().blas_create(o); }); };
    a.blas_destroy = [](void* h) { return boundary([&] { return adapter().blas_destroy(h); }); };
    a.blas_get_version = [](void* h, int32_t* o) {
      return boundary([&] { return adapter().blas_get_version(h, o); });
    };
    a.blas_set_stream = [](void* h, uint64_t s) {
      return boundary([&] { return adapter().blas_set_stream(h, s); });
    };
    a.blas_get_stream = [](void* h, uint64_t* o) {
      return boundary([&] { return adapter().blas_get_stream(h, o); });
    };
    a.blas_set_pointer_mode = [](void* h, uint32_t m) {
      return boundary([&] { return adapter().blas_set_pointer_mode(h, m); });
    };
    a.blas_get_pointer_mode = [](void* h, uint32_t* o) {
      return boundary([&] { return adapter().blas_get_pointer_mode(h, o); });
    };
    a.blas_set_math_mode = [](void* h, uint32_t m) {
      return boundary([&] { return adapter().blas_set_math_mode(h, m); });
    };
    a.blas_get_math_mode = [](void* h, uint32_t* o) {
      return boundary([&] { return adapter().blas_get_math_mode(h, o); });
    };
    a.blas_sgemm = [](void* h, uint32_t oa, uint32_t ob, int32_t m, int32_t n, int32_t k,
                      const float* al, const float* ap, int32_t lda, const float* bp, int32_t ldb,
                      const float* be, float* cp, int32_t ldc) {
      return boundary(
          [&] { return adapter().blas_sgemm(h, oa, ob, m, n, k, al, ap, lda, bp, ldb, be, cp, ldc); });
    };
    return a;
  }();
  return t;
}

} // namespace

xvram_status compat_runtime_info(xvram_b200_runtime_info_v1* out) { return adapter().extra(out); }

} // namespace xvram

extern "C" XVRAM_CUDA_COMPAT_API xvram_status XVRAM_CALL
xvram_cuda_compat_get_api(uint32_t requested, uint32_t size, void* output) {
  if (!output)
    return XVRAM_STATUS_INVALID_ARGUMENT;
  if (requested != XVRAM_CUDA_COMPAT_ABI_VERSION_1 || size < sizeof(xvram_cuda_compat_api_v1))
    return XVRAM_STATUS_INCOMPATIBLE_ABI;
  std::memcpy(output, &xvram::table(), sizeof(xvram_cuda_compat_api_v1));
  return XVRAM_STATUS_SUCCESS;
}
