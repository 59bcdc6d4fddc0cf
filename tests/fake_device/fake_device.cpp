// fake_device.cpp -- a host-memory stand-in for the library's Device interface, for tests.
//
// TEST INFRASTRUCTURE ONLY: built by tests/fake_device.py into tests/_build and installed
// with xvram_b200_test_set_device_factory.  It lets the CPU test suite drive the residency
// runtime, the out-of-core executor, transactions and the live budget without a GPU, the
// way the reference's fake driver tables do (reference
// tests/unit/residency_executor_fake_tests.cpp).  Nothing in the product links it.
//
// Memory model:
//   * "device addresses" are host addresses: va_reserve reserves an inaccessible range,
//     a physical handle is a memfd of the chunk size, map() places it at the address
//     (MAP_FIXED | MAP_SHARED) so contents survive unmap / remap like a VMM frame's;
//   * streams and events are immediate: every operation completes when it is issued;
//   * gemm is a plain loop per output in k order: FP32 fmaf for FP32 arithmetic (inputs
//     of any type widened exactly), FP64 fma for FP64, alpha / beta as the kernels apply
//     them; C of a narrower type is rounded to nearest even once;
//   * mem_get_info reports a settable free-byte figure (for the live budget);
//   * any operation can be made to fail after a number of calls (failure paths).
#include "device.hpp"

#include <sys/mman.h>
#include <unistd.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <vector>

namespace {

using WorkspaceFn = uint64_t (*)(uint32_t, uint32_t, int32_t, uint32_t, uint32_t, int64_t,
                                 int64_t, int64_t);
std::atomic<WorkspaceFn> g_workspace_fn{nullptr};
std::atomic<uint64_t> g_free{8ull << 30};
std::atomic<int> g_sm_count{148};
std::atomic<uint32_t> g_kernel_word{0};
std::atomic<uint64_t> g_gemm_calls{0}, g_prepares{0};
std::atomic<uint64_t> g_total{16ull << 30};
std::mutex g_fail_mu;
std::string g_fail_op;
long g_fail_after = -1; // calls of g_fail_op that still succeed; -1: never fail

bool should_fail(const char* op) {
  std::lock_guard<std::mutex> lk(g_fail_mu);
  if (g_fail_after < 0 || g_fail_op != op)
    return false;
  if (g_fail_after == 0) {
    g_fail_after = -1;
    return true;
  }
  --g_fail_after;
  return false;
}

xvram::Error injected(const char* op) {
  return xvram::cuda_error("fake_device", op, 999, "injected", "injected failure");
}

constexpr uint64_t kGranularity = 2ull << 20;

// IEEE binary16 / bfloat16 <-> float, round to nearest even, written from the format
// definitions (sign, biased exponent, fraction).
float half_to_float(uint16_t h) {
  const int sign = h >> 15, e = (h >> 10) & 31, f = h & 1023;
  float v;
  if (e == 0)
    v = std::ldexp(static_cast<float>(f), -24);
  else if (e == 31)
    v = f ? NAN : INFINITY;
  else
    v = std::ldexp(static_cast<float>(1024 + f), e - 25);
  return sign ? -v : v;
}
uint16_t float_to_half(float x) {
  const uint16_t sign = std::signbit(x) ? 0x8000 : 0;
  if (std::isnan(x))
    return sign | 0x7e00;
  const double ax = std::fabs(static_cast<double>(x));
  if (ax >= 65520.0) // at or past the midpoint between 65504 and 2^16
    return sign | 0x7c00;
  if (ax < std::ldexp(1.0, -14)) { // subnormal range: units of 2^-24
    const double q = std::nearbyint(std::ldexp(ax, 24));
    return sign | static_cast<uint16_t>(q); // q == 1024 is the smallest normal, as bits
  }
  int e = 0;
  std::frexp(ax, &e); // ax = fr * 2^e, fr in [0.5, 1)
  e -= 1;             // ax in [2^e, 2^(e+1))
  double q = std::nearbyint(std::ldexp(ax, 10 - e)); // [1024, 2048]
  if (q == 2048.0) {
    q = 1024.0;
    ++e;
  }
  if (e + 15 >= 31)
    return sign | 0x7c00;
  return sign | static_cast<uint16_t>(((e + 15) << 10) | (static_cast<int>(q) - 1024));
}
float bf16_to_float(uint16_t h) {
  const uint32_t u = static_cast<uint32_t>(h) << 16;
  float v;
  std::memcpy(&v, &u, 4);
  return v;
}
uint16_t float_to_bf16(float x) {
  uint32_t u;
  std::memcpy(&u, &x, 4);
  if (std::isnan(x))
    return static_cast<uint16_t>((u >> 16) | 0x40);
  u += 0x7fff + ((u >> 16) & 1); // round to nearest, ties to the even upper half
  return static_cast<uint16_t>(u >> 16);
}

double load(uint32_t type, uint64_t base, int64_t i) {
  switch (type) {
  case xvram::kFp16: return half_to_float(reinterpret_cast<const uint16_t*>(base)[i]);
  case xvram::kBf16: return bf16_to_float(reinterpret_cast<const uint16_t*>(base)[i]);
  case xvram::kFp32: return reinterpret_cast<const float*>(base)[i];
  default: return reinterpret_cast<const double*>(base)[i];
  }
}
void store(uint32_t type, uint64_t base, int64_t i, double v) {
  switch (type) {
  case xvram::kFp16: reinterpret_cast<uint16_t*>(base)[i] = float_to_half(static_cast<float>(v)); break;
  case xvram::kBf16: reinterpret_cast<uint16_t*>(base)[i] = float_to_bf16(static_cast<float>(v)); break;
  case xvram::kFp32: reinterpret_cast<float*>(base)[i] = static_cast<float>(v); break;
  default: reinterpret_cast<double*>(base)[i] = v; break;
  }
}

class FakeDevice final : public xvram::Device {
public:
  xvram::Error open(int ordinal, xvram::DeviceInfo* info) override {
    info->ordinal = ordinal;
    info->device_count = 1;
    info->name = "fake host-memory device";
    info->total_bytes = g_total.load();
    info->sm_count = g_sm_count.load();
    info->vmm_granularity = kGranularity;
    info->driver_version = 0;
    info->cc_major = 10;
    info->cc_minor = 0;
    return {};
  }
  xvram::Error close() override { return {}; }
  xvram::Error mem_get_info(uint64_t* free_bytes, uint64_t* total_bytes) override {
    *free_bytes = g_free.load();
    *total_bytes = g_total.load();
    return {};
  }

  xvram::Error va_reserve(uint64_t bytes, uint64_t* va) override {
    void* p = mmap(nullptr, bytes, PROT_NONE, MAP_PRIVATE | MAP_ANONYMOUS | MAP_NORESERVE, -1, 0);
    if (p == MAP_FAILED)
      return xvram::make_error(XVRAM_STATUS_HOST_OUT_OF_MEMORY, "fake_device", "va_reserve",
                               "mmap failed");
    *va = reinterpret_cast<uint64_t>(p);
    return {};
  }
  xvram::Error va_free(uint64_t va, uint64_t bytes) override {
    munmap(reinterpret_cast<void*>(va), bytes);
    return {};
  }
  xvram::Error handle_create(uint64_t bytes, uint64_t* handle) override {
    if (should_fail("handle_create"))
      return injected("handle_create");
    const int fd = memfd_create("xvram_fake_frame", 0);
    if (fd < 0 || ftruncate(fd, static_cast<off_t>(bytes)) != 0)
      return xvram::make_error(XVRAM_STATUS_HOST_OUT_OF_MEMORY, "fake_device", "handle_create",
                               "memfd failed");
    *handle = static_cast<uint64_t>(fd) + 1; // 0 is never a handle
    return {};
  }
  xvram::Error handle_release(uint64_t handle) override {
    ::close(static_cast<int>(handle - 1));
    return {};
  }
  xvram::Error map(uint64_t va, uint64_t bytes, uint64_t handle) override {
    if (should_fail("map"))
      return injected("map");
    void* p = mmap(reinterpret_cast<void*>(va), bytes, PROT_READ | PROT_WRITE,
                   MAP_SHARED | MAP_FIXED, static_cast<int>(handle - 1), 0);
    if (p == MAP_FAILED)
      return xvram::make_error(XVRAM_STATUS_INTERNAL, "fake_device", "map", "mmap failed");
    ++maps;
    return {};
  }
  xvram::Error unmap(uint64_t va, uint64_t bytes) override {
    // Put the reservation back: the range stays owned, its pages inaccessible.
    void* p = mmap(reinterpret_cast<void*>(va), bytes, PROT_NONE,
                   MAP_PRIVATE | MAP_ANONYMOUS | MAP_NORESERVE | MAP_FIXED, -1, 0);
    if (p == MAP_FAILED)
      return xvram::make_error(XVRAM_STATUS_INTERNAL, "fake_device", "unmap", "mmap failed");
    return {};
  }

  xvram::Error host_alloc(uint64_t bytes, void** out) override {
    *out = std::aligned_alloc(4096, (bytes + 4095) / 4096 * 4096);
    return *out ? xvram::Error{}
                : xvram::make_error(XVRAM_STATUS_HOST_OUT_OF_MEMORY, "fake_device",
                                    "host_alloc", "out of host memory");
  }
  xvram::Error host_free(void* p) override {
    std::free(p);
    return {};
  }

  xvram::Error stream_create(xvram::StreamId* out) override {
    *out = ++next_id;
    return {};
  }
  xvram::Error stream_destroy(xvram::StreamId) override { return {}; }
  xvram::Error stream_sync(xvram::StreamId) override { return {}; }
  xvram::Error event_create(xvram::EventId* out) override {
    *out = ++next_id;
    return {};
  }
  xvram::Error event_destroy(xvram::EventId) override { return {}; }
  xvram::Error event_record(xvram::EventId, xvram::StreamId) override { return {}; }
  xvram::Error stream_wait_event(xvram::StreamId, xvram::EventId) override { return {}; }
  xvram::Error event_sync(xvram::EventId) override { return {}; }
  xvram::Error event_elapsed_ms(xvram::EventId, xvram::EventId, float* ms) override {
    *ms = 0.0f;
    return {};
  }

  xvram::Error copy_2d(uint64_t dst, uint64_t dpitch, uint64_t src, uint64_t spitch,
                       uint64_t width, uint64_t height, xvram::CopyDir, xvram::StreamId) override {
    if (should_fail("copy_2d"))
      return injected("copy_2d");
    for (uint64_t r = 0; r < height; ++r)
      std::memcpy(reinterpret_cast<void*>(dst + r * dpitch),
                  reinterpret_cast<const void*>(src + r * spitch), width);
    return {};
  }
  xvram::Error memset_d32(uint64_t dst, uint32_t value, uint64_t count, xvram::StreamId) override {
    uint32_t* p = reinterpret_cast<uint32_t*>(dst);
    for (uint64_t i = 0; i < count; ++i)
      p[i] = value;
    return {};
  }

  xvram::Error gemm(const xvram::GemmTypes& t, int op_a, int op_b, int64_t m, int64_t n,
                    int64_t k, double alpha, uint64_t a, int64_t lda, uint64_t b, int64_t ldb,
                    double beta, uint64_t c, int64_t ldc, uint64_t, uint64_t,
                    xvram::StreamId) override {
    if (should_fail("sgemm"))
      return injected("sgemm");
    if (t.compute == xvram::kComputeFp64)
      contract<double>(t, op_a, op_b, m, n, k, alpha, a, lda, b, ldb, beta, c, ldc);
    else // strict FP32 (the fake computes TF32 requests in strict FP32 too)
      contract<float>(t, op_a, op_b, m, n, k, alpha, a, lda, b, ldb, beta, c, ldc);
    ++gemms;
    ++g_gemm_calls;
    return {};
  }
  // Per output: one FMA chain in k order in T, then alpha * acc (+ beta * C as one FMA),
  // stored to C's type.  Operands are widened first (exactly); loops run j, k, i so the
  // inner loop is contiguous.
  template <class T>
  void contract(const xvram::GemmTypes& t, int op_a, int op_b, int64_t m, int64_t n, int64_t k,
                double alpha, uint64_t a, int64_t lda, uint64_t b, int64_t ldb, double beta,
                uint64_t c, int64_t ldc) {
    std::vector<T> A(static_cast<size_t>(m * k)), col(static_cast<size_t>(k)),
        acc(static_cast<size_t>(m));
    for (int64_t kk = 0; kk < k; ++kk)
      for (int64_t i = 0; i < m; ++i)
        A[static_cast<size_t>(i + kk * m)] =
            static_cast<T>(load(t.ab, a, op_a == 0 ? i + kk * lda : kk + i * lda));
    for (int64_t j = 0; j < n; ++j) {
      for (int64_t kk = 0; kk < k; ++kk)
        col[static_cast<size_t>(kk)] =
            static_cast<T>(load(t.ab, b, op_b == 0 ? kk + j * ldb : j + kk * ldb));
      std::fill(acc.begin(), acc.end(), T(0));
      for (int64_t kk = 0; kk < k; ++kk) {
        const T y = col[static_cast<size_t>(kk)];
        const T* ak = A.data() + kk * m;
        T* ac = acc.data();
        for (int64_t i = 0; i < m; ++i)
          ac[i] = std::fma(ak[i], y, ac[i]);
      }
      for (int64_t i = 0; i < m; ++i) {
        const int64_t ci = i + j * ldc;
        const T v = static_cast<T>(alpha) * acc[static_cast<size_t>(i)];
        store(t.c, c, ci,
              beta == 0.0 ? v
                          : std::fma(static_cast<T>(beta), static_cast<T>(load(t.c, c, ci)), v));
      }
    }
  }
  // The workspace the real kernels would ask for (the library's own sizing function,
  // installed by the test), so the planner budgets exactly as on a GPU; the fake's loops
  // do not use it.
  uint64_t gemm_workspace(const xvram::GemmTypes& t, int op_a, int op_b, int64_t m, int64_t n,
                          int64_t k) override {
    return g_workspace_fn ? g_workspace_fn(t.ab, t.c, t.compute, static_cast<uint32_t>(op_a),
                                           static_cast<uint32_t>(op_b), m, n, k)
                          : 0;
  }
  xvram::Error convert(uint32_t st, uint64_t src, int64_t lds, uint32_t dt, uint64_t dst,
                       int64_t ldd, int64_t rows, int64_t cols, xvram::StreamId) override {
    for (int64_t j = 0; j < cols; ++j)
      for (int64_t i = 0; i < rows; ++i)
        store(dt, dst, i + j * ldd, load(st, src, i + j * lds));
    ++conversions;
    return {};
  }
  // The fake keeps the operands where they are: preparing records them, and a block is the
  // plain loop over C's columns [n0, n0 + nj) (op(B)'s columns n0.. are B's columns for
  // op N, its rows for op T).
  xvram::Error gemm_prepare(const xvram::GemmTypes& t, int op_a, int op_b, int64_t, int64_t,
                            int64_t, uint64_t a, int64_t lda, uint64_t b, int64_t ldb, uint64_t,
                            uint64_t, xvram::StreamId, xvram::PreparedGemm* out) override {
    if (should_fail("sgemm"))
      return injected("sgemm");
    *out = xvram::PreparedGemm{};
    out->compute = t.compute;
    out->op_a = op_a;
    out->op_b = op_b;
    out->a = a;
    out->b = b;
    out->lda = lda;
    out->ldb = ldb;
    ++g_prepares;
    return {};
  }
  xvram::Error gemm_block(const xvram::PreparedGemm& p, int64_t m, int64_t n0, int64_t nj,
                          int64_t k, double alpha, double beta, uint64_t c, int64_t ldc,
                          xvram::StreamId) override {
    if (should_fail("sgemm"))
      return injected("sgemm");
    const xvram::GemmTypes t{xvram::kFp32, xvram::kFp32, static_cast<int>(p.compute)};
    const uint64_t b = p.b + static_cast<uint64_t>(p.op_b == 0 ? n0 * p.ldb : n0) * 4;
    contract<float>(t, p.op_a, p.op_b, m, nj, k, alpha, p.a, p.lda, b, p.ldb, beta, c, ldc);
    ++gemms;
    ++g_gemm_calls;
    return {};
  }
  // The kernels' sticky error word: a test may set it to stand for a kernel whose bounded
  // wait ran out; reading clears it, as on the device.
  xvram::Error kernel_status(xvram::StreamId, uint32_t* word) override {
    *word = g_kernel_word.exchange(0);
    return {};
  }
  uint64_t native_stream(xvram::StreamId) override { return 0; }

  xvram::Error make_current(int* previous) override {
    *previous = 0;
    return {};
  }
  void restore_current(int) override {}
  xvram::Error mem_alloc(uint64_t bytes, uint64_t* out) override {
    if (should_fail("mem_alloc"))
      return injected("mem_alloc");
    void* p = std::aligned_alloc(256, (std::max<uint64_t>(bytes, 1) + 255) / 256 * 256);
    if (!p)
      return xvram::make_error(XVRAM_STATUS_DEVICE_OUT_OF_MEMORY, "fake", "mem_alloc", "no memory");
    *out = reinterpret_cast<uint64_t>(p);
    return {};
  }
  xvram::Error mem_free(uint64_t p) override {
    std::free(reinterpret_cast<void*>(p));
    return {};
  }
  xvram::Error event_query(xvram::EventId, bool* done) override {
    *done = true; // immediate streams: everything recorded has completed
    return {};
  }
  xvram::Error transpose_f32(uint64_t src, int64_t lds, uint64_t dst, int64_t ldd, int64_t rows,
                             int64_t cols, xvram::StreamId) override {
    const float* s = reinterpret_cast<const float*>(src);
    float* d = reinterpret_cast<float*>(dst);
    for (int64_t c = 0; c < cols; ++c)
      for (int64_t r = 0; r < rows; ++r)
        d[c + r * ldd] = s[r + c * lds];
    return {};
  }

  uint64_t next_id = 0;
  uint64_t maps = 0, gemms = 0, conversions = 0;
};

} // namespace

extern "C" {

__attribute__((visibility("default"))) void* fake_device_create() { return new FakeDevice(); }

__attribute__((visibility("default"))) void fake_device_set_memory(uint64_t free_bytes,
                                                                   uint64_t total_bytes) {
  g_free.store(free_bytes);
  g_total.store(total_bytes);
}

// The library's xvram_b200_gemm_typed_workspace_bytes (or null: no workspace).
__attribute__((visibility("default"))) void fake_device_set_workspace_fn(void* fn) {
  g_workspace_fn.store(reinterpret_cast<WorkspaceFn>(fn));
}

// SM count reported by open() (the runtime sizes GEMM column blocks by it).
__attribute__((visibility("default"))) void fake_device_set_sm_count(int n) { g_sm_count.store(n); }

// The error word the next kernel_status returns.
__attribute__((visibility("default"))) void fake_device_set_kernel_word(uint32_t w) {
  g_kernel_word.store(w);
}

// GEMM launches (whole GEMMs and column blocks) and column-block preparations since load.
__attribute__((visibility("default"))) uint64_t fake_device_gemm_calls() { return g_gemm_calls.load(); }
__attribute__((visibility("default"))) uint64_t fake_device_prepares() { return g_prepares.load(); }

// The (after + 1)-th call of `op` ("copy_2d", "map", "handle_create", "sgemm") fails with
// an injected CUDA error; after < 0 clears the injection.
__attribute__((visibility("default"))) void fake_device_fail(const char* op, long after) {
  std::lock_guard<std::mutex> lk(g_fail_mu);
  g_fail_op = op ? op : "";
  g_fail_after = after;
}

} // extern "C"
