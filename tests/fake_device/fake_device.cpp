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
//   * sgemm is a plain FP32 loop (fmaf in k order per output), alpha / beta as the
//     kernels apply them;
//   * mem_get_info reports a settable free-byte figure (for the live budget);
//   * any operation can be made to fail after a number of calls (failure paths).
#include "device.hpp"

#include <sys/mman.h>
#include <unistd.h>

#include <atomic>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <string>

namespace {

std::atomic<uint64_t> g_free{8ull << 30};
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

class FakeDevice final : public xvram::Device {
public:
  xvram::Error open(int ordinal, xvram::DeviceInfo* info) override {
    info->ordinal = ordinal;
    info->device_count = 1;
    info->name = "fake host-memory device";
    info->total_bytes = g_total.load();
    info->sm_count = 148;
    info->vmm_granularity = kGranularity;
    info->driver_version = 0;
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

  xvram::Error sgemm(int op_a, int op_b, int64_t m, int64_t n, int64_t k, float alpha,
                     uint64_t a, int64_t lda, uint64_t b, int64_t ldb, float beta, uint64_t c,
                     int64_t ldc, uint64_t, uint64_t, bool, xvram::StreamId) override {
    if (should_fail("sgemm"))
      return injected("sgemm");
    const float* A = reinterpret_cast<const float*>(a);
    const float* B = reinterpret_cast<const float*>(b);
    float* Cm = reinterpret_cast<float*>(c);
    for (int64_t j = 0; j < n; ++j)
      for (int64_t i = 0; i < m; ++i) {
        float acc = 0.0f;
        for (int64_t kk = 0; kk < k; ++kk) {
          const float x = op_a == 0 ? A[i + kk * lda] : A[kk + i * lda];
          const float y = op_b == 0 ? B[kk + j * ldb] : B[j + kk * ldb];
          acc = std::fmaf(x, y, acc);
        }
        float& out = Cm[i + j * ldc];
        const float v = alpha * acc;
        out = beta == 0.0f ? v : std::fmaf(beta, out, v);
      }
    ++gemms;
    return {};
  }
  uint64_t sgemm_workspace(int, int, int64_t, int64_t, int64_t, bool) override { return 0; }
  xvram::Error kernel_status(xvram::StreamId, uint32_t* word) override {
    *word = 0;
    return {};
  }
  uint64_t native_stream(xvram::StreamId) override { return 0; }

  uint64_t next_id = 0;
  uint64_t maps = 0, gemms = 0;
};

} // namespace

extern "C" {

__attribute__((visibility("default"))) void* fake_device_create() { return new FakeDevice(); }

__attribute__((visibility("default"))) void fake_device_set_memory(uint64_t free_bytes,
                                                                   uint64_t total_bytes) {
  g_free.store(free_bytes);
  g_total.store(total_bytes);
}

// The (after + 1)-th call of `op` ("copy_2d", "map", "handle_create", "sgemm") fails with
// an injected CUDA error; after < 0 clears the injection.
__attribute__((visibility("default"))) void fake_device_fail(const char* op, long after) {
  std::lock_guard<std::mutex> lk(g_fail_mu);
  g_fail_op = op ? op : "";
  g_fail_after = after;
}

} // extern "C"
