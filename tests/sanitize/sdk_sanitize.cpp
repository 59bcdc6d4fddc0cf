// sdk_sanitize.cpp -- the SDK v1 table (sessions, worker thread, operations) on the
// residency runtime, under the sanitizers, over the host-memory fake device.
//
// TEST INFRASTRUCTURE: tests/test_sanitize_cpu.py compiles this file with sdk_api.cpp,
// runtime.cpp, planner.cpp, validate.cpp, host_util.cpp and tests/fake_device/fake_device.cpp
// under -fsanitize=address,undefined and under -fsanitize=thread.  It supplies the
// library's device factory itself (the fake), so no CUDA is involved.
//
// One session (16 MiB budget, 2 MiB chunks, budget polled every millisecond by the
// runtime's sampler thread) runs, from the caller's thread while the session's worker
// thread executes them:
//   * an in-place FP32 GEMM (row-major) with gemm_execute;
//   * a streamed FP32 GEMM (C alone is 16 MiB) submitted as an operation, polled, waited;
//   * a second GEMM submitted behind it and cancelled (CANCELLED if still queued, BUSY
//     once running -- both are accepted);
//   * a transaction whose callback doubles C on the "device" (host memory in the fake);
//   * a prefetch, then every release and the session close.
// Results are checked against double-precision loops.  Exit status 0 means all passed.
#include "device.hpp"
#include "xvram/xvram.h"

#include <cmath>
#include <cstdio>
#include <cstring>
#include <memory>
#include <vector>

extern "C" void* fake_device_create();
extern "C" void fake_device_set_memory(uint64_t free_bytes, uint64_t total_bytes);

namespace xvram {
namespace {
std::unique_ptr<Device> make_fake() {
  return std::unique_ptr<Device>(static_cast<Device*>(fake_device_create()));
}
} // namespace
DeviceFactory& device_factory() {
  static DeviceFactory f = &make_fake;
  return f;
}
} // namespace xvram

namespace {

int failures = 0;

#define CHECK(call)                                                                          \
  do {                                                                                       \
    const xvram_status st_ = (call);                                                         \
    if (st_ != XVRAM_STATUS_SUCCESS) {                                                       \
      std::fprintf(stderr, "%s failed with status %d\n", #call, static_cast<int>(st_));       \
      ++failures;                                                                            \
      return;                                                                                \
    }                                                                                        \
  } while (0)

void expect(bool ok, const char* what) {
  if (!ok) {
    std::fprintf(stderr, "FAILED: %s\n", what);
    ++failures;
  }
}

float value(uint64_t i, uint32_t salt) {
  return static_cast<float>(static_cast<int>((i * 2654435761u + salt * 40503u) % 61u) - 30) /
         64.0f;
}

struct Host {
  std::vector<float> v;
  xvram_allocation a = nullptr;
};

xvram_status upload(const xvram_api_v1& api, xvram_session s, Host* h, uint64_t elems,
                    uint32_t salt) {
  h->v.resize(elems);
  for (uint64_t i = 0; i < elems; ++i)
    h->v[i] = value(i, salt);
  xvram_allocation_desc_v1 d = XVRAM_ALLOCATION_DESC_V1_INIT;
  d.size_bytes = elems * 4;
  if (xvram_status st = api.allocation_create(s, &d, &h->a); st != XVRAM_STATUS_SUCCESS)
    return st;
  return api.allocation_write(h->a, 0, h->v.data(), elems * 4);
}

// Row-major C (m x n) = alpha A (m x k) B (k x n) + beta C, all row-major.
xvram_gemm_desc_v1 row_major_gemm(const Host& a, const Host& b, const Host& c, uint64_t m,
                                  uint64_t n, uint64_t k, double alpha, double beta) {
  xvram_gemm_desc_v1 g = XVRAM_GEMM_DESC_V1_INIT;
  g.a.allocation = a.a;
  g.a.rows = m;
  g.a.columns = k;
  g.a.leading_dimension = k;
  g.b.allocation = b.a;
  g.b.rows = k;
  g.b.columns = n;
  g.b.leading_dimension = n;
  g.c.allocation = c.a;
  g.c.rows = m;
  g.c.columns = n;
  g.c.leading_dimension = n;
  g.compute_mode = XVRAM_COMPUTE_FP32_STRICT;
  g.alpha = alpha;
  g.beta = beta;
  return g;
}

double worst_error(const xvram_api_v1& api, const Host& a, const Host& b, const Host& c,
                   uint64_t m, uint64_t n, uint64_t k, double alpha, double beta,
                   double scale) {
  std::vector<float> got(m * n);
  if (api.allocation_read(c.a, 0, got.data(), got.size() * 4) != XVRAM_STATUS_SUCCESS)
    return INFINITY;
  double worst = 0;
  for (uint64_t i = 0; i < m; ++i)
    for (uint64_t j = 0; j < n; ++j) {
      double dot = 0;
      for (uint64_t p = 0; p < k; ++p)
        dot += static_cast<double>(a.v[i * k + p]) * static_cast<double>(b.v[p * n + j]);
      const double want = scale * (alpha * dot + beta * static_cast<double>(c.v[i * n + j]));
      worst = std::max(worst, std::fabs(got[i * n + j] - want));
    }
  return worst;
}

xvram_status XVRAM_CALL double_c(const xvram_transaction_context_v1* ctx, void*,
                                 xvram_error_info_v1*) {
  float* p = reinterpret_cast<float*>(ctx->ranges[0].device_address);
  for (uint64_t i = 0; i < ctx->ranges[0].length_bytes / 4; ++i)
    p[i] *= 2.0f;
  return XVRAM_STATUS_SUCCESS;
}

void run() {
  fake_device_set_memory(1ull << 30, 2ull << 30);
  xvram_api_v1 api;
  std::memset(&api, 0, sizeof api);
  CHECK(xvram_get_api(XVRAM_ABI_VERSION_1, static_cast<uint32_t>(sizeof api), &api));
  xvram_session_config_v1 cfg = XVRAM_SESSION_CONFIG_V1_INIT;
  cfg.cache_target_bytes = 16ull << 20;
  cfg.chunk_size_bytes = 2ull << 20;
  cfg.device_headroom_bytes = 0;
  cfg.budget_poll_ms = 1;
  xvram_session s = nullptr;
  CHECK(api.session_create(&cfg, &s));

  { // in place, gemm_execute
    const uint64_t m = 200, n = 300, k = 40;
    Host a, b, c;
    CHECK(upload(api, s, &a, m * k, 1));
    CHECK(upload(api, s, &b, k * n, 2));
    CHECK(upload(api, s, &c, m * n, 3));
    xvram_gemm_desc_v1 g = row_major_gemm(a, b, c, m, n, k, 0.5, 1.5);
    xvram_gemm_plan plan = nullptr;
    CHECK(api.gemm_plan_create(s, &g, &plan));
    CHECK(api.gemm_execute(plan, XVRAM_TIMEOUT_INFINITE));
    api.gemm_plan_release(plan);
    expect(worst_error(api, a, b, c, m, n, k, 0.5, 1.5, 1.0) <= 1e-6 * k, "in-place gemm");
    CHECK(api.allocation_release(a.a));
    CHECK(api.allocation_release(b.a));
    CHECK(api.allocation_release(c.a));
  }

  { // streamed, submitted; a second one submitted behind it and cancelled
    const uint64_t m = 2048, n = 2048, k = 16;
    Host a, b, c;
    CHECK(upload(api, s, &a, m * k, 4));
    CHECK(upload(api, s, &b, k * n, 5));
    CHECK(upload(api, s, &c, m * n, 6));
    xvram_gemm_desc_v1 g = row_major_gemm(a, b, c, m, n, k, 1.0, 1.0);
    xvram_gemm_plan plan = nullptr;
    CHECK(api.gemm_plan_create(s, &g, &plan));
    xvram_gemm_plan_info_v1 info = XVRAM_GEMM_PLAN_INFO_V1_INIT;
    CHECK(api.gemm_plan_get_info(plan, &info));
    expect(info.tile_count > 1, "the plan streams");
    xvram_operation first = nullptr, second = nullptr;
    CHECK(api.gemm_submit(plan, &first));
    CHECK(api.gemm_submit(plan, &second));
    const xvram_status cancel = api.operation_cancel(second);
    expect(cancel == XVRAM_STATUS_SUCCESS || cancel == XVRAM_STATUS_BUSY, "cancel answer");
    xvram_operation_info_v1 oi = XVRAM_OPERATION_INFO_V1_INIT;
    CHECK(api.operation_poll(first, &oi));
    CHECK(api.operation_wait(first, XVRAM_TIMEOUT_INFINITE, &oi));
    expect(oi.state == XVRAM_OPERATION_COMPLETED, "first gemm completed");
    xvram_operation_info_v1 oi2 = XVRAM_OPERATION_INFO_V1_INIT;
    const xvram_status w2 = api.operation_wait(second, XVRAM_TIMEOUT_INFINITE, &oi2);
    const bool cancelled = oi2.state == XVRAM_OPERATION_CANCELLED;
    expect(cancelled || (w2 == XVRAM_STATUS_SUCCESS && oi2.state == XVRAM_OPERATION_COMPLETED),
           "second gemm cancelled or completed");
    api.operation_release(first);
    api.operation_release(second);
    api.gemm_plan_release(plan);
    // With beta = 1 each completed GEMM adds A B once more.
    std::vector<float> got(m * n);
    CHECK(api.allocation_read(c.a, 0, got.data(), got.size() * 4));
    double worst = 0;
    const double runs = cancelled ? 1.0 : 2.0;
    for (uint64_t i = 0; i < m; i += 7)
      for (uint64_t j = 0; j < n; j += 5) {
        double dot = 0;
        for (uint64_t p = 0; p < k; ++p)
          dot += static_cast<double>(a.v[i * k + p]) * static_cast<double>(b.v[p * n + j]);
        worst = std::max(worst, std::fabs(got[i * n + j] - (runs * dot + c.v[i * n + j])));
      }
    expect(worst <= 1e-6 * k, "streamed gemm");
    // A transaction doubling C, then a prefetch.
    xvram_access_range_v1 r{c.a, 0, m * n * 4, XVRAM_ACCESS_READ_WRITE, 0};
    xvram_transaction_desc_v1 t{};
    t.struct_size = sizeof t;
    t.ranges = &r;
    t.range_count = 1;
    t.callback = &double_c;
    // The transaction's ranges must fit the budget: one 2 MiB chunk of C at a time.
    r.length_bytes = 2ull << 20;
    CHECK(api.transaction_execute(s, &t, XVRAM_TIMEOUT_INFINITE));
    std::vector<float> after(512 * 1024);
    CHECK(api.allocation_read(c.a, 0, after.data(), after.size() * 4));
    bool doubled = true;
    for (size_t i = 0; i < after.size(); i += 97)
      doubled = doubled && after[i] == 2.0f * got[i];
    expect(doubled, "transaction doubled C");
    xvram_prefetch_desc_v1 pd{};
    pd.struct_size = sizeof pd;
    xvram_access_range_v1 pr{a.a, 0, 4096, XVRAM_ACCESS_READ, 0};
    pd.ranges = &pr;
    pd.range_count = 1;
    xvram_operation pf = nullptr;
    CHECK(api.prefetch_submit(s, &pd, &pf));
    CHECK(api.operation_wait(pf, XVRAM_TIMEOUT_INFINITE, &oi));
    api.operation_release(pf);
    CHECK(api.allocation_release(a.a));
    CHECK(api.allocation_release(b.a));
    CHECK(api.allocation_release(c.a));
  }
  CHECK(api.session_close(s, XVRAM_TIMEOUT_INFINITE));
  api.session_release(s);
}

} // namespace

int main() {
  run();
  std::printf("%s (%d failures)\n", failures ? "FAILED" : "ok", failures);
  return failures ? 1 : 0;
}
