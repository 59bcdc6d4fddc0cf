// runtime_sanitize.cpp -- the residency runtime and planner under AddressSanitizer and
// UndefinedBehaviorSanitizer, driven over the host-memory fake device.
//
// TEST INFRASTRUCTURE: tests/test_sanitize_cpu.py compiles this file with runtime.cpp,
// planner.cpp, validate.cpp, host_util.cpp and tests/fake_device/fake_device.cpp under
// -fsanitize=address,undefined and runs it (the reference's CI runs its host code under
// the same sanitizers).  No CUDA is involved: the runtime reaches the device only through
// the Device interface, and the fake implements it on host memory.
//
// Scenarios, each checked against a plain double-precision loop:
//   1. in-place GEMM, synchronous, all four operations;
//   2. deferred GEMM split into column blocks (the fake reports 2 SMs), C read in pieces;
//   3. streamed (out-of-core) GEMM under a 16 MiB budget, with eviction and write-back;
//   4. a transaction writing C, a prefetch, and release of every allocation;
//   5. the live budget: a sampler thread polling every millisecond while free memory
//      drops and comes back.
// Exit status 0 means every check passed (and the sanitizers found nothing: they abort).
// Argument "quick" shortens K (for ThreadSanitizer, which runs the loops ~10x slower).
#include "device.hpp"
#include "runtime.hpp"

#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <memory>
#include <thread>
#include <vector>

extern "C" void* fake_device_create();
extern "C" void fake_device_set_memory(uint64_t free_bytes, uint64_t total_bytes);
extern "C" void fake_device_set_sm_count(int n);

namespace {

using namespace xvram;

int failures = 0;
uint64_t k_scale = 1; // K divisor for a quick run

void expect(bool ok, const char* what) {
  if (!ok) {
    std::fprintf(stderr, "FAILED: %s\n", what);
    ++failures;
  }
}

bool ok(const Error& e, const char* what) {
  if (e) {
    std::fprintf(stderr, "%s: status %d %s/%s %s\n", what, static_cast<int>(e.status),
                 e.stage.c_str(), e.operation.c_str(), e.message.c_str());
    ++failures;
    return false;
  }
  return true;
}

float value(uint64_t i, uint32_t salt) {
  return static_cast<float>(static_cast<int>((i * 2654435761u + salt * 40503u) % 61u) - 30) /
         64.0f;
}

struct Matrix {
  uint64_t id = 0, va = 0;
  std::vector<float> host;
};

Matrix make(Runtime& rt, uint64_t elems, uint32_t salt) {
  Matrix x;
  x.host.resize(elems);
  for (uint64_t i = 0; i < elems; ++i)
    x.host[i] = value(i, salt);
  ok(rt.allocate(elems * 4, &x.id, &x.va), "allocate");
  ok(rt.write(x.id, 0, x.host.data(), elems * 4), "write");
  return x;
}

MatrixRef ref(const Matrix& x, uint64_t rows, uint64_t cols, uint64_t ld) {
  MatrixRef r;
  r.allocation_id = x.id;
  r.allocation_bytes = x.host.size() * 4;
  r.rows = rows;
  r.columns = cols;
  r.ld = ld;
  return r;
}

// C (m x n, ldc) = alpha op(A) op(B) + beta C in double, from the host copies.
std::vector<double> reference(int op_a, int op_b, uint64_t m, uint64_t n, uint64_t k,
                              double alpha, const Matrix& a, uint64_t lda, const Matrix& b,
                              uint64_t ldb, double beta, const Matrix& c, uint64_t ldc) {
  std::vector<double> out(ldc * n);
  for (uint64_t j = 0; j < n; ++j)
    for (uint64_t i = 0; i < m; ++i) {
      double dot = 0;
      for (uint64_t p = 0; p < k; ++p)
        dot += static_cast<double>(a.host[op_a ? p + i * lda : i + p * lda]) *
               static_cast<double>(b.host[op_b ? j + p * ldb : p + j * ldb]);
      out[i + j * ldc] = alpha * dot + beta * static_cast<double>(c.host[i + j * ldc]);
    }
  return out;
}

void check_c(Runtime& rt, const Matrix& c, const std::vector<double>& want, uint64_t m,
             uint64_t n, uint64_t ldc, uint64_t k, bool in_pieces, const char* what) {
  std::vector<float> got(ldc * n);
  if (in_pieces) { // cuts that fall inside column blocks
    const uint64_t total = got.size() * 4;
    const uint64_t cuts[] = {0, 4 * (ldc * 37 + 5), 4 * (ldc * 300 + 1), total};
    for (int i = 0; i < 3; ++i)
      ok(rt.read(c.id, cuts[i], reinterpret_cast<char*>(got.data()) + cuts[i],
                 cuts[i + 1] - cuts[i]),
         "read piece");
  } else {
    ok(rt.read(c.id, 0, got.data(), got.size() * 4), "read");
  }
  double worst = 0;
  for (uint64_t j = 0; j < n; ++j)
    for (uint64_t i = 0; i < m; ++i)
      worst = std::max(worst, std::fabs(got[i + j * ldc] - want[i + j * ldc]));
  expect(worst <= 1e-6 * static_cast<double>(k), what);
}

std::unique_ptr<Device> fake() { return std::unique_ptr<Device>(static_cast<Device*>(fake_device_create())); }

void gemms(bool deferred) {
  fake_device_set_sm_count(2);
  fake_device_set_memory(1ull << 30, 2ull << 30);
  Runtime rt;
  RuntimeConfig cfg;
  cfg.chunk_bytes = 2ull << 20;
  cfg.headroom_bytes = 0;
  cfg.cache_target_bytes = 64ull << 20;
  if (!ok(rt.open(cfg, fake()), "open"))
    return;
  const uint64_t m = 300, n = 700, k = 48 / k_scale, ldc = m + 3;
  for (int op_a = 0; op_a < 2; ++op_a)
    for (int op_b = 0; op_b < 2; ++op_b) {
      const uint64_t lda = op_a ? k : m, ldb = op_b ? n : k;
      Matrix a = make(rt, lda * (op_a ? m : k), 1 + op_a);
      Matrix b = make(rt, ldb * (op_b ? k : n), 3 + op_b);
      Matrix c = make(rt, ldc * n, 5);
      GemmCall call;
      call.shape.m = m;
      call.shape.n = n;
      call.shape.k = k;
      call.shape.op_a = op_a;
      call.shape.op_b = op_b;
      call.shape.a = ref(a, op_a ? k : m, op_a ? m : k, lda);
      call.shape.b = ref(b, op_b ? n : k, op_b ? k : n, ldb);
      call.shape.c = ref(c, m, n, ldc);
      call.alpha = 0.5;
      call.beta = -1.5;
      call.defer_completion = deferred;
      ok(rt.gemm(call), "gemm");
      check_c(rt, c, reference(op_a, op_b, m, n, k, 0.5, a, lda, b, ldb, -1.5, c, ldc), m, n,
              ldc, k, deferred && op_a == 1, deferred ? "deferred gemm" : "in-place gemm");
      ok(rt.release(a.id), "release");
      ok(rt.release(b.id), "release");
      ok(rt.release(c.id), "release");
    }
  expect(!deferred || rt.extra().gemm_column_blocks > 4, "column blocks used");
  ok(rt.close(), "close");
}

void streamed_and_transaction() {
  fake_device_set_sm_count(148);
  fake_device_set_memory(1ull << 30, 2ull << 30);
  Runtime rt;
  RuntimeConfig cfg;
  cfg.chunk_bytes = 2ull << 20;
  cfg.headroom_bytes = 0;
  cfg.cache_target_bytes = 16ull << 20;
  if (!ok(rt.open(cfg, fake()), "open"))
    return;
  // 2048 x 2048 C (16 MiB) plus A and B: more chunks than the 8 frames
  const uint64_t m = 2048, n = 2048, k = 256 / k_scale;
  Matrix a = make(rt, m * k, 7), b = make(rt, k * n, 8), c = make(rt, m * n, 9);
  GemmCall call;
  call.shape.m = m;
  call.shape.n = n;
  call.shape.k = k;
  call.shape.a = ref(a, m, k, m);
  call.shape.b = ref(b, k, n, k);
  call.shape.c = ref(c, m, n, m);
  call.alpha = 1.0;
  call.beta = 1.0;
  ok(rt.gemm(call), "streamed gemm");
  expect(rt.extra().gemm_streamed == 1, "the gemm streamed");
  check_c(rt, c, reference(0, 0, m, n, k, 1.0, a, m, b, k, 1.0, c, m), m, n, m, k, false,
          "streamed gemm");
  // A transaction doubling C in place (the fake's device memory is host memory).
  std::vector<AccessRange> ranges{{c.id, 0, m * n * 4, 1}};
  ok(rt.transaction(ranges, 0,
                    [&](const std::vector<ResolvedRange>& r, uint64_t, uint64_t, uint64_t) {
                      float* p = reinterpret_cast<float*>(r[0].device_address);
                      for (uint64_t i = 0; i < m * n; ++i)
                        p[i] *= 2.0f;
                      return Error{};
                    }),
     "transaction");
  std::vector<float> got(m * n);
  ok(rt.read(c.id, 0, got.data(), got.size() * 4), "read");
  const std::vector<double> want = reference(0, 0, m, n, k, 1.0, a, m, b, k, 1.0, c, m);
  double worst = 0;
  for (uint64_t i = 0; i < m * n; ++i)
    worst = std::max(worst, std::fabs(got[i] - 2.0 * want[i]));
  expect(worst <= 2e-6 * k, "transaction result");
  ok(rt.prefetch({{a.id, 0, 4096, 0}}), "prefetch");
  ok(rt.release(a.id), "release");
  ok(rt.release(b.id), "release");
  ok(rt.release(c.id), "release");
  ok(rt.close(), "close");
}

void live_budget() {
  fake_device_set_memory(64ull << 20, 2ull << 30);
  Runtime rt;
  RuntimeConfig cfg;
  cfg.chunk_bytes = 2ull << 20;
  cfg.headroom_bytes = 0;
  cfg.budget_poll_ms = 1;
  if (!ok(rt.open(cfg, fake()), "open"))
    return;
  std::vector<Matrix> blocks;
  for (int i = 0; i < 12; ++i)
    blocks.push_back(make(rt, 512 * 1024, 20 + i));
  fake_device_set_memory(0, 2ull << 30);
  std::this_thread::sleep_for(std::chrono::milliseconds(20));
  ok(rt.prefetch({{blocks.back().id, 0, 4096, 0}}), "prefetch");
  expect(rt.counters().budget_shrinks >= 1, "budget shrank");
  for (const Matrix& x : blocks) {
    std::vector<float> got(x.host.size());
    ok(rt.read(x.id, 0, got.data(), got.size() * 4), "read");
    expect(std::memcmp(got.data(), x.host.data(), got.size() * 4) == 0, "data survives shrink");
  }
  fake_device_set_memory(64ull << 20, 2ull << 30);
  for (int i = 0; i < 6; ++i) {
    std::this_thread::sleep_for(std::chrono::milliseconds(5));
    ok(rt.prefetch({{blocks.back().id, 0, 4096, 0}}), "prefetch");
  }
  expect(rt.counters().budget_grows >= 1, "budget grew back");
  ok(rt.close(), "close");
}

} // namespace

int main(int argc, char** argv) {
  if (argc > 1 && std::strcmp(argv[1], "quick") == 0)
    k_scale = 4;
  gemms(false);
  gemms(true);
  streamed_and_transaction();
  live_budget();
  std::printf("%s (%d failures)\n", failures ? "FAILED" : "ok", failures);
  return failures ? 1 : 0;
}
