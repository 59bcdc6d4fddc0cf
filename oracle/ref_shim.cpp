// ref_shim.cpp -- C-callable wrappers over the reference's own CPU code.
//
// TEST INFRASTRUCTURE ONLY.  oracle/Makefile compiles this file together with the
// reference sources where they lie (src/compat_bench/pattern.cpp,
// src/gemm_bench/pattern.cpp, src/gemm/planner.cpp, src/residency/core.cpp) into
// oracle/_ref/libxvram_ref.so.  Nothing is copied out of the reference tree.  The
// library is used to pin the C oracle (tests/test_oracle_cpu.py), to generate
// tests/golden/ fixtures, and as bench.py's "reference" CPU baseline.
#include "compat_bench/pattern.hpp"
#include "gemm/planner.hpp"
#include "gemm_bench/pattern.hpp"

#include <cstring>
#include <string>
#include <cstdint>
#include <cstdio>
#include <thread>
#include <vector>

#define XR_EXPORT extern "C" __attribute__((visibility("default")))

namespace cb = xvram::compat_bench;
namespace gb = xvram::gemm_bench;
namespace gm = xvram::gemm;

XR_EXPORT float xr_cb_pattern_a(std::uint64_t row, std::uint64_t k, std::uint64_t seed) {
  return cb::pattern_a(row, k, seed);
}
XR_EXPORT float xr_cb_pattern_b(std::uint64_t k, std::uint64_t column, std::uint64_t seed) {
  return cb::pattern_b(k, column, seed);
}
XR_EXPORT float xr_cb_pattern_c(std::uint64_t row, std::uint64_t column) {
  return cb::pattern_c(row, column);
}
XR_EXPORT double xr_cb_reference_dot(std::uint64_t row, std::uint64_t column, std::uint64_t k,
                                     std::uint64_t seed, int full) {
  return cb::reference_dot(row, column, k, seed, full != 0);
}
XR_EXPORT double xr_cb_reference_result(std::uint64_t m, std::uint64_t n, std::uint64_t k,
                                        std::uint64_t row, std::uint64_t column,
                                        std::uint64_t seed, float alpha, float beta,
                                        std::uint32_t passes, int full) {
  cb::Shape s;
  s.m = m;
  s.n = n;
  s.k = k;
  return cb::reference_result(s, row, column, seed, alpha, beta, passes, full != 0);
}
// Fills `out` (count floats) exactly as the reference's compat bench fills a device
// allocation: padding value outside the matrix, pattern values inside.
XR_EXPORT int xr_cb_fill_pattern(float* out, std::uint64_t count, std::uint64_t start,
                                 std::uint64_t m, std::uint64_t n, std::uint64_t k,
                                 std::uint64_t padding, std::uint64_t offset, int transpose_a,
                                 int transpose_b, int operand, std::uint64_t seed) {
  cb::Shape s;
  s.m = m;
  s.n = n;
  s.k = k;
  s.padding = padding;
  s.offset = offset;
  s.transpose_a = transpose_a != 0;
  s.transpose_b = transpose_b != 0;
  const auto op = operand == 0 ? cb::Operand::a : (operand == 1 ? cb::Operand::b : cb::Operand::c);
  if (!cb::matrix_storage(s, op))
    return 1;
  cb::fill_pattern(std::span<float>(out, count), start, s, op, seed);
  return 0;
}
XR_EXPORT float xr_cb_padding_value() { return cb::padding_value; }

XR_EXPORT std::uint64_t xr_gb_a(std::uint64_t row, std::uint64_t k) {
  return gb::pattern_a_value(row, k);
}
XR_EXPORT std::uint64_t xr_gb_b(std::uint64_t k, std::uint64_t column) {
  return gb::pattern_b_value(k, column);
}
XR_EXPORT int xr_gb_expected(std::uint64_t row, std::uint64_t column, std::uint64_t k,
                             std::uint64_t* out) {
  const auto v = gb::pattern_expected_value(row, column, k);
  if (!v)
    return 1;
  *out = *v;
  return 0;
}

// gemm::validate_problem over a flat column-major FP32 problem description.  Returns the
// ProblemError enumerator value; *operand receives the operand letter (or 0).
XR_EXPORT int xr_validate_problem(std::uint64_t m, std::uint64_t n, std::uint64_t k, int op_a,
                                  int op_b, const std::uint64_t* alloc_ids,
                                  const std::uint64_t* alloc_bytes,
                                  const std::uint64_t* offsets, const std::uint64_t* rows,
                                  const std::uint64_t* cols, const std::uint64_t* lds,
                                  char* operand) {
  gm::GemmProblem p;
  p.m = m;
  p.n = n;
  p.k = k;
  gm::MatrixView* views[3] = {&p.a, &p.b, &p.c};
  for (int i = 0; i < 3; ++i) {
    views[i]->allocation_id.value = alloc_ids[i];
    views[i]->allocation_bytes = alloc_bytes[i];
    views[i]->offset_bytes = offsets[i];
    views[i]->rows = rows[i];
    views[i]->columns = cols[i];
    views[i]->leading_dimension = lds[i];
    views[i]->layout = gm::MatrixLayout::column_major;
    views[i]->element_type = gm::ElementType::fp32;
  }
  p.a_operation = op_a == 0 ? gm::MatrixOperation::none : gm::MatrixOperation::transpose;
  p.b_operation = op_b == 0 ? gm::MatrixOperation::none : gm::MatrixOperation::transpose;
  p.compute_mode = gm::ComputeMode::strict_fp32;
  const auto v = gm::validate_problem(p);
  *operand = v.operand;
  return static_cast<int>(v.error);
}

// The compat bench's report digest over `count` floats, as the 32 hex digits of its two
// lanes (b, then a, as Digest::string prints them; formatted here with snprintf so no
// iostream state crosses into the host process) plus the terminating zero in out.
XR_EXPORT void xr_cb_digest(const float* values, std::uint64_t count, char* out) {
  cb::Digest d;
  for (std::uint64_t i = 0; i < count; ++i)
    d.add(values[i]);
  std::snprintf(out, 33, "%016llx%016llx", static_cast<unsigned long long>(d.b),
                static_cast<unsigned long long>(d.a));
}

// gemm::validate_problem with element types (A, B, C; gemm::ElementType order) and a
// compute mode (gemm::ComputeMode order); values outside the enumerations pass through as
// they are (the reference's own checks classify them).
XR_EXPORT int xr_validate_problem_typed(std::uint64_t m, std::uint64_t n, std::uint64_t k,
                                        int op_a, int op_b, const std::uint64_t* alloc_ids,
                                        const std::uint64_t* alloc_bytes,
                                        const std::uint64_t* offsets, const std::uint64_t* rows,
                                        const std::uint64_t* cols, const std::uint64_t* lds,
                                        const std::uint32_t* types, int compute, char* operand) {
  gm::GemmProblem p;
  p.m = m;
  p.n = n;
  p.k = k;
  gm::MatrixView* views[3] = {&p.a, &p.b, &p.c};
  for (int i = 0; i < 3; ++i) {
    views[i]->allocation_id.value = alloc_ids[i];
    views[i]->allocation_bytes = alloc_bytes[i];
    views[i]->offset_bytes = offsets[i];
    views[i]->rows = rows[i];
    views[i]->columns = cols[i];
    views[i]->leading_dimension = lds[i];
    views[i]->layout = gm::MatrixLayout::column_major;
    views[i]->element_type = static_cast<gm::ElementType>(types[i]);
  }
  p.a_operation = op_a == 0 ? gm::MatrixOperation::none : gm::MatrixOperation::transpose;
  p.b_operation = op_b == 0 ? gm::MatrixOperation::none : gm::MatrixOperation::transpose;
  p.compute_mode = static_cast<gm::ComputeMode>(compute);
  const auto v = gm::validate_problem(p);
  *operand = v.operand;
  return static_cast<int>(v.error);
}

// The reference's CPU FP64 GEMM (cb::reference_result with the full k loop) over the
// output elements [first, first + count) of an m x n column-major C, on `threads` host
// threads.  Returns the sum of the results so the work cannot be elided.
XR_EXPORT double xr_cpu_gemm_sample(std::uint64_t m, std::uint64_t n, std::uint64_t k,
                                    std::uint64_t first, std::uint64_t count, float alpha,
                                    float beta, std::uint64_t seed, int threads) {
  if (threads < 1)
    threads = 1;
  cb::Shape s;
  s.m = m;
  s.n = n;
  s.k = k;
  std::vector<double> partial(static_cast<std::size_t>(threads), 0.0);
  std::vector<std::thread> pool;
  for (int t = 0; t < threads; ++t) {
    pool.emplace_back([&, t] {
      const std::uint64_t b = first + count * t / threads, e = first + count * (t + 1) / threads;
      double acc = 0.0;
      for (std::uint64_t idx = b; idx < e; ++idx)
        acc += cb::reference_result(s, idx % m, idx / m, seed, alpha, beta, 1, true);
      partial[static_cast<std::size_t>(t)] = acc;
    });
  }
  for (auto& th : pool)
    th.join();
  double total = 0.0;
  for (double v : partial)
    total += v;
  return total;
}
