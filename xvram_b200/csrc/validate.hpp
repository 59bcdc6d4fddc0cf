// validate.hpp -- GEMM problem validation with the reference's error taxonomy.
//
// Restates the rules of reference src/gemm/planner.cpp:40-110 (validate_matrix,
// matrix_bounds) and :785-859 (validate_problem) for column-major problems of any of the
// reference's element types: the same checks in the same order produce the same
// ProblemError enumerator, so a caller sees identical failure classes.
// tests/test_validate_cpu.py checks this against the reference's own function on the
// golden table in tests/golden/reference_vectors.json.
#pragma once

#include <cstdint>

namespace xvram {

// Enumerator values match reference src/gemm/planner.hpp:69-84.
enum class ProblemError : int {
  none = 0,
  zero_dimension = 1,
  invalid_allocation = 2,
  invalid_layout = 3,
  invalid_operation = 4,
  invalid_element_type = 5,
  invalid_compute_mode = 6,
  dimension_mismatch = 7,
  leading_dimension_too_small = 8,
  storage_overflow = 9,
  storage_out_of_bounds = 10,
  unsupported_type_combination = 11,
  output_aliases_input = 12,
  integer_limit_exceeded = 13,
};

const char* problem_error_name(ProblemError e);

// Element types, numbered as the reference's gemm::ElementType and the SDK's
// XVRAM_DATA_* (reference src/gemm/planner.hpp:25-30, include/xvram/xvram.h).
enum DataType : uint32_t { kFp16 = 0, kBf16 = 1, kFp32 = 2, kFp64 = 3 };
// Bytes per element; 0 for a value that is not an element type.
inline uint64_t element_bytes(uint32_t t) {
  return t == kFp16 || t == kBf16 ? 2 : t == kFp32 ? 4 : t == kFp64 ? 8 : 0;
}

// Arithmetic, numbered as the reference's gemm::ComputeMode (planner.hpp:32-36):
// strict FP32 (every product and sum an FP32 FMA), TF32 tensor cores (here the three-term
// TF32 kernel, FP32-accurate within the stated tolerance), FP64.
enum ComputeKind : int { kStrictFp32 = 0, kTf32 = 1, kComputeFp64 = 2 };

// A column-major matrix inside a managed allocation.
struct MatrixRef {
  uint64_t allocation_id = 0;
  uint64_t allocation_bytes = 0;
  uint64_t offset_bytes = 0;
  uint64_t rows = 0;
  uint64_t columns = 0;
  uint64_t ld = 0;
  uint32_t dtype = kFp32;
};

struct GemmShape {
  uint64_t m = 0, n = 0, k = 0;
  int op_a = 0, op_b = 0; // 0 = N, 1 = T
  int compute = kStrictFp32;
  MatrixRef a, b, c;
};

// The type rule of reference planner.cpp:819-842: A and B share a type; FP16 / BF16
// inputs give an FP16 / BF16 (same type) or FP32 C with strict FP32 arithmetic; FP32
// inputs give FP32 with strict or TF32 arithmetic; FP64 gives FP64 with FP64 arithmetic.
bool supported_types(uint32_t ab, uint32_t c, int compute);

struct Validation {
  ProblemError error = ProblemError::none;
  char operand = 0;
  explicit operator bool() const { return error == ProblemError::none; }
};

Validation validate_gemm(const GemmShape& s);

// First and one-past-last byte (relative to the allocation) a matrix touches.
bool matrix_byte_span(const MatrixRef& m, uint64_t* begin, uint64_t* end);

} // namespace xvram
