// validate.hpp -- GEMM problem validation with the reference's error taxonomy.
//
// Restates the rules of reference src/gemm/planner.cpp:40-110 (validate_matrix,
// matrix_bounds) and :785-859 (validate_problem) for column-major FP32 problems:
// the same checks in the same order produce the same ProblemError enumerator, so a
// caller sees identical failure classes.  tests/test_validate_cpu.py checks this
// against the reference's own function on the golden table in
// tests/golden/reference_vectors.json.
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

// A column-major FP32 matrix inside a managed allocation.
struct MatrixRef {
  uint64_t allocation_id = 0;
  uint64_t allocation_bytes = 0;
  uint64_t offset_bytes = 0;
  uint64_t rows = 0;
  uint64_t columns = 0;
  uint64_t ld = 0;
};

struct GemmShape {
  uint64_t m = 0, n = 0, k = 0;
  int op_a = 0, op_b = 0; // 0 = N, 1 = T
  MatrixRef a, b, c;
};

struct Validation {
  ProblemError error = ProblemError::none;
  char operand = 0;
  explicit operator bool() const { return error == ProblemError::none; }
};

Validation validate_gemm(const GemmShape& s);

// First and one-past-last byte (relative to the allocation) a matrix touches.
bool matrix_byte_span(const MatrixRef& m, uint64_t* begin, uint64_t* end);

} // namespace xvram
