// validate.cpp -- see validate.hpp.
#include "validate.hpp"

#include <climits>

namespace xvram {
namespace {

bool mul_ok(uint64_t a, uint64_t b, uint64_t* out) {
  if (a != 0 && b > UINT64_MAX / a)
    return false;
  *out = a * b;
  return true;
}
bool add_ok(uint64_t a, uint64_t b, uint64_t* out) {
  if (b > UINT64_MAX - a)
    return false;
  *out = a + b;
  return true;
}

// Per-matrix checks (reference planner.cpp validate_matrix): allocation identity,
// non-empty, leading dimension >= rows and <= INT_MAX, storage arithmetic that does not
// overflow, and storage that lies inside the allocation.
Validation check_matrix(const MatrixRef& m, char operand) {
  auto fail = [operand](ProblemError e) { return Validation{e, operand}; };
  if (m.allocation_id == 0 || m.allocation_bytes == 0)
    return fail(ProblemError::invalid_allocation);
  const uint64_t esize = element_bytes(m.dtype);
  if (esize == 0)
    return fail(ProblemError::invalid_element_type);
  if (m.rows == 0 || m.columns == 0)
    return fail(ProblemError::zero_dimension);
  if (m.ld < m.rows)
    return fail(ProblemError::leading_dimension_too_small);
  if (m.ld > static_cast<uint64_t>(INT_MAX))
    return fail(ProblemError::integer_limit_exceeded);
  uint64_t last_col = 0, last = 0, bytes = 0, end = 0;
  if (!mul_ok(m.columns - 1, m.ld, &last_col) || !add_ok(last_col, m.rows - 1, &last) ||
      !add_ok(last, 1, &last))
    return fail(ProblemError::storage_overflow);
  if (!mul_ok(last, esize, &bytes) || !add_ok(m.offset_bytes, bytes, &end))
    return fail(ProblemError::storage_overflow);
  if (m.offset_bytes >= m.allocation_bytes || end > m.allocation_bytes)
    return fail(ProblemError::storage_out_of_bounds);
  return {};
}

} // namespace

bool supported_types(uint32_t ab, uint32_t c, int compute) {
  switch (ab) {
  case kFp16:
  case kBf16:
    return (c == ab || c == kFp32) && compute == kStrictFp32;
  case kFp32:
    return c == kFp32 && (compute == kStrictFp32 || compute == kTf32);
  case kFp64:
    return c == kFp64 && compute == kComputeFp64;
  default:
    return false;
  }
}

bool matrix_byte_span(const MatrixRef& m, uint64_t* begin, uint64_t* end) {
  const uint64_t esize = element_bytes(m.dtype);
  if (m.rows == 0 || m.columns == 0 || esize == 0)
    return false;
  uint64_t last_col = 0, last = 0, bytes = 0, e = 0;
  if (!mul_ok(m.columns - 1, m.ld, &last_col) || !add_ok(last_col, m.rows, &last) ||
      !mul_ok(last, esize, &bytes) || !add_ok(m.offset_bytes, bytes, &e))
    return false;
  *begin = m.offset_bytes;
  *end = e;
  return true;
}

const char* problem_error_name(ProblemError e) {
  switch (e) {
  case ProblemError::none: return "none";
  case ProblemError::zero_dimension: return "zero_dimension";
  case ProblemError::invalid_allocation: return "invalid_allocation";
  case ProblemError::invalid_layout: return "invalid_layout";
  case ProblemError::invalid_operation: return "invalid_operation";
  case ProblemError::invalid_element_type: return "invalid_element_type";
  case ProblemError::invalid_compute_mode: return "invalid_compute_mode";
  case ProblemError::dimension_mismatch: return "dimension_mismatch";
  case ProblemError::leading_dimension_too_small: return "leading_dimension_too_small";
  case ProblemError::storage_overflow: return "storage_overflow";
  case ProblemError::storage_out_of_bounds: return "storage_out_of_bounds";
  case ProblemError::unsupported_type_combination: return "unsupported_type_combination";
  case ProblemError::output_aliases_input: return "output_aliases_input";
  case ProblemError::integer_limit_exceeded: return "integer_limit_exceeded";
  }
  return "invalid";
}

// Problem-level order (reference planner.cpp:785-859): empty problem, operations,
// compute mode, each matrix A, B, C, allocation identity consistency, operated shapes,
// element types, then overlap of C with an input in the same allocation.
Validation validate_gemm(const GemmShape& s) {
  if (s.m == 0 || s.n == 0 || s.k == 0)
    return {ProblemError::zero_dimension, 0};
  if (s.op_a != 0 && s.op_a != 1)
    return {ProblemError::invalid_operation, 'A'};
  if (s.op_b != 0 && s.op_b != 1)
    return {ProblemError::invalid_operation, 'B'};
  if (s.compute != kStrictFp32 && s.compute != kTf32 && s.compute != kComputeFp64)
    return {ProblemError::invalid_compute_mode, 0};
  const MatrixRef* mats[3] = {&s.a, &s.b, &s.c};
  const char names[3] = {'A', 'B', 'C'};
  for (int i = 0; i < 3; ++i)
    if (Validation v = check_matrix(*mats[i], names[i]); !v)
      return v;
  const auto same_id_other_size = [](const MatrixRef& x, const MatrixRef& y) {
    return x.allocation_id == y.allocation_id && x.allocation_bytes != y.allocation_bytes;
  };
  if (same_id_other_size(s.a, s.b) || same_id_other_size(s.a, s.c) ||
      same_id_other_size(s.b, s.c))
    return {ProblemError::invalid_allocation, 0};
  const uint64_t a_rows = s.op_a == 0 ? s.a.rows : s.a.columns;
  const uint64_t a_cols = s.op_a == 0 ? s.a.columns : s.a.rows;
  const uint64_t b_rows = s.op_b == 0 ? s.b.rows : s.b.columns;
  const uint64_t b_cols = s.op_b == 0 ? s.b.columns : s.b.rows;
  if (a_rows != s.m || a_cols != s.k || b_rows != s.k || b_cols != s.n || s.c.rows != s.m ||
      s.c.columns != s.n)
    return {ProblemError::dimension_mismatch, 0};
  if (s.a.dtype != s.b.dtype || !supported_types(s.a.dtype, s.c.dtype, s.compute))
    return {ProblemError::unsupported_type_combination, 0};
  uint64_t ab = 0, ae = 0, bb = 0, be = 0, cb = 0, ce = 0;
  if (!matrix_byte_span(s.a, &ab, &ae) || !matrix_byte_span(s.b, &bb, &be) ||
      !matrix_byte_span(s.c, &cb, &ce))
    return {ProblemError::storage_overflow, 0};
  const auto overlaps = [](uint64_t b0, uint64_t e0, uint64_t b1, uint64_t e1) {
    return b0 < e1 && b1 < e0;
  };
  if ((s.a.allocation_id == s.c.allocation_id && overlaps(ab, ae, cb, ce)) ||
      (s.b.allocation_id == s.c.allocation_id && overlaps(bb, be, cb, ce)))
    return {ProblemError::output_aliases_input, 'C'};
  return {};
}

} // namespace xvram
