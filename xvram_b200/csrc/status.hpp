// status.hpp -- error record carried through the runtime and published by get_error.
//
// Mirrors the reference's sdk::Error (src/sdk/status.hpp:11): a status code plus the
// stage/operation/native detail that xvram_error_info_v1 exposes
// (reference include/xvram/xvram.h:87-97).
#pragma once

#include "xvram/xvram.h"

#include <cstdint>
#include <cstring>
#include <string>

namespace xvram {

struct Error {
  xvram_status status = XVRAM_STATUS_SUCCESS;
  xvram_native_error_domain domain = XVRAM_NATIVE_ERROR_NONE;
  int64_t native_code = 0;
  std::string stage;
  std::string operation;
  std::string native_name;
  std::string message;

  explicit operator bool() const noexcept { return status != XVRAM_STATUS_SUCCESS; }
};

inline Error make_error(xvram_status status, const char* stage, const char* operation,
                        const std::string& message) {
  Error e;
  e.status = status;
  e.domain = XVRAM_NATIVE_ERROR_INTERNAL;
  if (status == XVRAM_STATUS_SUCCESS)
    e.domain = XVRAM_NATIVE_ERROR_NONE;
  e.stage = stage;
  e.operation = operation;
  e.message = message;
  return e;
}

inline Error cuda_error(const char* stage, const char* operation, int code, const char* name,
                        const std::string& message) {
  Error e;
  e.status = XVRAM_STATUS_CUDA_ERROR;
  e.domain = XVRAM_NATIVE_ERROR_CUDA;
  e.native_code = code;
  e.stage = stage;
  e.operation = operation;
  e.native_name = name ? name : "";
  e.message = message;
  return e;
}

inline void copy_field(char* dst, size_t cap, const std::string& src) {
  const size_t n = src.size() < cap - 1 ? src.size() : cap - 1;
  std::memcpy(dst, src.data(), n);
  dst[n] = '\0';
}

// Writes `e` into a caller-provided record, preserving the caller's struct_size.
inline void write_error_info(const Error& e, xvram_error_info_v1& out) {
  const uint32_t size = out.struct_size;
  std::memset(&out, 0, sizeof(out));
  out.struct_size = size;
  out.status = e.status;
  out.native_domain = e.domain;
  out.native_code = e.native_code;
  copy_field(out.stage, sizeof(out.stage), e.stage);
  copy_field(out.operation, sizeof(out.operation), e.operation);
  copy_field(out.native_name, sizeof(out.native_name), e.native_name);
  copy_field(out.message, sizeof(out.message), e.message);
}

} // namespace xvram
