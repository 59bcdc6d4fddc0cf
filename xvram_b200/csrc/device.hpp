// device.hpp -- the runtime's only window onto the GPU.
//
// The residency runtime, transfer engine and executor talk to the device through this
// interface, never to CUDA directly.  CudaDevice (cuda_device.cpp) is the only
// implementation; device_factory() is the seam where another one (a host-memory fake, as
// in the reference's tests/unit/residency_executor_fake_tests.cpp) would be installed.
//
// Addresses are plain 64-bit integers (device virtual addresses for the real device).
#pragma once

#include "status.hpp"
#include "validate.hpp"

#include <cstdint>
#include <memory>
#include <string>

namespace xvram {

struct DeviceInfo {
  int ordinal = 0;
  int device_count = 0;
  std::string name;
  uint64_t total_bytes = 0;
  int sm_count = 0;
  uint64_t vmm_granularity = 0; // physical allocation granularity for cuMemCreate
  int driver_version = 0;
  int cc_major = 0, cc_minor = 0;
};

using StreamId = uint64_t;
using EventId = uint64_t;

enum class CopyDir { h2d, d2h, d2d };

// The operands of one GEMM after gemm_prepare: addresses, leading dimensions and
// operations as the device's kernel reads them (a2 / b2: second terms, e.g. the low parts
// of a split).  Device-defined; the runtime only passes it back to gemm_block.
struct PreparedGemm {
  uint32_t compute = 0;
  int op_a = 0, op_b = 0;
  uint64_t a = 0, b = 0, a2 = 0, b2 = 0;
  int64_t lda = 0, ldb = 0;
};

// Element types and arithmetic of one device GEMM (validate.hpp's DataType / ComputeKind).
struct GemmTypes {
  uint32_t ab = kFp32; // A and B
  uint32_t c = kFp32;
  int compute = kStrictFp32;
};

class Device {
public:
  virtual ~Device() = default;

  virtual Error open(int ordinal, DeviceInfo* info) = 0;
  virtual Error close() = 0;
  virtual Error mem_get_info(uint64_t* free_bytes, uint64_t* total_bytes) = 0;

  // Virtual memory management: stable address ranges and physical frames.
  virtual Error va_reserve(uint64_t bytes, uint64_t* va) = 0;
  virtual Error va_free(uint64_t va, uint64_t bytes) = 0;
  virtual Error handle_create(uint64_t bytes, uint64_t* handle) = 0;
  virtual Error handle_release(uint64_t handle) = 0;
  // Maps `handle` (exactly `bytes`) at `va` and grants this device read/write access.
  virtual Error map(uint64_t va, uint64_t bytes, uint64_t handle) = 0;
  virtual Error unmap(uint64_t va, uint64_t bytes) = 0;

  // Page-locked host memory.
  virtual Error host_alloc(uint64_t bytes, void** out) = 0;
  virtual Error host_free(void* p) = 0;

  virtual Error stream_create(StreamId* out) = 0;
  virtual Error stream_destroy(StreamId s) = 0;
  virtual Error stream_sync(StreamId s) = 0;
  virtual Error event_create(EventId* out) = 0;
  virtual Error event_destroy(EventId e) = 0;
  virtual Error event_record(EventId e, StreamId s) = 0;
  virtual Error stream_wait_event(StreamId s, EventId e) = 0;
  virtual Error event_sync(EventId e) = 0;
  virtual Error event_elapsed_ms(EventId start, EventId stop, float* ms) = 0;

  // Pitched 2D copy of `height` rows of `width` bytes.
  virtual Error copy_2d(uint64_t dst, uint64_t dpitch, uint64_t src, uint64_t spitch,
                        uint64_t width, uint64_t height, CopyDir dir, StreamId s) = 0;
  virtual Error memset_d32(uint64_t dst, uint32_t value, uint64_t count, StreamId s) = 0;

  // C = alpha * op(A) op(B) + beta * C on device addresses (column-major), for the
  // element types and arithmetic in `t`: strict FP32 (FFMA kernel), three-term TF32
  // (tcgen05 kernel), FP16 / BF16 inputs (widened, FFMA kernel), FP64.  The workspace
  // (gemm_workspace bytes) holds canonicalised or widened operands.
  virtual Error gemm(const GemmTypes& t, int op_a, int op_b, int64_t m, int64_t n, int64_t k,
                     double alpha, uint64_t a, int64_t lda, uint64_t b, int64_t ldb, double beta,
                     uint64_t c, int64_t ldc, uint64_t workspace, uint64_t workspace_bytes,
                     StreamId s) = 0;
  // Workspace that gemm needs for this problem (0 if none).
  virtual uint64_t gemm_workspace(const GemmTypes& t, int op_a, int op_b, int64_t m, int64_t n,
                                  int64_t k) = 0;
  // dst (rows x cols, column-major, ldd) = src converted between FP16 / BF16 and FP32
  // (round to nearest even when narrowing).
  virtual Error convert(uint32_t src_type, uint64_t src, int64_t lds, uint32_t dst_type,
                        uint64_t dst, int64_t ldd, int64_t rows, int64_t cols, StreamId s) = 0;
  // An FP32 GEMM (strict or three-term TF32) in two parts, for launching C's column blocks
  // separately: gemm_prepare brings op(A) and op(B) into the workspace in the form the
  // kernel reads; gemm_block computes C's columns [n0, n0 + nj) (c = the address of column
  // n0) from them.  For n0 on a multiple of 256, every output equals that of one gemm call
  // over all of C.  The workspace must stay untouched until the last block has run.
  virtual Error gemm_prepare(const GemmTypes& t, int op_a, int op_b, int64_t m, int64_t n,
                             int64_t k, uint64_t a, int64_t lda, uint64_t b, int64_t ldb,
                             uint64_t workspace, uint64_t workspace_bytes, StreamId s,
                             PreparedGemm* out) = 0;
  virtual Error gemm_block(const PreparedGemm& p, int64_t m, int64_t n0, int64_t nj, int64_t k,
                           double alpha, double beta, uint64_t c, int64_t ldc, StreamId s) = 0;
  // Reads and clears the sticky error word of the library's kernels (synchronising s).
  virtual Error kernel_status(StreamId s, uint32_t* word) = 0;
  // The native handle of stream s (a cudaStream_t) handed to transaction callbacks.
  virtual uint64_t native_stream(StreamId s) = 0;

  // --- used by the multi-GPU executor (sharded.cpp) --------------------------------------
  // Makes this device the calling thread's current one; *previous receives the one that
  // was current, for restore_current.
  virtual Error make_current(int* previous) = 0;
  virtual void restore_current(int previous) = 0;
  // Plain device allocations (256-byte aligned) for the executor's own buffers.
  virtual Error mem_alloc(uint64_t bytes, uint64_t* out) = 0;
  virtual Error mem_free(uint64_t p) = 0;
  // *done = whether everything before event e's record has completed (non-blocking).
  virtual Error event_query(EventId e, bool* done) = 0;
  // dst (cols x rows, column-major, ldd) = src^T (src: rows x cols, column-major, lds):
  // FP32 values moved, not rounded.
  virtual Error transpose_f32(uint64_t src, int64_t lds, uint64_t dst, int64_t ldd, int64_t rows,
                              int64_t cols, StreamId s) = 0;
};

using DeviceFactory = std::unique_ptr<Device> (*)();

std::unique_ptr<Device> make_cuda_device();

// The factory the adapter uses; tests may replace it before initialize().
DeviceFactory& device_factory();

} // namespace xvram

// Testing seam (the role of the reference's fake driver tables in
// tests/unit/residency_executor_fake_tests.cpp): sessions and the compat adapter created
// after this call get their device from `create`, which returns a new object implementing
// the Device interface above, built with the same compiler -- the host-memory fake in
// tests/fake_device/.  NULL restores the CUDA device.  The product libraries do not export
// it; only the test suite's own link of the same objects does.
extern "C" __attribute__((visibility("default"))) xvram_status
xvram_b200_test_set_device_factory(void* (*create)(void));
