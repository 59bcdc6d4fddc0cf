// runtime.hpp -- residency runtime and GEMM executor.
//
// Replaces the reference's residency::Runtime (reference src/residency/runtime.hpp:317-372,
// runtime.cpp) and gemm::execute_tiled_gemm (reference src/gemm/executor.cpp:331-454).
//
// Memory model
//   * Every allocation owns a stable device virtual-address reservation (returned to
//     the caller as its "device pointer") cut into chunks of session.chunk_size_bytes,
//     and an optional page-locked host backing store created on first need.
//   * Device memory is a pool of physical frames (one cuMemCreate handle per chunk-sized
//     frame) capped by the device budget.  A resident chunk has a frame mapped at its
//     stable address; frames are created once and then reused (handle reuse), never
//     released before close.
//   * A chunk is dirty when the device holds newer data than the host backing; dirty
//     chunks are written back before their frame is reused (dirty eviction).
//
// GEMM execution
//   * In place: when the chunks under A, B and C fit in the frame pool at once they are
//     made resident and the sm_100a kernel runs directly on the stable addresses;
//     C stays resident and dirty (later reads come straight from HBM).
//   * Streamed (out of core): otherwise the runtime writes back and unmaps every
//     resident chunk, maps the pool's frames into a slot arena, and replays the panel
//     plan (planner.hpp): pitched H2D panel copies on a copy stream, one kernel per
//     (C block, K panel) step on the compute stream (beta applied on the block's first
//     K panel, 1 afterwards), C blocks written back on a third stream.  Slot reuse is
//     ordered by per-slot completion events, so copies run ahead of compute without
//     host waits.
#pragma once

#include "device.hpp"
#include "planner.hpp"
#include "validate.hpp"

#include <cstdint>
#include <functional>
#include <memory>
#include <vector>

namespace xvram {

struct RuntimeConfig {
  int device_ordinal = 0;
  uint64_t chunk_bytes = 64ull << 20;
  uint64_t cache_target_bytes = 0; // 0 = free device memory at open minus headroom
  uint64_t headroom_bytes = 512ull << 20;
  // Live budget: at operation boundaries, at most this often, the runtime samples the
  // device's free memory and shrinks (or, after repeated samples with room, regrows up to
  // the budget it opened with) its frame pool to free + own frames - headroom.
  uint64_t budget_poll_ms = 100;
  // Victim choice for resident chunks: 0 = CLOCK (the reference's default), 1 = LRU.
  // Streamed GEMMs evict panels by exact next use either way (the plan knows it).
  uint32_t cache_policy = 0;
  // Cap on the host ledger (the pinned host backing of allocations); 0 = none.  An
  // allocation whose backing would pass it fails with HOST_OUT_OF_MEMORY.
  uint64_t host_store_cap_bytes = 0;
  // Planning rates (estimates only; they steer geometry choice, never correctness).
  double flops_per_s = 70e12;
  double h2d_bytes_per_s = 50e9;
  double d2h_bytes_per_s = 50e9;
};

struct GemmCall {
  // Element types in shape.a/b/c.dtype, arithmetic in shape.compute: kTf32 is the
  // three-term TF32 tensor-core kernel (FP32-accurate within 1e-6 of the normalised error
  // bound).  alpha and beta are applied in FP32 for FP32 arithmetic, in FP64 for FP64.
  GemmShape shape;
  double alpha = 1.0, beta = 0.0;
  // Rates for planning this call (0 = the runtime's configured rates).
  double flops_per_s = 0;
  // Return once the kernels are queued, as cublasSgemm does, instead of after they finish.
  // An in-place FP32 GEMM (strict or TF32) is then launched as column blocks of C on two
  // streams,
  // and a later read of C copies each block home as soon as its own kernel is done, while
  // the next blocks compute.  The kernels' error word is read at the next read, synchronize
  // or close, which report a failed kernel.
  bool defer_completion = false;
};

// A byte range of an allocation that an operation touches (reference
// src/residency/core.cpp:128-277 access ranges).  mode: 0 read, 1 read-write, 2 write-only.
struct AccessRange {
  uint64_t allocation_id = 0;
  uint64_t offset_bytes = 0;
  uint64_t length_bytes = 0;
  int mode = 0;
};

// The same range once resident: device_address is where offset_bytes lives in HBM.
struct ResolvedRange {
  uint64_t allocation_id = 0;
  uint64_t offset_bytes = 0;
  uint64_t length_bytes = 0;
  uint64_t device_address = 0;
  int mode = 0;
};

// Device-side work of a transaction: enqueue only, on native_stream.
using TransactionBody = std::function<Error(const std::vector<ResolvedRange>& ranges,
                                            uint64_t workspace_address, uint64_t workspace_bytes,
                                            uint64_t native_stream)>;

// How gemm() would run a problem (for plan descriptions; nothing is executed).
struct GemmLayout {
  bool in_place = false;
  uint64_t tile_m = 0, tile_n = 0, tile_k = 0;
  uint64_t tiles = 0;
  uint64_t working_set_bytes = 0;
  uint64_t workspace_bytes = 0;
};

// Counters that are not part of xvram_session_telemetry_v1.
struct RuntimeExtra {
  uint64_t tiles_submitted = 0;
  uint64_t tiles_retired = 0;
  uint64_t gemm_in_place = 0;
  uint64_t gemm_streamed = 0;
  uint64_t host_backing_bytes = 0;
  uint64_t host_backing_peak_bytes = 0;
  // Tombstoned ranges of released allocations still reserved (current state; zero after
  // close), and those released at close (cumulative).
  uint64_t retired_va_reservations = 0;
  uint64_t retired_va_bytes = 0;
  uint64_t retired_va_reservations_freed = 0;
  uint64_t retired_va_bytes_freed = 0;
  // Last streamed plan.
  int64_t last_mb = 0, last_nb = 0, last_kb = 0;
  int64_t last_steps = 0;
  int32_t last_panel_slots = 0;
  double last_gemm_ms = 0;
  // In-place GEMMs that returned before their kernels finished, and the C column blocks
  // they were launched as.
  uint64_t gemm_deferred = 0;
  uint64_t gemm_column_blocks = 0;
  // Streamed GEMMs: panel loads into a slot that held another panel.  The slot's frames
  // stay mapped, so these are not evictions or handle reuses in the reference's sense
  // (those count VMM unmaps and remaps) and are counted here instead.
  uint64_t panel_slot_refills = 0;
};

class Runtime {
public:
  Runtime();
  ~Runtime();
  Runtime(const Runtime&) = delete;
  Runtime& operator=(const Runtime&) = delete;

  Error open(const RuntimeConfig& cfg, std::unique_ptr<Device> device);
  Error close();

  // zero_fill: bytes never written read as zero, on the host and on the device.
  Error allocate(uint64_t bytes, uint64_t* id, uint64_t* va, bool zero_fill = false);
  Error release(uint64_t id);
  Error write(uint64_t id, uint64_t offset, const void* src, uint64_t bytes);
  Error read(uint64_t id, uint64_t offset, void* dst, uint64_t bytes);
  Error gemm(const GemmCall& call);
  Error describe_gemm(const GemmCall& call, GemmLayout* out);
  // Starts making the ranges resident (uploads run on the H2D stream); returns without
  // waiting.  Later operations on these chunks wait for exactly their uploads.
  Error prefetch(const std::vector<AccessRange>& ranges);
  // Makes the ranges resident, gives `body` their device addresses, a workspace of
  // workspace_bytes and the compute stream, marks written ranges dirty and waits for the
  // stream.  BUDGET_PRESSURE when the ranges and workspace exceed the device budget.
  Error transaction(const std::vector<AccessRange>& ranges, uint64_t workspace_bytes,
                    const TransactionBody& body);
  bool live(uint64_t id) const;
  uint64_t allocation_bytes(uint64_t id) const;
  // Samples the device now (ignoring the poll interval) and applies the live budget.
  Error refresh_budget();
  Error synchronize();
  Error mem_get_info(uint64_t* free_bytes, uint64_t* total_bytes);

  const DeviceInfo& info() const;
  const xvram_session_telemetry_v1& counters() const;
  const RuntimeExtra& extra() const;
  uint64_t chunk_bytes() const;
  uint64_t frame_capacity() const;

  struct Impl;

private:
  std::unique_ptr<Impl> impl_;
};

} // namespace xvram
