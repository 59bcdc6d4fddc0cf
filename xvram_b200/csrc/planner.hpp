// planner.hpp -- out-of-core panel scheduler.
//
// Replaces the reference's geometry-fit planner (reference src/gemm/planner.cpp:1005-1153,
// tile loop m -> n -> k at :492-512, beta on the first K panel at :475-490) with a
// transfer-volume planner:
//
//   * C is processed in blocks of mb x nb that stay resident in HBM while every K panel
//     of op(A) (mb x kb) and op(B) (kb x nb) for that block streams through;
//   * panels are packed sub-rectangles copied with one pitched 2D copy each, so a
//     column-major panel costs exactly its own bytes (the reference moves whole 64 MiB
//     chunks of the allocation);
//   * panel slots are evicted by exact next use (Belady): the step sequence is known in
//     advance, so the slot holding the panel needed furthest in the future is reused;
//   * geometry and loop order are chosen by simulating that cache for every candidate
//     and minimising the predicted time max(FLOP / compute rate, H2D bytes / link rate,
//     D2H bytes / link rate) under the device budget.
//
// The plan is deterministic and contains every load decision, so the executor only
// replays it and the CPU tests can check it exhaustively.
#pragma once

#include <cstdint>
#include <functional>
#include <vector>

namespace xvram {

struct PlanProblem {
  int op_a = 0, op_b = 0; // 0 = N, 1 = T
  int64_t m = 0, n = 0, k = 0;
  bool beta_nonzero = false;
};

struct PlanLimits {
  uint64_t budget_bytes = 0;   // device bytes for C blocks + panel slots
  uint64_t quantum_bytes = 0;  // every slot is a whole number of physical frames
  double flops_per_s = 70e12;  // planning estimates only
  double h2d_bytes_per_s = 50e9;
  double d2h_bytes_per_s = 50e9;
  int64_t force_mb = 0, force_nb = 0, force_kb = 0; // 0 = search (tests pin geometry)
  // Per-step device workspace for canonicalising K-major panels: the kernel transposes
  // op(A) panels when transpose_a and op(B) panels when transpose_b.
  bool transpose_a = false, transpose_b = false;
  // Tensor-core steps instead: hi/lo split copies of both panels (2 x (mb + nb) x kb floats).
  bool tf32x3 = false;
  // When set, the per-step workspace for an mb x nb x kb step (replaces the three flags
  // above: the executor asks the device's kernel for it).
  std::function<uint64_t(int64_t mb, int64_t nb, int64_t kb)> step_workspace;
  // Element bytes: A / B panels and their host copies; the C block as the kernel
  // accumulates it in its slot; C on the host.  A C stored narrower than it accumulates
  // (FP16 / BF16 C of an FP32-arithmetic GEMM) also needs a staging copy of the block in
  // its slot for the conversions on the way in and out.
  uint32_t ab_bytes = 4, c_acc_bytes = 4, c_host_bytes = 4;
  int force_order = -1;                             // -1 search, 0 m-outer, 1 n-outer
};

// One panel load: copy panel (operand, block, kpanel) into slot `slot`.
struct PanelLoad {
  uint8_t operand = 0; // 0 = A (block = m block), 1 = B (block = n block)
  int32_t block = 0;
  int32_t kpanel = 0;
  int32_t slot = 0;
  bool evicts = false; // the slot held another panel before (a frame reuse)
};

struct PlanStep {
  int32_t bm = 0, bn = 0, bk = 0;
  int32_t slot_a = 0, slot_b = 0;
  int32_t c_slot = 0;
  bool first_k = false; // C block starts here (load C if beta != 0)
  bool last_k = false;  // C block completes here (write back)
  uint32_t load_begin = 0, load_count = 0; // range in Plan::loads issued before this step
};

struct Plan {
  int64_t mb = 0, nb = 0, kb = 0;
  bool n_outer = false;
  int64_t blocks_m = 0, blocks_n = 0, panels_k = 0;
  uint64_t slot_bytes = 0;   // panel slot size (multiple of quantum)
  uint64_t c_slot_bytes = 0; // C block slot size (multiple of quantum)
  uint64_t c_stage_offset = 0; // staging copy inside a C slot (0: none, C kept as stored)
  uint64_t workspace_bytes = 0; // per-step canonicalisation workspace (multiple of quantum)
  int32_t panel_slots = 0;
  int32_t c_slots = 0;
  std::vector<PlanStep> steps;
  std::vector<PanelLoad> loads;
  // Predictions from the simulation.
  uint64_t h2d_bytes = 0, d2h_bytes = 0;
  uint64_t panel_loads = 0, panel_hits = 0, panel_evictions = 0;
  double flops = 0, est_seconds = 0;
  int candidates_considered = 0;
};

enum class PlanStatus { ok = 0, invalid = 1, budget_too_small = 2 };

PlanStatus make_panel_plan(const PlanProblem& p, const PlanLimits& lim, Plan* out);

// Bytes of one panel / C block for a geometry (useful to tests and the executor).
inline uint64_t round_up(uint64_t v, uint64_t q) { return q ? (v + q - 1) / q * q : v; }

} // namespace xvram
