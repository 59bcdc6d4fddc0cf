// planner.cpp -- see planner.hpp.
#include "planner.hpp"
#include "tiling.hpp"

#include <algorithm>
#include <climits>
#include <cmath>
#include <set>
#include <utility>

namespace xvram {
namespace {

constexpr int64_t kTileM = 128;   // CTA tile rows of the contraction kernel
constexpr int64_t kTileN = 128;   // block width granularity (the kernel's tiles are 256 wide
                                  // when the block is wider than 128)
constexpr int64_t kTileK = 32;
constexpr int kSmCount = 148;
constexpr double kStepOverheadS = 15e-6; // launch + event bookkeeping per step
// Fixed time of one CTA tile besides its FFMAs: the TMA ring filling up and the C
// epilogue (read, alpha/beta, write).  Every wave of every step pays it, so deep K panels
// (fewer steps) amortise it; measured at ~1 ms per 16384 x 16384 step (55 waves).
constexpr double kTileFixedS = 12e-6;
constexpr int64_t kMaxSteps = 1 << 15;     // steps a plan may have
// Plans predicted within this fraction of the fastest are treated as equally fast, and the
// one that moves the fewest host bytes wins: the time model is approximate to about this
// much, while host traffic decides how far the link stays from saturation -- and links are
// shared when several GPUs of a node stream at once.
constexpr double kTrafficSlack = 0.02;
constexpr int kMaxSimulations = 96;          // candidates simulated per plan
constexpr int32_t kNever = INT32_MAX;

int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

std::vector<int64_t> block_candidates(int64_t dim, int64_t align, int64_t lo, int64_t hi) {
  std::vector<int64_t> v;
  const int64_t whole = round_up(static_cast<uint64_t>(dim), static_cast<uint64_t>(align));
  if (whole <= hi)
    v.push_back(whole);
  for (int64_t x = lo; x <= hi; x *= 2)
    if (x < whole)
      v.push_back(x);
  if (v.empty())
    v.push_back(std::min<int64_t>(hi, whole));
  std::sort(v.begin(), v.end());
  v.erase(std::unique(v.begin(), v.end()), v.end());
  return v;
}

struct Geo {
  int64_t mb, nb, kb;
  bool n_outer;
};

// CTA tiles of one kernel launch on an mr x nr block, in the tiling the kernel picks for it
// (tiling.hpp: 192 x 192, or 128 x 256 / 128 x 128 at 0.95 of that FMA rate), and the
// waves they take: one CTA per SM, and a last wave of at most half the SMs runs as
// half-width tiles in about half a tile's time.
int64_t launch_ctas(int64_t mr, int64_t nr) {
  const Tiling t = choose_tiling(mr, nr, kSmCount);
  return ceil_div(mr, t.tile_m) * ceil_div(nr, t.tile_n);
}
double launch_waves(int64_t mr, int64_t nr) { return tile_waves(launch_ctas(mr, nr), kSmCount); }
// Useful work per SM-wave slot of the launch, times the tiling's relative FMA rate.
double wave_efficiency(int64_t mr, int64_t nr) {
  const Tiling t = choose_tiling(mr, nr, kSmCount);
  return static_cast<double>(mr) * static_cast<double>(nr) /
         (launch_waves(mr, nr) * kSmCount * t.tile_m * t.tile_n) * t.rate;
}

// Per-step time that does not scale with kr: launch bookkeeping plus one tile fixed cost
// per wave of the step's C block.
double step_fixed_s(int64_t mr, int64_t nr) {
  return kStepOverheadS + launch_waves(mr, nr) * kTileFixedS;
}

// Builds the step sequence and replays the slot cache.  With `record` false only the
// predictions are filled in (the search path); with `record` true the steps and the
// loads are stored as well.
bool simulate(const PlanProblem& p, const PlanLimits& lim, const Geo& g, bool record, Plan* out) {
  Plan& pl = *out;
  pl = Plan{};
  pl.mb = g.mb;
  pl.nb = g.nb;
  pl.kb = g.kb;
  pl.n_outer = g.n_outer;
  pl.blocks_m = ceil_div(p.m, g.mb);
  pl.blocks_n = ceil_div(p.n, g.nb);
  pl.panels_k = ceil_div(p.k, g.kb);
  const int64_t nsteps = pl.blocks_m * pl.blocks_n * pl.panels_k;
  if (nsteps > kMaxSteps)
    return false;
  const uint64_t q = lim.quantum_bytes ? lim.quantum_bytes : 1;
  const uint64_t cblock = static_cast<uint64_t>(g.mb) * static_cast<uint64_t>(g.nb);
  pl.slot_bytes = round_up(static_cast<uint64_t>(std::max(g.mb, g.nb)) * g.kb * lim.ab_bytes, q);
  if (lim.c_host_bytes < lim.c_acc_bytes) { // accumulator, then the stored-type staging copy
    pl.c_stage_offset = round_up(cblock * lim.c_acc_bytes, 256);
    pl.c_slot_bytes = round_up(pl.c_stage_offset + cblock * lim.c_host_bytes, q);
  } else {
    pl.c_slot_bytes = round_up(cblock * lim.c_acc_bytes, q);
  }
  const int64_t blocks = pl.blocks_m * pl.blocks_n;
  pl.c_slots = blocks > 1 ? 2 : 1;
  {
    const auto up = [](uint64_t v, uint64_t m) { return (v + m - 1) / m * m; };
    uint64_t ws = 0;
    if (lim.step_workspace)
      ws = lim.step_workspace(g.mb, g.nb, g.kb);
    else if (lim.transpose_a)
      ws += up(up(static_cast<uint64_t>(g.mb), 4) * static_cast<uint64_t>(g.kb) * 4u, 256);
    if (!lim.step_workspace && lim.transpose_b)
      ws += up(up(static_cast<uint64_t>(g.nb), 4) * static_cast<uint64_t>(g.kb) * 4u, 256);
    if (!lim.step_workspace && lim.tf32x3)
      ws = 2 * up(static_cast<uint64_t>(g.mb) * up(static_cast<uint64_t>(g.kb), 4) * 4u, 256) +
           2 * up(static_cast<uint64_t>(g.nb) * up(static_cast<uint64_t>(g.kb), 4) * 4u, 256);
    pl.workspace_bytes = round_up(ws, q);
  }
  const uint64_t c_total =
      pl.c_slot_bytes * static_cast<uint64_t>(pl.c_slots) + pl.workspace_bytes;
  if (c_total >= lim.budget_bytes)
    return false;
  const int64_t distinct = (pl.blocks_m + pl.blocks_n) * pl.panels_k;
  const int64_t fit = static_cast<int64_t>((lim.budget_bytes - c_total) / pl.slot_bytes);
  const int64_t need = std::min<int64_t>(4, distinct);
  if (fit < need)
    return false;
  pl.panel_slots = static_cast<int32_t>(std::min<int64_t>({fit, distinct, INT32_MAX / 2}));

  // Step order: outer block index, serpentine middle index, K direction alternating
  // per C block so the panels loaded last are the first ones the next block needs.
  std::vector<PlanStep> steps;
  steps.reserve(static_cast<size_t>(nsteps));
  const int64_t outer = g.n_outer ? pl.blocks_n : pl.blocks_m;
  const int64_t inner = g.n_outer ? pl.blocks_m : pl.blocks_n;
  int64_t block_index = 0;
  for (int64_t o = 0; o < outer; ++o) {
    for (int64_t ii = 0; ii < inner; ++ii) {
      const int64_t i = (o % 2 == 0) ? ii : inner - 1 - ii;
      const int64_t bm = g.n_outer ? i : o;
      const int64_t bn = g.n_outer ? o : i;
      const bool forward = (block_index % 2) == 0;
      for (int64_t kk = 0; kk < pl.panels_k; ++kk) {
        PlanStep s;
        s.bm = static_cast<int32_t>(bm);
        s.bn = static_cast<int32_t>(bn);
        s.bk = static_cast<int32_t>(forward ? kk : pl.panels_k - 1 - kk);
        s.c_slot = static_cast<int32_t>(block_index % pl.c_slots);
        s.first_k = kk == 0;
        s.last_k = kk == pl.panels_k - 1;
        steps.push_back(s);
      }
      ++block_index;
    }
  }

  // Panel ids: A panels first, then B panels.
  const int64_t a_ids = pl.blocks_m * pl.panels_k;
  auto id_a = [&](const PlanStep& s) { return static_cast<int64_t>(s.bm) * pl.panels_k + s.bk; };
  auto id_b = [&](const PlanStep& s) {
    return a_ids + static_cast<int64_t>(s.bn) * pl.panels_k + s.bk;
  };
  // next_a[s] / next_b[s]: the next step after s that uses the same panel.
  std::vector<int32_t> next_a(static_cast<size_t>(nsteps)), next_b(static_cast<size_t>(nsteps));
  {
    std::vector<int32_t> last(static_cast<size_t>(distinct), kNever);
    for (int64_t s = nsteps - 1; s >= 0; --s) {
      const auto& st = steps[static_cast<size_t>(s)];
      next_a[static_cast<size_t>(s)] = last[static_cast<size_t>(id_a(st))];
      last[static_cast<size_t>(id_a(st))] = static_cast<int32_t>(s);
      next_b[static_cast<size_t>(s)] = last[static_cast<size_t>(id_b(st))];
      last[static_cast<size_t>(id_b(st))] = static_cast<int32_t>(s);
    }
  }

  std::vector<int64_t> slot_panel(static_cast<size_t>(pl.panel_slots), -1);
  std::vector<int32_t> slot_next(static_cast<size_t>(pl.panel_slots), kNever);
  std::vector<int32_t> panel_slot(static_cast<size_t>(distinct), -1);
  std::set<std::pair<int32_t, int32_t>> by_next; // (next use, slot) of occupied slots
  int32_t free_cursor = 0;

  const auto panel_bytes = [&](int operand, int64_t block, int64_t kp) -> uint64_t {
    const int64_t kr = std::min<int64_t>(g.kb, p.k - kp * g.kb);
    const int64_t rr = operand == 0 ? std::min<int64_t>(g.mb, p.m - block * g.mb)
                                    : std::min<int64_t>(g.nb, p.n - block * g.nb);
    return static_cast<uint64_t>(kr) * static_cast<uint64_t>(rr) * lim.ab_bytes;
  };

  double compute_s = 0;
  std::vector<PanelLoad> loads;
  if (record)
    loads.reserve(static_cast<size_t>(std::min<int64_t>(2 * nsteps, 1 << 22)));
  int32_t protect[4] = {-1, -1, -1, -1};
  for (int64_t s = 0; s < nsteps; ++s) {
    PlanStep& st = steps[static_cast<size_t>(s)];
    st.load_begin = static_cast<uint32_t>(loads.size());
    // Slots used by this step and the previous one are never victims, so a load
    // never has to wait for the kernel that was issued just before it.
    protect[0] = protect[2];
    protect[1] = protect[3];
    protect[2] = protect[3] = -1;
    for (int operand = 0; operand < 2; ++operand) {
      const int64_t id = operand == 0 ? id_a(st) : id_b(st);
      const int32_t nxt = operand == 0 ? next_a[static_cast<size_t>(s)] : next_b[static_cast<size_t>(s)];
      int32_t slot = panel_slot[static_cast<size_t>(id)];
      if (slot >= 0) {
        ++pl.panel_hits;
        by_next.erase({slot_next[static_cast<size_t>(slot)], slot});
      } else {
        bool evicts = false;
        if (free_cursor < pl.panel_slots) {
          slot = free_cursor++;
        } else {
          slot = -1;
          for (auto it = by_next.rbegin(); it != by_next.rend(); ++it) {
            const int32_t cand = it->second;
            if (cand == protect[0] || cand == protect[1] || cand == protect[2])
              continue;
            slot = cand;
            break;
          }
          if (slot < 0) // every occupied slot is protected: take the farthest anyway
            slot = by_next.rbegin()->second;
          by_next.erase({slot_next[static_cast<size_t>(slot)], slot});
          panel_slot[static_cast<size_t>(slot_panel[static_cast<size_t>(slot)])] = -1;
          evicts = true;
          ++pl.panel_evictions;
        }
        slot_panel[static_cast<size_t>(slot)] = id;
        panel_slot[static_cast<size_t>(id)] = slot;
        ++pl.panel_loads;
        const int64_t block = operand == 0 ? st.bm : st.bn;
        pl.h2d_bytes += panel_bytes(operand, block, st.bk);
        if (record) {
          PanelLoad ld;
          ld.operand = static_cast<uint8_t>(operand);
          ld.block = static_cast<int32_t>(block);
          ld.kpanel = st.bk;
          ld.slot = slot;
          ld.evicts = evicts;
          loads.push_back(ld);
        }
      }
      slot_next[static_cast<size_t>(slot)] = nxt;
      by_next.insert({nxt, slot});
      (operand == 0 ? st.slot_a : st.slot_b) = slot;
      protect[2 + operand] = slot;
    }
    st.load_count = static_cast<uint32_t>(loads.size()) - st.load_begin;
    const int64_t mr = std::min<int64_t>(g.mb, p.m - static_cast<int64_t>(st.bm) * g.mb);
    const int64_t nr = std::min<int64_t>(g.nb, p.n - static_cast<int64_t>(st.bn) * g.nb);
    const int64_t kr = std::min<int64_t>(g.kb, p.k - static_cast<int64_t>(st.bk) * g.kb);
    if (st.first_k && p.beta_nonzero)
      pl.h2d_bytes += static_cast<uint64_t>(mr) * static_cast<uint64_t>(nr) * lim.c_host_bytes;
    if (st.last_k)
      pl.d2h_bytes += static_cast<uint64_t>(mr) * static_cast<uint64_t>(nr) * lim.c_host_bytes;
    compute_s += 2.0 * mr * nr * kr / lim.flops_per_s / wave_efficiency(mr, nr) +
                 step_fixed_s(mr, nr);
  }

  pl.flops = 2.0 * static_cast<double>(p.m) * static_cast<double>(p.n) * static_cast<double>(p.k);
  // Pipeline estimate: the slowest of the three engines, plus filling the pipe with the
  // first step's operands and draining the last C block.
  const auto& s0 = steps.front();
  double head = (panel_bytes(0, s0.bm, s0.bk) + panel_bytes(1, s0.bn, s0.bk)) / lim.h2d_bytes_per_s;
  const double cblock_bytes = static_cast<double>(std::min<int64_t>(g.mb, p.m)) *
                              static_cast<double>(std::min<int64_t>(g.nb, p.n)) *
                              lim.c_host_bytes;
  if (p.beta_nonzero)
    head += cblock_bytes / lim.h2d_bytes_per_s;
  const double tail = cblock_bytes / lim.d2h_bytes_per_s;
  pl.est_seconds = std::max({compute_s, pl.h2d_bytes / lim.h2d_bytes_per_s,
                             pl.d2h_bytes / lim.d2h_bytes_per_s}) +
                   head + tail;
  if (record) {
    pl.steps = std::move(steps);
    pl.loads = std::move(loads);
  }
  return true;
}

} // namespace

PlanStatus make_panel_plan(const PlanProblem& p, const PlanLimits& lim, Plan* out) {
  if (p.m <= 0 || p.n <= 0 || p.k <= 0 || (p.op_a != 0 && p.op_a != 1) ||
      (p.op_b != 0 && p.op_b != 1) || lim.budget_bytes == 0 || lim.flops_per_s <= 0 ||
      lim.h2d_bytes_per_s <= 0 || lim.d2h_bytes_per_s <= 0 || lim.ab_bytes == 0 ||
      lim.c_acc_bytes == 0 || lim.c_host_bytes == 0)
    return PlanStatus::invalid;

  std::vector<int64_t> mbs = lim.force_mb ? std::vector<int64_t>{lim.force_mb}
                                          : block_candidates(p.m, kTileM, 512, 65536);
  std::vector<int64_t> nbs = lim.force_nb ? std::vector<int64_t>{lim.force_nb}
                                          : block_candidates(p.n, kTileN, 512, 65536);
  std::vector<int64_t> kbs = lim.force_kb ? std::vector<int64_t>{lim.force_kb}
                                          : block_candidates(p.k, kTileK, 256, 32768);
  for (int64_t v : mbs)
    if (v <= 0 || v % kTileM)
      return PlanStatus::invalid;
  for (int64_t v : nbs)
    if (v <= 0 || v % kTileN)
      return PlanStatus::invalid;
  for (int64_t v : kbs)
    if (v <= 0 || v % kTileK)
      return PlanStatus::invalid;

  // Rank candidates by a closed-form lower bound on their time -- compute at the block's
  // wave efficiency plus per-step overhead, or the unavoidable link traffic (every operand
  // byte once) -- and simulate only while the bound can still beat the best plan.
  struct Cand {
    Geo g;
    double lb;
  };
  std::vector<Cand> cands;
  const double flops = 2.0 * static_cast<double>(p.m) * static_cast<double>(p.n) *
                       static_cast<double>(p.k);
  const double min_h2d =
      static_cast<double>(lim.ab_bytes) *
          (static_cast<double>(p.m) * p.k + static_cast<double>(p.k) * p.n) +
      (p.beta_nonzero ? static_cast<double>(lim.c_host_bytes) * p.m * p.n : 0.0);
  const double min_d2h = static_cast<double>(lim.c_host_bytes) * p.m * p.n;
  const bool forced = lim.force_mb || lim.force_nb || lim.force_kb;
  bool found = false;
  Geo best{};
  Plan trial, best_plan;
  int considered = 0;
  // Blocks smaller than one wave of CTAs waste SMs on every launch: they are considered
  // only when nothing else fits the budget (second pass).
  for (int pass = 0; pass < 2; ++pass) {
    cands.clear();
    for (int64_t mb : mbs)
      for (int64_t nb : nbs)
        for (int64_t kb : kbs)
          for (int order = 0; order < 2; ++order) {
            if (lim.force_order >= 0 && order != lim.force_order)
              continue;
            const int64_t steps = ceil_div(p.m, mb) * ceil_div(p.n, nb) * ceil_div(p.k, kb);
            if (steps > kMaxSteps)
              continue;
            const bool small = launch_ctas(std::min(mb, p.m), std::min(nb, p.n)) < kSmCount &&
                               (mb < p.m || nb < p.n);
            if (!forced && small != (pass == 1))
              continue;
            const double lb = std::max({flops / lim.flops_per_s /
                                            wave_efficiency(std::min(mb, p.m), std::min(nb, p.n)) +
                                            steps * step_fixed_s(std::min(mb, p.m),
                                                                 std::min(nb, p.n)),
                                        min_h2d / lim.h2d_bytes_per_s,
                                        min_d2h / lim.d2h_bytes_per_s});
            cands.push_back({Geo{mb, nb, kb, order == 1}, lb});
          }
    std::stable_sort(cands.begin(), cands.end(),
                     [](const Cand& x, const Cand& y) { return x.lb < y.lb; });

    // Every simulated plan is kept; the choice is made once the search ends (fewest H2D
    // bytes among the plans within kTrafficSlack of the fastest, then fewest steps).
    std::vector<std::pair<Geo, Plan>> sims;
    double fastest = 0.0;
    for (const Cand& cd : cands) {
      if (!sims.empty() &&
          (cd.lb > fastest * (1 + kTrafficSlack) || considered >= kMaxSimulations))
        break;
      if (!simulate(p, lim, cd.g, false, &trial))
        continue;
      ++considered;
      if (sims.empty() || trial.est_seconds < fastest)
        fastest = trial.est_seconds;
      sims.emplace_back(cd.g, trial);
    }
    for (const auto& [g, pl] : sims) {
      if (pl.est_seconds > fastest * (1 + kTrafficSlack))
        continue;
      const bool better =
          !found || pl.h2d_bytes < best_plan.h2d_bytes ||
          (pl.h2d_bytes == best_plan.h2d_bytes &&
           (pl.blocks_m * pl.blocks_n * pl.panels_k <
                best_plan.blocks_m * best_plan.blocks_n * best_plan.panels_k ||
            (pl.blocks_m * pl.blocks_n * pl.panels_k ==
                 best_plan.blocks_m * best_plan.blocks_n * best_plan.panels_k &&
             pl.est_seconds < best_plan.est_seconds)));
      if (better) {
        found = true;
        best = g;
        best_plan = pl;
      }
    }
    if (found || forced)
      break;
  }
  if (!found)
    return PlanStatus::budget_too_small;
  simulate(p, lim, best, true, out);
  out->candidates_considered = considered;
  return PlanStatus::ok;
}

} // namespace xvram
