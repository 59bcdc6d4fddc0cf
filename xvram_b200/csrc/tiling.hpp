// tiling.hpp -- which C tile the TMA-fed FFMA kernel runs for an M-/N-major problem.
//
// Two tilings compute the same bits (every output is one FFMA chain in k order):
//   * 192 x 192 tiles, 12 warps, 12 x 8 accumulators per thread;
//   * 128 x 256 tiles (128 x 128 when n <= 128), 8 warps, 8 x 16 per thread.
// Both run one CTA per SM and split a last wave that is at most half full into half-width
// units.  The 12-warp form issues FMAs about 5 % faster per tile-FLOP (three warps per SM
// sub-partition instead of two; C 9216 x 9216 x 4096: 10.867 against 11.391 ms), so it
// runs unless its waves -- ragged edges and the tail included -- cost more than that.
// Shared by the kernel's dispatch (sgemm_ffma.cu) and the out-of-core planner's
// per-launch cost model (planner.cpp), so the two agree.
#pragma once

#include <cstdint>

namespace xvram {

constexpr double kTile256Rate = 0.95; // 128 x 256 FMA rate relative to 192 x 192

// Waves a launch of `tiles` one-CTA-per-SM tiles takes on `sms` SMs.
inline double tile_waves(int64_t tiles, int64_t sms) {
  const int64_t tail = tiles % sms;
  return static_cast<double>(tiles / sms) + (tail == 0 ? 0.0 : (2 * tail <= sms ? 0.5 : 1.0));
}

struct Tiling {
  int tile_m, tile_n;
  double rate; // FMA rate relative to the 192 x 192 form
};

inline Tiling choose_tiling(int64_t m, int64_t n, int64_t sms) {
  const Tiling t256{128, n > 128 ? 256 : 128, kTile256Rate};
  if (m <= 128 || n <= 128 || sms <= 0)
    return t256;
  const auto cdiv = [](int64_t a, int64_t b) { return (a + b - 1) / b; };
  const double c192 = tile_waves(cdiv(m, 192) * cdiv(n, 192), sms) * 192.0 * 192.0;
  const double c256 = tile_waves(cdiv(m, 128) * cdiv(n, 256), sms) * 128.0 * 256.0 / kTile256Rate;
  return c192 < c256 ? Tiling{192, 192, 1.0} : t256;
}

} // namespace xvram
