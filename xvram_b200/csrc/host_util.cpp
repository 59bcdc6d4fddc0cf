// host_util.cpp -- see host_util.hpp.
#include "host_util.hpp"

#include <algorithm>
#include <cstring>
#include <thread>
#include <vector>

namespace xvram {
namespace {

inline uint64_t mix64(uint64_t z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

template <class F> void parallel_for(uint64_t count, int threads, F&& body) {
  if (threads <= 1 || count < 2) {
    body(0, count);
    return;
  }
  std::vector<std::thread> pool;
  pool.reserve(static_cast<size_t>(threads - 1));
  for (int t = 1; t < threads; ++t)
    pool.emplace_back([&, t] { body(count * t / threads, count * (t + 1) / threads); });
  body(0, count / threads);
  for (auto& th : pool)
    th.join();
}

} // namespace

int host_threads() {
  const unsigned n = std::thread::hardware_concurrency();
  return n == 0 ? 1 : static_cast<int>(std::min(n, 64u));
}

void parallel_memcpy(void* dst, const void* src, uint64_t bytes) {
  constexpr uint64_t kSplit = 16ull << 20;
  if (bytes < kSplit) {
    std::memcpy(dst, src, bytes);
    return;
  }
  const int threads = static_cast<int>(std::min<uint64_t>(host_threads(), bytes / (4ull << 20)));
  const uint64_t lines = (bytes + 63) / 64;
  parallel_for(lines, threads, [&](uint64_t b, uint64_t e) {
    const uint64_t lo = b * 64, hi = std::min(bytes, e * 64);
    if (hi > lo)
      std::memcpy(static_cast<char*>(dst) + lo, static_cast<const char*>(src) + lo, hi - lo);
  });
}

float uniform_at(uint64_t seed, uint64_t index) {
  const uint64_t u = mix64(mix64(seed) ^ index);
  return static_cast<float>(static_cast<int32_t>(u >> 40) - 8388608) * (1.0f / 8388608.0f);
}

void fill_uniform(float* dst, uint64_t count, uint64_t seed, uint64_t first_index, int threads) {
  if (threads <= 0)
    threads = host_threads();
  const uint64_t s = mix64(seed);
  parallel_for(count, count < (1u << 20) ? 1 : threads, [&](uint64_t b, uint64_t e) {
    for (uint64_t i = b; i < e; ++i) {
      const uint64_t u = mix64(s ^ (first_index + i));
      dst[i] = static_cast<float>(static_cast<int32_t>(u >> 40) - 8388608) * (1.0f / 8388608.0f);
    }
  });
}

} // namespace xvram
