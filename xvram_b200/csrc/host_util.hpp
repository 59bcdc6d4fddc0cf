// host_util.hpp -- host-side helpers: parallel memcpy and the synthetic input generator.
#pragma once

#include <cstdint>

namespace xvram {

// memcpy split across host threads for large copies (page-locked backing stores are
// filled and drained at memory bandwidth rather than single-core speed).
void parallel_memcpy(void* dst, const void* src, uint64_t bytes);

// Element `index` of the uniform[-1, 1) stream `seed` (counter-based, SplitMix64
// finaliser): (q - 2^23) * 2^-23 for a 24-bit draw q, exact in binary32.
float uniform_at(uint64_t seed, uint64_t index);

// dst[i] = uniform_at(seed, first_index + i), filled on `threads` host threads
// (0 = all hardware threads).
void fill_uniform(float* dst, uint64_t count, uint64_t seed, uint64_t first_index, int threads);

// Host hardware threads available to the process.
int host_threads();

} // namespace xvram
