// probes.cu -- FP32 pipe peak probes.
//
// The FP32 (non-tensor) peak is the denominator of the SGEMM roofline.  It is not in
// the driver-measured peak file, so the bench measures it on the same device in the
// same run: 16 independent FMA chains per thread (no chain waits on its own latency),
// enough warps to keep all four SM sub-partitions busy, and no memory traffic.  Two
// forms: scalar FFMA (one FMA per lane per instruction) and packed FFMA2 (two per lane
// per instruction, which the SGEMM kernel's main loop uses); the roofline takes the
// higher of the two.
#include "kernels.hpp"

namespace xvram {
namespace {

__global__ void __launch_bounds__(256) ffma_peak_kernel(int iterations, float* sink) {
  float v[16];
#pragma unroll
  for (int j = 0; j < 16; ++j)
    v[j] = 1.0f + 1e-7f * static_cast<float>(threadIdx.x + j);
  const float x = 0.999999f, y = 1e-7f;
  for (int it = 0; it < iterations; ++it) {
#pragma unroll
    for (int r = 0; r < 32; ++r)
#pragma unroll
      for (int j = 0; j < 16; ++j)
        v[j] = fmaf(v[j], x, y);
  }
  float s = 0.0f;
#pragma unroll
  for (int j = 0; j < 16; ++j)
    s += v[j];
  if (s == 123.456f) // never true for these inputs; keeps the chains live
    sink[0] = s;
}

// Packed form: 8 float2 chains per thread, the same 512 FMAs per thread per iteration.
__global__ void __launch_bounds__(256) ffma2_peak_kernel(int iterations, float* sink) {
  float2 v[8];
#pragma unroll
  for (int j = 0; j < 8; ++j)
    v[j] = make_float2(1.0f + 1e-7f * static_cast<float>(threadIdx.x + 2 * j),
                       1.0f + 1e-7f * static_cast<float>(threadIdx.x + 2 * j + 1));
  const float2 x = make_float2(0.999999f, 0.999999f), y = make_float2(1e-7f, 1e-7f);
  for (int it = 0; it < iterations; ++it) {
#pragma unroll
    for (int r = 0; r < 32; ++r)
#pragma unroll
      for (int j = 0; j < 8; ++j)
        v[j] = __ffma2_rn(v[j], x, y);
  }
  float s = 0.0f;
#pragma unroll
  for (int j = 0; j < 8; ++j)
    s += v[j].x + v[j].y;
  if (s == 123.456f)
    sink[0] = s;
}

} // namespace

cudaError_t ffma_peak_probe(int blocks, int iterations, float* sink, cudaStream_t stream,
                            bool packed) {
  if (packed)
    ffma2_peak_kernel<<<blocks, 256, 0, stream>>>(iterations, sink);
  else
    ffma_peak_kernel<<<blocks, 256, 0, stream>>>(iterations, sink);
  return cudaGetLastError();
}

} // namespace xvram
