// probes.cu -- FP32 pipe peak probe.
//
// The FP32 (non-tensor) peak is the denominator of the SGEMM roofline.  It is not in
// the driver-measured peak file, so the bench measures it on the same device in the
// same run: 16 independent FFMA chains per thread (no chain waits on its own latency),
// enough warps to keep all four SM sub-partitions issuing an FFMA every cycle, and no
// memory traffic.
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

} // namespace

cudaError_t ffma_peak_probe(int blocks, int iterations, float* sink, cudaStream_t stream) {
  ffma_peak_kernel<<<blocks, 256, 0, stream>>>(iterations, sink);
  return cudaGetLastError();
}

} // namespace xvram
