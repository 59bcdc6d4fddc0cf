// epilogue.cu -- bias + activation over a resident column-major activation block.
//
// The SDK expresses "Linear + bias + ReLU" as a GEMM followed by a transaction whose
// callback launches this kernel on the transaction's stream (the reference's tiled GEMM
// takes no bias; its torch route rejects biased linear layers,
// reference python/xvram/torch_native.py:1913-1921).
//
//   Y[r, c] = act(Y[r, c] + bias[r])      r < rows (features), c < cols (batch)
//
// HBM-bound: one read and one write of Y, the bias vector from L1/L2.  Each thread
// handles float4 groups along the contiguous row dimension when ldy and the base are
// 16-byte aligned; the grid is sized in whole waves of the SM count.
#include "xvram_b200.h"

#include <cuda_runtime.h>

#include <cstdint>

namespace {

template <bool RELU, bool HAS_BIAS>
__global__ void __launch_bounds__(256)
    bias_act_vec4(float* __restrict__ y, long long ldy, long long rows4, long long cols,
                  const float* __restrict__ bias) {
  const long long total = rows4 * cols;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long c = i / rows4, r4 = i - c * rows4;
    float4* p = reinterpret_cast<float4*>(y + c * ldy) + r4;
    float4 v = *p;
    if constexpr (HAS_BIAS) {
      const float4 b = __ldg(reinterpret_cast<const float4*>(bias) + r4);
      v.x += b.x;
      v.y += b.y;
      v.z += b.z;
      v.w += b.w;
    }
    if constexpr (RELU) {
      v.x = fmaxf(v.x, 0.0f);
      v.y = fmaxf(v.y, 0.0f);
      v.z = fmaxf(v.z, 0.0f);
      v.w = fmaxf(v.w, 0.0f);
    }
    *p = v;
  }
}

template <bool RELU, bool HAS_BIAS>
__global__ void __launch_bounds__(256)
    bias_act_scalar(float* __restrict__ y, long long ldy, long long rows, long long cols,
                    const float* __restrict__ bias) {
  const long long total = rows * cols;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long c = i / rows, r = i - c * rows;
    float v = y[c * ldy + r];
    if constexpr (HAS_BIAS)
      v += __ldg(bias + r);
    if constexpr (RELU)
      v = fmaxf(v, 0.0f);
    y[c * ldy + r] = v;
  }
}

template <bool RELU, bool HAS_BIAS>
cudaError_t launch(float* y, long long ldy, long long rows, long long cols, const float* bias,
                   cudaStream_t s) {
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess)
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const bool vec = rows % 4 == 0 && ldy % 4 == 0 && (reinterpret_cast<uintptr_t>(y) & 15) == 0 &&
                   (!HAS_BIAS || (reinterpret_cast<uintptr_t>(bias) & 15) == 0);
  const long long work = vec ? rows / 4 * cols : rows * cols;
  long long blocks = (work + 255) / 256;
  const long long cap = static_cast<long long>(sms) * 8; // 8 resident 256-thread blocks per SM
  if (blocks > cap)
    blocks = cap;
  if (blocks < 1)
    blocks = 1;
  if (vec)
    bias_act_vec4<RELU, HAS_BIAS>
        <<<static_cast<unsigned>(blocks), 256, 0, s>>>(y, ldy, rows / 4, cols, bias);
  else
    bias_act_scalar<RELU, HAS_BIAS>
        <<<static_cast<unsigned>(blocks), 256, 0, s>>>(y, ldy, rows, cols, bias);
  return cudaGetLastError();
}

} // namespace

extern "C" XVRAM_B200_API xvram_status XVRAM_CALL xvram_b200_bias_activation(
    uint64_t y, int64_t ldy, int64_t rows, int64_t cols, uint64_t bias, uint32_t activation,
    uint64_t stream) {
  if (rows < 0 || cols < 0 || activation > XVRAM_B200_ACTIVATION_RELU || (rows > 0 && cols > 0 &&
      (!y || ldy < rows)))
    return XVRAM_STATUS_INVALID_ARGUMENT;
  if (rows == 0 || cols == 0)
    return XVRAM_STATUS_SUCCESS;
  float* yp = reinterpret_cast<float*>(y);
  const float* bp = reinterpret_cast<const float*>(bias);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const bool relu = activation == XVRAM_B200_ACTIVATION_RELU;
  cudaError_t e;
  if (relu)
    e = bp ? launch<true, true>(yp, ldy, rows, cols, bp, s)
           : launch<true, false>(yp, ldy, rows, cols, bp, s);
  else
    e = bp ? launch<false, true>(yp, ldy, rows, cols, bp, s)
           : launch<false, false>(yp, ldy, rows, cols, bp, s);
  return e == cudaSuccess ? XVRAM_STATUS_SUCCESS : XVRAM_STATUS_CUDA_ERROR;
}
