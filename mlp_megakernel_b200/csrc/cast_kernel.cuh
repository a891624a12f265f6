// fp32 <-> fp16 casts for the fp32-input forward (the reference's kernel.py
// accepts fp32 x and W, kernel.py:37-43 / 134-138: its products run on fp32
// operands, every hidden activation is rounded to fp16 (kernel.py:110, 117)
// and the fp16-rounded result is stored into an fp32 output).  The fp32 path
// of this library casts x and W to fp16 (round to nearest even), runs the fp16
// fused kernel and widens the fp16 result to fp32 -- the same rounding points
// for the activations and the output; the operands carry 10 mantissa bits in
// both (tf32 / fp16), fp16's narrower exponent range (|x| < 65504) being the
// difference.  HBM-bound elementwise kernels: 8 elements per thread per step,
// 16-byte loads and stores, grid-stride.
#pragma once
#include <cuda_fp16.h>

#include <cstdint>

namespace mlpk {

__global__ void __launch_bounds__(256) mlp_cast_f32_f16_kernel(const float* __restrict__ src,
                                                              __half* __restrict__ dst, int64_t n) {
  pdl_enter();
  const int64_t n8 = n / 8;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n8; i += stride) {
    const float4 a = reinterpret_cast<const float4*>(src)[2 * i];
    const float4 b = reinterpret_cast<const float4*>(src)[2 * i + 1];
    __half2 h[4] = {__floats2half2_rn(a.x, a.y), __floats2half2_rn(a.z, a.w), __floats2half2_rn(b.x, b.y),
                    __floats2half2_rn(b.z, b.w)};
    reinterpret_cast<uint4*>(dst)[i] = *reinterpret_cast<uint4*>(h);
  }
  for (int64_t i = 8 * n8 + blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n; i += stride)
    dst[i] = __float2half_rn(src[i]);
}

__global__ void __launch_bounds__(256) mlp_cast_f16_f32_kernel(const __half* __restrict__ src,
                                                              float* __restrict__ dst, int64_t n) {
  pdl_enter();
  const int64_t n8 = n / 8;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n8; i += stride) {
    uint4 v = reinterpret_cast<const uint4*>(src)[i];
    const __half2* h = reinterpret_cast<const __half2*>(&v);
    const float2 a = __half22float2(h[0]), b = __half22float2(h[1]), c = __half22float2(h[2]),
                 d = __half22float2(h[3]);
    reinterpret_cast<float4*>(dst)[2 * i] = make_float4(a.x, a.y, b.x, b.y);
    reinterpret_cast<float4*>(dst)[2 * i + 1] = make_float4(c.x, c.y, d.x, d.y);
  }
  for (int64_t i = 8 * n8 + blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n; i += stride)
    dst[i] = __half2float(src[i]);
}

}  // namespace mlpk
