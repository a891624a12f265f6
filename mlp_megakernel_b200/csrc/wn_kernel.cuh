// Weight normalisation W = g * v / ||v|| (per output neuron = per column of
// the [in, out] weight), forward and backward, ONE launch for all layers.
//
// Replaces the reference's _wn_fwd_kernel and _wn_bwd_from_dw_T_kernel
// (mlp_fused.md:466-483): contiguous parameter storage (v_all, g_all), the
// forward also returns inv_norm = 1/||v|| for the backward, and the backward
// reads the fp32 dW produced by the weight-gradient reduction directly.
//
// Layout: v_all = concat over layers of v_l [d_l][d_{l+1}] (row-major fp32),
// g_all = concat of g_l [d_{l+1}], inv_norm likewise; W_l are separate fp16
// tensors (the GEMM operands).  One thread per output column (d_{l+1} columns
// per layer): reads of a column are coalesced across the threads of a warp.
#pragma once
#include <cuda_fp16.h>

#include <cstdint>

namespace mlpk {

struct WnShape {
  int num_layers;
  int din[8];     // d_l
  int dout[8];    // d_{l+1}
  long long voff[8];  // element offset of v_l in v_all (and dW_l in dW_all)
  int goff[8];    // element offset of g_l in g_all
  int total_cols;
};

__device__ __forceinline__ int wn_layer_of(const WnShape& s, int c, int& j) {
  int l = 0;
  while (l + 1 < s.num_layers && c >= s.goff[l + 1]) ++l;
  j = c - s.goff[l];
  return l;
}

struct WnOut {
  __half* w[8];
};

__global__ void mlp_wn_fwd_kernel(WnShape s, const float* __restrict__ v_all,
                                  const float* __restrict__ g_all, WnOut out,
                                  float* __restrict__ inv_norm) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= s.total_cols) return;
  int j;
  const int l = wn_layer_of(s, c, j);
  const int K = s.din[l], N = s.dout[l];
  const float* v = v_all + s.voff[l];
  float ss = 0.0f;
  for (int i = 0; i < K; ++i) {
    const float a = v[static_cast<size_t>(i) * N + j];
    ss = fmaf(a, a, ss);
  }
  const float inv = 1.0f / sqrtf(ss);
  const float scale = g_all[c] * inv;
  __half* w = out.w[l];
  for (int i = 0; i < K; ++i)
    w[static_cast<size_t>(i) * N + j] = __float2half_rn(v[static_cast<size_t>(i) * N + j] * scale);
  inv_norm[c] = inv;
}

// dg_j = <dW_:j, v_:j> / ||v_:j||
// dv_:j = (g_j / ||v_:j||) dW_:j - (g_j dg_j / ||v_:j||^2) v_:j
__global__ void mlp_wn_bwd_kernel(WnShape s, const float* __restrict__ dw_all,
                                  const float* __restrict__ v_all, const float* __restrict__ g_all,
                                  const float* __restrict__ inv_norm, float* __restrict__ dv_all,
                                  float* __restrict__ dg_all) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= s.total_cols) return;
  int j;
  const int l = wn_layer_of(s, c, j);
  const int K = s.din[l], N = s.dout[l];
  const float* v = v_all + s.voff[l];
  const float* dw = dw_all + s.voff[l];
  float* dv = dv_all + s.voff[l];
  const float inv = inv_norm[c];
  const float gj = g_all[c];
  float dot = 0.0f;
  for (int i = 0; i < K; ++i) {
    const size_t e = static_cast<size_t>(i) * N + j;
    dot = fmaf(dw[e], v[e], dot);
  }
  const float dg = dot * inv;
  const float a = gj * inv;
  const float b = gj * dg * inv * inv;
  for (int i = 0; i < K; ++i) {
    const size_t e = static_cast<size_t>(i) * N + j;
    dv[e] = fmaf(a, dw[e], -b * v[e]);
  }
  dg_all[c] = dg;
}

}  // namespace mlpk
