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

// Block = one layer x 32 output columns; 1024 threads = 32 columns x 32 row
// groups.  Thread (c, r) holds rows r, r+32, ... (at most kWnMaxPer of them:
// widths up to 256) of column c in registers, so every value is read from
// global memory once, in one batch of independent loads; the per-column sums
// are combined through shared memory in a fixed order (row group 0, 1, ...),
// so the results are bitwise reproducible.  (The first version, 8 row groups
// re-reading v in a second pass, took ~9 us per launch for 3L128, two
// dependent chains of loads.)
constexpr int kWnCols = 32;
constexpr int kWnRowGroups = 32;
constexpr int kWnMaxPer = 8;  // rows per thread: 256 / 32

__device__ __forceinline__ int wn_block_layer(const WnShape& s, int b, int& col0) {
  int l = 0, nb = 0;
  while (true) {
    const int blocks_l = (s.dout[l] + kWnCols - 1) / kWnCols;
    if (b < nb + blocks_l || l + 1 == s.num_layers) {
      col0 = (b - nb) * kWnCols;
      return l;
    }
    nb += blocks_l;
    ++l;
  }
}

__device__ __forceinline__ float wn_col_sum(float v, float (*red)[kWnCols + 1], int c, int r) {
  red[r][c] = v;
  __syncthreads();
  float t = 0.0f;
#pragma unroll
  for (int k = 0; k < kWnRowGroups; ++k) t += red[k][c];  // fixed order
  __syncthreads();
  return t;
}

__global__ void __launch_bounds__(kWnCols * kWnRowGroups)
    mlp_wn_fwd_kernel(WnShape s, const float* __restrict__ v_all, const float* __restrict__ g_all,
                      WnOut out, float* __restrict__ inv_norm) {
  pdl_enter();
  __shared__ float red[kWnRowGroups][kWnCols + 1];
  const int c = threadIdx.x % kWnCols, r = threadIdx.x / kWnCols;
  int col0;
  const int l = wn_block_layer(s, blockIdx.x, col0);
  const int K = s.din[l], N = s.dout[l];
  const int j = col0 + c;
  const bool valid = j < N;
  const float* v = v_all + s.voff[l];
  float a[kWnMaxPer];
#pragma unroll
  for (int u = 0; u < kWnMaxPer; ++u) {
    const int i = r + u * kWnRowGroups;
    a[u] = (valid && i < K) ? v[static_cast<size_t>(i) * N + j] : 0.0f;
  }
  float ss = 0.0f;
#pragma unroll
  for (int u = 0; u < kWnMaxPer; ++u) ss = fmaf(a[u], a[u], ss);
  ss = wn_col_sum(ss, red, c, r);
  if (!valid) return;
  const float inv = 1.0f / sqrtf(ss);
  const float scale = g_all[s.goff[l] + j] * inv;
  __half* w = out.w[0];  // a constant-index pick: out.w[l] would copy out to the stack
#pragma unroll
  for (int k = 1; k < 8; ++k)
    if (k == l) w = out.w[k];
#pragma unroll
  for (int u = 0; u < kWnMaxPer; ++u) {
    const int i = r + u * kWnRowGroups;
    if (i < K) w[static_cast<size_t>(i) * N + j] = __float2half_rn(a[u] * scale);
  }
  if (r == 0) inv_norm[s.goff[l] + j] = inv;
}

// dg_j = <dW_:j, v_:j> / ||v_:j||
// dv_:j = (g_j / ||v_:j||) dW_:j - (g_j dg_j / ||v_:j||^2) v_:j
__global__ void __launch_bounds__(kWnCols * kWnRowGroups)
    mlp_wn_bwd_kernel(WnShape s, const float* __restrict__ dw_all, const float* __restrict__ v_all,
                      const float* __restrict__ g_all, const float* __restrict__ inv_norm,
                      float* __restrict__ dv_all, float* __restrict__ dg_all) {
  pdl_enter();
  __shared__ float red[kWnRowGroups][kWnCols + 1];
  const int c = threadIdx.x % kWnCols, r = threadIdx.x / kWnCols;
  int col0;
  const int l = wn_block_layer(s, blockIdx.x, col0);
  const int K = s.din[l], N = s.dout[l];
  const int j = col0 + c;
  const bool valid = j < N;
  const float* v = v_all + s.voff[l];
  const float* dw = dw_all + s.voff[l];
  float* dv = dv_all + s.voff[l];
  float gv[kWnMaxPer], vv[kWnMaxPer];
#pragma unroll
  for (int u = 0; u < kWnMaxPer; ++u) {
    const int i = r + u * kWnRowGroups;
    const bool in = valid && i < K;
    const size_t e = static_cast<size_t>(i) * N + j;
    gv[u] = in ? dw[e] : 0.0f;
    vv[u] = in ? v[e] : 0.0f;
  }
  float dot = 0.0f;
#pragma unroll
  for (int u = 0; u < kWnMaxPer; ++u) dot = fmaf(gv[u], vv[u], dot);
  dot = wn_col_sum(dot, red, c, r);
  if (!valid) return;
  const float inv = inv_norm[s.goff[l] + j];
  const float gj = g_all[s.goff[l] + j];
  const float dg = dot * inv;
  const float a = gj * inv;
  const float b = gj * dg * inv * inv;
#pragma unroll
  for (int u = 0; u < kWnMaxPer; ++u) {
    const int i = r + u * kWnRowGroups;
    if (i < K) dv[static_cast<size_t>(i) * N + j] = fmaf(a, gv[u], -b * vv[u]);
  }
  if (r == 0) dg_all[s.goff[l] + j] = dg;
}

__host__ __device__ inline int wn_num_blocks(const WnShape& s) {
  int n = 0;
  for (int l = 0; l < s.num_layers; ++l) n += (s.dout[l] + kWnCols - 1) / kWnCols;
  return n;
}

}  // namespace mlpk
