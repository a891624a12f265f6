// Test kernels of the device API (include/mlpk_device.cuh): a user kernel
// that encodes 3-d points (frequency encoding, sin/cos), runs the fused MLP
// on the encoded rows in registers and reduces the outputs to a per-row loss,
// all in one launch.  Built by mlp_megakernel_b200/build.py into
// tests/device_api/libmlpk_devtest.so; called by tests/test_device_api_gpu.py.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "../../include/mlpk_device.cuh"

namespace {

constexpr int kFreqs = 5;                 // 3 coords x (1 + 2 x 5) = 33 -> padded to 64 features
constexpr int kEnc = 64;
using SmallMLP = mlpk::device::FusedMLP<64, 64, 64, 16>;
using WideMLP = mlpk::device::FusedMLP<64, 128, 128, 128, 32>;

template <class MLP>
__global__ void __launch_bounds__(128, 1)
    encode_mlp_loss_kernel(const float* __restrict__ pts, int M, const __half* const* W, float* __restrict__ out,
                           float* __restrict__ loss, int* __restrict__ failed) {
  extern __shared__ uint8_t smem[];
  MLP mlp;
  const __half* ws[MLP::L];
  for (int l = 0; l < MLP::L; ++l) ws[l] = W[l];
  mlp.init(smem, ws);
  for (int tile = blockIdx.x; tile * 128 < M; tile += gridDim.x) {
    const int row = tile * 128 + static_cast<int>(threadIdx.x);
    const bool valid = row < M;
    float x[kEnc];
#pragma unroll
    for (int i = 0; i < kEnc; ++i) x[i] = 0.0f;
    if (valid) {
#pragma unroll
      for (int c = 0; c < 3; ++c) {
        const float p = pts[3 * row + c];
        x[c] = p;
        float f = 1.0f;
#pragma unroll
        for (int k = 0; k < kFreqs; ++k) {
          x[3 + 6 * k + 2 * c] = sinf(f * p);
          x[3 + 6 * k + 2 * c + 1] = cosf(f * p);
          f *= 2.0f;
        }
      }
    }
    float y[MLP::DL];
    const bool ok = mlp.forward(x, valid, y);
    if (!ok && threadIdx.x == 0) atomicOr(failed, 1);
    if (valid) {
      float s = 0.0f;
#pragma unroll
      for (int j = 0; j < MLP::DL; ++j) {
        out[static_cast<size_t>(row) * MLP::DL + j] = y[j];
        s += y[j] * y[j];
      }
      loss[row] = s;
    }
  }
  mlp.finish();
}

template <class MLP>
int run(const float* pts, int M, const void* const* W, float* out, float* loss, int* failed, int grid,
        cudaStream_t st) {
  const __half* const* w = reinterpret_cast<const __half* const*>(W);
  auto kern = encode_mlp_loss_kernel<MLP>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, MLP::SMEM_BYTES);
  if (e != cudaSuccess) return static_cast<int>(e);
  kern<<<grid, 128, MLP::SMEM_BYTES, st>>>(pts, M, w, out, loss, failed);
  return static_cast<int>(cudaGetLastError());
}

}  // namespace

// pts [M, 3] fp32; W: device array of device pointers to W_l fp16 [d_l][d_{l+1}];
// out [M, dL] fp32; loss [M] fp32; failed: device int set to 1 on a wait
// timeout.  net 0: 64-64-64-16, net 1: 64-128-128-128-32.  Returns a
// cudaError_t value.
extern "C" int mlpk_devtest_encode_mlp_loss(int net, const float* pts, int M, const void* const* W_dev,
                                            float* out, float* loss, int* failed, int grid, void* stream) {
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (net == 0) return run<SmallMLP>(pts, M, W_dev, out, loss, failed, grid, st);
  return run<WideMLP>(pts, M, W_dev, out, loss, failed, grid, st);
}
