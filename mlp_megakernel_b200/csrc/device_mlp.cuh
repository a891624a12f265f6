// A fused softplus MLP that a user's own CUDA kernel calls on rows it holds in
// registers (sm_100a), so that the step before the MLP (an input encoding)
// and the step after it (a loss, a reduction, a renderer's compositing) run
// in the same kernel instead of round-tripping through global memory.  The
// reference names this as the next step of its design (mlp_fused.md:406:
// "device-side MLP callable from user kernels", as tiny-cuda-nn inlines its
// fully fused MLP); the arithmetic is the library's forward: fp16 GEMM
// operands, fp32 accumulation in TMEM, softplus (beta 1, threshold 20) in
// fp32 registers, each hidden activation rounded to fp16 for the next GEMM
// and the output rounded to fp16 (kernel.py:108-123).
//
// Usage, inside a kernel launched with at least 128 threads per CTA and
// SMEM_BYTES of dynamic shared memory:
//
//   using MLP = mlpk::device::FusedMLP<64, 64, 64, 16>;   // widths d0 .. dL
//   extern __shared__ uint8_t smem[];
//   MLP mlp;
//   mlp.init(smem, weights);             // every thread of the CTA; W_l [d_l][d_{l+1}] fp16, global
//   for (each group of 128 rows) {
//     if (threadIdx.x < 128) {           // one row per thread of the first warpgroup
//       float x[64] = ...;               // the caller's encoding of its row
//       float y[16];
//       bool ok = mlp.forward(x, row_valid, y);
//       ...                              // the caller's use of y
//     }
//   }
//   mlp.finish();                        // every thread of the CTA
//
// forward() is called by threads 0..127 together (a warpgroup: warp w owns
// TMEM lanes 32w..32w+31, i.e. rows 32w..32w+31 of the tile); it uses named
// barrier 15 among them and returns false if one of its bounded waits on the
// tensor core expired (the outputs are then zeros).  Constraints: every
// width 16, 32 or a multiple of 64 and at most 256 (pad a narrower encoding
// with zero columns), hidden widths 32 or multiples of 64, the weights and one
// 128-row input tile in shared memory (SMEM_BYTES).
#pragma once
#include "fwd_kernel.cuh"

namespace mlpk {
namespace device {

constexpr int kNamedBarrier = 15;

template <int... Ds>
class FusedMLP {
 public:
  using NetT = Net<Ds...>;
  static constexpr int L = NetT::L;
  static constexpr int D0 = NetT::template D<0>();
  static constexpr int DL = NetT::template D<L>();
  static constexpr int HMAX = NetT::max_hidden_or_out();
  static constexpr int W_BYTES = NetT::w_total();
  static constexpr int X_BYTES = align_up(tile_bytes(kTileM, D0), 1024);
  static constexpr int OFF_X = W_BYTES;
  static constexpr int OFF_MISC = OFF_X + X_BYTES;  // mbarrier, TMEM base, abort flag
  static constexpr int SMEM_BYTES = OFF_MISC + 64 + 1024;  // + alignment slack
  static constexpr int SLOT = align_up(HMAX, 32);
  static constexpr int TMEM_COLS = 2 * SLOT <= 32 ? 32 : 2 * SLOT <= 64 ? 64 : 2 * SLOT <= 128 ? 128
                                   : 2 * SLOT <= 256 ? 256 : 512;
  static constexpr int THREADS = 128;

  // every operand row must be a swizzle-layout pitch: 16, 32 or a multiple
  // of 64 fp16 columns (32, 64 or 128-byte chunks)
  __host__ __device__ static constexpr bool dims_ok() {
    for (int i = 0; i <= L; ++i) {
      const int d = NetT::dim(i);
      if (!(d == 16 || d == 32 || d % 64 == 0) || d > 256) return false;
    }
    for (int i = 1; i < L; ++i)
      if (NetT::dim(i) % 32 != 0) return false;
    return true;
  }
  static_assert(L >= 1, "at least one layer");
  static_assert(dims_ok(), "widths: 16, 32 or multiples of 64, at most 256 (hidden: 32 or multiples of 64)");
  static_assert(SMEM_BYTES <= 232448, "weights and input tile exceed shared memory");

  // Copies the weights into shared memory (UMMA layout), allocates TMEM and
  // sets up the barrier.  Every thread of the CTA calls it (it synchronises
  // the CTA); W[l] is [d_l][d_{l+1}] fp16 row-major in global memory, 16-byte
  // aligned.
  __device__ void init(uint8_t* smem_raw, const __half* const* W) {
    const uint32_t raw = smem_u32(smem_raw);
    base_ = (raw + 1023u) & ~1023u;
    gbase_ = smem_raw + (base_ - raw);
    static_for<0, L>([&](auto lc) {
      constexpr int l = decltype(lc)::value;
      constexpr int K = NetT::template D<l>();
      constexpr int N = NetT::template D<l + 1>();
      constexpr int C = chunk_elems(N);
      constexpr int P = pitch_bytes(N);
      const uint4* src = reinterpret_cast<const uint4*>(W[l]);
      // 16-byte units: row k, columns 8u .. 8u+7, placed as a TMA box {C, K}
      // of the chunk the columns belong to would place them
      for (int i = threadIdx.x; i < K * N / 8; i += blockDim.x) {
        const int k = i / (N / 8), u = i % (N / 8);
        const int n0 = 8 * u;
        const uint4 v = __ldg(src + i);
        st_shared_v4(base_ + NetT::template w_off<l>() + (n0 / C) * K * P + swz_off<P>(k, (n0 % C) / 8), v.x,
                     v.y, v.z, v.w);
      }
    });
    if (threadIdx.x == 0) {
      mbar_init(bar(), 1);
      *abort_flag() = 0;
      fence_mbar_init();
    }
    if (threadIdx.x < 32) {
      tmem_alloc(base_ + OFF_MISC + 8, TMEM_COLS);
      tmem_relinquish();
    }
    fence_proxy_async_smem();  // the weights are read by the tensor core
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    tmem_ = *reinterpret_cast<volatile uint32_t*>(gbase_ + OFF_MISC + 8);
    phase_ = 0;
  }

  // One forward step of the 128-row tile the warpgroup holds: thread t
  // supplies row t (x[0..d0-1]; `valid` false for a row past the caller's
  // batch, which then computes on zeros) and receives y[0..dL-1].  Returns
  // false if a bounded wait expired.
  __device__ bool forward(const float* x, bool valid, float* y) {
    const uint32_t row = threadIdx.x;
    const uint32_t lane_off = (row & ~31u) << 16;
    // 1. the input row as the first GEMM's K-major A operand
    {
      constexpr int C = chunk_elems(D0);
      constexpr int P = pitch_bytes(D0);
#pragma unroll
      for (int u = 0; u < D0 / 8; ++u) {
        uint32_t w[4];
#pragma unroll
        for (int j = 0; j < 4; ++j)
          w[j] = valid ? pack_half2(x[8 * u + 2 * j], x[8 * u + 2 * j + 1]) : 0u;
        st_shared_v4(base_ + OFF_X + (8 * u / C) * (kTileM * P) + swz_off<P>(row, (8 * u % C) / 8), w[0],
                     w[1], w[2], w[3]);
      }
    }
    fence_proxy_async_smem();
    tc_fence_before();
    named_bar_sync(kNamedBarrier, THREADS);
    bool ok = true;
    // 2. layer 0 from shared memory, then every hidden layer from TMEM
    static_for<0, L>([&](auto lc) {
      constexpr int l = decltype(lc)::value;
      constexpr int K = NetT::template D<l>();
      constexpr int N = NetT::template D<l + 1>();
      constexpr uint32_t idesc = make_idesc_f16(kTileM, N, 0, 1);
      const uint32_t d_tmem = tmem_ + (l & 1) * SLOT;
      const uint32_t a_tmem = tmem_ + ((l & 1) ^ 1) * SLOT;
      if (!ok) return;
      if constexpr (l > 0) {
        // softplus of layer l-1's accumulator (this thread's row), packed
        // fp16 back into TMEM as layer l's A operand
        const uint32_t tb = tmem_ + lane_off + ((l - 1) & 1) * SLOT;
#pragma unroll
        for (int j = 0; j < K / 32; ++j) {
          uint32_t a[32];
          tmem_ld_wait_x32(tb + 32 * j, a);
          uint32_t w[16];
          pack_cols<16, true>(a, w);
          tmem_st_x16(tb + h_tmem_col(32 * j), w);
        }
        tmem_wait_st();
        tc_fence_before();
        named_bar_sync(kNamedBarrier, THREADS);
      }
      if (threadIdx.x == 0) {
        tc_fence_after();
        const uint64_t bdesc0 = mnmajor_base_desc<K, N>(base_ + NetT::template w_off<l>());
        if constexpr (l == 0) {
          const uint64_t adesc0 = kmajor_base_desc<K>(base_ + OFF_X);
#pragma unroll
          for (int k = 0; k < K / 16; ++k)
            umma_f16(d_tmem, adesc0 + (kmajor_koff<kTileM, K>(k) >> 4), bdesc0 + (mnmajor_koff<N>(k) >> 4), idesc,
                     k > 0 ? 1u : 0u);
        } else {
#pragma unroll
          for (int k = 0; k < K / 16; ++k)
            umma_f16_ts(d_tmem, a_tmem + h_tmem_col(16 * k), bdesc0 + (mnmajor_koff<N>(k) >> 4), idesc,
                        k > 0 ? 1u : 0u);
        }
        umma_commit(bar());
      }
      ok = mbar_wait(bar(), phase_ & 1, abort_flag(), kDevTimeoutEpi);
      ++phase_;
      tc_fence_after();
    });
    // 3. the output row: fp32 accumulator rounded to fp16 (the kernels' output)
    if (ok) {
      const uint32_t tb = tmem_ + lane_off + ((L - 1) & 1) * SLOT;
#pragma unroll
      for (int c = 0; c < DL; c += 16) {
        uint32_t r[16];
        tmem_ld_wait_x16(tb + c, r);
#pragma unroll
        for (int j = 0; j < 16; ++j) y[c + j] = __half2float(__float2half_rn(__uint_as_float(r[j])));
      }
    } else {
#pragma unroll
      for (int c = 0; c < DL; ++c) y[c] = 0.0f;
    }
    tc_fence_before();  // the next call's MMAs overwrite what this call read
    return ok;
  }

  // Frees TMEM; every thread that called init() calls it (it synchronises
  // the CTA).
  __device__ void finish() {
    tc_fence_before();
    __syncthreads();
    if (threadIdx.x < 32) {
      tc_fence_after();
      tmem_dealloc(tmem_, TMEM_COLS);
    }
  }

 private:
  __device__ uint32_t bar() const { return base_ + OFF_MISC; }
  __device__ volatile int* abort_flag() const { return reinterpret_cast<volatile int*>(gbase_ + OFF_MISC + 16); }
  uint32_t base_ = 0;
  uint8_t* gbase_ = nullptr;
  uint32_t tmem_ = 0;
  uint32_t phase_ = 0;
};

}  // namespace device
}  // namespace mlpk
