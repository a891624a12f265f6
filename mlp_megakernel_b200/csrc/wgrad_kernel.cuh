// Split-K weight gradients for the streamed backward (networks whose weight
// gradients do not fit in TMEM next to the data-gradient chain, e.g. the wide
// D = H = OUT = 256 network: 3 x 256 KB of fp32 dW).
//
//   dW_l = sum over rows of A_l^T B_l,  A_l = h_l (x for l = 0)  [M, d_l],
//                                       B_l = dz_{l+1} (grad_out for l = L-1)  [M, d_{l+1}]
//
// (the weight-gradient GEMMs of mlp_fused.md:92-94, which the reference sends
// to cuBLAS at large batch, mlp_fused.md:139-146).  Every layer gets P CTAs;
// CTA (l, p) accumulates dW_l over its contiguous share of 64-row stages in
// TMEM (d_l / 128 accumulators of 128 lanes x d_{l+1} fp32 columns) and
// writes one fp32 partial; mlp_reduce_kernel then sums the P partials of each
// layer in a fixed order, so dW is bitwise reproducible.
//
// Roles: warp 0 = TMA producer (A and B stages through a 3-deep ring), warp 1 =
// TMEM owner + MMA issuer (both operands MN-major from shared memory, K = the
// stage's 64 rows), warps 2..5 = dump of the partial (thread = dW row).
// Rows past M are zero-filled by TMA and add nothing.
#pragma once
#include "fwd_kernel.cuh"

namespace mlpk {

constexpr int kWgStageRows = 64;

template <int L>
struct alignas(64) WgradMaps {
  CUtensorMap a[L];  // h_l (x for l = 0), box {64, 64}
  CUtensorMap b[L];  // dz_{l+1} (grad_out for l = L-1), box {64, 64}
  float* partials;   // [gridDim.x][DA * DB] fp32, row-major dW_l of CTA (l, p)
};

template <int DA, int DB>
struct WgradCfg {
  static constexpr int MB = DA / 128;  // accumulator blocks (dW rows per block: 128)
  static constexpr int A_BYTES = kWgStageRows * DA * 2;
  static constexpr int B_BYTES = kWgStageRows * DB * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int NSTAGE = 3;
  static constexpr int OFF_BAR = NSTAGE * STAGE_BYTES;
  static constexpr int NUM_BARS = 2 * NSTAGE + 1;  // full[], empty[], done
  static constexpr int OFF_MISC = OFF_BAR + 8 * NUM_BARS;
  static constexpr int SMEM_BYTES = OFF_MISC + 16 + 1024;
  static constexpr int TMEM_COLS_RAW = MB * DB;
  static constexpr int TMEM_COLS = TMEM_COLS_RAW <= 128 ? 128 : TMEM_COLS_RAW <= 256 ? 256 : 512;
  static constexpr int THREADS = 6 * 32;
  static_assert(DA % 128 == 0 && DB % 64 == 0 && DB <= 256, "weight-gradient tile shape");
  static_assert(TMEM_COLS_RAW <= 512, "weight-gradient accumulators exceed TMEM");
  static_assert(SMEM_BYTES <= 232448, "shared memory budget exceeded");
};

template <int L, int DA, int DB>
__global__ void __launch_bounds__(WgradCfg<DA, DB>::THREADS, 1)
    mlp_wgrad_kernel(const __grid_constant__ WgradMaps<L> maps, int M, int ctas_per_layer) {
  using Cfg = WgradCfg<DA, DB>;
  constexpr int NST = Cfg::NSTAGE;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t sbase = (raw + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (sbase - raw);
  const uint32_t s_bar = sbase + Cfg::OFF_BAR;
  auto bar_full = [&](int b) { return s_bar + 8u * b; };
  auto bar_empty = [&](int b) { return s_bar + 8u * (NST + b); };
  const uint32_t bar_done = s_bar + 8u * (2 * NST);
  const uint32_t s_tmem_slot = sbase + Cfg::OFF_MISC;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(gbase + Cfg::OFF_MISC + 4);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  const int l = static_cast<int>(blockIdx.x) / ctas_per_layer;
  const int p = static_cast<int>(blockIdx.x) % ctas_per_layer;
  const int nst = (M + kWgStageRows - 1) / kWgStageRows;
  const int s0 = static_cast<int>(static_cast<long long>(p) * nst / ctas_per_layer);
  const int s1 = static_cast<int>(static_cast<long long>(p + 1) * nst / ctas_per_layer);

  if (threadIdx.x == 0) {
    for (int b = 0; b < NST; ++b) {
      mbar_init(bar_full(b), 1);
      mbar_init(bar_empty(b), 1);
    }
    mbar_init(bar_done, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(s_tmem_slot, Cfg::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *reinterpret_cast<volatile uint32_t*>(gbase + Cfg::OFF_MISC);
  pdl_enter();

  if (warp == 0) {
    if (lane == 0 && l < L) {
      bool ok = true;
      int issued = 0;
      for (int st = s0; ok && st < s1; ++st, ++issued) {
        const int slot = issued % NST;
        if (!mbar_wait(bar_empty(slot), ((issued / NST) & 1) ^ 1, abort_flag, kDevTimeoutEmpty)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(bar_full(slot), Cfg::STAGE_BYTES);
        const uint32_t da = sbase + slot * Cfg::STAGE_BYTES;
        const uint32_t db = da + Cfg::A_BYTES;
        // runtime layer index into the map arrays (parameter space)
#pragma unroll
        for (int c = 0; c < DA / 64; ++c)
          tma_load_2d(da + c * kWgStageRows * 128, &maps.a[l], bar_full(slot), c * 64, st * kWgStageRows);
#pragma unroll
        for (int c = 0; c < DB / 64; ++c)
          tma_load_2d(db + c * kWgStageRows * 128, &maps.b[l], bar_full(slot), c * 64, st * kWgStageRows);
      }
      volatile int no_abort = 0;
      for (int b = 0; b < NST; ++b) {
        const int uses = issued > b ? (issued - b + NST - 1) / NST : 0;
        if (uses > 0) mbar_wait(bar_full(b), (uses - 1) & 1, &no_abort, kDevTimeoutFull);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    const bool issuer = (lane == 0);
    constexpr uint32_t idesc = make_idesc_f16(kTileM, DB, 1, 1);
    bool ok = true;
    int used = 0;
    for (int st = s0; ok && l < L && st < s1; ++st, ++used) {
      const int slot = used % NST;
      ok = __all_sync(0xffffffffu, mbar_wait(bar_full(slot), (used / NST) & 1, abort_flag, kDevTimeoutMma));
      if (!ok) break;
      tc_fence_after();
      if (issuer) {
        const uint32_t da = sbase + slot * Cfg::STAGE_BYTES;
        const uint32_t db = da + Cfg::A_BYTES;
#pragma unroll
        for (int mb = 0; mb < Cfg::MB; ++mb) {
          // A block mb: dW rows [128mb, 128mb+128) = two 64-column chunks of the stage
          const uint64_t a0 = make_sdesc(da + mb * 2 * kWgStageRows * 128, kWgStageRows * 128, 1024, 2);
          const uint64_t b0 = make_sdesc(db, kWgStageRows * 128, 1024, 2);
#pragma unroll
          for (int kk = 0; kk < kWgStageRows / 16; ++kk)
            umma_f16(tmem_base + mb * DB, a0 + ((kk * 16 * 128) >> 4), b0 + ((kk * 16 * 128) >> 4), idesc,
                     (st > s0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(bar_empty(slot));
      }
      __syncwarp();
    }
    if (issuer) umma_commit(bar_done);
    __syncwarp();
    {
      volatile int no_abort = 0;
      mbar_wait(bar_done, 0, &no_abort, kDevTimeoutMma);
    }
    __syncwarp();
  } else {
    // dump: thread = row (lane) of accumulator block mb -> dW_l row 128mb + lane
    const int q = warp & 3;
    const uint32_t row = q * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(q * 32) << 16;
    bool ok = __all_sync(0xffffffffu, mbar_wait(bar_done, 0, abort_flag, kDevTimeoutEpi));
    tc_fence_after();
    if (ok && l < L) {
      float* part = maps.partials + static_cast<size_t>(blockIdx.x) * DA * DB;
      const bool empty = s1 <= s0;  // no rows: the accumulators were never written
#pragma unroll 1
      for (int mb = 0; mb < Cfg::MB; ++mb) {
#pragma unroll 1
        for (int c = 0; c < DB; c += 16) {
          uint32_t r[16];
          tmem_ld_wait_x16(tmem_base + lane_off + mb * DB + c, r);
          float4* dst = reinterpret_cast<float4*>(part + static_cast<size_t>(mb * 128 + row) * DB + c);
#pragma unroll
          for (int v = 0; v < 4; ++v)
            dst[v] = empty ? make_float4(0.f, 0.f, 0.f, 0.f)
                           : make_float4(__uint_as_float(r[4 * v]), __uint_as_float(r[4 * v + 1]),
                                         __uint_as_float(r[4 * v + 2]), __uint_as_float(r[4 * v + 3]));
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, Cfg::TMEM_COLS);
  }
}

}  // namespace mlpk
