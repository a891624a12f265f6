// Persistent fused backward of the softplus MLP for sm_100a.
//
// For each 128-row tile (weights W_l are [d_l, d_{l+1}], h_0 = x, h_l the
// saved fp16 activations, g = dL/dout):
//
//   dz_L = g
//   for l = L-1 .. 0:
//     dW_l += h_l^T dz_{l+1}                 (wgrad, UMMA M=d_l, K = tile rows)
//     dh_l  = dz_{l+1} W_l^T                 (dgrad, UMMA M=128, K = d_{l+1})
//     dz_l  = dh_l * (1 - exp(-h_l))  (l>0)  (softplus' from the saved h)
//   dx = dh_0
//
// This is the fused data-gradient chain plus weight gradients of the
// reference's training path (math: mlp_fused.md:80-95, sigmoid-h multiply:
// mlp_fused.md:134-137) with a different reduction: instead of fp32 atomics
// (mlp_fused.md:97-112) or a cuBLAS fallback (mlp_fused.md:130-146), every CTA
// accumulates dW_l for ALL of its tiles in TMEM (split-K level 1) and dumps one
// fp32 partial per CTA; mlpk_reduce sums the partials in a fixed order (level
// 2), so weight gradients are bitwise deterministic.
//
// Roles: warp 0 = TMA producer (weights once, then per tile g, h_l, x with
// prefetch as buffers free up), warp 1 = TMEM owner + MMA issuer (one lane),
// warps 2..5 = epilogue (thread = tile row; sigmoid multiply in registers,
// dz written straight into the swizzled smem tile that the next layer's two
// UMMAs read as K-major A (dgrad) and MN-major B (wgrad)).
//
// Shared memory: all weights (read as K-major B = W^T for dgrad), one buffer
// per h_l, x, and one "G" buffer that holds g, then each dz, then dx staging.
// TMEM: one fp32 accumulator per dW_l plus one dgrad accumulator.
#pragma once
#include "fwd_kernel.cuh"

namespace mlpk {

template <int L>
struct alignas(64) BwdMaps {
  CUtensorMap x;               // [M, d0] fp16 load
  CUtensorMap g;               // [M, dL] fp16 load (grad_out)
  CUtensorMap dx;              // [M, d0] fp16 store
  CUtensorMap h[L > 1 ? L - 1 : 1];  // h_1..h_{L-1}: [M, d_l] fp16 loads
  CUtensorMap w[L];            // [d_l, d_{l+1}] fp16 loads
  float* partials;             // [gridDim.x][sum_l d_l*d_{l+1}] fp32
};

template <class NetT>
struct BwdCfg {
  static constexpr int L = NetT::L;
  static constexpr int D0 = NetT::template D<0>();
  static constexpr int DL = NetT::template D<L>();
  static constexpr int H = NetT::template D<1>();
  static constexpr int DMAX = D0 > NetT::max_hidden_or_out() ? D0 : NetT::max_hidden_or_out();
  // Weight-gradient plan of layer l: UMMA M must be 64 or 128 and the
  // accumulator is read with the M = 128 layout (TMEM lane = row), so the GEMM
  // runs in the orientation with the wider M (dW_l = h_l^T dz, or, when
  // d_l < 64, dW_l^T = dz^T h_l), and an M of 64 is padded to 128 with a zeroed
  // shared-memory chunk (rows 64..127 of that accumulator stay zero).
  __host__ __device__ static constexpr bool wg_trans(int l) { return NetT::dim(l) < 64; }
  __host__ __device__ static constexpr int wg_m(int l) {
    return wg_trans(l) ? NetT::dim(l + 1) : NetT::dim(l);
  }
  __host__ __device__ static constexpr int wg_n(int l) {
    return wg_trans(l) ? NetT::dim(l) : NetT::dim(l + 1);
  }
  __host__ __device__ static constexpr bool wg_pad(int l) { return wg_m(l) < 128; }
  __host__ __device__ static constexpr bool any_pad() {
    for (int l = 0; l < L; ++l)
      if (wg_pad(l)) return true;
    return false;
  }
  __host__ __device__ static constexpr bool plans_ok() {
    for (int l = 0; l < L; ++l) {
      if (wg_m(l) != 64 && wg_m(l) != 128) return false;
      if (wg_n(l) % 16 != 0 || wg_n(l) < 16 || wg_n(l) > 256) return false;
    }
    return true;
  }
  // TMEM: dW_l (wg_n(l) columns each), then the dgrad accumulator
  __host__ __device__ static constexpr int dw_col(int l) {
    int c = 0;
    for (int i = 0; i < l; ++i) c += wg_n(i);
    return c;
  }
  static constexpr int TILE_BYTES = align_up(tile_bytes(kTileM, DMAX), 1024);
  static constexpr int W_TOTAL = NetT::w_total();
  static constexpr int OFF_G = W_TOTAL;
  static constexpr int OFF_X = OFF_G + TILE_BYTES;
  static constexpr int OFF_H = OFF_X + TILE_BYTES;                 // h_1 .. h_{L-1}
  static constexpr int OFF_ZERO = OFF_H + (L - 1) * TILE_BYTES;    // zero chunk (M padding)
  static constexpr int ZERO_BYTES = any_pad() ? 16384 : 0;         // 128 rows x 128 B
  static constexpr int OFF_BAR = OFF_ZERO + ZERO_BYTES;
  // barriers: w_full, g_full, g_empty, x_full, x_empty, acc_full, dz_full,
  //           acc_free, out_ready, mma_done, h_full[L-1], h_empty[L-1]
  static constexpr int NUM_BARS = 10 + 2 * (L - 1);
  static constexpr int OFF_MISC = OFF_BAR + 8 * NUM_BARS;
  static constexpr int SMEM_BYTES = OFF_MISC + 16 + 1024;
  static constexpr int ACC_COL = dw_col(L);
  static constexpr int TMEM_COLS_RAW = ACC_COL + align_up(DMAX, 32);
  static constexpr int TMEM_COLS = TMEM_COLS_RAW <= 128 ? 128 : TMEM_COLS_RAW <= 256 ? 256 : 512;
  static constexpr int PARTIAL_FLOATS = [] {
    int n = 0;
    for (int i = 0; i < L; ++i) n += NetT::dim(i) * NetT::dim(i + 1);
    return n;
  }();
  static constexpr int THREADS = 6 * 32;
  static_assert(plans_ok(), "weight-gradient GEMM shapes not supported");
  static_assert(NetT::hidden_uniform(), "all hidden layers must have the same width");
  static_assert(TMEM_COLS_RAW <= 512, "dW + dgrad accumulators exceed TMEM");
  static_assert(SMEM_BYTES <= 232448, "shared memory budget exceeded");
};

// this thread's row of an fp16 operand tile of extent N: 8 values at column c
template <int N>
__device__ __forceinline__ uint4 ld_tile_row8(uint32_t tile_base, uint32_t row, int c) {
  constexpr int C = chunk_elems(N);
  constexpr int P = pitch_bytes(N);
  uint4 v;
  asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(tile_base + (c / C) * (kTileM * P) + swz_off<P>(row, (c % C) / 8)));
  return v;
}
template <int N>
__device__ __forceinline__ void st_tile_row8(uint32_t tile_base, uint32_t row, int c, uint32_t a,
                                             uint32_t b, uint32_t d, uint32_t e) {
  constexpr int C = chunk_elems(N);
  constexpr int P = pitch_bytes(N);
  st_shared_v4(tile_base + (c / C) * (kTileM * P) + swz_off<P>(row, (c % C) / 8), a, b, d, e);
}

__device__ __forceinline__ float2 half2_to_float2(uint32_t v) {
  __half2 h = *reinterpret_cast<__half2*>(&v);
  return __half22float2(h);
}

// dz = dh * (1 - e^{-h}) for a pair (packed f32x2 math; softplus' via h).
__device__ __forceinline__ float2 dsoftplus_mul_x2(float2 dh, float2 h) {
  const float2 s = __fmul2_rn(h, make_float2(-kLog2e, -kLog2e));
  const float2 e = make_float2(ex2_approx(s.x), ex2_approx(s.y));  // e^{-h}, h >= 0
  return __ffma2_rn(make_float2(-e.x, -e.y), dh, dh);              // dh - dh*e
}

template <class NetT>
__global__ void __launch_bounds__(BwdCfg<NetT>::THREADS, 1)
    mlp_bwd_kernel(const __grid_constant__ BwdMaps<NetT::L> maps, int num_tiles) {
  using Cfg = BwdCfg<NetT>;
  constexpr int L = Cfg::L;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t sbase = (raw + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (sbase - raw);

  const uint32_t s_w = sbase;
  const uint32_t s_g = sbase + Cfg::OFF_G;
  const uint32_t s_xb = sbase + Cfg::OFF_X;
  auto s_h = [&](int l) { return sbase + Cfg::OFF_H + (l - 1) * Cfg::TILE_BYTES; };  // l >= 1
  const uint32_t s_bar = sbase + Cfg::OFF_BAR;
  const uint32_t bar_w_full = s_bar;
  const uint32_t bar_g_full = s_bar + 8;
  const uint32_t bar_g_empty = s_bar + 16;
  const uint32_t bar_x_full = s_bar + 24;
  const uint32_t bar_x_empty = s_bar + 32;
  const uint32_t bar_acc_full = s_bar + 40;
  const uint32_t bar_dz_full = s_bar + 48;
  const uint32_t bar_acc_free = s_bar + 56;
  const uint32_t bar_out_ready = s_bar + 64;
  const uint32_t bar_mma_done = s_bar + 72;
  auto bar_h_full = [&](int l) { return s_bar + 80 + 8u * (l - 1); };
  auto bar_h_empty = [&](int l) { return s_bar + 80 + 8u * (L - 1) + 8u * (l - 1); };
  const uint32_t s_tmem_slot = sbase + Cfg::OFF_MISC;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(gbase + Cfg::OFF_MISC + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    mbar_init(bar_w_full, 1);
    mbar_init(bar_g_full, 1);
    mbar_init(bar_g_empty, 1);
    mbar_init(bar_x_full, 1);
    mbar_init(bar_x_empty, 1);
    mbar_init(bar_acc_full, 1);
    mbar_init(bar_dz_full, 4);
    mbar_init(bar_acc_free, 4);
    mbar_init(bar_out_ready, 4);
    mbar_init(bar_mma_done, 1);
    for (int l = 1; l < L; ++l) {
      mbar_init(bar_h_full(l), 1);
      mbar_init(bar_h_empty(l), 4);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(s_tmem_slot, Cfg::TMEM_COLS);
    tmem_relinquish();
  }
  if constexpr (Cfg::ZERO_BYTES > 0) {  // zero chunk that pads a 64-wide wgrad M to 128
    for (int i = threadIdx.x; i < Cfg::ZERO_BYTES / 16; i += blockDim.x)
      st_shared_v4(sbase + Cfg::OFF_ZERO + 16 * i, 0u, 0u, 0u, 0u);
    fence_proxy_async_smem();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *reinterpret_cast<volatile uint32_t*>(gbase + Cfg::OFF_MISC);
  const int G = gridDim.x;
  auto tile_of = [&](int i) { return static_cast<int>(blockIdx.x) + i * G; };

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      mbar_arrive_expect_tx(bar_w_full, NetT::w_bytes_exact());
      static_for<0, L>([&](auto lc) {
        constexpr int l = decltype(lc)::value;
        constexpr int K = NetT::template D<l>();
        constexpr int N = NetT::template D<l + 1>();
        constexpr int C = chunk_elems(N);
        constexpr int P = pitch_bytes(N);
#pragma unroll
        for (int c = 0; c < N / C; ++c)
          tma_load_2d(s_w + NetT::template w_off<l>() + c * K * P, &maps.w[l], bar_w_full, c * C, 0);
      });
      auto load_tile = [&](const CUtensorMap* map, uint32_t dst, uint32_t bar, int d, int t) {
        const int C = d < 64 ? d : 64;
        const int P = 2 * C;
        mbar_arrive_expect_tx(bar, kTileM * d * 2);
        for (int c = 0; c < d / C; ++c) tma_load_2d(dst + c * kTileM * P, map, bar, c * C, t * kTileM);
      };
      bool ok = true;
      for (int i = 0; ok; ++i) {
        const int t = tile_of(i);
        if (t >= num_tiles) break;
        const uint32_t par = (i & 1) ^ 1;
        // in the order the buffers free up: h_{L-1} .. h_1, x, g
        static_for<1, L>([&](auto lc) {
          constexpr int l = L - decltype(lc)::value;  // L-1 .. 1
          if (!ok) return;
          ok = mbar_wait(bar_h_empty(l), par, abort_flag, kDevTimeoutEmpty);
          if (ok) load_tile(&maps.h[l - 1], s_h(l), bar_h_full(l), NetT::template D<l>(), t);
        });
        if (ok) ok = mbar_wait(bar_x_empty, par, abort_flag, kDevTimeoutEmpty);
        if (ok) load_tile(&maps.x, s_xb, bar_x_full, Cfg::D0, t);
        if (ok) ok = mbar_wait(bar_g_empty, par, abort_flag, kDevTimeoutEmpty);
        if (ok) load_tile(&maps.g, s_g, bar_g_full, Cfg::DL, t);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    const bool issuer = (lane == 0);
    bool ok = __all_sync(0xffffffffu, mbar_wait(bar_w_full, 0, abort_flag, kDevTimeoutMma));
    tc_fence_after();
    const uint32_t acc = tmem_base + Cfg::ACC_COL;
    for (int i = 0; ok; ++i) {
      if (tile_of(i) >= num_tiles) break;
      static_for<0, L>([&](auto lc) {
        constexpr int l = L - 1 - decltype(lc)::value;  // L-1 .. 0
        constexpr int DI = NetT::template D<l>();      // d_l
        constexpr int DO = NetT::template D<l + 1>();  // d_{l+1}
        if (!ok) return;
        // G holds dz_{l+1}: g for the last layer (TMA), else written by the epilogue
        if constexpr (l == L - 1) {
          ok = __all_sync(0xffffffffu, mbar_wait(bar_g_full, i & 1, abort_flag, kDevTimeoutMma)) &&
               __all_sync(0xffffffffu,
                          mbar_wait(bar_acc_free, (i & 1) ^ 1, abort_flag, kDevTimeoutMma));
        } else {
          ok = __all_sync(0xffffffffu, mbar_wait(bar_dz_full, (i * (L - 1) + (L - 2 - l)) & 1,
                                                 abort_flag, kDevTimeoutMma));
        }
        if (!ok) return;
        // A operand of the wgrad: h_l (x for l == 0)
        if constexpr (l == 0) {
          ok = __all_sync(0xffffffffu, mbar_wait(bar_x_full, i & 1, abort_flag, kDevTimeoutMma));
        } else {
          ok = __all_sync(0xffffffffu, mbar_wait(bar_h_full(l), i & 1, abort_flag, kDevTimeoutMma));
        }
        if (!ok) return;
        tc_fence_after();
        const uint32_t a_h = (l == 0) ? s_xb : s_h(l);
        if (issuer) {
          // wgrad over the 128 tile rows (K): dW_l += h_l^T dz (A = h_l, B = dz) or,
          // transposed, dW_l^T += dz^T h_l (A = dz, B = h_l); both operands
          // MN-major from shared memory; a 64-wide A is padded to M = 128 by
          // pointing its second 64-column chunk (LBO) at the zero chunk.
          {
            constexpr bool TR = Cfg::wg_trans(l);
            constexpr int MW = Cfg::wg_m(l);
            constexpr int NW = Cfg::wg_n(l);
            constexpr uint32_t idesc_w = make_idesc_f16(kTileM, NW, 1, 1);
            const uint32_t a_base = TR ? s_g : a_h;
            const uint32_t b_base = TR ? a_h : s_g;
            constexpr int PA = pitch_bytes(MW);
            const uint32_t lbo = (MW < 128) ? (sbase + Cfg::OFF_ZERO - a_base) : kTileM * PA;
            const uint64_t aw0 = make_sdesc(a_base, lbo, 8 * PA, umma_layout_code(PA));
            const uint64_t bw0 = mnmajor_base_desc<kTileM, NW>(b_base);
            const uint32_t dw = tmem_base + Cfg::dw_col(l);
#pragma unroll
            for (int k = 0; k < kTileM / 16; ++k)
              umma_f16(dw, aw0 + (mnmajor_koff<MW>(k) >> 4), bw0 + (mnmajor_koff<NW>(k) >> 4),
                       idesc_w, (i > 0 || k > 0) ? 1u : 0u);
          }
          // dgrad: dh_l[128 x d_l] = dz W_l^T: A = dz (K-major, K = d_{l+1}),
          // B = W_l as stored ([d_l rows][d_{l+1}] = K-major W_l^T)
          constexpr uint32_t idesc_d = make_idesc_f16(kTileM, DI, 0, 0);
          const uint64_t ad0 = kmajor_base_desc<DO>(s_g);
          const uint64_t bd0 = kmajor_base_desc<DO>(s_w + NetT::template w_off<l>());
#pragma unroll
          for (int k = 0; k < DO / 16; ++k)
            umma_f16(acc, ad0 + (kmajor_koff<kTileM, DO>(k) >> 4),
                     bd0 + (kmajor_koff<DI, DO>(k) >> 4), idesc_d, k > 0 ? 1u : 0u);
          umma_commit(bar_acc_full);
          if constexpr (l == 0) umma_commit(bar_x_empty);
        }
        __syncwarp();
      });
    }
    if (issuer) umma_commit(bar_mma_done);
    __syncwarp();
    {
      volatile int no_abort = 0;
      mbar_wait(bar_mma_done, 0, &no_abort, kDevTimeoutMma);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;
    const uint32_t row = q * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(q * 32) << 16;
    const uint32_t acc = tmem_base + lane_off + Cfg::ACC_COL;
    const bool store_leader = (warp == 2 && lane == 0);
    bool ok = true;
    for (int i = 0; ok; ++i) {
      const int t = tile_of(i);
      if (t >= num_tiles) break;
      static_for<0, L>([&](auto lc) {
        constexpr int l = L - 1 - decltype(lc)::value;  // dgrad result dh_l
        constexpr int DI = NetT::template D<l>();
        if (!ok) return;
        ok = __all_sync(0xffffffffu,
                        mbar_wait(bar_acc_full, (i * L + (L - 1 - l)) & 1, abort_flag, kDevTimeoutEpi));
        if (!ok) return;
        tc_fence_after();
        if constexpr (l > 0) {
          // dz_l = dh_l * softplus'(z_l) = dh_l * (1 - e^{-h_l}) -> G (fp16)
          const uint32_t hb = s_h(l);
#pragma unroll 1
          for (int c = 0; c < DI; c += 32) {
            uint32_t r[32];
            tmem_ld_wait_x32(acc + c, r);
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              const uint4 hv = ld_tile_row8<DI>(hb, row, c + 8 * u);
              const uint32_t hw[4] = {hv.x, hv.y, hv.z, hv.w};
              uint32_t o[4];
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                const float2 dz = dsoftplus_mul_x2(
                    make_float2(__uint_as_float(r[8 * u + 2 * j]), __uint_as_float(r[8 * u + 2 * j + 1])),
                    half2_to_float2(hw[j]));
                o[j] = pack_half2(dz.x, dz.y);
              }
              st_tile_row8<DI>(s_g, row, c + 8 * u, o[0], o[1], o[2], o[3]);
            }
          }
          fence_proxy_async_smem();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) {
            mbar_arrive(bar_dz_full);
            mbar_arrive(bar_h_empty(l));
          }
        } else {
          // dx = dh_0 -> fp16 staged in G -> TMA store
#pragma unroll 1
          for (int c = 0; c < DI; c += 32) {
            uint32_t r[32];
            tmem_ld_wait_x32(acc + c, r);
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              uint32_t o[4];
              pack_cols<4, false>(r + 8 * u, o);
              st_tile_row8<DI>(s_g, row, c + 8 * u, o[0], o[1], o[2], o[3]);
            }
          }
          fence_proxy_async_smem();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) {
            mbar_arrive(bar_acc_free);
            mbar_arrive(bar_out_ready);
          }
          if (store_leader) {
            ok = mbar_wait(bar_out_ready, i & 1, abort_flag, kDevTimeoutEpi);
            if (ok) {
              constexpr int C = chunk_elems(DI);
              constexpr int P = pitch_bytes(DI);
#pragma unroll
              for (int cc = 0; cc < DI / C; ++cc)
                tma_store_2d(&maps.dx, s_g + cc * kTileM * P, cc * C, t * kTileM);
              bulk_commit_group();
              bulk_wait_group_read<0>();
              mbar_arrive(bar_g_empty);  // G may take the next tile's g
            }
          }
          ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
        }
      });
    }
    // dump this CTA's dW partials: lane (row of dW_l) x d_{l+1} fp32
    if (ok) {
      ok = __all_sync(0xffffffffu, mbar_wait(bar_mma_done, 0, abort_flag, kDevTimeoutEpi));
      tc_fence_after();
    }
    if (ok) {
      float* part = maps.partials + static_cast<size_t>(blockIdx.x) * Cfg::PARTIAL_FLOATS;
      int off = 0;
      static_for<0, L>([&](auto lc) {
        constexpr int l = decltype(lc)::value;
        constexpr int DO = NetT::template D<l + 1>();
        constexpr bool TR = Cfg::wg_trans(l);
        constexpr int MW = Cfg::wg_m(l);
        constexpr int NW = Cfg::wg_n(l);
        const uint32_t dw = tmem_base + lane_off + Cfg::dw_col(l);
        // lane `row` of the accumulator: row of dW_l, or (transposed) column
        if (row < static_cast<uint32_t>(MW)) {
#pragma unroll 1
          for (int c = 0; c < NW; c += 16) {
            uint32_t r[16];
            tmem_ld_wait_x16(dw + c, r);
            if constexpr (!TR) {
              float4* dst = reinterpret_cast<float4*>(part + off + row * DO + c);
#pragma unroll
              for (int v = 0; v < 4; ++v)
                dst[v] = make_float4(__uint_as_float(r[4 * v]), __uint_as_float(r[4 * v + 1]),
                                     __uint_as_float(r[4 * v + 2]), __uint_as_float(r[4 * v + 3]));
            } else {
#pragma unroll
              for (int v = 0; v < 16; ++v) part[off + (c + v) * DO + row] = __uint_as_float(r[v]);
            }
          }
        } else {
          // lanes past M still take part in the warp-wide TMEM loads
#pragma unroll 1
          for (int c = 0; c < NW; c += 16) {
            uint32_t r[16];
            tmem_ld_wait_x16(dw + c, r);
          }
        }
        off += NetT::dim(l) * DO;
      });
    }
    if (store_leader) bulk_wait_group<0>();
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, Cfg::TMEM_COLS);
  }
}

// Level-2 reduction of the per-CTA partials: a block covers kReduceElems
// elements with kReduceSlices threads each; slice s sums partials p = s,
// s + kReduceSlices, ... in increasing p, and the slices are added in slice
// order.  The order is fixed, so dW is bitwise reproducible.  blockIdx.y
// selects an independent group (nparts partials of nfloats each, written to
// dw + y * nfloats), e.g. one group per layer of the split-K wgrad kernel.
constexpr int kReduceElems = 64;
constexpr int kReduceSlices = 4;

__global__ void __launch_bounds__(kReduceElems * kReduceSlices)
    mlp_reduce_kernel(const float* __restrict__ partials, int nparts, int nfloats,
                      float* __restrict__ dw) {
  __shared__ float red[kReduceSlices][kReduceElems];
  partials += static_cast<size_t>(blockIdx.y) * nparts * nfloats;
  dw += static_cast<size_t>(blockIdx.y) * nfloats;
  const int le = threadIdx.x % kReduceElems, sl = threadIdx.x / kReduceElems;
  const int e = blockIdx.x * kReduceElems + le;
  float acc = 0.0f;
  if (e < nfloats)
    for (int p = sl; p < nparts; p += kReduceSlices)
      acc += partials[static_cast<size_t>(p) * nfloats + e];
  red[sl][le] = acc;
  __syncthreads();
  if (sl == 0 && e < nfloats) {
    float t = red[0][le];
#pragma unroll
    for (int k = 1; k < kReduceSlices; ++k) t += red[k][le];
    dw[e] = t;
  }
}

}  // namespace mlpk
