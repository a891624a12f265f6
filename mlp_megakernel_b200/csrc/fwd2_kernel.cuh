// CTA-pair (2-SM) variant of the fused softplus-MLP forward for sm_100a.
//
// Same pipeline as fwd_kernel.cuh (persistent CTAs, NS tile slots, TMEM
// accumulators double-buffered per slot, activations kept in TMEM, chunked
// epilogue -> MMA hand-off), but every GEMM is one tcgen05.mma with
// cta_group::2 and M = 256 covering a pair of 128-row tiles held by the two
// CTAs of a cluster (the two SMs of a TPC):
//
//  * each CTA stores HALF of every weight matrix (its N/2 output columns) in
//    shared memory -- half the weight footprint and half the per-SM B-operand
//    shared-memory traffic of the 1-SM kernel;
//  * only the leader CTA (cluster rank 0) issues UMMAs: one instruction per
//    256 rows instead of two, halving the MMA warp's issue work per row;
//  * each CTA keeps its own 128 rows of x, of the accumulators and of the
//    activations (TMEM), and runs its own epilogue and TMA stores.
//
// Cross-CTA hand-offs: both producers' TMA loads complete on the leader's
// x_full / w_full barriers (cta_group::2 loads, no multicast); the peer's
// epilogue warps arrive on the leader's chunk barriers through cluster
// addresses; the leader's commits arrive on the barrier of both CTAs
// (tcgen05.commit multicast).  All waits are bounded.
#pragma once
#include "fwd_kernel.cuh"

namespace mlpk {

template <class NetT, int NS, int EPW>
struct Fwd2Cfg {
  static constexpr int L = NetT::L;
  static constexpr int D0 = NetT::template D<0>();
  static constexpr int DL = NetT::template D<L>();
  static constexpr int H = NetT::template D<1>();
  static constexpr int HMAX = NetT::max_hidden_or_out();
  static constexpr int X_BYTES = align_up(tile_bytes(kTileM, D0), 1024);
  static constexpr int O_BYTES = align_up(tile_bytes(kTileM, DL), 1024);
  // weight halves: layer l holds K rows x N/2 columns
  template <int l>
  __host__ __device__ static constexpr int wh_off() { return NetT::template w_half_off<l>(); }
  static constexpr int W_TOTAL = NetT::template w_half_off<L>();
  static constexpr int OFF_X = W_TOTAL;
  static constexpr int OFF_O = OFF_X + NS * X_BYTES;
  static constexpr int OFF_BAR = OFF_O + NS * O_BYTES;
  static constexpr int NG = EPW / 4;
  static constexpr int SPC = (HMAX / NG) / 32 >= 4 ? 2 : 1;
  static constexpr int MAXCH = ((HMAX / NG + 31) / 32 + SPC - 1) / SPC;
  static constexpr int NUM_BARS = 6 * NS + NS * MAXCH + 2;
  static constexpr int OFF_MISC = OFF_BAR + 8 * NUM_BARS;
  static constexpr int SMEM_BYTES = OFF_MISC + 16 + 1024;
  static constexpr int SLOT_COLS = align_up(HMAX, 32);
  static constexpr int TMEM_COLS_RAW = 2 * NS * SLOT_COLS;
  static constexpr int TMEM_COLS = TMEM_COLS_RAW <= 128 ? 128 : TMEM_COLS_RAW <= 256 ? 256 : 512;
  static constexpr int THREADS = (2 + NS * EPW) * 32;
  static constexpr int W_BYTES_HALF = NetT::w_half_bytes_exact();
  static_assert(EPW % 4 == 0, "epilogue warps come in groups of 4");
  static_assert(L >= 2 && NetT::hidden_uniform(), "uniform hidden widths, >= 2 layers");
  static_assert(TMEM_COLS_RAW <= 512, "accumulators exceed TMEM");
  static_assert(SMEM_BYTES <= 232448, "shared memory budget exceeded");
};

template <class NetT, int NS, int EPW>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(Fwd2Cfg<NetT, NS, EPW>::THREADS, 1)
    mlp_fwd2_kernel(const __grid_constant__ FwdMaps<NetT::L> maps, int num_pairs) {
  using Cfg = Fwd2Cfg<NetT, NS, EPW>;
  constexpr int L = Cfg::L;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t sbase = (raw + 1023u) & ~1023u;  // identical offset in both CTAs
  uint8_t* gbase = smem_raw + (sbase - raw);

  const uint32_t rank = cluster_ctarank();
  const bool leader = (rank == 0);
  const uint32_t s_w = sbase;
  const uint32_t s_x = sbase + Cfg::OFF_X;
  const uint32_t s_o = sbase + Cfg::OFF_O;
  const uint32_t s_bar = sbase + Cfg::OFF_BAR;
  auto bar_x_full = [&](int s) { return s_bar + 8u * s; };       // leader: count 2 (+tx)
  auto bar_x_empty = [&](int s) { return s_bar + 8u * (NS + s); }; // both: commit multicast
  // one accumulator-full barrier per slot and TMEM buffer (job g -> buffer
  // g & 1, parity (g >> 1) & 1), as in mlp_fwd_kernel: a single barrier per slot
  // could complete twice before a slow epilogue warp polls it
  auto bar_acc_full = [&](int s, int b) { return s_bar + 8u * (2 * NS + 2 * s + b); };
  auto bar_out_ready = [&](int s) { return s_bar + 8u * (4 * NS + s); };
  auto bar_store_free = [&](int s) { return s_bar + 8u * (5 * NS + s); };
  auto bar_chunk = [&](int s, int c) { return s_bar + 8u * (6 * NS + s * Cfg::MAXCH + c); };
  const uint32_t bar_w_full = s_bar + 8u * (6 * NS + NS * Cfg::MAXCH);
  const uint32_t bar_mma_done = bar_w_full + 8u;
  const uint32_t s_tmem_slot = sbase + Cfg::OFF_MISC;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(gbase + Cfg::OFF_MISC + 4);
  // the leader's copy of a barrier, as a cluster address
  auto to_leader = [&](uint32_t bar) { return mapa_shared(bar, 0); };

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(bar_x_full(s), 2);
      mbar_init(bar_x_empty(s), 1);
      mbar_init(bar_acc_full(s, 0), 1);
      mbar_init(bar_acc_full(s, 1), 1);
      mbar_init(bar_out_ready(s), EPW);
      mbar_init(bar_store_free(s), 1);
      for (int c = 0; c < Cfg::MAXCH; ++c) mbar_init(bar_chunk(s, c), 2 * EPW);
    }
    mbar_init(bar_w_full, 2);
    mbar_init(bar_mma_done, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc_pair(s_tmem_slot, Cfg::TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();  // barriers of both CTAs initialised before any remote arrive
  tc_fence_after();
  const uint32_t tmem_base = *reinterpret_cast<volatile uint32_t*>(gbase + Cfg::OFF_MISC);

  uint32_t cid, ncl;
  asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(cid));
  asm volatile("mov.u32 %0, %%nclusterid.x;" : "=r"(ncl));
  // pair tile index of slot s in round i; this CTA holds rows (2*pt + rank)*128
  auto pair_of = [&](int i, int s) { return static_cast<int>(cid) + (i * NS + s) * static_cast<int>(ncl); };

  if (warp == 0) {
    // ------------------------------------------------------------ producer (both CTAs)
    if (lane == 0) {
      tma_prefetch_desc(&maps.x);
      tma_prefetch_desc(&maps.out);
      mbar_arrive_expect_tx_cluster(to_leader(bar_w_full), Cfg::W_BYTES_HALF);
      static_for<0, L>([&](auto lc) {
        constexpr int l = decltype(lc)::value;
        constexpr int K = NetT::template D<l>();
        constexpr int NH = NetT::template D<l + 1>() / 2;
        constexpr int C = chunk_elems(NH);
        constexpr int P = pitch_bytes(NH);
#pragma unroll
        for (int c = 0; c < NH / C; ++c)
          tma_load_2d_pair(s_w + Cfg::template wh_off<l>() + c * K * P, &maps.w[l],
                           to_leader(bar_w_full), static_cast<int>(rank) * NH + c * C, 0);
      });
      constexpr int C0 = chunk_elems(Cfg::D0);
      constexpr int P0 = pitch_bytes(Cfg::D0);
      bool ok = true;
      for (int i = 0; ok; ++i) {
#pragma unroll
        for (int s = 0; s < NS; ++s) {
          const int pt = pair_of(i, s);
          if (pt >= num_pairs) {
            ok = false;
            break;
          }
          if (!mbar_wait_cluster(bar_x_empty(s), (i & 1) ^ 1, abort_flag, kDevTimeoutEmpty)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx_cluster(to_leader(bar_x_full(s)), kTileM * Cfg::D0 * 2);
          const int row0 = (2 * pt + static_cast<int>(rank)) * kTileM;
#pragma unroll
          for (int c = 0; c < Cfg::D0 / C0; ++c)
            tma_load_2d_pair(s_x + s * Cfg::X_BYTES + c * kTileM * P0, &maps.x,
                             to_leader(bar_x_full(s)), c * C0, row0);
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (leader)
    const bool issuer = leader && (lane == 0);
    bool ok = true;
    if (leader) {
      ok = __all_sync(0xffffffffu, mbar_wait_cluster(bar_w_full, 0, abort_flag, kDevTimeoutMma));
      tc_fence_after();
      for (int i = 0; ok; ++i) {
        if (pair_of(i, 0) >= num_pairs) break;
        static_for<0, L>([&](auto lc) {
          constexpr int l = decltype(lc)::value;
          constexpr int K = NetT::template D<l>();
          constexpr int N = NetT::template D<l + 1>();
          constexpr uint32_t idesc = make_idesc_f16(2 * kTileM, N, 0, 1);
          const uint64_t bdesc0 = mnmajor_base_desc<K, N / 2>(s_w + Cfg::template wh_off<l>());
#pragma unroll
          for (int s = 0; s < NS; ++s) {
            if (!ok || pair_of(i, s) >= num_pairs) break;
            const uint32_t d_tmem = tmem_base + (2 * s + ((i * L + l) & 1)) * Cfg::SLOT_COLS;
            if constexpr (l == 0) {
              ok = __all_sync(0xffffffffu,
                              mbar_wait_cluster(bar_x_full(s), i & 1, abort_flag, kDevTimeoutMma));
              if (!ok) break;
              tc_fence_after();
              const uint64_t adesc0 = kmajor_base_desc<K>(s_x + s * Cfg::X_BYTES);
              if (issuer) {
#pragma unroll
                for (int k = 0; k < K / 16; ++k)
                  umma_f16_pair(d_tmem, adesc0 + (kmajor_koff<kTileM, K>(k) >> 4),
                                bdesc0 + (mnmajor_koff<N / 2>(k) >> 4), idesc, k > 0 ? 1u : 0u);
                umma_commit_pair(bar_x_empty(s), 0x3);
              }
              __syncwarp();
            } else {
              constexpr int NGRP = Cfg::NG;
              constexpr int SPC = Cfg::SPC;
              constexpr int NCH = K / (32 * NGRP * SPC);
              static_assert(NCH >= 1 && K % (32 * NGRP * SPC) == 0, "hidden width vs chunks");
              const uint32_t a_tmem = tmem_base + (2 * s + ((i * L + l - 1) & 1)) * Cfg::SLOT_COLS;
              const uint32_t par = (i * (L - 1) + l - 1) & 1;
#pragma unroll
              for (int j = 0; j < NCH; ++j) {
                ok = __all_sync(0xffffffffu,
                                mbar_wait_cluster(bar_chunk(s, j), par, abort_flag, kDevTimeoutMma));
                if (!ok) break;
                tc_fence_after();
                if (issuer) {
#pragma unroll
                  for (int js = 0; js < SPC; ++js) {
#pragma unroll
                    for (int g = 0; g < NGRP; ++g) {
#pragma unroll
                      for (int kk = 0; kk < 2; ++kk) {
                        const int k = 2 * ((j * SPC + js) * NGRP + g) + kk;
                        umma_f16_pair_ts(d_tmem, a_tmem + h_tmem_col(16 * k),
                                         bdesc0 + (mnmajor_koff<N / 2>(k) >> 4), idesc,
                                         (j == 0 && js == 0 && g == 0 && kk == 0) ? 0u : 1u);
                      }
                    }
                  }
                }
                __syncwarp();
              }
              if (!ok) break;
            }
            if (issuer) umma_commit_pair(bar_acc_full(s, (i * L + l) & 1), 0x3);
            __syncwarp();
          }
        });
      }
      if (issuer) umma_commit_pair(bar_mma_done, 0x3);
      __syncwarp();
    }
    // both CTAs: every UMMA writing this CTA's TMEM has completed
    if (lane == 0) {
      volatile int no_abort = 0;
      mbar_wait_cluster(bar_mma_done, 0, &no_abort, kDevTimeoutMma);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue (both CTAs)
    const int e = warp - 2;
    const int s = e / EPW;
    const int ew = e % EPW;
    const int q = warp & 3;
    const int grp = ew >> 2;
    const uint32_t row = q * 32 + lane;
    const uint32_t t_lane = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + 2 * s * Cfg::SLOT_COLS;
    const uint32_t obuf = s_o + s * Cfg::O_BYTES;
    const bool store_leader = (ew == 0 && lane == 0);
    const uint32_t chunk0_leader = to_leader(bar_chunk(s, 0));
    bool ok = true;
    constexpr int H = Cfg::H;
    constexpr int NCOL_O = Cfg::DL / Cfg::NG;
    for (int i = 0; ok; ++i) {
      const int pt = pair_of(i, s);
      if (pt >= num_pairs) break;
      const int row0 = (2 * pt + static_cast<int>(rank)) * kTileM;
#pragma unroll 1
      for (int l = 0; l < L - 1; ++l) {
        ok = __all_sync(0xffffffffu, mbar_wait_cluster(bar_acc_full(s, (i * L + l) & 1),
                                                       ((i * L + l) >> 1) & 1, abort_flag,
                                                       kDevTimeoutEpi));
        if (!ok) break;
        tc_fence_after();
        if (l == 0 && i > 0) {
          if (store_leader) {
            bulk_wait_group_read<0>();
            mbar_arrive(bar_store_free(s));
          }
          __syncwarp();
          ok = __all_sync(0xffffffffu,
                          mbar_wait(bar_store_free(s), (i - 1) & 1, abort_flag, kDevTimeoutEpi));
          if (!ok) break;
        }
        const uint32_t t_buf = t_lane + ((i * L + l) & 1) * Cfg::SLOT_COLS;
        hidden_job<H, Cfg::NG, Cfg::SPC, true>(t_buf, grp, chunk0_leader);
      }
      if (!ok) break;
      {
        constexpr int l = L - 1;
        ok = __all_sync(0xffffffffu, mbar_wait_cluster(bar_acc_full(s, (i * L + l) & 1),
                                                       ((i * L + l) >> 1) & 1, abort_flag,
                                                       kDevTimeoutEpi));
        if (!ok) break;
        tc_fence_after();
        const uint32_t t_buf = t_lane + ((i * L + l) & 1) * Cfg::SLOT_COLS;
        out_job<Cfg::DL, NCOL_O>(t_buf, obuf, row, grp * NCOL_O);
        fence_proxy_async_smem();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar_out_ready(s));
        if (store_leader) ok = mbar_wait(bar_out_ready(s), i & 1, abort_flag, kDevTimeoutEpi);
        ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
        if (store_leader && ok) {
          constexpr int C = chunk_elems(Cfg::DL);
          constexpr int P = pitch_bytes(Cfg::DL);
#pragma unroll
          for (int c = 0; c < Cfg::DL / C; ++c)
            tma_store_2d(&maps.out, obuf + c * kTileM * P, c * C, row0);
          bulk_commit_group();
        }
      }
    }
    if (store_leader) bulk_wait_group<0>();
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync();  // no CTA leaves while its peer may still signal its barriers
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, Cfg::TMEM_COLS);
  }
}

}  // namespace mlpk
