// Persistent, warp-specialised fused softplus-MLP forward for sm_100a.
//
// out = softplus(...softplus(x @ W_0)...) @ W_{L-1}   (weights [in, out])
//
// This replaces the reference's Triton megakernel `_fused_mlp_recompute`
// (kernel.py:60-123) and its launch wrapper (kernel.py:130-156); the 5-layer
// chain is README.md:9.  Design (not a translation of the Triton loop nest):
//
//  * One CTA per SM (persistent).  Row tiles of 128 rows are assigned
//    round-robin: CTA b owns tiles b, b+G, b+2G, ...; the tiles are processed
//    NS at a time ("slots"), so the tensor core runs layer l of one slot while
//    the epilogue warps run the activation of another slot.
//  * warp 0 (one lane): TMA producer.  Loads every layer's fp16 weights into
//    shared memory ONCE per CTA, then streams x tiles into an NS-deep ring.
//  * warp 1: allocates TMEM; one lane issues tcgen05.mma (M=128, N=d_{l+1},
//    K=16 steps) for every layer of every tile; fp32 accumulators live in TMEM
//    (one accumulator region per slot, reused by all layers of that slot).
//  * warps 2..2+NEW-1: epilogue.  tcgen05.ld the accumulator (warp w owns TMEM
//    lanes 32*(w%4)..+31 = tile rows), softplus in fp32 registers, cast to fp16
//    and st.shared straight into the next layer's K-major, swizzled A operand;
//    for the last layer the fp16 result is staged in the same buffer and
//    written by TMA stores (OOB rows of the last tile are clipped by TMA).
//  * No activation touches HBM: HBM traffic is x in, out out (plus weights once
//    per CTA from L2).
//  * Hand-offs are mbarriers; all waits are bounded (ptx.cuh).
#pragma once
#include "layout.cuh"
#include "ptx.cuh"
#include "softplus.cuh"

namespace mlpk {

constexpr int kTileM = 128;

template <int... Ds>
struct Net {
  static constexpr int L = static_cast<int>(sizeof...(Ds)) - 1;
  template <int I>
  __host__ __device__ static constexpr int D() {
    constexpr int a[] = {Ds...};
    return a[I];
  }
  __host__ __device__ static constexpr int max_hidden_or_out() {
    constexpr int a[] = {Ds...};
    int m = 0;
    for (int i = 1; i < static_cast<int>(sizeof...(Ds)); ++i) m = a[i] > m ? a[i] : m;
    return m;
  }
  // Byte offset of W_l inside the weight region (each matrix 1024-aligned).
  template <int l>
  __host__ __device__ static constexpr int w_off() {
    constexpr int a[] = {Ds...};
    int o = 0;
    for (int i = 0; i < l; ++i) o += align_up(tile_bytes(a[i], a[i + 1]), 1024);
    return o;
  }
  __host__ __device__ static constexpr int w_total() { return w_off<L>(); }
  __host__ __device__ static constexpr int w_bytes_exact() {
    constexpr int a[] = {Ds...};
    int o = 0;
    for (int i = 0; i < L; ++i) o += tile_bytes(a[i], a[i + 1]);
    return o;
  }
};

template <int L>
struct alignas(64) FwdMaps {
  CUtensorMap x;       // [M, d0] fp16, box {chunk(d0), 128}
  CUtensorMap out;     // [M, dL] fp16, box {chunk(dL), 128}
  CUtensorMap w[L];    // [d_l, d_{l+1}] fp16, box {chunk(d_{l+1}), d_l}
};

template <int I, int N, class F>
__host__ __device__ __forceinline__ void static_for(F&& f) {
  if constexpr (I < N) {
    f(std::integral_constant<int, I>{});
    static_for<I + 1, N>(f);
  }
}

template <class NetT, int NS, int NEW>
struct FwdCfg {
  static constexpr int L = NetT::L;
  static constexpr int D0 = NetT::template D<0>();
  static constexpr int DL = NetT::template D<L>();
  static constexpr int HMAX = NetT::max_hidden_or_out();
  static constexpr int X_BYTES = align_up(tile_bytes(kTileM, D0), 1024);
  static constexpr int H_BYTES = align_up(tile_bytes(kTileM, HMAX), 1024);
  static constexpr int W_TOTAL = NetT::w_total();
  static constexpr int OFF_X = W_TOTAL;
  static constexpr int OFF_H = OFF_X + NS * X_BYTES;
  static constexpr int OFF_BAR = OFF_H + NS * H_BYTES;
  static constexpr int NUM_BARS = 7 * NS + 2;
  static constexpr int OFF_MISC = OFF_BAR + 8 * NUM_BARS;
  static constexpr int SMEM_BYTES = OFF_MISC + 16 + 1024;  // + alignment slack
  static constexpr int SLOT_COLS = align_up(HMAX, 32);
  static constexpr int TMEM_COLS_RAW = NS * SLOT_COLS;
  static constexpr int TMEM_COLS = TMEM_COLS_RAW <= 32    ? 32
                                   : TMEM_COLS_RAW <= 64  ? 64
                                   : TMEM_COLS_RAW <= 128 ? 128
                                   : TMEM_COLS_RAW <= 256 ? 256
                                                          : 512;
  static constexpr int THREADS = (2 + NEW) * 32;
  static constexpr int NG = NEW / 4;  // column groups of the epilogue
  static_assert(NEW % 4 == 0, "epilogue warps come in groups of 4 (one per TMEM lane quarter)");
  static_assert(TMEM_COLS_RAW <= 512, "accumulators exceed TMEM");
  static_assert(SMEM_BYTES <= 232448, "shared memory budget exceeded");
};

// Load NCOL consecutive fp32 accumulator columns of this thread's TMEM lane
// (load and wait in one statement, see ptx.cuh).
template <int NCOL>
__device__ __forceinline__ void tmem_load_cols(uint32_t taddr, float (&v)[NCOL]) {
  static_assert(NCOL == 8 || NCOL == 16 || NCOL == 32 || NCOL == 64, "unsupported width");
  uint32_t r[NCOL];
  if constexpr (NCOL == 8) tmem_ld_wait_x8(taddr, r);
  if constexpr (NCOL == 16) tmem_ld_wait_x16(taddr, r);
  if constexpr (NCOL == 32) tmem_ld_wait_x32(taddr, r);
  if constexpr (NCOL == 64) tmem_ld_wait_x64(taddr, r);
#pragma unroll
  for (int i = 0; i < NCOL; ++i) v[i] = __uint_as_float(r[i]);
}

// Write NCOL fp16 values (columns col0..col0+NCOL-1 of row `row`) into an
// operand tile of extent N stored as swizzled chunks.
template <int N, int NCOL, bool ACT>
__device__ __forceinline__ void store_row_chunk(uint32_t tile_base, uint32_t row, int col0,
                                                const float (&v)[NCOL]) {
  constexpr int C = chunk_elems(N);
  constexpr int P = pitch_bytes(N);
#pragma unroll
  for (int u = 0; u < NCOL / 8; ++u) {
    const int col = col0 + 8 * u;
    uint32_t w[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float a = v[8 * u + 2 * j], b = v[8 * u + 2 * j + 1];
      if constexpr (ACT) {
        a = softplus_f32(a);
        b = softplus_f32(b);
      }
      w[j] = pack_half2(a, b);
    }
    const uint32_t addr =
        tile_base + (col / C) * (kTileM * P) + swz_off<P>(row, (col % C) / 8);
    st_shared_v4(addr, w[0], w[1], w[2], w[3]);
  }
}

template <class NetT, int NS, int NEW>
__global__ void __launch_bounds__(FwdCfg<NetT, NS, NEW>::THREADS, 1)
    mlp_fwd_kernel(const __grid_constant__ FwdMaps<NetT::L> maps, int num_tiles) {
  using Cfg = FwdCfg<NetT, NS, NEW>;
  constexpr int L = Cfg::L;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t sbase = (raw + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (sbase - raw);

  const uint32_t s_w = sbase;
  const uint32_t s_x = sbase + Cfg::OFF_X;
  const uint32_t s_h = sbase + Cfg::OFF_H;
  const uint32_t s_bar = sbase + Cfg::OFF_BAR;
  auto bar_x_full = [&](int s) { return s_bar + 8u * s; };
  auto bar_x_empty = [&](int s) { return s_bar + 8u * (NS + s); };
  auto bar_acc_full = [&](int s) { return s_bar + 8u * (2 * NS + s); };
  auto bar_h_full = [&](int s) { return s_bar + 8u * (3 * NS + s); };
  auto bar_acc_empty = [&](int s) { return s_bar + 8u * (4 * NS + s); };
  auto bar_out_ready = [&](int s) { return s_bar + 8u * (5 * NS + s); };
  auto bar_store_free = [&](int s) { return s_bar + 8u * (6 * NS + s); };
  const uint32_t bar_w_full = s_bar + 8u * (7 * NS);
  const uint32_t bar_mma_done = s_bar + 8u * (7 * NS + 1);
  const uint32_t s_tmem_slot = sbase + Cfg::OFF_MISC;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(gbase + Cfg::OFF_MISC + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(bar_x_full(s), 1);
      mbar_init(bar_x_empty(s), 1);
      mbar_init(bar_acc_full(s), 1);
      mbar_init(bar_h_full(s), NEW);
      mbar_init(bar_acc_empty(s), NEW);
      mbar_init(bar_out_ready(s), NEW);
      mbar_init(bar_store_free(s), 1);
    }
    mbar_init(bar_w_full, 1);
    mbar_init(bar_mma_done, 1);
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

  const int G = gridDim.x;
  auto tile_of = [&](int p, int s) { return static_cast<int>(blockIdx.x) + (p * NS + s) * G; };

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      tma_prefetch_desc(&maps.x);
      tma_prefetch_desc(&maps.out);
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
      constexpr int C0 = chunk_elems(Cfg::D0);
      constexpr int P0 = pitch_bytes(Cfg::D0);
      bool ok = true;
      int issued[NS];
#pragma unroll
      for (int s = 0; s < NS; ++s) issued[s] = 0;
      for (int p = 0; ok; ++p) {
#pragma unroll
        for (int s = 0; s < NS; ++s) {
          const int t = tile_of(p, s);
          if (t >= num_tiles) {
            ok = false;
            break;
          }
          if (!mbar_wait(bar_x_empty(s), (p & 1) ^ 1, abort_flag, kDevTimeoutEmpty)) {
            ok = false;
            break;
          }
          ++issued[s];
          mbar_arrive_expect_tx(bar_x_full(s), kTileM * Cfg::D0 * 2);
#pragma unroll
          for (int c = 0; c < Cfg::D0 / C0; ++c)
            tma_load_2d(s_x + s * Cfg::X_BYTES + c * kTileM * P0, &maps.x, bar_x_full(s), c * C0,
                        t * kTileM);
        }
      }
      // Drain: never leave the CTA with a TMA load still writing shared memory.
      volatile int no_abort = 0;
      mbar_wait(bar_w_full, 0, &no_abort, kDevTimeoutFull);
#pragma unroll
      for (int s = 0; s < NS; ++s)
        if (issued[s] > 0) mbar_wait(bar_x_full(s), (issued[s] - 1) & 1, &no_abort, kDevTimeoutFull);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      bool ok = mbar_wait(bar_w_full, 0, abort_flag, kDevTimeoutMma);
      tc_fence_after();
      for (int p = 0; ok; ++p) {
        if (tile_of(p, 0) >= num_tiles) break;
        static_for<0, L>([&](auto lc) {
          constexpr int l = decltype(lc)::value;
          constexpr int K = NetT::template D<l>();
          constexpr int N = NetT::template D<l + 1>();
          constexpr uint32_t idesc = make_idesc_f16(kTileM, N, 0, 1);
#pragma unroll
          for (int s = 0; s < NS; ++s) {
            if (!ok || tile_of(p, s) >= num_tiles) break;
            if constexpr (l == 0) {
              ok = mbar_wait(bar_x_full(s), p & 1, abort_flag, kDevTimeoutMma) &&
                   mbar_wait(bar_acc_empty(s), (p & 1) ^ 1, abort_flag, kDevTimeoutMma);
            } else {
              ok = mbar_wait(bar_h_full(s), (p * (L - 1) + l - 1) & 1, abort_flag, kDevTimeoutMma);
            }
            if (!ok) break;
            tc_fence_after();
            const uint32_t a_base = (l == 0) ? s_x + s * Cfg::X_BYTES : s_h + s * Cfg::H_BYTES;
            const uint32_t b_base = s_w + NetT::template w_off<l>();
            const uint32_t d_tmem = tmem_base + s * Cfg::SLOT_COLS;
#pragma unroll
            for (int k = 0; k < K / 16; ++k) {
              const uint64_t ad = kmajor_desc<kTileM, K>(a_base, k);
              const uint64_t bd = mnmajor_desc<K, N>(b_base, k);
              umma_f16(d_tmem, ad, bd, idesc, k > 0 ? 1u : 0u);
            }
            umma_commit(bar_acc_full(s));
            if constexpr (l == 0) umma_commit(bar_x_empty(s));
          }
        });
      }
      // Drain: all issued MMAs complete before TMEM is freed.
      umma_commit(bar_mma_done);
      volatile int no_abort = 0;
      mbar_wait(bar_mma_done, 0, &no_abort, kDevTimeoutMma);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue
    const int e = warp - 2;
    const int q = warp & 3;           // TMEM lane quarter this warp may access
    const int grp = e >> 2;           // column group
    const uint32_t row = q * 32 + lane;
    const uint32_t lane_addr = static_cast<uint32_t>(q * 32) << 16;
    const bool leader = (e == 0 && lane == 0);
    bool ok = true;
    for (int p = 0; ok; ++p) {
      if (tile_of(p, 0) >= num_tiles) break;
      static_for<0, L>([&](auto lc) {
        constexpr int l = decltype(lc)::value;
        constexpr int N = NetT::template D<l + 1>();
        constexpr int NCOL = N / Cfg::NG;
        constexpr bool last = (l == L - 1);
        static_for<0, NS>([&](auto sc) {
          constexpr int s = decltype(sc)::value;
          if (!ok || tile_of(p, s) >= num_tiles) return;
          ok = __all_sync(0xffffffffu, mbar_wait(bar_acc_full(s), (p * L + l) & 1, abort_flag,
                                                 kDevTimeoutEpi));
          if (!ok) return;
          tc_fence_after();
          const uint32_t hbuf = s_h + s * Cfg::H_BYTES;
          if constexpr (l == 0) {
            // hbuf may still be the source of this slot's previous TMA store:
            // the leader waits for that store to finish reading, then frees it.
            if (p > 0) {
              if (leader) {
                bulk_wait_group_read<NS - 1 - s>();
                mbar_arrive(bar_store_free(s));
              }
              __syncwarp();
              ok = __all_sync(0xffffffffu,
                              mbar_wait(bar_store_free(s), (p - 1) & 1, abort_flag, kDevTimeoutEpi));
              if (!ok) return;
            }
          }
          const int col0 = grp * NCOL;
          float v[NCOL];
          tmem_load_cols<NCOL>(tmem_base + lane_addr + s * Cfg::SLOT_COLS + col0, v);
          if constexpr (last) {
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(bar_acc_empty(s));
          }
          store_row_chunk<N, NCOL, !last>(hbuf, row, col0, v);
          fence_proxy_async_smem();
          if constexpr (!last) {
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(bar_h_full(s));
          } else {
            __syncwarp();
            if (lane == 0) mbar_arrive(bar_out_ready(s));
            if (leader) ok = mbar_wait(bar_out_ready(s), p & 1, abort_flag, kDevTimeoutEpi);
            ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
            if (leader && ok) {
              constexpr int C = chunk_elems(N);
              constexpr int P = pitch_bytes(N);
              const int t = tile_of(p, s);
#pragma unroll
              for (int c = 0; c < N / C; ++c)
                tma_store_2d(&maps.out, hbuf + c * kTileM * P, c * C, t * kTileM);
              bulk_commit_group();
            }
          }
        });
      });
    }
    if (leader) bulk_wait_group<0>();
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, Cfg::TMEM_COLS);
  }
}

}  // namespace mlpk
