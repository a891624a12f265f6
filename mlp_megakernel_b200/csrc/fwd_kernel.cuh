// Persistent, warp-specialised fused softplus-MLP forward for sm_100a.
//
// out = softplus(...softplus(x @ W_0)...) @ W_{L-1}   (weights [in, out])
//
// This replaces the reference's Triton megakernel `_fused_mlp_recompute`
// (kernel.py:60-123) and its launch wrapper (kernel.py:130-156); the 5-layer
// chain is README.md:9.  Design (not a translation of the Triton loop nest):
//
//  * One CTA per SM (persistent).  Row tiles of 128 rows are assigned
//    round-robin: CTA b owns tiles b, b+G, b+2G, ...; tile b+(i*NS+s)*G runs in
//    "slot" s.  Each slot has its own x buffer, activation buffer, TMEM
//    accumulator and epilogue warp group, so the tensor core runs layer l of
//    one slot while the other slot's warps run their activation (ping-pong).
//  * warp 0 (one lane): TMA producer.  Loads every layer's fp16 weights into
//    shared memory ONCE per CTA, then streams x tiles into an NS-deep ring.
//  * warp 1: allocates TMEM; one lane issues tcgen05.mma (M=128, N=d_{l+1},
//    K=16 steps) for every layer of every tile; fp32 accumulators live in TMEM
//    (one accumulator region per slot, reused by all layers of that slot).
//  * warps 2..2+NS*EPW-1: epilogue, EPW warps per slot.  tcgen05.ld the
//    accumulator (warp w owns TMEM lanes 32*(w%4)..+31 = tile rows; the slot's
//    EPW/4 column groups split the columns), softplus in fp32 registers with
//    packed f32x2 math, cast to fp16 and st.shared straight into the next
//    layer's K-major, swizzled A operand; for the last layer the fp16 result is
//    staged in the same buffer and written by TMA stores (OOB rows of the last
//    tile are clipped by TMA).  TMEM loads are software-pipelined: the next 32
//    columns are in flight while the current 32 are computed.
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
  __host__ __device__ static constexpr bool hidden_uniform() {
    constexpr int a[] = {Ds...};
    for (int i = 2; i < L; ++i)
      if (a[i] != a[1]) return false;
    return true;
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

template <class NetT, int NS, int EPW>
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
  static constexpr int CHUNK = 32;                       // columns per h hand-off chunk
  static constexpr int MAXCH = (HMAX + CHUNK - 1) / CHUNK;  // chunks per layer, max
  // x_full, x_empty, acc_full, out_ready, store_free per slot; MAXCH h-chunk
  // barriers per slot; w_full; mma_done
  static constexpr int NUM_BARS = 5 * NS + NS * MAXCH + 2;
  static constexpr int OFF_MISC = OFF_BAR + 8 * NUM_BARS;
  static constexpr int SMEM_BYTES = OFF_MISC + 16 + 1024;  // + alignment slack
  static constexpr int SLOT_COLS = align_up(HMAX, 32);   // one accumulator buffer
  static constexpr int TMEM_COLS_RAW = 2 * NS * SLOT_COLS;  // two buffers per slot
  static constexpr int TMEM_COLS = TMEM_COLS_RAW <= 32    ? 32
                                   : TMEM_COLS_RAW <= 64  ? 64
                                   : TMEM_COLS_RAW <= 128 ? 128
                                   : TMEM_COLS_RAW <= 256 ? 256
                                                          : 512;
  static constexpr int THREADS = (2 + NS * EPW) * 32;
  static constexpr int NG = EPW / 4;  // column groups per slot
  static_assert(EPW % 4 == 0, "epilogue warps come in groups of 4 (one per TMEM lane quarter)");
  static_assert(L >= 2, "at least two layers");
  static constexpr int H = NetT::template D<1>();  // hidden width (all hidden layers)
  static_assert(NetT::hidden_uniform(), "all hidden layers must have the same width");
  static_assert(TMEM_COLS_RAW <= 512, "accumulators exceed TMEM");
  static_assert(SMEM_BYTES <= 232448, "shared memory budget exceeded");
};

// Converts CH fp32 accumulator values (columns col..col+CH-1 of row `row`) to
// fp16 -- through softplus when ACT -- and stores them as CH/8 16-byte units
// into an operand tile of extent N stored as swizzled chunks (layout.cuh).
template <int N, int CH, bool ACT>
__device__ __forceinline__ void emit_cols(const uint32_t (&r)[CH], uint32_t tile_base,
                                          uint32_t row, int col) {
  constexpr int C = chunk_elems(N);
  constexpr int P = pitch_bytes(N);
#pragma unroll
  for (int u = 0; u < CH / 8; ++u) {
    const int cc = col + 8 * u;
    uint32_t w[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float2 z = make_float2(__uint_as_float(r[8 * u + 2 * j]), __uint_as_float(r[8 * u + 2 * j + 1]));
      if constexpr (ACT) z = softplus_x2(z);
      w[j] = pack_half2(z.x, z.y);
    }
    st_shared_v4(tile_base + (cc / C) * (kTileM * P) + swz_off<P>(row, (cc % C) / 8), w[0], w[1],
                 w[2], w[3]);
  }
}

// Publishes one finished chunk of h: the smem writes become visible to the
// tensor core (async proxy), the chunk's TMEM reads are ordered before any
// later MMA, and lane 0 arrives on the chunk's barrier (count: 4 warps).
__device__ __forceinline__ void publish_chunk(uint32_t bar) {
  fence_proxy_async_smem();
  tc_fence_before();
  __syncwarp();
  if (lane_id() == 0) mbar_arrive(bar);
}

// One epilogue job of one warp: NCOL accumulator columns starting at TMEM
// address taddr (lane field = the warp's quarter) -> fp16 operand tile.  For a
// hidden layer (PUB) every 32 finished columns are published on
// chunk_bar0 + 8*(chunk index) so the next layer's MMA can start on them.
// Inlined; the epilogue calls it from one runtime loop over the hidden layers
// and once for the output layer, so the kernel holds two copies.
template <int N, int NCOL, bool ACT, bool PUB>
__device__ __forceinline__ void epi_job(uint32_t taddr, uint32_t tile_base, uint32_t row, int col0,
                                     uint32_t chunk_bar0) {
  static_assert(!PUB || NCOL % 32 == 0,
                "hidden widths must give every column group whole 32-column chunks");
  if constexpr (NCOL == 8) {
    uint32_t r[8];
    tmem_ld_wait_x8(taddr, r);
    emit_cols<N, 8, ACT>(r, tile_base, row, col0);
    if constexpr (PUB) publish_chunk(chunk_bar0 + 8 * (col0 / 32));
  } else if constexpr (NCOL == 16) {
    uint32_t r[16];
    tmem_ld_wait_x16(taddr, r);
    emit_cols<N, 16, ACT>(r, tile_base, row, col0);
    if constexpr (PUB) publish_chunk(chunk_bar0 + 8 * (col0 / 32));
  } else {
    static_assert(NCOL % 32 == 0, "columns per thread: 8, 16 or a multiple of 32");
    uint32_t a[32];
    tmem_ld_wait_x32(taddr, a);
#pragma unroll
    for (int c = 0; c < NCOL; c += 32) {
      uint32_t b[32];
      if (c + 32 < NCOL) tmem_ld_async_x32(taddr + c + 32, b);
      emit_cols<N, 32, ACT>(a, tile_base, row, col0 + c);
      if constexpr (PUB) publish_chunk(chunk_bar0 + 8 * ((col0 + c) / 32));
      if (c + 32 < NCOL) {
        tmem_wait_ld_bind_x32(b);
#pragma unroll
        for (int i = 0; i < 32; ++i) a[i] = b[i];
      }
    }
  }
}

template <class NetT, int NS, int EPW>
__global__ void __launch_bounds__(FwdCfg<NetT, NS, EPW>::THREADS, 1)
    mlp_fwd_kernel(const __grid_constant__ FwdMaps<NetT::L> maps, int num_tiles) {
  using Cfg = FwdCfg<NetT, NS, EPW>;
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
  auto bar_out_ready = [&](int s) { return s_bar + 8u * (3 * NS + s); };
  auto bar_store_free = [&](int s) { return s_bar + 8u * (4 * NS + s); };
  // h chunk c of slot s: columns [32c, 32c+32) of the activation in hbuf[s]
  auto bar_chunk = [&](int s, int c) { return s_bar + 8u * (5 * NS + s * Cfg::MAXCH + c); };
  const uint32_t bar_w_full = s_bar + 8u * (5 * NS + NS * Cfg::MAXCH);
  const uint32_t bar_mma_done = bar_w_full + 8u;
  const uint32_t s_tmem_slot = sbase + Cfg::OFF_MISC;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(gbase + Cfg::OFF_MISC + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(bar_x_full(s), 1);
      mbar_init(bar_x_empty(s), 1);
      mbar_init(bar_acc_full(s), 1);
      mbar_init(bar_out_ready(s), EPW);
      mbar_init(bar_store_free(s), 1);
      for (int c = 0; c < Cfg::MAXCH; ++c) mbar_init(bar_chunk(s, c), 4);
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
    // Job g = i*L + l of slot s accumulates into TMEM buffer (g & 1) of the
    // slot, so layer l+1 can run while the epilogue still reads layer l.
    // Layer 0 consumes the whole x tile; layer l >= 1 consumes h_{l-1} chunk by
    // chunk as the epilogue publishes it (fixed order -> deterministic sums).
    if (lane == 0) {
      bool ok = mbar_wait(bar_w_full, 0, abort_flag, kDevTimeoutMma);
      tc_fence_after();
      for (int i = 0; ok; ++i) {
        if (tile_of(i, 0) >= num_tiles) break;
        static_for<0, L>([&](auto lc) {
          constexpr int l = decltype(lc)::value;
          constexpr int K = NetT::template D<l>();
          constexpr int N = NetT::template D<l + 1>();
          constexpr uint32_t idesc = make_idesc_f16(kTileM, N, 0, 1);
          const uint32_t b_base = s_w + NetT::template w_off<l>();
#pragma unroll
          for (int s = 0; s < NS; ++s) {
            if (!ok || tile_of(i, s) >= num_tiles) break;
            const uint32_t d_tmem = tmem_base + (2 * s + ((i * L + l) & 1)) * Cfg::SLOT_COLS;
            if constexpr (l == 0) {
              ok = mbar_wait(bar_x_full(s), i & 1, abort_flag, kDevTimeoutMma);
              if (!ok) break;
              tc_fence_after();
              const uint32_t a_base = s_x + s * Cfg::X_BYTES;
#pragma unroll
              for (int k = 0; k < K / 16; ++k)
                umma_f16(d_tmem, kmajor_desc<kTileM, K>(a_base, k), mnmajor_desc<K, N>(b_base, k),
                         idesc, k > 0 ? 1u : 0u);
              umma_commit(bar_x_empty(s));
            } else {
              // chunks of h_{l-1}: 32 columns each, produced by column group g
              // as its sub-chunk j; consume sub-chunk-major (both groups' first
              // halves first).
              constexpr int KC = K < 32 ? K : 32;        // columns per chunk
              constexpr int NCH = K / KC;                 // chunks of this input
              constexpr int NGRP = Cfg::NG;               // producer column groups
              constexpr int SUBS = NCH / NGRP > 0 ? NCH / NGRP : 1;
              const uint32_t a_base = s_h + s * Cfg::H_BYTES;
              const uint32_t par = (i * (L - 1) + l - 1) & 1;
              int issued = 0;
#pragma unroll
              for (int j = 0; j < SUBS; ++j) {
#pragma unroll
                for (int g = 0; g < NGRP; ++g) {
                  const int c = g * SUBS + j;
                  if (c >= NCH) continue;
                  ok = mbar_wait(bar_chunk(s, c), par, abort_flag, kDevTimeoutMma);
                  if (!ok) break;
                  tc_fence_after();
#pragma unroll
                  for (int kk = 0; kk < KC / 16; ++kk) {
                    const int k = c * (KC / 16) + kk;
                    umma_f16(d_tmem, kmajor_desc<kTileM, K>(a_base, k),
                             mnmajor_desc<K, N>(b_base, k), idesc, issued > 0 ? 1u : 0u);
                    ++issued;
                  }
                }
                if (!ok) break;
              }
              if (!ok) break;
            }
            umma_commit(bar_acc_full(s));
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
    const int s = e / EPW;             // slot served by this warp
    const int ew = e % EPW;            // warp index inside the slot group
    const int q = warp & 3;            // TMEM lane quarter this warp may access
    const int grp = ew >> 2;           // column group
    const uint32_t row = q * 32 + lane;
    const uint32_t t_lane = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + 2 * s * Cfg::SLOT_COLS;
    const uint32_t hbuf = s_h + s * Cfg::H_BYTES;
    const bool leader = (ew == 0 && lane == 0);
    bool ok = true;
    constexpr int H = Cfg::H;
    constexpr int NCOL_H = H / Cfg::NG;
    constexpr int NCOL_O = Cfg::DL / Cfg::NG;
    for (int i = 0; ok; ++i) {
      const int t = tile_of(i, s);
      if (t >= num_tiles) break;
      // hidden layers: softplus, fp16 activation published chunk by chunk
#pragma unroll 1
      for (int l = 0; l < L - 1; ++l) {
        ok = __all_sync(0xffffffffu, mbar_wait(bar_acc_full(s), (i * L + l) & 1, abort_flag,
                                               kDevTimeoutEpi));
        if (!ok) break;
        tc_fence_after();
        if (l == 0 && i > 0) {
          // hbuf may still be the source of this slot's previous TMA store:
          // the leader waits for that store to finish reading, then frees it.
          if (leader) {
            bulk_wait_group_read<0>();
            mbar_arrive(bar_store_free(s));
          }
          __syncwarp();
          ok = __all_sync(0xffffffffu,
                          mbar_wait(bar_store_free(s), (i - 1) & 1, abort_flag, kDevTimeoutEpi));
          if (!ok) break;
        }
        const uint32_t t_buf = t_lane + ((i * L + l) & 1) * Cfg::SLOT_COLS;
        epi_job<H, NCOL_H, true, true>(t_buf + grp * NCOL_H, hbuf, row, grp * NCOL_H,
                                       bar_chunk(s, 0));
      }
      if (!ok) break;
      // output layer: fp16 result staged in hbuf, written by TMA
      {
        constexpr int l = L - 1;
        ok = __all_sync(0xffffffffu, mbar_wait(bar_acc_full(s), (i * L + l) & 1, abort_flag,
                                               kDevTimeoutEpi));
        if (!ok) break;
        tc_fence_after();
        const uint32_t t_buf = t_lane + ((i * L + l) & 1) * Cfg::SLOT_COLS;
        epi_job<Cfg::DL, NCOL_O, false, false>(t_buf + grp * NCOL_O, hbuf, row, grp * NCOL_O, 0);
        fence_proxy_async_smem();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar_out_ready(s));
        if (leader) ok = mbar_wait(bar_out_ready(s), i & 1, abort_flag, kDevTimeoutEpi);
        ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
        if (leader && ok) {
          constexpr int C = chunk_elems(Cfg::DL);
          constexpr int P = pitch_bytes(Cfg::DL);
#pragma unroll
          for (int c = 0; c < Cfg::DL / C; ++c)
            tma_store_2d(&maps.out, hbuf + c * kTileM * P, c * C, t * kTileM);
          bulk_commit_group();
        }
      }
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
