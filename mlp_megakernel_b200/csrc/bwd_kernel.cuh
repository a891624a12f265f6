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
// Roles: warp 0 = TMA producer (weights once; then, per tile, g, h_{L-1} ..
// h_1 and x through a ring of generic tile slots, as far ahead as the ring
// allows), warp 1 = TMEM owner + MMA issuer (one lane), 4*NG epilogue warps
// (thread = tile row, NG column groups; sigmoid multiply in registers, dz
// written straight into the swizzled smem tile "G" that the next layer's two
// UMMAs read as K-major A (dgrad) and MN-major B (wgrad)).
//
// Per layer the MMA warp issues the dgrad first and commits it, then the
// wgrad: the epilogue's sigmoid multiply of layer l overlaps the wgrad of
// layer l, and only its stores into G wait for the wgrad to have read G.
//
// Shared memory: all weights (read as K-major B = W^T for dgrad), G (each dz),
// the ring of tile slots (dx is staged in x's slot for its TMA store) and,
// for 64-wide layers, a zeroed chunk that pads a weight-gradient M to 128.
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
  // caller's d0 when the network is served by a larger one (the maps carry
  // the caller's extents; loads zero-fill, the dx store skips chunks that
  // start at or past this width)
  int dx_cols;
};

// H32: the saved activations are fp32 (the reference's storage, README.md:30).
// Each h_l arrives as two ring slots (columns [0, d_l/2) and [d_l/2, d_l), in
// 32-column fp32 chunks); the epilogue computes the sigmoid from the fp32
// values and then overwrites the two slots in place with the fp16 h_l (the
// weight-gradient operand, rounded as the forward rounded it for the next
// GEMM) and dz_l, so no separate dz tile is needed; each layer's
// weight-gradient GEMM is issued after that epilogue.  One tile in flight.
template <class NetT, bool H32 = false>
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
  // widest dgrad output (d_0 .. d_{L-1}); the epilogue has NG column groups of
  // 4 warps so that a thread handles at most 32 columns of a layer
  __host__ __device__ static constexpr int dgmax() {
    int m = 0;
    for (int l = 0; l < L; ++l) m = NetT::dim(l) > m ? NetT::dim(l) : m;
    return m;
  }
  static constexpr int NG = dgmax() >= 128 ? 4 : dgmax() >= 64 ? 2 : 1;
  static constexpr int EPI_WARPS = 4 * NG;  // per slot
  static constexpr int ACC_W = align_up(DMAX, 32);
  static constexpr int TILE_BYTES = align_up(tile_bytes(kTileM, DMAX), 1024);
  static constexpr int W_TOTAL = NetT::w_total();
  // zero rows that pad a 64-wide weight-gradient M to 128: one UMMA reads 16
  // K-rows of it, and every K-step's descriptor points at the same 16 rows
  static constexpr int ZERO_BYTES = any_pad() ? 2048 : 0;  // 16 rows x 128 B
  // deepest load ring (5-layer backward at 1M rows: 227.5 us with 8 slots,
  // 224 us with the 10 that fit)
  static constexpr int kMaxRing = 12;
  // ring slots that fit in shared memory next to the weights, `ns` x `ng` dz
  // tiles (G), the zero rows and the barriers: w_full, slot_full[kMaxRing],
  // slot_empty[kMaxRing], then per tile slot acc_full, acc_free, wg_done, dz_full,
  // out_ready; mma_done; rd_done
  __host__ __device__ static constexpr int ring_fit_g(int ns, int ng) {
    return (232448 - 1024 - 16 - 8 * (3 + 2 * kMaxRing + 5 * ns) - (W_TOTAL + ns * ng * TILE_BYTES) - ZERO_BYTES) /
           TILE_BYTES;
  }
  __host__ __device__ static constexpr int ring_cap(int r) { return r > kMaxRing ? kMaxRing : r; }
  // every hidden width splits into two fp32 halves of whole 32-column chunks,
  // each fitting a ring slot
  __host__ __device__ static constexpr bool h32_ok() {
    for (int l = 1; l < L; ++l)
      if ((NetT::dim(l) / 2) % 32 != 0 || kTileM * (NetT::dim(l) / 2) * 4 > TILE_BYTES) return false;
    return true;
  }
  // Tiles in flight ("slots"): two when TMEM holds a second dgrad accumulator
  // next to the dW accumulators and the ring can hold one tile's loads plus
  // the first two of the next (see the producer); the MMA warp then
  // alternates the slots' layer steps so one slot's epilogue overlaps the
  // other slot's MMAs.
  // Tiles in flight and dz tiles per tile slot: two tiles where TMEM holds a
  // second dgrad accumulator and the ring keeps one tile's loads plus the
  // first two of the next.  With one tile in flight, two dz tiles (the
  // epilogue writes dz_l while the MMAs still read dz_{l+1}, no wait for the
  // weight gradient) where the ring keeps 4 slots beside them (the 6- and
  // 7-layer 64-wide networks; 3L128 and the 2-layer 128-wide network have
  // room for one); with two tiles in flight the other tile's step already
  // covers that wait, and a second dz tile per slot measured slower (5-layer
  // backward 227.8 vs 229.4 us at 1M rows).  fp32 saved activations: one
  // tile, no dz tile (dz lives in h's high half-slot).
  static constexpr bool TMEM2 = dw_col(L) + 2 * ACC_W <= 512;
  static constexpr int NS = (!H32 && TMEM2 && ring_cap(ring_fit_g(2, 1)) >= L + 3) ? 2 : 1;
  static constexpr int G_TILES = H32 ? 0 : (NS == 2 ? 1 : (ring_cap(ring_fit_g(1, 2)) >= 4 ? 2 : 1));
  __host__ __device__ static constexpr int ring_fit(int ns) { return ring_fit_g(ns, G_TILES); }
  // loads per tile: g, then h_{L-1} .. h_1 (one slot each, or two fp32 halves
  // each), then x
  static constexpr int NLD = H32 ? 2 * L : L + 1;
  // load index (within a tile) of h_l: fp16 -> its slot; fp32 -> its low
  // half (the high half is the next load)
  __host__ __device__ static constexpr int h_load(int l) { return H32 ? 1 + 2 * (L - 1 - l) : L - l; }
  static constexpr int THREADS = (2 + NS * EPI_WARPS) * 32;
  __host__ __device__ static constexpr bool groups_ok() {
    for (int l = 0; l < L; ++l) {
      const int cw = NetT::dim(l) / NG;
      if (NetT::dim(l) % NG != 0 || (cw != 8 && cw != 16 && cw != 32 && cw != 64)) return false;
    }
    return true;
  }
  static constexpr int OFF_G = W_TOTAL;  // G b of slot s at OFF_G + (s * G_TILES + b) * TILE_BYTES
  static constexpr int OFF_RING = OFF_G + NS * G_TILES * TILE_BYTES;
  static constexpr int RING_FIT = ring_fit(NS);
  static constexpr int RING = RING_FIT > kMaxRing ? kMaxRing : RING_FIT;
  static constexpr int OFF_ZERO = OFF_RING + RING * TILE_BYTES;
  static constexpr int OFF_BAR = OFF_ZERO + ZERO_BYTES;
  static constexpr int NUM_BARS = 2 + 2 * RING + 5 * NS + 1;
  static constexpr int OFF_MISC = OFF_BAR + 8 * NUM_BARS;
  static constexpr int SMEM_BYTES = OFF_MISC + 16 + 1024;
  static constexpr int ACC_COL = dw_col(L);
  // Data-gradient GEMMs with A from TMEM: the epilogue also packs dz_l
  // (fp16, two per column) into a per-slot TMEM tile at ZT_COL that the next
  // dgrad reads as its A operand (the TS form reads only W from shared
  // memory: 2 of the 6 KB an SS 128x64x16 UMMA reads), where TMEM has room
  // for it beside the dW and dgrad accumulators (the 64-wide networks and the
  // 5-layer one; not 3L128, whose accumulators fill TMEM).  dz_L = g still
  // comes from its ring slot (SS).
  static constexpr int ZT_W = NetT::template D<1>() / 2;
  static constexpr bool DG_TS = !H32 && L >= 2 && ACC_COL + NS * (ACC_W + ZT_W) <= 512;
  static constexpr int ZT_COL = ACC_COL + NS * ACC_W;
  static constexpr int TMEM_COLS_RAW = ACC_COL + NS * ACC_W + (DG_TS ? NS * ZT_W : 0);
  static constexpr int TMEM_COLS = TMEM_COLS_RAW <= 128 ? 128 : TMEM_COLS_RAW <= 256 ? 256 : 512;
  static constexpr int PARTIAL_FLOATS = [] {
    int n = 0;
    for (int i = 0; i < L; ++i) n += NetT::dim(i) * NetT::dim(i + 1);
    return n;
  }();
  static_assert(plans_ok(), "weight-gradient GEMM shapes not supported");
  static_assert(groups_ok(), "layer widths vs epilogue column groups");
  static_assert(NetT::hidden_uniform(), "all hidden layers must have the same width");
  static_assert(RING >= 2, "the tile ring needs at least two slots");
  // with two tiles in flight the ring must hold one tile's loads plus the
  // first two of the next (see the producer)
  static_assert(NS == 1 || RING >= L + 3, "ring too shallow for two tiles in flight");
  static_assert(TMEM_COLS_RAW <= 512, "dW + dgrad accumulators exceed TMEM");
  static_assert(SMEM_BYTES <= 232448, "shared memory budget exceeded");
  // fp32 saved activations: a ring of 3 keeps every load's slot free of the
  // step that waits for it (see the producer)
  static_assert(!H32 || (RING >= 3 && h32_ok()), "fp32 saved activations: ring too shallow or widths");
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

// this thread's row of an fp32 tile stored as 32-column chunks (128-byte
// rows, 128B swizzle): 4 values at column c (c % 4 == 0)
__device__ __forceinline__ uint4 ld_tile_row4_f32(uint32_t tile_base, uint32_t row, int c) {
  uint4 v;
  asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(tile_base + (c / 32) * (kTileM * 128) + swz_off<128>(row, (c % 32) / 4)));
  return v;
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

// CW consecutive fp32 TMEM columns of this warp's lanes, loaded and waited.
template <int CW>
__device__ __forceinline__ void tmem_ld_cols(uint32_t taddr, uint32_t (&r)[CW]) {
  if constexpr (CW == 8) tmem_ld_wait_x8(taddr, r);
  else if constexpr (CW == 16) tmem_ld_wait_x16(taddr, r);
  else if constexpr (CW == 32) tmem_ld_wait_x32(taddr, r);
  else tmem_ld_wait_x64(taddr, r);
}

// N consecutive 32-bit TMEM columns of this warp's lanes from registers
// (complete with tmem_wait_st()).
template <int N>
__device__ __forceinline__ void tmem_st_cols(uint32_t taddr, const uint32_t (&r)[N]) {
  if constexpr (N == 4) {
    tmem_st_x4(taddr, r);
  } else if constexpr (N == 8) {
    tmem_st_x8(taddr, r);
  } else if constexpr (N == 16) {
    tmem_st_x16(taddr, r);
  } else {
    static_assert(N % 16 == 0, "TMEM store width");
#pragma unroll
    for (int c = 0; c < N; c += 16) {
      uint32_t w[16];
#pragma unroll
      for (int v = 0; v < 16; ++v) w[v] = r[c + v];
      tmem_st_x16(taddr + c, w);
    }
  }
}

// The layer index l = L - 1 - i of static_for iteration i, as a type.
template <int L, class IC>
__device__ __forceinline__ constexpr auto lc_rev(IC) {
  return std::integral_constant<int, L - 1 - IC::value>{};
}

template <class NetT, bool H32 = false>
__global__ void __launch_bounds__(BwdCfg<NetT, H32>::THREADS, 1)
    mlp_bwd_kernel(const __grid_constant__ BwdMaps<NetT::L> maps, int num_tiles) {
  using Cfg = BwdCfg<NetT, H32>;
  constexpr int L = Cfg::L;
  constexpr int R = Cfg::RING;
  // loads per tile: k = 0 g; fp16 h: k = 1..L-1 h_{L-k}; fp32 h: k = 1..2L-2
  // the halves (lo, hi) of h_{L-1}, .., h_1; k = NLD-1 x
  constexpr int NLD = Cfg::NLD;
  constexpr int NG = Cfg::NG;
  constexpr int EW = Cfg::EPI_WARPS;  // epilogue warps per slot
  constexpr int NS = Cfg::NS;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t sbase = (raw + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (sbase - raw);

  const uint32_t s_w = sbase;
  // dz tile of slot s written at the slot's step st (read by the next step)
  auto s_g = [&](int s, int st) {
    const int b = Cfg::G_TILES > 1 ? (st & 1) : 0;
    return sbase + Cfg::OFF_G + static_cast<uint32_t>(s * Cfg::G_TILES + b) * Cfg::TILE_BYTES;
  };
  auto slot_addr = [&](int r) { return sbase + Cfg::OFF_RING + static_cast<uint32_t>(r) * Cfg::TILE_BYTES; };
  const uint32_t s_zero = sbase + Cfg::OFF_ZERO;
  const uint32_t s_bar = sbase + Cfg::OFF_BAR;
  const uint32_t bar_w_full = s_bar;
  auto bar_slot_full = [&](int r) { return s_bar + 8u + 8u * r; };
  auto bar_slot_empty = [&](int r) { return s_bar + 8u + 8u * (R + r); };
  // per tile slot s
  auto bar_acc_full = [&](int s) { return s_bar + 8u + 16u * R + 40u * s; };  // dgrad accumulator written
  auto bar_acc_free = [&](int s) { return bar_acc_full(s) + 8; };   // ... and read (once per tile)
  auto bar_wg_done = [&](int s) { return bar_acc_full(s) + 16; };   // a wgrad read its operands
  auto bar_dz_full = [&](int s) { return bar_acc_full(s) + 24; };   // the next layer's dz is staged
  auto bar_out_ready = [&](int s) { return bar_acc_full(s) + 32; }; // dx staged
  const uint32_t bar_mma_done = bar_acc_full(NS);
  // (H32) every epilogue warp has read its fp32 h of the current layer: the
  // two half-slots may be overwritten in place
  const uint32_t bar_rd_done = bar_mma_done + 8u;
  const uint32_t s_tmem_slot = sbase + Cfg::OFF_MISC;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(gbase + Cfg::OFF_MISC + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    mbar_init(bar_w_full, 1);
    for (int r = 0; r < R; ++r) {
      mbar_init(bar_slot_full(r), 1);
      mbar_init(bar_slot_empty(r), 1 + EW);  // MMA commit + every epilogue warp
    }
    for (int s = 0; s < NS; ++s) {
      mbar_init(bar_acc_full(s), 1);
      mbar_init(bar_acc_free(s), EW);
      mbar_init(bar_wg_done(s), 1);
      mbar_init(bar_dz_full(s), EW);
      mbar_init(bar_out_ready(s), EW);
    }
    mbar_init(bar_mma_done, 1);
    mbar_init(bar_rd_done, EW);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(s_tmem_slot, Cfg::TMEM_COLS);
    tmem_relinquish();
  }
  if constexpr (Cfg::ZERO_BYTES > 0) {  // zero chunk that pads a 64-wide wgrad M to 128
    for (int i = threadIdx.x; i < Cfg::ZERO_BYTES / 16; i += blockDim.x)
      st_shared_v4(s_zero + 16 * i, 0u, 0u, 0u, 0u);
    fence_proxy_async_smem();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *reinterpret_cast<volatile uint32_t*>(gbase + Cfg::OFF_MISC);
  pdl_enter();
  const int G = gridDim.x;
  // Tiles from the last to the first (num_tiles = none left): the training
  // forward runs them first to last, so the rows it wrote (and read) last --
  // the saved activations and inputs of its final rounds, still in L2 when
  // the backward starts -- are the first this kernel loads (config 3 step
  // 211 -> 206 us at 262,144 rows, also with L2 flushed before each step).
  auto tile_of = [&](int i) {
    const int r = static_cast<int>(blockIdx.x) + i * G;
    return r < num_tiles ? num_tiles - 1 - r : num_tiles;
  };

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
      // L2 eviction priorities: the next tile's rows are prefetched as
      // evict_last, so they stay in L2 until their ring loads come, and the
      // ring loads read them as evict_first: a line is read once, and once
      // read it is the first to go (config 3 step 216 -> 208 us at 262,144
      // rows; the prefetched fp32 h used to lose lines before its loads)
      const uint64_t pol_keep = l2_policy_evict_last();
      const uint64_t pol_drop = l2_policy_evict_first();
      auto load_tile = [&](const CUtensorMap* map, uint32_t dst, uint32_t bar, int d, int t) {
        const int C = d < 64 ? d : 64;
        const int P = 2 * C;
        mbar_arrive_expect_tx(bar, kTileM * d * 2);
        for (int c = 0; c < d / C; ++c) tma_load_2d_hint(dst + c * kTileM * P, map, bar, c * C, t * kTileM, pol_drop);
      };
      // fp32 half `half` of an h tile of width d: d/64 chunks of 32 columns
      auto load_half_f32 = [&](const CUtensorMap* map, uint32_t dst, uint32_t bar, int d, int half, int t) {
        const int hw = d / 2;
        mbar_arrive_expect_tx(bar, kTileM * hw * 4);
        for (int c = 0; c < hw / 32; ++c)
          tma_load_2d_hint(dst + c * kTileM * 128, map, bar, half * hw + c * 32, t * kTileM, pol_drop);
      };
      auto prefetch_tile = [&](const CUtensorMap* map, int d, int t) {
        const int C = d < 64 ? d : 64;
        for (int c = 0; c < d / C; ++c) tma_prefetch_l2_2d_hint(map, c * C, t * kTileM, pol_keep);
      };
      auto prefetch_tile_f32 = [&](const CUtensorMap* map, int d, int t) {
        for (int c = 0; c < d / 32; ++c) tma_prefetch_l2_2d_hint(map, c * 32, t * kTileM, pol_keep);
      };
      bool ok = true;
      int issued = 0;
      for (int i = 0; ok; ++i) {
        const int t = tile_of(i);
        if (t >= num_tiles) break;
        // the ring holds about one tile: bring the NEXT tile's rows into L2 now,
        // so its ring loads later hit L2 (more bytes in flight per SM)
        if (tile_of(i + 1) < num_tiles) {
          const int tn = tile_of(i + 1);
          prefetch_tile(&maps.g, Cfg::DL, tn);
          static_for<1, L>([&](auto hc) {
            constexpr int l = decltype(hc)::value;
            if constexpr (H32) prefetch_tile_f32(&maps.h[l - 1], NetT::template D<l>(), tn);
            else prefetch_tile(&maps.h[l - 1], NetT::template D<l>(), tn);
          });
          prefetch_tile(&maps.x, Cfg::D0, tn);
        }
        static_for<0, NLD>([&](auto kc) {
          constexpr int k = decltype(kc)::value;
          if (!ok) return;
          const int n = i * NLD + k;
          const int r = n % R;
          ok = mbar_wait(bar_slot_empty(r), ((n / R) & 1) ^ 1, abort_flag, kDevTimeoutEmpty);
          if (!ok) return;
          if constexpr (k == 0) {
            load_tile(&maps.g, slot_addr(r), bar_slot_full(r), Cfg::DL, t);
          } else if constexpr (k == NLD - 1) {
            load_tile(&maps.x, slot_addr(r), bar_slot_full(r), Cfg::D0, t);
          } else if constexpr (H32) {
            constexpr int l = L - 1 - (k - 1) / 2;
            load_half_f32(&maps.h[l - 1], slot_addr(r), bar_slot_full(r), NetT::template D<l>(), (k - 1) % 2, t);
          } else {
            load_tile(&maps.h[L - k - 1], slot_addr(r), bar_slot_full(r), NetT::template D<L - k>(), t);
          }
          ++issued;
        });
      }
      // Drain: never leave the CTA with a TMA load still writing shared memory.
      volatile int no_abort = 0;
      mbar_wait(bar_w_full, 0, &no_abort, kDevTimeoutFull);
      for (int r = 0; r < R; ++r) {
        const int uses = issued > r ? (issued - r + R - 1) / R : 0;
        if (uses > 0) mbar_wait(bar_slot_full(r), (uses - 1) & 1, &no_abort, kDevTimeoutFull);
      }
    } else if (lane == 1) {
      // dx stores, off the epilogue warps' path: the epilogue stages each
      // tile's dx in x's ring slot; this lane TMA-stores it and, once the store
      // has read it, returns the slot to the producer
      bool ok = true;
      for (int i = 0; ok; ++i) {
        const int t = tile_of(i);
        if (t >= num_tiles) break;
        const int s = i % NS, j = i / NS;
        ok = mbar_wait(bar_out_ready(s), j & 1, abort_flag, kDevTimeoutEpi);
        if (!ok) break;
        const int nx = i * NLD + NLD - 1;
        const uint32_t xb = slot_addr(nx % R);
        constexpr int C = chunk_elems(Cfg::D0);
        constexpr int P = pitch_bytes(Cfg::D0);
#pragma unroll
        for (int cc = 0; cc < Cfg::D0 / C; ++cc)
          if (cc * C < maps.dx_cols) tma_store_2d(&maps.dx, xb + cc * kTileM * P, cc * C, t * kTileM);
        bulk_commit_group();
        bulk_wait_group_read<0>();
        mbar_arrive_cnt(bar_slot_empty(nx % R), EW);  // x's slot may take a new tile
      }
      bulk_wait_group<0>();
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    const bool issuer = (lane == 0);
    // dgrad: dh_l[128 x d_l] = dz_{l+1} W_l^T: A = dz (K-major, K = d_{l+1}),
    // B = W_l as stored ([d_l rows][d_{l+1}] = K-major W_l^T)
    // (DG_TS, l < L-1: A = the packed dz_{l+1} in TMEM at zt, 16 K-elements
    // per 8 columns)
    auto issue_dgrad = [&](auto lc, uint32_t acc, uint32_t zsrc, uint32_t zt) {
      constexpr int l = decltype(lc)::value;
      constexpr int DI = NetT::template D<l>();
      constexpr int DO = NetT::template D<l + 1>();
      constexpr uint32_t idesc_d = make_idesc_f16(kTileM, DI, 0, 0);
      const uint64_t bd0 = kmajor_base_desc<DO>(s_w + NetT::template w_off<l>());
      if constexpr (Cfg::DG_TS && l < L - 1) {
#pragma unroll
        for (int k = 0; k < DO / 16; ++k)
          umma_f16_ts(acc, zt + 8 * k, bd0 + (kmajor_koff<DI, DO>(k) >> 4), idesc_d, k > 0 ? 1u : 0u);
      } else {
        const uint64_t ad0 = kmajor_base_desc<DO>(zsrc);
#pragma unroll
        for (int k = 0; k < DO / 16; ++k)
          umma_f16(acc, ad0 + (kmajor_koff<kTileM, DO>(k) >> 4), bd0 + (kmajor_koff<DI, DO>(k) >> 4), idesc_d,
                   k > 0 ? 1u : 0u);
      }
    };
    // wgrad over the 128 tile rows (K): dW_l += h_l^T dz (A = h_l, B = dz) or,
    // transposed, dW_l^T += dz^T h_l (A = dz, B = h_l); both operands
    // MN-major from shared memory; a 64-wide A is padded to M = 128 by
    // pointing its second 64-column chunk (LBO) at the zero chunk.
    auto issue_wgrad = [&](auto lc, int i, uint32_t a_h, uint32_t zsrc) {
      constexpr int l = decltype(lc)::value;
      constexpr bool TR = Cfg::wg_trans(l);
      constexpr int MW = Cfg::wg_m(l);
      constexpr int NW = Cfg::wg_n(l);
      constexpr uint32_t idesc_w = make_idesc_f16(kTileM, NW, 1, 1);
      const uint32_t a_base = TR ? zsrc : a_h;
      const uint32_t b_base = TR ? a_h : zsrc;
      constexpr int PA = pitch_bytes(MW);
      const uint64_t bw0 = mnmajor_base_desc<kTileM, NW>(b_base);
      const uint32_t dw = tmem_base + Cfg::dw_col(l);
      // a 64-wide A: its second 64-column chunk (LBO) is the 16 zero rows, the
      // same for every K-step, so K-step k moves the start address up by
      // koff and the LBO down by as much: one 64-bit add of a constant per
      // K-step (no borrow: the zero rows lie past the ring and G, at least a
      // tile beyond a_base, and koff < a tile)
      const uint32_t lbo0 = (MW < 128) ? (s_zero - a_base) : kTileM * PA;
      const uint64_t aw0 = make_sdesc(a_base, lbo0, 8 * PA, umma_layout_code(PA));
#pragma unroll
      for (int k = 0; k < kTileM / 16; ++k) {
        const uint64_t ko = mnmajor_koff<MW>(k) >> 4;
        const uint64_t astep = (MW < 128) ? ko - (ko << 16) : ko;
        umma_f16(dw, aw0 + astep, bw0 + (mnmajor_koff<NW>(k) >> 4), idesc_w, (i > 0 || k > 0) ? 1u : 0u);
      }
    };
    bool ok = __all_sync(0xffffffffu, mbar_wait(bar_w_full, 0, abort_flag, kDevTimeoutMma));
    tc_fence_after();
    if constexpr (H32) {
      // One tile at a time.  Layer step l: dgrad(l) reads dz_{l+1} (g, or the
      // high half-slot of h_{l+1} where the epilogue of step l+1 put it), then
      // the weight gradient of layer l+1, whose operands the epilogue of step
      // l+1 has just written (fp16 h_{l+1} in its low half-slot) -- the last
      // read of h_{l+1}'s low slot and of dz_{l+2}'s slot.  After dgrad(0):
      // wgrad(0) from x and dz_1.
      const uint32_t acc = tmem_base + Cfg::ACC_COL;
      for (int i = 0; ok; ++i) {
        if (tile_of(i) >= num_tiles) break;
        const int base = i * NLD;
        auto slot_of = [&](int k) { return (base + k) % R; };
        auto full_par = [&](int k) { return static_cast<uint32_t>(((base + k) / R) & 1); };
        static_for<0, L>([&](auto sc) {
          constexpr int l = L - 1 - decltype(sc)::value;  // L-1 .. 0
          if (!ok) return;
          uint32_t zsrc;
          if constexpr (l == L - 1) {
            ok = __all_sync(0xffffffffu, mbar_wait(bar_slot_full(slot_of(0)), full_par(0), abort_flag,
                                                   kDevTimeoutMma)) &&
                 __all_sync(0xffffffffu, mbar_wait(bar_acc_free(0), (i & 1) ^ 1, abort_flag, kDevTimeoutMma));
            zsrc = slot_addr(slot_of(0));
          } else {
            ok = __all_sync(0xffffffffu, mbar_wait(bar_dz_full(0), (i * (L - 1) + (L - 2 - l)) & 1,
                                                   abort_flag, kDevTimeoutMma));
            zsrc = slot_addr(slot_of(Cfg::h_load(l + 1) + 1));  // dz_{l+1}: high half-slot of h_{l+1}
          }
          if (!ok) return;
          tc_fence_after();
          if (issuer) {
            issue_dgrad(std::integral_constant<int, l>{}, acc, zsrc, 0u);
            umma_commit(bar_acc_full(0));
            if constexpr (l < L - 1) {
              // weight gradient of layer l+1: A = fp16 h_{l+1} (low half-slot),
              // B = dz_{l+2} (g, or the high half-slot of h_{l+2})
              constexpr int kb = (l + 1 == L - 1) ? 0 : Cfg::h_load(l + 2) + 1;
              constexpr int ka = Cfg::h_load(l + 1);
              issue_wgrad(std::integral_constant<int, l + 1>{}, i, slot_addr(slot_of(ka)), slot_addr(slot_of(kb)));
              umma_commit(bar_slot_empty(slot_of(ka)));
              umma_commit(bar_slot_empty(slot_of(kb)));
            }
          }
          __syncwarp();
          if constexpr (l == 0) {
            ok = __all_sync(0xffffffffu, mbar_wait(bar_slot_full(slot_of(NLD - 1)), full_par(NLD - 1),
                                                   abort_flag, kDevTimeoutMma));
            if (!ok) return;
            tc_fence_after();
            if (issuer) {
              constexpr int kz = Cfg::h_load(1) + 1;  // dz_1: high half-slot of h_1
              issue_wgrad(std::integral_constant<int, 0>{}, i, slot_addr(slot_of(NLD - 1)), slot_addr(slot_of(kz)));
              umma_commit(bar_wg_done(0));  // x's slot may take dx
              umma_commit(bar_slot_empty(slot_of(kz)));
              umma_commit(bar_slot_empty(slot_of(NLD - 1)));
            }
            __syncwarp();
          }
        });
      }
    } else {
      // Tiles i = p*NS + s of round p; per layer, every slot's step in turn.
      // Per layer the dgrad is issued first and committed, then the wgrad:
      // the epilogue's sigmoid multiply of layer l overlaps the wgrad of
      // layer l, and only its stores into G wait for the wgrad to have read G.
      for (int p = 0; ok; ++p) {
        if (tile_of(p * NS) >= num_tiles) break;
        static_for<0, L>([&](auto lc) {
          constexpr int l = L - 1 - decltype(lc)::value;  // L-1 .. 0
#pragma unroll
          for (int s = 0; s < NS; ++s) {
            const int i = p * NS + s;
            if (!ok || tile_of(i) >= num_tiles) break;
            const uint32_t acc = tmem_base + Cfg::ACC_COL + s * Cfg::ACC_W;
            const int ng = i * NLD;            // g
            const int na = i * NLD + (L - l);  // h_l (x for l == 0)
            const int st = p * L + (L - 1 - l);  // this slot's step count
            // dz_{l+1}: g (a ring slot) for the last layer, else the G tile the
            // epilogue of the previous step wrote
            uint32_t zsrc = s_g(s, st - 1);
            if constexpr (l == L - 1) {
              ok = __all_sync(0xffffffffu, mbar_wait(bar_slot_full(ng % R), (ng / R) & 1, abort_flag,
                                                     kDevTimeoutMma)) &&
                   __all_sync(0xffffffffu,
                              mbar_wait(bar_acc_free(s), (p & 1) ^ 1, abort_flag, kDevTimeoutMma));
              zsrc = slot_addr(ng % R);
            } else {
              ok = __all_sync(0xffffffffu, mbar_wait(bar_dz_full(s), (p * (L - 1) + (L - 2 - l)) & 1,
                                                     abort_flag, kDevTimeoutMma));
            }
            if (!ok) break;
            ok = __all_sync(0xffffffffu,
                            mbar_wait(bar_slot_full(na % R), (na / R) & 1, abort_flag, kDevTimeoutMma));
            if (!ok) break;
            tc_fence_after();
            const uint32_t a_h = slot_addr(na % R);
            if (issuer) {
              issue_dgrad(lc_rev<L>(lc), acc, zsrc, tmem_base + Cfg::ZT_COL + s * Cfg::ZT_W);
              umma_commit(bar_acc_full(s));
              issue_wgrad(lc_rev<L>(lc), i, a_h, zsrc);
              umma_commit(bar_wg_done(s));
              umma_commit(bar_slot_empty(na % R));
              if constexpr (l == L - 1) umma_commit(bar_slot_empty(ng % R));
            }
            __syncwarp();
          }
        });
      }
    }
    // Drain: all issued MMAs complete before TMEM is freed.
    if (issuer) umma_commit(bar_mma_done);
    __syncwarp();
    {
      volatile int no_abort = 0;
      mbar_wait(bar_mma_done, 0, &no_abort, kDevTimeoutMma);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue
    const int e = warp - 2;
    const int s = e / EW;       // tile slot served by this warp
    const int ew = e % EW;
    const int q = warp & 3;     // TMEM lane quarter this warp may access
    const int grp = ew >> 2;    // column group
    const uint32_t row = q * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(q * 32) << 16;
    const uint32_t acc = tmem_base + lane_off + Cfg::ACC_COL + s * Cfg::ACC_W;
    bool ok = true;
    for (int j = 0; ok; ++j) {
      const int i = j * NS + s;  // this slot's j-th tile
      const int t = tile_of(i);
      if (t >= num_tiles) break;
      static_for<0, L>([&](auto lc) {
        constexpr int l = L - 1 - decltype(lc)::value;  // dgrad result dh_l
        constexpr int DI = NetT::template D<l>();
        constexpr int CW = DI / NG;                      // this group's columns
        if (!ok) return;
        const int step = j * L + (L - 1 - l);  // this slot's step count
        const int c0 = grp * CW;
        ok = __all_sync(0xffffffffu, mbar_wait(bar_acc_full(s), step & 1, abort_flag, kDevTimeoutEpi));
        if (!ok) return;
        tc_fence_after();
        // the g slot is only read by the MMAs: release this warp's share now
        if constexpr (l == L - 1)
          if (lane == 0) mbar_arrive(bar_slot_empty((i * NLD) % R));
        uint32_t r[CW];
        tmem_ld_cols<CW>(acc + c0, r);
        uint32_t o[CW / 2];
        if constexpr (l > 0 && H32) {
          // dz_l = dh_l * (1 - e^{-h_l}) with h_l in fp32 from its two
          // half-slots; then, in place, the fp16 h_l (weight-gradient operand)
          // into the low half-slot and dz_l into the high one
          const int nlo = i * NLD + Cfg::h_load(l);
          const uint32_t lo = slot_addr(nlo % R), hi = slot_addr((nlo + 1) % R);
          ok = __all_sync(0xffffffffu, mbar_wait(bar_slot_full(nlo % R), (nlo / R) & 1, abort_flag,
                                                 kDevTimeoutEpi)) &&
               __all_sync(0xffffffffu, mbar_wait(bar_slot_full((nlo + 1) % R), ((nlo + 1) / R) & 1,
                                                 abort_flag, kDevTimeoutEpi));
          if (!ok) return;
          uint32_t hp[CW / 2];
#pragma unroll
          for (int u = 0; u < CW / 4; ++u) {
            const int c = c0 + 4 * u;
            const uint4 hv = c < DI / 2 ? ld_tile_row4_f32(lo, row, c) : ld_tile_row4_f32(hi, row, c - DI / 2);
            const float2 h01 = make_float2(__uint_as_float(hv.x), __uint_as_float(hv.y));
            const float2 h23 = make_float2(__uint_as_float(hv.z), __uint_as_float(hv.w));
            const float2 d01 =
                dsoftplus_mul_x2(make_float2(__uint_as_float(r[4 * u]), __uint_as_float(r[4 * u + 1])), h01);
            const float2 d23 =
                dsoftplus_mul_x2(make_float2(__uint_as_float(r[4 * u + 2]), __uint_as_float(r[4 * u + 3])), h23);
            o[2 * u] = pack_half2(d01.x, d01.y);
            o[2 * u + 1] = pack_half2(d23.x, d23.y);
            hp[2 * u] = pack_half2(h01.x, h01.y);
            hp[2 * u + 1] = pack_half2(h23.x, h23.y);
          }
          // every warp's fp32 reads of both half-slots are done before any
          // warp overwrites them (the column groups share rows)
          __syncwarp();
          if (lane == 0) mbar_arrive(bar_rd_done);
          ok = __all_sync(0xffffffffu, mbar_wait(bar_rd_done, (j * (L - 1) + (L - 1 - l)) & 1, abort_flag,
                                                 kDevTimeoutEpi));
          if (!ok) return;
#pragma unroll
          for (int u = 0; u < CW / 8; ++u) {
            st_tile_row8<DI>(lo, row, c0 + 8 * u, hp[4 * u], hp[4 * u + 1], hp[4 * u + 2], hp[4 * u + 3]);
            st_tile_row8<DI>(hi, row, c0 + 8 * u, o[4 * u], o[4 * u + 1], o[4 * u + 2], o[4 * u + 3]);
          }
          fence_proxy_async_smem();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) {
            mbar_arrive(bar_dz_full(s));
            mbar_arrive(bar_slot_empty(nlo % R));        // this warp is done with both
            mbar_arrive(bar_slot_empty((nlo + 1) % R));  // half-slots; the MMAs still read them
          }
        } else if constexpr (l > 0) {
          // dz_l = dh_l * softplus'(z_l) = dh_l * (1 - e^{-h_l}), h_l from its slot
          const int nh = i * NLD + (L - l);
          const uint32_t hb = slot_addr(nh % R);
          ok = __all_sync(0xffffffffu,
                          mbar_wait(bar_slot_full(nh % R), (nh / R) & 1, abort_flag, kDevTimeoutEpi));
          if (!ok) return;
#pragma unroll
          for (int u = 0; u < CW / 8; ++u) {
            const uint4 hv = ld_tile_row8<DI>(hb, row, c0 + 8 * u);
            const uint32_t hw[4] = {hv.x, hv.y, hv.z, hv.w};
#pragma unroll
            for (int jj = 0; jj < 4; ++jj) {
              const float2 dz = dsoftplus_mul_x2(
                  make_float2(__uint_as_float(r[8 * u + 2 * jj]), __uint_as_float(r[8 * u + 2 * jj + 1])),
                  half2_to_float2(hw[jj]));
              o[4 * u + jj] = pack_half2(dz.x, dz.y);
            }
          }
          __syncwarp();
          if (lane == 0) mbar_arrive(bar_slot_empty(nh % R));  // h_l read
          if constexpr (Cfg::DG_TS) {
            // dz_l -> TMEM for dgrad(l-1); its previous contents, dz_{l+1},
            // were read by dgrad(l), complete since its acc_full commit
            tmem_st_cols<CW / 2>(tmem_base + lane_off + Cfg::ZT_COL + s * Cfg::ZT_W + c0 / 2, o);
          }
          if constexpr (Cfg::G_TILES == 1) {
            // G still holds dz_{l+1} until this layer's wgrad has read it
            ok = __all_sync(0xffffffffu, mbar_wait(bar_wg_done(s), step & 1, abort_flag, kDevTimeoutEpi));
            if (!ok) return;
          }
          // With two G tiles, this step's tile was last read by the previous
          // step's MMAs, all complete: the accumulator's commit (waited above)
          // tracks every MMA the issuing thread had issued before it.
          const uint32_t sg = s_g(s, step);
#pragma unroll
          for (int u = 0; u < CW / 8; ++u)
            st_tile_row8<DI>(sg, row, c0 + 8 * u, o[4 * u], o[4 * u + 1], o[4 * u + 2], o[4 * u + 3]);
          fence_proxy_async_smem();
          if constexpr (Cfg::DG_TS) tmem_wait_st();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(bar_dz_full(s));
        } else {
          // dx = dh_0 -> fp16, staged in x's slot (free once the wgrad read x) -> TMA store
#pragma unroll
          for (int u = 0; u < CW / 8; ++u) pack_cols<4, false>(r + 8 * u, o + 4 * u);
          const int nx = i * NLD + NLD - 1;
          const uint32_t xb = slot_addr(nx % R);
          // wg_done completes once per layer step (fp16 h) or once per tile,
          // after wgrad(0) (fp32 h)
          const int wg_phase = H32 ? j : step;
          ok = __all_sync(0xffffffffu, mbar_wait(bar_wg_done(s), wg_phase & 1, abort_flag, kDevTimeoutEpi));
          if (!ok) return;
          // accumulator read.  Released only after the wg_done wait: the next
          // tile's first step (which needs acc_free) commits wg_done again, and
          // a parity wait cannot tell that phase from this one.
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(bar_acc_free(s));
#pragma unroll
          for (int u = 0; u < CW / 8; ++u)
            st_tile_row8<DI>(xb, row, c0 + 8 * u, o[4 * u], o[4 * u + 1], o[4 * u + 2], o[4 * u + 3]);
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) mbar_arrive(bar_out_ready(s));  // warp 0, lane 1 stores it
        }
      });
    }
    // dump this CTA's dW partials: accumulator lane = row of dW_l (or, transposed,
    // column); 16-column pieces are shared round-robin by the column groups
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
#pragma unroll 1
        for (int c = 16 * (s * NG + grp); c < NW; c += 16 * NS * NG) {
          uint32_t rr[16];
          tmem_ld_wait_x16(dw + c, rr);  // every lane takes part in the warp-wide load
          if (row < static_cast<uint32_t>(MW)) {
            if constexpr (!TR) {
              float4* dst = reinterpret_cast<float4*>(part + off + row * DO + c);
#pragma unroll
              for (int v = 0; v < 4; ++v)
                dst[v] = make_float4(__uint_as_float(rr[4 * v]), __uint_as_float(rr[4 * v + 1]),
                                     __uint_as_float(rr[4 * v + 2]), __uint_as_float(rr[4 * v + 3]));
            } else {
#pragma unroll
              for (int v = 0; v < 16; ++v) part[off + (c + v) * DO + row] = __uint_as_float(rr[v]);
            }
          }
        }
        off += NetT::dim(l) * DO;
      });
    }
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, Cfg::TMEM_COLS);
  }
}

// Level-2 reduction of the per-CTA partials: a block covers kReduceElems x
// VEC elements with kReduceSlices threads each (a thread reads VEC
// neighbouring elements per load: 16-byte loads when nfloats is a multiple of
// 4); slice s sums partials p = s, s + kReduceSlices, ... in increasing p, and
// the slices are added in slice order.  The order is fixed, so dW is bitwise
// reproducible (and independent of VEC).  blockIdx.y selects an independent
// group (nparts partials of nfloats each, written to dw + y * nfloats), e.g.
// one group per layer of the split-K wgrad kernel.
constexpr int kReduceElems = 64;
constexpr int kReduceSlices = 4;

// Where the reduced weight gradients go.  layers == 0: the caller's flat dW has
// the kernel network's layout (element e of group y lands at y * nfloats + e).
// Otherwise the caller's network is smaller than the kernel's (served by zero
// padding): element e of the kernel's flat layout (all groups concatenated) is
// row r, column c of layer l's [k_l][n_l] block at kernel offset koff[l]; it
// goes to the caller's [rk_l][rn_l] block at roff[l] when r < rk_l and c <
// rn_l, and is dropped otherwise (it is an exact zero: padded activations and
// data gradients are zero).
struct DwLayout {
  int layers;
  long long koff[9];
  int kn[8];
  int rk[8];
  int rn[8];
  long long roff[8];
};

template <int VEC>
struct ReduceVec;
template <>
struct ReduceVec<1> {
  using T = float;
  static __device__ __forceinline__ void add(float* a, T v) { a[0] += v; }
};
template <>
struct ReduceVec<4> {
  using T = float4;
  static __device__ __forceinline__ void add(float* a, T v) {
    a[0] += v.x;
    a[1] += v.y;
    a[2] += v.z;
    a[3] += v.w;
  }
};

template <int VEC>
__global__ void __launch_bounds__(kReduceElems * kReduceSlices)
    mlp_reduce_kernel(const float* __restrict__ partials, int nparts, int nfloats,
                      float* __restrict__ dw, const __grid_constant__ DwLayout lay) {
  pdl_enter();
  using V = ReduceVec<VEC>;
  using T = typename V::T;
  __shared__ float red[kReduceSlices][kReduceElems * VEC];
  partials += static_cast<size_t>(blockIdx.y) * nparts * nfloats;
  const int le = threadIdx.x % kReduceElems, sl = threadIdx.x / kReduceElems;
  const int e = (blockIdx.x * kReduceElems + le) * VEC;  // nfloats is a multiple of VEC
  float acc[VEC];
#pragma unroll
  for (int k = 0; k < VEC; ++k) acc[k] = 0.0f;
  if (e < nfloats) {
    // U loads in flight, added in increasing p (the fixed order)
    constexpr int U = 8;
    const size_t stride = static_cast<size_t>(nfloats) / VEC;
    const T* src = reinterpret_cast<const T*>(partials) + e / VEC;
    int p = sl;
    for (; p + (U - 1) * kReduceSlices < nparts; p += U * kReduceSlices) {
      T v[U];
#pragma unroll
      for (int u = 0; u < U; ++u) v[u] = src[static_cast<size_t>(p + u * kReduceSlices) * stride];
#pragma unroll
      for (int u = 0; u < U; ++u) V::add(acc, v[u]);
    }
    for (; p < nparts; p += kReduceSlices) V::add(acc, src[static_cast<size_t>(p) * stride]);
  }
#pragma unroll
  for (int k = 0; k < VEC; ++k) red[sl][le * VEC + k] = acc[k];
  __syncthreads();
  // the first kReduceElems x VEC threads finish one element each
  const int fe = threadIdx.x;
  if (fe < kReduceElems * VEC) {
    const int eo = blockIdx.x * kReduceElems * VEC + fe;
    if (eo < nfloats) {
      float t = red[0][fe];
#pragma unroll
      for (int k = 1; k < kReduceSlices; ++k) t += red[k][fe];
      const long long eg = static_cast<long long>(blockIdx.y) * nfloats + eo;
      if (lay.layers == 0) {
        dw[eg] = t;
      } else {
        int l = 0;
        while (l + 1 < lay.layers && eg >= lay.koff[l + 1]) ++l;
        const long long q = eg - lay.koff[l];
        const int r = static_cast<int>(q / lay.kn[l]);
        const int c = static_cast<int>(q % lay.kn[l]);
        if (r < lay.rk[l] && c < lay.rn[l]) dw[lay.roff[l] + static_cast<long long>(r) * lay.rn[l] + c] = t;
      }
    }
  }
}

}  // namespace mlpk
