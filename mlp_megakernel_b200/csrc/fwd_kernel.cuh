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
//    (two accumulator buffers per slot, alternating between layers, so layer
//    l+1 accumulates while the epilogue still drains layer l).
//  * warps 2..2+NS*EPW-1: epilogue, EPW warps per slot.  tcgen05.ld the
//    accumulator (warp w owns TMEM lanes 32*(w%4)..+31 = tile rows; the slot's
//    EPW/4 column groups split the columns), softplus in fp32 registers with
//    packed f32x2 math, cast to fp16 and tcgen05.st the activation back into
//    TMEM, packed two per column over the accumulator columns it has consumed.
//    The next layer's UMMA takes that activation as its A operand straight from
//    TMEM (kind::f16 with [a_tmem]), so a hidden-layer UMMA reads only its
//    weight tile from shared memory -- an SS UMMA at M=N=128 needs the whole
//    shared-memory bandwidth and runs at about half the tensor rate.  For the
//    last layer the fp16 result is staged in shared memory and written by TMA
//    stores (OOB rows of the last tile are clipped by TMA).  TMEM loads are
//    software-pipelined: the next 32 columns are in flight while the current 32
//    are computed.
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
  __host__ __device__ static constexpr int dim(int i) {
    constexpr int a[] = {Ds...};
    return a[i];
  }
  __host__ __device__ static constexpr bool all_dims_are(int v) {
    constexpr int a[] = {Ds...};
    for (int i = 0; i <= L; ++i)
      if (a[i] != v) return false;
    return true;
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
  // training forward only: the saved hidden activations h_1..h_{L-1}, [M, d_l]
  // each: fp16 (the exact values fed to the next GEMM), box {chunk(d_l), 128};
  // or fp32 (H32), box {32, 32}
  CUtensorMap hsave[L > 1 ? L - 1 : 1];
  int M;
  // The caller's widths when they are smaller than the kernel's network (a
  // network served by a larger one): the maps above carry the caller's
  // extents, so TMA loads fill the missing rows / columns with zeros, and the
  // stores skip every chunk that starts at or past these widths (partially
  // covered chunks are clipped by TMA).
  int out_cols;                     // caller's d_L
  int h_cols[L > 1 ? L - 1 : 1];   // caller's d_1 .. d_{L-1}
};

template <int I, int N, class F>
__host__ __device__ __forceinline__ void static_for(F&& f) {
  if constexpr (I < N) {
    f(std::integral_constant<int, I>{});
    static_for<I + 1, N>(f);
  }
}

// H32: the training forward saves the hidden activations in fp32 (the
// reference's storage, README.md:30) instead of the fp16 operand copy.
template <class NetT, int NS, int EPW, bool H32 = false>
struct FwdCfg {
  static constexpr int L = NetT::L;
  static constexpr int D0 = NetT::template D<0>();
  static constexpr int DL = NetT::template D<L>();
  static constexpr int HMAX = NetT::max_hidden_or_out();
  static constexpr int X_BYTES = align_up(tile_bytes(kTileM, D0), 1024);
  static constexpr int H1 = NetT::template D<1>();
  // staging tile of a slot: the output, and in the training forward also every
  // hidden activation (both written to HBM by TMA stores); with fp32 saved
  // activations at least two 16 KB piece buffers (4 warps x 32 x 32 fp32)
  static constexpr int O_BYTES_BASE = align_up(tile_bytes(kTileM, DL > H1 ? DL : H1), 1024);
  static constexpr int O_BYTES = H32 && O_BYTES_BASE < 2 * 16384 ? 2 * 16384 : O_BYTES_BASE;
  static constexpr int NPB = O_BYTES / 16384;  // fp32 piece buffers per slot (H32)
  static constexpr int W_TOTAL = NetT::w_total();
  static constexpr int OFF_X = W_TOTAL;
  static constexpr int OFF_O = OFF_X + NS * X_BYTES;
  static constexpr int OFF_BAR = OFF_O + NS * O_BYTES;
  // Hidden activations are handed to the MMA warp in chunks: a chunk is one
  // 32-column stripe from every column group (32*NG columns); its barrier
  // counts all EPW warps of the slot.
  // SPC: stripes per chunk per column group (chunk = SPC*NG stripes).
  static constexpr int SPC = (HMAX / (EPW / 4)) / 32 >= 4 ? 2 : 1;
  static constexpr int MAXCH = ((HMAX / (EPW / 4) + 31) / 32 + SPC - 1) / SPC;  // chunks/layer
  // x_full, x_empty, out_ready, store_free per slot; acc_full per slot and
  // accumulator buffer; MAXCH h-chunk barriers per slot; w_full per layer;
  // mma_done; (H32) pieces_done per slot
  static constexpr int NUM_BARS = 6 * NS + NS * MAXCH + L + 1 + NS;
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
  static_assert(!H32 || EPW == 4, "fp32 saved activations: one column group (a warp owns 32 rows)");
  static_assert(!H32 || H % 32 == 0, "fp32 saved activations are stored in 32-column pieces");
};

// TMEM column (relative to the accumulator buffer) where the fp16 activation
// of accumulator column `col` is stored: columns are processed in 32-column
// stripes, and each stripe's activation is packed two per 32-bit TMEM column
// into the first 16 columns of that stripe's own range.
__host__ __device__ constexpr int h_tmem_col(int col) { return (col / 32) * 32 + (col % 32) / 2; }

// Packs 2*NP fp32 values to NP half2 words, through softplus when ACT.
template <int NP, bool ACT>
__device__ __forceinline__ void pack_cols(const uint32_t* r, uint32_t* w) {
#pragma unroll
  for (int j = 0; j < NP; ++j) {
    float2 z = make_float2(__uint_as_float(r[2 * j]), __uint_as_float(r[2 * j + 1]));
    if constexpr (ACT) z = softplus_x2(z);
    w[j] = pack_half2(z.x, z.y);
  }
}

// Publishes one finished chunk of h to the MMA issuer: the TMEM stores are
// complete and ordered (with this chunk's TMEM loads) before the arrive.
__device__ __forceinline__ void publish_chunk(uint32_t bar) {
  tmem_wait_st();
  tc_fence_before();
  __syncwarp();
  if (lane_id() == 0) mbar_arrive(bar);
}

// Hidden-layer job of one warp of column group `grp` (of NG): stripes
// grp, grp+NG, grp+2NG, ... (32 columns each) of the accumulator buffer at
// TMEM address tbuf (lane field = the warp's quarter) -> softplus -> fp16 back
// into TMEM at h_tmem_col(); after every SPC stripes it arrives on the next
// chunk barrier (chunk_bar0 + 8*(j/SPC)), which completes once all NG groups
// finished those stripes.  SAVE = 1 also writes the fp16 activation to this
// thread's row in global memory (hrow), SAVE = 2 into the swizzled staging
// tile at stage_base (row `row`) for a TMA store.  A
// column is always loaded before the packed activation overwrites it: a
// stripe's packed columns lie in its own range, and the async load of the
// next stripe is issued before this stripe's store.
// Where SAVE = 3 (fp32 saved activations) stages and stores one warp's
// stripes: NPB piece buffers of 4 KB per warp (32 rows x 32 fp32, 128-byte
// rows, 128B swizzle: the layout of a TMA box {32, 32} of an fp32 tensor).
// Stripe k of the warp goes to piece buffer k % NPB at
// base + (k % NPB) * (4 * 4096) + quarter * 4096; the warp's lane 0 stores it
// to rows [row0, row0 + 32) and columns [col, col + 32) of the saved tensor
// (TMA clips rows past M; a box that starts at or past M or past the
// caller's width hcols is skipped) and keeps at most NPB stores in flight.
struct F32Save {
  const CUtensorMap* map;
  uint32_t base;  // the slot's staging region (1024-aligned)
  int quarter;    // this warp's TMEM lane quarter (its 32 rows of the tile)
  int row0;       // first tile row of this warp in the tensor
  int M;
  int hcols;
  int* count;     // pieces this warp has written so far (across layers and tiles)
};

template <int NPB>
__device__ __forceinline__ uint32_t f32_piece_begin(const F32Save& fs) {
  const int k = *fs.count;
  if (k >= NPB) {  // the store that used this buffer NPB pieces ago must have read it
    if (lane_id() == 0) bulk_wait_group_read<NPB - 1>();
    __syncwarp();
  }
  return fs.base + static_cast<uint32_t>((k % NPB) * 4 + fs.quarter) * 4096u;
}

template <int NPB>
__device__ __forceinline__ void f32_piece_end(const F32Save& fs, uint32_t buf, int col) {
  fence_proxy_async_smem();
  __syncwarp();
  if (lane_id() == 0) {
    if (fs.row0 < fs.M && col < fs.hcols) tma_store_2d(fs.map, buf, col, fs.row0);
    bulk_commit_group();  // one group per piece (possibly empty): the ring arithmetic stays exact
  }
  ++*fs.count;
}

template <int N, int NG, int SPC, int SAVE = 0, int NPB = 2>
__device__ __forceinline__ void hidden_job(uint32_t tbuf, int grp, uint32_t chunk_bar0,
                                           uint8_t* hrow = nullptr, uint32_t stage_base = 0,
                                           uint32_t row = 0, const F32Save* fs = nullptr) {
  static_assert(N % (32 * NG) == 0, "hidden width must be a multiple of 32 * column groups");
  constexpr int SUBS = N / (32 * NG);
  static_assert(SUBS % SPC == 0, "stripes per chunk must divide the stripes per group");
  uint32_t a[32];
  tmem_ld_wait_x32(tbuf + 32 * grp, a);
#pragma unroll
  for (int j = 0; j < SUBS; ++j) {
    const int col = 32 * (j * NG + grp);
    uint32_t b[32];
    if (j + 1 < SUBS) tmem_ld_async_x32(tbuf + col + 32 * NG, b);
    uint32_t w[16];
    if constexpr (SAVE == 3) {
      // fp32 h of this stripe into the warp's piece buffer (row = lane), then
      // one TMA store of the warp's 32 x 32 box; the fp16 pack feeds TMEM
      const uint32_t buf = f32_piece_begin<NPB>(*fs);
      const uint32_t lane = lane_id();
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const float2 z0 = softplus_x2(make_float2(__uint_as_float(a[4 * u]), __uint_as_float(a[4 * u + 1])));
        const float2 z1 = softplus_x2(make_float2(__uint_as_float(a[4 * u + 2]), __uint_as_float(a[4 * u + 3])));
        st_shared_v4(buf + swz_off<128>(lane, u), __float_as_uint(z0.x), __float_as_uint(z0.y),
                     __float_as_uint(z1.x), __float_as_uint(z1.y));
        w[2 * u] = pack_half2(z0.x, z0.y);
        w[2 * u + 1] = pack_half2(z1.x, z1.y);
      }
      f32_piece_end<NPB>(*fs, buf, col);
    } else {
      pack_cols<16, true>(a, w);
    }
    tmem_st_x16(tbuf + h_tmem_col(col), w);
    if constexpr (SAVE == 1) {
      if (hrow != nullptr) {  // this thread's row exists (row < M): save h for backward
        uint4* dst = reinterpret_cast<uint4*>(hrow + 2 * col);
#pragma unroll
        for (int v = 0; v < 4; ++v)
          dst[v] = make_uint4(w[4 * v], w[4 * v + 1], w[4 * v + 2], w[4 * v + 3]);
      }
    } else if constexpr (SAVE == 2) {
      constexpr int C = chunk_elems(N);
      constexpr int P = pitch_bytes(N);
#pragma unroll
      for (int v = 0; v < 4; ++v) {
        const int cc = col + 8 * v;
        st_shared_v4(stage_base + (cc / C) * (kTileM * P) + swz_off<P>(row, (cc % C) / 8), w[4 * v],
                     w[4 * v + 1], w[4 * v + 2], w[4 * v + 3]);
      }
    }
    if ((j + 1) % SPC == 0) publish_chunk(chunk_bar0 + 8 * (j / SPC));
    if (j + 1 < SUBS) {
      tmem_wait_ld_bind_x32(b);
#pragma unroll
      for (int i = 0; i < 32; ++i) a[i] = b[i];
    }
  }
}

// Output-layer job of one warp: NCOL accumulator columns -> fp16 -> the
// swizzled smem staging tile of extent N (TMA-store layout, layout.cuh).
template <int N, int NCOL>
__device__ __forceinline__ void out_job(uint32_t tbuf, uint32_t tile_base, uint32_t row, int col0) {
  constexpr int C = chunk_elems(N);
  constexpr int P = pitch_bytes(N);
  constexpr int CH = NCOL < 32 ? NCOL : 32;
  static_assert(NCOL % CH == 0 && CH % 8 == 0, "unsupported width");
#pragma unroll
  for (int c = 0; c < NCOL; c += CH) {
    uint32_t r[CH];
    if constexpr (CH == 32) tmem_ld_wait_x32(tbuf + col0 + c, r);
    if constexpr (CH == 16) tmem_ld_wait_x16(tbuf + col0 + c, r);
    if constexpr (CH == 8) tmem_ld_wait_x8(tbuf + col0 + c, r);
#pragma unroll
    for (int u = 0; u < CH / 8; ++u) {
      uint32_t w[4];
      pack_cols<4, false>(r + 8 * u, w);
      const int cc = col0 + c + 8 * u;
      st_shared_v4(tile_base + (cc / C) * (kTileM * P) + swz_off<P>(row, (cc % C) / 8), w[0],
                   w[1], w[2], w[3]);
    }
  }
}

template <class NetT, int NS, int EPW, bool TRAIN = false, bool H32 = false>
__global__ void __launch_bounds__(FwdCfg<NetT, NS, EPW, H32>::THREADS, 1)
    mlp_fwd_kernel(const __grid_constant__ FwdMaps<NetT::L> maps, int num_tiles) {
  using Cfg = FwdCfg<NetT, NS, EPW, H32>;
  static_assert(TRAIN || !H32, "fp32 saved activations belong to the training forward");
  constexpr int L = Cfg::L;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t sbase = (raw + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (sbase - raw);

  const uint32_t s_w = sbase;
  const uint32_t s_x = sbase + Cfg::OFF_X;
  const uint32_t s_o = sbase + Cfg::OFF_O;
  const uint32_t s_bar = sbase + Cfg::OFF_BAR;
  auto bar_x_full = [&](int s) { return s_bar + 8u * s; };
  auto bar_x_empty = [&](int s) { return s_bar + 8u * (NS + s); };
  // Accumulator of job g (= i*L + l) of slot s is complete: one barrier per
  // TMEM buffer (g & 1), waited with parity (g >> 1) & 1.  A single barrier per
  // slot could complete two phases before a slow epilogue warp polls it (a
  // layer-0 job of the next tile depends on no epilogue work), and a parity
  // wait cannot tell phase p from p + 2.  Per buffer this cannot happen: of
  // jobs g + 1 and g + 2 at least one has layer >= 1 and waits for the
  // epilogue's activation of the job before it, so the epilogue has consumed
  // job g before job g + 2 can commit.
  auto bar_acc_full = [&](int s, int b) { return s_bar + 8u * (2 * NS + 2 * s + b); };
  auto bar_out_ready = [&](int s) { return s_bar + 8u * (4 * NS + s); };
  auto bar_store_free = [&](int s) { return s_bar + 8u * (5 * NS + s); };
  // h chunk c of slot s: activation columns [32c, 32c+32), packed in TMEM
  auto bar_chunk = [&](int s, int c) { return s_bar + 8u * (6 * NS + s * Cfg::MAXCH + c); };
  // layer l's weights have landed (one barrier per layer, so layer 0 of the
  // first tile starts while the later layers' weights are still in flight)
  auto bar_w_full = [&](int l) { return s_bar + 8u * (6 * NS + NS * Cfg::MAXCH + l); };
  const uint32_t bar_mma_done = bar_w_full(L);
  // (H32) every warp of slot s has seen its fp32 piece stores read: the
  // output tile may overwrite the staging region
  auto bar_pieces_done = [&](int s) { return bar_mma_done + 8u + 8u * s; };
  const uint32_t s_tmem_slot = sbase + Cfg::OFF_MISC;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(gbase + Cfg::OFF_MISC + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(bar_x_full(s), 1);
      mbar_init(bar_x_empty(s), 1);
      mbar_init(bar_acc_full(s, 0), 1);
      mbar_init(bar_acc_full(s, 1), 1);
      mbar_init(bar_out_ready(s), EPW);
      mbar_init(bar_store_free(s), 1);
      for (int c = 0; c < Cfg::MAXCH; ++c) mbar_init(bar_chunk(s, c), EPW);
      mbar_init(bar_pieces_done(s), EPW);
    }
    for (int l = 0; l < L; ++l) mbar_init(bar_w_full(l), 1);
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
  pdl_enter();

  const int G = gridDim.x;
  auto tile_of = [&](int p, int s) { return static_cast<int>(blockIdx.x) + (p * NS + s) * G; };

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      tma_prefetch_desc(&maps.x);
      tma_prefetch_desc(&maps.out);
      // weights of layers [l0, l1), each on its own barrier
      auto load_weights = [&](auto l0c, auto l1c) {
        static_for<decltype(l0c)::value, decltype(l1c)::value>([&](auto lc) {
          constexpr int l = decltype(lc)::value;
          constexpr int K = NetT::template D<l>();
          constexpr int N = NetT::template D<l + 1>();
          constexpr int C = chunk_elems(N);
          constexpr int P = pitch_bytes(N);
          mbar_arrive_expect_tx(bar_w_full(l), tile_bytes(K, N));
#pragma unroll
          for (int c = 0; c < N / C; ++c)
            tma_load_2d(s_w + NetT::template w_off<l>() + c * K * P, &maps.w[l], bar_w_full(l), c * C, 0);
        });
      };
      // layer 0's weights, then the first round of x tiles, then the rest
      load_weights(std::integral_constant<int, 0>{}, std::integral_constant<int, 1>{});
      bool rest_loaded = false;
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
        if (!rest_loaded) {
          load_weights(std::integral_constant<int, 1>{}, std::integral_constant<int, L>{});
          rest_loaded = true;
        }
      }
      if (!rest_loaded) load_weights(std::integral_constant<int, 1>{}, std::integral_constant<int, L>{});
      // Drain: never leave the CTA with a TMA load still writing shared memory.
      volatile int no_abort = 0;
      for (int l = 0; l < L; ++l) mbar_wait(bar_w_full(l), 0, &no_abort, kDevTimeoutFull);
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
    // The whole warp runs the loop (waits and descriptors are warp-uniform, so
    // they live in uniform registers); lane 0 issues the tcgen05 instructions.
    const bool issuer = (lane == 0);
    bool ok = true;
    for (int i = 0; ok; ++i) {
      if (tile_of(i, 0) >= num_tiles) break;
      static_for<0, L>([&](auto lc) {
        constexpr int l = decltype(lc)::value;
        constexpr int K = NetT::template D<l>();
        constexpr int N = NetT::template D<l + 1>();
        constexpr uint32_t idesc = make_idesc_f16(kTileM, N, 0, 1);
        const uint64_t bdesc0 = mnmajor_base_desc<K, N>(s_w + NetT::template w_off<l>());
        if (i == 0 && ok) {  // this layer's weights, before their first use
          ok = __all_sync(0xffffffffu, mbar_wait(bar_w_full(l), 0, abort_flag, kDevTimeoutMma));
          tc_fence_after();
        }
#pragma unroll
        for (int s = 0; s < NS; ++s) {
          if (!ok || tile_of(i, s) >= num_tiles) break;
          const uint32_t d_tmem = tmem_base + (2 * s + ((i * L + l) & 1)) * Cfg::SLOT_COLS;
          if constexpr (l == 0) {
            ok = __all_sync(0xffffffffu,
                            mbar_wait(bar_x_full(s), i & 1, abort_flag, kDevTimeoutMma));
            if (!ok) break;
            tc_fence_after();
            const uint64_t adesc0 = kmajor_base_desc<K>(s_x + s * Cfg::X_BYTES);
            if (issuer) {
#pragma unroll
              for (int k = 0; k < K / 16; ++k)
                umma_f16(d_tmem, adesc0 + (kmajor_koff<kTileM, K>(k) >> 4),
                         bdesc0 + (mnmajor_koff<N>(k) >> 4), idesc, k > 0 ? 1u : 0u);
              umma_commit(bar_x_empty(s));
            }
            __syncwarp();
          } else {
            // chunk j of h_{l-1} = stripe j of every column group (32*NG
            // columns), complete once all epilogue warps of the slot arrived.
            // A comes from TMEM: the previous job's buffer, where the
            // epilogue packed h_{l-1} (h_tmem_col).
            constexpr int NGRP = Cfg::NG;
            constexpr int SPC = Cfg::SPC;
            constexpr int NCH = K / (32 * NGRP * SPC);
            static_assert(NCH >= 1 && K % (32 * NGRP * SPC) == 0, "hidden width vs chunks");
            const uint32_t a_tmem = tmem_base + (2 * s + ((i * L + l - 1) & 1)) * Cfg::SLOT_COLS;
            const uint32_t par = (i * (L - 1) + l - 1) & 1;
#pragma unroll
            for (int j = 0; j < NCH; ++j) {
              ok = __all_sync(0xffffffffu,
                              mbar_wait(bar_chunk(s, j), par, abort_flag, kDevTimeoutMma));
              if (!ok) break;
              tc_fence_after();
              if (issuer) {
#pragma unroll
                for (int js = 0; js < SPC; ++js) {
#pragma unroll
                  for (int g = 0; g < NGRP; ++g) {
#pragma unroll
                    for (int kk = 0; kk < 2; ++kk) {
                      const int k = 2 * ((j * SPC + js) * NGRP + g) + kk;  // K-step
                      umma_f16_ts(d_tmem, a_tmem + h_tmem_col(16 * k),
                                  bdesc0 + (mnmajor_koff<N>(k) >> 4), idesc,
                                  (j == 0 && js == 0 && g == 0 && kk == 0) ? 0u : 1u);
                    }
                  }
                }
              }
              __syncwarp();
            }
            if (!ok) break;
          }
          if (issuer) umma_commit(bar_acc_full(s, (i * L + l) & 1));
          __syncwarp();
        }
      });
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
    const int s = e / EPW;             // slot served by this warp
    const int ew = e % EPW;            // warp index inside the slot group
    const int q = warp & 3;            // TMEM lane quarter this warp may access
    const int grp = ew >> 2;           // column group
    const uint32_t row = q * 32 + lane;
    const uint32_t t_lane = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + 2 * s * Cfg::SLOT_COLS;
    const uint32_t obuf = s_o + s * Cfg::O_BYTES;
    const bool leader = (ew == 0 && lane == 0);
    bool ok = true;
    constexpr int H = Cfg::H;
    constexpr int NCOL_H = H / Cfg::NG;
    constexpr int NCOL_O = Cfg::DL / Cfg::NG;
    int pieces = 0;  // (H32) fp32 pieces this warp has staged
    for (int i = 0; ok; ++i) {
      const int t = tile_of(i, s);
      if (t >= num_tiles) break;
      // hidden layers: softplus, fp16 activation published chunk by chunk
#pragma unroll 1
      for (int l = 0; l < L - 1; ++l) {
        ok = __all_sync(0xffffffffu, mbar_wait(bar_acc_full(s, (i * L + l) & 1),
                                               ((i * L + l) >> 1) & 1, abort_flag, kDevTimeoutEpi));
        if (!ok) break;
        tc_fence_after();
        // obuf may still be the source of this slot's previous TMA store: the
        // leader waits for that store to finish reading, then frees it.  Uses
        // of obuf by the leader's stores: one per tile (the output) or, in the
        // fp16 training forward, one per layer (every h_l, then the output).
        // The fp32 training forward stages h in per-warp pieces, each warp
        // pacing its own stores (F32Save), so only the output counts.
        constexpr bool kLayerUses = TRAIN && !H32;
        const int use = kLayerUses ? i * L + l : i;
        if ((kLayerUses || l == 0) && use > 0) {
          if (leader) {
            bulk_wait_group_read<0>();
            mbar_arrive(bar_store_free(s));
          }
          __syncwarp();
          ok = __all_sync(0xffffffffu,
                          mbar_wait(bar_store_free(s), (use - 1) & 1, abort_flag, kDevTimeoutEpi));
          if (!ok) break;
        }
        const uint32_t t_buf = t_lane + ((i * L + l) & 1) * Cfg::SLOT_COLS;
        if constexpr (H32) {
          // h_l -> TMEM (next layer's A, fp16) and, in fp32, per-warp pieces
          // -> TMA stores
          const F32Save fs{&maps.hsave[l], obuf, q, t * kTileM + q * 32, maps.M, maps.h_cols[l], &pieces};
          hidden_job<H, Cfg::NG, Cfg::SPC, 3, Cfg::NPB>(t_buf, grp, bar_chunk(s, 0), nullptr, 0, row, &fs);
        } else if constexpr (TRAIN) {
          // h_l -> TMEM (next layer's A) and the staging tile -> TMA store
          hidden_job<H, Cfg::NG, Cfg::SPC, 2>(t_buf, grp, bar_chunk(s, 0), nullptr, obuf, row);
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) mbar_arrive(bar_out_ready(s));
          if (leader) {
            ok = mbar_wait(bar_out_ready(s), use & 1, abort_flag, kDevTimeoutEpi);
            if (ok) {
              constexpr int C = chunk_elems(H);
              constexpr int P = pitch_bytes(H);
#pragma unroll
              for (int c = 0; c < H / C; ++c)
                if (c * C < maps.h_cols[l]) tma_store_2d(&maps.hsave[l], obuf + c * kTileM * P, c * C, t * kTileM);
              bulk_commit_group();
            }
          }
          ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
          if (!ok) break;
        } else {
          hidden_job<H, Cfg::NG, Cfg::SPC>(t_buf, grp, bar_chunk(s, 0));
        }
      }
      if (!ok) break;
      // output layer: fp16 result staged in obuf, written by TMA
      {
        constexpr int l = L - 1;
        ok = __all_sync(0xffffffffu, mbar_wait(bar_acc_full(s, (i * L + l) & 1),
                                               ((i * L + l) >> 1) & 1, abort_flag, kDevTimeoutEpi));
        if (!ok) break;
        tc_fence_after();
        constexpr bool kLayerUses = TRAIN && !H32;
        const int use = kLayerUses ? i * L + l : i;
        if constexpr (H32) {
          // the output tile overlaps every warp's piece buffers: each warp
          // waits for its own piece stores to have read them, then all warps
          // of the slot meet
          if (lane == 0) bulk_wait_group_read<0>();
          __syncwarp();
          if (lane == 0) mbar_arrive(bar_pieces_done(s));
          ok = __all_sync(0xffffffffu, mbar_wait(bar_pieces_done(s), i & 1, abort_flag, kDevTimeoutEpi));
          if (!ok) break;
        } else if constexpr (TRAIN) {  // obuf held h_{L-1}: wait until its store has read it
          if (leader) {
            bulk_wait_group_read<0>();
            mbar_arrive(bar_store_free(s));
          }
          __syncwarp();
          ok = __all_sync(0xffffffffu,
                          mbar_wait(bar_store_free(s), (use - 1) & 1, abort_flag, kDevTimeoutEpi));
          if (!ok) break;
        }
        const uint32_t t_buf = t_lane + ((i * L + l) & 1) * Cfg::SLOT_COLS;
        out_job<Cfg::DL, NCOL_O>(t_buf, obuf, row, grp * NCOL_O);
        fence_proxy_async_smem();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar_out_ready(s));
        if (leader) ok = mbar_wait(bar_out_ready(s), use & 1, abort_flag, kDevTimeoutEpi);
        ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
        if (leader && ok) {
          constexpr int C = chunk_elems(Cfg::DL);
          constexpr int P = pitch_bytes(Cfg::DL);
#pragma unroll
          for (int c = 0; c < Cfg::DL / C; ++c)
            if (c * C < maps.out_cols) tma_store_2d(&maps.out, obuf + c * kTileM * P, c * C, t * kTileM);
          bulk_commit_group();
        }
      }
    }
    // every store this warp issued (the leader's tiles, and with fp32 saved
    // activations every warp's pieces) completes before the CTA exits
    if (lane == 0) bulk_wait_group<0>();
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
