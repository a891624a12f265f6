// Fused softplus-MLP chain with STREAMED weights, for networks whose fp16
// weights do not fit in shared memory next to the activation tiles (the
// wide D = H = OUT = 256 network: 3 x 128 KB of weights).
//
// One kernel template serves two chains:
//
//  * forward (kStreamFwd), the reference's _fused_mlp_recompute
//    (kernel.py:60-123) for the wide network, plus the training forward that
//    also saves every hidden activation (mlp_fused.md:52-61):
//      stage s: z = h_s @ W_s (K = d_s, N = d_{s+1}); h_{s+1} = softplus(z)
//  * data-gradient chain (kStreamDgrad) of the backward (mlp_fused.md:87-95):
//      stage s (layer l = L-1-s): dh_l = dz_{l+1} @ W_l^T; dz_l = dh_l * (1 - e^{-h_l})
//    which also writes every dz_l to global memory for the weight-gradient
//    kernel (wgrad_kernel.cuh) and dx for the last stage.
//
// Design (persistent, one CTA per SM, one 128-row tile in flight):
//  * warp 0, one lane: TMA producer.  The input tile (x, or grad_out) into a
//    shared buffer; then, for every stage of the tile, the weight in 64-row
//    K-chunks through a 3-deep ring (64 x 256 fp16 = 32 KB per chunk).  The
//    forward reads W_s as stored ([K][N], N contiguous: MN-major B); the
//    data-gradient chain reads W_l^T, i.e. K-chunks of W_l's columns
//    ([N rows][64 K]: K-major B).  Weights come from L2 after the first tile.
//  * warp 1: TMEM owner and MMA issuer.  Two accumulator buffers of up to 256
//    fp32 columns (TMEM = 512 columns); job g = tile*L + stage uses buffer
//    g & 1.  Stage 0 takes A from the input tile in shared memory; later
//    stages take A from TMEM, where the epilogue packed the previous stage's
//    fp16 result (tcgen05.mma ... [a_tmem]), chunk by chunk as published.
//  * EPW epilogue warps (4 per column group): tcgen05.ld the accumulator,
//    apply the stage's elementwise function in fp32, tcgen05.st the fp16
//    result back into TMEM for the next stage; a saved stage result (h in the
//    training forward, dz in the data-gradient chain) and the last stage's
//    output go through one shared-memory staging tile and TMA stores.
//  * All hand-offs are mbarriers and every wait is bounded (ptx.cuh).
#pragma once
#include "bwd_kernel.cuh"

namespace mlpk {

constexpr int kStreamK = 64;  // K rows of one streamed weight chunk
enum StreamMode : int { kStreamFwd = 0, kStreamDgrad = 1 };

// Net<d_L, ..., d_0> from Net<d_0, ..., d_L>: the data-gradient chain.
template <class Acc, class Rest>
struct NetRevImpl;
template <int... A>
struct NetRevImpl<Net<A...>, Net<>> {
  using type = Net<A...>;
};
template <int... A, int D, int... R>
struct NetRevImpl<Net<A...>, Net<D, R...>> {
  using type = typename NetRevImpl<Net<D, A...>, Net<R...>>::type;
};
template <class NetT>
using NetReverse = typename NetRevImpl<Net<>, NetT>::type;

template <int L>
struct alignas(64) StreamMaps {
  CUtensorMap in;    // stage-0 input [M, d_0 of the chain], box {64, 128}
  CUtensorMap out;   // last-stage output [M, d_L of the chain], box {64, 128}
  CUtensorMap w[L];  // stage s weight chunks (see the producer)
  // fp16 [M, d_{s+1}] result of hidden stage s, box {64, 128} (written when SAVE)
  CUtensorMap save[L > 1 ? L - 1 : 1];
  const void* hact[L > 1 ? L - 1 : 1];  // dgrad: saved h_l read by stage s (l = L-1-s)
  int M;
  // The caller's widths when they are smaller than the kernel's network (a
  // network served by a larger one): the maps carry the caller's extents, so
  // TMA loads fill the missing rows / columns with zeros; stores skip every
  // 64-column chunk that starts at or past these widths (partially covered
  // chunks are clipped by TMA); hact rows have hact_cols columns and the
  // columns past them read as zero.
  int out_cols;
  int save_cols[L > 1 ? L - 1 : 1];
  int hact_cols[L > 1 ? L - 1 : 1];
};

// TF32: fp32 input, weights and output, tf32 tensor-core GEMMs and fp32
// hidden activations (the reference's INPUT_DTYPE fp32 design,
// mlp_fused.md:159-166); inference forward only.  Every shared-memory row is
// 128 bytes: 32 fp32 columns per chunk instead of 64 fp16 ones.
template <class ChainT, int EPW, bool TF32 = false>
struct StreamCfg {
  static constexpr int L = ChainT::L;
  static constexpr int D0 = ChainT::template D<0>();
  static constexpr int DL = ChainT::template D<L>();
  static constexpr int H = ChainT::template D<1>();
  static constexpr int HMAX = ChainT::max_hidden_or_out();
  static constexpr int NG = EPW / 4;  // column groups
  static constexpr int NWBUF = 3;
  static constexpr int ES = TF32 ? 4 : 2;   // element bytes
  static constexpr int CB = 128 / ES;       // columns of one 128-byte chunk
  static constexpr int KSTEP = TF32 ? 8 : 16;  // K of one UMMA
  static constexpr int WCH_BYTES = kStreamK * HMAX * ES;
  static constexpr int X_BYTES = align_up(kTileM * D0 * ES, 1024);
  static constexpr int O_BYTES = align_up(kTileM * DL * ES, 1024);
  static constexpr int OFF_W = 0;
  static constexpr int OFF_X = NWBUF * WCH_BYTES;
  static constexpr int OFF_O = OFF_X + X_BYTES;
  static constexpr int OFF_BAR = OFF_O + O_BYTES;
  // hidden results are published in chunks of CH_COLS columns (SPC stripes of
  // 32 columns from every column group)
  static constexpr int SPC = (H / NG) / 32 >= 4 ? 2 : 1;
  static constexpr int CH_COLS = 32 * NG * SPC;
  static constexpr int MAXCH = H / CH_COLS;
  // x_full, x_empty, w_full[NWBUF], w_empty[NWBUF], acc_full[2], out_ready,
  // store_free, chunk[MAXCH], mma_done
  static constexpr int NUM_BARS = 2 + 2 * NWBUF + 2 + 2 + MAXCH + 1;
  static constexpr int OFF_MISC = OFF_BAR + 8 * NUM_BARS;
  static constexpr int SMEM_BYTES = OFF_MISC + 16 + 1024;
  static constexpr int SLOT_COLS = align_up(HMAX, 32);
  static constexpr int TMEM_COLS_RAW = 2 * SLOT_COLS;
  static constexpr int TMEM_COLS = TMEM_COLS_RAW <= 128 ? 128 : TMEM_COLS_RAW <= 256 ? 256 : 512;
  static constexpr int THREADS = (2 + EPW) * 32;
  __host__ __device__ static constexpr bool dims_ok() {
    for (int i = 0; i <= L; ++i)
      if (ChainT::dim(i) % CB != 0 || ChainT::dim(i) > (TF32 ? 128 : 256)) return false;
    return true;
  }
  static_assert(EPW % 4 == 0, "epilogue warps come in groups of 4");
  static_assert(dims_ok(), "streamed chain needs every width a multiple of 64 (fp32: 32), at most 256 (fp32: 128)");
  static_assert(ChainT::hidden_uniform(), "all hidden layers must have the same width");
  static_assert(H % CH_COLS == 0, "hidden width vs publish chunks");
  static_assert(TMEM_COLS_RAW <= 512, "accumulators exceed TMEM");
  static_assert(SMEM_BYTES <= 232448, "shared memory budget exceeded");
};

// Loads this thread's saved activations of stripe j of one data-gradient
// stage: stripe j of column group grp covers columns 32*(j*NG + grp) .. +31
// (64 bytes).  Rows past M (hrow == nullptr) and columns at or past the row's
// width hcols (a multiple of 8) get zeros.
template <int NG>
__device__ __forceinline__ void dgrad_load_h(uint4 (&hv)[4], const uint8_t* hrow, int grp, int j,
                                             int hcols) {
  const int col = 32 * (j * NG + grp);
#pragma unroll
  for (int v = 0; v < 4; ++v)
    hv[v] = (hrow && col + 8 * v < hcols) ? __ldg(reinterpret_cast<const uint4*>(hrow + 2 * col) + v)
                                          : make_uint4(0, 0, 0, 0);
}

// Data-gradient stage epilogue of one warp (mirrors hidden_job): dz = dh *
// (1 - e^{-h}) for the thread's row over the group's stripes, fp16 result
// packed into TMEM at h_tmem_col() for the next stage's A operand, optionally
// staged for a TMA store (SAVE), chunks published as in hidden_job.  hv holds the
// first two stripes' h (loaded before the accumulator wait); each later
// stripe's h is loaded two stripes ahead, into the registers just consumed.
template <int N, int NG, int SPC, bool SAVE>
__device__ __forceinline__ void dgrad_job(uint32_t tbuf, int grp, uint32_t chunk_bar0, uint4 (&hv)[2][4],
                                          const uint8_t* hrow, int hcols, uint32_t stage_base, uint32_t row) {
  constexpr int SUBS = N / (32 * NG);
  static_assert(SUBS % SPC == 0, "stripes per chunk must divide the stripes per group");
  uint32_t a[32];
  tmem_ld_wait_x32(tbuf + 32 * grp, a);
#pragma unroll
  for (int j = 0; j < SUBS; ++j) {
    const int col = 32 * (j * NG + grp);
    uint32_t b[32];
    if (j + 1 < SUBS) tmem_ld_async_x32(tbuf + col + 32 * NG, b);
    uint4(&hc)[4] = hv[j & 1];
    const uint32_t hw[16] = {hc[0].x, hc[0].y, hc[0].z, hc[0].w, hc[1].x, hc[1].y, hc[1].z, hc[1].w,
                             hc[2].x, hc[2].y, hc[2].z, hc[2].w, hc[3].x, hc[3].y, hc[3].z, hc[3].w};
    if (j + 2 < SUBS) dgrad_load_h<NG>(hc, hrow, grp, j + 2, hcols);
    uint32_t w[16];
#pragma unroll
    for (int p = 0; p < 16; ++p) {
      const float2 dz = dsoftplus_mul_x2(
          make_float2(__uint_as_float(a[2 * p]), __uint_as_float(a[2 * p + 1])), half2_to_float2(hw[p]));
      w[p] = pack_half2(dz.x, dz.y);
    }
    tmem_st_x16(tbuf + h_tmem_col(col), w);
    if constexpr (SAVE) {  // into the swizzled staging tile (TMA-store layout)
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

// fp32 hidden-stage job (TF32 chain) of one warp: like hidden_job, but the
// softplus result stays fp32 and goes back into the accumulator columns it
// came from (one 32-bit TMEM column per element: the next stage's tf32 A).
template <int N, int NG, int SPC>
__device__ __forceinline__ void hidden_job_f32(uint32_t tbuf, int grp, uint32_t chunk_bar0) {
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
#pragma unroll
    for (int p = 0; p < 16; ++p) {
      const float2 z = softplus_x2(make_float2(__uint_as_float(a[2 * p]), __uint_as_float(a[2 * p + 1])));
      a[2 * p] = __float_as_uint(z.x);
      a[2 * p + 1] = __float_as_uint(z.y);
    }
    tmem_st_x32(tbuf + col, a);
    if ((j + 1) % SPC == 0) publish_chunk(chunk_bar0 + 8 * (j / SPC));
    if (j + 1 < SUBS) {
      tmem_wait_ld_bind_x32(b);
#pragma unroll
      for (int i = 0; i < 32; ++i) a[i] = b[i];
    }
  }
}

// fp32 output job (TF32 chain): NCOL accumulator columns -> the fp32 staging
// tile (32-column chunks, 128-byte rows, 128B swizzle: the TMA-store layout).
template <int NCOL>
__device__ __forceinline__ void out_job_f32(uint32_t tbuf, uint32_t tile_base, uint32_t row, int col0) {
  constexpr int CH = NCOL < 32 ? NCOL : 32;
  static_assert(NCOL % CH == 0 && (CH == 16 || CH == 32), "unsupported width");
#pragma unroll
  for (int c = 0; c < NCOL; c += CH) {
    uint32_t r[CH];
    if constexpr (CH == 32) tmem_ld_wait_x32(tbuf + col0 + c, r);
    else tmem_ld_wait_x16(tbuf + col0 + c, r);
#pragma unroll
    for (int u = 0; u < CH / 4; ++u) {
      const int cc = col0 + c + 4 * u;
      st_shared_v4(tile_base + (cc / 32) * (kTileM * 128) + swz_off<128>(row, (cc % 32) / 4), r[4 * u],
                   r[4 * u + 1], r[4 * u + 2], r[4 * u + 3]);
    }
  }
}

template <class ChainT, int EPW, int MODE, bool SAVE, bool TF32 = false>
__global__ void __launch_bounds__(StreamCfg<ChainT, EPW, TF32>::THREADS, 1)
    mlp_stream_kernel(const __grid_constant__ StreamMaps<ChainT::L> maps, int num_tiles) {
  using Cfg = StreamCfg<ChainT, EPW, TF32>;
  static_assert(!TF32 || (MODE == kStreamFwd && !SAVE), "the tf32 chain is the inference forward");
  constexpr int L = Cfg::L;
  constexpr int NWBUF = Cfg::NWBUF;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t sbase = (raw + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (sbase - raw);

  const uint32_t s_w = sbase + Cfg::OFF_W;
  const uint32_t s_x = sbase + Cfg::OFF_X;
  const uint32_t s_o = sbase + Cfg::OFF_O;
  const uint32_t s_bar = sbase + Cfg::OFF_BAR;
  const uint32_t bar_x_full = s_bar;
  const uint32_t bar_x_empty = s_bar + 8;
  auto bar_w_full = [&](int b) { return s_bar + 16u + 8u * b; };
  auto bar_w_empty = [&](int b) { return s_bar + 16u + 8u * (NWBUF + b); };
  // one accumulator-full barrier per TMEM buffer (job g -> buffer g & 1,
  // parity (g >> 1) & 1; see mlp_fwd_kernel for why not one per kernel)
  auto bar_acc_full = [&](int b) { return s_bar + 16u + 8u * (2 * NWBUF + b); };
  const uint32_t bar_out_ready = s_bar + 16u + 8u * (2 * NWBUF + 2);
  const uint32_t bar_store_free = bar_out_ready + 8u;
  auto bar_chunk = [&](int c) { return bar_store_free + 8u + 8u * c; };
  const uint32_t bar_mma_done = bar_chunk(Cfg::MAXCH);
  const uint32_t s_tmem_slot = sbase + Cfg::OFF_MISC;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(gbase + Cfg::OFF_MISC + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    mbar_init(bar_x_full, 1);
    mbar_init(bar_x_empty, 1);
    for (int b = 0; b < NWBUF; ++b) {
      mbar_init(bar_w_full(b), 1);
      mbar_init(bar_w_empty(b), 1);
    }
    mbar_init(bar_acc_full(0), 1);
    mbar_init(bar_acc_full(1), 1);
    mbar_init(bar_out_ready, EPW);
    mbar_init(bar_store_free, 1);
    for (int c = 0; c < Cfg::MAXCH; ++c) mbar_init(bar_chunk(c), EPW);
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

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      tma_prefetch_desc(&maps.in);
      tma_prefetch_desc(&maps.out);
      bool ok = true;
      int n = 0;       // weight chunks issued (ring position)
      int xs = 0;      // input tiles issued
      for (int i = 0; ok; ++i) {
        const int t = static_cast<int>(blockIdx.x) + i * G;
        if (t >= num_tiles) break;
        if (!mbar_wait(bar_x_empty, (i & 1) ^ 1, abort_flag, kDevTimeoutEmpty)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(bar_x_full, kTileM * Cfg::D0 * Cfg::ES);
#pragma unroll
        for (int c = 0; c < Cfg::D0 / Cfg::CB; ++c)
          tma_load_2d(s_x + c * kTileM * 128, &maps.in, bar_x_full, c * Cfg::CB, t * kTileM);
        ++xs;
        if constexpr (MODE == kStreamDgrad) {
          // the epilogue reads the saved activations with plain loads: bring
          // this tile's (first tile) and the next tile's rows into L2 early,
          // as evict_last so they stay until read (W256 backward 1,466 ->
          // 1,439 us at 1M rows, A/B on one box)
          for (int tt = (i == 0 ? t : t + G); tt <= t + G && tt < num_tiles; tt += G) {
            const int rows = maps.M - tt * kTileM < kTileM ? maps.M - tt * kTileM : kTileM;
#pragma unroll 1
            for (int s = 0; s + 1 < L; ++s)
              prefetch_l2_bulk_hint(static_cast<const uint8_t*>(maps.hact[s]) +
                                        static_cast<size_t>(tt) * kTileM * maps.hact_cols[s] * 2,
                                    static_cast<uint32_t>(rows) * maps.hact_cols[s] * 2, l2_policy_evict_last());
          }
        }
        static_for<0, L>([&](auto sc) {
          constexpr int s = decltype(sc)::value;
          constexpr int K = ChainT::template D<s>();
          constexpr int N = ChainT::template D<s + 1>();
          for (int kc = 0; ok && kc < K / kStreamK; ++kc) {
            const int slot = n % NWBUF;
            if (!mbar_wait(bar_w_empty(slot), ((n / NWBUF) & 1) ^ 1, abort_flag, kDevTimeoutEmpty)) {
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(bar_w_full(slot), kStreamK * N * Cfg::ES);
            const uint32_t dst = s_w + slot * Cfg::WCH_BYTES;
            if constexpr (MODE == kStreamFwd) {
              // W_s rows [64kc, 64kc+64), all N columns: N/CB boxes {CB, 64}
#pragma unroll
              for (int c = 0; c < N / Cfg::CB; ++c)
                tma_load_2d(dst + c * kStreamK * 128, &maps.w[s], bar_w_full(slot), c * Cfg::CB, kc * kStreamK);
            } else {
              // W_l^T chunk: columns [64kc, 64kc+64) of W_l, all N = d_l rows
              tma_load_2d(dst, &maps.w[s], bar_w_full(slot), kc * kStreamK, 0);
            }
            ++n;
          }
        });
      }
      // Drain: never leave the CTA with a TMA load still writing shared memory.
      volatile int no_abort = 0;
      if (xs > 0) mbar_wait(bar_x_full, (xs - 1) & 1, &no_abort, kDevTimeoutFull);
      for (int b = 0; b < NWBUF; ++b) {
        const int uses = n > b ? (n - b + NWBUF - 1) / NWBUF : 0;
        if (uses > 0) mbar_wait(bar_w_full(b), (uses - 1) & 1, &no_abort, kDevTimeoutFull);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    const bool issuer = (lane == 0);
    bool ok = true;
    int n = 0;
    for (int i = 0; ok; ++i) {
      if (static_cast<int>(blockIdx.x) + i * G >= num_tiles) break;
      static_for<0, L>([&](auto sc) {
        constexpr int s = decltype(sc)::value;
        constexpr int K = ChainT::template D<s>();
        constexpr int N = ChainT::template D<s + 1>();
        constexpr uint32_t idesc = TF32 ? make_idesc_tf32(kTileM, N, 0, 1)
                                        : make_idesc_f16(kTileM, N, 0, MODE == kStreamFwd ? 1 : 0);
        if (!ok) return;
        const int g = i * L + s;
        const uint32_t d_tmem = tmem_base + (g & 1) * Cfg::SLOT_COLS;
        const uint32_t a_tmem = tmem_base + ((g & 1) ^ 1) * Cfg::SLOT_COLS;
        const uint32_t par = (i * (L - 1) + s - 1) & 1;
        if constexpr (s == 0) {
          ok = __all_sync(0xffffffffu, mbar_wait(bar_x_full, i & 1, abort_flag, kDevTimeoutMma));
          if (!ok) return;
        }
        int next_ch = 0;
        for (int kc = 0; kc < K / kStreamK; ++kc) {
          if constexpr (s > 0) {
            // every chunk of the previous stage's result this weight chunk reads
            const int need = (kc * kStreamK + kStreamK - 1) / Cfg::CH_COLS;
            for (; ok && next_ch <= need; ++next_ch)
              ok = __all_sync(0xffffffffu, mbar_wait(bar_chunk(next_ch), par, abort_flag, kDevTimeoutMma));
            if (!ok) break;
          }
          const int slot = n % NWBUF;
          ok = __all_sync(0xffffffffu,
                          mbar_wait(bar_w_full(slot), (n / NWBUF) & 1, abort_flag, kDevTimeoutMma));
          if (!ok) break;
          tc_fence_after();
          if (issuer) {
            const uint32_t wb = s_w + slot * Cfg::WCH_BYTES;
#pragma unroll
            for (int kk = 0; kk < kStreamK / Cfg::KSTEP; ++kk) {
              const int k = kc * (kStreamK / Cfg::KSTEP) + kk;
              const uint32_t accum = (kc > 0 || kk > 0) ? 1u : 0u;
              if constexpr (TF32) {
                // W chunks in the 32-byte-atom swizzle (the one MN-major
                // tf32 layout); a K-step is 8 rows of 128 bytes
                const uint64_t bdesc = mnmajor_tf32_base_desc<kStreamK>(wb) + ((kk * Cfg::KSTEP * 128) >> 4);
                if constexpr (s == 0)
                  umma_tf32(d_tmem,
                            kmajor_base_desc<2 * Cfg::D0>(s_x) + (kmajor_koff<kTileM, 2 * Cfg::D0>(k) >> 4),
                            bdesc, idesc, accum);
                else
                  umma_tf32_ts(d_tmem, a_tmem + Cfg::KSTEP * k, bdesc, idesc, accum);
              } else {
                uint64_t bdesc;
                if constexpr (MODE == kStreamFwd)
                  bdesc = mnmajor_base_desc<kStreamK, N>(wb) + (mnmajor_koff<N>(kk) >> 4);
                else
                  bdesc = kmajor_base_desc<kStreamK>(wb) + ((kk * 32) >> 4);
                if constexpr (s == 0)
                  umma_f16(d_tmem, kmajor_base_desc<Cfg::D0>(s_x) + (kmajor_koff<kTileM, Cfg::D0>(k) >> 4),
                           bdesc, idesc, accum);
                else
                  umma_f16_ts(d_tmem, a_tmem + h_tmem_col(16 * k), bdesc, idesc, accum);
              }
            }
            umma_commit(bar_w_empty(slot));
          }
          __syncwarp();
          ++n;
        }
        if (!ok) return;
        if (issuer) {
          if constexpr (s == 0) umma_commit(bar_x_empty);
          umma_commit(bar_acc_full(g & 1));
        }
        __syncwarp();
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
    const int q = warp & 3;     // TMEM lane quarter this warp may access
    const int grp = e >> 2;     // column group
    const uint32_t row = q * 32 + lane;
    const uint32_t t_lane = tmem_base + (static_cast<uint32_t>(q * 32) << 16);
    const bool leader = (e == 0 && lane == 0);
    constexpr int H = Cfg::H;
    constexpr int NG = Cfg::NG;
    constexpr int NCOL_O = Cfg::DL / NG;
    bool ok = true;
    for (int i = 0; ok; ++i) {
      const int t = static_cast<int>(blockIdx.x) + i * G;
      if (t >= num_tiles) break;
      const int grow = t * kTileM + static_cast<int>(row);
      const bool valid = grow < maps.M;
#pragma unroll 1
      for (int s = 0; s < L - 1; ++s) {
        const int g = i * L + s;
        uint4 hv[2][4];
        const uint8_t* hrow = nullptr;
        int hcols = H;
        if constexpr (MODE == kStreamDgrad) {
          hcols = maps.hact_cols[s];
          hrow = valid ? static_cast<const uint8_t*>(maps.hact[s]) + static_cast<size_t>(grow) * hcols * 2
                       : nullptr;
          dgrad_load_h<NG>(hv[0], hrow, grp, 0, hcols);
          if (H / (32 * NG) > 1) dgrad_load_h<NG>(hv[1], hrow, grp, 1, hcols);
        }
        ok = __all_sync(0xffffffffu,
                        mbar_wait(bar_acc_full(g & 1), (g >> 1) & 1, abort_flag, kDevTimeoutEpi));
        if (!ok) break;
        tc_fence_after();
        // the staging tile may still be the source of its previous TMA store:
        // the leader waits for it to be read, then frees it.  Uses: one per
        // tile (the output) or, when stage results are saved, one per stage.
        const int use = SAVE ? g : i;
        if ((SAVE || s == 0) && use > 0) {
          if (leader) {
            bulk_wait_group_read<0>();
            mbar_arrive(bar_store_free);
          }
          __syncwarp();
          ok = __all_sync(0xffffffffu,
                          mbar_wait(bar_store_free, (use - 1) & 1, abort_flag, kDevTimeoutEpi));
          if (!ok) break;
        }
        const uint32_t t_buf = t_lane + (g & 1) * Cfg::SLOT_COLS;
        if constexpr (TF32)
          hidden_job_f32<H, NG, Cfg::SPC>(t_buf, grp, bar_chunk(0));
        else if constexpr (MODE == kStreamFwd)
          hidden_job<H, NG, Cfg::SPC, SAVE ? 2 : 0>(t_buf, grp, bar_chunk(0), nullptr, s_o, row);
        else
          dgrad_job<H, NG, Cfg::SPC, SAVE>(t_buf, grp, bar_chunk(0), hv, hrow, hcols, s_o, row);
        if constexpr (SAVE) {
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) mbar_arrive(bar_out_ready);
          if (leader) {
            ok = mbar_wait(bar_out_ready, use & 1, abort_flag, kDevTimeoutEpi);
            if (ok) {
#pragma unroll
              for (int c = 0; c < H / 64; ++c)
                if (c * 64 < maps.save_cols[s]) tma_store_2d(&maps.save[s], s_o + c * kTileM * 128, c * 64, t * kTileM);
              bulk_commit_group();
            }
          }
          ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
          if (!ok) break;
        }
      }
      if (!ok) break;
      {
        // last stage: fp16 result staged in shared memory, written by TMA
        const int g = i * L + L - 1;
        ok = __all_sync(0xffffffffu,
                        mbar_wait(bar_acc_full(g & 1), (g >> 1) & 1, abort_flag, kDevTimeoutEpi));
        if (!ok) break;
        tc_fence_after();
        const int use = SAVE ? g : i;
        if constexpr (SAVE) {  // the tile held the last saved stage: wait for its store's read
          if (leader) {
            bulk_wait_group_read<0>();
            mbar_arrive(bar_store_free);
          }
          __syncwarp();
          ok = __all_sync(0xffffffffu,
                          mbar_wait(bar_store_free, (use - 1) & 1, abort_flag, kDevTimeoutEpi));
          if (!ok) break;
        }
        const uint32_t t_buf = t_lane + (g & 1) * Cfg::SLOT_COLS;
        if constexpr (TF32)
          out_job_f32<NCOL_O>(t_buf, s_o, row, grp * NCOL_O);
        else
          out_job<Cfg::DL, NCOL_O>(t_buf, s_o, row, grp * NCOL_O);
        fence_proxy_async_smem();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar_out_ready);
        if (leader) ok = mbar_wait(bar_out_ready, use & 1, abort_flag, kDevTimeoutEpi);
        ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
        if (leader && ok) {
#pragma unroll
          for (int c = 0; c < Cfg::DL / Cfg::CB; ++c)
            if (c * Cfg::CB < maps.out_cols)
              tma_store_2d(&maps.out, s_o + c * kTileM * 128, c * Cfg::CB, t * kTileM);
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
