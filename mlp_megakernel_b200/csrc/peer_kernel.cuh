// Cross-GPU sum of the fp32 weight gradients over NVLink peer memory, for
// data-parallel training on the GPUs of one node (the all_reduce(SUM) of the
// reference's DP recipe, done without NCCL).
//
// Every rank owns one exported ("peer") buffer of
//   [in: n floats][slot 0: n floats][slot 1: n floats]
//   [ready[kPeerMaxRanks][kPeerMaxCtas]][epoch[kPeerMaxCtas]] (uint32 words)
// opened by every other rank through CUDA IPC.  Step e of CTA c (every call
// launches the same grid; CTA c owns the same float4s every time):
//   1. the backward's reduction has written this rank's dW into `in`;
//   2. CTA c copies its float4s of `in` into slot e % 2, then stores e into
//      ready[rank][c] of every rank's buffer (release, system scope), waits
//      until its own ready[q][c] >= e for every rank q (acquire, bounded),
//      and sums slot e % 2 of ranks 0 .. W-1 in rank order over its float4s.
//      Every rank adds the same values in the same order, so the sum is
//      bitwise identical on all ranks (NCCL's ring / tree orders do not
//      promise that);
//   3. CTA c records e in its epoch word (read by CTA c of the next call).
// Why two slots and no closing barrier: rank r rewrites slot e % 2 in step
// e + 2, after its CTA c passed the ready wait of step e + 1; rank q signals
// that step only from its next kernel, i.e. after it finished reading rank
// r's slot e % 2 in step e.  So one flag hand-off per step suffices (the
// first version closed every step with a second, "done" hand-off and a count
// of finished CTAs).  `in` is never read by the other ranks: the next
// backward may rewrite it as soon as this kernel returns.  The other ranks
// may still be reading this rank's slots then, so a buffer is freed only
// after every rank synchronized its device and met a host barrier.
// The step number lives in device memory, so the kernel can be replayed from
// a CUDA graph.  Plain peer loads and stores only (no multicast objects, no
// TMA).  Every wait is bounded: on expiry the kernel records kDevTimeoutFlag in
// the device status word and returns (without the result if the data never
// became ready).
#pragma once
#include "ptx.cuh"

namespace mlpk {

constexpr int kPeerMaxRanks = 8;
constexpr int kPeerMaxCtas = 256;  // CTAs of one call (the host caps the grid)
// 32-bit words after the three float regions
constexpr int kPeerFlagWords = kPeerMaxRanks * kPeerMaxCtas + kPeerMaxCtas;

struct PeerPtrs {
  float* buf[kPeerMaxRanks];  // every rank's peer buffer (this rank's own included)
};

// A release of several flags is ONE system-scope fence followed by relaxed
// stores (a st.release per flag would fence each time: measured ~1.8 us per
// remote flag); an acquire of several flags is relaxed polls followed by one
// fence.
__device__ __forceinline__ void fence_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }
__device__ __forceinline__ void st_relaxed_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_relaxed_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.relaxed.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Bounded wait until every word flags[q * stride], q < world, is >= epoch
// (acquire).
__device__ __forceinline__ bool peer_wait_all(const uint32_t* flags, int stride, int world, uint32_t epoch) {
  const uint64_t t0 = globaltimer_ns();
  for (int q = 0; q < world; ++q) {
    while (static_cast<int32_t>(ld_relaxed_sys(flags + static_cast<size_t>(q) * stride) - epoch) < 0) {
      if (globaltimer_ns() - t0 > MLPK_WAIT_TIMEOUT_NS) {
        atomicOr(&g_device_status, kDevTimeoutFlag);
        return false;
      }
    }
  }
  fence_sys();
  return true;
}

__global__ void __launch_bounds__(256)
    mlp_peer_allreduce_kernel(PeerPtrs peers, int world, int rank, int n, float* __restrict__ out) {
  pdl_enter();
  const int c = blockIdx.x;
  auto flags = [&](int q) { return reinterpret_cast<uint32_t*>(peers.buf[q] + 3 * static_cast<size_t>(n)); };
  uint32_t* const epoch_word = flags(rank) + kPeerMaxRanks * kPeerMaxCtas + c;
  __shared__ int s_ok;
  __shared__ uint32_t s_epoch;
  if (threadIdx.x == 0) s_epoch = *reinterpret_cast<volatile uint32_t*>(epoch_word) + 1u;
  __syncthreads();
  const uint32_t e = s_epoch;
  const size_t slot = static_cast<size_t>(n) * (1 + (e & 1u));
  // n is a multiple of 4 (checked by the host); CTA c's float4s: a grid stride
  const int i0 = c * blockDim.x + threadIdx.x, stride = gridDim.x * blockDim.x;
  {
    const float4* in = reinterpret_cast<const float4*>(peers.buf[rank]);
    float4* mine = reinterpret_cast<float4*>(peers.buf[rank] + slot);
    for (int i4 = i0; 4 * i4 < n; i4 += stride) mine[i4] = in[i4];
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    // release this CTA's copy (the CTA barrier above orders every thread's
    // stores before this fence), then acquire every rank's
    fence_sys();
    for (int q = 0; q < world; ++q) st_relaxed_sys(flags(q) + rank * kPeerMaxCtas + c, e);
    s_ok = peer_wait_all(flags(rank) + c, kPeerMaxCtas, world, e) ? 1 : 0;
  }
  __syncthreads();
  if (s_ok) {
    for (int i4 = i0; 4 * i4 < n; i4 += stride) {
      // all ranks' loads in flight at once (one NVLink round trip), then the
      // adds in fixed rank order: identical sums on every rank
      float4 v[kPeerMaxRanks];
#pragma unroll
      for (int q = 0; q < kPeerMaxRanks; ++q)
        if (q < world) v[q] = __ldcv(reinterpret_cast<const float4*>(peers.buf[q] + slot) + i4);
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int q = 0; q < kPeerMaxRanks; ++q) {
        if (q < world) {
          acc.x += v[q].x;
          acc.y += v[q].y;
          acc.z += v[q].z;
          acc.w += v[q].w;
        }
      }
      reinterpret_cast<float4*>(out)[i4] = acc;
    }
  }
  // the step is done for this CTA index (also after a timeout, so that the
  // step numbers of later calls stay in line with the other ranks')
  if (threadIdx.x == 0) *reinterpret_cast<volatile uint32_t*>(epoch_word) = e;
}

}  // namespace mlpk
