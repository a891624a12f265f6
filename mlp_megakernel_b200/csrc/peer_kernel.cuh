// Cross-GPU sum of the fp32 weight gradients over NVLink peer memory, for
// data-parallel training on the GPUs of one node (the all_reduce(SUM) of the
// reference's DP recipe, done without NCCL).
//
// Every rank owns one exported ("peer") buffer of
//   [slot: n floats][ready[8]][done[8]][count][epoch] (uint32 words)
// opened by every other rank through CUDA IPC.  In each step:
//   1. the backward's reduction writes this rank's dW into its slot;
//   2. mlp_peer_allreduce_kernel: every CTA reads the step number
//      e = epoch + 1 from its own buffer; thread 0 of CTA 0 stores e into
//      ready[rank] of every rank's buffer (release, system scope); every CTA
//      waits until its own ready[q] >= e for all q (acquire, bounded), then its
//      threads sum the slots of ranks 0 .. W-1 in rank order and write the
//      result.  Every rank adds the same values in the same order, so the sum
//      is bitwise identical on all ranks (NCCL's ring / tree orders do not
//      promise that);
//   3. completion: every CTA counts itself done in `count`; CTA 0 then stores
//      e into done[rank] of every rank's buffer, waits for its own done[q] >= e
//      and finally sets epoch = e.  So when the kernel returns on a rank, every
//      rank has finished reading that rank's slot (it may be rewritten by the
//      next backward, freed, or the process may exit) and no rank will write
//      into that rank's buffer again in this step.
// The step number lives in device memory, so the kernel can be replayed from
// a CUDA graph.  Plain peer loads and stores only (no multicast objects, no
// TMA).  Every wait is bounded: on expiry the kernel records kDevTimeoutFlag in
// the device status word and returns (without the result if the data never
// became ready).
#pragma once
#include "ptx.cuh"

namespace mlpk {

constexpr int kPeerMaxRanks = 8;

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

// Bounded wait until every word flags[0 .. world-1] >= epoch (acquire).
__device__ __forceinline__ bool peer_wait_all(const uint32_t* flags, int world, uint32_t epoch) {
  const uint64_t t0 = globaltimer_ns();
  for (int q = 0; q < world; ++q) {
    while (static_cast<int32_t>(ld_relaxed_sys(flags + q) - epoch) < 0) {
      if (globaltimer_ns() - t0 > MLPK_WAIT_TIMEOUT_NS) {
        atomicOr(&g_device_status, kDevTimeoutFlag);
        return false;
      }
    }
  }
  fence_sys();
  return true;
}

// Release: everything this thread (and, after a CTA barrier, its CTA) wrote
// or read before is ordered before the flag stores.
__device__ __forceinline__ void peer_signal_all(const PeerPtrs& peers, int world, int n, int word,
                                                uint32_t epoch) {
  fence_sys();
  for (int q = 0; q < world; ++q)
    st_relaxed_sys(reinterpret_cast<uint32_t*>(peers.buf[q] + static_cast<size_t>(n)) + word, epoch);
}

__global__ void __launch_bounds__(256)
    mlp_peer_allreduce_kernel(PeerPtrs peers, int world, int rank, int n, float* __restrict__ out) {
  pdl_enter();
  auto words = [&](int q) { return reinterpret_cast<uint32_t*>(peers.buf[q] + static_cast<size_t>(n)); };
  uint32_t* const ready = words(rank);                  // ready[kPeerMaxRanks]
  uint32_t* const done = ready + kPeerMaxRanks;         // done[kPeerMaxRanks]
  uint32_t* const count = ready + 2 * kPeerMaxRanks;    // CTAs finished, all steps
  uint32_t* const epoch_word = count + 1;               // steps completed
  __shared__ int s_ok;
  __shared__ uint32_t s_epoch;
  if (threadIdx.x == 0) {
    // epoch only changes at the very end of CTA 0, after every CTA counted itself
    const uint32_t e = *reinterpret_cast<volatile uint32_t*>(epoch_word) + 1u;
    s_epoch = e;
    // this rank's slot was completed by the previous kernel on this stream
    if (blockIdx.x == 0) peer_signal_all(peers, world, n, rank, e);
    s_ok = peer_wait_all(ready, world, e) ? 1 : 0;
  }
  __syncthreads();
  const uint32_t e = s_epoch;
  if (s_ok) {
    // n is a multiple of 4 (checked by the host); grid-stride over float4s
    // (the host keeps the grid at most one CTA per SM: every CTA is resident)
    for (int i4 = blockIdx.x * blockDim.x + threadIdx.x; 4 * i4 < n; i4 += gridDim.x * blockDim.x) {
      // all ranks' loads in flight at once (one NVLink round trip), then the
      // adds in fixed rank order: identical sums on every rank
      float4 v[kPeerMaxRanks];
#pragma unroll
      for (int q = 0; q < kPeerMaxRanks; ++q)
        if (q < world) v[q] = __ldcv(reinterpret_cast<const float4*>(peers.buf[q]) + i4);
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
  __syncthreads();  // this CTA's peer reads are complete
  if (threadIdx.x == 0) {
    __threadfence();
    atomicAdd(count, 1u);
    if (blockIdx.x == 0) {
      // every CTA of this kernel (count is cumulative over steps) ...
      const uint32_t target = e * gridDim.x;
      const uint64_t t0 = globaltimer_ns();
      bool ok = s_ok != 0;
      while (ok && static_cast<int32_t>(ld_relaxed_sys(count) - target) < 0) {
        if (globaltimer_ns() - t0 > MLPK_WAIT_TIMEOUT_NS) {
          atomicOr(&g_device_status, kDevTimeoutFlag);
          ok = false;
        }
      }
      // ... then every rank is done with the others' buffers for this step
      if (ok) {
        peer_signal_all(peers, world, n, kPeerMaxRanks + rank, e);
        peer_wait_all(done, world, e);
      }
      *reinterpret_cast<volatile uint32_t*>(epoch_word) = e;
    }
  }
}

}  // namespace mlpk
