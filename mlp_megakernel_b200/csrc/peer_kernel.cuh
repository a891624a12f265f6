// Cross-GPU sum of the fp32 weight gradients over NVLink peer memory, for
// data-parallel training on the GPUs of one node (the all_reduce(SUM) of the
// reference's DP recipe, done without NCCL).
//
// Every rank owns one exported ("peer") buffer of
//   [slot 0: n floats][slot 1: n floats][ready[8]][done[8]][count] (uint32 words)
// opened by every other rank through CUDA IPC.  In step `epoch` (1, 2, ...):
//   1. the backward's reduction writes this rank's dW into its own slot
//      (epoch & 1);
//   2. mlp_peer_allreduce_kernel: thread 0 of CTA 0 stores `epoch` into
//      ready[rank] of every rank's buffer (release, system scope); every CTA
//      waits until its own buffer's ready[q] >= epoch for all q (acquire,
//      bounded), then its threads sum slot (epoch & 1) of ranks 0 .. W-1 in
//      rank order and write the result.  Every rank adds the same values in
//      the same order, so the sum is bitwise identical on all ranks (NCCL's
//      ring / tree orders do not promise that).
//   3. completion: every CTA counts itself done in `count`; CTA 0 then stores
//      `epoch` into done[rank] of every rank's buffer and waits for its own
//      done[q] >= epoch.  So when the kernel returns on any rank, no rank reads
//      or writes that rank's buffer again in this step: a rank may free its
//      buffer or exit right after its last step.
// Slots alternate by epoch parity: a rank can write its slot for epoch e only
// after its step e-1 returned, i.e. after every rank finished reading epoch
// e-1 -- and, one step earlier, epoch e-2 (the same slot).
//
// Plain peer loads and stores only (no multicast objects, no TMA).  Every wait
// is bounded: on expiry the kernel records kDevTimeoutFlag in the device
// status word and returns (without writing the result if the data never
// became ready).
#pragma once
#include "ptx.cuh"

namespace mlpk {

constexpr int kPeerMaxRanks = 8;

struct PeerPtrs {
  float* buf[kPeerMaxRanks];  // every rank's peer buffer (this rank's own included)
};

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Bounded wait until every word flags[0 .. world-1] >= epoch.
__device__ __forceinline__ bool peer_wait_all(const uint32_t* flags, int world, uint32_t epoch) {
  const uint64_t t0 = globaltimer_ns();
  for (int q = 0; q < world; ++q) {
    while (static_cast<int32_t>(ld_acquire_sys(flags + q) - epoch) < 0) {
      if (globaltimer_ns() - t0 > MLPK_WAIT_TIMEOUT_NS) {
        atomicOr(&g_device_status, kDevTimeoutFlag);
        return false;
      }
    }
  }
  return true;
}

__global__ void __launch_bounds__(256)
    mlp_peer_allreduce_kernel(PeerPtrs peers, int world, int rank, int n, uint32_t epoch,
                              float* __restrict__ out) {
  const size_t slot_off = static_cast<size_t>(epoch & 1u) * n;
  auto words = [&](int q) { return reinterpret_cast<uint32_t*>(peers.buf[q] + 2 * static_cast<size_t>(n)); };
  uint32_t* const ready = words(rank);                  // ready[kPeerMaxRanks]
  uint32_t* const done = ready + kPeerMaxRanks;         // done[kPeerMaxRanks]
  uint32_t* const count = ready + 2 * kPeerMaxRanks;    // CTAs finished, all steps
  __shared__ int s_ok;
  if (threadIdx.x == 0) {
    if (blockIdx.x == 0) {
      // this rank's slot was completed by the previous kernel on this stream
      asm volatile("fence.acq_rel.sys;" ::: "memory");
      for (int q = 0; q < world; ++q) st_release_sys(words(q) + rank, epoch);
    }
    s_ok = peer_wait_all(ready, world, epoch) ? 1 : 0;
  }
  __syncthreads();
  if (s_ok) {
    // n is a multiple of 4 (checked by the host); grid-stride over float4s
    // (the host keeps the grid at most one CTA per SM: every CTA is resident)
    for (int i4 = blockIdx.x * blockDim.x + threadIdx.x; 4 * i4 < n; i4 += gridDim.x * blockDim.x) {
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int q = 0; q < world; ++q) {  // fixed rank order: identical sums on every rank
        const float4 v = __ldcv(reinterpret_cast<const float4*>(peers.buf[q] + slot_off) + i4);
        acc.x += v.x;
        acc.y += v.y;
        acc.z += v.z;
        acc.w += v.w;
      }
      reinterpret_cast<float4*>(out)[i4] = acc;
    }
  }
  __syncthreads();  // this CTA's peer reads are complete
  if (threadIdx.x == 0) {
    __threadfence();
    atomicAdd(count, 1u);
    if (blockIdx.x == 0 && s_ok) {
      // every CTA of this kernel (count is cumulative over steps) ...
      const uint32_t target = epoch * gridDim.x;
      const uint64_t t0 = globaltimer_ns();
      bool ok = true;
      while (static_cast<int32_t>(ld_acquire_sys(count) - target) < 0) {
        if (globaltimer_ns() - t0 > MLPK_WAIT_TIMEOUT_NS) {
          atomicOr(&g_device_status, kDevTimeoutFlag);
          ok = false;
          break;
        }
      }
      // ... then every rank is done with the others' buffers for this step
      if (ok) {
        asm volatile("fence.acq_rel.sys;" ::: "memory");
        for (int q = 0; q < world; ++q) st_release_sys(words(q) + kPeerMaxRanks + rank, epoch);
        peer_wait_all(done, world, epoch);
      }
    }
  }
}

}  // namespace mlpk
