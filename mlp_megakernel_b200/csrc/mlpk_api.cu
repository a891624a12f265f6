// C-ABI entry points of libmlpk (declared in include/mlpk.h).
//
// Host responsibilities: validate shapes and pointers, encode the TMA tensor
// maps (driver entry point fetched through the runtime, so the library does
// not link libcuda), size the persistent grid from the SM count, and launch on
// the caller's stream.  Nothing here allocates device memory or synchronises.
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <cstdint>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <set>
#include <utility>

#include "../../include/mlpk.h"
#include "bwd_kernel.cuh"
#include "cast_kernel.cuh"
#include "stream_kernel.cuh"
#include "peer_kernel.cuh"
#include "wgrad_kernel.cuh"
#include "wn_kernel.cuh"

namespace {

using mlpk::FwdCfg;
using mlpk::FwdMaps;
using mlpk::Net;

// ------------------------------------------------------------------ device
constexpr int kMaxDevices = 64;
struct DevInfo {
  int sm_count = 0;
  int major = 0;
  int minor = 0;
  bool valid = false;
};
DevInfo g_dev[kMaxDevices];
std::mutex g_dev_mu;

// The CUDA failure behind this thread's most recent MLPK_ERR_CUDA (reported by
// mlpk_last_cuda_error).
thread_local char t_last_cuda_error[160] = "no error";

int cuda_status(cudaError_t e) {
  if (e == cudaSuccess) return MLPK_OK;
  std::snprintf(t_last_cuda_error, sizeof(t_last_cuda_error), "%s: %s", cudaGetErrorName(e),
                cudaGetErrorString(e));
  return MLPK_ERR_CUDA;
}

int driver_status(const char* what, int result) {
  if (result == 0) return MLPK_OK;
  std::snprintf(t_last_cuda_error, sizeof(t_last_cuda_error), "%s returned CUresult %d", what, result);
  return MLPK_ERR_CUDA;
}

// Launch through cudaLaunchKernelEx so that the status returned is that of
// THIS launch, not an error left earlier on the calling thread.  With `early`
// the kernel is launched with programmatic stream serialization: it may start
// while the kernel before it on the stream is still running (every kernel of
// the library calls pdl_enter() before touching global memory, ptx.cuh), so
// its setup overlaps that kernel's tail.  The inference forward launches this
// way (back-to-back small calls: 6.0 -> 5.2 us per call at 64 rows); the
// training kernels do not (the config-3 step measured 40.8 us at 16,384 rows
// without it, 42.4 with it).
template <typename... KArgs, typename... Args>
int launch_kernel_cfg(bool early, void (*kern)(KArgs...), dim3 grid, unsigned block, size_t smem,
                      cudaStream_t st, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(block, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = early ? 1 : 0;
  return cuda_status(cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...));
}
template <typename... KArgs, typename... Args>
int launch_kernel(void (*kern)(KArgs...), dim3 grid, unsigned block, size_t smem, cudaStream_t st,
                  Args&&... args) {
  return launch_kernel_cfg(false, kern, grid, block, smem, st, std::forward<Args>(args)...);
}
template <typename... KArgs, typename... Args>
int launch_kernel_early(void (*kern)(KArgs...), dim3 grid, unsigned block, size_t smem, cudaStream_t st,
                        Args&&... args) {
  return launch_kernel_cfg(true, kern, grid, block, smem, st, std::forward<Args>(args)...);
}

int current_device_info(DevInfo* out, int* dev_out) {
  int dev = 0;
  int rc = cuda_status(cudaGetDevice(&dev));
  if (rc != MLPK_OK) return rc;
  if (dev < 0 || dev >= kMaxDevices) return MLPK_ERR_DEVICE;
  // The tensor maps are encoded through the driver API, which needs the
  // device's context current on THIS thread.  A thread that has only asked the
  // runtime for its device (torch's autograd worker, for one) may have none
  // bound yet; cudaSetDevice binds the primary context.
  thread_local int t_bound_dev = -1;
  if (t_bound_dev != dev) {
    if ((rc = cuda_status(cudaSetDevice(dev))) != MLPK_OK) return rc;
    t_bound_dev = dev;
  }
  std::lock_guard<std::mutex> lk(g_dev_mu);
  DevInfo& d = g_dev[dev];
  if (!d.valid) {
    if ((rc = cuda_status(cudaDeviceGetAttribute(&d.sm_count, cudaDevAttrMultiProcessorCount, dev))) ||
        (rc = cuda_status(cudaDeviceGetAttribute(&d.major, cudaDevAttrComputeCapabilityMajor, dev))) ||
        (rc = cuda_status(cudaDeviceGetAttribute(&d.minor, cudaDevAttrComputeCapabilityMinor, dev))))
      return rc;
    d.valid = true;
  }
  *out = d;
  if (dev_out) *dev_out = dev;
  return d.major == 10 ? MLPK_OK : MLPK_ERR_ARCH;
}

// ------------------------------------------------------------------ TMA maps
using EncodeFn = PFN_cuTensorMapEncodeTiled_v12000;
EncodeFn get_encode() {
  static EncodeFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeFn>(p);
  });
  return fn;
}

// 2-D tensor [outer][inner] (inner contiguous) of fp16 (elem_bytes 2) or fp32
// (elem_bytes 4), box {box_inner, box_outer}, swizzle chosen from the box's
// row pitch (box_inner * elem_bytes); atom32: 128-byte rows swizzled in
// 32-byte granules (the MN-major tf32 operand layout, layout.cuh).
int make_map_2d(CUtensorMap* map, const void* ptr, uint64_t inner, uint64_t outer,
                uint32_t box_inner, uint32_t box_outer, uint32_t elem_bytes = 2, bool atom32 = false) {
  EncodeFn enc = get_encode();
  if (!enc) return driver_status("cudaGetDriverEntryPoint(cuTensorMapEncodeTiled)", -1);
  const uint32_t pitch = box_inner * elem_bytes;
  if (atom32 && pitch != 128) return MLPK_ERR_SHAPE;
  CUtensorMapSwizzle swz = atom32         ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B
                           : pitch == 128 ? CU_TENSOR_MAP_SWIZZLE_128B
                           : pitch == 64  ? CU_TENSOR_MAP_SWIZZLE_64B
                                          : CU_TENSOR_MAP_SWIZZLE_32B;
  cuuint64_t gdim[2] = {inner, outer};
  cuuint64_t gstride[1] = {inner * elem_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estride[2] = {1, 1};
  CUresult r = enc(map, elem_bytes == 4 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
                   const_cast<void*>(ptr), gdim, gstride, box, estride, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return driver_status("cuTensorMapEncodeTiled", static_cast<int>(r));
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Raise a kernel's dynamic shared-memory limit once per (kernel, device).
template <class Kern>
bool set_smem_once(Kern kern, int bytes, int dev) {
  static std::mutex mu;
  static std::set<std::pair<const void*, int>> done;
  std::lock_guard<std::mutex> lk(mu);
  const auto key = std::make_pair(reinterpret_cast<const void*>(kern), dev);
  if (done.count(key)) return true;
  if (cuda_status(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes)))
    return false;
  done.insert(key);
  return true;
}

// ------------------------------------------------------------------ descriptor cache
// Encoded tensor maps of recent calls, per host thread: a serving loop calls
// the forward again and again on the same buffers, and re-encoding every TMA
// descriptor would be most of the host work of a small call.  The key holds
// everything the maps encode (device, rows, every pointer, the caller's
// widths, the saved-activation precision); four entries, replaced round robin.
template <class Maps>
struct MapCache {
  static constexpr int kEntries = 4;
  static constexpr int kKey = 40;
  struct Entry {
    bool valid = false;
    uint64_t key[kKey];
    Maps maps;
  };
  Entry e[kEntries];
  int next = 0;
  const Maps* find(const uint64_t* key) const {
    for (const Entry& x : e)
      if (x.valid && std::memcmp(x.key, key, sizeof(x.key)) == 0) return &x.maps;
    return nullptr;
  }
  void insert(const uint64_t* key, const Maps& m) {
    Entry& x = e[next];
    next = (next + 1) % kEntries;
    std::memcpy(x.key, key, sizeof(x.key));
    x.maps = m;
    x.valid = true;
  }
};

// ------------------------------------------------------------------ forward
// Every launcher takes the caller's widths rd[0..L] (each at most the kernel
// network's width, a multiple of 8): tensor maps of the caller's tensors carry
// the caller's extents with the kernel network's boxes, so a smaller network
// is served by the larger kernel through TMA zero fill (rd equal to the kernel
// network's widths is the plain case).
template <class NetT, int NS, int EPW>
int launch_fwd(const int* rd, const void* x, const void* const* W, void* out, int64_t M,
               void* const* hsave, bool h32, cudaStream_t st) {
  using Cfg = FwdCfg<NetT, NS, EPW>;
  using Cfg32 = FwdCfg<NetT, NS, EPW, true>;
  constexpr int L = NetT::L;
  DevInfo di;
  int dev = 0;
  int rc = current_device_info(&di, &dev);
  if (rc != MLPK_OK) return rc;
  if (M == 0) return MLPK_OK;
  if (M > (int64_t(1) << 31) - 256) return MLPK_ERR_SHAPE;

  thread_local MapCache<FwdMaps<L>> cache;
  uint64_t key[MapCache<FwdMaps<L>>::kKey] = {};
  {
    int k = 0;
    key[k++] = static_cast<uint64_t>(dev);
    key[k++] = static_cast<uint64_t>(M);
    key[k++] = reinterpret_cast<uintptr_t>(x);
    key[k++] = reinterpret_cast<uintptr_t>(out);
    key[k++] = (hsave ? 1u : 0u) | (h32 ? 2u : 0u);
    for (int l = 0; l < L; ++l) key[k++] = reinterpret_cast<uintptr_t>(W[l]);
    for (int l = 0; hsave && l + 1 < L; ++l) key[k++] = reinterpret_cast<uintptr_t>(hsave[l]);
    for (int i = 0; i <= L; ++i) key[k++] = static_cast<uint64_t>(rd[i]);
  }
  const int num_tiles = static_cast<int>((M + mlpk::kTileM - 1) / mlpk::kTileM);
  const int grid = num_tiles < di.sm_count ? num_tiles : di.sm_count;
  FwdMaps<L> maps;
  if (const FwdMaps<L>* hit = cache.find(key)) {
    maps = *hit;
  } else {
    std::memset(&maps, 0, sizeof(maps));
    rc = make_map_2d(&maps.x, x, rd[0], M, mlpk::chunk_elems(Cfg::D0), mlpk::kTileM);
    if (rc) return rc;
    rc = make_map_2d(&maps.out, out, rd[L], M, mlpk::chunk_elems(Cfg::DL), mlpk::kTileM);
    if (rc) return rc;
    int wrc = MLPK_OK;
    mlpk::static_for<0, L>([&](auto lc) {
      constexpr int l = decltype(lc)::value;
      constexpr int K = NetT::template D<l>();
      constexpr int N = NetT::template D<l + 1>();
      if (wrc == MLPK_OK) wrc = make_map_2d(&maps.w[l], W[l], rd[l + 1], rd[l], mlpk::chunk_elems(N), K);
    });
    if (wrc) return wrc;
    maps.M = static_cast<int>(M);
    maps.out_cols = rd[L];
    for (int l = 0; l + 1 < L; ++l) maps.h_cols[l] = rd[l + 1];
    if (hsave) {
      for (int l = 0; l + 1 < L; ++l) {
        if (!hsave[l]) return MLPK_ERR_NULL;
        // fp32: every warp stores its 32 rows x 32 columns per piece
        rc = h32 ? make_map_2d(&maps.hsave[l], hsave[l], rd[l + 1], M, 32, 32, 4)
                 : make_map_2d(&maps.hsave[l], hsave[l], rd[l + 1], M, mlpk::chunk_elems(Cfg::H), mlpk::kTileM);
        if (rc) return rc;
      }
    }
    cache.insert(key, maps);
  }
  if (!hsave && num_tiles <= di.sm_count) {
    // Small batches (every CTA gets at most one row tile): the latency
    // configuration -- one tile in flight and up to four column groups of
    // epilogue warps, so each warp runs one 32-column stripe of a layer
    // instead of all of them (the tile's MMA -> softplus -> MMA chain is the
    // whole kernel time here, not the throughput of several tiles).
    constexpr int kLatEpw = 4 * (Cfg::H / 32 < 4 ? Cfg::H / 32 : 4);
    using CfgL = FwdCfg<NetT, 1, kLatEpw>;
    auto kern = mlpk::mlp_fwd_kernel<NetT, 1, kLatEpw, false>;
    if (!set_smem_once(kern, CfgL::SMEM_BYTES, dev)) return MLPK_ERR_CUDA;
    return launch_kernel_early(kern, grid, CfgL::THREADS, CfgL::SMEM_BYTES, st, maps, num_tiles);
  }
  if (hsave && h32) {
    auto kern = mlpk::mlp_fwd_kernel<NetT, NS, EPW, true, true>;
    if (!set_smem_once(kern, Cfg32::SMEM_BYTES, dev)) return MLPK_ERR_CUDA;
    return launch_kernel(kern, grid, Cfg32::THREADS, Cfg32::SMEM_BYTES, st, maps, num_tiles);
  }
  if (hsave) {
    auto kern = mlpk::mlp_fwd_kernel<NetT, NS, EPW, true>;
    if (!set_smem_once(kern, Cfg::SMEM_BYTES, dev)) return MLPK_ERR_CUDA;
    return launch_kernel(kern, grid, Cfg::THREADS, Cfg::SMEM_BYTES, st, maps, num_tiles);
  }
  auto kern = mlpk::mlp_fwd_kernel<NetT, NS, EPW, false>;
  if (!set_smem_once(kern, Cfg::SMEM_BYTES, dev)) return MLPK_ERR_CUDA;
  return launch_kernel_early(kern, grid, Cfg::THREADS, Cfg::SMEM_BYTES, st, maps, num_tiles);
}

// ------------------------------------------------------------------ backward
template <class NetT>
int64_t bwd_grid(int64_t M, int sm_count) {
  const int64_t tiles = (M + mlpk::kTileM - 1) / mlpk::kTileM;
  return tiles < sm_count ? tiles : sm_count;
}

template <class NetT>
size_t bwd_workspace(int64_t M, int sm_count) {  // the same for fp16 and fp32 saved activations
  return static_cast<size_t>(bwd_grid<NetT>(M, sm_count)) * mlpk::BwdCfg<NetT>::PARTIAL_FLOATS *
         sizeof(float);
}

// Output layout of the weight-gradient reduction for the caller's widths rd
// (identity when they are the kernel network's widths).
template <class NetT>
mlpk::DwLayout dw_layout(const int* rd) {
  constexpr int L = NetT::L;
  mlpk::DwLayout lay;
  std::memset(&lay, 0, sizeof(lay));
  bool same = true;
  for (int i = 0; i <= L; ++i) same = same && rd[i] == NetT::dim(i);
  if (same) return lay;
  lay.layers = L;
  long long ko = 0, ro = 0;
  for (int l = 0; l < L; ++l) {
    lay.koff[l] = ko;
    lay.kn[l] = NetT::dim(l + 1);
    lay.rk[l] = rd[l];
    lay.rn[l] = rd[l + 1];
    lay.roff[l] = ro;
    ko += static_cast<long long>(NetT::dim(l)) * NetT::dim(l + 1);
    ro += static_cast<long long>(rd[l]) * rd[l + 1];
  }
  lay.koff[L] = ko;
  return lay;
}

// Fixed-order sum of `groups` groups of nparts partials (nfloats each) into dw;
// 16-byte loads when the partial rows stay 16-byte aligned (bitwise the same
// sums either way).
inline int launch_reduce(const float* partials, int nparts, int nfloats, int groups, float* dw,
                         const mlpk::DwLayout& lay, cudaStream_t st) {
  const int threads = mlpk::kReduceElems * mlpk::kReduceSlices;
  if (nfloats % 4 == 0 && reinterpret_cast<uintptr_t>(partials) % 16 == 0) {
    const int per = mlpk::kReduceElems * 4;
    return launch_kernel(mlpk::mlp_reduce_kernel<4>, dim3((nfloats + per - 1) / per, groups, 1), threads, 0,
                         st, partials, nparts, nfloats, dw, lay);
  }
  return launch_kernel(mlpk::mlp_reduce_kernel<1>,
                       dim3((nfloats + mlpk::kReduceElems - 1) / mlpk::kReduceElems, groups, 1), threads, 0,
                       st, partials, nparts, nfloats, dw, lay);
}

template <class NetT>
int launch_bwd(const int* rd, const void* x, const void* const* W, const void* const* h, bool h32,
               const void* g, void* dx, float* ws, size_t ws_bytes, float* dw, int64_t M, cudaStream_t st) {
  using Cfg = mlpk::BwdCfg<NetT>;
  using Cfg32 = mlpk::BwdCfg<NetT, true>;
  constexpr int L = NetT::L;
  DevInfo di;
  int dev = 0;
  int rc = current_device_info(&di, &dev);
  if (rc != MLPK_OK) return rc;
  if (M > (int64_t(1) << 31) - 256) return MLPK_ERR_SHAPE;
  const int nfloats = Cfg::PARTIAL_FLOATS;
  const int grid = static_cast<int>(bwd_grid<NetT>(M, di.sm_count));
  if (grid > 0) {
    if (ws_bytes < bwd_workspace<NetT>(M, di.sm_count)) return MLPK_ERR_SHAPE;
    mlpk::BwdMaps<L> maps;
    std::memset(&maps, 0, sizeof(maps));
    if ((rc = make_map_2d(&maps.x, x, rd[0], M, mlpk::chunk_elems(Cfg::D0), mlpk::kTileM))) return rc;
    if ((rc = make_map_2d(&maps.g, g, rd[L], M, mlpk::chunk_elems(Cfg::DL), mlpk::kTileM))) return rc;
    if ((rc = make_map_2d(&maps.dx, dx, rd[0], M, mlpk::chunk_elems(Cfg::D0), mlpk::kTileM))) return rc;
    int wrc = MLPK_OK;
    mlpk::static_for<0, L>([&](auto lc) {
      constexpr int l = decltype(lc)::value;
      constexpr int K = NetT::template D<l>();
      constexpr int N = NetT::template D<l + 1>();
      if (wrc == MLPK_OK) wrc = make_map_2d(&maps.w[l], W[l], rd[l + 1], rd[l], mlpk::chunk_elems(N), K);
      if constexpr (l >= 1)
        if (wrc == MLPK_OK)  // fp32: 32-column chunks of the two halves
          wrc = h32 ? make_map_2d(&maps.h[l - 1], h[l - 1], rd[l], M, 32, mlpk::kTileM, 4)
                    : make_map_2d(&maps.h[l - 1], h[l - 1], rd[l], M, mlpk::chunk_elems(K), mlpk::kTileM);
    });
    if (wrc) return wrc;
    maps.partials = ws;
    maps.dx_cols = rd[0];
    const int num_tiles = static_cast<int>((M + mlpk::kTileM - 1) / mlpk::kTileM);
    if (h32) {
      auto kern = mlpk::mlp_bwd_kernel<NetT, true>;
      if (!set_smem_once(kern, Cfg32::SMEM_BYTES, dev)) return MLPK_ERR_CUDA;
      if ((rc = launch_kernel(kern, grid, Cfg32::THREADS, Cfg32::SMEM_BYTES, st, maps, num_tiles))) return rc;
    } else {
      auto kern = mlpk::mlp_bwd_kernel<NetT>;
      if (!set_smem_once(kern, Cfg::SMEM_BYTES, dev)) return MLPK_ERR_CUDA;
      if ((rc = launch_kernel(kern, grid, Cfg::THREADS, Cfg::SMEM_BYTES, st, maps, num_tiles))) return rc;
    }
  }
  return launch_reduce(static_cast<const float*>(ws), grid, nfloats, 1, dw, dw_layout<NetT>(rd), st);
}

// ------------------------------------------------------------------ streamed weights
// Networks whose weights do not fit in shared memory (D = H = OUT = 256).
constexpr int kStreamEpw = 8;

template <class NetT>
int launch_stream_fwd(const int* rd, const void* x, const void* const* W, void* out, int64_t M,
                      void* const* hsave, bool h32, cudaStream_t st) {
  if (hsave && h32) return MLPK_ERR_UNSUPPORTED;  // streamed networks save fp16 activations
  using Cfg = mlpk::StreamCfg<NetT, kStreamEpw>;
  constexpr int L = NetT::L;
  DevInfo di;
  int dev = 0;
  int rc = current_device_info(&di, &dev);
  if (rc != MLPK_OK) return rc;
  if (M == 0) return MLPK_OK;
  if (M > (int64_t(1) << 31) - 256) return MLPK_ERR_SHAPE;
  mlpk::StreamMaps<L> maps;
  std::memset(&maps, 0, sizeof(maps));
  if ((rc = make_map_2d(&maps.in, x, rd[0], M, 64, mlpk::kTileM))) return rc;
  if ((rc = make_map_2d(&maps.out, out, rd[L], M, 64, mlpk::kTileM))) return rc;
  int wrc = MLPK_OK;
  mlpk::static_for<0, L>([&](auto lc) {
    constexpr int l = decltype(lc)::value;
    // W_l [d_l][d_{l+1}]: K-chunks of 64 rows read as {64 columns, 64 rows} boxes
    if (wrc == MLPK_OK) wrc = make_map_2d(&maps.w[l], W[l], rd[l + 1], rd[l], 64, mlpk::kStreamK);
  });
  if (wrc) return wrc;
  if (hsave) {
    for (int l = 0; l + 1 < L; ++l) {
      if (!hsave[l]) return MLPK_ERR_NULL;
      if ((rc = make_map_2d(&maps.save[l], hsave[l], rd[l + 1], M, 64, mlpk::kTileM))) return rc;
    }
  }
  maps.M = static_cast<int>(M);
  maps.out_cols = rd[L];
  for (int l = 0; l + 1 < L; ++l) maps.save_cols[l] = maps.hact_cols[l] = rd[l + 1];
  const int64_t tiles = (M + mlpk::kTileM - 1) / mlpk::kTileM;
  const int grid = static_cast<int>(tiles < di.sm_count ? tiles : di.sm_count);
  if (hsave) {
    auto kern = mlpk::mlp_stream_kernel<NetT, kStreamEpw, mlpk::kStreamFwd, true>;
    if (!set_smem_once(kern, Cfg::SMEM_BYTES, dev)) return MLPK_ERR_CUDA;
    return launch_kernel(kern, grid, Cfg::THREADS, Cfg::SMEM_BYTES, st, maps, static_cast<int>(tiles));
  }
  auto kern = mlpk::mlp_stream_kernel<NetT, kStreamEpw, mlpk::kStreamFwd, false>;
  if (!set_smem_once(kern, Cfg::SMEM_BYTES, dev)) return MLPK_ERR_CUDA;
  return launch_kernel_early(kern, grid, Cfg::THREADS, Cfg::SMEM_BYTES, st, maps, static_cast<int>(tiles));
}

// fp32 forward on tf32 tensor cores (networks up to 128 wide): x, W and out
// fp32, every GEMM kind::tf32, hidden activations fp32 in TMEM.
template <class NetT>
int launch_stream_fwd_tf32(const int* rd, const void* x, const void* const* W, void* out, int64_t M,
                           cudaStream_t st) {
  using Cfg = mlpk::StreamCfg<NetT, kStreamEpw, true>;
  constexpr int L = NetT::L;
  DevInfo di;
  int dev = 0;
  int rc = current_device_info(&di, &dev);
  if (rc != MLPK_OK) return rc;
  if (M == 0) return MLPK_OK;
  if (M > (int64_t(1) << 31) - 256) return MLPK_ERR_SHAPE;
  mlpk::StreamMaps<L> maps;
  std::memset(&maps, 0, sizeof(maps));
  if ((rc = make_map_2d(&maps.in, x, rd[0], M, 32, mlpk::kTileM, 4))) return rc;
  if ((rc = make_map_2d(&maps.out, out, rd[L], M, 32, mlpk::kTileM, 4))) return rc;
  for (int l = 0; l < L; ++l)  // K-chunks of 64 rows, boxes {32 columns, 64 rows}, 32-byte atoms
    if ((rc = make_map_2d(&maps.w[l], W[l], rd[l + 1], rd[l], 32, mlpk::kStreamK, 4, true))) return rc;
  maps.M = static_cast<int>(M);
  maps.out_cols = rd[L];
  const int64_t tiles = (M + mlpk::kTileM - 1) / mlpk::kTileM;
  const int grid = static_cast<int>(tiles < di.sm_count ? tiles : di.sm_count);
  auto kern = mlpk::mlp_stream_kernel<NetT, kStreamEpw, mlpk::kStreamFwd, false, true>;
  if (!set_smem_once(kern, Cfg::SMEM_BYTES, dev)) return MLPK_ERR_CUDA;
  return launch_kernel_early(kern, grid, Cfg::THREADS, Cfg::SMEM_BYTES, st, maps, static_cast<int>(tiles));
}

// Workspace of the streamed backward: the data-gradient chain's dz_1..dz_{L-1}
// (fp16 [M, H] each, read back by the weight-gradient kernel), then the fp32
// partials of the weight-gradient CTAs.
template <class NetT>
struct StreamBwdLayout {
  static constexpr int L = NetT::L;
  static constexpr int DA = NetT::template D<0>();
  static constexpr int DB = NetT::template D<1>();
  static_assert(NetT::all_dims_are(DA), "streamed backward serves equal widths");
  static int ctas_per_layer(int sm_count) { return sm_count / L > 0 ? sm_count / L : 1; }
  static size_t dz_bytes(int64_t M) { return static_cast<size_t>(M) * DB * 2; }
  static size_t partial_offset(int64_t M) {
    return (static_cast<size_t>(L - 1) * dz_bytes(M) + 255) / 256 * 256;
  }
  static size_t total(int64_t M, int sm_count) {
    return partial_offset(M) +
           static_cast<size_t>(ctas_per_layer(sm_count)) * L * DA * DB * sizeof(float);
  }
};

template <class NetT>
size_t stream_bwd_workspace(int64_t M, int sm_count) {
  return StreamBwdLayout<NetT>::total(M, sm_count);
}

template <class NetT>
int launch_stream_bwd(const int* rd, const void* x, const void* const* W, const void* const* h, bool h32,
                      const void* g, void* dx, float* ws, size_t ws_bytes, float* dw, int64_t M,
                      cudaStream_t st) {
  if (h32) return MLPK_ERR_UNSUPPORTED;  // streamed networks save fp16 activations
  using Lay = StreamBwdLayout<NetT>;
  using Chain = mlpk::NetReverse<NetT>;
  using Cfg = mlpk::StreamCfg<Chain, kStreamEpw>;
  using WCfg = mlpk::WgradCfg<Lay::DA, Lay::DB>;
  constexpr int L = NetT::L;
  DevInfo di;
  int dev = 0;
  int rc = current_device_info(&di, &dev);
  if (rc != MLPK_OK) return rc;
  if (M > (int64_t(1) << 31) - 256) return MLPK_ERR_SHAPE;
  if (ws_bytes < Lay::total(M, di.sm_count)) return MLPK_ERR_SHAPE;
  uint8_t* wsb = reinterpret_cast<uint8_t*>(ws);
  void* dz[L > 1 ? L - 1 : 1];  // dz[l - 1] = dz_l, l = 1 .. L-1
  for (int l = 1; l < L; ++l) dz[l - 1] = wsb + static_cast<size_t>(l - 1) * Lay::dz_bytes(M);
  float* partials = reinterpret_cast<float*>(wsb + Lay::partial_offset(M));
  const int P = Lay::ctas_per_layer(di.sm_count);
  if (M > 0) {
    // 1. data-gradient chain: stage s handles layer l = L-1-s
    mlpk::StreamMaps<L> maps;
    std::memset(&maps, 0, sizeof(maps));
    if ((rc = make_map_2d(&maps.in, g, rd[L], M, 64, mlpk::kTileM))) return rc;
    if ((rc = make_map_2d(&maps.out, dx, rd[0], M, 64, mlpk::kTileM))) return rc;
    int wrc = MLPK_OK;
    mlpk::static_for<0, L>([&](auto sc) {
      constexpr int s = decltype(sc)::value;
      constexpr int l = L - 1 - s;
      // W_l [d_l][d_{l+1}] read as W_l^T K-chunks: boxes {64 columns, all d_l rows}
      if (wrc == MLPK_OK)
        wrc = make_map_2d(&maps.w[s], W[l], rd[l + 1], rd[l], 64, NetT::template D<l>());
    });
    if (wrc) return wrc;
    for (int s = 0; s + 1 < L; ++s) {
      const int l = L - 1 - s;
      maps.hact[s] = h[l - 1];
      maps.hact_cols[s] = rd[l];
      // dz_l is this library's scratch: the kernel network's width
      maps.save_cols[s] = Cfg::H;
      if ((rc = make_map_2d(&maps.save[s], dz[l - 1], Cfg::H, M, 64, mlpk::kTileM))) return rc;
    }
    maps.M = static_cast<int>(M);
    maps.out_cols = rd[0];
    const int64_t tiles = (M + mlpk::kTileM - 1) / mlpk::kTileM;
    const int grid = static_cast<int>(tiles < di.sm_count ? tiles : di.sm_count);
    auto kern = mlpk::mlp_stream_kernel<Chain, kStreamEpw, mlpk::kStreamDgrad, true>;
    if (!set_smem_once(kern, Cfg::SMEM_BYTES, dev)) return MLPK_ERR_CUDA;
    if ((rc = launch_kernel(kern, grid, Cfg::THREADS, Cfg::SMEM_BYTES, st, maps, static_cast<int>(tiles))))
      return rc;
  }
  // 2. split-K weight gradients: P CTAs per layer (an empty share writes zeros)
  {
    mlpk::WgradMaps<L> wm;
    std::memset(&wm, 0, sizeof(wm));
    const int64_t rows = M > 0 ? M : 1;  // a map needs a non-empty tensor; no stage reads it at M = 0
    for (int l = 0; l < L; ++l) {
      const void* a = l == 0 ? x : h[l - 1];
      const void* b = l == L - 1 ? g : dz[l];
      int acols = rd[l], bcols = l == L - 1 ? rd[L] : Lay::DB;  // dz_l: scratch, full width
      if (M == 0) {  // never read
        a = b = ws;
        acols = Lay::DA;
        bcols = Lay::DB;
      }
      if ((rc = make_map_2d(&wm.a[l], a, acols, rows, 64, mlpk::kWgStageRows))) return rc;
      if ((rc = make_map_2d(&wm.b[l], b, bcols, rows, 64, mlpk::kWgStageRows))) return rc;
    }
    wm.partials = partials;
    auto kern = mlpk::mlp_wgrad_kernel<L, Lay::DA, Lay::DB>;
    if (!set_smem_once(kern, WCfg::SMEM_BYTES, dev)) return MLPK_ERR_CUDA;
    if ((rc = launch_kernel(kern, P * L, WCfg::THREADS, WCfg::SMEM_BYTES, st, wm, static_cast<int>(M), P)))
      return rc;
  }
  // 3. fixed-order sum of each layer's P partials
  constexpr int nfloats = Lay::DA * Lay::DB;
  return launch_reduce(static_cast<const float*>(partials), P, nfloats, L, dw, dw_layout<NetT>(rd), st);
}

// ------------------------------------------------------------------ dispatch
using Fwd = int (*)(const int*, const void*, const void* const*, void*, int64_t, void* const*, bool,
                   cudaStream_t);
using Bwd = int (*)(const int*, const void*, const void* const*, const void* const*, bool, const void*,
                    void*, float*, size_t, float*, int64_t, cudaStream_t);
using BwdWs = size_t (*)(int64_t, int);
using Fwd32 = int (*)(const int*, const void*, const void* const*, void*, int64_t, cudaStream_t);

struct ShapeOps {
  Fwd fwd = nullptr;
  Bwd bwd = nullptr;
  BwdWs bwd_ws = nullptr;
  bool h32 = false;  // fp32 saved activations served (the fused kernels)
  Fwd32 fwd32 = nullptr;  // fp32 forward on tf32 tensor cores (up to 128 wide)
};

// The compiled networks, smallest first.  A caller's network is served by the
// first one of its depth that covers it: every width at most the compiled
// width and a multiple of 8 (16-byte rows, the TMA stride rule).  The missing
// rows and columns are zero-filled by TMA on the way in and clipped on the
// way out; zero inputs and weights contribute exact zeros, and the padded
// hidden units feed only zero weight rows, so the caller's outputs and
// gradients are those of its own network.  The reference's widths are all
// multiples of 16 (its tl.dot tiles, kernel.py:25-53).
template <class NetT>
bool covers(const mlpk_shape* s) {
  if (s->num_layers != NetT::L) return false;
  for (int i = 0; i <= NetT::L; ++i)
    if (s->dims[i] > NetT::dim(i) || s->dims[i] % 8 != 0) return false;
  return true;
}

// Row tiles in flight per CTA of the forward (slots): 2 for 128-wide layers
// (2 slots x 2 accumulators x 128 columns fill TMEM), 3 for 64-wide ones
// (384 columns; measured at 1M rows: 5-layer forward 135 -> 123 us, training
// forward 170 -> 132 us; 64^3 forward 80 -> 74 us).
ShapeOps pick_ops(const mlpk_shape* s, bool training) {
  using N64 = Net<64, 64, 64, 64>;
  using N3 = Net<128, 128, 128, 128>;
  using N256 = Net<256, 256, 256, 256>;
  using N5 = Net<32, 64, 64, 64, 64, 16>;
  using N5w64 = Net<64, 64, 64, 64, 64, 64>;
  using N5w128 = Net<128, 128, 128, 128, 128, 128>;
  using N5w256 = Net<256, 256, 256, 256, 256, 256>;
  using N2w64 = Net<64, 64, 64>;
  using N2w128 = Net<128, 128, 128>;
  using N2w256 = Net<256, 256, 256>;
  using N4w64 = Net<64, 64, 64, 64, 64>;
  using N4w128 = Net<128, 128, 128, 128, 128>;
  using N4w256 = Net<256, 256, 256, 256, 256>;
  // deeper uniform networks, up to MLPK_MAX_LAYERS: 64 wide on the fused
  // kernels while the backward's weight gradients fit in TMEM (6 and 7
  // layers; an 8-layer 64-wide network runs on the 128-wide kernels), 128 and
  // 256 wide on the streamed-weight kernels
  using N6w64 = Net<64, 64, 64, 64, 64, 64, 64>;
  using N7w64 = Net<64, 64, 64, 64, 64, 64, 64, 64>;
  using N6w128 = Net<128, 128, 128, 128, 128, 128, 128>;
  using N7w128 = Net<128, 128, 128, 128, 128, 128, 128, 128>;
  using N8w128 = Net<128, 128, 128, 128, 128, 128, 128, 128, 128>;
  using N6w256 = Net<256, 256, 256, 256, 256, 256, 256>;
  using N7w256 = Net<256, 256, 256, 256, 256, 256, 256, 256>;
  using N8w256 = Net<256, 256, 256, 256, 256, 256, 256, 256, 256>;
  ShapeOps o;
  if (covers<N64>(s)) {
    o.fwd = &launch_fwd<N64, 3, 4>;
    o.bwd = &launch_bwd<N64>;
    o.bwd_ws = &bwd_workspace<N64>;
    o.fwd32 = &launch_stream_fwd_tf32<N64>;
    o.h32 = true;
  } else if (covers<N3>(s)) {
    o.fwd = &launch_fwd<N3, 2, 4>;
    o.bwd = &launch_bwd<N3>;
    o.bwd_ws = &bwd_workspace<N3>;
    o.fwd32 = &launch_stream_fwd_tf32<N3>;
    o.h32 = true;
  } else if (covers<N256>(s)) {
    o.fwd = &launch_stream_fwd<N256>;
    o.bwd = &launch_stream_bwd<N256>;
    o.bwd_ws = &stream_bwd_workspace<N256>;
  } else if (covers<N5>(s)) {
    o.fwd = &launch_fwd<N5, 3, 4>;
    o.bwd = &launch_bwd<N5>;
    o.bwd_ws = &bwd_workspace<N5>;
    o.fwd32 = &launch_stream_fwd_tf32<N5w64>;
    o.h32 = true;
  } else if (covers<N5w64>(s)) {
    o.fwd = &launch_fwd<N5w64, 3, 4>;
    o.bwd = &launch_bwd<N5w64>;
    o.bwd_ws = &bwd_workspace<N5w64>;
    o.fwd32 = &launch_stream_fwd_tf32<N5w64>;
    o.h32 = true;
  } else if (covers<N5w128>(s)) {
    o.fwd = &launch_stream_fwd<N5w128>;
    o.bwd = &launch_stream_bwd<N5w128>;
    o.bwd_ws = &stream_bwd_workspace<N5w128>;
    o.fwd32 = &launch_stream_fwd_tf32<N5w128>;
  } else if (covers<N5w256>(s)) {
    o.fwd = &launch_stream_fwd<N5w256>;
    o.bwd = &launch_stream_bwd<N5w256>;
    o.bwd_ws = &stream_bwd_workspace<N5w256>;
  } else if (covers<N2w64>(s)) {  // one hidden layer
    o.fwd = &launch_fwd<N2w64, 3, 4>;
    o.bwd = &launch_bwd<N2w64>;
    o.bwd_ws = &bwd_workspace<N2w64>;
    o.fwd32 = &launch_stream_fwd_tf32<N2w64>;
    o.h32 = true;
  } else if (covers<N2w128>(s)) {
    o.fwd = &launch_fwd<N2w128, 2, 4>;
    o.bwd = &launch_bwd<N2w128>;
    o.bwd_ws = &bwd_workspace<N2w128>;
    o.fwd32 = &launch_stream_fwd_tf32<N2w128>;
    o.h32 = true;
  } else if (covers<N2w256>(s)) {
    o.fwd = &launch_stream_fwd<N2w256>;
    o.bwd = &launch_stream_bwd<N2w256>;
    o.bwd_ws = &stream_bwd_workspace<N2w256>;
  } else if (covers<N4w64>(s)) {  // three hidden layers
    o.fwd = &launch_fwd<N4w64, 3, 4>;
    o.bwd = &launch_bwd<N4w64>;
    o.bwd_ws = &bwd_workspace<N4w64>;
    o.fwd32 = &launch_stream_fwd_tf32<N4w64>;
    o.h32 = true;
  } else if (covers<N4w128>(s)) {
    o.fwd = &launch_stream_fwd<N4w128>;
    o.bwd = &launch_stream_bwd<N4w128>;
    o.bwd_ws = &stream_bwd_workspace<N4w128>;
    o.fwd32 = &launch_stream_fwd_tf32<N4w128>;
  } else if (covers<N4w256>(s)) {
    o.fwd = &launch_stream_fwd<N4w256>;
    o.bwd = &launch_stream_bwd<N4w256>;
    o.bwd_ws = &stream_bwd_workspace<N4w256>;
  } else if (covers<N6w64>(s)) {  // five hidden layers
    o.fwd = &launch_fwd<N6w64, 3, 4>;
    o.bwd = &launch_bwd<N6w64>;
    o.bwd_ws = &bwd_workspace<N6w64>;
    o.fwd32 = &launch_stream_fwd_tf32<N6w64>;
    o.h32 = true;
  } else if (covers<N6w128>(s)) {
    o.fwd = &launch_stream_fwd<N6w128>;
    o.bwd = &launch_stream_bwd<N6w128>;
    o.bwd_ws = &stream_bwd_workspace<N6w128>;
    o.fwd32 = &launch_stream_fwd_tf32<N6w128>;
  } else if (covers<N6w256>(s)) {
    o.fwd = &launch_stream_fwd<N6w256>;
    o.bwd = &launch_stream_bwd<N6w256>;
    o.bwd_ws = &stream_bwd_workspace<N6w256>;
  } else if (covers<N7w64>(s)) {  // six hidden layers
    o.fwd = &launch_fwd<N7w64, 3, 4>;
    o.bwd = &launch_bwd<N7w64>;
    o.bwd_ws = &bwd_workspace<N7w64>;
    o.fwd32 = &launch_stream_fwd_tf32<N7w64>;
    o.h32 = true;
  } else if (covers<N7w128>(s)) {
    o.fwd = &launch_stream_fwd<N7w128>;
    o.bwd = &launch_stream_bwd<N7w128>;
    o.bwd_ws = &stream_bwd_workspace<N7w128>;
    o.fwd32 = &launch_stream_fwd_tf32<N7w128>;
  } else if (covers<N7w256>(s)) {
    o.fwd = &launch_stream_fwd<N7w256>;
    o.bwd = &launch_stream_bwd<N7w256>;
    o.bwd_ws = &stream_bwd_workspace<N7w256>;
  } else if (covers<N8w128>(s)) {  // seven hidden layers (64 wide included)
    o.fwd = &launch_stream_fwd<N8w128>;
    o.bwd = &launch_stream_bwd<N8w128>;
    o.bwd_ws = &stream_bwd_workspace<N8w128>;
    o.fwd32 = &launch_stream_fwd_tf32<N8w128>;
  } else if (covers<N8w256>(s)) {
    o.fwd = &launch_stream_fwd<N8w256>;
    o.bwd = &launch_stream_bwd<N8w256>;
    o.bwd_ws = &stream_bwd_workspace<N8w256>;
  }
  return o;
}

int check_shape(const mlpk_shape* s) {
  if (!s) return MLPK_ERR_NULL;
  if (s->num_layers < 1 || s->num_layers > MLPK_MAX_LAYERS) return MLPK_ERR_SHAPE;
  for (int i = 0; i <= s->num_layers; ++i)
    if (s->dims[i] <= 0) return MLPK_ERR_SHAPE;
  return MLPK_OK;
}

}  // namespace

extern "C" {

const char* mlpk_status_string(int status) {
  switch (status) {
    case MLPK_OK: return "ok";
    case MLPK_ERR_SHAPE: return "invalid shape";
    case MLPK_ERR_UNSUPPORTED: return "no kernel compiled for this shape";
    case MLPK_ERR_ARCH: return "device is not sm_100 (B200)";
    case MLPK_ERR_CUDA: return "CUDA runtime/driver call failed";
    case MLPK_ERR_ALIGN: return "pointer not 16-byte aligned";
    case MLPK_ERR_NULL: return "required pointer is NULL";
    case MLPK_ERR_DEVICE: return "kernel recorded a device-side error";
    case MLPK_ERR_SCRATCH:
      return "problem needs more scratch than the allocation-free entry point's static buffer";
    default: return "unknown status";
  }
}

int mlpk_shape_supported(const mlpk_shape* shape) {
  if (check_shape(shape) != MLPK_OK) return 0;
  return pick_ops(shape, false).fwd != nullptr ? 1 : 0;
}

int mlpk_shape_supported_ex(const mlpk_shape* shape, int dtype) {
  if (check_shape(shape) != MLPK_OK) return 0;
  const ShapeOps o = pick_ops(shape, false);
  if (dtype == MLPK_DT_F16) return o.fwd != nullptr ? 1 : 0;
  if (dtype == MLPK_DT_F32) return o.fwd32 != nullptr ? 1 : 0;
  return 0;
}

int mlpk_train_supported_ex(const mlpk_shape* shape, int h_dtype) {
  if (check_shape(shape) != MLPK_OK) return 0;
  if (h_dtype != MLPK_H_F16 && h_dtype != MLPK_H_F32) return 0;
  const ShapeOps o = pick_ops(shape, true);
  return (o.fwd != nullptr && o.bwd != nullptr && (h_dtype == MLPK_H_F16 || o.h32)) ? 1 : 0;
}

int mlpk_train_supported(const mlpk_shape* shape) { return mlpk_train_supported_ex(shape, MLPK_H_F16); }

namespace {
int check_fwd_args(const mlpk_shape* shape, int64_t M, const void* x, const void* const* W,
                   const void* out) {
  int rc = check_shape(shape);
  if (rc) return rc;
  if (M < 0) return MLPK_ERR_SHAPE;
  if (!W) return MLPK_ERR_NULL;
  if (M > 0 && (!x || !out)) return MLPK_ERR_NULL;
  for (int l = 0; l < shape->num_layers; ++l) {
    if (!W[l]) return MLPK_ERR_NULL;
    if (!aligned16(W[l])) return MLPK_ERR_ALIGN;
  }
  if (!aligned16(x) || !aligned16(out)) return MLPK_ERR_ALIGN;
  return MLPK_OK;
}
}  // namespace

int mlpk_fwd(const mlpk_shape* shape, int64_t M, const void* x, const void* const* W, void* out,
             mlpk_stream_t stream) {
  int rc = check_fwd_args(shape, M, x, W, out);
  if (rc) return rc;
  Fwd f = pick_ops(shape, false).fwd;
  if (!f) return MLPK_ERR_UNSUPPORTED;
  return f(shape->dims, x, W, out, M, nullptr, false, static_cast<cudaStream_t>(stream));
}

int mlpk_fwd_ex(const mlpk_shape* shape, int64_t M, const void* x, const void* const* W, void* out, int dtype,
                mlpk_stream_t stream) {
  if (dtype == MLPK_DT_F16) return mlpk_fwd(shape, M, x, W, out, stream);
  if (dtype != MLPK_DT_F32) return MLPK_ERR_SHAPE;
  int rc = check_fwd_args(shape, M, x, W, out);
  if (rc) return rc;
  const Fwd32 f = pick_ops(shape, false).fwd32;
  if (!f) return MLPK_ERR_UNSUPPORTED;
  return f(shape->dims, x, W, out, M, static_cast<cudaStream_t>(stream));
}

int mlpk_train_fwd_ex(const mlpk_shape* shape, int64_t M, const void* x, const void* const* W,
                      void* out, void* const* h_saved, int h_dtype, mlpk_stream_t stream) {
  int rc = check_fwd_args(shape, M, x, W, out);
  if (rc) return rc;
  if (h_dtype != MLPK_H_F16 && h_dtype != MLPK_H_F32) return MLPK_ERR_SHAPE;
  if (!h_saved) return MLPK_ERR_NULL;
  for (int l = 0; l + 1 < shape->num_layers; ++l) {
    if (M > 0 && !h_saved[l]) return MLPK_ERR_NULL;
    if (!aligned16(h_saved[l])) return MLPK_ERR_ALIGN;
  }
  const ShapeOps o = pick_ops(shape, true);
  if (!o.fwd || !o.bwd || (h_dtype == MLPK_H_F32 && !o.h32)) return MLPK_ERR_UNSUPPORTED;
  return o.fwd(shape->dims, x, W, out, M, h_saved, h_dtype == MLPK_H_F32, static_cast<cudaStream_t>(stream));
}

int mlpk_train_fwd(const mlpk_shape* shape, int64_t M, const void* x, const void* const* W,
                   void* out, void* const* h_saved, mlpk_stream_t stream) {
  return mlpk_train_fwd_ex(shape, M, x, W, out, h_saved, MLPK_H_F16, stream);
}

int64_t mlpk_bwd_workspace_size(const mlpk_shape* shape, int64_t M) {
  if (check_shape(shape) != MLPK_OK || M < 0) return -1;
  const ShapeOps o = pick_ops(shape, true);
  if (!o.bwd_ws) return -1;
  DevInfo di;
  if (current_device_info(&di, nullptr) != MLPK_OK) return -1;
  return static_cast<int64_t>(o.bwd_ws(M, di.sm_count));
}

int mlpk_bwd_ex(const mlpk_shape* shape, int64_t M, const void* x, const void* const* W,
                const void* const* h_saved, int h_dtype, const void* grad_out, void* dx, void* workspace,
                int64_t workspace_bytes, float* dW, mlpk_stream_t stream) {
  int rc = check_fwd_args(shape, M, x, W, grad_out);
  if (rc) return rc;
  if (h_dtype != MLPK_H_F16 && h_dtype != MLPK_H_F32) return MLPK_ERR_SHAPE;
  if (!dW || (M > 0 && (!dx || !h_saved || !workspace))) return MLPK_ERR_NULL;
  if (!aligned16(dx) || !aligned16(dW) || !aligned16(workspace)) return MLPK_ERR_ALIGN;
  for (int l = 0; M > 0 && l + 1 < shape->num_layers; ++l) {
    if (!h_saved[l]) return MLPK_ERR_NULL;
    if (!aligned16(h_saved[l])) return MLPK_ERR_ALIGN;
  }
  if (workspace_bytes < 0) return MLPK_ERR_SHAPE;
  const ShapeOps o = pick_ops(shape, true);
  if (!o.bwd || (h_dtype == MLPK_H_F32 && !o.h32)) return MLPK_ERR_UNSUPPORTED;
  return o.bwd(shape->dims, x, W, h_saved, h_dtype == MLPK_H_F32, grad_out, dx, static_cast<float*>(workspace),
               static_cast<size_t>(workspace_bytes), dW, M, static_cast<cudaStream_t>(stream));
}

int mlpk_bwd(const mlpk_shape* shape, int64_t M, const void* x, const void* const* W,
             const void* const* h_saved, const void* grad_out, void* dx, void* workspace,
             int64_t workspace_bytes, float* dW, mlpk_stream_t stream) {
  return mlpk_bwd_ex(shape, M, x, W, h_saved, MLPK_H_F16, grad_out, dx, workspace, workspace_bytes, dW, stream);
}

namespace {
int make_wn_shape(const mlpk_shape* s, mlpk::WnShape* w) {
  int rc = check_shape(s);
  if (rc) return rc;
  w->num_layers = s->num_layers;
  long long vo = 0;
  int go = 0;
  for (int l = 0; l < s->num_layers; ++l) {
    // a column's rows live in the registers of 32 row-group threads
    if (s->dims[l] > mlpk::kWnRowGroups * mlpk::kWnMaxPer) return MLPK_ERR_UNSUPPORTED;
    w->din[l] = s->dims[l];
    w->dout[l] = s->dims[l + 1];
    w->voff[l] = vo;
    w->goff[l] = go;
    vo += static_cast<long long>(s->dims[l]) * s->dims[l + 1];
    go += s->dims[l + 1];
  }
  w->total_cols = go;
  return MLPK_OK;
}
}  // namespace

int mlpk_wn_fwd(const mlpk_shape* shape, const float* v_all, const float* g_all, void* const* W,
                float* inv_norm, mlpk_stream_t stream) {
  mlpk::WnShape ws;
  int rc = make_wn_shape(shape, &ws);
  if (rc) return rc;
  if (!v_all || !g_all || !W || !inv_norm) return MLPK_ERR_NULL;
  mlpk::WnOut out;
  for (int l = 0; l < shape->num_layers; ++l) {
    if (!W[l]) return MLPK_ERR_NULL;
    out.w[l] = static_cast<__half*>(W[l]);
  }
  DevInfo di;
  if ((rc = current_device_info(&di, nullptr)) != MLPK_OK) return rc;
  return launch_kernel(mlpk::mlp_wn_fwd_kernel, mlpk::wn_num_blocks(ws),
                       mlpk::kWnCols * mlpk::kWnRowGroups, 0, static_cast<cudaStream_t>(stream), ws,
                       v_all, g_all, out, inv_norm);
}

int mlpk_wn_bwd(const mlpk_shape* shape, const float* dW_all, const float* v_all,
                const float* g_all, const float* inv_norm, float* dv_all, float* dg_all,
                mlpk_stream_t stream) {
  mlpk::WnShape ws;
  int rc = make_wn_shape(shape, &ws);
  if (rc) return rc;
  if (!dW_all || !v_all || !g_all || !inv_norm || !dv_all || !dg_all) return MLPK_ERR_NULL;
  DevInfo di;
  if ((rc = current_device_info(&di, nullptr)) != MLPK_OK) return rc;
  return launch_kernel(mlpk::mlp_wn_bwd_kernel, mlpk::wn_num_blocks(ws),
                       mlpk::kWnCols * mlpk::kWnRowGroups, 0, static_cast<cudaStream_t>(stream), ws,
                       dW_all, v_all, g_all, inv_norm, dv_all, dg_all);
}

// ------------------------------------------------------------------ allocation-free backward
// Backward for callers that cannot allocate device memory when they call it
// (plain C / FFI callers that hold only their input and output buffers and no
// device allocator, serving processes whose device memory is fixed at
// start-up).  Instead of a caller-provided workspace, the per-CTA
// weight-gradient partials live in this file-scope array, which every GPU that
// loads the library holds until the process exits.
}  // extern "C"

static __device__ __align__(256) unsigned char g_bwd_noalloc_scratch[MLPK_BWD_NOALLOC_SCRATCH_BYTES];

namespace {
void* g_noalloc_scratch_ptr[kMaxDevices] = {};
std::mutex g_noalloc_mu;

// The device address of the scratch array on the current device.  In host
// code the array's name is only a host-side stand-in, so the address is looked
// up once per device (with that device current) and cached.
int noalloc_scratch(void** out) {
  int dev = 0;
  const int drc = cuda_status(cudaGetDevice(&dev));
  if (drc) return drc;
  if (dev < 0 || dev >= kMaxDevices) return MLPK_ERR_DEVICE;
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (!g_noalloc_scratch_ptr[dev]) {
    void* p = nullptr;
    const int rc = cuda_status(cudaGetSymbolAddress(&p, g_bwd_noalloc_scratch));
    if (rc) return rc;
    if (p == nullptr) return driver_status("cudaGetSymbolAddress gave NULL", -1);
    g_noalloc_scratch_ptr[dev] = p;
  }
  *out = g_noalloc_scratch_ptr[dev];
  return MLPK_OK;
}
}  // namespace

extern "C" {

int mlpk_bwd_noalloc(const mlpk_shape* shape, int64_t M, const void* x, const void* const* W,
                     const void* const* h_saved, const void* grad_out, void* dx, float* dW,
                     mlpk_stream_t stream) {
  int rc = check_shape(shape);
  if (rc) return rc;
  if (M < 0) return MLPK_ERR_SHAPE;
  const ShapeOps o = pick_ops(shape, true);
  if (!o.bwd_ws) return MLPK_ERR_UNSUPPORTED;
  DevInfo di;
  if ((rc = current_device_info(&di, nullptr)) != MLPK_OK) return rc;  // CUDA failure or not sm_100
  const size_t need = o.bwd_ws(M, di.sm_count);
  if (need > static_cast<size_t>(MLPK_BWD_NOALLOC_SCRATCH_BYTES)) return MLPK_ERR_SCRATCH;
  void* scratch = nullptr;
  if ((rc = noalloc_scratch(&scratch)) != MLPK_OK) return rc;
  // Every call reuses the same array: the backward kernel overwrites the
  // partials of every CTA it launches before the reduction reads them, so no
  // stale contents from an earlier call are ever read.
  return mlpk_bwd(shape, M, x, W, h_saved, grad_out, dx, scratch,
                  static_cast<int64_t>(MLPK_BWD_NOALLOC_SCRATCH_BYTES), dW, stream);
}

// ------------------------------------------------------------------ host-resident rows
namespace {
constexpr int kPipeBufs = MLPK_FWD_HOST_BUFFERS;

// Copy streams and events of one host thread on one device (created on first
// use, kept for the thread's lifetime).
struct HostPipe {
  bool ready = false;
  cudaStream_t h2d = nullptr, d2h = nullptr;
  cudaEvent_t start = nullptr;
  cudaEvent_t in_ready[kPipeBufs] = {};   // chunk copied into x buffer b
  cudaEvent_t comp_done[kPipeBufs] = {};  // forward of buffer b done (x_b free, out_b written)
  cudaEvent_t out_done[kPipeBufs] = {};   // out buffer b copied out (free again)
};

int host_pipe(int dev, HostPipe** out) {
  thread_local HostPipe pipes[kMaxDevices];
  HostPipe& p = pipes[dev];
  if (!p.ready) {
    int rc;
    if ((rc = cuda_status(cudaStreamCreateWithFlags(&p.h2d, cudaStreamNonBlocking))) ||
        (rc = cuda_status(cudaStreamCreateWithFlags(&p.d2h, cudaStreamNonBlocking))) ||
        (rc = cuda_status(cudaEventCreateWithFlags(&p.start, cudaEventDisableTiming))))
      return rc;
    for (int b = 0; b < kPipeBufs; ++b)
      if ((rc = cuda_status(cudaEventCreateWithFlags(&p.in_ready[b], cudaEventDisableTiming))) ||
          (rc = cuda_status(cudaEventCreateWithFlags(&p.comp_done[b], cudaEventDisableTiming))) ||
          (rc = cuda_status(cudaEventCreateWithFlags(&p.out_done[b], cudaEventDisableTiming))))
        return rc;
    p.ready = true;
  }
  *out = &p;
  return MLPK_OK;
}

size_t host_chunk_bytes(int64_t rows, int width) {
  return (static_cast<size_t>(rows) * width * 2 + 255) / 256 * 256;
}
}  // namespace

int64_t mlpk_fwd_host_workspace_size(const mlpk_shape* shape, int64_t chunk_rows) {
  if (check_shape(shape) != MLPK_OK || chunk_rows < 0) return -1;
  if (chunk_rows == 0) chunk_rows = MLPK_FWD_HOST_CHUNK_ROWS;
  const int L = shape->num_layers;
  return static_cast<int64_t>(kPipeBufs * (host_chunk_bytes(chunk_rows, shape->dims[0]) +
                                           host_chunk_bytes(chunk_rows, shape->dims[L])));
}

int mlpk_fwd_host(const mlpk_shape* shape, int64_t M, const void* x_host, const void* const* W,
                  void* out_host, int64_t chunk_rows, void* workspace, int64_t workspace_bytes,
                  mlpk_stream_t stream) {
  int rc = check_shape(shape);
  if (rc) return rc;
  if (M < 0 || chunk_rows < 0) return MLPK_ERR_SHAPE;
  if (chunk_rows == 0) chunk_rows = MLPK_FWD_HOST_CHUNK_ROWS;
  if (!W) return MLPK_ERR_NULL;
  for (int l = 0; l < shape->num_layers; ++l) {
    if (!W[l]) return MLPK_ERR_NULL;
    if (!aligned16(W[l])) return MLPK_ERR_ALIGN;
  }
  const Fwd f = pick_ops(shape, false).fwd;
  if (!f) return MLPK_ERR_UNSUPPORTED;
  if (M == 0) return MLPK_OK;
  if (!x_host || !out_host || !workspace) return MLPK_ERR_NULL;
  if (!aligned16(workspace)) return MLPK_ERR_ALIGN;
  if (workspace_bytes < mlpk_fwd_host_workspace_size(shape, chunk_rows)) return MLPK_ERR_SHAPE;
  DevInfo di;
  int dev = 0;
  if ((rc = current_device_info(&di, &dev)) != MLPK_OK) return rc;
  HostPipe* p = nullptr;
  if ((rc = host_pipe(dev, &p)) != MLPK_OK) return rc;

  const int L = shape->num_layers;
  const int d0 = shape->dims[0], dL = shape->dims[L];
  const size_t xb = host_chunk_bytes(chunk_rows, d0), ob = host_chunk_bytes(chunk_rows, dL);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  auto xbuf = [&](int b) { return ws + b * xb; };
  auto obuf = [&](int b) { return ws + kPipeBufs * xb + b * ob; };
  const auto* xh = static_cast<const uint8_t*>(x_host);
  auto* oh = static_cast<uint8_t*>(out_host);
  cudaStream_t st = static_cast<cudaStream_t>(stream);

  // The copy streams start after the work already queued on `stream` (which
  // may still use the workspace or produce the weights).
  if ((rc = cuda_status(cudaEventRecord(p->start, st))) ||
      (rc = cuda_status(cudaStreamWaitEvent(p->h2d, p->start, 0))) ||
      (rc = cuda_status(cudaStreamWaitEvent(p->d2h, p->start, 0))))
    return rc;
  const int64_t nchunks = (M + chunk_rows - 1) / chunk_rows;
  auto rows_of = [&](int64_t k) { return k + 1 < nchunks ? chunk_rows : M - k * chunk_rows; };
  // copy in chunk k (its buffer is free once the forward of chunk k - B read it)
  auto copy_in = [&](int64_t k) {
    const int b = static_cast<int>(k % kPipeBufs);
    int r = MLPK_OK;
    if (k >= kPipeBufs) r = cuda_status(cudaStreamWaitEvent(p->h2d, p->comp_done[b], 0));
    if (!r)
      r = cuda_status(cudaMemcpyAsync(xbuf(b), xh + static_cast<size_t>(k * chunk_rows) * d0 * 2,
                                      static_cast<size_t>(rows_of(k)) * d0 * 2, cudaMemcpyHostToDevice,
                                      p->h2d));
    if (!r) r = cuda_status(cudaEventRecord(p->in_ready[b], p->h2d));
    return r;
  };
  for (int64_t k = 0; k < nchunks && k < kPipeBufs - 1; ++k)
    if ((rc = copy_in(k))) return rc;
  for (int64_t k = 0; k < nchunks; ++k) {
    const int b = static_cast<int>(k % kPipeBufs);
    // keep B - 1 chunks of input in flight ahead of the forward
    if (k + kPipeBufs - 1 < nchunks && (rc = copy_in(k + kPipeBufs - 1))) return rc;
    // forward of chunk k: its input has arrived and its output buffer is free
    if ((rc = cuda_status(cudaStreamWaitEvent(st, p->in_ready[b], 0)))) return rc;
    if (k >= kPipeBufs && (rc = cuda_status(cudaStreamWaitEvent(st, p->out_done[b], 0)))) return rc;
    if ((rc = f(shape->dims, xbuf(b), W, obuf(b), rows_of(k), nullptr, false, st))) return rc;
    if ((rc = cuda_status(cudaEventRecord(p->comp_done[b], st)))) return rc;
    // copy out chunk k
    if ((rc = cuda_status(cudaStreamWaitEvent(p->d2h, p->comp_done[b], 0))) ||
        (rc = cuda_status(cudaMemcpyAsync(oh + static_cast<size_t>(k * chunk_rows) * dL * 2, obuf(b),
                                          static_cast<size_t>(rows_of(k)) * dL * 2, cudaMemcpyDeviceToHost,
                                          p->d2h))) ||
        (rc = cuda_status(cudaEventRecord(p->out_done[b], p->d2h))))
      return rc;
  }
  // `stream` reaches this point only after the last copy out (and, through
  // it, every earlier one: the copy-out stream is in order)
  const int last = static_cast<int>((nchunks - 1) % kPipeBufs);
  return cuda_status(cudaStreamWaitEvent(st, p->out_done[last], 0));
}

int mlpk_device_status(int clear, int* status_out) {
  int v = 0;
  int rc = cuda_status(cudaMemcpyFromSymbol(&v, mlpk::g_device_status, sizeof(int)));
  if (rc) return rc;
  if (status_out) *status_out = v;
  if (clear) {
    const int z = 0;
    if ((rc = cuda_status(cudaMemcpyToSymbol(mlpk::g_device_status, &z, sizeof(int))))) return rc;
  }
  return MLPK_OK;
}

// ------------------------------------------------------------------ fp32 <-> fp16 casts
namespace {
int cast_grid(int64_t n) {
  DevInfo di;
  if (current_device_info(&di, nullptr) != MLPK_OK) return 0;
  const int64_t want = (n / 8 + 255) / 256;
  const int64_t cap = static_cast<int64_t>(di.sm_count) * 8;
  return static_cast<int>(want < 1 ? 1 : want < cap ? want : cap);
}
}  // namespace

int mlpk_cast_f32_f16(const float* src, void* dst, int64_t n, mlpk_stream_t stream) {
  if (n < 0) return MLPK_ERR_SHAPE;
  if (n == 0) return MLPK_OK;
  if (!src || !dst) return MLPK_ERR_NULL;
  if (!aligned16(src) || !aligned16(dst)) return MLPK_ERR_ALIGN;
  DevInfo di;
  int rc = current_device_info(&di, nullptr);
  if (rc != MLPK_OK) return rc;
  return launch_kernel(mlpk::mlp_cast_f32_f16_kernel, cast_grid(n), 256, 0, static_cast<cudaStream_t>(stream),
                       src, static_cast<__half*>(dst), n);
}

int mlpk_cast_f16_f32(const void* src, float* dst, int64_t n, mlpk_stream_t stream) {
  if (n < 0) return MLPK_ERR_SHAPE;
  if (n == 0) return MLPK_OK;
  if (!src || !dst) return MLPK_ERR_NULL;
  if (!aligned16(src) || !aligned16(dst)) return MLPK_ERR_ALIGN;
  DevInfo di;
  int rc = current_device_info(&di, nullptr);
  if (rc != MLPK_OK) return rc;
  return launch_kernel(mlpk::mlp_cast_f16_f32_kernel, cast_grid(n), 256, 0, static_cast<cudaStream_t>(stream),
                       static_cast<const __half*>(src), dst, n);
}

// ------------------------------------------------------------------ peer-memory dW sum
int mlpk_peer_alloc(int64_t n, void** buf_out, void* handle_out) {
  if (!buf_out || !handle_out) return MLPK_ERR_NULL;
  if (n <= 0 || n % 4 != 0) return MLPK_ERR_SHAPE;
  static_assert(sizeof(cudaIpcMemHandle_t) == MLPK_PEER_HANDLE_BYTES, "IPC handle size");
  // `in`, slot 0 and slot 1 (n floats each), then the ready and epoch words
  const size_t bytes = 3 * static_cast<size_t>(n) * sizeof(float) + mlpk::kPeerFlagWords * sizeof(uint32_t);
  void* p = nullptr;
  int rc = cuda_status(cudaMalloc(&p, bytes));
  if (rc) return rc;
  if ((rc = cuda_status(cudaMemset(p, 0, bytes))) ||
      (rc = cuda_status(cudaIpcGetMemHandle(static_cast<cudaIpcMemHandle_t*>(handle_out), p)))) {
    cudaFree(p);
    return rc;
  }
  *buf_out = p;
  return MLPK_OK;
}

int mlpk_peer_open(const void* handle, void** buf_out) {
  if (!handle || !buf_out) return MLPK_ERR_NULL;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  return cuda_status(cudaIpcOpenMemHandle(buf_out, h, cudaIpcMemLazyEnablePeerAccess));
}

int mlpk_peer_close(void* peer_buf) {
  if (!peer_buf) return MLPK_ERR_NULL;
  return cuda_status(cudaIpcCloseMemHandle(peer_buf));
}

int mlpk_peer_free(void* buf) {
  if (!buf) return MLPK_ERR_NULL;
  return cuda_status(cudaFree(buf));
}

int mlpk_peer_allreduce(void* const* bufs, int world, int rank, int64_t n, float* dW_out,
                        mlpk_stream_t stream) {
  if (!bufs || !dW_out) return MLPK_ERR_NULL;
  if (world < 1 || world > mlpk::kPeerMaxRanks || rank < 0 || rank >= world) return MLPK_ERR_SHAPE;
  if (n <= 0 || n % 4 != 0 || n > (int64_t(1) << 30)) return MLPK_ERR_SHAPE;
  if (!aligned16(dW_out)) return MLPK_ERR_ALIGN;
  mlpk::PeerPtrs peers;
  std::memset(&peers, 0, sizeof(peers));
  for (int q = 0; q < world; ++q) {
    if (!bufs[q]) return MLPK_ERR_NULL;
    peers.buf[q] = static_cast<float*>(bufs[q]);
  }
  DevInfo di;
  int rc = current_device_info(&di, nullptr);
  if (rc != MLPK_OK) return rc;
  // the same grid on every call and every rank (CTA c always owns the same
  // elements and flags): at most one CTA per SM, all resident
  int64_t blocks = (n / 4 + 255) / 256;
  if (blocks > di.sm_count) blocks = di.sm_count;
  if (blocks > mlpk::kPeerMaxCtas) blocks = mlpk::kPeerMaxCtas;
  const int grid = static_cast<int>(blocks);
  return launch_kernel(mlpk::mlp_peer_allreduce_kernel, grid, 256, 0, static_cast<cudaStream_t>(stream),
                       peers, world, rank, static_cast<int>(n), dW_out);
}

const char* mlpk_last_cuda_error(void) {
  return t_last_cuda_error;
}

}  // extern "C"
