/*
 * mlpk -- B200 (sm_100a) fused softplus MLP, C ABI.
 *
 * The drop-in boundary for the reference's fused-MLP path
 * (Marcelo5444/mlp-megakernel).  Every entry point takes plain device
 * pointers, sizes and a CUDA stream; no torch types cross this boundary.  The
 * Python package binds these symbols with ctypes.
 *
 * Conventions (mirroring the reference, kernel.py:130-156):
 *   - weights are [in, out] row-major (out = x @ W), fp16;
 *   - activations x / out / grad_out / dx are [M, d] row-major fp16;
 *   - saved training activations are fp16 (the next GEMM's operand) or, with
 *     the _ex entry points, fp32; weight gradients and weight-norm parameters
 *     fp32;
 *   - every pointer must be 16-byte aligned and tensors contiguous;
 *   - all work is enqueued on `stream`; no entry point synchronises the host
 *     (except mlpk_device_status, which reads a device word);
 *   - return value: MLPK_OK or an MLPK_ERR_* code (mlpk_status_string).
 */
#ifndef MLPK_H_
#define MLPK_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef void* mlpk_stream_t; /* a cudaStream_t */

#define MLPK_MAX_LAYERS 8

/* Network shape: num_layers GEMMs, dims[0] = in features, dims[num_layers] =
 * out features, dims[1..num_layers-1] = hidden widths. */
typedef struct mlpk_shape {
  int32_t num_layers;
  int32_t dims[MLPK_MAX_LAYERS + 1];
} mlpk_shape;

enum {
  MLPK_OK = 0,
  MLPK_ERR_SHAPE = 1,       /* dims/num_layers invalid or M < 0 */
  MLPK_ERR_UNSUPPORTED = 2, /* no kernel built for this shape */
  MLPK_ERR_ARCH = 3,        /* device is not sm_100 */
  MLPK_ERR_CUDA = 4,        /* a CUDA runtime/driver call failed */
  MLPK_ERR_ALIGN = 5,       /* a pointer is not 16-byte aligned */
  MLPK_ERR_NULL = 6,        /* a required pointer is NULL */
  MLPK_ERR_DEVICE = 7,      /* a kernel recorded a device-side error */
  MLPK_ERR_SCRATCH = 8      /* mlpk_bwd_noalloc: problem exceeds its static scratch */
};

/* Human-readable text for a status code. */
const char* mlpk_status_string(int status);

/* 1 if a kernel serves this shape, else 0.  Compiled networks: 2, 3 and 4
 * layers at 64, 128 and 256 wide; 5 layers at 32-64-64-64-64-16 and 64, 128
 * and 256 wide; 6 and 7 layers at 64, 128 and 256 wide; 8 layers at 128 and
 * 256 wide (the networks whose weights or weight gradients do not fit on the
 * SM -- 256 wide, and 128 wide from 4 layers on -- run the streamed-weight
 * kernels).  A network of the
 * same depth whose every width is a multiple of 8 and at most the compiled
 * width is served by the smallest such kernel (its missing rows / columns are
 * zero-filled on load and clipped on store; results are those of the
 * caller's network).  Hidden widths need not be equal.  The reference's
 * kernel takes the widths its tiles divide (kernel.py:25-53); all of them
 * up to 256 wide are served, at 3 and 5 layers and every depth from 2 to
 * MLPK_MAX_LAYERS. */
int mlpk_shape_supported(const mlpk_shape* shape);

/* Inference forward: out[M, dL] = MLP(x[M, d0]).
 * Replaces _fused_mlp_fwd (kernel.py:130-156) / ModelNew.forward
 * (kernel.py:174-180) and the 5-layer forward (README.md:9). */
int mlpk_fwd(const mlpk_shape* shape, int64_t M, const void* x, const void* const* W, void* out,
             mlpk_stream_t stream);

/* ---- fp32 inference on tf32 tensor cores.  The reference's design keeps
 * fp32 operands fp32 through the whole chain (INPUT_DTYPE fp32,
 * mlp_fused.md:159-166; its kernel.py selects fp32 tiles at kernel.py:37-43
 * but fails at the second GEMM on them).  mlpk_fwd_ex with MLPK_DT_F32: x, W
 * and out fp32; every GEMM is a tf32 tensor-core GEMM (the inputs' 10
 * mantissa bits, fp32's exponent range) with fp32 accumulation, the hidden
 * activations stay fp32.  Served for networks up to 128 wide
 * (mlpk_shape_supported_ex); MLPK_DT_F16 is mlpk_fwd. */
#define MLPK_DT_F16 0
#define MLPK_DT_F32 1
int mlpk_shape_supported_ex(const mlpk_shape* shape, int dtype);
int mlpk_fwd_ex(const mlpk_shape* shape, int64_t M, const void* x, const void* const* W, void* out, int dtype,
                mlpk_stream_t stream);

/* 1 if training (mlpk_train_fwd + mlpk_bwd) serves this shape (the same
 * rule as mlpk_shape_supported). */
int mlpk_train_supported(const mlpk_shape* shape);

/* Training forward: as mlpk_fwd, and also writes every hidden activation
 * h_l = softplus(z_l), l = 1..num_layers-1, to h_saved[l-1] ([M, dims[l]],
 * fp16 -- the exact operand the next GEMM consumed).
 * Replaces the training forward of the reference (mlp_fused.md:52-61;
 * fused_mlp.py is named at README.md:18 but absent from its tree). */
int mlpk_train_fwd(const mlpk_shape* shape, int64_t M, const void* x, const void* const* W,
                   void* out, void* const* h_saved, mlpk_stream_t stream);

/* ---- Saved-activation precision.  The reference's training forward stores
 * the hidden activations in fp32 "to avoid numerical loss in the backward
 * sigmoid derivative" (README.md:30; mlp_fused.md:52-61); the _ex entry points
 * below take that choice: MLPK_H_F32 saves h_l in fp32 (the backward computes
 * softplus' = 1 - e^{-h} from it and rounds h to fp16 only as its
 * weight-gradient operand, the value the forward's next GEMM consumed),
 * MLPK_H_F16 saves the fp16 operand copy (half the traffic; what
 * mlpk_train_fwd / mlpk_bwd do).  fp32 is served by every network of the fused
 * backward (mlpk_train_supported_ex); the streamed-weight networks (256 wide,
 * 128 wide at 4 and 5 layers) save fp16 only. */
#define MLPK_H_F16 0
#define MLPK_H_F32 1
int mlpk_train_supported_ex(const mlpk_shape* shape, int h_dtype);
/* mlpk_train_fwd with h_saved[l] of h_dtype ([M, dims[l+1]] fp16 or fp32). */
int mlpk_train_fwd_ex(const mlpk_shape* shape, int64_t M, const void* x, const void* const* W,
                      void* out, void* const* h_saved, int h_dtype, mlpk_stream_t stream);

/* Bytes of device workspace mlpk_bwd (and mlpk_bwd_ex, either precision)
 * needs for M rows on the current device (one fp32 weight-gradient partial
 * per persistent CTA); -1 if unsupported. */
int64_t mlpk_bwd_workspace_size(const mlpk_shape* shape, int64_t M);

/* Backward: from x, W, the saved h and grad_out ([M, dims[L]] fp16) writes
 * dx ([M, dims[0]] fp16) and dW (fp32, all layers concatenated, layer l is
 * [dims[l], dims[l+1]] row-major).  dW is a deterministic fixed-order sum over
 * the per-CTA partials kept in `workspace` (>= mlpk_bwd_workspace_size bytes).
 * Replaces the fused backward megakernel and its cuBLAS fallback
 * (mlp_fused.md:80-146). */
int mlpk_bwd(const mlpk_shape* shape, int64_t M, const void* x, const void* const* W,
             const void* const* h_saved, const void* grad_out, void* dx, void* workspace,
             int64_t workspace_bytes, float* dW, mlpk_stream_t stream);
/* mlpk_bwd reading h_saved of h_dtype (as written by mlpk_train_fwd_ex). */
int mlpk_bwd_ex(const mlpk_shape* shape, int64_t M, const void* x, const void* const* W,
                const void* const* h_saved, int h_dtype, const void* grad_out, void* dx, void* workspace,
                int64_t workspace_bytes, float* dW, mlpk_stream_t stream);

/* Weight norm forward, all layers in one launch: W_l = g_l * v_l / ||v_l||
 * per output column.  v_all: fp32 concat of v_l [dims[l], dims[l+1]]; g_all and
 * inv_norm: fp32 concat of per-column vectors; W[l]: fp16 outputs.
 * Replaces _wn_fwd_kernel (mlp_fused.md:466-480). */
int mlpk_wn_fwd(const mlpk_shape* shape, const float* v_all, const float* g_all, void* const* W,
                float* inv_norm, mlpk_stream_t stream);

/* Weight norm backward, all layers in one launch: (dv_all, dg_all) from the
 * fp32 dW_all of mlpk_bwd.  Replaces _wn_bwd_from_dw_T_kernel
 * (mlp_fused.md:481-483). */
int mlpk_wn_bwd(const mlpk_shape* shape, const float* dW_all, const float* v_all,
                const float* g_all, const float* inv_norm, float* dv_all, float* dg_all,
                mlpk_stream_t stream);

/* Allocation-free backward.  No counterpart in the reference: it exists for
 * callers that cannot allocate device memory at the time they call it (plain
 * C / FFI callers that hold only their input and output buffers and have no
 * device allocator of their own, serving processes that reserve all their
 * device memory at start-up and must not allocate afterwards).  Same
 * arguments and results as mlpk_bwd minus the workspace: the scratch mlpk_bwd
 * keeps in its workspace lives in a static device array of
 * MLPK_BWD_NOALLOC_SCRATCH_BYTES (32 MiB) that every GPU which loads the
 * library holds until the process exits.  Returns MLPK_ERR_SCRATCH, before
 * any launch, when the problem needs more than that (mlpk_bwd_workspace_size
 * > 32 MiB).  On a 148-SM B200 that serves: every network of the fused
 * backward (the 64- and 128-wide 2- and 3-layer networks, the 64-wide 4- and
 * 5-layer ones and the 5-layer 32-64-64-64-64-16) at any M (3L128 needs at
 * most 29 MB); the streamed 128-wide 4-layer network up to about 31,000 rows
 * and the 5-layer one up to about 23,000 rows (their data gradients are kept
 * in the scratch); no 256-wide network (their weight-gradient partials alone
 * take about 38 MB).  Calls no allocator.  The first call on a
 * device looks up the array's device address (cudaGetSymbolAddress) with that
 * device current; make that first call before any stream capture.  All calls
 * share the array, so calls that overlap on the GPU (other streams, other
 * host threads) race: serialise them. */
#define MLPK_BWD_NOALLOC_SCRATCH_BYTES (32u << 20)
int mlpk_bwd_noalloc(const mlpk_shape* shape, int64_t M, const void* x, const void* const* W,
                     const void* const* h_saved, const void* grad_out, void* dx, float* dW,
                     mlpk_stream_t stream);

/* ---- Inference on host-resident rows.  No counterpart in the reference (its
 * forward takes device tensors, kernel.py:130-156): for serving batches that
 * live in host memory.  out_host[M, dL] = MLP(x_host[M, d0]); x_host and
 * out_host are host buffers (page-locked for the copies to overlap), W the
 * device weights as for mlpk_fwd.  The rows stream through the GPU in chunks
 * of chunk_rows (0 = MLPK_FWD_HOST_CHUNK_ROWS): chunk k+1 is copied in and
 * chunk k-1 copied out (one cudaMemcpyAsync each, on two copy streams of the
 * library) while chunk k runs the fused forward on `stream`, through
 * MLPK_FWD_HOST_BUFFERS device buffers of each kind in `workspace`
 * (mlpk_fwd_host_workspace_size bytes).  Asynchronous: the results are in
 * out_host once `stream` has reached the point of the call (the copy streams
 * wait for `stream` at entry and `stream` waits for the last copy out).  The
 * copy streams and events are per host thread and device; concurrent calls
 * from one host thread on different streams are serialised by them. */
#define MLPK_FWD_HOST_CHUNK_ROWS 131072
#define MLPK_FWD_HOST_BUFFERS 3
int64_t mlpk_fwd_host_workspace_size(const mlpk_shape* shape, int64_t chunk_rows);
int mlpk_fwd_host(const mlpk_shape* shape, int64_t M, const void* x_host, const void* const* W,
                  void* out_host, int64_t chunk_rows, void* workspace, int64_t workspace_bytes,
                  mlpk_stream_t stream);

/* Reads (and optionally clears) the device-side status word of the current
 * device: bit flags set by bounded waits that expired (each wait gives up
 * after 1 s, records its flag and lets the kernel return).  Synchronises. */
#define MLPK_DEVST_TIMEOUT_FULL 1   /* a consumer waited too long for data */
#define MLPK_DEVST_TIMEOUT_EMPTY 2  /* a producer waited too long for a free buffer */
#define MLPK_DEVST_TIMEOUT_MMA 4    /* the tensor-core issuer waited too long */
#define MLPK_DEVST_TIMEOUT_EPI 8    /* an epilogue warp waited too long */
#define MLPK_DEVST_TIMEOUT_FLAG 16  /* a cross-CTA or cross-GPU flag wait expired */
int mlpk_device_status(int clear, int* status_out);

/* ---- fp32 <-> fp16 casts (round to nearest even), for the fp32-input
 * forward: the reference's kernel.py accepts fp32 x and W (kernel.py:37-43,
 * 134-138) and stores its fp16-rounded result into an fp32 output; the
 * library casts x and W to fp16, runs mlpk_fwd and widens the result.  n
 * elements; pointers 16-byte aligned. */
int mlpk_cast_f32_f16(const float* src, void* dst_f16, int64_t n, mlpk_stream_t stream);
int mlpk_cast_f16_f32(const void* src_f16, float* dst, int64_t n, mlpk_stream_t stream);

/* ---- Data-parallel weight-gradient sum over NVLink peer memory (one node).
 * Replaces the all_reduce(SUM) of the fp32 dW buffer in the reference's
 * data-parallel recipe (BASELINE: "training all-reduces the weight gradients
 * over NVLink"); the reference itself calls NCCL through torch.distributed.
 * Each rank allocates one peer buffer for n floats (n a multiple of 4), shares
 * its IPC handle (MLPK_PEER_HANDLE_BYTES bytes) with the other ranks and opens
 * theirs.  Per step: the backward writes this rank's dW into its own buffer
 * (the first n floats), then mlpk_peer_allreduce sums every rank's dW in rank
 * order into dW_out (bitwise identical on all ranks).  Every rank must call it
 * once per step, in the same order; the step count lives in device memory, so
 * the call can be captured in a CUDA graph.  When it returns (on the stream),
 * this rank's dW input (the first n floats) may be rewritten; the other ranks
 * may still be reading the rest of this rank's buffer until they return from
 * the same step, so free a buffer (mlpk_peer_free) only after every rank has
 * synchronized its device and met a host barrier.  If a peer does not
 * arrive within the bounded wait (1 s), the kernel sets MLPK_DEVST_TIMEOUT_FLAG
 * (16) in the device status word (mlpk_device_status).  At most 8 ranks;
 * mlpk_peer_alloc and mlpk_peer_open allocate / map device memory (set-up
 * calls, not per step). */
#define MLPK_PEER_HANDLE_BYTES 64
#define MLPK_PEER_MAX_RANKS 8
int mlpk_peer_alloc(int64_t n, void** buf_out, void* handle_out);
int mlpk_peer_open(const void* handle, void** buf_out);
int mlpk_peer_close(void* peer_buf);
int mlpk_peer_free(void* buf);
int mlpk_peer_allreduce(void* const* bufs, int world, int rank, int64_t n, float* dW_out,
                        mlpk_stream_t stream);

/* Text of the CUDA runtime / driver failure behind the calling thread's most
 * recent MLPK_ERR_CUDA ("no error" if none).  The reference reports failures as
 * Python exceptions carrying the CUDA message (cutile_mlp.py:388); this is the
 * message for the C caller.  The string stays valid until the thread's next
 * failing call. */
const char* mlpk_last_cuda_error(void);

#ifdef __cplusplus
}
#endif

#endif /* MLPK_H_ */
