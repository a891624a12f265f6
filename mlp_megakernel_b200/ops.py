"""The C-ABI entry points as torch custom operators (``torch.ops.mlpk.*``).

Each operator's real implementation calls libmlpk through ctypes on the
current CUDA stream (no CPU path: CPU tensors raise); its fake implementation
gives only the output shapes and dtypes, so ``torch.compile`` (fullgraph),
FakeTensor / meta tracing and CUDA-graph capture see an ordinary operator
instead of an opaque Python call.  Operators:

* ``mlpk::fwd(x, weights) -> out`` -- the inference forward (kernel.py:130-156),
  fp16 operands, or fp32 ones on tf32 tensor cores with fp32 activations
  (networks up to 128 wide; wider ones are cast to fp16 around the fp16
  kernel);
* ``mlpk::fwd_out(x, weights, out) -> ()`` -- the same into a caller buffer;
* ``mlpk::train_fwd(x, weights, h_fp32) -> [out, h_1, .., h_{L-1}]`` --
  the training forward, saved activations in fp32 or fp16;
* ``mlpk::bwd(x, weights, hs, grad_out) -> [dx, dW_flat]`` -- the fused
  backward with its deterministic split-K weight gradients;
* ``mlpk::wn_fwd(v_all, g_all, dims) -> [W_0, .., W_{L-1}, inv_norm]`` and
  ``mlpk::wn_bwd(dW_flat, v_all, g_all, inv_norm, dims) -> [dv_all, dg_all]``
  -- the single-launch weight norm (mlp_fused.md:466-483).

Buffers are allocated by torch's caching allocator (the reference's
ownership convention: the callee allocates its outputs, kernel.py:136);
misaligned inputs are copied to 16-byte-aligned storage first.
"""
from __future__ import annotations

import ctypes

import torch
from torch import Tensor

from . import _lib


def _stream(dev) -> int:
    return torch.cuda.current_stream(dev).cuda_stream


def _aligned(t: Tensor) -> Tensor:
    t = t.contiguous()
    if t.data_ptr() % 16 != 0:
        t = t.clone()
    return t


def _dims_of(x: Tensor, weights) -> list:
    return [x.shape[1]] + [w.shape[1] for w in weights]


def _ptrs(ts) -> ctypes.Array:
    return _lib.ptr_array([t.data_ptr() for t in ts])


def _require_cuda(*ts):
    for t in ts:
        if not t.is_cuda:
            raise RuntimeError("fused MLP runs on CUDA (sm_100) only; got a CPU tensor")


def _cast(lib, t: Tensor, dtype, stream) -> Tensor:
    """fp32 -> fp16 copy of a contiguous tensor with the library's cast kernel."""
    dst = torch.empty(t.shape, device=t.device, dtype=dtype)
    _lib.check("mlpk_cast_f32_f16", lib.mlpk_cast_f32_f16(t.data_ptr(), dst.data_ptr(), t.numel(), stream))
    return dst


def _forward_into(x: Tensor, weights, out: Tensor) -> None:
    _require_cuda(x, out, *weights)
    M = x.shape[0]
    if M == 0:
        return
    dims = _dims_of(x, weights)
    lib = _lib.lib()
    shape = _lib.shape_struct(dims)
    with torch.cuda.device(x.device):
        stream = _stream(x.device)
        x = _aligned(x)
        ws = [_aligned(w) for w in weights]
        if x.dtype == torch.float32 and lib.mlpk_shape_supported_ex(ctypes.byref(shape), _lib.DT_F32):
            # fp32 operands on tf32 tensor cores, fp32 hidden activations
            # (the reference's INPUT_DTYPE fp32 design, mlp_fused.md:159-166)
            _lib.check("mlpk_fwd_ex", lib.mlpk_fwd_ex(ctypes.byref(shape), M, x.data_ptr(), _ptrs(ws),
                                                      out.data_ptr(), _lib.DT_F32, stream))
            return
        if x.dtype == torch.float32:
            # networks wider than the tf32 kernels (256 wide): operands rounded
            # to fp16 by the library's cast kernel, the fp16 result widened
            if not lib.mlpk_shape_supported(ctypes.byref(shape)):
                _lib.check("mlpk_fwd", 2)
            x16 = _cast(lib, x, torch.float16, stream)
            w16 = [_cast(lib, w, torch.float16, stream) for w in ws]
            out16 = torch.empty((M, dims[-1]), device=x.device, dtype=torch.float16)
            _lib.check("mlpk_fwd", lib.mlpk_fwd(ctypes.byref(shape), M, x16.data_ptr(), _ptrs(w16),
                                                out16.data_ptr(), stream))
            _lib.check("mlpk_cast_f16_f32", lib.mlpk_cast_f16_f32(out16.data_ptr(), out.data_ptr(),
                                                                  out.numel(), stream))
            return
        _lib.check("mlpk_fwd", lib.mlpk_fwd(ctypes.byref(shape), M, x.data_ptr(), _ptrs(ws), out.data_ptr(),
                                            stream))


@torch.library.custom_op("mlpk::fwd", mutates_args=())
def fwd(x: Tensor, weights: list[Tensor]) -> Tensor:
    out = torch.empty((x.shape[0], weights[-1].shape[1]), device=x.device, dtype=x.dtype)
    _forward_into(x, weights, out)
    return out


@fwd.register_fake
def _fwd_fake(x, weights):
    return x.new_empty((x.shape[0], weights[-1].shape[1]))


@torch.library.custom_op("mlpk::fwd_out", mutates_args=("out",))
def fwd_out(x: Tensor, weights: list[Tensor], out: Tensor) -> None:
    if out.data_ptr() % 16 != 0:
        raise ValueError("out must be 16-byte aligned")
    _forward_into(x, weights, out)


@fwd_out.register_fake
def _fwd_out_fake(x, weights, out):
    return None


@torch.library.custom_op("mlpk::train_fwd", mutates_args=())
def train_fwd(x: Tensor, weights: list[Tensor], h_fp32: bool) -> list[Tensor]:
    _require_cuda(x, *weights)
    dims = _dims_of(x, weights)
    M = x.shape[0]
    h_dtype = torch.float32 if h_fp32 else torch.float16
    out = torch.empty((M, dims[-1]), device=x.device, dtype=torch.float16)
    hs = [torch.empty((M, d), device=x.device, dtype=h_dtype) for d in dims[1:-1]]
    if M > 0:
        lib = _lib.lib()
        with torch.cuda.device(x.device):
            x = _aligned(x)
            ws = [_aligned(w) for w in weights]
            rc = lib.mlpk_train_fwd_ex(ctypes.byref(_lib.shape_struct(dims)), M, x.data_ptr(), _ptrs(ws),
                                       out.data_ptr(), _ptrs(hs), _lib.H_F32 if h_fp32 else _lib.H_F16,
                                       _stream(x.device))
        _lib.check("mlpk_train_fwd_ex", rc)
    return [out] + hs


@train_fwd.register_fake
def _train_fwd_fake(x, weights, h_fp32):
    dims = _dims_of(x, weights)
    M = x.shape[0]
    h_dtype = torch.float32 if h_fp32 else torch.float16
    return [x.new_empty((M, dims[-1]), dtype=torch.float16)] + \
        [x.new_empty((M, d), dtype=h_dtype) for d in dims[1:-1]]


def backward_into(x: Tensor, weights, hs, grad_out: Tensor, dx: Tensor, dw: Tensor) -> None:
    """mlpk_bwd_ex writing dx and the flat fp32 dW into the given buffers (the
    saved activations' dtype is read from ``hs``)."""
    _require_cuda(x, grad_out, *weights, *hs)
    dims = _dims_of(x, weights)
    M = x.shape[0]
    lib = _lib.lib()
    shape = _lib.shape_struct(dims)
    with torch.cuda.device(x.device):
        wsb = lib.mlpk_bwd_workspace_size(ctypes.byref(shape), M)
        if wsb < 0:
            raise _lib.MlpkError("mlpk_bwd_workspace_size", 2)
        work = torch.empty(max(int(wsb), 16), device=x.device, dtype=torch.uint8)
        x = _aligned(x)
        ws = [_aligned(w) for w in weights]
        hs = [_aligned(h) for h in hs]
        g = _aligned(grad_out)
        h_code = _lib.H_F32 if (hs and hs[0].dtype == torch.float32) else _lib.H_F16
        rc = lib.mlpk_bwd_ex(ctypes.byref(shape), M, x.data_ptr(), _ptrs(ws), _ptrs(hs), h_code, g.data_ptr(),
                             dx.data_ptr(), work.data_ptr(), int(work.numel()), dw.data_ptr(), _stream(x.device))
    _lib.check("mlpk_bwd_ex", rc)


@torch.library.custom_op("mlpk::bwd", mutates_args=())
def bwd(x: Tensor, weights: list[Tensor], hs: list[Tensor], grad_out: Tensor) -> list[Tensor]:
    dims = _dims_of(x, weights)
    dx = torch.empty(x.shape, device=x.device, dtype=torch.float16)
    dw = torch.empty(sum(a * b for a, b in zip(dims[:-1], dims[1:])), device=x.device, dtype=torch.float32)
    backward_into(x, weights, hs, grad_out, dx, dw)
    return [dx, dw]


@bwd.register_fake
def _bwd_fake(x, weights, hs, grad_out):
    dims = _dims_of(x, weights)
    return [x.new_empty(x.shape, dtype=torch.float16),
            x.new_empty((sum(a * b for a, b in zip(dims[:-1], dims[1:])),), dtype=torch.float32)]


@torch.library.custom_op("mlpk::wn_fwd", mutates_args=())
def wn_fwd(v_all: Tensor, g_all: Tensor, dims: list[int]) -> list[Tensor]:
    _require_cuda(v_all, g_all)
    ws = [torch.empty((a, b), device=v_all.device, dtype=torch.float16) for a, b in zip(dims[:-1], dims[1:])]
    inv = torch.empty(g_all.shape, device=g_all.device, dtype=torch.float32)
    lib = _lib.lib()
    with torch.cuda.device(v_all.device):
        v = _aligned(v_all)
        g = _aligned(g_all)
        rc = lib.mlpk_wn_fwd(ctypes.byref(_lib.shape_struct(dims)), v.data_ptr(), g.data_ptr(), _ptrs(ws),
                             inv.data_ptr(), _stream(v_all.device))
    _lib.check("mlpk_wn_fwd", rc)
    return ws + [inv]


@wn_fwd.register_fake
def _wn_fwd_fake(v_all, g_all, dims):
    return [v_all.new_empty((a, b), dtype=torch.float16) for a, b in zip(dims[:-1], dims[1:])] + \
        [g_all.new_empty(g_all.shape, dtype=torch.float32)]


@torch.library.custom_op("mlpk::wn_bwd", mutates_args=())
def wn_bwd(dw: Tensor, v_all: Tensor, g_all: Tensor, inv: Tensor, dims: list[int]) -> list[Tensor]:
    _require_cuda(dw, v_all, g_all, inv)
    dv = torch.empty(v_all.shape, device=v_all.device, dtype=torch.float32)
    dg = torch.empty(g_all.shape, device=g_all.device, dtype=torch.float32)
    lib = _lib.lib()
    with torch.cuda.device(v_all.device):
        d, v, g, i = (_aligned(t) for t in (dw, v_all, g_all, inv))
        rc = lib.mlpk_wn_bwd(ctypes.byref(_lib.shape_struct(dims)), d.data_ptr(), v.data_ptr(), g.data_ptr(),
                             i.data_ptr(), dv.data_ptr(), dg.data_ptr(), _stream(v_all.device))
    _lib.check("mlpk_wn_bwd", rc)
    return [dv, dg]


@wn_bwd.register_fake
def _wn_bwd_fake(dw, v_all, g_all, inv, dims):
    return [v_all.new_empty(v_all.shape, dtype=torch.float32), g_all.new_empty(g_all.shape, dtype=torch.float32)]
