"""Functional API of the fused softplus MLP (forward).

Mirrors the reference's functional surface:

* ``_fused_mlp_fwd(x, w1, w2, w3)`` -- kernel.py:130-156 (same argument
  meaning: x ``[M, K1]``, ``w_i`` ``[in, out]``, returns a new ``[M, N3]``
  tensor in x's dtype; inputs are made contiguous first, as at kernel.py:132-133);
* ``fused_mlp_fwd(x, *weights)`` -- the same for any depth (the 5-layer chain of
  README.md:9);
* ``ModelNew`` -- the nn.Module shim of kernel.py:174-180.

Every call runs the sm_100a kernel in libmlpk through its C ABI on the current
CUDA stream.  x and the weights are fp16, or fp32.  fp32 operands run the
reference's fp32 design (INPUT_DTYPE fp32 throughout, mlp_fused.md:159-166):
every GEMM on tf32 tensor cores with fp32 accumulation, the hidden
activations fp32, an fp32 output -- for networks up to 128 wide; wider ones
are rounded to fp16 by the library's cast kernel around the fp16 kernel (the
inference kernel's rounding points, kernel.py:110, 117, 121-124).  The
reference's own kernel.py selects fp32 tile configurations (kernel.py:37-43,
138) but fails on fp32 operands at the second GEMM (it dots the fp16-cast h1
with the fp32 W2: "Both operands must be same dtype").
There is no CPU or PyTorch fallback: CPU tensors, other dtypes or unsupported
shapes raise.
"""
from __future__ import annotations

import ctypes

import torch
import torch.nn as nn

from . import _lib, ops  # noqa: F401  (ops registers torch.ops.mlpk.*)
from .ops import _aligned


def _check_operands(x: torch.Tensor, weights) -> list:
    if not isinstance(x, torch.Tensor) or x.dim() != 2:
        raise ValueError("x must be a 2-D tensor [M, in_features]")
    if not x.is_cuda:
        raise RuntimeError("fused MLP runs on CUDA (sm_100) only; got a CPU tensor")
    dt = x.dtype
    if dt is not torch.float16 and dt is not torch.float32:
        raise TypeError(f"fused MLP takes fp16 or fp32 inputs (fp16 operands, fp32 accumulate); "
                        f"got x.dtype={x.dtype}")
    if len(weights) < 1:
        raise ValueError("need at least one weight matrix")
    dev = x.device
    dims = [x.shape[1]]
    for i, w in enumerate(weights):
        if w.dim() != 2 or w.dtype is not dt or w.device != dev:
            raise ValueError(f"weight {i} must be a 2-D {x.dtype} tensor on {x.device}")
        if w.shape[0] != dims[-1]:
            raise ValueError(
                f"weight {i} has {w.shape[0]} input features, expected {dims[-1]} "
                f"(weights are [in, out], out = x @ W)"
            )
        dims.append(w.shape[1])
    return dims


def _current_stream(dev_index: int) -> int:
    """Raw handle of the current CUDA stream of a device."""
    try:
        return torch._C._cuda_getCurrentRawStream(dev_index)
    except AttributeError:  # older torch: through the Stream object
        return torch.cuda.current_stream(dev_index).cuda_stream


try:
    from torch._subclasses.fake_tensor import is_fake as _is_fake
except ImportError:  # no FakeTensor support: every tensor is real
    def _is_fake(t) -> bool:
        return False


def _eager_fwd(x: torch.Tensor, weights, out: torch.Tensor) -> None:
    """The fp16 forward straight through the C ABI (no operator dispatch):
    the per-call cost of an eager call is the host work here, so it is kept to
    one pointer array and one ctypes call."""
    dev = x.get_device()
    if dev != torch.cuda.current_device():
        with torch.cuda.device(dev):
            return _eager_fwd(x, weights, out)
    x = _aligned(x)
    ws = [_aligned(w) for w in weights]
    dims = [x.shape[1]] + [w.shape[1] for w in ws]
    lib = _lib.lib()
    ptrs = (ctypes.c_void_p * len(ws))(*[w.data_ptr() for w in ws])
    _lib.check("mlpk_fwd", lib.mlpk_fwd(ctypes.byref(_lib.shape_struct(dims)), x.shape[0], x.data_ptr(), ptrs,
                                        out.data_ptr(), _current_stream(dev)))


def fused_mlp_fwd(x: torch.Tensor, *weights: torch.Tensor, out: torch.Tensor = None) -> torch.Tensor:
    """``softplus(...softplus(x @ W_0)...) @ W_{L-1}`` in one kernel launch.

    Softplus is beta=1, threshold=20 (kernel.py:108); products accumulate in
    fp32 and every hidden activation is rounded to fp16 before the next GEMM
    (kernel.py:110, kernel.py:117).  Like the reference (kernel.py:136) the
    result is a new tensor unless ``out`` (contiguous, ``[M, out_features]``,
    x's dtype and device) is given, which lets a serving loop reuse one buffer.
    Under torch.compile it is the custom operator ``torch.ops.mlpk.fwd``
    (``fwd_out`` with ``out``), traced as one operator; eager fp16 calls go
    straight to the C ABI.
    """
    dims = _check_operands(x, weights)
    M = x.shape[0]
    if out is not None and (out.shape != (M, dims[-1]) or out.dtype != x.dtype or out.device != x.device
                            or not out.is_contiguous()):
        raise ValueError("out must be a contiguous, 16-byte aligned "
                         f"[{M}, {dims[-1]}] {x.dtype} tensor on {x.device}")
    if torch.compiler.is_compiling() or x.dtype != torch.float16 or _is_fake(x):
        if out is None:
            return torch.ops.mlpk.fwd(x, list(weights))
        torch.ops.mlpk.fwd_out(x, list(weights), out)
        return out
    if out is None:
        out = torch.empty((M, dims[-1]), device=x.device, dtype=x.dtype)
    elif out.data_ptr() % 16 != 0:
        raise ValueError("out must be 16-byte aligned")
    if M > 0:
        _eager_fwd(x, weights, out)
    return out


@torch.compiler.disable
def fused_mlp_fwd_host(x: torch.Tensor, *weights: torch.Tensor, out: torch.Tensor = None,
                       chunk_rows: int = _lib.FWD_HOST_CHUNK_ROWS) -> torch.Tensor:
    """The fused forward on rows that live in HOST memory (serving from host
    buffers; no counterpart in the reference, whose forward takes device
    tensors).

    ``x`` is a CPU fp16 tensor ``[M, in_features]`` (page-locked -- e.g.
    ``.pin_memory()`` -- for the copies to overlap), the weights are fp16 CUDA
    tensors; returns a CPU fp16 tensor ``[M, out_features]`` (``out``, if
    given: contiguous, CPU, fp16), complete when the call returns.  The rows
    stream through the GPU in chunks of ``chunk_rows``: the copy in of the next
    chunk and the copy out of the previous one overlap the forward of the
    current one (the host link runs both directions at once), on the current
    CUDA stream of the weights' device (mlpk_fwd_host).
    """
    if not isinstance(x, torch.Tensor) or x.dim() != 2 or x.is_cuda:
        raise ValueError("x must be a 2-D CPU tensor [M, in_features] (host rows)")
    if x.dtype != torch.float16:
        raise TypeError(f"fused_mlp_fwd_host takes fp16 rows; got {x.dtype}")
    if not weights or not all(w.is_cuda for w in weights):
        raise ValueError("the weights must be CUDA tensors")
    dev = weights[0].device
    dims = [x.shape[1]]
    for i, w in enumerate(weights):
        if w.dim() != 2 or w.dtype != torch.float16 or w.device != dev or w.shape[0] != dims[-1]:
            raise ValueError(f"weight {i} must be a 2-D fp16 [{dims[-1]}, out] tensor on {dev}")
        dims.append(w.shape[1])
    x = x.contiguous()
    ws = [_aligned(w) for w in weights]
    M = x.shape[0]
    if out is None:
        out = torch.empty((M, dims[-1]), dtype=torch.float16, pin_memory=x.is_pinned())
    elif (out.shape != (M, dims[-1]) or out.dtype != torch.float16 or out.is_cuda
          or not out.is_contiguous()):
        raise ValueError(f"out must be a contiguous CPU [{M}, {dims[-1]}] fp16 tensor")
    if M == 0:
        return out
    lib = _lib.lib()
    shape = _lib.shape_struct(dims)
    with torch.cuda.device(dev):
        wsb = lib.mlpk_fwd_host_workspace_size(ctypes.byref(shape), chunk_rows)
        if wsb < 0:
            raise ValueError(f"invalid chunk_rows {chunk_rows}")
        work = torch.empty(int(wsb), dtype=torch.uint8, device=dev)
        stream = torch.cuda.current_stream(dev)
        rc = lib.mlpk_fwd_host(ctypes.byref(shape), M, x.data_ptr(), _lib.ptr_array([w.data_ptr() for w in ws]),
                               out.data_ptr(), chunk_rows, work.data_ptr(), int(work.numel()),
                               stream.cuda_stream)
        _lib.check("mlpk_fwd_host", rc)
        stream.synchronize()  # the rows are in `out` once the stream got there
    return out


def _fused_mlp_fwd(x, w1, w2, w3):
    """3-layer inference forward -- drop-in for kernel.py:130-156."""
    return fused_mlp_fwd(x, w1, w2, w3)


class ModelNew(nn.Module):
    """Fused 3-layer softplus MLP, weights passed per call (kernel.py:174-180)."""

    def forward(self, x, w1, w2, w3):
        return _fused_mlp_fwd(x, w1, w2, w3)
