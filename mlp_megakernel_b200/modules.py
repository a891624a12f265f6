"""Module API: FusedMLPSoftplus and FusedMLPSoftplusWN (training + inference).

Mirrors the reference's module surface (README.md:58-70): constructed as
``FusedMLPSoftplus(D=128, H=128, out_features=128)``, moved with
``.cuda().half()``, called as ``model(x)`` followed by ``loss.backward()``.
The reference's classes live in fused_mlp.py / fused_mlp5.py, which its
published tree does not contain (README.md:18-19); their behaviour is known
from mlp_fused.md:52-172 and mlp_fused.md:461-486, and is restated here:

* one autograd.Function per model, with ``torch.amp.custom_fwd(device_type=
  "cuda", cast_inputs=torch.float16)`` / ``custom_bwd`` (mlp_fused.md:168-172);
* forward = one fused kernel launch that also saves the hidden activations;
  backward = one fused kernel (data gradients + weight gradients) plus a
  fixed-order reduction, called through the C ABI -- no per-op Python dispatch
  (the cost the reference reports at mlp_fused.md:272-280);
* the weight-norm model keeps all directions and gains in two contiguous
  parameters ``v_all`` / ``g_all`` (mlp_fused.md:478-480) and normalises every
  layer in one launch per direction.

``num_layers`` selects the depth (3 or 5 in the reference; README.md:9); all
hidden layers have width H.  ``activation_dtype`` is the precision of the
hidden activations saved for the backward: ``torch.float32`` as the
reference stores them (README.md:30; the backward computes softplus' from the
fp32 value and rounds it to fp16 only as its weight-gradient operand) or
``torch.float16`` (the fp16 operand copy: half the traffic).  The default,
None, is fp32 where the network's kernels offer it (every network of the
fused backward) and fp16 on the streamed-weight networks (256 wide; 128 wide
at 4 and 5 layers), which save fp16 only.  Data-parallel training: pass a
``torch.distributed`` process group and the fp32 weight gradients are summed
over the ranks on the current stream between the backward kernel and the
weight-norm backward (so every rank applies the same update): on one node by
this library's NVLink peer-memory kernel, otherwise by NCCL (``grad_reduce``
= "auto", "peer" or "nccl"; see dp.make_grad_reducer).
"""
from __future__ import annotations

import math

import torch
import torch.nn as nn

from . import _lib, ops
from .dp import make_grad_reducer


def _dims(D: int, H: int, out_features: int, num_layers: int):
    if num_layers < 2:
        raise ValueError("num_layers must be >= 2")
    return tuple([D] + [H] * (num_layers - 1) + [out_features])


def _stream(dev):
    return torch.cuda.current_stream(dev).cuda_stream


_H_CODE = {torch.float16: _lib.H_F16, torch.float32: _lib.H_F32}


def _resolve_activation_dtype(dims, activation_dtype):
    """The saved-activation dtype of a network: the requested one (raising if
    its kernels do not offer it), or fp32 where offered and else fp16."""
    if activation_dtype is None:
        return torch.float32 if _lib.train_supported(dims, _lib.H_F32) else torch.float16
    if activation_dtype not in _H_CODE:
        raise TypeError(f"activation_dtype must be torch.float32 or torch.float16, got {activation_dtype}")
    if not _lib.train_supported(dims, _H_CODE[activation_dtype]):
        raise ValueError(f"no training kernels for dims {tuple(dims)} with {activation_dtype} saved activations")
    return activation_dtype


def _train_forward(x: torch.Tensor, ws, dims, h_dtype=torch.float16):
    """The training forward (torch.ops.mlpk.train_fwd): returns
    (out, [h_1..h_{L-1}]), the saved activations in ``h_dtype``."""
    res = torch.ops.mlpk.train_fwd(x, list(ws), h_dtype == torch.float32)
    return res[0], list(res[1:])


class _GradSum:
    """Data-parallel weight-gradient sum of one module: the reducer is made on
    the first backward (a collective set-up on every rank of the group)."""

    def __init__(self, process_group, kind: str = "auto"):
        self.process_group = process_group
        self.kind = kind
        self._reducer = None

    def reducer(self, n: int):
        if self._reducer is None or self._reducer.n != n:
            if self._reducer is not None:
                self._reducer.close()
            self._reducer = make_grad_reducer(n, self.process_group, self.kind)
        return self._reducer


def _backward(x, ws, hs, grad_out, dims, grad_sum: _GradSum = None):
    """The fused backward: returns (dx fp16, dW_flat fp32).  Without a
    gradient sum it is the operator torch.ops.mlpk.bwd; with one, the backward
    writes this rank's dW where the reducer wants it and the reducer sums it
    over the ranks."""
    g = grad_out.to(torch.float16)
    if grad_sum is None:
        dx, dw = torch.ops.mlpk.bwd(x, list(ws), list(hs), g)
        return dx, dw
    dx = torch.empty(x.shape, device=x.device, dtype=torch.float16)
    nflat = sum(a * b for a, b in zip(dims[:-1], dims[1:]))
    dw = torch.empty(nflat, device=x.device, dtype=torch.float32)
    red = grad_sum.reducer(nflat)
    local = red.local_buffer(dw)
    ops.backward_into(x, ws, hs, g, dx, local)
    red.reduce(local, dw)
    return dx, dw


def _split_flat(flat: torch.Tensor, dims):
    out, off = [], 0
    for a, b in zip(dims[:-1], dims[1:]):
        out.append(flat[off:off + a * b].view(a, b))
        off += a * b
    return out


def _check_input(x: torch.Tensor, d0: int) -> torch.Tensor:
    if not x.is_cuda:
        raise RuntimeError("fused MLP runs on CUDA (sm_100) only; got a CPU tensor")
    if x.dim() != 2 or x.shape[1] != d0:
        raise ValueError(f"x must be [M, {d0}]")
    return x.to(torch.float16).contiguous()


class _FusedMLPFn(torch.autograd.Function):
    @staticmethod
    @torch.amp.custom_fwd(device_type="cuda", cast_inputs=torch.float16)
    def forward(ctx, x, dims, grad_sum, h_dtype, *weights):
        x = _check_input(x, dims[0])
        ws = [w.to(torch.float16).contiguous() for w in weights]
        out, hs = _train_forward(x, ws, dims, h_dtype)
        ctx.dims = dims
        ctx.grad_sum = grad_sum
        ctx.w_dtypes = [w.dtype for w in weights]
        ctx.save_for_backward(x, *ws, *hs)
        return out

    @staticmethod
    @torch.amp.custom_bwd(device_type="cuda")
    def backward(ctx, grad_out):
        dims = ctx.dims
        L = len(dims) - 1
        saved = ctx.saved_tensors
        x, ws, hs = saved[0], list(saved[1:1 + L]), list(saved[1 + L:])
        dx, dw = _backward(x, ws, hs, grad_out, dims, ctx.grad_sum)
        dws = [d.to(t) for d, t in zip(_split_flat(dw, dims), ctx.w_dtypes)]
        return (dx if ctx.needs_input_grad[0] else None, None, None, None, *dws)


class _FusedMLPWNFn(torch.autograd.Function):
    @staticmethod
    @torch.amp.custom_fwd(device_type="cuda", cast_inputs=torch.float16)
    def forward(ctx, x, dims, grad_sum, h_dtype, v_all, g_all):
        x = _check_input(x, dims[0])
        v32 = v_all.detach().to(torch.float32).contiguous()
        g32 = g_all.detach().to(torch.float32).contiguous()
        res = torch.ops.mlpk.wn_fwd(v32, g32, list(dims))
        ws, inv = list(res[:-1]), res[-1]
        out, hs = _train_forward(x, ws, dims, h_dtype)
        ctx.dims = dims
        ctx.grad_sum = grad_sum
        ctx.dtypes = (v_all.dtype, g_all.dtype)
        ctx.save_for_backward(x, v32, g32, inv, *ws, *hs)
        return out

    @staticmethod
    @torch.amp.custom_bwd(device_type="cuda")
    def backward(ctx, grad_out):
        dims = ctx.dims
        L = len(dims) - 1
        saved = ctx.saved_tensors
        x, v32, g32, inv = saved[:4]
        ws, hs = list(saved[4:4 + L]), list(saved[4 + L:])
        dx, dw = _backward(x, ws, hs, grad_out, dims, ctx.grad_sum)
        dv, dg = torch.ops.mlpk.wn_bwd(dw, v32, g32, inv, list(dims))
        return (dx if ctx.needs_input_grad[0] else None, None, None, None,
                dv.to(ctx.dtypes[0]), dg.to(ctx.dtypes[1]))


# The autograd Functions call the library through torch.ops.mlpk.* custom
# operators, so torch.compile traces them (fullgraph).  With a data-parallel
# gradient sum the backward also runs the reducer, a Python object over
# peer-memory buffers or NCCL: that case stays opaque to torch.compile and
# runs eagerly at a graph break.
@torch.compiler.disable
def _apply_fused_dp(x, dims, grad_sum, h_dtype, *weights):
    return _FusedMLPFn.apply(x, dims, grad_sum, h_dtype, *weights)


@torch.compiler.disable
def _apply_fused_wn_dp(x, dims, grad_sum, h_dtype, v_all, g_all):
    return _FusedMLPWNFn.apply(x, dims, grad_sum, h_dtype, v_all, g_all)


def _apply_fused(x, dims, grad_sum, h_dtype, *weights):
    if grad_sum is not None:
        return _apply_fused_dp(x, dims, grad_sum, h_dtype, *weights)
    return _FusedMLPFn.apply(x, dims, None, h_dtype, *weights)


def _apply_fused_wn(x, dims, grad_sum, h_dtype, v_all, g_all):
    if grad_sum is not None:
        return _apply_fused_wn_dp(x, dims, grad_sum, h_dtype, v_all, g_all)
    return _FusedMLPWNFn.apply(x, dims, None, h_dtype, v_all, g_all)


class FusedMLPSoftplus(nn.Module):
    """``softplus(...softplus(x @ W_1)...) @ W_L`` with fused training kernels.

    Weights are ``[in, out]`` parameters ``w1 .. wL`` initialised
    U(-1/sqrt(in), 1/sqrt(in)).
    """

    def __init__(self, D: int = 128, H: int = 128, out_features: int = 128, num_layers: int = 3,
                 process_group=None, grad_reduce: str = "auto", activation_dtype=None):
        super().__init__()
        self.dims = _dims(D, H, out_features, num_layers)
        self.activation_dtype = _resolve_activation_dtype(self.dims, activation_dtype)
        self.process_group = process_group
        self._grad_sum = _GradSum(process_group, grad_reduce) if process_group is not None else None
        for i, (a, b) in enumerate(zip(self.dims[:-1], self.dims[1:])):
            w = torch.empty(a, b)
            nn.init.uniform_(w, -1.0 / math.sqrt(a), 1.0 / math.sqrt(a))
            self.register_parameter(f"w{i + 1}", nn.Parameter(w))

    @property
    def weights(self):
        return [getattr(self, f"w{i + 1}") for i in range(len(self.dims) - 1)]

    def forward(self, x):
        return _apply_fused(x, self.dims, self._grad_sum, self.activation_dtype, *self.weights)


class FusedMLPSoftplusWN(nn.Module):
    """Weight-normalised fused MLP: ``W_l = g_l * v_l / ||v_l||`` per output column.

    ``v_all`` holds every v_l ([in, out], row-major) back to back, ``g_all``
    every g_l; at construction v_l ~ U(+-1/sqrt(in)) and g_l = ||v_l||, so the
    effective weights start equal to v.  ``weight(l)`` returns the effective
    W_l.
    """

    def __init__(self, D: int = 128, H: int = 128, out_features: int = 128, num_layers: int = 3,
                 process_group=None, grad_reduce: str = "auto", activation_dtype=None):
        super().__init__()
        self.dims = _dims(D, H, out_features, num_layers)
        self.activation_dtype = _resolve_activation_dtype(self.dims, activation_dtype)
        self.process_group = process_group
        self._grad_sum = _GradSum(process_group, grad_reduce) if process_group is not None else None
        vs, gs = [], []
        for a, b in zip(self.dims[:-1], self.dims[1:]):
            v = torch.empty(a, b)
            nn.init.uniform_(v, -1.0 / math.sqrt(a), 1.0 / math.sqrt(a))
            vs.append(v.reshape(-1))
            gs.append(v.norm(dim=0))
        self.v_all = nn.Parameter(torch.cat(vs))
        self.g_all = nn.Parameter(torch.cat(gs))

    def v(self, l: int) -> torch.Tensor:
        off = sum(a * b for a, b in zip(self.dims[:l], self.dims[1:l + 1]))
        a, b = self.dims[l], self.dims[l + 1]
        return self.v_all[off:off + a * b].view(a, b)

    def g(self, l: int) -> torch.Tensor:
        off = sum(self.dims[1:l + 1])
        return self.g_all[off:off + self.dims[l + 1]]

    def weight(self, l: int) -> torch.Tensor:
        v = self.v(l).float()
        return self.g(l).float() * v / v.norm(dim=0, keepdim=True)

    @torch.no_grad()
    def load_weights(self, weights):
        """Set v = W and g = ||W|| (per column) from plain [in, out] weights."""
        for l, w in enumerate(weights):
            self.v(l).copy_(w)
            self.g(l).copy_(w.float().norm(dim=0))

    def forward(self, x):
        return _apply_fused_wn(x, self.dims, self._grad_sum, self.activation_dtype, self.v_all, self.g_all)
