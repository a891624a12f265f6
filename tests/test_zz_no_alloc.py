"""The allocation-free backward (mlpk_bwd_noalloc) against the allocating one.

mlpk_bwd_noalloc serves callers that cannot allocate device memory when they
call the backward -- C / FFI callers that hold only their inputs and outputs
and no device allocator, serving processes whose device memory is fixed at
start-up.
It keeps its scratch (the per-CTA weight-gradient partials, and for the
streamed-weight networks the data gradients) in a static 32 MiB
device array inside the library instead of a caller workspace.  This test calls
it through the C ABI twice in a row -- a large batch, then a small one that
launches fewer CTAs, so the second call runs on an array still holding the
first call's partials -- and checks dx and dW against mlpk_bwd with the
tolerance of the other gradient tests (relative L2 <= 1e-2).  It also checks a
streamed 128-wide 4-layer network (whose data gradients share the array with
the partials) and that a problem larger than the array is refused with
MLPK_ERR_SCRATCH before anything is launched.  The file is named to be
collected last.
"""
import ctypes

import numpy as np
import pytest
import torch

from mlp_megakernel_b200 import _lib
from mlp_megakernel_b200.modules import _backward, _stream, _train_forward
from mlp_megakernel_b200.synthetic import make_inputs

pytestmark = pytest.mark.gpu

DIMS = (128, 128, 128, 128)
GRAD_TOL = 1e-2


def _rel_l2(a, b):
    a = a.double().cpu().numpy()
    b = b.double().cpu().numpy()
    return np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30)


def _bwd_noalloc(x, ws, hs, g, dims=DIMS):
    lib = _lib.lib()
    dx = torch.empty_like(x)
    dw = torch.empty(sum(a * b for a, b in zip(dims[:-1], dims[1:])), device=x.device,
                     dtype=torch.float32)
    rc = lib.mlpk_bwd_noalloc(ctypes.byref(_lib.shape_struct(dims)), x.shape[0], x.data_ptr(),
                              _lib.ptr_array([w.data_ptr() for w in ws]),
                              _lib.ptr_array([h.data_ptr() for h in hs]), g.data_ptr(),
                              dx.data_ptr(), dw.data_ptr(), _stream(x.device))
    _lib.check("mlpk_bwd_noalloc", rc)
    return dx, dw


def test_noalloc_backward_matches_allocating_backward(built_lib):
    _lib.device_status(clear=True)
    for M in (262144, 5000):  # two calls in a row; the second launches fewer CTAs
        x, ws, g = make_inputs("3L128", M, with_grad=True)
        x, ws, g = x.cuda(), [w.cuda() for w in ws], g.cuda()
        _, hs = _train_forward(x, ws, DIMS)
        dx_ref, dw_ref = _backward(x, ws, hs, g, DIMS)
        dx, dw = _bwd_noalloc(x, ws, hs, g)
        torch.cuda.synchronize()
        assert _rel_l2(dx, dx_ref) <= GRAD_TOL
        assert _rel_l2(dw, dw_ref) <= GRAD_TOL
        assert torch.isfinite(dw).all()
    assert _lib.device_status() == 0


def test_noalloc_streamed_network_and_scratch_limit(built_lib):
    """A streamed network (128 wide, 4 layers: its dz_1..dz_3 live in the
    array next to the weight-gradient partials) at a batch that fits, two calls
    in a row; then the 256-wide network, whose partials alone exceed the
    array: refused with MLPK_ERR_SCRATCH and nothing launched (null buffers)."""
    from mlp_megakernel_b200.synthetic import make_grad, make_weights, make_x

    dims = (128, 128, 128, 128, 128)
    _lib.device_status(clear=True)
    for M in (20000, 3000):
        x = make_x(M, dims[0], "normal", 21).cuda()
        ws = [w.cuda() for w in make_weights(dims, seed=22)]
        g = make_grad(M, dims[-1], seed=23).cuda()
        _, hs = _train_forward(x, ws, dims)
        dx_ref, dw_ref = _backward(x, ws, hs, g, dims)
        dx, dw = _bwd_noalloc(x, ws, hs, g, dims)
        torch.cuda.synchronize()
        assert _rel_l2(dx, dx_ref) <= GRAD_TOL
        assert _rel_l2(dw, dw_ref) <= GRAD_TOL
    assert _lib.device_status() == 0
    lib = _lib.lib()
    wide = (256, 256, 256, 256)
    null3 = _lib.ptr_array([0, 0, 0])
    rc = lib.mlpk_bwd_noalloc(ctypes.byref(_lib.shape_struct(wide)), 128, None, null3, null3, None, None,
                              None, _stream(torch.device("cuda", 0)))
    assert _lib.STATUS_NAMES[rc] == "MLPK_ERR_SCRATCH"
