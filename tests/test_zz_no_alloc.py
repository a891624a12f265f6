"""The allocation-free backward (mlpk_bwd_noalloc) against the allocating one.

mlpk_bwd_noalloc serves callers that cannot allocate device memory when they
call the backward -- C / FFI callers that hold only their inputs and outputs
and no device allocator, serving processes whose device memory is fixed at
start-up.
It keeps its scratch (the per-CTA weight-gradient partials) in a static 32 MiB
device array inside the library instead of a caller workspace.  This test calls
it through the C ABI twice in a row -- a large batch, then a small one that
launches fewer CTAs, so the second call runs on an array still holding the
first call's partials -- and checks dx and dW against mlpk_bwd with the
tolerance of the other gradient tests (relative L2 <= 1e-2).  The file is named
to be collected last.
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


def _bwd_noalloc(x, ws, hs, g):
    lib = _lib.lib()
    dx = torch.empty_like(x)
    dw = torch.empty(sum(a * b for a, b in zip(DIMS[:-1], DIMS[1:])), device=x.device,
                     dtype=torch.float32)
    rc = lib.mlpk_bwd_noalloc(ctypes.byref(_lib.shape_struct(DIMS)), x.shape[0], x.data_ptr(),
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
