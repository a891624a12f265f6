"""Training gradients at the BASELINE row counts.

dW sums over every row, so a row subsample cannot stand in for it: here the
kernels' dx and dW at M = 1,048,576 for BASELINE config 4 (5 layers,
32-64-64-64-64-16, x ~ U(-1, 1)) and config 5 (D = H = OUT = 256) are
checked against the reference's formula (kernel.py:163-171: GEMMs with
F.softplus between them) differentiated by torch.autograd in fp32 on the
same GPU, with TF32 off (the checker; the product path is the library's
kernels alone).  Tolerance: gradients relative L2 <= 1e-2 (north star).
"""
import pytest
import torch

from mlp_megakernel_b200 import _lib
from mlp_megakernel_b200.modules import _backward, _train_forward
from mlp_megakernel_b200.synthetic import make_inputs

pytestmark = pytest.mark.gpu

GRAD_TOL = 1e-2
M_FULL = 1024 * 1024


def _rel_l2(a, b):
    a, b = a.double(), b.double()
    return float((a - b).norm() / b.norm().clamp_min(1e-30))


def _torch_fp32_grads(x, ws, g):
    """Reference formula in fp32 with torch.autograd (TF32 disabled)."""
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        xt = x.float().requires_grad_(True)
        wt = [w.float().requires_grad_(True) for w in ws]
        h = xt
        for i, w in enumerate(wt):
            h = h @ w
            if i < len(wt) - 1:
                h = torch.nn.functional.softplus(h)
        h.backward(g.float())
        return xt.grad, [w.grad for w in wt]
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev


@pytest.mark.parametrize("config", ["5L", "W256"])
def test_gradients_at_full_config_rows(config, built_lib):
    x, ws, g = make_inputs(config, M_FULL, device="cuda", with_grad=True)
    dims = tuple([x.shape[1]] + [w.shape[1] for w in ws])
    _lib.device_status(clear=True)
    _, hs = _train_forward(x, ws, dims)
    dx, dw = _backward(x, ws, hs, g, dims)
    torch.cuda.synchronize()
    assert _lib.device_status() == 0
    del hs
    ref_dx, ref_dws = _torch_fp32_grads(x, ws, g)
    assert _rel_l2(dx, ref_dx) <= GRAD_TOL
    off = 0
    for l, (a, b) in enumerate(zip(dims[:-1], dims[1:])):
        err = _rel_l2(dw[off:off + a * b].view(a, b), ref_dws[l])
        assert err <= GRAD_TOL, (l, err)
        off += a * b
