"""GPU parity for networks served by a larger compiled network (zero padding
through TMA): the caller's widths need only be multiples of 8 and at most the
compiled widths of the same depth (64, 128 and 256 wide for 2, 3 and 4 layers;
32-64-64-64-64-16, 64, 128 and 256 wide for 5; 64 (6 and 7 layers), 128 and
256 wide for 6 to 8), hidden widths may differ from each other.

The reference's kernel accepts any widths its tl.dot tiles divide
(kernel.py:25-53, kernel.py:130-156) and its modules take D, H, out_features
(README.md:58-70); these tests hold such networks to the same oracle and
tolerances as the compiled widths: outputs max|d| <= 1e-2 * max|ref| (and the
3e-3 implementation bar for the forward), gradients relative L2 <= 1e-2.
"""
import numpy as np
import pytest
import torch

import oracle
from mlp_megakernel_b200 import FusedMLPSoftplus, FusedMLPSoftplusWN, _lib, fused_mlp_fwd
from mlp_megakernel_b200.modules import _backward, _train_forward
from mlp_megakernel_b200.synthetic import make_grad, make_weights, make_x

pytestmark = pytest.mark.gpu

TIGHT = 3e-3
GRAD_TOL = 1e-2

# (dims, served by)
SHAPES = [
    ((128, 96, 64, 32), "128^3"),
    ((32, 64, 64, 16), "64^3"),
    ((16, 16, 16, 16), "64^3"),
    ((48, 128, 80, 24), "128^3"),
    ((8, 120, 128, 8), "128^3"),
    ((200, 136, 256, 72), "256^3"),
    ((256, 160, 200, 256), "256^3"),
    ((16, 32, 48, 64, 40, 8), "5-layer"),
    ((32, 64, 64, 64, 64, 16), "5-layer (exact)"),
    ((64, 64, 64, 64, 64, 64), "5-layer 64-wide (exact)"),
    ((48, 64, 32, 64, 56, 24), "5-layer 64-wide"),
    ((128, 128, 128, 128, 128, 128), "5-layer 128-wide streamed (exact)"),
    ((96, 128, 64, 128, 112, 16), "5-layer 128-wide streamed"),
    ((256, 256, 256, 256, 256, 256), "5-layer 256-wide streamed (exact)"),
    ((200, 136, 256, 72, 128, 64), "5-layer 256-wide streamed"),
    ((64, 64, 64), "2-layer 64-wide (exact)"),
    ((32, 48, 16), "2-layer 64-wide"),
    ((128, 128, 128), "2-layer 128-wide (exact)"),
    ((128, 96, 16), "2-layer 128-wide"),
    ((256, 200, 64), "2-layer 256-wide streamed"),
    ((64, 64, 64, 64, 64), "4-layer 64-wide (exact)"),
    ((32, 64, 48, 64, 8), "4-layer 64-wide"),
    ((128, 96, 128, 112, 16), "4-layer 128-wide streamed"),
    ((200, 128, 64, 256, 8), "4-layer 256-wide streamed"),
    ((64,) * 7, "6-layer 64-wide (exact)"),
    ((32, 64, 16, 64, 48, 64, 8), "6-layer 64-wide"),
    ((64,) * 8, "7-layer 64-wide (exact)"),
    ((64,) * 9, "8-layer 64-wide, on the 128-wide kernels"),
    ((128,) * 7, "6-layer 128-wide streamed (exact)"),
    ((96, 128, 128, 64, 128, 128, 128, 128, 24), "8-layer 128-wide streamed"),
    ((256,) * 8, "7-layer 256-wide streamed (exact)"),
    ((200, 256, 8, 256, 64, 256, 256), "6-layer 256-wide streamed"),
]


def rel_l2(a, b):
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30)


def rel_max(a, b):
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return np.abs(a - b).max() / max(np.abs(b).max(), 1e-30)


@pytest.fixture(autouse=True)
def _status(built_lib):
    _lib.device_status(clear=True)
    yield
    assert _lib.device_status() == 0, "a kernel recorded a device-side timeout"


def _split(dw, dims):
    out, off = [], 0
    for a, b in zip(dims[:-1], dims[1:]):
        out.append(dw[off:off + a * b].reshape(a, b))
        off += a * b
    return out


@pytest.mark.parametrize("dims,served", SHAPES, ids=[str(s[0]) for s in SHAPES])
@pytest.mark.parametrize("M", [1, 300, 148 * 128 + 77])
def test_forward_covered_shapes(dims, served, M):
    assert _lib.shape_supported(dims) and _lib.train_supported(dims)
    x = make_x(M, dims[0], "normal", 7)
    ws = make_weights(dims, seed=11)
    out = fused_mlp_fwd(x.cuda(), *[w.cuda() for w in ws])
    assert out.shape == (M, dims[-1])
    ref = oracle.mlp_forward(x.numpy(), [w.numpy() for w in ws])
    assert rel_max(out.cpu().numpy(), ref) <= TIGHT, served


@pytest.mark.parametrize("dims,served", SHAPES, ids=[str(s[0]) for s in SHAPES])
@pytest.mark.parametrize("M", [1, 300, 148 * 128 + 77])
def test_training_covered_shapes(dims, served, M):
    """Training forward (saved activations at the caller's widths), fused or
    streamed backward, dx and the fixed-order dW reduction written in the
    caller's [d_l, d_{l+1}] layout."""
    x = make_x(M, dims[0], "normal", 7)
    ws = make_weights(dims, seed=11)
    g = make_grad(M, dims[-1], seed=13)
    xg, wg = x.cuda(), [w.cuda() for w in ws]
    out, hs = _train_forward(xg, wg, dims)
    assert [tuple(h.shape) for h in hs] == [(M, d) for d in dims[1:-1]]
    dx, dw = _backward(xg, wg, hs, g.cuda(), dims)
    torch.cuda.synchronize()
    wn = [w.numpy() for w in ws]
    ref_out, ref_hs = oracle.mlp_forward_train(x.numpy(), wn)
    assert rel_max(out.cpu().numpy(), ref_out) <= TIGHT, served
    for h, rh in zip(hs, ref_hs):
        assert rel_max(h.cpu().numpy(), rh) <= TIGHT
    ref_dx, ref_dws = oracle.mlp_backward(x.numpy(), wn, ref_hs, g.numpy())
    assert dx.shape == (M, dims[0]) and dw.numel() == sum(a * b for a, b in zip(dims[:-1], dims[1:]))
    assert rel_l2(dx.cpu().numpy(), ref_dx) <= GRAD_TOL, served
    for d, rd in zip(_split(dw.cpu().numpy(), dims), ref_dws):
        assert rel_l2(d, rd) <= GRAD_TOL, served
    _, dw2 = _backward(xg, wg, hs, g.cuda(), dims)
    assert torch.equal(dw, dw2), "weight gradients are not deterministic"


def test_padded_network_equals_compiled_network_exactly():
    """A 96-wide network run on the 128^3 kernel gives bitwise the same
    outputs as the 128^3 network with explicitly zero-padded weights (the
    padding is exact: zero operands contribute exact zeros)."""
    dims = (128, 96, 96, 128)
    M = 5000
    x = make_x(M, 128, "normal", 3).cuda()
    ws = [w.cuda() for w in make_weights(dims, seed=5)]
    out = fused_mlp_fwd(x, *ws)
    pad = [torch.zeros(128, 128, dtype=torch.float16, device="cuda") for _ in range(3)]
    pad[0][:, :96] = ws[0]
    pad[1][:96, :96] = ws[1]
    pad[2][:96, :] = ws[2]
    ref = fused_mlp_fwd(x, *pad)
    assert torch.equal(out, ref)


@pytest.mark.parametrize("cls", [FusedMLPSoftplus, FusedMLPSoftplusWN])
@pytest.mark.parametrize("kw", [dict(D=48, H=96, out_features=24),
                                dict(D=64, H=200, out_features=40),
                                dict(D=16, H=48, out_features=8, num_layers=5),
                                dict(D=64, H=160, out_features=32, num_layers=5),
                                dict(D=32, H=96, out_features=8, num_layers=2),
                                dict(D=48, H=64, out_features=16, num_layers=4)],
                         ids=["3L-96", "3L-200", "5L-48", "5L-160", "2L-96", "4L-64"])
def test_modules_with_other_widths(cls, kw):
    """The reference's modules take any D, H, out_features (README.md:58-70):
    gradients through autograd against torch's own autograd in fp32 on the same
    (fp16-rounded) weights."""
    torch.manual_seed(0)
    model = cls(**kw).cuda()
    M = 2000
    x = torch.randn(M, kw["D"], device="cuda").half()
    g = torch.randn(M, kw["out_features"], device="cuda").half()
    out = model(x)
    out.backward(g)
    params = [p for p in model.parameters()]
    ref_params = [p.detach().float().clone().requires_grad_(True) for p in params]
    if cls is FusedMLPSoftplus:
        ws = [p.half().float() for p in ref_params]
    else:
        ws = []
        for l in range(len(model.dims) - 1):
            off_v = sum(a * b for a, b in zip(model.dims[:l], model.dims[1:l + 1]))
            off_g = sum(model.dims[1:l + 1])
            a, b = model.dims[l], model.dims[l + 1]
            vv = ref_params[0][off_v:off_v + a * b].view(a, b)
            gg = ref_params[1][off_g:off_g + b]
            ws.append((gg * vv / vv.norm(dim=0, keepdim=True)).half().float())
    h = x.float()
    for i, w in enumerate(ws):
        h = h @ w
        if i + 1 < len(ws):
            h = torch.nn.functional.softplus(h).half().float()
    h.backward(g.float())
    assert rel_max(out.detach().float().cpu().numpy(), h.detach().cpu().numpy()) <= 1e-2
    for p, rp in zip(params, ref_params):
        assert rel_l2(p.grad.float().cpu().numpy(), rp.grad.cpu().numpy()) <= GRAD_TOL
