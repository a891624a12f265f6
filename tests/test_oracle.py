"""CPU tests of the oracle: pinned to the reference's own kernel, and its
closed-form backward / weight norm checked against torch.autograd."""
import numpy as np
import pytest
import torch

import oracle
from tests.golden_io import case_names, load_case


@pytest.mark.parametrize("name", case_names())
def test_oracle_matches_reference_kernel(name):
    """The oracle (kernel.py:163-171 restated, fp16 recast of h as at
    kernel.py:110/117) reproduces the reference Triton kernel's outputs."""
    x, ws, rows, out_ref, rec = load_case(name)
    got = oracle.mlp_forward(x.numpy()[rows], [w.numpy() for w in ws])
    ref = out_ref.astype(np.float64)
    scale = max(np.abs(ref).max(), 1e-6)
    err = np.abs(got - ref).max() / scale
    # tighter than the parity tolerance (1e-2 * max|ref|): the two differ only
    # by accumulation order and fp16 rounding-boundary flips
    assert err <= 2e-3, f"{name}: oracle vs reference kernel rel-max err {err:.3e}"
    assert np.mean(np.abs(got - ref)) / scale <= 2e-4


def test_softplus_threshold_semantics():
    z = np.array([-100.0, -20.0, -1.0, 0.0, 1.0, 19.999, 20.0, 20.001, 50.0])
    ref = torch.nn.functional.softplus(torch.tensor(z, dtype=torch.float64)).numpy()
    np.testing.assert_allclose(oracle.softplus(z), ref, rtol=1e-12, atol=1e-300)


def _rand(shape, seed, scale=1.0):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(*shape, generator=g, dtype=torch.float64) * scale)


@pytest.mark.parametrize("dims", [(16, 32, 24, 8), (32, 64, 64, 64, 64, 16)])
def test_backward_closed_form_matches_autograd(dims):
    """mlp_fused.md:80-95 closed forms == autograd of the forward formula."""
    M = 37
    x = _rand((M, dims[0]), 0)
    ws = [_rand((i, o), 1 + k, 1.0 / np.sqrt(i)) for k, (i, o) in enumerate(zip(dims[:-1], dims[1:]))]
    g = _rand((M, dims[-1]), 99)
    xt = x.clone().requires_grad_(True)
    wts = [w.clone().requires_grad_(True) for w in ws]
    h = xt
    hs = []
    for i, w in enumerate(wts):
        z = h @ w
        if i < len(wts) - 1:
            h = torch.nn.functional.softplus(z)
            hs.append(h.detach().numpy())
        else:
            h = z
    (h * g).sum().backward()
    # oracle with rounding disabled: feed float64 values that are exactly
    # representable to avoid the fp16 operand rounding of the GPU model
    dx, dws = _backward_f64(x.numpy(), [w.numpy() for w in ws], hs, g.numpy())
    np.testing.assert_allclose(dx, xt.grad.numpy(), rtol=1e-10, atol=1e-12)
    for a, b in zip(dws, wts):
        np.testing.assert_allclose(a, b.grad.numpy(), rtol=1e-10, atol=1e-12)


def _backward_f64(x, ws, hs, g):
    # same algebra as oracle.mlp_backward, without the fp16 operand rounding
    L = len(ws)
    a_in = [x] + hs
    dz = g
    dws = [None] * L
    for l in range(L - 1, -1, -1):
        dws[l] = a_in[l].T @ dz
        dh = dz @ ws[l].T
        if l > 0:
            dz = dh * (1.0 - np.exp(-hs[l - 1]))
        else:
            dx = dh
    return dx, dws


def test_oracle_backward_rounding_model_close_to_exact():
    dims = (32, 64, 64, 16)
    M = 64
    x = _rand((M, dims[0]), 3).numpy().astype(np.float16).astype(np.float64)
    ws = [(_rand((i, o), 4 + k).numpy() / np.sqrt(i)).astype(np.float16).astype(np.float64)
          for k, (i, o) in enumerate(zip(dims[:-1], dims[1:]))]
    g = _rand((M, dims[-1]), 5).numpy().astype(np.float16).astype(np.float64)
    out, hs = oracle.mlp_forward_train(x, ws)
    dx, dws = oracle.mlp_backward(x, ws, hs, g)
    dx_e, dws_e = _backward_f64(x, ws, hs, g)
    rel = lambda a, b: np.linalg.norm(a - b) / np.linalg.norm(b)
    assert rel(dx, dx_e) < 2e-3
    for a, b in zip(dws, dws_e):
        assert rel(a, b) < 2e-3


def test_weight_norm_matches_autograd():
    v = _rand((24, 10), 7)
    gvec = _rand((10,), 8).abs() + 0.5
    dW = _rand((24, 10), 9)
    vt = v.clone().requires_grad_(True)
    gt = gvec.clone().requires_grad_(True)
    W = gt[None, :] * vt / vt.norm(dim=0, keepdim=True)
    (W * dW).sum().backward()
    Wo, inv = oracle.weight_norm_forward(v.numpy(), gvec.numpy())
    np.testing.assert_allclose(Wo, W.detach().numpy(), rtol=1e-12)
    np.testing.assert_allclose(inv, 1.0 / v.norm(dim=0).numpy(), rtol=1e-12)
    dv, dg = oracle.weight_norm_backward(v.numpy(), gvec.numpy(), dW.numpy())
    np.testing.assert_allclose(dv, vt.grad.numpy(), rtol=1e-10, atol=1e-12)
    np.testing.assert_allclose(dg, gt.grad.numpy(), rtol=1e-10, atol=1e-12)


def test_planted_error_is_caught():
    """A mistake planted in the oracle (on CPU) is detected by the golden check."""
    x, ws, rows, out_ref, _ = load_case("ragged_M300")
    bad = [w.numpy().copy() for w in ws]
    bad[1][3, 5] += 0.5
    got = oracle.mlp_forward(x.numpy()[rows], bad)
    ref = out_ref.astype(np.float64)
    assert np.abs(got - ref).max() / np.abs(ref).max() > 2e-3
