"""Training parity pinned to the REFERENCE's own PyTorch model.

The fixtures ``tests/golden/train_*.npz`` hold the outputs and gradients of
the reference's ``Model`` (kernel.py:163-171, imported from the reference by
tests/golden/make_golden.py) on weight-normed weights W_l = g_l v_l / ||v_l||,
run in fp32 and differentiated by torch.autograd (BASELINE config 3 at
M = 16,384 and 262,144).  These tests check

* on the CPU: the oracle's closed-form backward (oracle/mlp_oracle.py, float64
  with the kernels' fp16 GEMM operands) against the fixtures, so the oracle
  itself is pinned to the reference for training;
* on the GPU: the training kernels through the module API (weight-norm
  forward, training forward, fused backward, weight-norm backward) against
  the fixtures, for both saved-activation precisions.

Tolerance (north star): outputs max|d| <= 1e-2 * max|ref|; gradients
relative L2 <= 1e-2.
"""
import hashlib

import numpy as np
import pytest
import torch

import oracle
from tests.golden.cases import TRAIN_CASES, make_train_inputs
from tests.golden_io import GOLDEN_DIR

GRAD_TOL = 1e-2
OUT_TOL = 1e-2


def _digest(*ts) -> str:
    return hashlib.sha256(b"".join(t.contiguous().numpy().tobytes() for t in ts)).hexdigest()


def load_train_case(name):
    rec = dict(np.load(f"{GOLDEN_DIR}/train_{name}.npz"))
    dims, M, _ = TRAIN_CASES[name]
    x, g, vs, gs = make_train_inputs(dims, M)
    if (_digest(x) != str(rec["x_sha256"]) or _digest(g) != str(rec["grad_sha256"])
            or _digest(*vs) != str(rec["v_sha256"])):
        raise AssertionError(f"{name}: regenerated inputs do not match the fixture digests")
    return dims, x, g, vs, gs, rec


def rel_l2(a, b):
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30)


def rel_max(a, b):
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return np.abs(a - b).max() / max(np.abs(b).max(), 1e-30)


@pytest.mark.parametrize("name", sorted(TRAIN_CASES))
def test_oracle_training_matches_reference_model(name):
    """The oracle's forward, closed-form backward and weight-norm backward
    reproduce the reference Model's autograd gradients."""
    dims, x, g, vs, gs, rec = load_train_case(name)
    rows = rec["rows"]
    ws = [oracle.weight_norm_forward(v.numpy(), gg.numpy())[0] for v, gg in zip(vs, gs)]
    ws16 = [w.astype(np.float16) for w in ws]  # the kernels' fp16 weights
    out, hs = oracle.mlp_forward_train(x.numpy(), ws16)
    assert rel_max(out[rows], rec["out_ref"]) <= OUT_TOL
    dx, dws = oracle.mlp_backward(x.numpy(), ws16, hs, g.numpy())
    assert rel_l2(dx[rows], rec["dx_ref"]) <= GRAD_TOL
    dw_flat = np.concatenate([d.reshape(-1) for d in dws])
    assert rel_l2(dw_flat, rec["dw_ref"]) <= GRAD_TOL
    dv, dg = [], []
    for v, gg, d in zip(vs, gs, dws):
        a, b = oracle.weight_norm_backward(v.numpy(), gg.numpy(), d)
        dv.append(a.reshape(-1))
        dg.append(b)
    assert rel_l2(np.concatenate(dv), rec["dv_ref"]) <= GRAD_TOL
    assert rel_l2(np.concatenate(dg), rec["dg_ref"]) <= GRAD_TOL


@pytest.mark.gpu
@pytest.mark.parametrize("h_dtype", [torch.float32, torch.float16])
@pytest.mark.parametrize("name", sorted(TRAIN_CASES))
def test_kernels_training_match_reference_model(name, h_dtype, built_lib):
    """FusedMLPSoftplusWN (weight-norm forward, training forward, fused
    backward, weight-norm backward) against the reference Model's autograd:
    out and dx on the recorded rows, dv and dg in full; and the backward's
    dW of the effective weights in full."""
    from mlp_megakernel_b200 import FusedMLPSoftplusWN, _lib
    from mlp_megakernel_b200.modules import _backward, _train_forward

    dims, x, g, vs, gs, rec = load_train_case(name)
    rows = torch.as_tensor(rec["rows"]).cuda()
    _lib.device_status(clear=True)
    model = FusedMLPSoftplusWN(D=dims[0], H=dims[1], out_features=dims[-1],
                               activation_dtype=h_dtype).cuda()
    with torch.no_grad():
        model.v_all.copy_(torch.cat([v.reshape(-1) for v in vs]))
        model.g_all.copy_(torch.cat(gs))
    xg = x.cuda().requires_grad_(True)
    out = model(xg)
    out.backward(g.cuda())
    torch.cuda.synchronize()
    assert rel_max(out.detach()[rows].float().cpu().numpy(), rec["out_ref"]) <= OUT_TOL
    assert rel_l2(xg.grad[rows].float().cpu().numpy(), rec["dx_ref"]) <= GRAD_TOL
    assert rel_l2(model.v_all.grad.cpu().numpy(), rec["dv_ref"]) <= GRAD_TOL
    assert rel_l2(model.g_all.grad.cpu().numpy(), rec["dg_ref"]) <= GRAD_TOL
    # dW of the effective (weight-normed) weights straight from the backward
    ws = [model.weight(l).detach().half().contiguous() for l in range(len(dims) - 1)]
    xs = x.cuda()
    _, hs = _train_forward(xs, ws, dims, h_dtype)
    _, dw = _backward(xs, ws, hs, g.cuda(), dims)
    assert rel_l2(dw.cpu().numpy(), rec["dw_ref"]) <= GRAD_TOL
    assert _lib.device_status() == 0
