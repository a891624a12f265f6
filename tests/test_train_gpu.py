"""GPU parity of the training path: training forward, fused backward (dx and
the deterministic split-K weight gradients), weight norm, and the module API
through torch.autograd.

Tolerances (north star): outputs max|d| <= 1e-2 * max|ref|; gradients
relative L2 <= 1e-2.  The oracle is the closed-form backward of
oracle/mlp_oracle.py (float64, fp16 GEMM operands), itself checked against
torch.autograd in tests/test_oracle.py.
"""
import numpy as np
import pytest
import torch

import oracle
from mlp_megakernel_b200 import FusedMLPSoftplus, FusedMLPSoftplusWN, _lib, fused_mlp_fwd
from mlp_megakernel_b200.modules import _backward, _train_forward
from mlp_megakernel_b200.synthetic import make_grad, make_inputs, make_weights, make_x, weight_norm_init

pytestmark = pytest.mark.gpu

DIMS = (128, 128, 128, 128)
GRAD_TOL = 1e-2
OUT_TOL = 1e-2


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


def _run(x, ws, g, dims=DIMS):
    xg, wg, gg = x.cuda(), [w.cuda() for w in ws], g.cuda()
    out, hs = _train_forward(xg, wg, dims)
    dx, dw = _backward(xg, wg, hs, gg, dims)
    torch.cuda.synchronize()
    return out, hs, dx, dw


def _split(dw, dims=DIMS):
    out, off = [], 0
    for a, b in zip(dims[:-1], dims[1:]):
        out.append(dw[off:off + a * b].reshape(a, b))
        off += a * b
    return out


@pytest.mark.parametrize("config,M", [("5L", 1), ("5L", 300), ("5L", 65536), ("5L", 148 * 128 * 3 + 5)])
def test_train_5layer_matches_oracle(config, M):
    """BASELINE config 4 shape: 32 -> 64 -> 64 -> 64 -> 64 -> 16 (x ~ U(-1,1))."""
    dims = (32, 64, 64, 64, 64, 16)
    x, ws, g = make_inputs(config, M, with_grad=True)
    out, hs, dx, dw = _run(x, ws, g, dims)
    ref_out, ref_hs = oracle.mlp_forward_train(x.numpy(), [w.numpy() for w in ws])
    assert rel_max(out.cpu().numpy(), ref_out) <= OUT_TOL
    ref_dx, ref_dws = oracle.mlp_backward(x.numpy(), [w.numpy() for w in ws], ref_hs, g.numpy())
    assert rel_l2(dx.cpu().numpy(), ref_dx) <= GRAD_TOL
    for d, rd in zip(_split(dw.cpu().numpy(), dims), ref_dws):
        assert rel_l2(d, rd) <= GRAD_TOL
    dx2, dw2 = _backward(x.cuda(), [w.cuda() for w in ws], hs, g.cuda(), dims)
    assert torch.equal(dw, dw2)


@pytest.mark.parametrize("M", [1, 300, 40000])
def test_train_w256_matches_oracle(M):
    """BASELINE config 5 shape (D = H = OUT = 256): streamed-weight training
    forward, data-gradient chain, split-K weight gradients."""
    dims = (256, 256, 256, 256)
    x, ws, g = make_inputs("W256", M, with_grad=True)
    out, hs, dx, dw = _run(x, ws, g, dims)
    assert torch.equal(out, fused_mlp_fwd(x.cuda(), *[w.cuda() for w in ws]))
    ref_out, ref_hs = oracle.mlp_forward_train(x.numpy(), [w.numpy() for w in ws])
    assert rel_max(out.cpu().numpy(), ref_out) <= OUT_TOL
    for h, rh in zip(hs, ref_hs):
        assert rel_max(h.cpu().numpy(), rh) <= 2e-3
    ref_dx, ref_dws = oracle.mlp_backward(x.numpy(), [w.numpy() for w in ws], ref_hs, g.numpy())
    assert rel_l2(dx.cpu().numpy(), ref_dx) <= GRAD_TOL
    for d, rd in zip(_split(dw.cpu().numpy(), dims), ref_dws):
        assert rel_l2(d, rd) <= GRAD_TOL
    dx2, dw2 = _backward(x.cuda(), [w.cuda() for w in ws], hs, g.cuda(), dims)
    assert torch.equal(dw, dw2) and torch.equal(dx, dx2)


def test_module_w256_wn_autograd():
    """FusedMLPSoftplusWN(D=H=OUT=256) through autograd (BASELINE config 5 shape)."""
    torch.manual_seed(5)
    model = FusedMLPSoftplusWN(D=256, H=256, out_features=256).cuda()
    M = 3000
    x, _, g = make_inputs("W256", M, with_grad=True)
    x, g = x.cuda(), g.cuda()
    out = model(x)
    out.backward(g)
    torch.cuda.synchronize()
    v = model.v_all.detach().double().cpu().requires_grad_(True)
    gg = model.g_all.detach().double().cpu().requires_grad_(True)
    ws, off, goff = [], 0, 0
    for a, b in zip(model.dims[:-1], model.dims[1:]):
        vl = v[off:off + a * b].view(a, b)
        ws.append(gg[goff:goff + b] * vl / vl.norm(dim=0, keepdim=True))
        off += a * b
        goff += b
    ref = x.cpu().double()
    for i, w in enumerate(ws):
        ref = ref @ w
        if i < len(ws) - 1:
            ref = torch.nn.functional.softplus(ref)
    ref.backward(g.cpu().double())
    assert rel_max(out.detach().cpu().numpy(), ref.detach().numpy()) <= OUT_TOL
    assert rel_l2(model.v_all.grad.cpu().numpy(), v.grad.numpy()) <= GRAD_TOL
    assert rel_l2(model.g_all.grad.cpu().numpy(), gg.grad.numpy()) <= GRAD_TOL


def test_train_64wide_matches_oracle():
    dims = (64, 64, 64, 64)
    M = 3000
    x = make_x(M, 64, "normal", 7)
    ws = make_weights(dims)
    g = make_grad(M, 64, seed=8)
    out, hs, dx, dw = _run(x, ws, g, dims)
    ref_out, ref_hs = oracle.mlp_forward_train(x.numpy(), [w.numpy() for w in ws])
    ref_dx, ref_dws = oracle.mlp_backward(x.numpy(), [w.numpy() for w in ws], ref_hs, g.numpy())
    assert rel_l2(dx.cpu().numpy(), ref_dx) <= GRAD_TOL
    for d, rd in zip(_split(dw.cpu().numpy(), dims), ref_dws):
        assert rel_l2(d, rd) <= GRAD_TOL


def test_module_5layer_wn_autograd():
    """FusedMLPSoftplusWN with 5 layers (D=32, H=64, OUT=16) through autograd."""
    torch.manual_seed(3)
    model = FusedMLPSoftplusWN(D=32, H=64, out_features=16, num_layers=5).cuda()
    M = 20000
    x, _, g = make_inputs("5L", M, with_grad=True)
    x, g = x.cuda(), g.cuda()
    out = model(x)
    torch.cuda.synchronize()
    out.backward(g)
    torch.cuda.synchronize()
    v = model.v_all.detach().double().cpu().requires_grad_(True)
    gg = model.g_all.detach().double().cpu().requires_grad_(True)
    ws, off, goff = [], 0, 0
    for a, b in zip(model.dims[:-1], model.dims[1:]):
        vl = v[off:off + a * b].view(a, b)
        ws.append(gg[goff:goff + b] * vl / vl.norm(dim=0, keepdim=True))
        off += a * b
        goff += b
    ref = x.cpu().double()
    for i, w in enumerate(ws):
        ref = ref @ w
        if i < len(ws) - 1:
            ref = torch.nn.functional.softplus(ref)
    ref.backward(g.cpu().double())
    assert rel_max(out.detach().cpu().numpy(), ref.detach().numpy()) <= OUT_TOL
    assert rel_l2(model.v_all.grad.cpu().numpy(), v.grad.numpy()) <= GRAD_TOL
    assert rel_l2(model.g_all.grad.cpu().numpy(), gg.grad.numpy()) <= GRAD_TOL


@pytest.mark.parametrize("M", [1, 127, 129, 1000, 16384, 148 * 128 + 1])
def test_train_forward_and_backward_match_oracle(M):
    x, ws, g = make_inputs("3L128", M, with_grad=True)
    out, hs, dx, dw = _run(x, ws, g)
    # training forward == inference forward, bitwise
    assert torch.equal(out, fused_mlp_fwd(x.cuda(), *[w.cuda() for w in ws]))
    ref_out, ref_hs = oracle.mlp_forward_train(x.numpy(), [w.numpy() for w in ws])
    assert rel_max(out.cpu().numpy(), ref_out) <= OUT_TOL
    for h, rh in zip(hs, ref_hs):  # saved activations (fp16 of the fp32 softplus)
        assert rel_max(h.cpu().numpy(), rh) <= 2e-3
    ref_dx, ref_dws = oracle.mlp_backward(x.numpy(), [w.numpy() for w in ws], ref_hs, g.numpy())
    assert rel_l2(dx.cpu().numpy(), ref_dx) <= GRAD_TOL
    for d, rd in zip(_split(dw.cpu().numpy()), ref_dws):
        assert rel_l2(d, rd) <= GRAD_TOL


def test_backward_split_k_regime_and_determinism():
    """BASELINE config 3, M = 262,144 (split-K regime): full weight gradients
    against the oracle, and bitwise-identical dW over repeated runs."""
    M = 262144
    x, ws, g = make_inputs("3L128", M, with_grad=True)
    out, hs, dx, dw = _run(x, ws, g)
    dx2, dw2 = _backward(x.cuda(), [w.cuda() for w in ws], hs, g.cuda(), DIMS)
    torch.cuda.synchronize()
    assert torch.equal(dw, dw2), "weight gradients are not deterministic"
    assert torch.equal(dx, dx2)
    ref_out, ref_hs = oracle.mlp_forward_train(x.numpy(), [w.numpy() for w in ws])
    ref_dx, ref_dws = oracle.mlp_backward(x.numpy(), [w.numpy() for w in ws], ref_hs, g.numpy())
    for d, rd in zip(_split(dw.cpu().numpy()), ref_dws):
        assert rel_l2(d, rd) <= GRAD_TOL
    assert rel_l2(dx.cpu().numpy(), ref_dx) <= GRAD_TOL


@pytest.mark.parametrize("config,dims", [("3L128", DIMS), ("5L", (32, 64, 64, 64, 64, 16)),
                                         ("W256", (256, 256, 256, 256))])
def test_backward_empty_batch(config, dims):
    x, ws, g = make_inputs(config, 0, with_grad=True)
    out, hs, dx, dw = _run(x, ws, g, dims)
    assert out.shape == (0, dims[-1]) and dx.shape == (0, dims[0])
    assert float(dw.abs().max()) == 0.0


def test_weight_norm_kernels_match_oracle():
    from mlp_megakernel_b200.modules import _stream
    import ctypes

    ws = make_weights(DIMS)
    vs = [(w.float() + 0.01 * torch.randn(w.shape, generator=torch.Generator().manual_seed(i)))
          for i, w in enumerate(ws)]
    gs = [v.norm(dim=0) * (1.0 + 0.1 * i) for i, v in enumerate(vs)]
    v_all = torch.cat([v.reshape(-1) for v in vs]).cuda()
    g_all = torch.cat(gs).cuda()
    W = [torch.empty(a, b, dtype=torch.float16, device="cuda") for a, b in zip(DIMS[:-1], DIMS[1:])]
    inv = torch.empty_like(g_all)
    lib = _lib.lib()
    shape = _lib.shape_struct(DIMS)
    _lib.check("mlpk_wn_fwd", lib.mlpk_wn_fwd(ctypes.byref(shape), v_all.data_ptr(), g_all.data_ptr(),
                                              _lib.ptr_array([w.data_ptr() for w in W]),
                                              inv.data_ptr(), _stream(v_all.device)))
    dW = [torch.randn(a, b, generator=torch.Generator().manual_seed(10 + i))
          for i, (a, b) in enumerate(zip(DIMS[:-1], DIMS[1:]))]
    dw_all = torch.cat([d.reshape(-1) for d in dW]).cuda()
    dv = torch.empty_like(v_all)
    dg = torch.empty_like(g_all)
    _lib.check("mlpk_wn_bwd", lib.mlpk_wn_bwd(ctypes.byref(shape), dw_all.data_ptr(), v_all.data_ptr(),
                                              g_all.data_ptr(), inv.data_ptr(), dv.data_ptr(),
                                              dg.data_ptr(), _stream(v_all.device)))
    torch.cuda.synchronize()
    voff = goff = 0
    for l, (a, b) in enumerate(zip(DIMS[:-1], DIMS[1:])):
        rW, rinv = oracle.weight_norm_forward(vs[l].numpy(), gs[l].numpy())
        assert rel_max(W[l].cpu().numpy(), rW) <= 1e-3
        assert rel_max(inv[goff:goff + b].cpu().numpy(), rinv) <= 1e-5
        rdv, rdg = oracle.weight_norm_backward(vs[l].numpy(), gs[l].numpy(), dW[l].numpy())
        assert rel_l2(dv[voff:voff + a * b].cpu().numpy().reshape(a, b), rdv) <= 1e-5
        assert rel_l2(dg[goff:goff + b].cpu().numpy(), rdg) <= 1e-5
        voff += a * b
        goff += b


def _torch_reference(x, weights, grad):
    xt = x.detach().double().requires_grad_(True)
    out = xt
    for i, w in enumerate(weights):
        out = out @ w
        if i < len(weights) - 1:
            out = torch.nn.functional.softplus(out)
    out.backward(grad.double())
    return out.detach(), xt.grad


def test_module_fused_mlp_softplus_autograd():
    """FusedMLPSoftplus(...).cuda().half(); model(x); loss.backward() (README.md:58-70)."""
    torch.manual_seed(0)
    model = FusedMLPSoftplus(D=128, H=128, out_features=128).cuda().half()
    M = 4096
    x = make_x(M, 128, "normal", 0).cuda().requires_grad_(True)
    g = make_grad(M, 128).cuda()
    out = model(x)
    out.backward(g)
    torch.cuda.synchronize()
    ws_ref = [w.detach().double().cpu().requires_grad_(True) for w in model.weights]
    ref_out, ref_dx = _torch_reference(x.detach().cpu(), ws_ref, g.cpu())
    assert rel_max(out.detach().cpu().numpy(), ref_out.numpy()) <= OUT_TOL
    assert rel_l2(x.grad.cpu().numpy(), ref_dx.numpy()) <= GRAD_TOL
    for w, wr in zip(model.weights, ws_ref):
        assert w.grad is not None and w.grad.dtype == torch.float16
        assert rel_l2(w.grad.float().cpu().numpy(), wr.grad.numpy()) <= GRAD_TOL


def test_module_fused_mlp_softplus_wn_autograd():
    """FusedMLPSoftplusWN: gradients of v_all, g_all and x against explicit
    weight norm + MLP under torch.autograd in float64."""
    torch.manual_seed(1)
    model = FusedMLPSoftplusWN(D=128, H=128, out_features=128).cuda()
    with torch.no_grad():  # g != ||v|| so the weight norm is not the identity
        model.g_all.mul_(1.3)
    M = 16384
    x = make_x(M, 128, "normal", 0).cuda()
    g = make_grad(M, 128).cuda()
    out = model(x)
    out.backward(g)
    torch.cuda.synchronize()
    v = model.v_all.detach().double().cpu().requires_grad_(True)
    gg = model.g_all.detach().double().cpu().requires_grad_(True)
    ws, off, goff = [], 0, 0
    for a, b in zip(model.dims[:-1], model.dims[1:]):
        vl = v[off:off + a * b].view(a, b)
        gl = gg[goff:goff + b]
        ws.append(gl * vl / vl.norm(dim=0, keepdim=True))
        off += a * b
        goff += b
    xr = x.cpu().double()
    ref = xr
    for i, w in enumerate(ws):
        ref = ref @ w
        if i < len(ws) - 1:
            ref = torch.nn.functional.softplus(ref)
    ref.backward(g.cpu().double())
    assert rel_max(out.detach().cpu().numpy(), ref.detach().numpy()) <= OUT_TOL
    assert rel_l2(model.v_all.grad.cpu().numpy(), v.grad.numpy()) <= GRAD_TOL
    assert rel_l2(model.g_all.grad.cpu().numpy(), gg.grad.numpy()) <= GRAD_TOL


def test_module_under_autocast_and_fp32_params():
    """custom_fwd(cast_inputs=fp16): fp32 inputs/params under autocast work and
    gradients come back in the parameters' dtype."""
    model = FusedMLPSoftplus().cuda()
    x = torch.randn(1000, 128, device="cuda", requires_grad=True)
    with torch.autocast("cuda", dtype=torch.float16):
        out = model(x)
    out.float().sum().backward()
    assert out.dtype == torch.float16
    assert x.grad is not None and x.grad.dtype == torch.float32
    assert all(w.grad.dtype == torch.float32 for w in model.weights)


@pytest.mark.parametrize("config,dims,M", [("5L", (32, 64, 64, 64, 64, 16), 1048576),
                                           ("3L128", DIMS, 1048576),
                                           ("W256", (256, 256, 256, 256), 262144)])
def test_repeated_launches_are_stable(config, dims, M):
    """Many back-to-back inference and training forwards and backwards: every
    repetition bitwise equal to the first and no bounded wait expired (the
    fixture checks the device status word).  Catches hand-off races between
    the warp roles that a single launch may not hit."""
    x, ws, g = make_inputs(config, M, with_grad=True)
    x, ws, g = x.cuda(), [w.cuda() for w in ws], g.cuda()
    ref = fused_mlp_fwd(x, *ws)
    ref_t, hs = _train_forward(x, ws, dims)
    dx0, dw0 = _backward(x, ws, hs, g, dims)
    assert torch.equal(ref, ref_t)
    for _ in range(20):
        out = fused_mlp_fwd(x, *ws)
        out_t, hs2 = _train_forward(x, ws, dims)
        dx, dw = _backward(x, ws, hs2, g, dims)
        assert torch.equal(out, ref) and torch.equal(out_t, ref)
        assert torch.equal(dx, dx0) and torch.equal(dw, dw0)
    assert _lib.device_status() == 0


def test_module_under_autocast():
    """AMP (mlp_fused.md:168-172): fp32 parameters and input under torch.autocast
    run the fp16 kernels (custom_fwd casts the inputs); gradients come back in
    the parameters' dtype."""
    torch.manual_seed(11)
    model = FusedMLPSoftplus(D=128, H=128, out_features=128).cuda()  # fp32 parameters
    M = 5000
    x, _, g = make_inputs("3L128", M, with_grad=True)
    xf = x.float().cuda()
    with torch.autocast("cuda", dtype=torch.float16):
        out = model(xf)
    assert out.dtype == torch.float16
    out.backward(g.cuda())
    assert all(w.grad.dtype == torch.float32 for w in model.weights)
    ws = [w.detach().half().float().cpu() for w in model.weights]
    ref_out, ref_hs = oracle.mlp_forward_train(x.numpy(), [w.numpy() for w in ws])
    assert rel_max(out.detach().cpu().numpy(), ref_out) <= OUT_TOL
    _, ref_dws = oracle.mlp_backward(x.numpy(), [w.numpy() for w in ws], ref_hs, g.numpy())
    for w, rd in zip(model.weights, ref_dws):
        assert rel_l2(w.grad.cpu().numpy(), rd) <= GRAD_TOL


def test_training_step_in_cuda_graph():
    """A whole training step (weight-normed module forward + backward) captured
    in a CUDA graph after one eager warm-up step, replayed on new inputs copied
    into the static buffers: same gradients as eager."""
    torch.manual_seed(12)
    model = FusedMLPSoftplusWN(D=32, H=64, out_features=16, num_layers=5).cuda()
    M = 30000
    x1, _, g1 = make_inputs("5L", M, with_grad=True)
    sx, sg = x1.cuda().clone(), g1.cuda().clone()
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream):  # warm-up (sets kernel attributes, caches)
        model(sx).backward(sg)
    torch.cuda.current_stream().wait_stream(stream)
    graph = torch.cuda.CUDAGraph()
    model.v_all.grad.zero_()
    model.g_all.grad.zero_()
    with torch.cuda.graph(graph):
        model(sx).backward(sg)
    # new data through the static buffers
    x2 = (x1.float() * 0.5).half()
    g2 = (g1.float() * -1.5).half()
    sx.copy_(x2.cuda())
    sg.copy_(g2.cuda())
    model.v_all.grad.zero_()
    model.g_all.grad.zero_()
    graph.replay()
    torch.cuda.synchronize()
    gv, gg = model.v_all.grad.clone(), model.g_all.grad.clone()
    model.v_all.grad = None
    model.g_all.grad = None
    model(x2.cuda()).backward(g2.cuda())
    torch.cuda.synchronize()
    assert torch.equal(gv, model.v_all.grad) and torch.equal(gg, model.g_all.grad)


@pytest.mark.parametrize("wn", [False, True])
def test_module_under_torch_compile(wn):
    """torch.compile(fullgraph=True) of the fused modules: the autograd
    Function calls the library through torch.ops.mlpk.* custom operators,
    so dynamo traces forward and backward without a graph break; same
    outputs and gradients as eager."""
    torch.manual_seed(13)
    if wn:
        model = FusedMLPSoftplusWN(D=128, H=128, out_features=128).cuda()
        params = [model.v_all, model.g_all]
    else:
        model = FusedMLPSoftplus(D=128, H=128, out_features=128).cuda().half()
        params = list(model.weights)
    x, _, g = make_inputs("3L128", 4000, with_grad=True)
    x, g = x.cuda(), g.cuda()
    out_e = model(x)
    out_e.backward(g)
    grads_e = [p.grad.clone() for p in params]
    for p in params:
        p.grad = None
    torch._dynamo.reset()
    compiled = torch.compile(model, fullgraph=True)
    out_c = compiled(x)
    out_c.backward(g)
    torch.cuda.synchronize()
    assert torch.equal(out_c, out_e)
    for p, ge in zip(params, grads_e):
        assert torch.equal(p.grad, ge)


def test_functional_forward_under_torch_compile():
    """fused_mlp_fwd inside a compiled function (fullgraph): one mlpk::fwd
    operator between ordinary torch ops."""
    x, ws = make_inputs("3L128", 3000)
    xg, wg = x.cuda(), [w.cuda() for w in ws]

    def f(a):  # exact fp16 arithmetic around the operator: results bitwise comparable
        return fused_mlp_fwd(a * 2, *wg) * 0.5

    torch._dynamo.reset()
    ref = f(xg)
    got = torch.compile(f, fullgraph=True)(xg)
    assert torch.equal(ref, got)
