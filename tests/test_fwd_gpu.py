"""GPU parity of the fused forward (libmlpk through its C ABI) against the
reference kernel's golden outputs and the CPU oracle.

Tolerance (from the task's north star): max|out - ref| <= 1e-2 * max|ref|.
The kernel is also held to a tighter implementation bar (3e-3) because it
computes the same fp16-operand / fp32-accumulate chain as the reference.
"""
import ctypes

import numpy as np
import pytest
import torch

import oracle
from mlp_megakernel_b200 import ModelNew, _fused_mlp_fwd, fused_mlp_fwd, fused_mlp_fwd_host
from mlp_megakernel_b200 import _lib
from mlp_megakernel_b200.synthetic import make_inputs, make_weights, make_x
from tests.golden_io import case_names, load_case

pytestmark = pytest.mark.gpu

TOL = 1e-2      # north-star parity tolerance, relative to max|ref|
TIGHT = 3e-3    # implementation bar
TF32_TOL = 1e-2  # tf32 operands: 10 mantissa bits per GEMM input


def _rel_max(got, ref):
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    return np.abs(got - ref).max() / max(np.abs(ref).max(), 1e-6)


def _gpu(ts):
    return [t.cuda() for t in ts]


@pytest.fixture(autouse=True)
def _lib_loaded(built_lib):
    _lib.device_status(clear=True)
    yield
    assert _lib.device_status() == 0, "a kernel recorded a device-side timeout"


@pytest.mark.parametrize("name", case_names())
def test_fwd_matches_reference_kernel_golden(name):
    x, ws, rows, out_ref, rec = load_case(name)
    dims = [x.shape[1]] + [w.shape[1] for w in ws]
    if not _lib.shape_supported(dims):
        pytest.skip(f"no forward kernel for dims {dims} yet")
    out = fused_mlp_fwd(x.cuda(), *_gpu(ws)).cpu().numpy()[rows]
    err = _rel_max(out, out_ref)
    assert err <= TOL, f"{name}: {err:.3e}"
    assert err <= TIGHT, f"{name}: {err:.3e} (parity ok, implementation bar missed)"


@pytest.mark.parametrize("config,M", [("3L128", 4096), ("5L", 8192), ("3L128", 148 * 128 * 3 + 77),
                                      ("W256", 1), ("W256", 129), ("W256", 5000),
                                      ("W256", 148 * 128 * 2 + 3)])
def test_fwd_matches_oracle(config, M):
    x, ws = make_inputs(config, M)
    out = fused_mlp_fwd(x.cuda(), *_gpu(ws)).cpu().numpy()
    ref = oracle.mlp_forward(x.numpy(), [w.numpy() for w in ws])
    assert _rel_max(out, ref) <= TIGHT


@pytest.mark.parametrize("M", [1, 2, 64, 127, 128, 129, 255, 256, 1000, 148 * 128, 148 * 128 + 1])
def test_fwd_ragged_batch_sizes(M):
    x, ws = make_inputs("3L128", M)
    out = fused_mlp_fwd(x.cuda(), *_gpu(ws)).cpu().numpy()
    ref = oracle.mlp_forward(x.numpy(), [w.numpy() for w in ws])
    assert out.shape == (M, 128)
    assert _rel_max(out, ref) <= TIGHT


@pytest.mark.parametrize("M", [148 * 256 + 128, 1 << 20])
def test_fwd_multi_round_batches(M):
    """Batches that give every CTA several rounds of row tiles (and a ragged
    last round): edge and strided rows against the oracle."""
    x, ws = make_inputs("3L128", M)
    out = fused_mlp_fwd(x.cuda(), *_gpu(ws))
    torch.cuda.synchronize()
    rows = np.unique(np.concatenate([np.arange(min(M, 512)), np.arange(max(0, M - 512), M),
                                     np.arange(0, M, max(1, M // 512))]))
    ref = oracle.mlp_forward(x.numpy()[rows], [w.numpy() for w in ws])
    assert _rel_max(out.cpu().numpy()[rows], ref) <= TIGHT


@pytest.mark.parametrize("dims", [(128, 128, 128), (96, 128, 80, 40), (64, 128, 128, 16), (32, 128, 128, 128)])
def test_fwd_throughput_config_networks(dims):
    """Inference batches of more than one row tile per SM (the throughput
    configuration) on networks served with 128-wide hidden layers: the 2-layer
    network and narrower widths by zero fill, against the oracle, ragged last
    tile included."""
    M = 148 * 128 * 2 + 77
    x = make_x(M, dims[0], "normal", 11)
    ws = make_weights(dims, seed=12)
    out = fused_mlp_fwd(x.cuda(), *_gpu(ws)).cpu().numpy()
    ref = oracle.mlp_forward(x.numpy(), [w.numpy() for w in ws])
    assert out.shape == (M, dims[-1])
    assert _rel_max(out, ref) <= TIGHT


def test_fwd_empty_batch():
    x, ws = make_inputs("3L128", 0)
    out = fused_mlp_fwd(x.cuda(), *_gpu(ws))
    assert out.shape == (0, 128)


def test_fwd_large_batch_properties():
    """M = 4,194,304 (top of the batch sweep): a strided + edge row sample
    against the oracle, bitwise determinism, and row-permutation equivariance
    (each row's result is independent of its tile)."""
    M = 4 * 1024 * 1024
    dims = (128, 128, 128, 128)
    x = make_x(M, 128, "normal", 0, device="cuda")
    ws = make_weights(dims, device="cuda")
    out = fused_mlp_fwd(x, *ws)
    out2 = fused_mlp_fwd(x, *ws)
    torch.cuda.synchronize()
    assert torch.equal(out, out2), "forward is not deterministic"
    rows = torch.cat([torch.arange(0, 2048), torch.arange(M - 2048, M), torch.arange(0, M, 1024)])
    ref = oracle.mlp_forward(x[rows].cpu().numpy(), [w.cpu().numpy() for w in ws])
    assert _rel_max(out[rows].cpu().numpy(), ref) <= TIGHT
    perm = torch.randperm(M, device="cuda", generator=torch.Generator("cuda").manual_seed(5))
    outp = fused_mlp_fwd(x[perm].contiguous(), *ws)
    assert torch.equal(outp, out[perm])
    assert torch.isfinite(out).all()


def test_fwd_large_preactivations_threshold_branch():
    """z > 20 (linear branch) and z << 0 (softplus underflow side)."""
    x, ws = make_inputs("3L128", 1024)
    ws = [(w.float() * 12).half() for w in ws]
    out = fused_mlp_fwd(x.cuda(), *_gpu(ws)).cpu().numpy()
    ref = oracle.mlp_forward(x.numpy(), [w.numpy() for w in ws])
    assert _rel_max(out, ref) <= TIGHT


def test_fwd_noncontiguous_inputs():
    """Non-contiguous x and weights are made contiguous first (kernel.py:132-133)."""
    x, ws = make_inputs("3L128", 999)
    ref = oracle.mlp_forward(x.numpy(), [w.numpy() for w in ws])
    xg = x.cuda().t().contiguous().t()
    wg = [w.cuda().t().contiguous().t() for w in ws]
    assert not xg.is_contiguous() and not wg[0].is_contiguous()
    out = fused_mlp_fwd(xg, *wg).cpu().numpy()
    assert _rel_max(out, ref) <= TIGHT


def test_fwd_misaligned_device_view():
    x, ws = make_inputs("3L128", 300)
    buf = torch.zeros(300 * 128 + 1, dtype=torch.float16, device="cuda")
    buf[1:] = x.reshape(-1).cuda()
    xv = buf[1:].view(300, 128)
    assert xv.data_ptr() % 16 != 0
    out = fused_mlp_fwd(xv, *_gpu(ws)).cpu().numpy()
    ref = oracle.mlp_forward(x.numpy(), [w.numpy() for w in ws])
    assert _rel_max(out, ref) <= TIGHT


def test_fwd_out_buffer():
    x, ws = make_inputs("3L128", 700)
    xg, wg = x.cuda(), _gpu(ws)
    ref = fused_mlp_fwd(xg, *wg)
    buf = torch.full((700, 128), float("nan"), dtype=torch.float16, device="cuda")
    got = fused_mlp_fwd(xg, *wg, out=buf)
    assert got.data_ptr() == buf.data_ptr() and torch.equal(got, ref)
    with pytest.raises(ValueError):
        fused_mlp_fwd(xg, *wg, out=torch.empty(700, 64, dtype=torch.float16, device="cuda"))


def test_fwd_reference_api_names():
    x, ws = make_inputs("3L128", 512)
    xg, wg = x.cuda(), _gpu(ws)
    a = _fused_mlp_fwd(xg, *wg)
    b = ModelNew()(xg, *wg)
    assert torch.equal(a, b)
    assert a.dtype == torch.float16 and a.shape == (512, 128)


def test_fwd_cuda_graph_and_side_stream():
    x, ws = make_inputs("3L128", 8192)
    xg, wg = x.cuda(), _gpu(ws)
    eager = fused_mlp_fwd(xg, *wg)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        side = fused_mlp_fwd(xg, *wg)
    s.synchronize()
    assert torch.equal(side, eager)
    g = torch.cuda.CUDAGraph()
    static_x = xg.clone()
    fused_mlp_fwd(static_x, *wg)  # warm-up (attribute setup) outside capture
    torch.cuda.synchronize()
    with torch.cuda.graph(g):
        static_out = fused_mlp_fwd(static_x, *wg)
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(static_out, eager)


def test_fwd_errors_are_loud():
    x, ws = make_inputs("3L128", 16)
    with pytest.raises(RuntimeError):
        fused_mlp_fwd(x, *ws)  # CPU tensors: no fallback
    with pytest.raises(TypeError):
        fused_mlp_fwd(x.double().cuda(), *[w.double().cuda() for w in ws])
    with pytest.raises(ValueError):  # fp32 x with fp16 weights: dtypes must agree
        fused_mlp_fwd(x.float().cuda(), *[w.cuda() for w in ws])
    with pytest.raises(ValueError):
        fused_mlp_fwd(x.cuda(), ws[0].cuda(), ws[1][:64].cuda(), ws[2].cuda())
    # a width that is not a multiple of 8: no kernel serves it
    bad = [torch.zeros(128, 100, dtype=torch.float16, device="cuda"),
           torch.zeros(100, 128, dtype=torch.float16, device="cuda")]
    with pytest.raises(_lib.MlpkError):
        fused_mlp_fwd(x.cuda(), *bad)


@pytest.mark.parametrize("config,M", [("3L128", 4096), ("3L128", 300), ("5L", 5000)])
def test_fwd_fp32_inputs(config, M):
    """fp32 x and W (the reference accepts them, kernel.py:134-138): the result
    is fp32 from the tf32 chain (fp32 hidden activations), within tf32's
    tolerance of the formula in float64 on the fp32 operands and of the fp16
    path on the fp16-rounded operands; the out= form gives the same bits."""
    x, ws = make_inputs(config, M)
    x32 = (x.float() + 1e-4 * torch.randn(x.shape, generator=torch.Generator().manual_seed(3))).cuda()
    w32 = [(w.float() * 1.0003).cuda() for w in ws]
    out = fused_mlp_fwd(x32, *w32)
    assert out.dtype == torch.float32 and out.shape == (M, ws[-1].shape[1])
    ref = _f64_forward(x32.cpu().numpy(), [w.cpu().numpy() for w in w32])
    assert _rel_max(out.cpu().numpy(), ref) <= TF32_TOL
    ref16 = fused_mlp_fwd(x32.half(), *[w.half() for w in w32]).float()
    assert _rel_max(out.cpu().numpy(), ref16.cpu().numpy()) <= TF32_TOL
    buf = torch.empty_like(out)
    assert fused_mlp_fwd(x32, *w32, out=buf) is buf and torch.equal(buf, out)


def test_fwd_rejects_other_dtypes():
    x, ws = make_inputs("3L128", 64)
    with pytest.raises(TypeError):
        fused_mlp_fwd(x.cuda().bfloat16(), *[w.cuda().bfloat16() for w in ws])


@pytest.mark.parametrize("dims,M,chunk,pinned", [
    ((128, 128, 128, 128), 1, 0, True),
    ((128, 128, 128, 128), 300, 128, True),
    ((128, 128, 128, 128), 2 * 131072 + 5, 0, True),
    ((128, 128, 128, 128), 1 << 20, 65536, True),
    ((128, 128, 128, 128), 5000, 1000, False),
    ((32, 64, 64, 64, 64, 16), 70001, 8192, True),
    ((48, 128, 80, 24), 9999, 1024, True),
])
def test_fwd_host_rows_equal_device_forward(dims, M, chunk, pinned):
    """Host-resident rows streamed through the GPU in chunks give bitwise the
    device forward's result (every chunk runs the same kernel on its rows)."""
    x = make_x(M, dims[0], "normal", 21)
    ws = [w.cuda() for w in make_weights(dims, seed=22)]
    ref = fused_mlp_fwd(x.cuda(), *ws).cpu()
    xh = x.pin_memory() if pinned else x
    out = fused_mlp_fwd_host(xh, *ws, chunk_rows=chunk)
    assert not out.is_cuda and out.shape == (M, dims[-1])
    assert torch.equal(out, ref)
    buf = torch.full((M, dims[-1]), float("nan"), dtype=torch.float16)
    assert fused_mlp_fwd_host(xh, *ws, out=buf, chunk_rows=chunk) is buf and torch.equal(buf, ref)


def test_fwd_host_rows_errors():
    x, ws = make_inputs("3L128", 64)
    wg = _gpu(ws)
    with pytest.raises(ValueError):
        fused_mlp_fwd_host(x.cuda(), *wg)   # device rows: use fused_mlp_fwd
    with pytest.raises(TypeError):
        fused_mlp_fwd_host(x.float(), *wg)
    with pytest.raises(ValueError):
        fused_mlp_fwd_host(x, *ws)          # CPU weights
    assert fused_mlp_fwd_host(x[:0], *wg).shape == (0, 128)


# ---------------------------------------------------------------- fp32 on tf32 tensor cores


def _f64_forward(x, ws):
    """The reference formula (kernel.py:163-171) in float64, no fp16 rounding."""
    return oracle.mlp_forward(x, ws, round_h=False, round_out=False)


@pytest.mark.parametrize("dims", [(128, 128, 128, 128), (32, 64, 64, 64, 64, 16), (64, 64, 64, 64),
                                  (48, 128, 80, 24), (128, 128, 128, 128, 128, 128)])
@pytest.mark.parametrize("M", [1, 300, 148 * 128 + 77])
def test_fp32_forward_on_tf32_cores(dims, M):
    """fp32 x and W: the tf32 chain (fp32 hidden activations, fp32 output)
    against the formula in float64."""
    assert _lib.lib().mlpk_shape_supported_ex(ctypes.byref(_lib.shape_struct(dims)), _lib.DT_F32)
    x = make_x(M, dims[0], "normal", 5, dtype=torch.float32)
    ws = make_weights(dims, seed=6, dtype=torch.float32)
    out = fused_mlp_fwd(x.cuda(), *[w.cuda() for w in ws])
    assert out.dtype == torch.float32
    ref = _f64_forward(x.numpy(), [w.numpy() for w in ws])
    assert _rel_max(out.cpu().numpy(), ref) <= TF32_TOL


def test_fp32_forward_keeps_fp32_range():
    """Inputs far beyond fp16's range (|x| ~ 1e6, weights ~ 1e-6 and 1e5):
    fp16 operands would overflow or flush; the tf32 chain keeps fp32's
    exponent range."""
    dims = (128, 128, 128, 128)
    M = 4096
    x = make_x(M, 128, "normal", 7, dtype=torch.float32) * 1e6
    ws = make_weights(dims, seed=8, dtype=torch.float32)
    ws = [ws[0] * 1e-6, ws[1] * 1e5, ws[2] * 1e-5]
    out = fused_mlp_fwd(x.cuda(), *[w.cuda() for w in ws])
    assert torch.isfinite(out).all()
    ref = _f64_forward(x.numpy(), [w.numpy() for w in ws])
    assert _rel_max(out.cpu().numpy(), ref) <= TF32_TOL


def test_fp32_forward_wide_network_uses_fp16_operands():
    """256-wide networks have no tf32 kernel: fp32 operands are rounded to
    fp16 around the fp16 kernel (the inference kernel's rounding points)."""
    dims = (256, 256, 256, 256)
    assert not _lib.lib().mlpk_shape_supported_ex(ctypes.byref(_lib.shape_struct(dims)), _lib.DT_F32)
    x, ws = make_inputs("W256", 500)
    out = fused_mlp_fwd(x.float().cuda(), *[w.float().cuda() for w in ws])
    ref = oracle.mlp_forward(x.numpy(), [w.numpy() for w in ws])
    assert out.dtype == torch.float32 and _rel_max(out.cpu().numpy(), ref) <= TIGHT
