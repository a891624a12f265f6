"""The custom operators' fake implementations (CPU, no GPU needed).

torch.ops.mlpk.* must give correct output shapes and dtypes under FakeTensor
tracing (what torch.compile and meta-analysis see) without touching device
memory.  Here every operator, and the module API's forward, runs on fake CUDA
tensors.
"""
import pytest
import torch
from torch._subclasses.fake_tensor import FakeTensorMode

import mlp_megakernel_b200  # noqa: F401  (registers torch.ops.mlpk.*)
from mlp_megakernel_b200 import FusedMLPSoftplus, FusedMLPSoftplusWN, fused_mlp_fwd


@pytest.fixture
def fake():
    with FakeTensorMode() as m:
        yield m


def test_registered_ops():
    for name in ("fwd", "fwd_out", "train_fwd", "bwd", "wn_fwd", "wn_bwd"):
        assert hasattr(torch.ops.mlpk, name), name


@pytest.mark.parametrize("dtype", [torch.float16, torch.float32])
def test_functional_forward_shapes(fake, dtype, built_lib):
    x = torch.empty(1000, 48, device="cuda", dtype=dtype)
    ws = [torch.empty(48, 96, device="cuda", dtype=dtype), torch.empty(96, 96, device="cuda", dtype=dtype),
          torch.empty(96, 24, device="cuda", dtype=dtype)]
    out = fused_mlp_fwd(x, *ws)
    assert out.shape == (1000, 24) and out.dtype == dtype and out.device.type == "cuda"


@pytest.mark.parametrize("h_dtype", [torch.float32, torch.float16])
def test_train_ops_shapes(fake, h_dtype, built_lib):
    dims = (32, 64, 64, 64, 64, 16)
    x = torch.empty(777, 32, device="cuda", dtype=torch.float16)
    ws = [torch.empty(a, b, device="cuda", dtype=torch.float16) for a, b in zip(dims[:-1], dims[1:])]
    res = torch.ops.mlpk.train_fwd(x, ws, h_dtype == torch.float32)
    assert res[0].shape == (777, 16) and res[0].dtype == torch.float16
    assert [tuple(h.shape) for h in res[1:]] == [(777, 64)] * 4 and all(h.dtype == h_dtype for h in res[1:])
    g = torch.empty(777, 16, device="cuda", dtype=torch.float16)
    dx, dw = torch.ops.mlpk.bwd(x, ws, list(res[1:]), g)
    assert dx.shape == x.shape and dw.shape == (sum(a * b for a, b in zip(dims[:-1], dims[1:])),)
    assert dw.dtype == torch.float32


@pytest.mark.parametrize("wn", [False, True])
def test_module_forward_on_fake_tensors(fake, wn, built_lib):
    """The module forward (its autograd Function: weight norm, training
    forward) on fake CUDA tensors.  (The backward's operators are checked
    above; running autograd's engine itself needs a CUDA device.)"""
    with torch.device("cuda"):  # parameters created as fake CUDA tensors
        if wn:
            model = FusedMLPSoftplusWN(D=128, H=128, out_features=128)
        else:
            model = FusedMLPSoftplus(D=128, H=128, out_features=128)
    x = torch.empty(4096, 128, device="cuda", dtype=torch.float16, requires_grad=True)
    out = model(x)
    assert out.shape == (4096, 128) and out.dtype == torch.float16 and out.requires_grad


def test_weight_norm_ops_shapes(fake, built_lib):
    dims = [128, 128, 128, 128]
    n = sum(a * b for a, b in zip(dims[:-1], dims[1:]))
    v = torch.empty(n, device="cuda")
    g = torch.empty(sum(dims[1:]), device="cuda")
    res = torch.ops.mlpk.wn_fwd(v, g, dims)
    assert [tuple(w.shape) for w in res[:-1]] == [(128, 128)] * 3 and res[0].dtype == torch.float16
    assert res[-1].shape == g.shape
    dv, dg = torch.ops.mlpk.wn_bwd(torch.empty(n, device="cuda"), v, g, res[-1], dims)
    assert dv.shape == v.shape and dg.shape == g.shape
