"""The device-side MLP (include/mlpk_device.cuh) called from a user kernel.

tests/device_api/devtest.cu is such a user kernel: it frequency-encodes 3-d
points (sin/cos), runs mlpk::device::FusedMLP on the encoded rows in
registers and reduces each output row to a loss (sum of squares), in one
launch.  Checked against the oracle (oracle/mlp_oracle.py) on the same
encoding computed in float64 and rounded to fp16 as the kernel's GEMM
operand: outputs max|d| <= 1e-2 * max|ref|, losses relative L2 <= 1e-2.
"""
import ctypes

import numpy as np
import pytest
import torch

import oracle

NETS = {0: (64, 64, 64, 16), 1: (64, 128, 128, 128, 32)}
FREQS = 5


@pytest.fixture(scope="module")
def devlib():
    from mlp_megakernel_b200 import build as _build

    path = _build.build_devtest()
    lib = ctypes.CDLL(path)
    fn = lib.mlpk_devtest_encode_mlp_loss
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_int, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p,
                   ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p]
    return lib


def test_devtest_library_builds_and_exports(devlib):
    assert hasattr(devlib, "mlpk_devtest_encode_mlp_loss")


def _encode(pts: np.ndarray) -> np.ndarray:
    """The kernel's frequency encoding in float64: [p, sin(2^k p), cos(2^k p)]
    per coordinate, zero-padded to 64 features."""
    M = pts.shape[0]
    x = np.zeros((M, 64))
    x[:, :3] = pts
    for k in range(FREQS):
        f = 2.0 ** k
        for c in range(3):
            x[:, 3 + 6 * k + 2 * c] = np.sin(f * pts[:, c])
            x[:, 3 + 6 * k + 2 * c + 1] = np.cos(f * pts[:, c])
    return x


@pytest.mark.gpu
@pytest.mark.parametrize("M", [1, 1000, 70_000])
@pytest.mark.parametrize("net", sorted(NETS))
def test_user_kernel_encode_mlp_loss(devlib, net, M):
    dims = NETS[net]
    g = torch.Generator().manual_seed(net * 1000 + M)
    pts = (torch.rand(M, 3, generator=g) * 2 - 1).float()
    ws = [((torch.rand(a, b, generator=g) * 2 - 1) / a ** 0.5).half() for a, b in zip(dims[:-1], dims[1:])]
    dev = torch.device("cuda", 0)
    pts_d = pts.to(dev)
    ws_d = [w.to(dev) for w in ws]
    wptr = torch.tensor([w.data_ptr() for w in ws_d], dtype=torch.int64, device=dev)
    out = torch.empty(M, dims[-1], dtype=torch.float32, device=dev)
    loss = torch.empty(M, dtype=torch.float32, device=dev)
    failed = torch.zeros(1, dtype=torch.int32, device=dev)
    grid = min(148, (M + 127) // 128)
    rc = devlib.mlpk_devtest_encode_mlp_loss(net, pts_d.data_ptr(), M, wptr.data_ptr(), out.data_ptr(),
                                            loss.data_ptr(), failed.data_ptr(), grid,
                                            torch.cuda.current_stream().cuda_stream)
    assert rc == 0
    torch.cuda.synchronize()
    assert int(failed.item()) == 0, "a bounded wait of the device MLP expired"
    x16 = _encode(pts.numpy().astype(np.float64)).astype(np.float16)
    ref = oracle.mlp_forward(x16, [w.numpy() for w in ws])
    got = out.cpu().numpy()
    assert np.abs(got - ref).max() <= 1e-2 * np.abs(ref).max()
    ref_loss = (ref ** 2).sum(axis=1)
    got_loss = loss.cpu().numpy()
    assert np.linalg.norm(got_loss - ref_loss) <= 1e-2 * np.linalg.norm(ref_loss)
