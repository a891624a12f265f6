"""Failure detection on the device: a bounded wait that expires.

Every wait in the library's kernels gives up after a bounded time, records a
bit in the device status word (mlpk_device_status) and returns, so a missing
peer or a lost hand-off becomes an error the host reads instead of a hung GPU.
This test makes one such wait run out on purpose, with no second GPU and no
fault: the cross-GPU weight-gradient sum (mlpk_peer_allreduce) is called as
rank 0 of a world of 2 whose "rank 1" buffer is a second buffer on this GPU
that no kernel ever signals.  The kernel waits for rank 1's ready flag, gives
up after its limit (1 s), sets the cross-GPU flag timeout bit (value 16) and
returns; the context stays usable (a clean call and a forward run after it).
"""
import ctypes
import time

import pytest
import torch

from mlp_megakernel_b200 import _lib, fused_mlp_fwd
from mlp_megakernel_b200.dp import _DevicePtr
from mlp_megakernel_b200.synthetic import make_inputs

pytestmark = pytest.mark.gpu

DEV_TIMEOUT_FLAG = 16  # MLPK_DEVST_TIMEOUT_FLAG in include/mlpk.h


def _alloc(lib, n):
    buf = ctypes.c_void_p()
    handle = (ctypes.c_uint8 * _lib.PEER_HANDLE_BYTES)()
    _lib.check("mlpk_peer_alloc", lib.mlpk_peer_alloc(n, ctypes.byref(buf), handle))
    return buf.value


def test_peer_wait_expires_reports_and_recovers(built_lib):
    lib = _lib.lib()
    torch.cuda.set_device(0)
    n = 1024  # one CTA
    own, silent = _alloc(lib, n), _alloc(lib, n)
    try:
        dev = torch.device("cuda", 0)
        own_t = torch.as_tensor(_DevicePtr(own, n), device=dev)
        own_t.copy_(torch.arange(n, dtype=torch.float32, device=dev))
        out = torch.zeros(n, dtype=torch.float32, device=dev)
        stream = torch.cuda.current_stream().cuda_stream
        torch.cuda.synchronize()
        _lib.device_status(clear=True)

        t0 = time.perf_counter()
        rc = lib.mlpk_peer_allreduce(_lib.ptr_array([own, silent]), 2, 0, n, out.data_ptr(), stream)
        _lib.check("mlpk_peer_allreduce", rc)
        torch.cuda.synchronize()
        waited = time.perf_counter() - t0
        status = _lib.device_status(clear=True)
        assert status & DEV_TIMEOUT_FLAG, f"expected the cross-GPU timeout bit, status {status}"
        assert 0.5 <= waited < 30.0, waited  # the 1 s limit, not a hang
        assert _lib.device_status() == 0  # cleared

        # the context is usable: a clean one-rank sum and a forward
        rc = lib.mlpk_peer_allreduce(_lib.ptr_array([own]), 1, 0, n, out.data_ptr(), stream)
        _lib.check("mlpk_peer_allreduce", rc)
        torch.cuda.synchronize()
        assert torch.equal(out, own_t)
        x, ws = make_inputs("3L128", 300)
        y = fused_mlp_fwd(x.cuda(), *[w.cuda() for w in ws])
        torch.cuda.synchronize()
        assert torch.isfinite(y.float()).all()
        assert _lib.device_status() == 0
    finally:
        torch.cuda.synchronize()
        lib.mlpk_peer_free(ctypes.c_void_p(own))
        lib.mlpk_peer_free(ctypes.c_void_p(silent))
