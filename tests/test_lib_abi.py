"""CPU tests of the C ABI: libmlpk.so builds, loads without a GPU, exports
every function declared in include/mlpk.h, and validates arguments before it
touches the device."""
import ctypes
import os
import re

import pytest

from mlp_megakernel_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared_functions():
    names = []
    for hdr in sorted(os.listdir(os.path.join(ROOT, "include"))):
        if hdr.endswith(".h"):
            txt = open(os.path.join(ROOT, "include", hdr)).read()
            txt = re.sub(r"/\*.*?\*/", "", txt, flags=re.S)
            names += re.findall(r"\b(mlpk_[a-z0-9_]+)\s*\(", txt)
    return sorted(set(names))


def test_header_declares_entry_points():
    names = _declared_functions()
    assert "mlpk_fwd" in names and "mlpk_status_string" in names


def test_library_exports_every_declared_symbol(built_lib):
    for name in _declared_functions():
        assert hasattr(built_lib, name), f"libmlpk.so does not export {name}"
        assert name in _lib.SIGNATURES, f"{name} has no ctypes signature in _lib.SIGNATURES"


def test_status_strings(built_lib):
    assert _lib.status_string(0) == "ok"
    for code in range(1, 9):
        assert _lib.status_string(code) != "unknown status"


@pytest.mark.parametrize("dims,ok", [
    ((128, 128, 128, 128), True),
    ((32, 64, 64, 64, 64, 16), True),
    ((64, 64, 64, 64), True),
    ((256, 256, 256, 256), True),
    # served by a larger compiled network: widths multiples of 8, at most the
    # compiled widths of the same depth, hidden widths free
    ((128, 96, 128, 128), True),
    ((8, 8, 8, 8), True),
    ((200, 136, 256, 72), True),
    ((16, 32, 48, 64, 40, 8), True),
    ((64, 64, 64, 64, 64, 64), True),
    ((96, 128, 64, 128, 112, 16), True),
    ((256, 256, 256, 256, 256, 256), True),
    # not served
    ((128, 100, 128, 128), False),   # 100 is not a multiple of 8
    ((264, 256, 256, 256), False),   # wider than every 3-layer kernel
    ((64, 64, 64, 64, 64, 264), False),  # wider than every 5-layer kernel
    # 2 and 4 layers (one and three hidden layers)
    ((64, 64, 64), True),
    ((128, 96, 16), True),
    ((256, 256, 256), True),
    ((64, 64, 64, 64, 64), True),
    ((200, 128, 64, 256, 8), True),
    # 6 to 8 layers (MLPK_MAX_LAYERS): uniform 64 (6, 7 layers), 128 and 256
    # wide compiled; 64-wide 8-layer networks run on the 128-wide kernels
    ((64, 64, 64, 64, 64, 64, 64), True),
    ((32, 64, 16, 64, 48, 64, 8), True),
    ((64,) * 8, True),
    ((64,) * 9, True),
    ((128,) * 7, True),
    ((96, 128, 128, 64, 128, 128, 128, 128, 24), True),
    ((256,) * 9, True),
    ((200, 256, 8, 256, 64, 256, 256), True),
    ((264,) * 7, False),
    ((128, 128), False),
])
def test_shape_supported(built_lib, dims, ok):
    assert _lib.shape_supported(dims) == ok
    assert _lib.train_supported(dims) == ok


def test_depth_beyond_max_layers_rejected(built_lib):
    """9 layers is more than MLPK_MAX_LAYERS: the C ABI reports no kernel and
    the Python binding refuses to build the shape."""
    s = _lib.MlpkShape()
    s.num_layers = 9
    assert built_lib.mlpk_shape_supported(ctypes.byref(s)) == 0
    with pytest.raises(ValueError):
        _lib.shape_struct((64,) * 10)


def test_fwd_rejects_bad_arguments_without_touching_the_device(built_lib):
    lib = built_lib
    shape = _lib.shape_struct((128, 128, 128, 128))
    w = _lib.ptr_array([256, 512, 768])
    # NULL shape
    assert lib.mlpk_fwd(None, 16, 256, w, 512, None) == 6
    # negative M
    assert lib.mlpk_fwd(ctypes.byref(shape), -1, 256, w, 512, None) == 1
    # NULL weight pointer
    wn = _lib.ptr_array([256, 0, 768])
    assert lib.mlpk_fwd(ctypes.byref(shape), 16, 256, wn, 512, None) == 6
    # misaligned x
    assert lib.mlpk_fwd(ctypes.byref(shape), 16, 258, w, 512, None) == 5
    # unsupported shape
    bad = _lib.MlpkShape()
    bad.num_layers = 3
    for i, d in enumerate((128, 100, 128, 128)):
        bad.dims[i] = d
    assert lib.mlpk_fwd(ctypes.byref(bad), 16, 256, w, 512, None) == 2
    # zero layers
    z = _lib.MlpkShape()
    z.num_layers = 0
    assert lib.mlpk_fwd(ctypes.byref(z), 16, 256, w, 512, None) == 1


def test_fwd_host_rejects_bad_arguments_without_touching_the_device(built_lib):
    lib = built_lib
    shape = _lib.shape_struct((128, 128, 128, 128))
    w = _lib.ptr_array([256, 512, 768])
    assert lib.mlpk_fwd_host_workspace_size(ctypes.byref(shape), -1) == -1
    ws0 = lib.mlpk_fwd_host_workspace_size(ctypes.byref(shape), 0)
    assert ws0 == lib.mlpk_fwd_host_workspace_size(ctypes.byref(shape), _lib.FWD_HOST_CHUNK_ROWS)
    assert ws0 == 3 * 2 * _lib.FWD_HOST_CHUNK_ROWS * 128 * 2  # x and out buffers, 3 of each
    # NULL shape, negative M / chunk, NULL weight, unsupported shape, M = 0
    assert lib.mlpk_fwd_host(None, 16, 256, w, 512, 0, 1024, ws0, None) == 6
    assert lib.mlpk_fwd_host(ctypes.byref(shape), -1, 256, w, 512, 0, 1024, ws0, None) == 1
    assert lib.mlpk_fwd_host(ctypes.byref(shape), 16, 256, w, 512, -5, 1024, ws0, None) == 1
    assert lib.mlpk_fwd_host(ctypes.byref(shape), 16, 256, _lib.ptr_array([256, 0, 768]), 512, 0,
                             1024, ws0, None) == 6
    bad = _lib.shape_struct((128, 100, 128, 128))
    assert lib.mlpk_fwd_host(ctypes.byref(bad), 16, 256, w, 512, 0, 1024, ws0, None) == 2
    assert lib.mlpk_fwd_host(ctypes.byref(shape), 0, None, w, None, 0, None, 0, None) == 0
    # too small a workspace
    assert lib.mlpk_fwd_host(ctypes.byref(shape), 16, 256, w, 512, 0, 1024, ws0 - 1, None) == 1
