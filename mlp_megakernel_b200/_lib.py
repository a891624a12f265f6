"""ctypes binding of libmlpk.so (the C ABI declared in include/mlpk.h).

Loading the library needs no GPU; calling a compute entry point needs an
sm_100 device.  There is no fallback: if the library is missing, every op
raises.
"""
from __future__ import annotations

import ctypes
import os
import threading

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "lib", "libmlpk.so")
MAX_LAYERS = 8

MLPK_OK = 0
MLPK_ERR_CUDA = 4
STATUS_NAMES = {
    0: "MLPK_OK",
    1: "MLPK_ERR_SHAPE",
    2: "MLPK_ERR_UNSUPPORTED",
    3: "MLPK_ERR_ARCH",
    4: "MLPK_ERR_CUDA",
    5: "MLPK_ERR_ALIGN",
    6: "MLPK_ERR_NULL",
    7: "MLPK_ERR_DEVICE",
    8: "MLPK_ERR_SCRATCH",
}

# Every symbol declared in include/mlpk.h, with (restype, argtypes).
_vp = ctypes.c_void_p


class MlpkShape(ctypes.Structure):
    _fields_ = [("num_layers", ctypes.c_int32), ("dims", ctypes.c_int32 * (MAX_LAYERS + 1))]


_SHAPE_P = ctypes.POINTER(MlpkShape)
_VPP = ctypes.POINTER(ctypes.c_void_p)

SIGNATURES = {
    "mlpk_status_string": (ctypes.c_char_p, [ctypes.c_int]),
    "mlpk_shape_supported": (ctypes.c_int, [_SHAPE_P]),
    "mlpk_fwd": (ctypes.c_int, [_SHAPE_P, ctypes.c_int64, _vp, _VPP, _vp, _vp]),
    "mlpk_train_supported": (ctypes.c_int, [_SHAPE_P]),
    "mlpk_train_fwd": (ctypes.c_int, [_SHAPE_P, ctypes.c_int64, _vp, _VPP, _vp, _VPP, _vp]),
    "mlpk_train_supported_ex": (ctypes.c_int, [_SHAPE_P, ctypes.c_int]),
    "mlpk_shape_supported_ex": (ctypes.c_int, [_SHAPE_P, ctypes.c_int]),
    "mlpk_fwd_ex": (ctypes.c_int, [_SHAPE_P, ctypes.c_int64, _vp, _VPP, _vp, ctypes.c_int, _vp]),
    "mlpk_train_fwd_ex": (ctypes.c_int, [_SHAPE_P, ctypes.c_int64, _vp, _VPP, _vp, _VPP, ctypes.c_int, _vp]),
    "mlpk_bwd_workspace_size": (ctypes.c_int64, [_SHAPE_P, ctypes.c_int64]),
    "mlpk_bwd": (ctypes.c_int, [_SHAPE_P, ctypes.c_int64, _vp, _VPP, _VPP, _vp, _vp, _vp,
                                ctypes.c_int64, _vp, _vp]),
    "mlpk_bwd_ex": (ctypes.c_int, [_SHAPE_P, ctypes.c_int64, _vp, _VPP, _VPP, ctypes.c_int, _vp, _vp, _vp,
                                   ctypes.c_int64, _vp, _vp]),
    "mlpk_bwd_noalloc": (ctypes.c_int, [_SHAPE_P, ctypes.c_int64, _vp, _VPP, _VPP, _vp, _vp, _vp,
                                        _vp]),
    "mlpk_wn_fwd": (ctypes.c_int, [_SHAPE_P, _vp, _vp, _VPP, _vp, _vp]),
    "mlpk_wn_bwd": (ctypes.c_int, [_SHAPE_P, _vp, _vp, _vp, _vp, _vp, _vp, _vp]),
    "mlpk_device_status": (ctypes.c_int, [ctypes.c_int, ctypes.POINTER(ctypes.c_int)]),
    "mlpk_last_cuda_error": (ctypes.c_char_p, []),
    "mlpk_cast_f32_f16": (ctypes.c_int, [_vp, _vp, ctypes.c_int64, _vp]),
    "mlpk_cast_f16_f32": (ctypes.c_int, [_vp, _vp, ctypes.c_int64, _vp]),
    "mlpk_peer_alloc": (ctypes.c_int, [ctypes.c_int64, ctypes.POINTER(ctypes.c_void_p), ctypes.c_void_p]),
    "mlpk_peer_open": (ctypes.c_int, [ctypes.c_void_p, ctypes.POINTER(ctypes.c_void_p)]),
    "mlpk_peer_close": (ctypes.c_int, [ctypes.c_void_p]),
    "mlpk_peer_free": (ctypes.c_int, [ctypes.c_void_p]),
    "mlpk_peer_allreduce": (ctypes.c_int, [_VPP, ctypes.c_int, ctypes.c_int, ctypes.c_int64, _vp, _vp]),
    "mlpk_fwd_host_workspace_size": (ctypes.c_int64, [_SHAPE_P, ctypes.c_int64]),
    "mlpk_fwd_host": (ctypes.c_int, [_SHAPE_P, ctypes.c_int64, _vp, _VPP, _vp, ctypes.c_int64, _vp,
                                     ctypes.c_int64, _vp]),
}
FWD_HOST_CHUNK_ROWS = 131072
H_F16 = 0  # MLPK_H_F16: saved activations in fp16
H_F32 = 1  # MLPK_H_F32: saved activations in fp32 (the reference's storage)
DT_F16 = 0  # MLPK_DT_F16: fp16 operands
DT_F32 = 1  # MLPK_DT_F32: fp32 operands on tf32 tensor cores
PEER_HANDLE_BYTES = 64
PEER_MAX_RANKS = 8

_lock = threading.Lock()
_lib = None


class MlpkError(RuntimeError):
    """Raised when a libmlpk entry point returns a non-zero status."""

    def __init__(self, fn: str, status: int):
        self.status = status
        name = STATUS_NAMES.get(status, str(status))
        msg = f"{fn} failed: {name} ({status_string(status)})"
        if status == MLPK_ERR_CUDA:
            msg += f": {lib().mlpk_last_cuda_error().decode()}"
        super().__init__(msg)


def lib() -> ctypes.CDLL:
    """Load libmlpk.so once; raise if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise RuntimeError(
                    f"{LIB_PATH} not found: build it with `python -m mlp_megakernel_b200.build` "
                    "(there is no CPU fallback)"
                )
            handle = ctypes.CDLL(LIB_PATH)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(handle, name)
                fn.restype = res
                fn.argtypes = args
            _lib = handle
    return _lib


def status_string(status: int) -> str:
    return lib().mlpk_status_string(status).decode()


def check(fn: str, status: int) -> None:
    if status != MLPK_OK:
        raise MlpkError(fn, status)


_shape_cache: dict = {}


def shape_struct(dims) -> MlpkShape:
    dims = tuple(int(d) for d in dims)
    s = _shape_cache.get(dims)
    if s is None:
        if len(dims) < 2 or len(dims) - 1 > MAX_LAYERS:
            raise ValueError(f"unsupported number of layers: {len(dims) - 1}")
        s = MlpkShape()
        s.num_layers = len(dims) - 1
        for i, d in enumerate(dims):
            s.dims[i] = d
        _shape_cache[dims] = s
    return s


def shape_supported(dims) -> bool:
    return bool(lib().mlpk_shape_supported(ctypes.byref(shape_struct(dims))))


def train_supported(dims, h_dtype: int = H_F16) -> bool:
    return bool(lib().mlpk_train_supported_ex(ctypes.byref(shape_struct(dims)), h_dtype))


def ptr_array(ptrs) -> ctypes.Array:
    arr = (ctypes.c_void_p * len(ptrs))()
    for i, p in enumerate(ptrs):
        arr[i] = p
    return arr


def device_status(clear: bool = False) -> int:
    """Device-side status word of the current device (synchronises)."""
    v = ctypes.c_int(0)
    check("mlpk_device_status", lib().mlpk_device_status(int(clear), ctypes.byref(v)))
    return v.value
