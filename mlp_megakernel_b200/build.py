"""Build libmlpk.so (the C-ABI CUDA library) in-tree for sm_100a.

Usage: ``python -m mlp_megakernel_b200.build`` (or ``__graft_entry__.build()``).
The library is written next to this file as ``lib/libmlpk.so`` so it travels
with the source tree; nothing is installed into site-packages.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
LIBDIR = os.path.join(HERE, "lib")
LIB = os.path.join(LIBDIR, "libmlpk.so")

SOURCES = ["mlpk_api.cu"]
DEPS = ["ptx.cuh", "layout.cuh", "softplus.cuh", "fwd_kernel.cuh",
        "bwd_kernel.cuh", "wn_kernel.cuh", "stream_kernel.cuh", "wgrad_kernel.cuh", "peer_kernel.cuh", "cast_kernel.cuh"]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "--expt-relaxed-constexpr",
    "-Xcompiler", "-fPIC", "-shared",
    "-diag-suppress", "20013",
]


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found; the CUDA library cannot be built")


def _stale() -> bool:
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    files = [os.path.join(CSRC, f) for f in SOURCES + DEPS]
    files.append(os.path.join(ROOT, "include", "mlpk.h"))
    files.append(os.path.abspath(__file__))
    return any(os.path.getmtime(f) > t for f in files if os.path.exists(f))


DEVTEST_SRC = os.path.join(ROOT, "tests", "device_api", "devtest.cu")
DEVTEST_LIB = os.path.join(ROOT, "tests", "device_api", "libmlpk_devtest.so")


def build_devtest(force: bool = False, verbose: bool = False) -> str:
    """Compile the device-API test kernels (tests/device_api/devtest.cu, a
    user kernel calling include/mlpk_device.cuh) if missing or stale."""
    deps = [DEVTEST_SRC, os.path.join(ROOT, "include", "mlpk_device.cuh")] + \
        [os.path.join(CSRC, f) for f in DEPS + ["device_mlp.cuh"]]
    if not force and os.path.exists(DEVTEST_LIB) and \
            all(os.path.getmtime(f) <= os.path.getmtime(DEVTEST_LIB) for f in deps if os.path.exists(f)):
        return DEVTEST_LIB
    tmp = DEVTEST_LIB + ".tmp"
    cmd = [nvcc_path(), *NVCC_FLAGS, "-o", tmp, DEVTEST_SRC]
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError("nvcc failed:\n" + res.stdout + res.stderr)
    os.replace(tmp, DEVTEST_LIB)
    return DEVTEST_LIB


def build(force: bool = False, verbose: bool = False, ptxas_info: bool = False) -> str:
    """Compile libmlpk.so if missing or older than its sources; return its path."""
    if not force and not _stale():
        return LIB
    os.makedirs(LIBDIR, exist_ok=True)
    tmp = LIB + ".tmp"
    cmd = [nvcc_path(), *NVCC_FLAGS]
    if ptxas_info:
        cmd += ["-Xptxas", "-v"]
    cmd += ["-o", tmp] + [os.path.join(CSRC, s) for s in SOURCES]
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError("nvcc failed:\n" + res.stdout + res.stderr)
    if verbose or ptxas_info:
        sys.stderr.write(res.stdout + res.stderr)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True, ptxas_info="-v" in sys.argv))
