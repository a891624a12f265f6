"""Generate the golden forward vectors from the REFERENCE's own fused kernel.

Runs the reference's Triton megakernel ``_fused_mlp_fwd`` (kernel.py:130-156,
kernel.py:60-123) on the CPU through Triton's interpreter
(``TRITON_INTERPRET=1``), on seeded fp16 inputs, and records inputs and
outputs as ``.npz`` fixtures.  The reference reads the SM count of device 0
at import (kernel.py:18); with no GPU in this container that query is answered
with 148 (a B200's SM count) -- it only sizes the persistent grid, not the
arithmetic.

Needs the reference checkout (default /root/reference, or $MLPK_REFERENCE)
and only ever runs in the development container; the GPU box and the tests
use the committed fixtures.  Usage:

    python tests/golden/make_golden.py
"""
from __future__ import annotations

import hashlib
import importlib.util
import os
import sys

import numpy as np

os.environ["TRITON_INTERPRET"] = "1"

import torch  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from tests.golden.cases import CASES, make_case_inputs  # noqa: E402

REF = os.environ.get("MLPK_REFERENCE", "/root/reference")


class _Props:
    multi_processor_count = 148
    name = "interpreter"


def load_reference():
    torch.cuda.get_device_properties = lambda *_a, **_k: _Props()
    spec = importlib.util.spec_from_file_location("ref_kernel", os.path.join(REF, "kernel.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def make_case(mod, dims, M, dist, seed, scale):
    x, ws = make_case_inputs(dims, M, dist, seed, scale)
    out = mod._fused_mlp_fwd(x, *ws)
    ref32 = mod.Model()(x.float(), *[w.float() for w in ws])  # kernel.py:163-171 in fp32
    return x, ws, out, ref32


def main():
    mod = load_reference()
    for f in os.listdir(HERE):
        if f.startswith("fwd_") and f.endswith(".npz"):
            os.remove(os.path.join(HERE, f))
    for name, (dims, M, dist, seed, scale, sub) in CASES.items():
        x, ws, out, ref32 = make_case(mod, dims, M, dist, seed, scale)
        rec = {
            "dims": np.array(dims, dtype=np.int32),
            "M": np.int64(M),
            "x_dist": dist,
            "x_seed": np.int64(seed),
            "w_scale": np.float64(-1.0 if scale is None else scale),
            # inputs are regenerated from their seeds by the tests and checked
            # against these digests, so only the outputs are stored
            "x_sha256": hashlib.sha256(x.numpy().tobytes()).hexdigest(),
            "w_sha256": hashlib.sha256(b"".join(w.numpy().tobytes() for w in ws)).hexdigest(),
            "max_abs_kernel_vs_model_fp32": np.float64((out.float() - ref32).abs().max().item()),
        }
        if sub:
            rows = np.unique(np.concatenate([np.arange(0, 64), np.arange(M - 64, M),
                                             np.arange(0, M, M // sub)]))
        else:
            rows = np.arange(M)
        rec["rows"] = rows.astype(np.int64)
        rec["out_ref_kernel"] = out.numpy()[rows]
        path = os.path.join(HERE, f"fwd_{name}.npz")
        np.savez_compressed(path, **rec)
        d = (out.float() - ref32).abs().max().item()
        print(f"{name}: M={M} dims={dims} |kernel-Model| max {d:.3e} "
              f"max|ref| {ref32.abs().max().item():.3f} -> {os.path.getsize(path)} bytes")


if __name__ == "__main__":
    main()
