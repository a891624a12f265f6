"""Generate the golden forward vectors from the REFERENCE's own fused kernel.

Runs the reference's Triton megakernel ``_fused_mlp_fwd`` (kernel.py:130-156,
kernel.py:60-123) on the CPU through Triton's interpreter
(``TRITON_INTERPRET=1``), on seeded fp16 inputs, and records inputs and
outputs as ``.npz`` fixtures.  The reference reads the SM count of device 0
at import (kernel.py:18); with no GPU in this container that query is answered
with 148 (a B200's SM count) -- it only sizes the persistent grid, not the
arithmetic.

It also records TRAINING fixtures from the reference's own PyTorch model:
``Model`` (kernel.py:163-171) imported from the reference, fed the effective
weights of an explicit weight norm W_l = g_l v_l / ||v_l|| (per output column,
the weight norm of mlp_fused.md:466-480), run in fp32 on the CPU and
differentiated by torch.autograd: out and dx on a row subsample, the full
gradients of the effective weights dW_l and of the weight-norm parameters
dv_l, dg_l (BASELINE config 3 at M = 16,384 and 262,144).

Needs the reference checkout at $MLPK_REFERENCE (a directory holding its
kernel.py) and only ever runs in the development container; the GPU box and
the tests use the committed fixtures.  Usage:

    MLPK_REFERENCE=<reference checkout> python tests/golden/make_golden.py [--train-only]
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

from tests.golden.cases import CASES, TRAIN_CASES, make_case_inputs, make_train_inputs, train_rows  # noqa: E402

REF = os.environ.get("MLPK_REFERENCE")


class _Props:
    multi_processor_count = 148
    name = "interpreter"


def load_reference():
    if not REF or not os.path.exists(os.path.join(REF, "kernel.py")):
        raise SystemExit("set MLPK_REFERENCE to the reference checkout (the directory holding kernel.py)")
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


def _digest(*ts) -> str:
    return hashlib.sha256(b"".join(t.contiguous().numpy().tobytes() for t in ts)).hexdigest()


def make_train_case(mod, name, dims, M, nrows):
    """Reference Model (kernel.py:163-171) on weight-normed weights, fp32,
    torch.autograd; records the gradients the training kernels must match."""
    x16, g16, vs, gs = make_train_inputs(dims, M)
    x = x16.float().requires_grad_(True)
    vs = [v.clone().requires_grad_(True) for v in vs]
    gs = [g.clone().requires_grad_(True) for g in gs]
    ws = [g * v / v.norm(dim=0, keepdim=True) for v, g in zip(vs, gs)]
    for w in ws:
        w.retain_grad()
    out = mod.Model()(x, *ws)
    out.backward(g16.float())
    rows = train_rows(M, nrows)
    rec = {
        "dims": np.array(dims, dtype=np.int32),
        "M": np.int64(M),
        "x_sha256": _digest(x16),
        "grad_sha256": _digest(g16),
        "v_sha256": _digest(*[v.detach() for v in vs]),
        "rows": rows,
        "out_ref": out.detach().numpy()[rows],
        "dx_ref": x.grad.numpy()[rows],
        "dw_ref": np.concatenate([w.grad.reshape(-1).numpy() for w in ws]),
        "dv_ref": np.concatenate([v.grad.reshape(-1).numpy() for v in vs]),
        "dg_ref": np.concatenate([g.grad.numpy() for g in gs]),
    }
    path = os.path.join(HERE, f"train_{name}.npz")
    np.savez_compressed(path, **rec)
    print(f"train {name}: M={M} dims={dims} |dv| {np.linalg.norm(rec['dv_ref']):.4e} "
          f"-> {os.path.getsize(path)} bytes")


def main():
    mod = load_reference()
    for name, (dims, M, nrows) in TRAIN_CASES.items():
        make_train_case(mod, name, dims, M, nrows)
    if "--train-only" in sys.argv[1:]:
        return
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
