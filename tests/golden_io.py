"""Load the golden fixtures and regenerate their inputs (digest-checked)."""
from __future__ import annotations

import glob
import hashlib
import os

import numpy as np

from tests.golden.cases import CASES, make_case_inputs

GOLDEN_DIR = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def case_names():
    return sorted(os.path.basename(p)[4:-4] for p in glob.glob(os.path.join(GOLDEN_DIR, "fwd_*.npz")))


def load_case(name):
    """(x fp16 [M,d0], ws fp16, rows, out_ref_kernel fp16[rows], record)."""
    rec = dict(np.load(os.path.join(GOLDEN_DIR, f"fwd_{name}.npz")))
    dims, M, dist, seed, scale, _sub = CASES[name]
    x, ws = make_case_inputs(dims, M, dist, seed, scale)
    xd = hashlib.sha256(x.numpy().tobytes()).hexdigest()
    wd = hashlib.sha256(b"".join(w.numpy().tobytes() for w in ws)).hexdigest()
    if xd != str(rec["x_sha256"]) or wd != str(rec["w_sha256"]):
        raise AssertionError(f"{name}: regenerated inputs do not match the fixture digests")
    return x, ws, rec["rows"], rec["out_ref_kernel"], rec
