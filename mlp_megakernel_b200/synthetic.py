"""Seeded synthetic inputs for the benchmark configurations.

The reference measures on random tensors only (profile.py:307-310); the
configurations this library is benchmarked on are:

* ``3L128``  -- 128 -> 128 -> 128 -> 128, x ~ N(0, 1) (seed 0),
  W_i ~ U(+-1/sqrt(in)) (seed 1, drawn in layer order), grad_out ~ N(0, 1) (seed 2);
* ``5L``     -- 32 -> 64 -> 64 -> 64 -> 64 -> 16, x ~ U(-1, 1) (seed 3), W seed 1,
  grad_out seed 2;
* ``W256``   -- 256 -> 256 -> 256 -> 256, x ~ N(0, 1) (seed 4), W seed 1,
  grad_out seed 2.

Values are drawn in fp32 from ``torch.Generator(device)`` and rounded to fp16.
On CPU the bytes are reproducible across runs, so the CPU oracle and the GPU
see identical inputs; large benchmark inputs are drawn on the GPU with the
same distributions.
"""
from __future__ import annotations

import math

import torch

CONFIGS = {
    "3L128": {"dims": (128, 128, 128, 128), "x_dist": "normal", "x_seed": 0},
    "5L": {"dims": (32, 64, 64, 64, 64, 16), "x_dist": "uniform", "x_seed": 3},
    "W256": {"dims": (256, 256, 256, 256), "x_dist": "normal", "x_seed": 4},
}
W_SEED = 1
GRAD_SEED = 2


def _gen(seed: int, device) -> torch.Generator:
    g = torch.Generator(device=torch.device(device))
    g.manual_seed(seed)
    return g


def make_weights(dims, seed: int = W_SEED, device="cpu", dtype=torch.float16):
    """W_i ~ U(-1/sqrt(in), 1/sqrt(in)), shape [in, out], drawn in layer order."""
    g = _gen(seed, device)
    ws = []
    for i, o in zip(dims[:-1], dims[1:]):
        w = (torch.rand(i, o, generator=g, device=device) * 2 - 1) / math.sqrt(i)
        ws.append(w.to(dtype))
    return ws


def make_x(M: int, d0: int, dist: str = "normal", seed: int = 0, device="cpu",
           dtype=torch.float16):
    g = _gen(seed, device)
    if dist == "normal":
        x = torch.randn(M, d0, generator=g, device=device)
    elif dist == "uniform":
        x = torch.rand(M, d0, generator=g, device=device) * 2 - 1
    else:
        raise ValueError(dist)
    return x.to(dtype)


def make_grad(M: int, dL: int, seed: int = GRAD_SEED, device="cpu", dtype=torch.float16):
    g = _gen(seed, device)
    return torch.randn(M, dL, generator=g, device=device).to(dtype)


def make_inputs(config: str, M: int, device="cpu", with_grad: bool = False):
    """(x, weights[, grad_out]) for a named configuration."""
    c = CONFIGS[config]
    dims = c["dims"]
    x = make_x(M, dims[0], c["x_dist"], c["x_seed"], device)
    ws = make_weights(dims, W_SEED, device)
    if with_grad:
        return x, ws, make_grad(M, dims[-1], GRAD_SEED, device)
    return x, ws


def weight_norm_init(ws):
    """(v, g) with v = W (fp32) and g = ||v|| per output column, so g*v/||v|| == W."""
    vs = [w.float().clone() for w in ws]
    gs = [v.norm(dim=0) for v in vs]
    return vs, gs
