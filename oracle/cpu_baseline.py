"""The reference's PyTorch path on the host CPU -- TEST/BENCH INFRASTRUCTURE.

A restatement of ``Model.forward`` (kernel.py:163-171; identical to
``pytorch_fwd`` at profile.py:282-286) generalised to L layers, in fp32 on
torch's CPU backend with every host thread.  It is the timed CPU baseline of
``bench.py`` (its ``cpu_baseline`` leg and ``--impl reference`` arm) and is
never part of the product path.  ``train_step`` is the same model's
forward+backward through torch.autograd (the reference's training formulas,
mlp_fused.md:80-95), for the fwd+bwd baseline.
"""
from __future__ import annotations

import os
import time

import torch
import torch.nn.functional as F


def set_all_threads() -> int:
    n = os.cpu_count() or 1
    torch.set_num_threads(n)
    return torch.get_num_threads()


def model_forward(x: torch.Tensor, weights) -> torch.Tensor:
    """kernel.py:163-171 for any depth: softplus between GEMMs, none after the last."""
    h = x
    for i, w in enumerate(weights):
        h = h @ w
        if i < len(weights) - 1:
            h = F.softplus(h)
    return h


def train_step(x: torch.Tensor, weights, grad_out: torch.Tensor):
    ws = [w.detach().requires_grad_(True) for w in weights]
    out = model_forward(x, ws)
    out.backward(grad_out)
    return out, [w.grad for w in ws]


def train_step_wn(x: torch.Tensor, vs, gs, grad_out: torch.Tensor):
    """One weight-normed training step: W_l = g_l v_l / ||v_l|| per output
    column (mlp_fused.md:466-480), the forward above, and torch.autograd back
    to dx and (dv_l, dg_l) for every layer."""
    x = x.detach().requires_grad_(True)
    vs = [v.detach().requires_grad_(True) for v in vs]
    gs = [g.detach().requires_grad_(True) for g in gs]
    ws = [g * v / v.norm(dim=0, keepdim=True) for v, g in zip(vs, gs)]
    out = model_forward(x, ws)
    out.backward(grad_out)
    return out, x.grad, [v.grad for v in vs], [g.grad for g in gs]


def time_rows_per_s(fn, rows_per_call: int, min_seconds: float = 10.0, max_calls: int = 1000):
    """Call fn() repeatedly for at least min_seconds; return rows/s and calls made."""
    fn()  # warm-up
    calls = 0
    t0 = time.perf_counter()
    while True:
        fn()
        calls += 1
        dt = time.perf_counter() - t0
        if dt >= min_seconds or calls >= max_calls:
            break
    return rows_per_call * calls / dt, calls, dt
