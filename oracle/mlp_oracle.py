"""CPU restatement of the reference's fused softplus MLP -- TEST INFRASTRUCTURE.

This module is the parity checker.  It is imported only by ``tests/``,
``__graft_entry__.smoke()`` and the CPU legs of ``bench.py``; the product
package never imports it and has no CPU fallback.

What it restates (reference = Marcelo5444/mlp-megakernel):

* forward: ``Model.forward`` (kernel.py:163-171), i.e.
  ``h1 = softplus(x @ w1); h2 = softplus(h1 @ w2); out = h2 @ w3``, generalised
  to L layers (README.md:9 gives the 5-layer chain).  With ``round_h=True`` it
  also restates the fused kernel's operand casts: each hidden activation is
  rounded to fp16 before it feeds the next GEMM (kernel.py:110, kernel.py:117)
  and the output is rounded to the dtype of x (kernel.py:122, kernel.py:136).
* softplus: ``F.softplus`` with beta=1, threshold=20 (kernel.py:169-170), which
  the fused kernel writes as ``where(z > 20, z, log(exp(z) + 1))``
  (kernel.py:108, kernel.py:112).
* training forward: the forward plus the post-activation h_l saved in fp32
  (mlp_fused.md:52-61; README.md:30).
* backward: the closed forms of mlp_fused.md:80-95 --
  ``dz_l = (dz_{l+1} @ W_{l+1}^T) * (1 - exp(-h_l))``, ``dW_l = h_{l-1}^T @ dz_l``,
  ``dx = dz_1 @ W_1^T``.  The fused training kernels of the reference are not in
  its published tree (fused_mlp.py is absent), so the training path is pinned by
  these formulas and by ``torch.autograd`` (tests/test_oracle.py), not by
  reference code.
* weight norm: ``W = g * v / ||v||`` per output neuron (mlp_fused.md:466-480);
  with weights stored ``[in, out]`` that is per output column.  Backward:
  ``dg_j = <dW_:j, v_:j> / ||v_:j||``,
  ``dv_:j = (g_j / ||v_:j||) dW_:j - (g_j dg_j / ||v_:j||^2) v_:j``
  (mlp_fused.md:481-483 names the kernel; the formula is the chain rule).

All arithmetic is numpy float64 unless stated; inputs are taken as given
(callers pass the fp16-rounded tensors the GPU sees).
"""
from __future__ import annotations

import numpy as np

SOFTPLUS_THRESHOLD = 20.0  # F.softplus default, kernel.py:108


def _f64(a) -> np.ndarray:
    if hasattr(a, "detach"):  # torch tensor
        a = a.detach().cpu().float().numpy()
    return np.asarray(a, dtype=np.float64)


def _round_fp16(a: np.ndarray) -> np.ndarray:
    return a.astype(np.float16).astype(np.float64)


def softplus(z: np.ndarray) -> np.ndarray:
    """``where(z > 20, z, log1p(exp(z)))`` -- F.softplus(beta=1, threshold=20).

    Follows kernel.py:169-170 (``F.softplus``) and kernel.py:108.
    """
    z = np.asarray(z, dtype=np.float64)
    with np.errstate(over="ignore"):
        return np.where(z > SOFTPLUS_THRESHOLD, z, np.log1p(np.exp(np.minimum(z, SOFTPLUS_THRESHOLD))))


def mlp_forward(x, weights, round_h: bool = True, round_out: bool = True) -> np.ndarray:
    """L-layer softplus MLP forward; weights are ``[in, out]`` so ``x @ W``.

    Restates kernel.py:163-171 (``Model.forward``) for any depth.  With
    ``round_h`` each hidden activation is rounded to fp16 before the next GEMM,
    as the fused kernel does (kernel.py:110, kernel.py:117); with ``round_out``
    the result is rounded to fp16 (kernel.py:122).
    """
    h = _f64(x)
    ws = [_f64(w) for w in weights]
    for i, w in enumerate(ws):
        z = h @ w
        if i < len(ws) - 1:
            h = softplus(z)
            if round_h:
                h = _round_fp16(h)
        else:
            h = z
    return _round_fp16(h) if round_out else h


def mlp_forward_train(x, weights):
    """Forward that also returns the post-activation h_1..h_{L-1} (fp32 storage).

    Restates the training forward variant (mlp_fused.md:52-61): same chain as
    the inference forward, plus the stores of every hidden h in fp32.  The
    returned ``hs`` are the fp32 values (not fp16-rounded); the next GEMM still
    consumes the fp16 rounding of each h, as on the GPU.
    """
    h = _f64(x)
    ws = [_f64(w) for w in weights]
    hs = []
    for i, w in enumerate(ws):
        z = h @ w
        if i < len(ws) - 1:
            h32 = softplus(z).astype(np.float32).astype(np.float64)
            hs.append(h32)
            h = _round_fp16(h32)
        else:
            h = z
    return _round_fp16(h), hs


def mlp_backward(x, weights, hs, grad_out):
    """Closed-form backward (mlp_fused.md:80-95).

    ``hs`` are the saved fp32 activations.  GEMM operands are fp16-rounded as
    on the GPU (h and dz enter the tensor cores as fp16); everything else is
    float64.  Returns ``dx`` and the list of ``dW_l`` (float64).
    """
    ws = [_f64(w) for w in weights]
    L = len(ws)
    a_in = [_f64(x)] + [_round_fp16(_f64(h)) for h in hs]  # GEMM operands h_{l-1}
    dz = _f64(grad_out)
    dws = [None] * L
    for l in range(L - 1, -1, -1):
        dws[l] = a_in[l].T @ dz
        dh = dz @ ws[l].T
        if l > 0:
            h = _f64(hs[l - 1])
            dz = _round_fp16(dh * (1.0 - np.exp(-h)))
        else:
            dx = dh
    return dx, dws


def weight_norm_forward(v, g):
    """``W[:, j] = g[j] * v[:, j] / ||v[:, j]||`` for ``v`` of shape ``[in, out]``.

    Weight norm per output neuron (mlp_fused.md:466-480).  Returns (W, inv_norm).
    """
    v = _f64(v)
    g = _f64(g).reshape(-1)
    inv = 1.0 / np.sqrt((v * v).sum(axis=0))
    return v * (g * inv)[None, :], inv


def weight_norm_backward(v, g, dW):
    """(dv, dg) from dW for ``W = g * v / ||v||`` (chain rule; mlp_fused.md:481-483)."""
    v = _f64(v)
    g = _f64(g).reshape(-1)
    dW = _f64(dW)
    inv = 1.0 / np.sqrt((v * v).sum(axis=0))
    dg = (dW * v).sum(axis=0) * inv
    dv = dW * (g * inv)[None, :] - v * (g * dg * inv * inv)[None, :]
    return dv, dg
