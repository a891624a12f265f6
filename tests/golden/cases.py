"""Golden forward cases: names, seeds and input regeneration.

The fixtures ``fwd_<name>.npz`` hold the outputs of the REFERENCE's own fused
kernel on these inputs (made by make_golden.py); tests regenerate the inputs
from the seeds below and check them against the recorded SHA-256 digests.
"""
from __future__ import annotations

import torch

from mlp_megakernel_b200.synthetic import make_weights, make_x


# name -> (dims, M, x_dist, x_seed, weight scale, subsample_rows)
CASES = {
    # 3L128 forward at M=4096, x~N(0,1) seed 0, W~U(+-1/sqrt(in)) seed 1.
    "cfg1_3L128_M4096": ((128, 128, 128, 128), 4096, "normal", 0, 1.0, 256),
    # ragged batch sizes (tile = 128 rows): M=1, 127, 129, 300
    "ragged_M1": ((128, 128, 128, 128), 1, "normal", 10, 1.0, 0),
    "ragged_M127": ((128, 128, 128, 128), 127, "normal", 11, 1.0, 0),
    "ragged_M129": ((128, 128, 128, 128), 129, "normal", 12, 1.0, 0),
    "ragged_M300": ((128, 128, 128, 128), 300, "normal", 13, 1.0, 0),
    # large |pre-activation|: weights x12 push z past the threshold (z > 20)
    # and far below zero (softplus underflow side)
    "large_preact_M256": ((128, 128, 128, 128), 256, "normal", 14, 12.0, 0),
    # the reference's own benchmark distribution: x, W ~ 0.02*N(0,1) (profile.py:307-310)
    "profile_dist_M512": ((128, 128, 128, 128), 512, "normal", 15, None, 0),
    # wide 3-layer network D=H=OUT=256 (BASELINE config 5 shape), x seed 4
    "w256_M384": ((256, 256, 256, 256), 384, "normal", 4, 1.0, 0),
    # narrow 3-layer network D=H=OUT=64
    "d64_M200": ((64, 64, 64, 64), 200, "normal", 16, 1.0, 0),
    # mixed widths the reference's tiles accept (kernel.py:25-53: BK1 =
    # min(64, K1), BK2 = min(128, N1), BK3 = min(128, N2), BN3 = min(128, N3)
    # dividing their dims); served here by a larger compiled network
    "mixed_32_128_64_16_M300": ((32, 128, 64, 16), 300, "normal", 17, 1.0, 0),
    "mixed_128_64_32_128_M200": ((128, 64, 32, 128), 200, "normal", 18, 1.0, 0),
    "mixed_16_32_64_32_M129": ((16, 32, 64, 32), 129, "normal", 19, 1.0, 0),
    "mixed_192_256_128_256_M130": ((192, 256, 128, 256), 130, "normal", 20, 1.0, 0),
}


def make_case_inputs(dims, M, dist, seed, scale):
    """Regenerate a case's fp16 inputs from its seeds (used by the tests too)."""
    x = make_x(M, dims[0], dist, seed)
    if scale is None:  # profile.py:307-310 distribution
        g = torch.Generator().manual_seed(seed + 1000)
        x = (torch.randn(M, dims[0], generator=g) * 0.02).half()
        ws = [(torch.randn(i, o, generator=g) * 0.02).half() for i, o in zip(dims[:-1], dims[1:])]
    else:
        ws = [(w.float() * scale).half() for w in make_weights(dims)]
    return x, ws


# Training cases (fixtures ``train_<name>.npz``): BASELINE config 3 -- 3L128
# with weight norm W_l = g_l v_l / ||v_l|| (per output column), v_l ~
# U(+-1/sqrt(in)) seed 1 (the fp16 weights of make_weights, widened), g_l =
# ||v_l||, x ~ N(0,1) seed 0, grad_out ~ N(0,1) seed 2, fp16 inputs.
# name -> (dims, M, rows recorded for out / dx (0 = all))
TRAIN_CASES = {
    "cfg3_M16384": ((128, 128, 128, 128), 16384, 512),
    "cfg3_M262144": ((128, 128, 128, 128), 262144, 512),
}


def make_train_inputs(dims, M):
    """(x fp16, grad_out fp16, v fp32 list, g fp32 list) of a training case."""
    from mlp_megakernel_b200.synthetic import make_grad

    x = make_x(M, dims[0], "normal", 0)
    grad = make_grad(M, dims[-1], seed=2)
    vs = [w.float() for w in make_weights(dims)]
    gs = [v.norm(dim=0) for v in vs]
    return x, grad, vs, gs


def train_rows(M, n):
    """The recorded row subsample of a training case: the first and last 64
    rows and an even stride over the batch."""
    import numpy as np

    if n == 0 or n >= M:
        return np.arange(M)
    return np.unique(np.concatenate([np.arange(0, 64), np.arange(M - 64, M),
                                     np.arange(0, M, max(1, M // n))])).astype(np.int64)
