"""CPU oracle for the fused softplus MLP (test infrastructure only).

This package is the checker, never the product: only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline / reference arm may
import it.  The product path (``mlp_megakernel_b200``) never imports it and has
no CPU fallback.
"""
from .mlp_oracle import (  # noqa: F401
    softplus,
    mlp_forward,
    mlp_forward_train,
    mlp_backward,
    weight_norm_forward,
    weight_norm_backward,
)
