"""mlp_megakernel_b200 -- B200-native (sm_100a) fused softplus MLP.

Drop-in for the fused-MLP path of Marcelo5444/mlp-megakernel: the functional
forward ``_fused_mlp_fwd`` / ``ModelNew`` (kernel.py:130-180) and the module API
``FusedMLPSoftplus`` / ``FusedMLPSoftplusWN`` (README.md:58-70).  All compute
runs in hand-written CUDA kernels (libmlpk.so, C ABI in include/mlpk.h).
"""
from .functional import ModelNew, _fused_mlp_fwd, fused_mlp_fwd, fused_mlp_fwd_host  # noqa: F401
from .modules import FusedMLPSoftplus, FusedMLPSoftplusWN  # noqa: F401

__all__ = ["fused_mlp_fwd", "fused_mlp_fwd_host", "_fused_mlp_fwd", "ModelNew", "FusedMLPSoftplus",
           "FusedMLPSoftplusWN"]
