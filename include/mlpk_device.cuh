/*
 * mlpk device API -- the fused softplus MLP as a device-side object that a
 * user's own sm_100a kernel calls on rows it holds in registers, so that the
 * work before the MLP (an input encoding) and after it (a loss, a reduction)
 * stay in the same kernel.  No counterpart in the reference's code: its
 * design notes name it as the next step (mlp_fused.md:406, "device-side MLP
 * callable from user kernels").  Header-only; compile with
 * -gencode arch=compute_100a,code=sm_100a -std=c++17 --expt-relaxed-constexpr
 * and this repository's root on the include path.  See
 * mlpk::device::FusedMLP for the calling convention.
 */
#pragma once
#include "../mlp_megakernel_b200/csrc/device_mlp.cuh"
