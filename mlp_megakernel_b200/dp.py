"""Data-parallel plumbing for the fused MLP (one process per GPU).

The rows of a batch are independent, so the path shards by rows:

* inference: rank r runs the forward on its own rows; there is no collective;
* training: every rank runs the training forward and the fused backward on its
  rows, then the fp32 weight gradients (one flat buffer, every layer's dW back
  to back) are summed over ranks with ONE all-reduce, and the weight-norm
  backward runs replicated, so every rank holds identical dv / dg.

The split of a global batch follows the reference's benchmark recipe: rank r
of W takes rows ``[r*M/W, (r+1)*M/W)`` (integer division spreads a remainder
over the ranks).  ``torch.distributed`` supplies the process group: NCCL on the
GPUs, gloo in the CPU tests of this host logic.
"""
from __future__ import annotations

import torch


def shard_rows(M: int, rank: int, world: int) -> tuple[int, int]:
    """Half-open row range ``[start, stop)`` of rank ``rank`` out of ``world``."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} out of range for world size {world}")
    if M < 0:
        raise ValueError("M must be >= 0")
    return rank * M // world, (rank + 1) * M // world


def allreduce_weight_grads(dw: torch.Tensor, process_group=None) -> torch.Tensor:
    """Sum the flat fp32 weight gradients over the ranks of ``process_group``, in
    place, on the current stream (the gradients of the summed loss)."""
    import torch.distributed as dist

    if dw.dtype != torch.float32 or not dw.is_contiguous():
        raise ValueError("weight gradients must be one contiguous fp32 buffer")
    dist.all_reduce(dw, op=dist.ReduceOp.SUM, group=process_group)
    return dw


@torch.no_grad()
def broadcast_parameters(module: torch.nn.Module, process_group=None, src: int = 0) -> None:
    """Copy ``src``'s parameters to every rank so that all replicas start equal."""
    import torch.distributed as dist

    for p in module.parameters():
        dist.broadcast(p.data, src=src, group=process_group)
