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

The weight-gradient sum has two implementations behind ``make_grad_reducer``:

* ``PeerGradReducer`` -- all ranks on one node (up to 8): this library's own
  kernel sums the ranks' dW over NVLink peer memory (CUDA IPC buffers, bounded
  flag hand-off), in rank order, so every rank gets bitwise the same dW;
* ``NcclGradReducer`` -- anything else: ``all_reduce(SUM)`` over NCCL.
"""
from __future__ import annotations

import ctypes
import os

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


class NcclGradReducer:
    """dW sum over ``torch.distributed`` (NCCL across nodes)."""

    def __init__(self, n: int, process_group=None):
        self.n = n
        self.process_group = process_group

    def local_buffer(self, like: torch.Tensor) -> torch.Tensor:
        """Where the backward writes this rank's dW (here: the output itself)."""
        return like

    def reduce(self, local: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
        if local.data_ptr() != out.data_ptr():
            out.copy_(local)
        return allreduce_weight_grads(out, self.process_group)

    def close(self):
        pass


class PeerSetupError(RuntimeError):
    """The ranks could not set up peer-memory buffers (every rank raises it)."""


class _DevicePtr:
    """A raw device pointer seen by torch as a float32 tensor (no copy)."""

    def __init__(self, ptr: int, n: int):
        self.__cuda_array_interface__ = {"shape": (n,), "typestr": "<f4", "data": (ptr, False),
                                         "version": 3, "strides": None}


class PeerGradReducer:
    """Deterministic dW sum over NVLink peer memory for the ranks of one node.

    Set-up (collective): every rank allocates a peer buffer through the C ABI
    (``mlpk_peer_alloc``), the IPC handles are exchanged with
    ``all_gather_object`` and every rank opens the others' buffers.  Per step:
    the backward writes this rank's dW into ``local_buffer()`` and
    ``reduce()`` launches ``mlpk_peer_allreduce``, which sums the ranks' dW in
    rank order on the current stream.  Every rank must run the same steps in
    the same order; the step count is kept on the device, so steps may be
    replayed from a CUDA graph.
    """

    def __init__(self, n: int, process_group=None):
        import torch.distributed as dist

        from . import _lib

        if n % 4:
            raise ValueError("the gradient length must be a multiple of 4")
        self.n = n
        self.process_group = process_group
        self.world = dist.get_world_size(process_group)
        self.rank = dist.get_rank(process_group)
        if self.world > _lib.PEER_MAX_RANKS:
            raise ValueError(f"peer-memory reduction serves at most {_lib.PEER_MAX_RANKS} ranks")
        self._lib = _lib.lib()
        self._own = None
        self._opened = []
        # Every step below is agreed by all ranks, so a failure on one rank
        # (no CUDA IPC, out of memory) makes every rank give up together
        # instead of leaving the others in a collective.
        own = ctypes.c_void_p()
        handle = (ctypes.c_uint8 * _lib.PEER_HANDLE_BYTES)()
        ok = self._lib.mlpk_peer_alloc(n, ctypes.byref(own), handle) == 0
        if ok:
            self._own = own.value
        shared = [None] * self.world
        dist.all_gather_object(shared, (ok, bytes(handle)), group=process_group)
        if not all(flag for flag, _ in shared):
            self.close(sync=False)
            raise PeerSetupError("a rank could not allocate its peer buffer")
        ptrs = []
        ok = True
        for q, (_, h) in enumerate(shared):
            if q == self.rank:
                ptrs.append(self._own)
                continue
            p = ctypes.c_void_p()
            hb = (ctypes.c_uint8 * _lib.PEER_HANDLE_BYTES).from_buffer_copy(h)
            if self._lib.mlpk_peer_open(hb, ctypes.byref(p)) != 0:
                ok = False
                break
            self._opened.append(p.value)
            ptrs.append(p.value)
        flags = [None] * self.world
        dist.all_gather_object(flags, ok, group=process_group)
        if not all(flags):
            self.close(sync=False)
            raise PeerSetupError("a rank could not map the other ranks' peer buffers")
        self._ptrs = _lib.ptr_array(ptrs)
        self._local = torch.as_tensor(_DevicePtr(self._own, n),
                                      device=torch.device("cuda", torch.cuda.current_device()))

    def local_buffer(self, like: torch.Tensor = None) -> torch.Tensor:
        """This rank's dW slot (the backward writes dW here)."""
        return self._local

    def reduce(self, local: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
        from . import _lib

        if local.data_ptr() != self._own:
            raise RuntimeError("local dW is not in this rank's peer slot (use local_buffer())")
        if out.dtype != torch.float32 or not out.is_contiguous() or out.numel() != self.n:
            raise ValueError("output must be a contiguous fp32 buffer of the gradient length")
        _lib.check("mlpk_peer_allreduce",
                   self._lib.mlpk_peer_allreduce(self._ptrs, self.world, self.rank, self.n, out.data_ptr(),
                                                 torch.cuda.current_stream(out.device).cuda_stream))
        return out

    def close(self, sync: bool = True):
        """Unmap the peers' buffers and free this rank's.  Collective: a rank's
        last reduction may return while the other ranks still read its buffer,
        so every rank synchronizes its device and meets the others at a
        barrier before anything is unmapped or freed (``sync=False``: set-up
        failures only, before any reduction ran)."""
        if sync:
            import torch.distributed as dist

            torch.cuda.synchronize()
            if self.world > 1:
                dist.barrier(group=self.process_group)
        self._local = None
        for p in self._opened:
            self._lib.mlpk_peer_close(ctypes.c_void_p(p))
        self._opened = []
        if self._own is not None:
            self._lib.mlpk_peer_free(ctypes.c_void_p(self._own))
            self._own = None


def single_node(process_group=None) -> bool:
    """True when every rank of the group runs on this node (torchrun's
    LOCAL_WORLD_SIZE equals the group size)."""
    import torch.distributed as dist

    local = int(os.environ.get("LOCAL_WORLD_SIZE", "-1"))
    return local == dist.get_world_size(process_group)


def make_grad_reducer(n: int, process_group=None, kind: str = "auto"):
    """The dW reducer for ``process_group``: peer memory on one node (up to 8
    ranks), NCCL otherwise.  ``kind`` = "auto", "peer" or "nccl"."""
    import torch.distributed as dist

    if kind not in ("auto", "peer", "nccl"):
        raise ValueError(f"unknown reducer kind {kind!r}")
    if kind == "peer":
        return PeerGradReducer(n, process_group)
    if (kind == "auto" and dist.get_backend(process_group) == "nccl" and single_node(process_group)
            and dist.get_world_size(process_group) <= 8 and n % 4 == 0):
        try:
            return PeerGradReducer(n, process_group)
        except PeerSetupError:
            pass  # every rank of the group lands here together
    return NcclGradReducer(n, process_group)
