"""Data-parallel training on 2 GPUs: the 5-layer weight-normed module (BASELINE
config 4 shape) trained on row shards with its process group gives the
full-batch gradients of one GPU, identical on both ranks -- with the dW sum
done by this library's NVLink peer-memory kernel and by NCCL; and the
peer-memory reducer itself over several consecutive steps (the slot is
rewritten each step; the device-side step number advances) against the exact
sum, bitwise equal on every rank.

Needs two sm_100 GPUs; skipped otherwise.  Two processes are spawned, one per
GPU, rendezvous on 127.0.0.1 with a short process-group timeout.
"""
import datetime
import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

WORLD = 2
M = 200_003  # odd: the shards differ by one row


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, port, out_dir, kind):
    import torch.distributed as dist

    from mlp_megakernel_b200 import FusedMLPSoftplusWN
    from mlp_megakernel_b200.dp import broadcast_parameters, shard_rows
    from mlp_megakernel_b200.synthetic import make_inputs

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=WORLD,
                            timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        torch.manual_seed(100 + rank)  # different local init: the broadcast must fix it
        model = FusedMLPSoftplusWN(D=32, H=64, out_features=16, num_layers=5,
                                   process_group=dist.group.WORLD, grad_reduce=kind).cuda()
        broadcast_parameters(model)
        x, _, g = make_inputs("5L", M, with_grad=True)
        a, b = shard_rows(M, rank, WORLD)
        out = model(x[a:b].cuda())
        out.backward(g[a:b].cuda())
        torch.cuda.synchronize()
        np.save(os.path.join(out_dir, f"v{rank}.npy"), model.v_all.grad.cpu().numpy())
        np.save(os.path.join(out_dir, f"g{rank}.npy"), model.g_all.grad.cpu().numpy())
        if rank == 0:
            # full batch on one GPU, same parameters, no process group
            ref = FusedMLPSoftplusWN(D=32, H=64, out_features=16, num_layers=5).cuda()
            with torch.no_grad():
                ref.v_all.copy_(model.v_all)
                ref.g_all.copy_(model.g_all)
            ref(x.cuda()).backward(g.cuda())
            torch.cuda.synchronize()
            np.save(os.path.join(out_dir, "v_full.npy"), ref.v_all.grad.cpu().numpy())
            np.save(os.path.join(out_dir, "g_full.npy"), ref.g_all.grad.cpu().numpy())
        torch.cuda.synchronize()
        dist.barrier()
        if model._grad_sum is not None and model._grad_sum._reducer is not None:
            model._grad_sum._reducer.close()
    finally:
        dist.destroy_process_group()


def _run(target, args, tmp_path):
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=target, args=(r, port, str(tmp_path)) + args) for r in range(WORLD)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]


@pytest.mark.parametrize("kind", ["peer", "nccl"])
def test_dp_two_gpus_matches_full_batch(built_lib, tmp_path, kind):
    if torch.cuda.device_count() < WORLD:
        pytest.skip("needs two GPUs")
    _run(_worker, (kind,), tmp_path)
    for name in ("v", "g"):
        r0 = np.load(tmp_path / f"{name}0.npy")
        r1 = np.load(tmp_path / f"{name}1.npy")
        full = np.load(tmp_path / f"{name}_full.npy").astype(np.float64)
        assert np.array_equal(r0, r1), "ranks hold different gradients after the all-reduce"
        err = np.linalg.norm(r0 - full) / np.linalg.norm(full)
        assert err <= 1e-4, f"{name}: data-parallel vs full-batch rel-L2 {err:.2e}"


def _reducer_worker(rank, port, out_dir):
    import torch.distributed as dist

    from mlp_megakernel_b200 import _lib
    from mlp_megakernel_b200.dp import PeerGradReducer

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=WORLD,
                            timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        n = 49152  # the 3L128 weight-gradient length
        red = PeerGradReducer(n)
        out = torch.empty(n, device="cuda")
        for step in range(5):  # the slot rewritten, the step number advanced
            gen = torch.Generator().manual_seed(1000 * step + rank)
            red.local_buffer(out).copy_(torch.randn(n, generator=gen).cuda())
            red.reduce(red.local_buffer(out), out)
            torch.cuda.synchronize()
            np.save(os.path.join(out_dir, f"r{rank}_s{step}.npy"), out.cpu().numpy())
        assert _lib.device_status() == 0
        red.close()
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_peer_reducer_exact_and_identical_on_ranks(built_lib, tmp_path):
    if torch.cuda.device_count() < WORLD:
        pytest.skip("needs two GPUs")
    _run(_reducer_worker, (), tmp_path)
    n = 49152
    for step in range(5):
        parts = [torch.randn(n, generator=torch.Generator().manual_seed(1000 * step + r)).numpy()
                 for r in range(WORLD)]
        expect = parts[0].astype(np.float32)
        for p in parts[1:]:
            expect = expect + p.astype(np.float32)  # rank order, fp32: what the kernel computes
        r0 = np.load(tmp_path / f"r0_s{step}.npy")
        r1 = np.load(tmp_path / f"r1_s{step}.npy")
        assert np.array_equal(r0, r1)
        assert np.array_equal(r0, expect)
