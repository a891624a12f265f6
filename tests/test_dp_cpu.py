"""Data-parallel host logic on CPU: two gloo ranks (world_size 2, 127.0.0.1).

Checks that sharding the rows and summing the per-rank weight gradients with
mlp_megakernel_b200.dp gives exactly the full-batch gradients of the oracle
(the data-parallel training step of the reference's DP recipe: per-rank
backward, all_reduce(SUM) of fp32 dW, replicated weight-norm backward), and
that parameter broadcast makes the replicas identical.  No GPU is involved.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle
from mlp_megakernel_b200.dp import allreduce_weight_grads, broadcast_parameters, shard_rows
from mlp_megakernel_b200.synthetic import make_inputs

WORLD = 2


@pytest.mark.parametrize("M", [0, 1, 7, 128, 1000, 262145])
@pytest.mark.parametrize("world", [1, 2, 3, 8])
def test_shard_rows_partitions_exactly(M, world):
    ranges = [shard_rows(M, r, world) for r in range(world)]
    assert ranges[0][0] == 0 and ranges[-1][1] == M
    for (a, b), (c, d) in zip(ranges[:-1], ranges[1:]):
        assert b == c and a <= b
    sizes = [b - a for a, b in ranges]
    assert max(sizes) - min(sizes) <= 1


def test_shard_rows_rejects_bad_rank():
    with pytest.raises(ValueError):
        shard_rows(10, 2, 2)
    with pytest.raises(ValueError):
        shard_rows(-1, 0, 2)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _flat(dws):
    return np.concatenate([d.reshape(-1) for d in dws])


def _worker(rank, port, config, M, result_dir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=WORLD)
    try:
        x, ws, g = make_inputs(config, M, with_grad=True)
        a, b = shard_rows(M, rank, WORLD)
        wn = [w.numpy() for w in ws]
        _, hs = oracle.mlp_forward_train(x.numpy()[a:b], wn)
        _, dws = oracle.mlp_backward(x.numpy()[a:b], wn, hs, g.numpy()[a:b])
        dw = torch.from_numpy(_flat(dws).astype(np.float32)).contiguous()
        allreduce_weight_grads(dw)
        # replicas from different seeds become equal after the broadcast
        torch.manual_seed(100 + rank)
        mod = torch.nn.Linear(8, 4)
        broadcast_parameters(mod)
        params = torch.cat([p.detach().reshape(-1) for p in mod.parameters()])
        np.save(os.path.join(result_dir, f"dw{rank}.npy"), dw.numpy())
        np.save(os.path.join(result_dir, f"p{rank}.npy"), params.numpy())
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("config,M", [("3L128", 1001), ("5L", 777)])
def test_dp_gradient_sum_equals_full_batch(config, M, tmp_path):
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, port, config, M, str(tmp_path)))
             for r in range(WORLD)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]

    x, ws, g = make_inputs(config, M, with_grad=True)
    wn = [w.numpy() for w in ws]
    _, hs = oracle.mlp_forward_train(x.numpy(), wn)
    _, dws = oracle.mlp_backward(x.numpy(), wn, hs, g.numpy())
    full = _flat(dws)
    dw0 = np.load(tmp_path / "dw0.npy")
    dw1 = np.load(tmp_path / "dw1.npy")
    assert np.array_equal(dw0, dw1), "ranks disagree after the all-reduce"
    err = np.linalg.norm(dw0 - full) / np.linalg.norm(full)
    assert err <= 1e-6, err
    assert np.array_equal(np.load(tmp_path / "p0.npy"), np.load(tmp_path / "p1.npy"))


def _fallback_worker(rank, port, result_dir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=WORLD)
    try:
        from mlp_megakernel_b200.dp import (NcclGradReducer, PeerGradReducer, PeerSetupError,
                                            make_grad_reducer)

        # no GPU here: the peer buffer cannot be allocated on any rank, and
        # every rank must learn it together (no rank left in a collective)
        raised = False
        try:
            PeerGradReducer(16)
        except PeerSetupError:
            raised = True
        red = make_grad_reducer(16)  # "auto": not NCCL here -> the collective reducer
        out = torch.full((16,), float(rank + 1))
        red.reduce(red.local_buffer(out), out)
        np.save(os.path.join(result_dir, f"f{rank}.npy"),
                np.array([raised, isinstance(red, NcclGradReducer), float(out[0])]))
    finally:
        dist.destroy_process_group()


def test_peer_reducer_setup_failure_is_collective(tmp_path):
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_fallback_worker, args=(r, port, str(tmp_path))) for r in range(WORLD)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    for r in range(WORLD):
        raised, is_nccl, val = np.load(tmp_path / f"f{r}.npy")
        assert raised and is_nccl and val == 3.0
