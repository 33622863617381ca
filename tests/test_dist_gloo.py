"""Multi-rank host logic on CPU with gloo (world size 2 and 4): contiguous
row shards, per-rank gradient scale 1/B_global, one scalar all-reduce.  The
per-rank compute is the oracle (this tests the sharding and the exchange,
which are the only multi-GPU parts of the path); the same reduce_loss_sum /
shard_rows functions run over NCCL in bench.py."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, B, C, out):
    import sys

    repo = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    for p in (repo, os.path.join(repo, "fast-familywise-loss_b200")):
        if p not in sys.path:
            sys.path.insert(0, p)
    from fwloss_b200.distributed import reduce_loss_sum, shard_rows
    from oracle import fw_oracle as O

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    rng = np.random.default_rng(5)
    z = rng.standard_normal((B, C)).astype(np.float32)
    y = rng.integers(0, C, B)
    a, b = shard_rows(B, rank, world)
    s = O.solve(z[a:b], y[a:b], 1.0 / B)
    local = torch.tensor(float(s["loss"].sum() / B), dtype=torch.float64)
    total = reduce_loss_sum(local)
    out[rank] = (float(total), s["grad"], a, b)
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_sharded_loss_and_grad_equal_global(world):
    B, C = 37, 300
    mgr = mp.get_context("spawn").Manager()
    out = mgr.dict()
    mp.start_processes(_worker, args=(world, _free_port(), B, C, out), nprocs=world, join=True,
                       start_method="spawn")
    from oracle import fw_oracle as O

    rng = np.random.default_rng(5)
    z = rng.standard_normal((B, C)).astype(np.float32)
    y = rng.integers(0, C, B)
    full = O.solve(z, y, 1.0 / B)
    totals = [out[r][0] for r in range(world)]
    assert all(t == totals[0] for t in totals)
    np.testing.assert_allclose(totals[0], full["loss"].mean(), rtol=1e-12)
    g = np.concatenate([out[r][1] for r in range(world)])
    np.testing.assert_allclose(g, full["grad"], rtol=1e-12, atol=1e-15)
    assert [out[r][2] for r in range(world)] == sorted(out[r][2] for r in range(world))
