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


class _OracleExt:
    """Stands in for the native module on CPU tensors (test only): the three
    kernel calls the row-sharded autograd function makes, computed by the
    oracle, so that the function's host logic (scale 1/B_global, loss
    reduction, all-reduce, backward scaling) runs unchanged under gloo."""

    def __init__(self):
        from oracle import fw_oracle as O

        self.O = O
        self.calls = []

    def fused_fwd_bwd(self, z, y, scale, status):
        self.calls.append(("fused_fwd_bwd", scale))
        s = self.O.solve(z.numpy(), y.numpy(), scale)
        return (torch.from_numpy(s["grad"].astype(np.float32)), torch.from_numpy(s["H"].astype(np.float32)),
                torch.from_numpy(s["loss"].astype(np.float32)), torch.from_numpy(s["kappa"].astype(np.int32)))

    def forward_rows(self, z, y, status):
        self.calls.append(("forward_rows",))
        s = self.O.solve(z.numpy(), y.numpy(), 1.0)
        return (torch.from_numpy(s["H"].astype(np.float32)), torch.from_numpy(s["loss"].astype(np.float32)),
                torch.from_numpy(s["kappa"].astype(np.int32)))

    def loss_reduce(self, losses, scale):
        self.calls.append(("loss_reduce", scale))
        return torch.tensor(float(losses.double().sum()) * scale, dtype=torch.float32)

    def scale_grad(self, grad, grad_output, per_row, assumed):
        self.calls.append(("scale_grad", per_row))
        f = grad_output.double() / assumed
        grad.mul_((f.reshape(-1, 1) if per_row else f.reshape(())).to(grad.dtype))


def _worker_autograd(rank, world, port, B, C, out):
    import sys

    repo = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    for p in (repo, os.path.join(repo, "fast-familywise-loss_b200")):
        if p not in sys.path:
            sys.path.insert(0, p)
    from fwloss_b200 import distributed as D

    fake = _OracleExt()
    D.ext = lambda: fake               # the kernels, on the CPU (test only)
    D._check_inputs = lambda z, y: None  # the product path requires CUDA tensors
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    rng = np.random.default_rng(7)
    z = rng.standard_normal((B, C)).astype(np.float32)
    y = rng.integers(0, C, B)
    a, b = D.shard_rows(B, rank, world)
    zl = torch.from_numpy(z[a:b].copy()).requires_grad_(True)
    yl = torch.from_numpy(y[a:b].copy())
    loss = D.sharded_familywise_loss(zl, yl, B)
    (loss * 3.0).backward()
    with torch.no_grad():
        nograd = D.sharded_familywise_loss(zl, yl, B)
    no_exchange = D.loss_exchange() is None  # gloo: the loss sum is reduction + all-reduce
    out[rank] = (float(loss), zl.grad.numpy().copy(), a, b, float(nograd), list(fake.calls), no_exchange)
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_sharded_autograd_function_host_logic(world):
    """sharded_familywise_loss forward/backward under gloo with the kernel
    calls stubbed: every rank returns the global mean loss, its rows of the
    global gradient times the upstream factor, the fused kernel runs with the
    global scale 1/B, the no-grad call takes the forward-only kernel, and a
    gloo group sums the loss by reduction + all-reduce (no peer exchange)."""
    B, C = 29, 150
    mgr = mp.get_context("spawn").Manager()
    out = mgr.dict()
    mp.start_processes(_worker_autograd, args=(world, _free_port(), B, C, out), nprocs=world, join=True,
                       start_method="spawn")
    from oracle import fw_oracle as O

    rng = np.random.default_rng(7)
    z = rng.standard_normal((B, C)).astype(np.float32)
    y = rng.integers(0, C, B)
    full = O.solve(z, y, 1.0 / B)
    mean = full["loss"].mean()
    for r in range(world):
        loss, g, a, b, nograd, calls, no_exchange = out[r]
        assert no_exchange
        np.testing.assert_allclose(loss, mean, rtol=1e-6)
        np.testing.assert_allclose(nograd, mean, rtol=1e-6)
        np.testing.assert_allclose(g, 3.0 * full["grad"][a:b], rtol=1e-6, atol=1e-9)
        assert calls[0] == ("fused_fwd_bwd", 1.0 / B) and ("loss_reduce", 1.0 / B) in calls
        assert ("scale_grad", False) in calls and ("forward_rows",) in calls
    assert sorted(out[r][2] for r in range(world)) == [out[r][2] for r in range(world)]
    assert sum(out[r][3] - out[r][2] for r in range(world)) == B


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
