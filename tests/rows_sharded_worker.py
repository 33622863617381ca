"""One rank of the row-sharded check (launched by
tests/test_gpu_rows_sharded.py through torchrun, one or more ranks): every
rank holds a contiguous row block of one batch and calls the public
fwloss_b200.distributed.sharded_familywise_loss over NCCL.  Checked on every
rank against familywise_loss on the whole batch (computed by every rank on
its own GPU):

  * the loss (global mean) and this rank's rows of the gradient, with the
    implicit upstream gradient 1 and with an upstream factor of 3;
  * the forward-only path (torch.no_grad): the same loss;
  * the step captured once in a CUDA graph (forward kernel, loss reduction,
    the cross-GPU loss sum and the backward) and replayed on new logits, as
    bench.py runs it;
  * the cross-GPU loss sum over peer memory (fw_loss_allreduce) itself: used
    whenever every pair of GPUs has peer access, equal on every rank to the
    bit, within 1e-6 of the loss reduction + NCCL all-reduce over several
    calls in a row (both epoch parities), fp32 and fp64 losses;
  * its bounded wait: on a separate exchange only rank 0 calls (0.3 s limit),
    and gets NaN and FWB_STATUS_TIMEOUT instead of waiting for good.

Exits non-zero when any rank failed."""
import datetime
import os
import sys

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path[:0] = [REPO, os.path.join(REPO, "fast-familywise-loss_b200")]

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

from fwloss_b200 import familywise_loss, workloads  # noqa: E402
from fwloss_b200._native import ext  # noqa: E402
from fwloss_b200.distributed import (PeerLossExchange, loss_exchange, reduce_loss_sum,  # noqa: E402
                                     shard_rows, sharded_familywise_loss)


def full_reference(z, y):
    zr = z.clone().requires_grad_(True)
    loss = familywise_loss(zr, y, reduction="mean")
    loss.backward()
    return loss.detach(), zr.grad


def close(a, b):
    return abs(float(a) - float(b)) <= 1e-6 * max(1.0, abs(float(b)))


def main():
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    rank, world = dist.get_rank(), dist.get_world_size()
    ok = True
    B = 97  # not a multiple of the rank count: blocks differ by one row
    z, y = workloads.make("cfg2", rows=B)
    z, y = z.to(dev), y.to(dev)
    lo, hi = shard_rows(B, rank, world)
    ref_loss, ref_grad = full_reference(z, y)

    # eager, upstream gradient 1 and 3
    for factor in (1.0, 3.0):
        zl = z[lo:hi].clone().requires_grad_(True)
        loss = sharded_familywise_loss(zl, y[lo:hi], B)
        (loss * factor if factor != 1.0 else loss).backward()
        ok &= close(loss.detach(), ref_loss)
        ok &= torch.allclose(zl.grad, ref_grad[lo:hi] * factor, rtol=1e-6, atol=1e-9)

    # forward only
    with torch.no_grad():
        ok &= close(sharded_familywise_loss(z[lo:hi], y[lo:hi], B), ref_loss)

    # one CUDA graph holding the whole step, replayed on new logits
    static_z = z[lo:hi].clone().requires_grad_(True)
    static_y = y[lo:hi].clone()
    side = torch.cuda.Stream(dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(side):
        for _ in range(2):  # warm-up outside the capture (NCCL communicator, allocator)
            static_z.grad = None
            sharded_familywise_loss(static_z, static_y, B).backward()
    torch.cuda.current_stream(dev).wait_stream(side)
    torch.cuda.synchronize(dev)
    g = torch.cuda.CUDAGraph()
    static_z.grad = None
    with torch.cuda.graph(g):
        static_loss = sharded_familywise_loss(static_z, static_y, B)
        static_loss.backward()
    for seed in (11, 12):
        z2 = torch.randn(B, z.shape[1], generator=torch.Generator().manual_seed(seed)).mul_(2.0).to(dev)
        y2 = torch.randint(0, z.shape[1], (B,), generator=torch.Generator().manual_seed(seed + 100)).to(dev)
        with torch.no_grad():
            static_z.copy_(z2[lo:hi])
            static_y.copy_(y2[lo:hi])
        g.replay()
        torch.cuda.synchronize(dev)
        r_loss, r_grad = full_reference(z2, y2)
        ok &= close(static_loss, r_loss)
        ok &= torch.allclose(static_z.grad, r_grad[lo:hi], rtol=1e-6, atol=1e-9)
    del g, static_loss  # release the graph (it holds an NCCL call) before the group goes
    torch.cuda.synchronize(dev)

    ok &= check_peer_sum(dev, rank, world)

    flag = torch.tensor([0 if ok else 1], device=dev)
    dist.all_reduce(flag)
    dist.destroy_process_group()
    print(f"rank {rank}/{world}: ok={bool(ok)}")
    sys.exit(int(flag.item() != 0))


def check_peer_sum(dev, rank, world):
    ok = True
    peer_ok = all(torch.cuda.can_device_access_peer(dev.index, d) for d in range(torch.cuda.device_count())
                  if d != dev.index)
    ex = loss_exchange(None, dev)
    if world > 1 and peer_ok and torch.cuda.device_count() >= world:
        ok &= ex is not None  # the peer-memory path is the one that runs
    if ex is None:
        return ok
    g = torch.Generator().manual_seed(100 + rank)
    for i in range(5):  # epochs 1..5 of this exchange's own calls: both parities
        for dt in (torch.float32, torch.float64):
            losses = (torch.rand(37 + 11 * rank + i, generator=g, dtype=torch.float64) * 3).to(dt).to(dev)
            scale = 1.0 / 1000.0
            got = ex.reduce(losses, scale)
            ref = reduce_loss_sum(ext().loss_reduce(losses, scale))
            every = [torch.zeros((), dtype=dt, device=dev) for _ in range(world)]
            dist.all_gather(every, got.reshape(()).contiguous())
            ok &= all(bool(torch.equal(e, every[0])) for e in every)
            ok &= abs(float(got) - float(ref)) <= 1e-6 * max(1.0, abs(float(ref)))
    torch.cuda.synchronize(dev)
    ex.check()

    # bounded wait: a second exchange on which only rank 0 calls
    solo = PeerLossExchange(None, dev, timeout_s=0.3)
    if solo.available:
        if rank == 0:
            out = solo.reduce(torch.ones(8, device=dev), 1.0)
            torch.cuda.synchronize(dev)
            if world > 1:
                ok &= bool(torch.isnan(out)) and int(solo.status.item()) == 4
            else:
                ok &= float(out) == 8.0 and int(solo.status.item()) == 0
        solo.close()
    return ok


if __name__ == "__main__":
    main()
