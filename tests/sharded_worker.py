"""One rank of the two-GPU class-sharded check (launched by
tests/test_gpu_sharded.py::test_two_gpu_nccl through torchrun): every rank
holds a column shard of cfg4-like rows, runs class_sharded_familywise_loss over
NCCL, and compares its gradient shard and the loss with the unsharded fused
kernel on the full rows."""
import datetime
import os
import sys

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path[:0] = [REPO, os.path.join(REPO, "fast-familywise-loss_b200")]

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

from fwloss_b200 import capi, workloads  # noqa: E402
from fwloss_b200.sharded import class_sharded_familywise_loss, even_col_start  # noqa: E402


def main():
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    rank, world = dist.get_rank(), dist.get_world_size()
    z, y = workloads.make("cfg4", rows=64)
    z[5] = 0.25  # a constant row: its shard supports exceed K -> exact full-row path
    z, y = z.to(dev), y.to(dev)
    cs = even_col_start(z.shape[1], world)
    zl = z[:, cs[rank]:cs[rank + 1]].contiguous().requires_grad_(True)
    loss = class_sharded_familywise_loss(zl, y, cs, reduction="mean", K=16)
    loss.backward()
    g_full, H, l_full, k = capi.fused_fwd_bwd(z, y, 1.0 / z.shape[0])
    ok = torch.allclose(zl.grad, g_full[:, cs[rank]:cs[rank + 1]], rtol=1e-5, atol=1e-6)
    ok &= abs(loss.item() - l_full.double().mean().item()) <= 1e-5 * max(1.0, abs(loss.item()))
    flag = torch.tensor([0 if ok else 1], device=dev)
    dist.all_reduce(flag)
    dist.destroy_process_group()
    print(f"rank {rank}: ok={ok}")
    sys.exit(int(flag.item() != 0))


if __name__ == "__main__":
    main()
