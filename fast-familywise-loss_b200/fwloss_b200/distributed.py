"""Row-sharded data parallelism for the FW loss (one process per GPU).

Rows are independent, so a batch of B rows is split into contiguous row
blocks, one per rank; each rank runs the fused kernel on its block with the
gradient scaled by 1/B (global batch), and the only cross-GPU traffic is one
all-reduce of a scalar loss sum (NCCL over NVLink on B200 nodes, gloo on CPU
for tests).  The reference has no multi-device code; this is the sharding
its row-wise formulation admits.
"""
import torch
import torch.distributed as dist

from ._native import ext
from .functional import _check_inputs


def shard_rows(global_batch, rank, world_size):
    """[start, stop) of rank's contiguous row block (sizes differ by <= 1)."""
    base, extra = divmod(int(global_batch), int(world_size))
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def reduce_loss_sum(local_sum, group=None):
    """All-reduces a 0-d/1-element loss sum in place and returns it."""
    buf = local_sum.reshape(1)
    dist.all_reduce(buf, op=dist.ReduceOp.SUM, group=group)
    return buf.reshape(())


class _ShardedFW(torch.autograd.Function):
    @staticmethod
    def forward(ctx, logits, target, global_batch, group):
        scale = 1.0 / global_batch
        grad, H, losses, kappa = ext().fused_fwd_bwd(logits.detach(), target, scale, None)
        ctx.grad = grad
        local = ext().loss_reduce(losses, scale)
        return reduce_loss_sum(local, group)

    @staticmethod
    def backward(ctx, g):
        grad = ctx.grad
        ctx.grad = None
        ext().scale_grad(grad, g.reshape(1), False, 1.0)
        return grad, None, None, None


def sharded_familywise_loss(local_logits, local_target, global_batch, group=None):
    """Mean FW loss over the global batch from this rank's row block.

    Every rank must call it (it contains one all-reduce).  The returned 0-d
    tensor is the global mean; backward gives this rank's rows of the global
    gradient.  Without a possible gradient (no_grad, or logits that do not
    require grad) the forward-only kernel runs (no gradient is written).
    """
    _check_inputs(local_logits, local_target)
    if not (torch.is_grad_enabled() and local_logits.requires_grad):
        _, losses, _ = ext().forward_rows(local_logits.detach(), local_target, None)
        return reduce_loss_sum(ext().loss_reduce(losses, 1.0 / int(global_batch)), group)
    return _ShardedFW.apply(local_logits, local_target, int(global_batch), group)
