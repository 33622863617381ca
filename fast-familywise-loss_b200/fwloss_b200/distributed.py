"""Row-sharded data parallelism for the FW loss (one process per GPU).

Rows are independent, so a batch of B rows is split into contiguous row
blocks, one per rank; each rank runs the fused kernel on its block with the
gradient scaled by 1/B (global batch), and the only cross-GPU traffic is one
sum of a scalar loss.  On GPUs that reach each other's memory (NVLink /
NVSwitch, one node) that sum is one kernel, fw_loss_allreduce: the loss
reduction stores its partial into every rank's exchange buffer over peer
memory and adds the partials in rank order (PeerLossExchange); elsewhere
(other backends, no peer access, gloo on CPU for tests) it is the loss
reduction followed by an all-reduce of the scalar.  The reference has no
multi-device code; this is the sharding its row-wise formulation admits.
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


class PeerLossExchange:
    """The exchange buffers of the cross-GPU loss sum for one process group:
    this rank's buffer (on its current CUDA device) and every other rank's,
    mapped through CUDA IPC.  Built collectively: every rank of the group
    constructs it at the same point (it all-gathers the buffers' handles),
    outside any CUDA graph capture (it allocates and synchronises).

    `available` is False on every rank when any rank could not map every
    peer's buffer (GPUs without peer access, ranks on other hosts); callers
    then fall back to an all-reduce.  `reduce(losses, scale)` returns the
    0-d scale * (sum of every rank's losses), the same value on every rank;
    all ranks must make the same sequence of reduce calls, one stream at a
    time per rank.  A rank whose peers do not publish within `timeout_s`
    seconds gets NaN and the status bit checked by `check()`; the exchange is
    unusable after that."""

    def __init__(self, group=None, device=None, timeout_s=10.0):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        self.timeout_s = float(timeout_s)
        self.own, self.peers, self.bufs = None, [], []
        ok, handle = self.world <= 8, None
        if ok:
            try:
                with torch.cuda.device(self.device):
                    self.own, handle = ext().peer_buffer_create()
            except RuntimeError:
                ok = False
        handles = [None] * self.world
        dist.all_gather_object(handles, handle if ok else None, group=group)
        if all(h is not None for h in handles):
            try:
                with torch.cuda.device(self.device):
                    for r, h in enumerate(handles):
                        if r == self.rank:
                            self.bufs.append(self.own)
                        else:
                            p = ext().peer_buffer_open(h)
                            self.peers.append(p)
                            self.bufs.append(p)
            except RuntimeError:
                ok = False
        else:
            ok = False
        flags = [None] * self.world
        dist.all_gather_object(flags, ok, group=group)
        self.available = all(flags)
        if not self.available:
            self._release()
        self.status = torch.zeros(1, dtype=torch.int32, device=self.device)

    def reduce(self, losses, scale):
        return ext().loss_allreduce(losses, float(scale), self.bufs, self.rank, self.status, self.timeout_s)

    def check(self):
        """Raises if a reduce on this rank gave up waiting for its peers
        (reads the device status word: synchronises)."""
        if int(self.status.item()) & 4:
            raise RuntimeError("fwloss_b200: the cross-GPU loss sum timed out waiting for a peer rank")

    def _release(self):
        with torch.cuda.device(self.device):
            for p in self.peers:
                ext().peer_buffer_close(p)
            if self.own is not None:
                ext().peer_buffer_destroy(self.own)
        self.own, self.peers, self.bufs = None, [], []

    def close(self):
        """Collective: unmaps and frees the buffers once every rank is done."""
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        self._release()
        self.available = False


_EXCHANGES = {}


def loss_exchange(group=None, device=None):
    """The group's PeerLossExchange for `device` (collective on first use;
    None when the group's backend is not NCCL or a rank lacks peer access)."""
    if "nccl" not in str(dist.get_backend(group)):
        return None
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    key = (group, dev.index)
    ex = _EXCHANGES.get(key)
    if ex is None:
        ex = _EXCHANGES[key] = PeerLossExchange(group, dev)
    return ex if ex.available else None


def global_loss_sum(losses, scale, group=None):
    """scale * (sum of every rank's per-row losses), 0-d, on every rank: one
    kernel over peer memory where the GPUs allow it, else the loss reduction
    and an all-reduce."""
    ex = loss_exchange(group, losses.device) if losses.is_cuda else None
    if ex is not None:
        return ex.reduce(losses, scale)
    return reduce_loss_sum(ext().loss_reduce(losses, scale), group)


class _ShardedFW(torch.autograd.Function):
    @staticmethod
    def forward(ctx, logits, target, global_batch, group):
        scale = 1.0 / global_batch
        grad, H, losses, kappa = ext().fused_fwd_bwd(logits.detach(), target, scale, None)
        ctx.grad = grad
        return global_loss_sum(losses, scale, group)

    @staticmethod
    def backward(ctx, g):
        grad = ctx.grad
        ctx.grad = None
        ext().scale_grad(grad, g.reshape(1), False, 1.0)
        return grad, None, None, None


def sharded_familywise_loss(local_logits, local_target, global_batch, group=None):
    """Mean FW loss over the global batch from this rank's row block.

    Every rank must call it (it contains the cross-GPU loss sum).  The
    returned 0-d tensor is the global mean; backward gives this rank's rows of
    the global gradient.  Without a possible gradient (no_grad, or logits that
    do not require grad) the forward-only kernel runs (no gradient is
    written).  On an NCCL group the first call builds the group's
    PeerLossExchange (collective, allocating): make it outside CUDA graph
    capture.
    """
    _check_inputs(local_logits, local_target)
    if not (torch.is_grad_enabled() and local_logits.requires_grad):
        _, losses, _ = ext().forward_rows(local_logits.detach(), local_target, None)
        return global_loss_sum(losses, 1.0 / int(global_batch), group)
    return _ShardedFW.apply(local_logits, local_target, int(global_batch), group)
