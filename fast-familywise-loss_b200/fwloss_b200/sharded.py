"""Class-sharded FW loss: each rank holds a column shard of every row
(vocabulary-parallel LM heads), one process per GPU.

    from fwloss_b200.sharded import class_sharded_familywise_loss
    # local_logits: [B, C_q] fp32 (this rank's classes), target: [B] global class ids
    loss = class_sharded_familywise_loss(local_logits, target, col_start)   # every rank calls it
    loss.backward()                       # local_logits.grad = this rank's gradient shard

The global threshold h* of a row is >= the threshold each shard would have on
its own, so the part of the global support held by shard q lies inside shard
q's own support (usually a handful of entries).  Per step:
  1. fw_shard_scan      local solve, zero gradient shard, summary per row
  2. all-gather         summaries [world, B, 4 + K] int32 (B * (4 + K) * 4 bytes per rank)
  3. fw_shard_solve     global threshold from the union of the shard supports,
                        patch of the local gradient shard, loss where the
                        label lives here
  4. all-reduce         the scalar loss sum
Rows where a shard's own support exceeds K entries (near-constant rows) are
listed by step 3 and solved exactly from their full rows (gathered for those
rows only, then the unsharded fused kernel); reading that count is one 4-byte
device-to-host copy per step, issued after the step's other work is queued.
"""
import torch
import torch.distributed as dist

from ._native import ext

DEFAULT_K = 32


def even_col_start(num_classes, world_size):
    """Shard offsets [world + 1] for an even split (sizes differ by <= 1)."""
    base, extra = divmod(int(num_classes), int(world_size))
    out = [0]
    for q in range(world_size):
        out.append(out[-1] + base + (1 if q < extra else 0))
    return out


def _nccl_all_gather(local, group):
    world = dist.get_world_size(group)
    out = torch.empty((world,) + tuple(local.shape), dtype=local.dtype, device=local.device)
    dist.all_gather_into_tensor(out, local.contiguous(), group=group)
    return out


def _nccl_all_reduce(t, group):
    dist.all_reduce(t, group=group)
    return t


def scan_phase(z_local, K=DEFAULT_K):
    """Step 1: (zero-filled grad shard, summary [B, 4 + K], local_idx [B, K])."""
    return ext().shard_scan(z_local, K)


def solve_phase(gathered, z_local, target, col_start, rank, scale, grad, local_idx):
    """Step 3 on one rank.  Returns (H, kappa, loss_part, fb_rows, fb_count);
    grad is patched in place; rows listed in fb_rows[:fb_count] are not solved
    yet (finish_rows)."""
    return ext().shard_solve(gathered, rank, list(col_start), z_local, target, float(scale), grad, local_idx)


def finish_rows(fb_rows, fb_count, z_local, target, col_start, rank, scale, all_gather, grad, H, kappa,
                loss_part):
    """Exact path for the rows step 3 could not solve.  Reads the row count
    (one 4-byte device-to-host copy; identical on all ranks because it is
    computed from the same gathered data).  Returns the count."""
    nfb = int(fb_count.item())
    if nfb:
        rows = fb_rows[:nfb].long().sort().values
        _solve_full_rows(z_local, target, col_start, rank, scale, all_gather, rows, grad, H, kappa, loss_part)
    return nfb


def sharded_step(z_local, target, col_start, rank, scale, all_gather, K=DEFAULT_K):
    """Steps 1-3 for one rank.  Returns (grad shard, H, kappa, loss_part)
    where loss_part[r] is row r's loss on the rank that owns the label and 0
    elsewhere."""
    grad, summary, local_idx = scan_phase(z_local, K)
    H, kappa, loss_part, fb_rows, fb_count = solve_phase(all_gather(summary), z_local, target, col_start, rank,
                                                         scale, grad, local_idx)
    finish_rows(fb_rows, fb_count, z_local, target, col_start, rank, scale, all_gather, grad, H, kappa, loss_part)
    return grad, H, kappa, loss_part


def sharded_loss_step(z_local, target, col_start, rank, scale, all_gather, all_reduce, K=DEFAULT_K):
    """One full step for one rank, with the host read of the exact-path row
    count placed after all common-path work is queued: (grad shard, global
    loss sum * scale as a 0-d tensor)."""
    fw = ext()
    grad, summary, local_idx = scan_phase(z_local, K)
    H, kappa, loss_part, fb_rows, fb_count = solve_phase(all_gather(summary), z_local, target, col_start, rank,
                                                         scale, grad, local_idx)
    loss = all_reduce(fw.loss_reduce(loss_part, float(scale)).reshape(1))
    nfb = int(fb_count.item())
    if nfb:  # rare: solve those rows from their full rows, then add their losses
        rows = fb_rows[:nfb].long().sort().values
        before = loss_part[rows].clone()
        _solve_full_rows(z_local, target, col_start, rank, scale, all_gather, rows, grad, H, kappa, loss_part)
        corr = ((loss_part[rows] - before).double().sum() * scale).float().reshape(1)
        loss = loss + all_reduce(corr)
    return grad, loss.reshape(())


def _solve_full_rows(z_local, target, col_start, rank, scale, all_gather, rows, grad, H, kappa, loss_part):
    """Exact path for listed rows: gather their full rows and run the
    unsharded fused kernel; keep this rank's columns of the gradient."""
    widths = [col_start[q + 1] - col_start[q] for q in range(len(col_start) - 1)]
    wmax = max(widths)
    F = rows.numel()
    mine = torch.full((F, wmax), float("-inf"), dtype=z_local.dtype, device=z_local.device)
    mine[:, : widths[rank]] = z_local[rows]
    parts = all_gather(mine)  # [world, F, wmax]
    full = torch.cat([parts[q, :, : widths[q]] for q in range(len(widths))], dim=1)
    yr = target[rows]
    g, h, l, k = ext().fused_fwd_bwd(full, yr, float(scale), None)
    lo, hi = col_start[rank], col_start[rank + 1]
    grad[rows] = g[:, lo:hi]
    H[rows] = h
    kappa[rows] = k
    own = (yr >= lo) & (yr < hi)
    loss_part[rows] = torch.where(own, l, torch.zeros_like(l))


class _ClassSharded(torch.autograd.Function):
    @staticmethod
    def forward(ctx, z_local, target, col_start, scale, group, K):
        rank = dist.get_rank(group)
        grad, loss = sharded_loss_step(z_local.detach(), target, col_start, rank, scale,
                                       lambda x: _nccl_all_gather(x, group),
                                       lambda t: _nccl_all_reduce(t, group), K)
        ctx.grad = grad
        return loss

    @staticmethod
    def backward(ctx, g):
        grad = ctx.grad
        ctx.grad = None
        ext().scale_grad(grad, g.reshape(1), False, 1.0)
        return grad, None, None, None, None, None


def class_sharded_familywise_loss(local_logits, target, col_start, reduction="mean", group=None, K=DEFAULT_K):
    """FW loss of rows whose classes are split across the ranks of `group`.

    local_logits: [B, col_start[rank+1] - col_start[rank]] fp32 CUDA (this
    rank's classes); target: [B] int64 global class ids (the same on every
    rank); col_start: the world + 1 shard offsets (even_col_start for an even
    split).  Returns the global "mean" or "sum" loss (0-d, equal on all ranks);
    backward yields this rank's gradient shard.
    """
    if reduction not in ("mean", "sum"):
        raise ValueError(f"Invalid reduction mode: {reduction}")
    if not local_logits.is_cuda or local_logits.dtype != torch.float32 or local_logits.dim() != 2:
        raise TypeError("class_sharded_familywise_loss: local_logits must be a 2-D float32 CUDA tensor")
    world = dist.get_world_size(group)
    if len(col_start) != world + 1:
        raise ValueError("col_start must have world_size + 1 entries")
    B = local_logits.shape[0]
    scale = (1.0 / B if B else float("nan")) if reduction == "mean" else 1.0
    return _ClassSharded.apply(local_logits, target, tuple(int(c) for c in col_start), scale, group, int(K))
