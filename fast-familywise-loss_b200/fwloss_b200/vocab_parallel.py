"""FW loss on a vocabulary-parallel LM head: every rank of a process group
holds the same hidden states and labels and the weight rows of its own slice
of the classes (Megatron-style tensor-parallel output layer), one process per
GPU.

    from fwloss_b200.vocab_parallel import vocab_parallel_lm_head_loss
    # hidden [B, D] (same on every rank), weight_shard [C_q, D] = classes
    # col_start[rank] .. col_start[rank + 1], target [B] global class ids
    loss = vocab_parallel_lm_head_loss(hidden, weight_shard, target, col_start)
    loss.backward()   # weight_shard.grad: this rank's rows; hidden.grad: full

Per step, on every rank:
  1. the rank's logits are produced and reduced to per-(chunk, row) summary
     records chunk by chunk (the tcgen05 kernel for bf16 on sm_100, else a
     GEMM per chunk and the fused FW kernel), as for one GPU;
  2. all-gather of the records and the local support columns (the global
     chunk list is the ranks' chunk lists in rank order), all-reduce of the
     label logits (each row's label lives on one rank; the others add 0);
  3. fw_chunks_solve on the gathered records, identical on every rank: H,
     kappa, the loss and the global support columns.  No logit crosses
     NVLink, only B * nchunks * (4 + 2K) int32 words per rank;
  4. backward: each rank's part of dhidden (its support columns and label
     rows of W, fp32) is all-reduced while dweight is computed; dweight is
     local (sorted contribution keys of the local classes, deterministic).
Rows whose chunk supports exceed K entries (near-constant logits) are solved
from their full logit rows: each rank computes its columns of those rows,
they are all-gathered, and the unsharded fused kernel runs on them.
"""
import torch
import torch.distributed as dist

from ._native import ext
from .lm_head import DEFAULT_K, FUSED_TILE, STATUS_TIMEOUT, _fused_ok, _logits_chunk, chunk_summaries, \
    fused_nchunks, tile_col_start
from .sharded import even_col_start

MAX_CHUNKS = 16     # chunk records combined per row (all ranks together)
LIST_CAP = 256      # nchunks * K limit of the combined solve


def chunks_per_rank(world, B, col_start, K, fused, sms):
    """Chunks per rank, the same on every rank (it fixes the global chunk list
    and the shapes of the all-gathers), at most what the narrowest shard can
    be split into."""
    cap = max(1, min(MAX_CHUNKS // world, LIST_CAP // (K * world)))
    widths = [col_start[q + 1] - col_start[q] for q in range(world)]
    if fused:
        cap = min(cap, min(-(-w // FUSED_TILE) for w in widths))
        return max(1, fused_nchunks(B, max(widths), sms, max_chunks=cap))
    cap = min(cap, min(widths))
    return max(1, min(cap, -(-max(widths) // 16384)))


def local_chunk_starts(C_local, n, fused):
    return tile_col_start(C_local, n) if fused else even_col_start(C_local, n)


def global_chunk_starts(col_start, n, fused):
    """Column offsets of every rank's chunks, in rank order, ending at C."""
    out = []
    for q in range(len(col_start) - 1):
        out += [col_start[q] + c for c in local_chunk_starts(col_start[q + 1] - col_start[q], n, fused)[:-1]]
    return out + [col_start[-1]]


def scan_phase(hidden, weight_shard, target, c0, cs_local, K, fused):
    """Step 1 on one rank: (summaries [n, B, 4 + K], local_idx [n, B, K],
    zy part [B] (0 where the label is another rank's), status [1])."""
    return chunk_summaries(hidden, weight_shard, target, cs_local, K, fused, c0)


def solve_phase(summaries_all, local_idx_all, cs_global, zy, target):
    """Step 3 (every rank, same result): (H, kappa, loss_rows, sup_cols,
    fb_rows, fb_count) from the gathered records."""
    return ext().chunks_solve(summaries_all, local_idx_all, list(cs_global), zy, target)


def full_rows(hidden_rows, weight_shard, col_start, rank, all_gather):
    """Full fp32 logit rows [F, C] of the listed rows: this rank's columns,
    all-gathered (padded to the widest shard)."""
    widths = [col_start[q + 1] - col_start[q] for q in range(len(col_start) - 1)]
    mine = torch.full((hidden_rows.shape[0], max(widths)), float("-inf"), dtype=torch.float32,
                      device=hidden_rows.device)
    mine[:, : widths[rank]] = _logits_chunk(hidden_rows, weight_shard)
    parts = all_gather(mine)  # [world, F, wmax]
    return torch.cat([parts[q, :, : widths[q]] for q in range(len(widths))], dim=1)


def backward_parts(hidden, weight_shard, c0, target, kappa, sup_cols, scale, go, rows=None, g_rows=None,
                   need_dh=True, need_dw=True):
    """Step 4 on one rank before the all-reduce: (dhidden part [B, D] fp32 or
    None, dweight of the local classes or None).  rows / g_rows: the rows
    solved from their full logits and their unscaled dense gradient [F, C]."""
    fw = ext()
    C_local = weight_shard.shape[0]
    dH = dW = None
    gr = None
    if rows is not None:
        gr = (g_rows[:, c0:c0 + C_local] * (go * scale)).float()
    if need_dh:
        dH = fw.sparse_grad_hidden_shard(weight_shard, c0, sup_cols, kappa, target, scale, go, False)
        if gr is not None:
            dH[rows] += gr @ weight_shard.float()
    if need_dw:
        dW = torch.zeros(weight_shard.shape, dtype=weight_shard.dtype, device=weight_shard.device)
        keys = torch.sort(fw.weight_grad_keys_shard(sup_cols, kappa, target, c0, C_local)).values
        fw.segment_grad_weight(hidden, keys, kappa, scale, go, False, dW)
        if gr is not None:
            dW += (gr.t() @ hidden[rows].float()).to(dW.dtype)
    return dH, dW


def _all_gather(t, group):
    world = dist.get_world_size(group)
    out = torch.empty((world,) + tuple(t.shape), dtype=t.dtype, device=t.device)
    dist.all_gather_into_tensor(out, t.contiguous(), group=group)
    return out


class _VocabParallelLMHead(torch.autograd.Function):
    @staticmethod
    def forward(ctx, hidden, weight_shard, target, col_start, scale, group, n, K, fused):
        fw = ext()
        world, rank = dist.get_world_size(group), dist.get_rank(group)
        c0 = col_start[rank]
        B = hidden.shape[0]
        cs_local = local_chunk_starts(weight_shard.shape[0], n, fused)
        summ, lidx, zy, status = scan_phase(hidden, weight_shard, target, c0, cs_local, K, fused)
        summ_all = _all_gather(summ, group).reshape(-1, B, 4 + K)
        lidx_all = _all_gather(lidx, group).reshape(-1, B, K)
        dist.all_reduce(zy, group=group)
        H, kappa, loss_rows, sup_cols, fb_rows, fb_count = solve_phase(
            summ_all, lidx_all, global_chunk_starts(col_start, n, fused), zy, target)
        out = fw.loss_reduce(loss_rows, float(scale))
        # one small exchange after the step's work is queued: the exact-path
        # row count (the same on every rank) and any rank's timeout bit
        flags = torch.cat([fb_count, status])
        dist.all_reduce(flags, op=dist.ReduceOp.MAX, group=group)
        nfb, st = flags.tolist()
        if st & STATUS_TIMEOUT:
            raise RuntimeError("fw_lmhead_fused_scan: a bounded on-chip wait timed out")
        rows = g_rows = None
        if nfb:  # rare: rows solved from their full logit rows; their losses were 0 in `out`
            rows = fb_rows[:nfb].long().sort().values
            zf = full_rows(hidden[rows], weight_shard, col_start, rank, lambda t: _all_gather(t, group))
            g_rows, h, l, k = fw.fused_fwd_bwd(zf, target[rows], 1.0, None)
            loss_rows[rows] = l
            H[rows] = h
            out = out + (l.double().sum() * scale).float()
        ctx.save_for_backward(hidden, weight_shard, target, kappa, sup_cols)
        ctx.rows, ctx.g_rows, ctx.scale, ctx.c0, ctx.group = rows, g_rows, float(scale), c0, group
        return out if hidden.dtype == torch.float32 else out.to(hidden.dtype)

    @staticmethod
    def backward(ctx, g):
        hidden, weight_shard, target, kappa, sup_cols = ctx.saved_tensors
        go = g.float().reshape(1)
        args = (hidden, weight_shard, ctx.c0, target, kappa, sup_cols, ctx.scale, go, ctx.rows, ctx.g_rows)
        dH = dW = work = None
        if ctx.needs_input_grad[0]:
            dH, _ = backward_parts(*args, need_dh=True, need_dw=False)
            # fp32 partial sums of every rank's classes, summed while dweight is computed
            work = dist.all_reduce(dH, group=ctx.group, async_op=True)
        if ctx.needs_input_grad[1]:
            _, dW = backward_parts(*args, need_dh=False, need_dw=True)
        if work is not None:
            work.wait()
            dH = dH.to(hidden.dtype)
        return dH, dW, None, None, None, None, None, None, None


def vocab_parallel_lm_head_loss(hidden, weight_shard, target, col_start=None, reduction="mean", group=None,
                                K=DEFAULT_K, impl="auto"):
    """Mean/sum FW loss of logits = hidden @ weight^T where the rows of weight
    (the classes) are split across the ranks of `group`.

    hidden [B, D] and target [B] (global class ids) are the same on every
    rank; weight_shard [C_q, D] holds classes col_start[rank] ..
    col_start[rank + 1] (default: the shards' sizes all-gathered, in rank
    order).  hidden / weight_shard: CUDA, both float32 or both bfloat16.
    impl: "fused" (bf16 on sm_100: tcgen05 kernel), "staged" (GEMM per chunk)
    or "auto".  Every rank must call it with the same B, K and impl.  Returns
    the loss (equal on all ranks); backward gives hidden.grad (all-reduced)
    and weight_shard.grad (this rank's classes)."""
    if reduction not in ("mean", "sum"):
        raise ValueError(f"Invalid reduction mode: {reduction}")
    if impl not in ("staged", "fused", "auto"):
        raise ValueError(f"Invalid impl: {impl}")
    if not (hidden.is_cuda and weight_shard.is_cuda and hidden.dim() == 2 and weight_shard.dim() == 2):
        raise TypeError("vocab_parallel_lm_head_loss: hidden [B, D] and weight_shard [C_q, D] must be CUDA matrices")
    if hidden.dtype != weight_shard.dtype or hidden.dtype not in (torch.float32, torch.bfloat16):
        raise TypeError("vocab_parallel_lm_head_loss: hidden and weight_shard must both be float32 or bfloat16")
    if hidden.shape[1] != weight_shard.shape[1]:
        raise ValueError("vocab_parallel_lm_head_loss: hidden and weight_shard disagree on D")
    world = dist.get_world_size(group)
    if col_start is None:
        n = torch.tensor([weight_shard.shape[0]], dtype=torch.int64, device=hidden.device)
        sizes = _all_gather(n, group).reshape(-1).tolist()
        col_start = [0]
        for c in sizes:
            col_start.append(col_start[-1] + int(c))
    col_start = tuple(int(c) for c in col_start)
    if len(col_start) != world + 1:
        raise ValueError("col_start must have world_size + 1 entries")
    if K * world > LIST_CAP or world > MAX_CHUNKS:
        raise ValueError(f"vocab_parallel_lm_head_loss: K * world_size must be <= {LIST_CAP} and world_size <= "
                         f"{MAX_CHUNKS}")
    B = hidden.shape[0]
    scale = (1.0 / B if B else float("nan")) if reduction == "mean" else 1.0
    hidden, weight_shard = hidden.contiguous(), weight_shard.contiguous()
    fused = impl != "staged" and _fused_ok(hidden, weight_shard)
    if impl == "fused" and not fused:
        raise TypeError("vocab_parallel_lm_head_loss(impl='fused'): needs bfloat16 hidden/weight, D % 8 == 0, "
                        "16-byte aligned data and an sm_100 GPU")
    sms = torch.cuda.get_device_properties(hidden.device).multi_processor_count
    n = chunks_per_rank(world, B, col_start, int(K), fused, sms)
    return _VocabParallelLMHead.apply(hidden, weight_shard, target, col_start, scale, group, n, int(K), fused)
