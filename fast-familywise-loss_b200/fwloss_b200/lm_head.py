"""FW loss on top of an LM head without materialising [B, C] logits or their
gradient.

    from fwloss_b200.lm_head import fw_lm_head_loss
    loss = fw_lm_head_loss(hidden, weight, target)     # hidden [B, D], weight [C, D]
    loss.backward()                                    # hidden.grad, weight.grad

Forward: the logits are produced one column chunk at a time by the GEMM
(cuBLAS through torch.mm, fp32 output; bf16 inputs are accumulated in fp32)
and each chunk is reduced at once to per-row summaries by the fused kernel
(chunk max, the chunk's own support, up to K values) -- only one chunk of
logits exists at a time.  The chunk summaries are then combined per row
(fw_chunks_solve), which gives H, kappa, the loss and the support columns.

Backward: the logit gradient of a row has kappa + 1 non-zeros
(scale / kappa on the support, -scale at the label), so
dhidden = G W and dweight = G^T hidden become gathers and scatter-adds of
kappa + 1 rows per sample (fw_sparse_grad_hidden / fw_sparse_grad_weight)
instead of two dense [B, C] x [C, D] GEMMs.  dweight is written row by row
(fw_segment_grad_weight): the non-zeros are sorted by column and each touched
row of dweight sums its contributions in a fixed order, so the result is
deterministic and only touched rows are written.

Rows where a chunk's own support exceeds K entries (near-constant logits) are
solved exactly from their full logit rows, and their gradient rows are
applied densely; counting them costs one 4-byte device-to-host read per step.

impl="fused" (bf16 only) replaces the chunk GEMMs and scans by one
tensor-core kernel (fw_lmhead_fused_scan, sm_100a tcgen05) whose epilogue
writes the same chunk summaries straight from the accumulators: no logit
chunk is written to memory.  impl="staged" is the GEMM + scan form above;
impl="auto" (the default) picks the fused kernel where it applies (B200,
B = 8192, D = 4096, C = 128256: 7.45 ms per forward+backward fused, 8.77 ms
staged).
"""
import torch

from ._native import ext
from .sharded import even_col_start

DEFAULT_K = 16
FUSED_TILE = 256  # column tile of the fused kernel: chunk starts are multiples of it
DEFAULT_IMPL = "auto"
STATUS_TIMEOUT = 4


def tile_col_start(num_classes, nchunks, tile=FUSED_TILE):
    """Chunk offsets whose starts are multiples of `tile`: the column tiles
    are dealt out evenly (chunk sizes differ by at most one tile), at most
    nchunks chunks, fewer when there are fewer tiles."""
    C = int(num_classes)
    tiles = -(-C // tile)
    n = max(1, min(int(nchunks), tiles))
    base, extra = divmod(tiles, n)
    out, t = [0], 0
    for q in range(n):
        t += base + (1 if q < extra else 0)
        out.append(min(t * tile, C))
    return out


def fused_nchunks(batch, num_classes, sms, max_chunks=16, tile=FUSED_TILE):
    """Chunk count for the fused kernel.  Its persistent CTAs (one per SM)
    take (128-row block, chunk) work items of equal size round-robin, so the
    last round leaves SMs idle unless the item count is close to a multiple
    of the SM count: pick the count in [1, max_chunks] with the best filled
    fraction of the rounds, the largest such count on ties (within 1 %):
    smaller items also keep the weight columns that run concurrently in L2
    (B200, B = 8192, C = 128256: 16 chunks 6.4 ms, 9 chunks 6.85 ms, both
    97 % filled)."""
    mblocks = -(-int(batch) // 128)
    tiles = -(-int(num_classes) // tile)
    best, best_eff = 1, -1.0
    for n in range(1, max(1, min(max_chunks, tiles)) + 1):
        items = mblocks * n
        per_item = -(-tiles // n)  # the largest item's tiles
        rounds = -(-items // sms)
        eff = (mblocks * tiles) / (rounds * sms * per_item)
        if eff >= best_eff - 0.01:
            if eff > best_eff:
                best_eff = eff
            best = n
    return best


def _fused_ok(hidden, weight):
    return (hidden.dtype == torch.bfloat16 and weight.dtype == torch.bfloat16 and hidden.shape[1] % 8 == 0
            and hidden.data_ptr() % 16 == 0 and weight.data_ptr() % 16 == 0
            and torch.cuda.get_device_capability(hidden.device) == (10, 0))


def _logits_chunk(hidden, w_chunk):
    if hidden.dtype == torch.float32:
        return torch.mm(hidden, w_chunk.t())
    return torch.mm(hidden, w_chunk.t(), out_dtype=torch.float32)


_SIDE = {}


def _side_stream(dev):
    if dev not in _SIDE:
        _SIDE[dev] = torch.cuda.Stream(dev)
    return _SIDE[dev]


def _full_logits(hidden_rows, weight):
    return _logits_chunk(hidden_rows, weight)


def chunk_summaries(hidden, weight, target, col_start, K, fused, c0=0):
    """Per-(chunk, row) summary records of logits = hidden @ weight^T for the
    column chunks col_start (offsets into weight's rows).  weight holds the
    classes [c0, c0 + C) of the model (c0 = 0 for a whole weight); target
    carries global class ids.  Returns (summaries [n, B, 4 + K],
    local_idx [n, B, K], zy [B], status [1]) where zy[r] is the label logit
    when the label lies in this weight's classes and 0 otherwise."""
    fw = ext()
    B = hidden.shape[0]
    nchunks = len(col_start) - 1
    dev = hidden.device
    summaries = torch.empty((nchunks, B, 4 + K), dtype=torch.int32, device=dev)
    local_idx = torch.empty((nchunks, B, K), dtype=torch.int32, device=dev)
    zy = torch.zeros(B, dtype=torch.float32, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    if fused:
        y_local = target - c0 if c0 else target
        fw.lmhead_fused_scan(hidden, weight, y_local, col_start, summaries, local_idx, zy, status)
    else:
        # The GEMM of chunk q+1 (tensor cores) runs while chunk q is being
        # summarised on a second stream (HBM-bound); a chunk's memory is
        # released only after its scan (record_stream).
        main = torch.cuda.current_stream(dev)
        side = _side_stream(dev)
        side.wait_stream(main)
        for q in range(nchunks):
            q0, q1 = col_start[q], col_start[q + 1]
            z = _logits_chunk(hidden, weight[q0:q1])
            ready = torch.cuda.Event()
            ready.record(main)
            with torch.cuda.stream(side):
                side.wait_event(ready)
                fw.shard_scan_into(z, K, summaries[q], local_idx[q])
                fw.label_logits(z, target, c0 + q0, zy)
            z.record_stream(side)
            del z
        main.wait_stream(side)
    return summaries, local_idx, zy, status


class _FWLMHead(torch.autograd.Function):
    @staticmethod
    def forward(ctx, hidden, weight, target, scale, nchunks, K, fused):
        fw = ext()
        C = weight.shape[0]
        col_start = tile_col_start(C, nchunks) if fused else even_col_start(C, nchunks)
        summaries, local_idx, zy, status = chunk_summaries(hidden, weight, target, col_start, K, fused)
        H, kappa, loss_rows, sup_cols, fb_rows, fb_count = fw.chunks_solve(summaries, local_idx, col_start, zy, target)
        out = fw.loss_reduce(loss_rows, float(scale))
        # one read after the step's work is queued: exact-path row count and
        # the fused kernel's status word
        nfb, st = torch.cat([fb_count, status]).tolist()
        if st & STATUS_TIMEOUT:
            raise RuntimeError("fw_lmhead_fused_scan: a bounded on-chip wait timed out")
        rows = g_rows = None
        if nfb:  # rare: rows solved from their full logit rows; their losses were 0 in `out`
            rows = fb_rows[:nfb].long().sort().values
            zf = _full_logits(hidden[rows], weight)
            g_rows, h, l, k = fw.fused_fwd_bwd(zf, target[rows], 1.0, None)
            loss_rows[rows] = l
            H[rows] = h
            out = out + (l.double().sum() * scale).float()
        ctx.save_for_backward(hidden, weight, target, kappa, sup_cols)
        ctx.rows, ctx.g_rows, ctx.scale = rows, g_rows, float(scale)
        return out if hidden.dtype == torch.float32 else out.to(hidden.dtype)

    @staticmethod
    def backward(ctx, g):
        fw = ext()
        hidden, weight, target, kappa, sup_cols = ctx.saved_tensors
        go = g.float().reshape(1)
        dH = dW = None
        if ctx.needs_input_grad[0]:
            dH = fw.sparse_grad_hidden(weight, sup_cols, kappa, target, ctx.scale, go, False)
        if ctx.needs_input_grad[1]:
            dW = torch.zeros(weight.shape, dtype=weight.dtype, device=weight.device)
            keys = torch.sort(fw.weight_grad_keys(sup_cols, kappa, target, weight.shape[0])).values
            fw.segment_grad_weight(hidden, keys, kappa, ctx.scale, go, False, dW)
        if ctx.rows is not None:  # rows solved from their full logits: dense gradient rows
            gr = ctx.g_rows * (go * ctx.scale)
            if dH is not None:
                dH[ctx.rows] = (gr @ weight.float()).to(dH.dtype)
            if dW is not None:
                dW += (gr.t() @ hidden[ctx.rows].float()).to(dW.dtype)
        return dH, dW, None, None, None, None, None


def fw_lm_head_loss(hidden, weight, target, reduction="mean", nchunks=None, K=DEFAULT_K, impl=None):
    """Mean/sum FW loss of logits = hidden @ weight^T.

    hidden [B, D] and weight [C, D]: CUDA, both float32 or both bfloat16;
    target [B] int64.  `nchunks` column chunks (default: chunks of ~16k
    classes, at most 16) bound the logit memory to B x C / nchunks fp32
    (staged form).  impl: "staged", "fused" (bf16, sm_100a; raises where it
    does not apply) or "auto" (fused where it applies); default DEFAULT_IMPL."""
    if reduction not in ("mean", "sum"):
        raise ValueError(f"Invalid reduction mode: {reduction}")
    impl = DEFAULT_IMPL if impl is None else impl
    if impl not in ("staged", "fused", "auto"):
        raise ValueError(f"Invalid impl: {impl}")
    if not (hidden.is_cuda and weight.is_cuda and hidden.dim() == 2 and weight.dim() == 2):
        raise TypeError("fw_lm_head_loss: hidden [B, D] and weight [C, D] must be CUDA matrices")
    if hidden.dtype != weight.dtype or hidden.dtype not in (torch.float32, torch.bfloat16):
        raise TypeError("fw_lm_head_loss: hidden and weight must both be float32 or both bfloat16")
    if hidden.shape[1] != weight.shape[1]:
        raise ValueError("fw_lm_head_loss: hidden and weight disagree on D")
    C = weight.shape[0]
    B = hidden.shape[0]
    scale = (1.0 / B if B else float("nan")) if reduction == "mean" else 1.0
    hidden, weight = hidden.contiguous(), weight.contiguous()
    fused = impl != "staged" and _fused_ok(hidden, weight)
    if impl == "fused" and not fused:
        raise TypeError("fw_lm_head_loss(impl='fused'): needs bfloat16 hidden/weight, D % 8 == 0, "
                        "16-byte aligned data and an sm_100 GPU")
    if nchunks is None:
        if fused:
            sms = torch.cuda.get_device_properties(hidden.device).multi_processor_count
            nchunks = fused_nchunks(B, C, sms, max_chunks=min(16, 256 // int(K)))
        else:
            nchunks = max(1, min(16, -(-C // 16384)))
    nchunks = max(1, min(int(nchunks), C, 16, 256 // int(K)))
    return _FWLMHead.apply(hidden, weight, target, scale, nchunks, int(K), fused)
