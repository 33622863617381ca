"""Vocabulary-parallel LM head (fwloss_b200.vocab_parallel).

The protocol is emulated on one GPU: every "rank" runs the real kernels on
its slice of the weight rows, and the collectives become concatenations and
sums of the ranks' tensors.  The loss and the gradients must equal the
one-GPU LM head on the whole weight (fw_lm_head_loss): the loss to fp32
rounding, dweight exactly (each class's rows are summed by the same kernel in
the same order), dhidden to the rounding of the summed fp32 partials.  A real
two-process NCCL run is in test_two_gpu_vocab_parallel (needs two GPUs)."""
import os
import subprocess
import sys

import numpy as np
import pytest
import torch

from fwloss_b200._native import ext
from fwloss_b200.lm_head import fw_lm_head_loss
from fwloss_b200.sharded import even_col_start
from fwloss_b200.vocab_parallel import (backward_parts, chunks_per_rank, global_chunk_starts, local_chunk_starts,
                                        scan_phase, solve_phase)

pytestmark = pytest.mark.gpu
WORKER = os.path.join(os.path.dirname(os.path.abspath(__file__)), "vocab_parallel_worker.py")


def make(B, D, C, seed, dtype=torch.bfloat16, temp=4.0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    hidden = (torch.randn(B, D, generator=g, device="cuda") / D ** 0.5 * temp).to(dtype)
    weight = torch.randn(C, D, generator=g, device="cuda").to(dtype)
    target = torch.randint(0, C, (B,), generator=g, device="cuda")
    return hidden, weight, target


def emulate(hidden, weight, target, world, K, fused, scale):
    """All ranks of one step on one device: (loss, dhidden fp32, dweight, kappa, nfb)."""
    fw = ext()
    B, C = hidden.shape[0], weight.shape[0]
    col_start = even_col_start(C, world)
    shards = [weight[col_start[q]:col_start[q + 1]].contiguous() for q in range(world)]
    sms = torch.cuda.get_device_properties(hidden.device).multi_processor_count
    n = chunks_per_rank(world, B, col_start, K, fused, sms)
    scans = [scan_phase(hidden, shards[q], target, col_start[q], local_chunk_starts(shards[q].shape[0], n, fused),
                        K, fused) for q in range(world)]
    assert all(int(s[3].item()) == 0 for s in scans)
    summ_all = torch.cat([s[0] for s in scans])
    lidx_all = torch.cat([s[1] for s in scans])
    zy = sum(s[2] for s in scans)
    H, kappa, loss_rows, sup_cols, fb_rows, fb_count = solve_phase(summ_all, lidx_all,
                                                                   global_chunk_starts(col_start, n, fused), zy,
                                                                   target)
    nfb = int(fb_count.item())
    rows = g_rows = None
    if nfb:
        rows = fb_rows[:nfb].long().sort().values
        zf = torch.cat([hidden[rows].float() @ s.float().t() for s in shards], dim=1)
        g_rows, h, l, k = fw.fused_fwd_bwd(zf, target[rows], 1.0, None)
        loss_rows[rows] = l
    loss = float(loss_rows.double().sum().item() * scale)
    go = torch.ones(1, device="cuda")
    parts = [backward_parts(hidden, shards[q], col_start[q], target, kappa, sup_cols, scale, go, rows, g_rows)
             for q in range(world)]
    dH = sum(p[0] for p in parts)
    dW = torch.cat([p[1] for p in parts])
    return loss, dH, dW, kappa, nfb


def one_gpu(hidden, weight, target, K, impl, reduction):
    h = hidden.clone().requires_grad_(True)
    w = weight.clone().requires_grad_(True)
    loss = fw_lm_head_loss(h, w, target, reduction=reduction, K=K, impl=impl)
    loss.backward()
    return loss, h.grad, w.grad


CASES = [
    # (B, D, C, world, dtype, impl)
    (200, 256, 5000, 2, torch.bfloat16, "fused"),
    (257, 512, 33000, 4, torch.bfloat16, "fused"),
    (130, 128, 12345, 2, torch.float32, "staged"),
    (96, 256, 20000, 4, torch.bfloat16, "staged"),
]


@pytest.mark.parametrize("B,D,C,world,dtype,impl", CASES)
def test_emulated_ranks_match_one_gpu(B, D, C, world, dtype, impl):
    K = 16
    hidden, weight, target = make(B, D, C, seed=B + C + world, dtype=dtype)
    fused = impl == "fused"
    loss, dH, dW, kappa, nfb = emulate(hidden, weight, target, world, K, fused, 1.0 / B)
    ref_loss, ref_dH, ref_dW = one_gpu(hidden, weight, target, K, impl, "mean")
    tol = 1e-5 if dtype == torch.float32 else 2e-2
    np.testing.assert_allclose(loss, ref_loss.float().item(), rtol=1e-5 if dtype == torch.float32 else 1e-2)
    np.testing.assert_allclose(dH.to(dtype).float().cpu().numpy(), ref_dH.float().cpu().numpy(), rtol=tol, atol=1e-6)
    np.testing.assert_array_equal(dW.float().cpu().numpy(), ref_dW.float().cpu().numpy())
    assert (kappa.cpu().numpy() >= 1).all() and nfb == 0


@pytest.mark.parametrize("impl", ["fused", "staged"])
def test_emulated_ranks_rows_needing_the_exact_path(impl):
    """All-zero hidden rows give constant logits: every chunk record
    overflows, and the rows are solved from their full logit rows, gathered
    from the ranks' columns."""
    B, D, C, world, K = 150, 128, 6000, 2, 8
    hidden, weight, target = make(B, D, C, seed=31)
    hidden[:4] = 0
    hidden[100:102] = 0
    loss, dH, dW, kappa, nfb = emulate(hidden, weight, target, world, K, impl == "fused", 1.0)
    assert nfb == 6
    ref_loss, ref_dH, ref_dW = one_gpu(hidden, weight, target, K, impl, "sum")
    np.testing.assert_allclose(loss, ref_loss.float().item(), rtol=1e-2)
    np.testing.assert_allclose(dH.to(hidden.dtype).float().cpu().numpy(), ref_dH.float().cpu().numpy(), rtol=2e-2,
                               atol=1e-5)
    np.testing.assert_allclose(dW.float().cpu().numpy(), ref_dW.float().cpu().numpy(), rtol=2e-2, atol=1e-5)


def test_shard_entry_points_skip_other_ranks_classes():
    """fw_sparse_grad_hidden_shard / fw_weight_grad_keys_shard: a rank's
    parts, summed over ranks, equal the whole-weight kernels."""
    fw = ext()
    B, D, C = 64, 96, 3000
    hidden, weight, target = make(B, D, C, seed=5, dtype=torch.float32)
    S = 6
    g = torch.Generator(device="cuda").manual_seed(6)
    sup = torch.randint(0, C, (B, S), generator=g, device="cuda", dtype=torch.int32)
    kappa = torch.randint(0, S + 1, (B,), generator=g, device="cuda", dtype=torch.int32)
    go = torch.tensor([0.75], device="cuda")
    whole = fw.sparse_grad_hidden(weight, sup, kappa, target, 0.5, go, False)
    cs = [0, 1000, 2200, C]
    part = sum(fw.sparse_grad_hidden_shard(weight[cs[q]:cs[q + 1]].contiguous(), cs[q], sup, kappa, target, 0.5, go,
                                           False) for q in range(3))
    np.testing.assert_allclose(part.cpu().numpy(), whole.cpu().numpy(), rtol=1e-5, atol=1e-6)
    keys = fw.weight_grad_keys(sup, kappa, target, C)
    local = [fw.weight_grad_keys_shard(sup, kappa, target, cs[q], cs[q + 1] - cs[q]) for q in range(3)]
    no_key = 0x7fffffffffffffff
    back = []
    for q in range(3):
        k = local[q][local[q] != no_key]
        back.append(k + (cs[q] << 32))  # local class ids back to global
    np.testing.assert_array_equal(np.sort(torch.cat(back).cpu().numpy()), np.sort(keys[keys != no_key].cpu().numpy()))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_gpu_vocab_parallel():
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
           "--master-addr", "127.0.0.1", "--master-port", "29541", WORKER]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
