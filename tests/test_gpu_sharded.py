"""Class-sharded FW loss (rows split by columns across ranks).

The protocol is emulated on one GPU: every "rank" runs the real kernels on
its column shard, and the collectives become stacks of the ranks' tensors.
The result must equal the unsharded fused kernel (and the oracle): the same
kappa and H on every rank, the gradient shards tiling the full gradient, and
the per-row losses summing to the full losses.  A real two-process NCCL run
is in test_two_gpu_nccl (needs two GPUs)."""
import os
import subprocess
import sys

import numpy as np
import pytest
import torch

import cases
from fwloss_b200 import capi, workloads
from fwloss_b200.sharded import _solve_full_rows, even_col_start, scan_phase, solve_phase
from fwloss_b200._native import ext
from oracle import fw_oracle as O

pytestmark = pytest.mark.gpu
RTOL, ATOL = 1e-5, 1e-6


def emulate(z, y, col_start, scale, K):
    """Runs the sharded protocol for all ranks on one device."""
    world = len(col_start) - 1
    shards = [z[:, col_start[q]:col_start[q + 1]].contiguous() for q in range(world)]
    scans = [scan_phase(s, K) for s in shards]
    gathered = torch.stack([sc[1] for sc in scans])
    out = []
    for q in range(world):
        grad, _, local_idx = scans[q]
        H, kappa, loss_part, fb_rows, fb_count = solve_phase(gathered, shards[q], y, col_start, q, scale, grad,
                                                             local_idx)
        nfb = int(fb_count.item())
        if nfb:
            rows = fb_rows[:nfb].long().sort().values
            widths = [col_start[r + 1] - col_start[r] for r in range(world)]

            def all_gather(mine, rows=rows, widths=widths):
                parts = []
                for r in range(world):
                    blk = torch.full_like(mine, float("-inf"))
                    blk[:, : widths[r]] = shards[r][rows]
                    parts.append(blk)
                return torch.stack(parts)

            _solve_full_rows(shards[q], y, col_start, q, scale, all_gather, rows, grad, H, kappa, loss_part)
        out.append((grad, H, kappa, loss_part, nfb))
    return out


def check(z_np, y_np, col_start, K=32, scale=None):
    B = len(y_np)
    scale = 1.0 / B if scale is None else scale
    z = torch.from_numpy(z_np).cuda()
    y = torch.from_numpy(y_np).cuda()
    ref = O.solve(z_np, y_np, scale)
    out = emulate(z, y, col_start, scale, K)
    torch.cuda.synchronize()
    grads = [o[0].cpu().numpy() for o in out]
    np.testing.assert_allclose(np.concatenate(grads, axis=1), ref["grad"], rtol=RTOL, atol=ATOL)
    for grad, H, kappa, loss_part, nfb in out:
        np.testing.assert_array_equal(kappa.cpu().numpy(), ref["kappa"])
        np.testing.assert_allclose(H.cpu().numpy(), ref["H"], rtol=RTOL, atol=ATOL)
    losses = sum(o[3].double().cpu().numpy() for o in out)
    fin = np.isfinite(ref["loss"])
    np.testing.assert_allclose(losses[fin], ref["loss"][fin], rtol=RTOL, atol=ATOL)
    return max(o[4] for o in out)


@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("name", ["gauss_mid_C10000", "gauss_mid_C32000", "gauss_mid_C100000", "ties_C5000",
                                  "outlier_C50000", "neginf_C12000", "mag1e30_C5000", "zeros_C9000",
                                  "exact_ties", "gauss_C1000", "twolevel_C700"])
def test_sharded_matches_unsharded(world, name):
    z, y = dict(cases.parity_cases())[name]()
    if z.shape[1] < world:
        pytest.skip("fewer classes than shards")
    check(z, y, even_col_start(z.shape[1], world))


def test_sharded_uneven_widths_and_cfg4():
    z, y = workloads.make("cfg4", rows=16)
    z, y = z.numpy(), y.numpy()
    C = z.shape[1]
    check(z, y, [0, 1000, 40000, 40001, 90000, C])
    check(z, y, even_col_start(C, 8))


def test_sharded_dense_rows_take_the_exact_path():
    z, y = cases.gauss(6, 40000, 1e-3, seed=5)()  # supports of thousands of entries
    nfb = check(z, y, even_col_start(40000, 4), K=16)
    assert nfb == 6


def test_sharded_nonfinite_rows():
    z, y = dict(cases.nonfinite_cases())["nonfinite_C3000"]()
    C = z.shape[1]
    col_start = even_col_start(C, 4)
    zt, yt = torch.from_numpy(z).cuda(), torch.from_numpy(y).cuda()
    ref = O.solve(z, y, 1.0)
    out = emulate(zt, yt, col_start, 1.0, 32)
    grads = np.concatenate([o[0].cpu().numpy() for o in out], axis=1)
    np.testing.assert_allclose(grads, ref["grad"], rtol=RTOL, atol=ATOL)
    for o in out:
        np.testing.assert_array_equal(o[2].cpu().numpy(), ref["kappa"])
        np.testing.assert_array_equal(o[1].cpu().numpy(), ref["H"])


WORKER = os.path.join(os.path.dirname(__file__), "sharded_worker.py")


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_gpu_nccl():
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
           "--master-addr", "127.0.0.1", "--master-port", "29533", WORKER]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
