"""Row-sharded FW loss through the public API
(fwloss_b200.distributed.sharded_familywise_loss) over NCCL, one process per
GPU: in a one-rank group on any GPU box and across two and four GPUs where the
box has them.  The checks themselves are in tests/rows_sharded_worker.py (loss and
gradient rows against familywise_loss on the whole batch, the forward-only
path, and the step captured in a CUDA graph with its NCCL all-reduce)."""
import os
import socket
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu

WORKER = os.path.join(os.path.dirname(__file__), "rows_sharded_worker.py")


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


@pytest.mark.parametrize("nproc", [1, 2, 4])
def test_rows_sharded_nccl(nproc):
    if torch.cuda.device_count() < nproc:
        pytest.skip(f"needs {nproc} GPUs")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", str(nproc),
           "--master-addr", "127.0.0.1", "--master-port", str(_free_port()), WORKER]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert r.stdout.count("ok=True") == nproc, r.stdout[-3000:]
