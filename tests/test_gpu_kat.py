"""The reference's shipped known answers on the GPU path: for every
(distribution, sigma, K) of benchmarks/cpu_benchmarks/results/*.json the mean
support size over its 32 rows (`kbar`) must come out exactly, from inputs
replayed from the reference benchmark's own seed and draw order (tests/kat.py).
K runs from 10 to 1e6 and sigma from 1e-3 (kappa in the thousands: the dense
radix path) to 100 (kappa = 1)."""
import numpy as np
import pytest
import torch

import kat
from fwloss_b200 import capi

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("fname", sorted(kat.load().keys()))
def test_gpu_reproduces_reference_kbar(fname):
    entry = kat.load()[fname]
    bad = []
    for s, K, kbar, Z, y in kat.replay(entry):
        z = torch.from_numpy(Z).cuda()
        yt = torch.from_numpy(y).cuda()
        grad, H, loss, kappa = capi.fused_fwd_bwd(z, yt, 1.0 / len(y))
        k = kappa.cpu().numpy().astype(np.int64)
        if float(np.mean(k)) != kbar:
            bad.append((s, K, float(np.mean(k)), kbar))
        # the mask form and the gradient agree with kappa
        sel = (z > H[:, None]).sum(1).to(torch.int32)
        assert torch.equal(sel, kappa), (s, K)
        nz = (grad != 0).sum(1)
        assert int(nz.max()) <= int(kappa.max()) + 1
    assert not bad, bad
