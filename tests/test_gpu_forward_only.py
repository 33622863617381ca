"""Forward-only path: fw_forward_rows / fw_forward_rows_f64 (through the C
ABI) and the autograd layer when no gradient can be asked for (under
torch.no_grad, or logits that do not require grad).

The forward-only kernels run the same threshold search as the fused
forward+backward, so H, loss and kappa must be bit-identical to the fused
kernel's on the same inputs, at every tier (register rows, CTA rows,
clusters, dense radix rows) and element type; kappa is also checked against
the oracle.  They write nothing of the logits' size."""
import numpy as np
import pytest
import torch

import cases
from fwloss_b200 import FWLoss, capi, familywise_loss, fw_rows, workloads
from oracle import fw_oracle as O

pytestmark = pytest.mark.gpu

PARITY = dict(cases.parity_cases())
NAMES = ["gauss_C1", "gauss_C37", "gauss_C128", "gauss_C1000", "gauss_C2048", "gauss_mid_C2049",
         "gauss_mid_C32000", "gauss_mid_C100000", "ties_C128", "ties_C5000", "const_C40000",
         "dense_s1e-3_C1000", "dense_s1e-3_C40000", "dense_s1e-2_C100000", "exact_ties", "neginf_C12000",
         "zeros_C9000", "mag1e30_C5000"]
DTYPES = {"f32": torch.float32, "bf16": torch.bfloat16, "f16": torch.float16, "f64": torch.float64}


def _both(z, y):
    st1 = torch.zeros(1, dtype=torch.int32, device=z.device)
    st2 = torch.zeros(1, dtype=torch.int32, device=z.device)
    _, H1, l1, k1 = capi.fused_fwd_bwd(z, y, 1.0, status=st1)
    H2, l2, k2 = capi.forward_rows(z, y, status=st2)
    torch.cuda.synchronize()
    return [t.cpu().numpy() for t in (H1, l1, k1, st1, H2, l2, k2, st2)]


@pytest.mark.parametrize("dtype", list(DTYPES))
@pytest.mark.parametrize("name", NAMES)
def test_forward_rows_equals_fused(name, dtype):
    z32, y = PARITY[name]()
    z = torch.from_numpy(z32).to(DTYPES[dtype]).cuda()
    H1, l1, k1, s1, H2, l2, k2, s2 = _both(z, torch.from_numpy(y).cuda())
    np.testing.assert_array_equal(k2, k1)
    np.testing.assert_array_equal(H2, H1)
    np.testing.assert_array_equal(l2, l1)
    assert s1[0] == s2[0]
    if dtype == "f32":
        np.testing.assert_array_equal(k2, O.solve(z32, y)["kappa"])


@pytest.mark.parametrize("name,gen", cases.nonfinite_cases(), ids=[n for n, _ in cases.nonfinite_cases()])
def test_forward_rows_nonfinite_policy(name, gen):
    z32, y = gen()
    H1, l1, k1, s1, H2, l2, k2, s2 = _both(torch.from_numpy(z32).cuda(), torch.from_numpy(y).cuda())
    np.testing.assert_array_equal(k2, k1)
    np.testing.assert_array_equal(H2, H1)
    np.testing.assert_array_equal(l2, l1)
    assert s1[0] == s2[0] and (s2[0] & capi.FWB_STATUS_NONFINITE)


@pytest.mark.parametrize("C", [100, 1000, 3001, 40000])
def test_forward_rows_padded_and_sliced_rows(C):
    """Row stride > C (a column slice of a wider matrix)."""
    z32, y = cases.gauss(9, C, 1.0, seed=300 + C)()
    wide = torch.full((9, C + 5), float("nan"), device="cuda")
    wide[:, :C] = torch.from_numpy(z32).cuda()
    H1, l1, k1, _, H2, l2, k2, _ = _both(wide[:, :C], torch.from_numpy(y).cuda())
    np.testing.assert_array_equal(k2, k1)
    np.testing.assert_array_equal(H2, H1)
    np.testing.assert_array_equal(k2, O.solve(z32, y)["kappa"])


@pytest.mark.parametrize("name", ["cfg1", "cfg2", "cfg3"])
def test_forward_rows_reduced_configs(name):
    z, y = workloads.make(name, rows={"cfg1": 512, "cfg2": 64, "cfg3": 2048}[name])
    H1, l1, k1, _, H2, l2, k2, _ = _both(z.cuda(), y.cuda())
    np.testing.assert_array_equal(k2, k1)
    np.testing.assert_array_equal(H2, H1)
    np.testing.assert_array_equal(l2, l1)


@pytest.mark.parametrize("reduction", ["mean", "sum", "none"])
@pytest.mark.parametrize("dtype", ["f32", "bf16", "f64"])
def test_autograd_layer_without_gradient(reduction, dtype):
    """familywise_loss under torch.no_grad and on logits that do not require
    grad gives the values of the differentiable call, with no graph."""
    z, y = workloads.make("cfg2", rows=48)
    zd = z.to(DTYPES[dtype]).cuda()
    yd = y.cuda()
    ref = familywise_loss(zd.clone().requires_grad_(True), yd, reduction=reduction).detach()
    with torch.no_grad():
        a = familywise_loss(zd.clone().requires_grad_(True), yd, reduction=reduction)
    b = familywise_loss(zd, yd, reduction=reduction)
    torch.cuda.synchronize()
    for out in (a, b):
        assert not out.requires_grad and out.grad_fn is None
        assert out.dtype == ref.dtype and out.shape == ref.shape
        assert torch.equal(out, ref)


def test_fwloss_module_in_evaluation():
    """FWLoss on logits without grad (evaluation) returns the same H, losses,
    mean and kappas as with grad."""
    z, y = workloads.make("cfg1", rows=256)
    zd, yd = z.cuda(), y.cuda()
    fw = FWLoss(z.shape[1])
    Hg, lg, mg, kg = fw(zd.clone().requires_grad_(True), yd)
    He, le, me, ke = fw(zd, yd)
    assert not le.requires_grad and not me.requires_grad
    assert torch.equal(He, Hg) and torch.equal(le, lg.detach()) and torch.equal(ke, kg)
    assert torch.equal(me, mg.detach())
    losses, H, kappa = fw_rows(zd, yd)
    assert torch.equal(kappa.long(), kg) and torch.equal(H, Hg)
