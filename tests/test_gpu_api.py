"""GPU tests of the Python-facing drop-in APIs: the `fw_radix_cuda` module
(same four functions as the reference's extension, src/cuda/binding.cpp:8-13),
`familywise_loss` (as src/cpu/fwcpp.py) and `FWLoss` (as
reference_impl.FWLoss), checked against the oracle, the golden reference
outputs and, where it is cheap, the reference's own Python code semantics
re-expressed by the oracle."""
import numpy as np
import pytest
import torch

import cases
from fwloss_b200 import FWLoss, familywise_loss, fw_rows, workloads
from fwloss_b200._native import ext
from oracle import fw_oracle as O

pytestmark = pytest.mark.gpu
RTOL, ATOL = 1e-5, 1e-6


def _inputs(name, rows):
    z, y = workloads.make(name, rows=rows)
    return z.cuda(), y.cuda(), z.numpy(), y.numpy()


@pytest.mark.parametrize("name,rows", [("cfg0", 256), ("cfg1", 512), ("cfg3", 1024)])
def test_legacy_small_pair(name, rows):
    import fw_radix_cuda

    z, y, zn, yn = _inputs(name, rows)
    ref = O.solve(zn, yn)
    H, losses, mean, kappa, selected = fw_radix_cuda.fw_forward_small(z, y)
    assert H.dtype == torch.float32 and losses.dtype == torch.float32 and mean.dim() == 0
    assert kappa.dtype == torch.int32 and selected.dtype == torch.bool and selected.shape == z.shape
    grad = fw_radix_cuda.fw_backward_small(y, selected, kappa)
    np.testing.assert_array_equal(kappa.cpu().numpy(), ref["kappa"])
    np.testing.assert_array_equal(selected.cpu().numpy(), ref["mask"])
    np.testing.assert_allclose(losses.cpu().numpy(), ref["loss"], rtol=RTOL, atol=ATOL)
    np.testing.assert_allclose(mean.item(), ref["loss"].mean(), rtol=RTOL, atol=ATOL)
    np.testing.assert_allclose(grad.cpu().numpy(), ref["grad"], rtol=RTOL, atol=ATOL)


@pytest.mark.parametrize("name,rows", [("cfg2", 128), ("cfg4", 16)])
def test_legacy_large_pair(name, rows):
    import fw_radix_cuda

    z, y, zn, yn = _inputs(name, rows)
    ref = O.solve(zn, yn)
    out = fw_radix_cuda.fw_forward(z, y)
    assert len(out) == 7
    H, losses, mean, kappa, cbuf, cidx, ccnt = out
    assert cbuf.shape == z.shape and cidx.dtype == torch.int32 and ccnt.dtype == torch.int32
    grad = fw_radix_cuda.fw_backward(z, y, H, kappa, cbuf, cidx, ccnt)
    np.testing.assert_array_equal(kappa.cpu().numpy(), ref["kappa"])
    np.testing.assert_array_equal(ccnt.cpu().numpy(), ref["kappa"])
    np.testing.assert_allclose(losses.cpu().numpy(), ref["loss"], rtol=RTOL, atol=ATOL)
    np.testing.assert_allclose(grad.cpu().numpy(), ref["grad"], rtol=RTOL, atol=ATOL)


def test_legacy_checks_raise():
    import fw_radix_cuda

    with pytest.raises(RuntimeError):
        fw_radix_cuda.fw_forward_small(torch.randn(4, 10), torch.zeros(4, dtype=torch.long))
    with pytest.raises(RuntimeError):
        fw_radix_cuda.fw_forward(torch.randn(4, 10, device="cuda").double(),
                                 torch.zeros(4, dtype=torch.long, device="cuda"))
    with pytest.raises(RuntimeError):
        fw_radix_cuda.fw_forward_small(torch.randn(4, 10, device="cuda"),
                                       torch.zeros(3, dtype=torch.long, device="cuda"))


@pytest.mark.parametrize("reduction", ["mean", "sum", "none"])
@pytest.mark.parametrize("C", [100, 1000, 32000])
def test_familywise_loss_autograd(reduction, C):
    zn, yn = cases.gauss(48, C, 1.0, seed=C + 7)()
    B = zn.shape[0]
    scale = 1.0 / B if reduction == "mean" else 1.0
    ref = O.solve(zn, yn, scale)
    z = torch.from_numpy(zn).cuda().requires_grad_(True)
    y = torch.from_numpy(yn).cuda()
    out = familywise_loss(z, y, reduction=reduction)
    if reduction == "none":
        assert out.shape == (B,)
        np.testing.assert_allclose(out.detach().cpu().numpy(), ref["loss"], rtol=RTOL, atol=ATOL)
        w = torch.linspace(0.5, 2.0, B, device="cuda")
        (out * w).sum().backward()
        np.testing.assert_allclose(z.grad.cpu().numpy(), ref["grad"] * w.cpu().numpy()[:, None],
                                   rtol=RTOL, atol=ATOL)
    else:
        assert out.dim() == 0
        want = ref["loss"].mean() if reduction == "mean" else ref["loss"].sum()
        np.testing.assert_allclose(out.item(), want, rtol=RTOL, atol=ATOL)
        (2.5 * out).backward()
        np.testing.assert_allclose(z.grad.cpu().numpy(), 2.5 * ref["grad"], rtol=RTOL, atol=ATOL)


def test_fwloss_module_matches_reference_outputs():
    zn, yn = workloads.make("cfg1", rows=300)
    zn, yn = zn.numpy(), yn.numpy()
    ref = O.solve(zn, yn)
    z = torch.from_numpy(zn).cuda().requires_grad_(True)
    y = torch.from_numpy(yn).cuda()
    H, losses, mean, kappas = FWLoss(zn.shape[1], reduction="mean", device="cuda")(z, y)
    assert kappas.dtype == torch.int64 and H.dtype == torch.float32
    np.testing.assert_array_equal(kappas.cpu().numpy(), ref["kappa"])
    np.testing.assert_allclose(H.detach().cpu().numpy(), ref["H"], rtol=RTOL, atol=ATOL)
    np.testing.assert_allclose(losses.detach().cpu().numpy(), ref["loss"], rtol=RTOL, atol=ATOL)
    mean.backward()
    np.testing.assert_allclose(z.grad.cpu().numpy(), ref["grad"], rtol=RTOL, atol=ATOL)
    # sum and none reductions
    z.grad = None
    s = FWLoss(zn.shape[1], reduction="sum")(z, y)
    s.backward()
    np.testing.assert_allclose(z.grad.cpu().numpy(), ref["grad"] * len(yn), rtol=RTOL, atol=ATOL)
    n = FWLoss(zn.shape[1], reduction="none")(z, y)
    assert n.shape == (len(yn),)


def test_no_cpu_fallback():
    with pytest.raises(TypeError):
        familywise_loss(torch.randn(4, 10), torch.zeros(4, dtype=torch.long))


def test_status_word_and_rows():
    zn, yn = cases.gauss(8, 700, 1.0, seed=3)()
    yn = yn.copy()
    yn[0] = 700
    st = torch.zeros(1, dtype=torch.int32, device="cuda")
    losses, H, kappa = fw_rows(torch.from_numpy(zn).cuda(), torch.from_numpy(yn).cuda(), 1.0, st)
    torch.cuda.synchronize()
    assert st.item() & 1
    assert torch.isnan(losses[0]) and torch.isfinite(losses[1:]).all()
    assert ext().version() == "0.1.0"
