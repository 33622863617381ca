"""GPU parity of the float64 kernel (fw_fused_fwd_bwd_f64), called through
the C ABI (ctypes), against the float64 oracle (oracle.fw_oracle.solve_f64)
and the reference CPU kernel's float64 outputs
(tests/golden/reference_outputs_f64.npz).

Contract: kappa and the selected set bit-exact; the gradient bit-exact (it is
scale / kappa on the set and -scale at the label, both formed in fp64); H and
the loss to fp64 rounding: rtol 1e-12 against the oracle, rtol 1e-9 against
the reference, whose float64 branch sums unshifted logits.
"""
import os

import numpy as np
import pytest
import torch

import cases
from fwloss_b200 import FWLoss, capi, familywise_loss
from oracle import fw_oracle as O

pytestmark = pytest.mark.gpu

RTOL, ATOL = 1e-12, 1e-12
GOLDEN64 = np.load(os.path.join(os.path.dirname(__file__), "golden", "reference_outputs_f64.npz"))


def _to_dev64(z, y, ld=None, offset=0):
    """Device copies; ld > C pads the rows, offset moves the base pointer off
    its 16-byte alignment (both select the 8-byte access path)."""
    B, C = z.shape
    ld = C if ld is None else ld
    buf = torch.full((B * ld + offset + 2,), float("nan"), dtype=torch.float64, device="cuda")
    view = buf[offset:offset + B * ld].view(B, ld)[:, :C]
    view.copy_(torch.from_numpy(z))
    return view, torch.from_numpy(y).cuda()


def _fused64(z, y, scale, **kw):
    zt, yt = _to_dev64(z, y, **kw)
    st = torch.zeros(1, dtype=torch.int32, device="cuda")
    grad, H, loss, kappa = capi.fused_fwd_bwd(zt, yt, scale, status=st)
    torch.cuda.synchronize()
    assert grad.dtype == H.dtype == loss.dtype == torch.float64
    return dict(grad=grad.cpu().numpy(), H=H.cpu().numpy(), loss=loss.cpu().numpy(),
                kappa=kappa.cpu().numpy().astype(np.int64), status=int(st.item()))


def _check(out, ref, name):
    np.testing.assert_array_equal(out["kappa"], ref["kappa"], err_msg=f"{name}: kappa")
    np.testing.assert_array_equal(out["grad"], ref["grad"], err_msg=f"{name}: grad (support)")
    np.testing.assert_allclose(out["H"], ref["H"], rtol=RTOL, atol=ATOL, err_msg=f"{name}: H")
    np.testing.assert_allclose(out["loss"], ref["loss"], rtol=RTOL, atol=ATOL, err_msg=f"{name}: loss")


F64 = cases.f64_cases()


@pytest.mark.parametrize("name,gen", F64, ids=[n for n, _ in F64])
def test_f64_matches_oracle_and_reference(name, gen):
    z, y = gen()
    scale = 1.0 / len(y)
    ref = O.solve_f64(z, y, scale)
    out = _fused64(z, y, scale)
    _check(out, ref, name)
    assert out["status"] == 0
    assert cases.golden_inputs_match(GOLDEN64, name, z, y), f"{name}: inputs differ from the golden fixtures'"
    np.testing.assert_array_equal(out["kappa"], GOLDEN64[f"{name}/kappa_cpu64"], err_msg="kappa vs ref CPU")
    np.testing.assert_allclose(out["loss"], GOLDEN64[f"{name}/loss_cpu64"], rtol=1e-9, atol=1e-12)
    g = np.zeros(z.shape, np.float64)
    g[GOLDEN64[f"{name}/grad_cpu64_r"], GOLDEN64[f"{name}/grad_cpu64_c"]] = GOLDEN64[f"{name}/grad_cpu64_v"]
    np.testing.assert_allclose(out["grad"], g, rtol=1e-15, atol=0, err_msg="grad vs ref CPU")


@pytest.mark.parametrize("C", [3, 100, 1001, 1025, 3001, 40001])
@pytest.mark.parametrize("layout", ["padded", "offset"])
def test_f64_unaligned_rows(C, layout):
    z, y = cases.gauss64(5, C, seed=C)()
    kw = {"ld": C + 1} if layout == "padded" else {"offset": 1}
    _check(_fused64(z, y, 0.2, **kw), O.solve_f64(z, y, 0.2), f"C{C}/{layout}")


@pytest.mark.parametrize("name,gen", cases.f64_nonfinite_cases(), ids=[n for n, _ in cases.f64_nonfinite_cases()])
def test_f64_nonfinite_policy(name, gen):
    z, y = gen()
    ref = O.solve_f64(z, y, 0.5)
    out = _fused64(z, y, 0.5)
    np.testing.assert_array_equal(out["kappa"], ref["kappa"])
    np.testing.assert_array_equal(out["grad"], ref["grad"])
    np.testing.assert_array_equal(out["H"], ref["H"])          # NaN == NaN here
    np.testing.assert_allclose(out["loss"], ref["loss"], rtol=RTOL, atol=ATOL, equal_nan=True)
    assert out["status"] & 2


@pytest.mark.parametrize("C", [40, 5000])
def test_f64_label_out_of_range(C):
    z, y = cases.gauss64(4, C, seed=7)()
    y[0], y[2] = -1, C
    ref = O.solve_f64(z, y, 0.25)
    out = _fused64(z, y, 0.25)
    assert out["status"] & 1
    assert np.isnan(out["loss"][[0, 2]]).all() and np.isfinite(out["loss"][[1, 3]]).all()
    np.testing.assert_array_equal(out["grad"], ref["grad"])
    np.testing.assert_array_equal(out["kappa"], ref["kappa"])


@pytest.mark.parametrize("B,C", [(20000, 64), (3000, 2000)])
def test_f64_rows_looped_over(B, C):
    """More rows than resident CTAs: each team loops over rows."""
    z, y = cases.gauss64(B, C, seed=B)()
    _check(_fused64(z, y, 1.0 / B), O.solve_f64(z, y, 1.0 / B), f"B{B}")


def test_f64_deterministic_and_empty():
    z, y = cases.fine64(4, 3000, 1e-4, seed=3)()
    a = _fused64(z, y, 0.25)
    b = _fused64(z, y, 0.25)
    for k in ("grad", "H", "loss", "kappa"):
        np.testing.assert_array_equal(a[k], b[k])
    e = torch.empty((0, 17), dtype=torch.float64, device="cuda")
    grad, H, loss, kappa = capi.fused_fwd_bwd(e, torch.empty(0, dtype=torch.int64, device="cuda"), 1.0)
    assert grad.shape == (0, 17) and H.numel() == 0


@pytest.mark.parametrize("reduction", ["mean", "sum", "none"])
@pytest.mark.parametrize("C", [100, 5000])
def test_f64_familywise_loss_autograd(reduction, C):
    z, y = cases.gauss64(64, C, seed=C + 1)()
    B = len(y)
    zt = torch.from_numpy(z).cuda().requires_grad_(True)
    loss = familywise_loss(zt, torch.from_numpy(y).cuda(), reduction)
    assert loss.dtype == torch.float64
    ref = O.solve_f64(z, y, 1.0)
    if reduction == "none":
        up = torch.linspace(-1.0, 2.0, B, dtype=torch.float64, device="cuda")
        loss.backward(up)
        np.testing.assert_allclose(loss.detach().cpu().numpy(), ref["loss"], rtol=RTOL, atol=ATOL)
        want = ref["grad"] * up.cpu().numpy()[:, None]
    else:
        s = 1.0 / B if reduction == "mean" else 1.0
        (loss * 3.0).backward()
        np.testing.assert_allclose(loss.item(), ref["loss"].sum() * s, rtol=1e-12)
        want = ref["grad"] * (3.0 * s)
    np.testing.assert_allclose(zt.grad.cpu().numpy(), want, rtol=1e-14, atol=1e-300)


def test_f64_fwloss_module_and_reduce():
    z, y = cases.gauss64(32, 700, seed=9)()
    zt = torch.from_numpy(z).cuda().requires_grad_(True)
    H, losses, mean, kappas = FWLoss(700)(zt, torch.from_numpy(y).cuda())
    ref = O.solve_f64(z, y)
    assert H.dtype == losses.dtype == mean.dtype == torch.float64 and kappas.dtype == torch.int64
    np.testing.assert_array_equal(kappas.cpu().numpy(), ref["kappa"])
    np.testing.assert_allclose(H.cpu().numpy(), ref["H"], rtol=RTOL, atol=ATOL)
    mean.backward()
    np.testing.assert_allclose(zt.grad.cpu().numpy(), ref["grad"], rtol=1e-14, atol=1e-300)
    l = torch.from_numpy(np.random.default_rng(1).standard_normal(5001)).cuda()
    out = capi.loss_reduce(l, 0.5)
    assert out.dtype == torch.float64
    np.testing.assert_allclose(out.item(), 0.5 * l.cpu().numpy().sum(), rtol=1e-13)
