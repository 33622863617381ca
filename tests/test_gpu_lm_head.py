"""LM-head FW loss (chunked logits, sparse backward) against the dense path:
logits = hidden @ weight^T materialised, the fused FW kernel on them, and
autograd through the GEMM.  The chunked forward sees the same logit values
(one GEMM per column chunk), so kappa and the loss match exactly up to GEMM
rounding; the sparse backward matches the dense one to fp32 rounding."""
import numpy as np
import pytest
import torch

from fwloss_b200 import familywise_loss
from fwloss_b200.lm_head import fw_lm_head_loss
from oracle import fw_oracle as O

pytestmark = pytest.mark.gpu


def dense_reference(hidden, weight, target, reduction):
    h = hidden.detach().clone().requires_grad_(True)
    w = weight.detach().clone().requires_grad_(True)
    z = h.float() @ w.float().t()  # bf16 values, fp32 GEMM (same values as bf16 x bf16 -> fp32)
    loss = familywise_loss(z, target, reduction=reduction)
    loss.backward()
    return loss.detach().float(), h.grad.float(), w.grad.float(), z.detach()


def make(B, D, C, dtype, seed, temp=4.0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    hidden = torch.randn(B, D, generator=g, device="cuda") / D ** 0.5 * temp
    weight = torch.randn(C, D, generator=g, device="cuda")
    target = torch.randint(0, C, (B,), generator=g, device="cuda")
    return hidden.to(dtype), weight.to(dtype), target


@pytest.mark.parametrize("dtype,tol", [(torch.float32, 2e-5), (torch.bfloat16, 2e-2)])
@pytest.mark.parametrize("B,D,C,nchunks", [(64, 256, 5000, 4), (128, 512, 32000, 2), (33, 128, 3001, 3),
                                           (256, 1024, 50000, 8)])
def test_lm_head_matches_dense(dtype, tol, B, D, C, nchunks):
    hidden, weight, target = make(B, D, C, dtype, seed=B + C)
    ref_loss, ref_dh, ref_dw, z = dense_reference(hidden, weight, target, "mean")
    h = hidden.clone().requires_grad_(True)
    w = weight.clone().requires_grad_(True)
    loss = fw_lm_head_loss(h, w, target, reduction="mean", nchunks=nchunks, impl="staged")
    loss.backward()
    assert h.grad.dtype == dtype and w.grad.dtype == dtype
    np.testing.assert_allclose(loss.float().item(), ref_loss.item(), rtol=1e-5 if dtype == torch.float32 else 1e-2)
    np.testing.assert_allclose(h.grad.float().cpu().numpy(), ref_dh.cpu().numpy(), rtol=tol, atol=1e-6)
    np.testing.assert_allclose(w.grad.float().cpu().numpy(), ref_dw.cpu().numpy(), rtol=tol, atol=1e-6)
    # kappa/H from the oracle on the same logits
    ref = O.solve(z.cpu().numpy(), target.cpu().numpy())
    np.testing.assert_allclose(loss.float().item(), ref["loss"].mean(), rtol=1e-5 if dtype == torch.float32 else 1e-2)


def test_lm_head_rows_needing_the_exact_path():
    B, D, C = 48, 64, 4096
    hidden, weight, target = make(B, D, C, torch.float32, seed=3)
    hidden[:5] = 0.0          # logits all 0: support = every class
    hidden[7] *= 1e-4         # near-constant logits
    ref_loss, ref_dh, ref_dw, _ = dense_reference(hidden, weight, target, "sum")
    h = hidden.clone().requires_grad_(True)
    w = weight.clone().requires_grad_(True)
    loss = fw_lm_head_loss(h, w, target, reduction="sum", nchunks=4, K=8, impl="staged")
    (3.0 * loss).backward()
    np.testing.assert_allclose(loss.item(), ref_loss.item(), rtol=1e-5)
    np.testing.assert_allclose(h.grad.cpu().numpy(), 3.0 * ref_dh.cpu().numpy(), rtol=2e-5, atol=1e-6)
    np.testing.assert_allclose(w.grad.cpu().numpy(), 3.0 * ref_dw.cpu().numpy(), rtol=2e-5, atol=1e-6)
