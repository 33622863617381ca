"""The fused LM-head kernel (fw_lmhead_fused_scan: tcgen05 GEMM whose
epilogue writes the chunk summaries) against logits materialised by an fp32
GEMM on the same bf16 values, and the fused forward + sparse backward
against the dense path.

The accumulation order of the tensor cores differs from the reference GEMM,
so logit values agree to fp32 rounding (rtol/atol 1e-5 here); the supports
(kappa per chunk and per row) agree exactly on these inputs, whose logits
have no near-ties at the threshold."""
import numpy as np
import pytest
import torch

from fwloss_b200 import capi
from fwloss_b200.lm_head import fw_lm_head_loss, tile_col_start
from fwloss_b200._native import ext
from oracle import fw_oracle as O

pytestmark = pytest.mark.gpu

SHAPES = [(100, 64, 1000, 4), (300, 200, 5000, 3), (128, 512, 12345, 5), (257, 1024, 33000, 16)]


def make(B, D, C, seed, temp=4.0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    hidden = (torch.randn(B, D, generator=g, device="cuda") / D ** 0.5 * temp).to(torch.bfloat16)
    weight = torch.randn(C, D, generator=g, device="cuda").to(torch.bfloat16)
    target = torch.randint(0, C, (B,), generator=g, device="cuda")
    return hidden, weight, target


def fused_scan(hidden, weight, target, nchunks, K):
    B, C = hidden.shape[0], weight.shape[0]
    cs = tile_col_start(C, nchunks)
    n = len(cs) - 1
    dev = hidden.device
    summ = torch.full((n, B, 4 + K), -7, dtype=torch.int32, device=dev)
    lidx = torch.full((n, B, K), -7, dtype=torch.int32, device=dev)
    zy = torch.full((B,), float("nan"), device=dev)
    st = torch.zeros(1, dtype=torch.int32, device=dev)
    ext().lmhead_fused_scan(hidden, weight, target, cs, summ, lidx, zy, st)
    torch.cuda.synchronize()
    return cs, summ.cpu().numpy(), lidx.cpu().numpy(), zy.cpu().numpy(), int(st.item())


@pytest.mark.parametrize("B,D,C,nchunks", SHAPES)
def test_fused_summaries_match_materialised_logits(B, D, C, nchunks):
    K = 16
    hidden, weight, target = make(B, D, C, seed=B * 7 + C)
    cs, summ, lidx, zy, st = fused_scan(hidden, weight, target, nchunks, K)
    assert st == 0
    z = (hidden.float() @ weight.float().t()).cpu().numpy()
    y = target.cpu().numpy()
    np.testing.assert_allclose(zy, z[np.arange(B), y], rtol=1e-5, atol=1e-5)
    for q in range(len(cs) - 1):
        zq = z[:, cs[q]:cs[q + 1]]
        rec = summ[q]
        M = rec[:, 0].view(np.float32)
        np.testing.assert_allclose(M, zq.max(1), rtol=1e-5, atol=1e-5, err_msg=f"chunk {q}: max")
        ref = O.solve(zq, np.zeros(B, dtype=np.int64))
        np.testing.assert_array_equal(rec[:, 1], ref["kappa"], err_msg=f"chunk {q}: own support size")
        assert (rec[:, 2] == 0).all() and (rec[:, 3] == -1).all()
        for r in range(B):
            k = min(rec[r, 1], K)
            cols = lidx[q, r, :k]
            vals = rec[r, 4:4 + k].view(np.float32)
            assert sorted(cols) == sorted(np.nonzero(ref["mask"][r])[0][:k]) or rec[r, 1] > K
            np.testing.assert_allclose(vals, zq[r, cols], rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("B,D,C,nchunks", SHAPES)
def test_fused_loss_and_grads_match_dense(B, D, C, nchunks):
    from fwloss_b200 import familywise_loss

    hidden, weight, target = make(B, D, C, seed=B + C)
    h = hidden.detach().clone().requires_grad_(True)
    w = weight.detach().clone().requires_grad_(True)
    zr = h.float() @ w.float().t()
    ref = familywise_loss(zr, target, reduction="mean")
    ref.backward()
    h2 = hidden.clone().requires_grad_(True)
    w2 = weight.clone().requires_grad_(True)
    loss = fw_lm_head_loss(h2, w2, target, reduction="mean", nchunks=nchunks, impl="fused")
    loss.backward()
    np.testing.assert_allclose(loss.float().item(), ref.item(), rtol=1e-2)
    # loss in fp32 before the cast to bf16 output: compare the staged form too
    staged = fw_lm_head_loss(hidden, weight, target, reduction="mean", nchunks=nchunks, impl="staged")
    np.testing.assert_allclose(loss.float().item(), staged.float().item(), rtol=1e-2)
    np.testing.assert_allclose(h2.grad.float().cpu().numpy(), h.grad.float().cpu().numpy(), rtol=2e-2, atol=1e-6)
    np.testing.assert_allclose(w2.grad.float().cpu().numpy(), w.grad.float().cpu().numpy(), rtol=2e-2, atol=1e-6)


def test_fused_rows_needing_the_exact_path():
    """All-zero hidden rows give constant logits: the on-chip candidate list
    overflows, the chunk is recorded with kappa = K + 1 and the row is solved
    from its full logit row."""
    B, D, C = 200, 128, 6000
    hidden, weight, target = make(B, D, C, seed=5)
    hidden[:5] = 0
    hidden[130:133] = 0
    K = 8
    cs, summ, lidx, zy, st = fused_scan(hidden, weight, target, 4, K)
    assert st == 0
    assert (summ[:, :5, 1] == K + 1).all() and (summ[:, 130:133, 1] == K + 1).all()
    h = hidden.detach().clone().requires_grad_(True)
    w = weight.detach().clone().requires_grad_(True)
    from fwloss_b200 import familywise_loss

    ref = familywise_loss(h.float() @ w.float().t(), target, reduction="sum")
    ref.backward()
    h2 = hidden.clone().requires_grad_(True)
    w2 = weight.clone().requires_grad_(True)
    loss = fw_lm_head_loss(h2, w2, target, reduction="sum", nchunks=4, K=K, impl="fused")
    loss.backward()
    np.testing.assert_allclose(loss.float().item(), ref.item(), rtol=1e-2)
    np.testing.assert_allclose(h2.grad.float().cpu().numpy(), h.grad.float().cpu().numpy(), rtol=2e-2, atol=1e-5)
    np.testing.assert_allclose(w2.grad.float().cpu().numpy(), w.grad.float().cpu().numpy(), rtol=2e-2, atol=1e-5)


def test_fused_nonfinite_rows_match_staged():
    """A hidden row holding +inf gives +-inf logits: the chunk records carry
    the first column of the maximum, and the combined row (H, kappa, support
    column) equals the staged form's."""
    B, D, C = 64, 64, 3000
    hidden, weight, target = make(B, D, C, seed=9)
    hidden[3, 10] = float("inf")
    hidden[40, 0] = float("nan")
    fw = ext()
    out = {}
    for impl, cs in (("fused", tile_col_start(C, 4)), ("staged", None)):
        if impl == "fused":
            cs, summ, lidx, zy, st = fused_scan(hidden, weight, target, 4, 16)
            summ_t, lidx_t, zy_t = (torch.from_numpy(summ).cuda(), torch.from_numpy(lidx).cuda(),
                                    torch.from_numpy(zy).cuda())
        else:
            from fwloss_b200.sharded import even_col_start

            cs = even_col_start(C, 4)
            n = len(cs) - 1
            summ_t = torch.empty((n, B, 20), dtype=torch.int32, device="cuda")
            lidx_t = torch.empty((n, B, 16), dtype=torch.int32, device="cuda")
            zy_t = torch.empty(B, device="cuda")
            for q in range(n):
                zq = (hidden @ weight[cs[q]:cs[q + 1]].t()).float()
                fw.shard_scan_into(zq, 16, summ_t[q], lidx_t[q])
                fw.label_logits(zq, target, cs[q], zy_t)
        H, kappa, loss, sup, fb_rows, fb_count = fw.chunks_solve(summ_t, lidx_t, cs, zy_t, target)
        out[impl] = (H.cpu().numpy(), kappa.cpu().numpy(), sup[:, 0].cpu().numpy(), int(fb_count.item()))
    Hf, kf, sf, nf = out["fused"]
    Hs, ks, ss, ns = out["staged"]
    for r in (3, 40):
        assert kf[r] == ks[r] == 1
        assert sf[r] == ss[r]
        assert (np.isnan(Hf[r]) and np.isnan(Hs[r])) or Hf[r] == Hs[r]


def test_fused_argument_checks():
    lib = capi.load()
    import ctypes

    P = None
    dummy = ctypes.c_void_p(256)
    cs = (ctypes.c_int64 * 3)(0, 300, 1000)  # 300 is not a multiple of 256
    assert lib.fw_lmhead_fused_scan(1, dummy, 4, 64, dummy, 1000, 2, cs, 8, dummy, dummy, dummy, dummy, P,
                                    P) == 1
    cs = (ctypes.c_int64 * 3)(0, 256, 1000)
    assert lib.fw_lmhead_fused_scan(0, dummy, 4, 64, dummy, 1000, 2, cs, 8, dummy, dummy, dummy, dummy, P,
                                    P) == 5
    assert lib.fw_lmhead_fused_scan(1, dummy, 4, 60, dummy, 1000, 2, cs, 8, dummy, dummy, dummy, dummy, P,
                                    P) == 1
