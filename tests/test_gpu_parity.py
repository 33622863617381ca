"""GPU parity of the CUDA kernels, called through the C ABI (ctypes), against
the CPU oracle and the reference's own outputs (tests/golden).

Contract (north star): kappa and the selected set bit-exact; H, per-row loss
and gradient within rtol 1e-5 / atol 1e-6 (fp32).
"""
import numpy as np
import pytest
import torch

import cases
from fwloss_b200 import capi, workloads
from oracle import fw_oracle as O

pytestmark = pytest.mark.gpu

RTOL, ATOL = 1e-5, 1e-6
GOLDEN = np.load(__import__("os").path.join(__import__("os").path.dirname(__file__), "golden",
                                            "reference_outputs.npz"))
CONFIG_ROWS = {"cfg0": 256, "cfg1": 512, "cfg2": 64, "cfg3": 2048, "cfg4": 8}


def _to_dev(z, y, ld=None, offset=0):
    """Device copies; ld > C gives padded rows, offset shifts the base pointer
    off its 16-byte alignment (both force the 32-bit access path)."""
    B, C = z.shape
    ld = C if ld is None else ld
    buf = torch.full((B * ld + offset + 4,), float("nan"), dtype=torch.float32, device="cuda")
    view = buf[offset:offset + B * ld].view(B, ld)[:, :C]
    view.copy_(torch.from_numpy(z))
    return view, torch.from_numpy(y).cuda()


def _fused(z, y, scale, **kw):
    zt, yt = _to_dev(z, y, **kw)
    st = torch.zeros(1, dtype=torch.int32, device="cuda")
    grad, H, loss, kappa = capi.fused_fwd_bwd(zt, yt, scale, status=st)
    torch.cuda.synchronize()
    return dict(grad=grad.cpu().numpy(), H=H.cpu().numpy(), loss=loss.cpu().numpy(),
                kappa=kappa.cpu().numpy().astype(np.int64), status=int(st.item()), z=zt)


def _check_row_outputs(out, z, y, ref, name=""):
    np.testing.assert_array_equal(out["kappa"], ref["kappa"], err_msg=f"{name}: kappa")
    np.testing.assert_allclose(out["H"], ref["H"], rtol=RTOL, atol=ATOL, err_msg=f"{name}: H")
    np.testing.assert_allclose(out["loss"], ref["loss"], rtol=RTOL, atol=ATOL, err_msg=f"{name}: loss")
    # H is rounded toward -inf: the mask z > H is exactly the support
    sel = (z > out["H"][:, None])
    fin = np.isfinite(ref["M"])
    np.testing.assert_array_equal(sel[fin].sum(1), out["kappa"][fin], err_msg=f"{name}: |z > H|")
    np.testing.assert_array_equal(sel[fin], ref["mask"][fin], err_msg=f"{name}: support")


def _check_golden(name, out, z, y):
    if f"{name}/kappa_cpu" not in GOLDEN.files:
        return False
    # a host whose torch CPU generator draws other inputs fails here rather
    # than silently comparing with the oracle only (the committed-input test
    # below pins these cases on any host)
    assert cases.golden_inputs_match(GOLDEN, name, z, y), \
        f"{name}: this host regenerates other inputs than the golden fixtures were made from"
    np.testing.assert_array_equal(out["kappa"], GOLDEN[f"{name}/kappa_cpu"], err_msg=f"{name}: kappa vs ref CPU")
    np.testing.assert_allclose(out["loss"], GOLDEN[f"{name}/loss_cpu"], rtol=RTOL, atol=ATOL,
                               err_msg=f"{name}: loss vs ref CPU")
    B, C = out["grad"].shape
    g = np.zeros((B, C), np.float32)
    g[GOLDEN[f"{name}/grad_cpu_r"], GOLDEN[f"{name}/grad_cpu_c"]] = GOLDEN[f"{name}/grad_cpu_v"]
    np.testing.assert_allclose(out["grad"], g, rtol=RTOL, atol=ATOL, err_msg=f"{name}: grad vs ref CPU")
    return True


PARITY = cases.parity_cases()


@pytest.mark.parametrize("name,gen", PARITY, ids=[n for n, _ in PARITY])
def test_fused_matches_oracle_and_reference(name, gen):
    z, y = gen()
    scale = 1.0 / len(y)
    ref = O.solve(z, y, scale)
    out = _fused(z, y, scale)
    _check_row_outputs(out, z, y, ref, name)
    np.testing.assert_allclose(out["grad"], ref["grad"], rtol=RTOL, atol=ATOL, err_msg=f"{name}: grad")
    _check_golden(name, out, z, y)
    assert out["status"] == 0


@pytest.mark.parametrize("name", list(CONFIG_ROWS))
def test_configs_reduced_match_reference(name):
    z, y = workloads.make(name, rows=CONFIG_ROWS[name])
    z, y = z.numpy(), y.numpy()
    ref = O.solve(z, y)
    out = _fused(z, y, 1.0 / len(y))
    _check_row_outputs(out, z, y, ref, name)
    np.testing.assert_allclose(out["grad"], ref["grad"], rtol=RTOL, atol=ATOL)
    if _check_golden(name, out, z, y):
        # the float32 reference_impl agrees bit-exactly on kappa for all five configs
        np.testing.assert_array_equal(out["kappa"], GOLDEN[f"{name}/kappa_ref32"])
        np.testing.assert_allclose(out["H"], GOLDEN[f"{name}/H_ref32"], rtol=RTOL, atol=ATOL)
        np.testing.assert_allclose(out["loss"], GOLDEN[f"{name}/loss_ref32"], rtol=RTOL, atol=ATOL)


@pytest.mark.parametrize("name", list(CONFIG_ROWS))
def test_configs_committed_inputs_match_reference(name):
    """The reduced configurations from their committed inputs (no
    regeneration on this host) against the reference's own outputs: kappa
    bit-exact against the reference CPU kernel and reference_impl, loss and
    gradient within tolerance."""
    z, y, case_rows = cases.committed_config_inputs(name)
    ref = cases.golden_first_rows(GOLDEN, name, len(y), z.shape[1])
    out = _fused(z, y, 1.0 / case_rows)
    np.testing.assert_array_equal(out["kappa"], ref["kappa_cpu"])
    np.testing.assert_array_equal(out["kappa"], ref["kappa_ref32"])
    np.testing.assert_allclose(out["H"], ref["H_ref32"], rtol=RTOL, atol=ATOL)
    np.testing.assert_allclose(out["loss"], ref["loss_cpu"], rtol=RTOL, atol=ATOL)
    np.testing.assert_allclose(out["grad"], ref["grad_cpu"], rtol=RTOL, atol=ATOL)
    assert out["status"] == 0


@pytest.mark.parametrize("C", [3, 64, 100, 1000, 1001, 2048, 3001, 40000])
@pytest.mark.parametrize("layout", ["padded", "offset"])
def test_unaligned_rows(C, layout):
    z, y = cases.gauss(7, C, 1.0, seed=100 + C)()
    ref = O.solve(z, y, 0.5)
    kw = {"ld": C + 3} if layout == "padded" else {"offset": 1}
    out = _fused(z, y, 0.5, **kw)
    _check_row_outputs(out, z, y, ref, f"C{C}-{layout}")
    np.testing.assert_allclose(out["grad"], ref["grad"], rtol=RTOL, atol=ATOL)


@pytest.mark.parametrize("name,gen", cases.nonfinite_cases(), ids=[n for n, _ in cases.nonfinite_cases()])
def test_nonfinite_policy(name, gen):
    z, y = gen()
    ref = O.solve(z, y, 1.0)
    out = _fused(z, y, 1.0)
    np.testing.assert_array_equal(out["kappa"], ref["kappa"])
    np.testing.assert_array_equal(out["H"], ref["H"])  # NaN == NaN here
    np.testing.assert_allclose(out["loss"], ref["loss"].astype(np.float32), rtol=RTOL, atol=ATOL, equal_nan=True)
    np.testing.assert_allclose(out["grad"], ref["grad"], rtol=RTOL, atol=ATOL)
    assert out["status"] & capi.FWB_STATUS_NONFINITE


def test_label_out_of_range_flags_and_nan():
    z, y = cases.gauss(4, 300, 1.0, seed=5)()
    y = y.copy()
    y[1] = -1
    y[2] = 300
    out = _fused(z, y, 1.0)
    assert out["status"] & capi.FWB_STATUS_LABEL_RANGE
    assert np.isnan(out["loss"][1]) and np.isnan(out["loss"][2])
    assert np.isfinite(out["loss"][[0, 3]]).all()
    # rows with a bad label still get their support, with no label term
    ref = O.solve(z, np.where((y < 0) | (y >= 300), 0, y), 1.0)
    np.testing.assert_array_equal(out["kappa"], ref["kappa"])
    g = out["grad"]
    np.testing.assert_allclose(g[1].sum(), 1.0, rtol=1e-5)


@pytest.mark.parametrize("name,gen", [c for c in PARITY if c[0] in (
    "gauss_C1", "gauss_C37", "gauss_C1000", "gauss_mid_C10000", "ties_C128", "dense_s1e-3_C1000",
    "dense_s1e-3_C40000", "const_C40000", "exact_ties", "mag1e30_C5000", "gauss_mid_C31623",
    "neginf_C12000", "zeros_C9000")])
def test_mask_and_candidate_forms(name, gen):
    z, y = gen()
    B, C = z.shape
    ref = O.solve(z, y, 1.0 / B)
    zt, yt = _to_dev(z, y)
    H, loss, kappa, mask = capi.forward_mask(zt, yt)
    g_mask = capi.backward_mask(yt, mask, kappa, 1.0 / B)
    H2, loss2, kappa2, cv, ci, cc = capi.forward_candidates(zt, yt)
    g_cand = capi.backward_candidates(cv, ci, cc, H2, kappa2, yt, 1.0 / B)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(mask.cpu().numpy(), ref["mask"])
    np.testing.assert_array_equal(kappa.cpu().numpy(), ref["kappa"])
    np.testing.assert_array_equal(kappa2.cpu().numpy(), ref["kappa"])
    np.testing.assert_array_equal(cc.cpu().numpy(), ref["kappa"])
    np.testing.assert_array_equal(H.cpu().numpy(), H2.cpu().numpy())
    np.testing.assert_allclose(loss.cpu().numpy(), ref["loss"], rtol=RTOL, atol=ATOL)
    # candidate rows hold exactly the support
    cvn, cin, ccn = cv.cpu().numpy(), ci.cpu().numpy(), cc.cpu().numpy()
    for r in range(B):
        cols = np.sort(cin[r, : ccn[r]])
        np.testing.assert_array_equal(cols, np.nonzero(ref["mask"][r])[0])
        np.testing.assert_array_equal(cvn[r, : ccn[r]], z[r, cin[r, : ccn[r]]])
    np.testing.assert_allclose(g_mask.cpu().numpy(), ref["grad"], rtol=RTOL, atol=ATOL)
    np.testing.assert_allclose(g_cand.cpu().numpy(), ref["grad"], rtol=RTOL, atol=ATOL)


def test_scale_grad_and_loss_reduce():
    z, y = cases.gauss(64, 5000, 1.0, seed=9)()
    ref = O.solve(z, y, 1.0)
    zt, yt = _to_dev(z, y)
    grad, H, loss, kappa = capi.fused_fwd_bwd(zt, yt, 1.0)
    go = torch.linspace(-2.0, 2.0, 64, device="cuda")
    go[5] = 1.0
    capi.scale_grad(grad, go, True, 1.0)
    np.testing.assert_allclose(grad.cpu().numpy(), ref["grad"] * go.cpu().numpy()[:, None],
                               rtol=RTOL, atol=ATOL)
    s = capi.loss_reduce(loss, 1.0 / 64)
    np.testing.assert_allclose(s.item(), ref["loss"].mean(), rtol=1e-6)
    g2, *_ = capi.fused_fwd_bwd(zt, yt, 1.0 / 64)
    capi.scale_grad(g2, torch.tensor([3.0], device="cuda"), False, 1.0)
    np.testing.assert_allclose(g2.cpu().numpy(), ref["grad"] * 3.0 / 64, rtol=RTOL, atol=ATOL)


def test_empty_batch_is_noop():
    z = torch.empty((0, 100), dtype=torch.float32, device="cuda")
    y = torch.empty((0,), dtype=torch.int64, device="cuda")
    grad, H, loss, kappa = capi.fused_fwd_bwd(z, y, 1.0)
    torch.cuda.synchronize()
    assert grad.shape == (0, 100)


def test_deterministic_repeat():
    z, y = workloads.make("cfg2", rows=256)
    zt, yt = z.cuda(), y.cuda()
    a = capi.fused_fwd_bwd(zt, yt, 1.0 / 256)
    b = capi.fused_fwd_bwd(zt, yt, 1.0 / 256)
    for u, v in zip(a, b):
        assert torch.equal(u, v)


def _full_size_properties(z, y, out_grad, H, loss, kappa, scale, sample_rows=48):
    """Size-independent checks at full configuration size (on the device),
    plus an oracle comparison on a random sample of rows."""
    B, C = z.shape
    sel = z > H[:, None]
    assert torch.equal(sel.sum(1).to(torch.int32), kappa)
    nz = (out_grad != 0).sum(1)
    ysel = sel[torch.arange(B, device=z.device), y]
    assert torch.equal(nz, kappa.long() + (~ysel).long() - (ysel & (kappa == 1)).long())
    rs = out_grad.double().sum(1)
    assert rs.abs().max().item() <= 1e-6 * max(1.0, scale * 10)
    # threshold optimality: sum_j max(z_j - h, 0) == 1 at h = H (up to the round-down of H)
    f = torch.clamp(z.double() - H.double()[:, None], min=0).sum(1)
    ulp = torch.abs(H.double()) * 2.0 ** -23 + 1e-30
    assert ((f - 1.0).abs() <= kappa.double() * ulp * 2 + 1e-9).all()
    zy = z[torch.arange(B, device=z.device), y].double()
    np.testing.assert_allclose(loss.double().cpu().numpy(), (1.0 - zy + H.double()).cpu().numpy(),
                               rtol=RTOL, atol=ATOL)
    g = torch.Generator().manual_seed(0)
    rows = torch.randperm(B, generator=g)[:sample_rows].sort().values
    zs = z[rows.cuda()].cpu().numpy()
    ys = y[rows.cuda()].cpu().numpy()
    ref = O.solve(zs, ys, scale)
    np.testing.assert_array_equal(kappa[rows.cuda()].cpu().numpy(), ref["kappa"])
    np.testing.assert_allclose(out_grad[rows.cuda()].cpu().numpy(), ref["grad"], rtol=RTOL, atol=ATOL)


@pytest.mark.parametrize("name", ["cfg1", "cfg2", "cfg3", "cfg4"])
def test_full_size_configs_match_reference_cpu_kernel(name):
    """Every row of the full-size configuration against the reference's own
    CPU kernel (src/cpu/fw_cpu.cpp, fw_loss_grad, compiled into oracle/_ref),
    as the reference's benchmark checks the whole batch
    (benchmarks/cuda_benchmarks/CE_FW_perf.py:137-177): kappa equal for all
    rows, per-row loss and the gradient within rtol 1e-5 / atol 1e-6; the
    forward-only kernel's kappa too."""
    from oracle import ref_cpu

    assert ref_cpu.ref_available(), "the reference CPU kernel (oracle/_ref) is not built"
    z, y = workloads.make(name)
    B = z.shape[0]
    torch.set_num_threads(max(1, __import__("os").cpu_count() or 1))
    L, G, K = ref_cpu.ref_loss_grad(z.numpy(), y.numpy(), 1.0 / B)
    zd, yd = z.cuda(), y.cuda()
    del z
    grad, H, loss, kappa = capi.fused_fwd_bwd(zd, yd, 1.0 / B)
    _, _, kappa_f = capi.forward_rows(zd, yd)
    torch.cuda.synchronize()
    K = torch.from_numpy(K)
    assert torch.equal(kappa.cpu().long(), K), f"{name}: kappa differs from the reference CPU kernel"
    assert torch.equal(kappa_f.cpu().long(), K)
    np.testing.assert_allclose(loss.cpu().numpy(), L, rtol=RTOL, atol=ATOL)
    Gd = torch.from_numpy(G).cuda()
    del G
    bad = (grad - Gd).abs() > (ATOL + RTOL * Gd.abs())
    assert not bool(bad.any()), f"{name}: {int(bad.sum())} gradient entries outside rtol/atol"
    del grad, Gd, bad, zd
    torch.cuda.empty_cache()


@pytest.mark.parametrize("name", ["cfg1", "cfg2", "cfg3", "cfg4"])
def test_full_size_configs(name):
    z, y = workloads.make(name)
    z, y = z.cuda(), y.cuda()
    B = z.shape[0]
    grad, H, loss, kappa = capi.fused_fwd_bwd(z, y, 1.0 / B)
    torch.cuda.synchronize()
    _full_size_properties(z, y, grad, H, loss, kappa, 1.0 / B)
    del grad
    torch.cuda.empty_cache()


HALF_TYPES = {"bf16": (torch.bfloat16, 2.0 ** -8), "f16": (torch.float16, 2.0 ** -11)}


@pytest.mark.parametrize("dtype", list(HALF_TYPES))
@pytest.mark.parametrize("name", ["gauss_C37", "gauss_C128", "gauss_C1000", "gauss_C2048", "gauss_mid_C3000",
                                  "gauss_mid_C31623", "gauss_mid_C32000", "ties_C128", "ties_C5000",
                                  "dense_s1e-1_C3000", "dense_s1e-3_C1000", "dense_s1e-3_C40000",
                                  "exact_ties", "neginf_C12000"])
def test_half_precision_logits(dtype, name):
    """16-bit logits: the oracle runs on the rounded values, so kappa, the
    support, H and the loss must match as for fp32; the gradient carries the
    element type's rounding (relative tolerance = its unit roundoff)."""
    tdt, rtol = HALF_TYPES[dtype]
    z32, y = dict(PARITY)[name]()
    zh = torch.from_numpy(z32).to(tdt)
    z = zh.float().numpy()  # the values the kernel sees
    B = len(y)
    ref = O.solve(z, y, 1.0 / B)
    zt = zh.cuda()
    yt = torch.from_numpy(y).cuda()
    grad, H, loss, kappa = capi.fused_fwd_bwd(zt, yt, 1.0 / B)
    torch.cuda.synchronize()
    assert grad.dtype == tdt
    np.testing.assert_array_equal(kappa.cpu().numpy(), ref["kappa"], err_msg=name)
    np.testing.assert_allclose(H.cpu().numpy(), ref["H"], rtol=RTOL, atol=ATOL)
    np.testing.assert_allclose(loss.cpu().numpy(), ref["loss"], rtol=RTOL, atol=ATOL)
    np.testing.assert_array_equal((z > H.cpu().numpy()[:, None]), ref["mask"])
    np.testing.assert_allclose(grad.float().cpu().numpy(), ref["grad"], rtol=rtol, atol=ATOL)
    # device-side upstream scaling on the 16-bit gradient
    capi.scale_grad(grad, torch.tensor([2.0], device="cuda"), False, 1.0)
    np.testing.assert_allclose(grad.float().cpu().numpy(), 2.0 * ref["grad"], rtol=2 * rtol, atol=ATOL)


def _half_shape_switches():
    """16-bit batches on both sides of the streaming tier's 16-bit launch-plan
    switches (148 SMs on a B200): the narrow shape (short rows, >= 64 Mi
    elements), the staged4 shape (>= 49152 columns over more than one wide
    wave), one wide launch, and a wide launch followed by a second launch of
    the rows left over after its whole wave."""
    sms = torch.cuda.get_device_properties(0).multi_processor_count if torch.cuda.is_available() else 148
    deep, wide = 2 * sms, 5 * sms
    n64 = 64 << 20
    return [(n64 // 32000 + 1, 32000), (n64 // 32000 - 1, 32000), (wide + 1, 49152), (wide + 1, 49151),
            (wide + 20, 30000), (n64 // 8192 + 3, 8192)]


HALF_SWITCHES = _half_shape_switches()


@pytest.mark.parametrize("dtype", list(HALF_TYPES))
@pytest.mark.parametrize("B,C", HALF_SWITCHES, ids=[f"B{b}_C{c}" for b, c in HALF_SWITCHES])
def test_half_precision_launch_shapes(dtype, B, C):
    """16-bit logits through every launch shape the plan picks for them:
    kappa bit-exact and H, loss within tolerance against the C oracle on the
    rounded values, the gradient within the element type's unit roundoff;
    odd rows are near-ties (sigma 1e-2 in 16-bit: many candidates)."""
    from oracle import ref_cpu

    tdt, rtol = HALF_TYPES[dtype]
    rng = np.random.default_rng(B + 7 * C)
    z32 = rng.standard_normal((B, C)).astype(np.float32)
    z32[1::2] *= np.float32(1e-2)
    zh = torch.from_numpy(z32).to(tdt)
    z = zh.float().numpy()
    del z32
    y = rng.integers(0, C, B).astype(np.int64)
    tau, kap, M, loss = ref_cpu.c_solve(z, y)
    grad, H, lo, kappa = capi.fused_fwd_bwd(zh.cuda(), torch.from_numpy(y).cuda(), 1.0 / B)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(kappa.cpu().numpy(), kap)
    Hr = O.threshold_f32(tau, M)
    np.testing.assert_allclose(H.cpu().numpy(), Hr, rtol=RTOL, atol=ATOL)
    np.testing.assert_allclose(lo.cpu().numpy(), loss, rtol=RTOL, atol=ATOL)
    g = grad.float().cpu().numpy()
    del grad
    expect = (z > Hr[:, None]).astype(np.float32) / kap[:, None].astype(np.float32) / np.float32(B)
    expect[np.arange(B), y] -= np.float32(1.0 / B)
    np.testing.assert_allclose(g, expect, rtol=rtol, atol=ATOL)
    torch.cuda.empty_cache()


@pytest.mark.parametrize("dtype", list(HALF_TYPES))
@pytest.mark.parametrize("C", [100, 5000])
def test_half_precision_subnormal_candidates(dtype, C):
    """Rows whose candidates are subnormal numbers of the 16-bit type, in both
    tiers (C = 100: register tier, C = 5000: streaming tier).  float16: a
    maximum of 1.0 makes the candidate threshold 0, and the positive
    subnormals (>= 2^-24, resolvable in the fp64 shifted sums) are
    candidates.  bfloat16 subnormals (~1e-39) are below the fp64 resolution
    of z - M next to M = 1, so there the maximum is itself a small normal
    number and the subnormals sit within 1 of it."""
    tdt, rtol = HALF_TYPES[dtype]
    tiny = float(torch.finfo(tdt).smallest_normal) / 4  # a subnormal of the type
    top = 1.0 if tdt == torch.float16 else float(torch.finfo(tdt).smallest_normal) * 8
    rng = np.random.default_rng(C)
    B = 6
    z = np.full((B, C), -2.0, np.float32)
    for r in range(B):
        cols = rng.choice(C, size=3 + 5 * r, replace=False)
        z[r, cols] = tiny * rng.integers(1, 4, size=cols.size)
        z[r, cols[0]] = top
    z = torch.from_numpy(z).to(tdt).float().numpy()  # exact in the type
    y = rng.integers(0, C, B).astype(np.int64)
    ref = O.solve(z, y, 1.0 / B)
    assert (ref["kappa"] > 1).sum() >= B - 1  # the subnormals decide the support
    zt = torch.from_numpy(z).to(tdt).cuda()
    grad, H, loss, kappa = capi.fused_fwd_bwd(zt, torch.from_numpy(y).cuda(), 1.0 / B)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(kappa.cpu().numpy(), ref["kappa"])
    np.testing.assert_array_equal((z > H.cpu().numpy()[:, None]), ref["mask"])
    np.testing.assert_allclose(loss.cpu().numpy(), ref["loss"], rtol=RTOL, atol=ATOL)
    np.testing.assert_allclose(grad.float().cpu().numpy(), ref["grad"], rtol=rtol, atol=ATOL)


@pytest.mark.parametrize("dtype", list(HALF_TYPES))
def test_half_precision_autograd(dtype):
    from fwloss_b200 import familywise_loss

    tdt, rtol = HALF_TYPES[dtype]
    z32, y = cases.gauss(64, 5000, 1.0, seed=77)()
    zh = torch.from_numpy(z32).to(tdt)
    ref = O.solve(zh.float().numpy(), y, 1.0 / 64)
    z = zh.cuda().requires_grad_(True)
    out = familywise_loss(z, torch.from_numpy(y).cuda(), reduction="mean")
    assert out.dtype == tdt
    out.backward()
    assert z.grad.dtype == tdt
    np.testing.assert_allclose(out.float().item(), ref["loss"].mean(), rtol=rtol)
    np.testing.assert_allclose(z.grad.float().cpu().numpy(), ref["grad"], rtol=rtol, atol=ATOL)


def _shape_switches():
    """Batch sizes around the streaming tier's launch-plan switches for this
    GPU's SM count (148 on a B200): deep shape with clusters of 8/4/2 or one
    CTA per row (B <= 2 CTAs per SM), one wide launch (B <= 5 per SM, or a
    last wave of more than 2 per SM), staged tiles (2 or 4 CTAs per SM) for
    long rows, the narrow staged shape (8 CTAs per SM) for short rows in
    batches of >= 64 Mi elements, and a wide launch followed by a second,
    staged launch of the rows left over after its one whole wave (one CTA or
    a cluster per leftover row)."""
    sms = torch.cuda.get_device_properties(0).multi_processor_count if torch.cuda.is_available() else 148
    deep, wide = 2 * sms, 5 * sms
    return [(1, 300000), (2, 65536), (deep // 8, 40000), (deep // 8 + 1, 40000), (deep // 4 - 1, 20000),
            (deep // 4, 20000), (deep // 2 - 1, 9000), (deep // 2 + 1, 9000), (deep - 1, 8200), (deep + 1, 8200),
            (deep + 10, 45000), (wide + 10, 70000), (600, 2049), (wide + 20, 3000), (wide + 10, 30000),
            (2 * wide + 3, 24600), ((64 << 20) // 12287 + 1, 12287), ((64 << 20) // 12287, 12287),
            (wide + deep - 6, 9000), (wide + deep + 4, 9000), (2 * wide + 7, 4100)]


SHAPE_SWITCHES = _shape_switches()


@pytest.mark.parametrize("B,C", SHAPE_SWITCHES, ids=[f"B{b}_C{c}" for b, c in SHAPE_SWITCHES])
def test_streaming_launch_shape_switches(B, C):
    """kappa bit-exact and H, loss, gradient within tolerance against the C
    oracle on both sides of every launch-shape switch, with Gaussian rows
    (a handful of candidates) and rows of near-ties (sigma 1e-3: the dense
    radix path for half of them)."""
    from oracle import ref_cpu

    rng = np.random.default_rng(B * 1000 + C)
    z = rng.standard_normal((B, C)).astype(np.float32)
    z[1::2] *= np.float32(1e-3)
    y = rng.integers(0, C, B).astype(np.int64)
    tau, kap, M, loss = ref_cpu.c_solve(z, y)
    out = _fused(z, y, 1.0 / B)
    np.testing.assert_array_equal(out["kappa"], kap)
    H = O.threshold_f32(tau, M)
    np.testing.assert_allclose(out["H"], H, rtol=RTOL, atol=ATOL)
    np.testing.assert_allclose(out["loss"], loss, rtol=RTOL, atol=ATOL)
    g = out["grad"]
    sel = z > H[:, None]
    expect = sel.astype(np.float64) / kap[:, None] / B
    expect[np.arange(B), y] -= 1.0 / B
    np.testing.assert_allclose(g, expect, rtol=RTOL, atol=ATOL)


@pytest.mark.parametrize("B,C", SHAPE_SWITCHES[-5:], ids=[f"B{b}_C{c}" for b, c in SHAPE_SWITCHES[-5:]])
def test_split_launch_followed_by_reduction(B, C):
    """Where the rows left over after the wide launch's whole waves run as a
    second, programmatically dependent launch, the loss reduction queued
    right after (no host synchronisation in between) sees every row, and the
    forward-only kernel gives the same kappa."""
    from oracle import ref_cpu

    rng = np.random.default_rng(7 * B + C)
    z = rng.standard_normal((B, C)).astype(np.float32)
    y = rng.integers(0, C, B).astype(np.int64)
    _, kap, _, loss = ref_cpu.c_solve(z, y)
    zt, yt = torch.from_numpy(z).cuda(), torch.from_numpy(y).cuda()
    for _ in range(3):
        _, _, l, k = capi.fused_fwd_bwd(zt, yt, 1.0 / B)
        s = capi.loss_reduce(l, 1.0 / B)
        _, _, kf = capi.forward_rows(zt, yt)
        torch.cuda.synchronize()
        np.testing.assert_allclose(s.item(), loss.mean(), rtol=1e-6)
        np.testing.assert_array_equal(k.cpu().numpy(), kap)
        np.testing.assert_array_equal(kf.cpu().numpy(), kap)


@pytest.mark.parametrize("B,C", [(6, 31623), (4, 300001), (9, 40002), (700, 30001)],
                         ids=["cta_C31623", "cluster_C300001", "cluster_C40002", "wide_C30001"])
def test_label_logit_captured_while_streaming(B, C):
    """The streaming tier records the label's logit while it streams the row
    (and a cluster's leader fetches it from the CTA whose segment holds it):
    labels at column 0, in every CTA's segment, and in the C % 4 tail
    columns give the oracle's per-row loss."""
    rng = np.random.default_rng(B + C)
    z = rng.standard_normal((B, C)).astype(np.float32)
    y = np.linspace(0, C - 1, B).astype(np.int64)
    y[0], y[-1] = 0, C - 1
    if B > 2:
        y[1] = C - 2
    ref = O.solve(z, y, 1.0 / B)
    out = _fused(z, y, 1.0 / B)
    _check_row_outputs(out, z, y, ref, f"B{B}_C{C}")
    np.testing.assert_allclose(out["grad"], ref["grad"], rtol=RTOL, atol=ATOL)
