"""CPU oracle for the FW-loss hot path -- TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may use
this module, and only as the checker or the timed CPU baseline; the product
path (fast-familywise-loss_b200/) never imports it.

Parity is pinned (tests/test_oracle_pins.py): the functions below reproduce
the reference's own known answers (the `kbar` fields of
benchmarks/cpu_benchmarks/results/*.json, regenerated from their seeds) and
the outputs of the reference code run in the build container
(tests/golden/, written by tests/golden/gen_golden.py from
reference_impl.py and src/cpu/fw_cpu.cpp).

Every function works on numpy arrays, one row per line, and returns per-row
results.  All arithmetic is float64.
"""
import numpy as np


def fw_sort_fp64(z, y):
    """Restates reference_impl.FWLoss.forward (reference_impl.py:11-26) in
    float64, which is the oracle the reference's CUDA benchmark compares
    against (benchmarks/cuda_benchmarks/CE_FW_perf.py:137-168):

        z_sorted = sort(z, descending);  S = cumsum(z_sorted)
        H_k = (S_k - 1) / k;  H = max_k H_k;  kappa = first argmax + 1
        loss = 1 - z[y] + H

    Returns (H [B] f64, kappa [B] i64, loss [B] f64).
    """
    z = np.asarray(z, dtype=np.float64)
    B, K = z.shape
    zs = -np.sort(-z, axis=1)
    S = np.cumsum(zs, axis=1)
    Hk = (S - 1.0) / np.arange(1, K + 1, dtype=np.float64)[None, :]
    idx = np.argmax(Hk, axis=1)          # first maximal index, as torch.max(dim)
    H = Hk[np.arange(B), idx]
    zy = z[np.arange(B), np.asarray(y)]
    return H, idx.astype(np.int64) + 1, 1.0 - zy + H


def fw_shifted_fp64(z, y):
    """Same search on the shifted logits d = z - max(z), as the reference CPU
    kernel does for robustness (src/cpu/fw_cpu.cpp:1-10, its "shifted"
    fallback).  Identical to fw_sort_fp64 whenever the unshifted prefix sums
    are exact; it stays exact for magnitudes where S_k - 1 == S_k in float64
    (e.g. logits ~1e30).  Rows with a non-finite maximum follow
    nonfinite_policy().

    Returns (tau [B] f64 = h* - M, kappa [B] i64, M [B] f64, loss [B] f64).
    """
    z = np.asarray(z, dtype=np.float64)
    B, K = z.shape
    y = np.asarray(y)
    M = np.max(z, axis=1)
    tau = np.zeros(B)
    kappa = np.ones(B, dtype=np.int64)
    loss = np.empty(B)
    finite = np.isfinite(M) & ~np.isnan(z).any(axis=1)
    if finite.any():
        zf = z[finite]
        d = zf - M[finite][:, None]
        ds = -np.sort(-d, axis=1)
        S = np.cumsum(ds, axis=1)
        hk = (S - 1.0) / np.arange(1, K + 1, dtype=np.float64)[None, :]
        idx = np.argmax(hk, axis=1)
        tau[finite] = hk[np.arange(len(idx)), idx]
        kappa[finite] = idx + 1
        rows = np.nonzero(finite)[0]
        loss[finite] = 1.0 + (M[finite] - z[rows, y[finite]]) + tau[finite]
    for r in np.nonzero(~finite)[0]:
        j, Mr = nonfinite_policy(z[r])
        M[r] = Mr
        tau[r] = 0.0
        kappa[r] = 1
        loss[r] = np.float32(1.0) - np.float32(z[r, y[r]]) + np.float32(Mr)
    return tau, kappa, M, loss


def nonfinite_policy(row):
    """Policy (not a reference restatement) for a row whose maximum is NaN or
    +-inf, where the reference's arithmetic is undefined: kappa = 1 at the
    first column holding the maximum (the first NaN if any), H = that maximum.
    Returns (column, maximum)."""
    row = np.asarray(row, dtype=np.float64)
    nan = np.isnan(row)
    if nan.any():
        return int(np.argmax(nan)), float("nan")
    m = row.max()
    return int(np.argmax(row == m)), float(m)


def round_down_f32(x):
    """Largest float32 <= x (x float64), elementwise; NaN and +-inf pass."""
    x = np.asarray(x, dtype=np.float64)
    f = x.astype(np.float32)
    over = f.astype(np.float64) > x
    f = np.where(over, np.nextafter(f, np.float32(-np.inf)), f)
    return f.astype(np.float32)


def threshold_f32(tau, M):
    """H as the kernels emit it: round_down_f32(M + tau), with the sum taken
    exactly (M + tau is formed in float64 and corrected by its rounding
    error, so the result is the float32 just below the real threshold)."""
    tau = np.asarray(tau, dtype=np.float64)
    M = np.asarray(M, dtype=np.float64)
    s = M + tau
    # two-sum error term: s + err == M + tau exactly
    bb = s - M
    err = (M - (s - bb)) + (tau - bb)
    f = round_down_f32(s)
    # s rounded up past the real value and landed on a float32: step down
    fix = (f.astype(np.float64) == s) & (err < 0)
    f = np.where(fix, np.nextafter(f, np.float32(-np.inf)), f)
    nf = ~np.isfinite(M)
    return np.where(nf, M.astype(np.float32), f).astype(np.float32)


def support_mask(z, tau, M, kappa):
    """Boolean support: z - M > tau (shifted domain); non-finite rows select
    the nonfinite_policy() column."""
    z = np.asarray(z, dtype=np.float64)
    mask = (z - M[:, None]) > tau[:, None]
    for r in np.nonzero(~np.isfinite(M) | np.isnan(z).any(axis=1))[0]:
        mask[r] = False
        mask[r, nonfinite_policy(z[r])[0]] = True
    return mask


def dense_grad(mask, kappa, y, scale):
    """grad = scale * (mask / kappa - e_y), float64 (reference:
    src/cuda/fw_radix_argmax.cu:1358-1379, src/cpu/fw_cpu.cpp:601-615)."""
    B = mask.shape[0]
    g = mask.astype(np.float64) * (scale / np.asarray(kappa, dtype=np.float64))[:, None]
    g[np.arange(B), np.asarray(y)] -= scale
    return g


def solve(z, y, scale=None):
    """Everything the kernels produce for logits z [B, C] (float32 values) and
    labels y: dict with tau, M, kappa, H (float32), loss (float64), mask and
    the dense gradient (float64) for `scale` (default 1/B)."""
    z = np.asarray(z, dtype=np.float32)
    B = z.shape[0]
    if scale is None:
        scale = 1.0 / B if B else 1.0
    tau, kappa, M, loss = fw_shifted_fp64(z, y)
    mask = support_mask(z, tau, M, kappa)
    return {
        "tau": tau, "M": M, "kappa": kappa, "loss": loss,
        "H": threshold_f32(tau, M), "mask": mask,
        "grad": dense_grad(mask, kappa, y, scale),
    }


def round_down_minus1_f64(M):
    """t0 of the float64 kernels: the largest float64 <= M - 1, elementwise
    (NaN and +-inf pass).  M - 1 is formed in float64 and corrected by its
    exact rounding error (two-sum)."""
    M = np.asarray(M, dtype=np.float64)
    with np.errstate(invalid="ignore"):
        s = M - 1.0
        bb = s - M
        err = (M - (s - bb)) + (-1.0 - bb)   # s + err == M - 1 exactly
        return np.where(np.isfinite(s) & (err < 0), np.nextafter(s, -np.inf), s)


def solve_f64(z, y, scale=None):
    """Everything fw_fused_fwd_bwd_f64 produces for float64 logits z [B, C]:
    dict with tau, M, kappa, H = M + tau, loss, mask and the dense gradient
    (all float64).

    Restates reference_impl.FWLoss.forward (reference_impl.py:11-26) on
    float64 rows, on the candidates above t0 = M - 1 rounded down and in the
    shifted domain d = fl(z - M) (as the reference CPU kernel's float64 path
    falls back to, src/cpu/fw_cpu.cpp:462-468): sort d descending,
    h_k = (S_k - 1)/k, tau = h at the first argmax, support
    {z > t0 and d > tau}, loss = (1 + (M - z_y)) + tau.  Rows with a
    non-finite maximum follow nonfinite_policy(); rows whose label is outside
    [0, C) get a NaN loss and no label term in the gradient.
    """
    z = np.asarray(z, dtype=np.float64)
    y = np.asarray(y, dtype=np.int64)
    B, C = z.shape
    if scale is None:
        scale = 1.0 / B if B else 1.0
    ok_y = (y >= 0) & (y < C)
    yc = np.where(ok_y, y, 0)
    M = np.max(z, axis=1) if C else np.zeros(B)
    tau = np.zeros(B)
    kappa = np.ones(B, dtype=np.int64)
    loss = np.empty(B)
    mask = np.zeros((B, C), dtype=bool)
    finite = np.isfinite(M) & ~np.isnan(z).any(axis=1)
    t0 = round_down_minus1_f64(M)
    for r in np.nonzero(finite)[0]:
        d = z[r] - M[r]
        cand = z[r] > t0[r]
        ds = -np.sort(-d[cand])
        S = np.cumsum(ds)
        hk = (S - 1.0) / np.arange(1, ds.size + 1, dtype=np.float64)
        k = int(np.argmax(hk))            # first maximal index
        tau[r] = hk[k]
        kappa[r] = k + 1
        mask[r] = cand & (d > tau[r])
        loss[r] = (1.0 + (M[r] - z[r, yc[r]])) + tau[r]
    for r in np.nonzero(~finite)[0]:
        j, Mr = nonfinite_policy(z[r])
        M[r] = Mr
        mask[r, j] = True
        loss[r] = 1.0 - z[r, yc[r]] + Mr
    loss = np.where(ok_y, loss, np.nan)
    inv = scale / kappa.astype(np.float64)
    grad = mask.astype(np.float64) * inv[:, None]
    rows = np.nonzero(ok_y)[0]
    grad[rows, y[rows]] -= scale
    H = np.where(finite, M + tau, M)
    return {"tau": tau, "M": M, "kappa": kappa, "loss": loss, "H": H, "mask": mask, "grad": grad}
