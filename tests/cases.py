"""Seeded parity cases shared by the fixture generator and the tests.

Each case is (name, generator) where generator() -> (z float32 [B, C],
y int64 [B]) as numpy arrays, fully determined by its seed.  The coverage
follows what the reference's CPU test suite is described to cover
(src/cpu/README.md "Files": ties, constant, sorted, two-level and outlier
inputs, magnitudes up to 1e30, K from 1 to 40,000) plus the GPU-specific
shapes: every warp-tier slot width, unaligned row strides, the streaming
tier with and without clusters, and dense rows that take the radix path.
"""
import hashlib

import numpy as np


def input_sha256(z, y):
    """Fingerprint of a case's inputs (the golden fixtures store it per case)."""
    return hashlib.sha256(np.ascontiguousarray(z).tobytes() + np.ascontiguousarray(y).tobytes()).hexdigest()


def golden_inputs_match(golden, name, z, y):
    """True when (z, y) are the inputs the golden outputs of case `name` were
    made from.  Cases drawn with numpy match on every host; the benchmark
    configurations are drawn with torch's CPU generator, whose float32 normal
    kernel gives different values on hosts where it runs its scalar code
    instead of the AVX2/AVX-512 one."""
    key = f"{name}/input_sha256"
    return key in golden.files and str(golden[key]) == input_sha256(z, y)


def committed_config_inputs(name):
    """(z [n, C] float32, y [n] int64, rows of the fixture case) of a reduced
    benchmark configuration, read from tests/golden/config_inputs.npz (its
    first n rows, stored by tests/golden/gen_golden.py --config-inputs)."""
    import os

    d = np.load(os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "config_inputs.npz"))
    return d[f"{name}/z"], d[f"{name}/y"], int(d[f"{name}/case_rows"])


def golden_first_rows(golden, name, n, C):
    """The golden outputs of case `name` for its first n rows: the reference
    CPU kernel's kappa, loss and dense gradient, and reference_impl's fp32
    kappa, H and loss."""
    out = {k: golden[f"{name}/{k}"][:n] for k in ("kappa_cpu", "loss_cpu", "kappa_ref32", "H_ref32", "loss_ref32")}
    r, c, v = (golden[f"{name}/grad_cpu_{s}"] for s in "rcv")
    keep = r < n
    g = np.zeros((n, C), np.float32)
    g[r[keep], c[keep]] = v[keep]
    out["grad_cpu"] = g
    return out


def _rng(seed):
    return np.random.default_rng(seed)


def _labels(rng, B, C):
    return rng.integers(0, C, B).astype(np.int64)


def gauss(B, C, sigma=1.0, seed=0):
    def g():
        r = _rng(seed)
        z = (r.standard_normal((B, C)) * sigma).astype(np.float32)
        return z, _labels(r, B, C)
    return g


def levels(B, C, lv, seed=0):
    def g():
        r = _rng(seed)
        z = np.asarray(lv, dtype=np.float32)[r.integers(0, len(lv), (B, C))]
        return z, _labels(r, B, C)
    return g


def constant(B, C, v=0.5, seed=0):
    def g():
        r = _rng(seed)
        return np.full((B, C), v, dtype=np.float32), _labels(r, B, C)
    return g


def sorted_rows(B, C, seed=0):
    def g():
        r = _rng(seed)
        z = np.sort(r.standard_normal((B, C)).astype(np.float32) * 0.3, axis=1)
        z[1::2] = z[1::2, ::-1]
        return np.ascontiguousarray(z), _labels(r, B, C)
    return g


def two_level(B, C, seed=0):
    def g():
        r = _rng(seed)
        a = r.standard_normal(B).astype(np.float32)[:, None]
        gap = r.uniform(0.0, 1.5, B).astype(np.float32)[:, None]
        hi = r.random((B, C)) < 0.3
        z = np.where(hi, a, a - gap).astype(np.float32)
        return z, _labels(r, B, C)
    return g


def outliers(B, C, seed=0):
    def g():
        r = _rng(seed)
        z = r.standard_normal((B, C)).astype(np.float32)
        cols = r.integers(0, C, B)
        z[np.arange(B), cols] = np.where(np.arange(B) % 2 == 0, 1e3, -1e3).astype(np.float32)
        return z, _labels(r, B, C)
    return g


def magnitude(B, C, scale, seed=0):
    def g():
        r = _rng(seed)
        z = (r.standard_normal((B, C)) * scale).astype(np.float32)
        # duplicated maxima at huge magnitude: S_k - 1 == S_k in float64
        z[0, : max(1, C // 3)] = z[0].max()
        return z, _labels(r, B, C)
    return g


def signed_zeros(B, C, seed=0):
    def g():
        r = _rng(seed)
        z = r.choice(np.array([0.0, -0.0, -0.5, -1.0, 0.25], dtype=np.float32), (B, C))
        z[: B // 2, :] = np.where(r.random((B // 2, C)) < 0.5, np.float32(0.0), np.float32(-0.0))
        return z.astype(np.float32), _labels(r, B, C)
    return g


def neg_inf(B, C, seed=0):
    def g():
        r = _rng(seed)
        z = r.standard_normal((B, C)).astype(np.float32)
        z[r.random((B, C)) < 0.4] = -np.inf
        z[:, 0] = r.standard_normal(B).astype(np.float32)  # at least one finite per row
        return z, _labels(r, B, C)
    return g


def exact_ties(seed=0):
    """Rows where z_(k+1) == h_k exactly (first-argmax must stop at k)."""
    def g():
        rows = [
            [3.5, 2.5, 0.0, -1.0],          # h1 = 2.5 == z2 -> kappa 1
            [1.0, 0.0, 0.0, 0.0],           # h1 = 0 == z2
            [2.0, 2.0, 1.5, -3.0],          # h2 = 1.5 == z3 -> kappa 2
            [0.0, -0.0, -1.0, -1.0],        # +-0 tie, h2 = -0.5
            [0.5, 0.5, 0.5, 0.5],           # constant -> kappa 4
            [1.0, 1.0, 0.0, 0.0],           # h2 = 0.5 > 0 -> kappa 2
            [4.0, 3.0, 3.0, 3.0],           # h1 = 3 == z2 -> kappa 1
            [0.75, 0.25, -0.25, -0.25],     # h2 = 0 > -0.25 -> kappa 2
        ]
        z = np.asarray(rows, dtype=np.float32)
        return z, _rng(seed).integers(0, 4, len(rows)).astype(np.int64)
    return g


def parity_cases(full=False):
    """List of (name, generator).  `full` adds the slow, large cases."""
    cases = []
    for C in list(range(1, 65)) + [100, 127, 128, 129, 255, 256, 257, 511, 512, 513, 1000, 1023,
                                   1024, 1025, 2047, 2048]:
        cases.append((f"gauss_C{C}", gauss(6, C, 1.0, seed=C)))
    for C in [2049, 3000, 4096, 10000, 31623, 32000, 100000]:
        cases.append((f"gauss_mid_C{C}", gauss(5, C, 1.0, seed=C)))
    cases += [
        ("ties_C128", levels(64, 128, [-3.5, -2.5, -1.5, -0.5, 0.5, 1.5, 2.5, 3.5], seed=1)),
        ("ties_C5000", levels(16, 5000, [-1.0, 0.0, 1.0, 2.0], seed=2)),
        ("ties_C40000", levels(4, 40000, [0.0, 0.5, 1.0], seed=3)),
        ("const_C1", constant(4, 1)),
        ("const_C5", constant(4, 5, 2.0)),
        ("const_C1000", constant(4, 1000, -3.0)),
        ("const_C3000", constant(3, 3000, 1.0)),
        ("const_C40000", constant(2, 40000, 0.1)),
        ("sorted_C1000", sorted_rows(8, 1000, seed=4)),
        ("sorted_C40000", sorted_rows(4, 40000, seed=5)),
        ("twolevel_C700", two_level(16, 700, seed=6)),
        ("twolevel_C20000", two_level(8, 20000, seed=7)),
        ("outlier_C1000", outliers(8, 1000, seed=8)),
        ("outlier_C50000", outliers(4, 50000, seed=9)),
        ("mag1e30_C64", magnitude(6, 64, 1e30, seed=10)),
        ("mag1e30_C5000", magnitude(4, 5000, 1e30, seed=11)),
        ("mag1e20_C300", magnitude(6, 300, 1e20, seed=12)),
        ("mag1e-30_C300", magnitude(6, 300, 1e-30, seed=13)),
        ("zeros_C100", signed_zeros(16, 100, seed=14)),
        ("zeros_C9000", signed_zeros(4, 9000, seed=15)),
        ("neginf_C500", neg_inf(8, 500, seed=16)),
        ("neginf_C12000", neg_inf(4, 12000, seed=17)),
        ("dense_s1e-3_C1000", gauss(8, 1000, 1e-3, seed=18)),
        ("dense_s1e-3_C40000", gauss(4, 40000, 1e-3, seed=19)),
        ("dense_s1e-2_C100000", gauss(2, 100000, 1e-2, seed=20)),
        ("dense_s1e-1_C3000", gauss(8, 3000, 1e-1, seed=21)),
        ("exact_ties", exact_ties(seed=22)),
    ]
    if full:
        cases += [
            ("dense_s1e-3_C300000", gauss(2, 300000, 1e-3, seed=23)),
            ("gauss_C1000000", gauss(2, 1000000, 1.0, seed=24)),
        ]
    return cases


def nonfinite_cases():
    """Rows whose maximum is NaN or +-inf (policy, not reference, semantics)."""
    def g_nan():
        r = _rng(30)
        z = r.standard_normal((6, 3000)).astype(np.float32)
        z[0, 17] = np.nan
        z[1, 5] = np.inf
        z[2, :] = -np.inf
        z[3, 2999] = np.nan
        z[3, 10] = np.inf
        return z, _labels(r, 6, 3000)

    def g_small():
        r = _rng(31)
        z = r.standard_normal((5, 40)).astype(np.float32)
        z[0, 3] = np.nan
        z[1, 39] = np.inf
        z[2, :] = -np.inf
        z[3, 0] = -np.inf
        return z, _labels(r, 5, 40)

    return [("nonfinite_C3000", g_nan), ("nonfinite_C40", g_small)]


# --------------------------------------------------------------- float64 rows
def as_f64(gen):
    """A float32 case's values, as float64 rows."""
    def g():
        z, y = gen()
        return z.astype(np.float64), y
    return g


def gauss64(B, C, sigma=1.0, seed=0, offset=0.0):
    """float64 values with bits below float32 resolution."""
    def g():
        r = _rng(seed)
        z = offset + r.standard_normal((B, C)) * sigma
        return z, _labels(r, B, C)
    return g


def fine64(B, C, step, seed=0):
    """Rows 0.5 + j * step in random order: neighbours closer than a float32
    ulp, so the support is decided by float64 bits only."""
    def g():
        r = _rng(seed)
        z = 0.5 + np.stack([r.permutation(C) for _ in range(B)]).astype(np.float64) * step
        return z, _labels(r, B, C)
    return g


def magnitude64(B, C, scale, seed=0):
    def g():
        r = _rng(seed)
        z = r.standard_normal((B, C)) * scale
        z[0, : max(1, C // 3)] = z[0].max()
        return z, _labels(r, B, C)
    return g


def f64_cases():
    """(name, generator) for float64 logits; generators return float64 z."""
    cases = []
    for C in [1, 2, 3, 7, 31, 32, 33, 100, 128, 511, 1023, 1024, 1025, 2048, 5001, 32000]:
        cases.append((f"f64_gauss_C{C}", gauss64(6, C, 1.0, seed=100 + C)))
    cases += [
        ("f64_gauss_off1e6_C700", gauss64(6, 700, 0.5, seed=201, offset=1e6)),
        ("f64_gauss_off1e6_C9000", gauss64(4, 9000, 0.5, seed=202, offset=1e6)),
        ("f64_fine_C200", fine64(6, 200, 1e-12, seed=203)),          # dense, one warp per row
        ("f64_fine_C3000", fine64(4, 3000, 1e-4, seed=204)),          # dense, one CTA per row
        ("f64_fine_C2000_s1e-3", fine64(4, 2000, 1e-3, seed=205)),   # support ~ sqrt(2000)
        ("f64_dense_s1e-3_C1000", gauss64(6, 1000, 1e-3, seed=206)),
        ("f64_dense_s1e-3_C40000", gauss64(2, 40000, 1e-3, seed=207)),
        ("f64_ties_C128", as_f64(levels(32, 128, [-3.5, -2.5, -1.5, -0.5, 0.5, 1.5, 2.5, 3.5], seed=208))),
        ("f64_ties_C5000", as_f64(levels(8, 5000, [-1.0, 0.0, 1.0, 2.0], seed=209))),
        ("f64_const_C5", as_f64(constant(4, 5, 2.0))),
        ("f64_const_C3000", as_f64(constant(3, 3000, 1.0))),
        ("f64_sorted_C1000", as_f64(sorted_rows(8, 1000, seed=210))),
        ("f64_twolevel_C20000", as_f64(two_level(4, 20000, seed=211))),
        ("f64_outlier_C1000", as_f64(outliers(8, 1000, seed=212))),
        ("f64_zeros_C100", as_f64(signed_zeros(16, 100, seed=213))),
        ("f64_neginf_C500", as_f64(neg_inf(8, 500, seed=214))),
        ("f64_neginf_C12000", as_f64(neg_inf(4, 12000, seed=215))),
        ("f64_exact_ties", as_f64(exact_ties(seed=216))),
        ("f64_mag1e200_C64", magnitude64(6, 64, 1e200, seed=217)),
        ("f64_mag1e200_C5000", magnitude64(4, 5000, 1e200, seed=218)),
        ("f64_mag1e-200_C300", magnitude64(6, 300, 1e-200, seed=219)),
    ]
    return cases


def f64_nonfinite_cases():
    return [(name.replace("nonfinite", "f64_nonfinite"), as_f64(g)) for name, g in nonfinite_cases()]
