"""Replays the input generation of the reference's CPU benchmark, whose result
files carry exact known answers: `kbar`, the mean support size kappa over the
N rows of each (distribution, sigma, K) (benchmarks/cpu_benchmarks/
results/*.json, copied into tests/golden/kat_kbar.json by gen_golden.py).

Draw order (benchmarks/cpu_benchmarks/bench_cpu_e2e.py:26-41): one
numpy.random.default_rng(0) for the whole file; for each sigma in file
order, for each K: Z = gen(K, sigma).astype(float32), then
y = rng.integers(0, K, N), where gen is
  gaussian: standard_normal((N, K)) * sigma
  laplace:  laplace(0, sigma / sqrt(2), (N, K))
  mixture:  pick = random((N, K)) < 0.5;
            where(pick, standard_normal((N, K)), mix_mean + sigma * standard_normal((N, K)))
"""
import json
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
KAT_PATH = os.path.join(HERE, "golden", "kat_kbar.json")


def load():
    with open(KAT_PATH) as f:
        return json.load(f)


def replay(entry):
    """Yields (sigma_str, K, kbar, Z float32 [N, K], y int64 [N]) in draw order."""
    rng = np.random.default_rng(0)
    N = entry["N"]
    dist = entry["dist"]
    mm = entry["mix_mean"]
    for s in entry["stds"]:
        std = float(s)
        for K, kbar in zip(entry["Ks"], entry["kbar"][s]):
            if dist == "gaussian":
                Z = rng.standard_normal((N, K)) * std
            elif dist == "laplace":
                Z = rng.laplace(0.0, std / np.sqrt(2.0), (N, K))
            else:
                pick = rng.random((N, K)) < 0.5
                Z = np.where(pick, rng.standard_normal((N, K)), mm + std * rng.standard_normal((N, K)))
            Z = Z.astype(np.float32)
            y = rng.integers(0, K, N)
            yield s, K, kbar, Z, y.astype(np.int64)
