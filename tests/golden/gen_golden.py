"""Writes the golden fixtures of tests/golden/ from the REFERENCE itself.

Run in a container that has the reference checkout (the directory named by the
environment variable FW_REF_PATH, or else a checkout named `reference` beside
this repository) and the reference CPU extension built by oracle/build.py:

    python tests/golden/gen_golden.py

Outputs (inputs are not stored: every case regenerates them from its seed,
see tests/cases.py and fwloss_b200.workloads; each case records the sha256 of
the regenerated inputs as `<case>/input_sha256`, so that a test on another
host can tell whether its inputs are the ones these outputs were made from --
torch's CPU normal generator gives different float32 values on hosts that run
its scalar kernels instead of the AVX2/AVX-512 ones):
  reference_outputs.npz  per case: what reference_impl.FWLoss (float32, CPU;
                         reference_impl.py:3-35) and the reference CPU
                         extension (src/cpu/fw_cpu.cpp, fw_loss_grad) return:
                         kappa, H, per-row loss and the gradient (sparse:
                         row, col, value) for reduction "mean".
  reference_outputs_f64.npz
                         the same for the float64 cases (cases.f64_cases):
                         reference_impl.FWLoss on float64 tensors and the
                         CPU extension's float64 branch (fw_cpu.cpp:698-704);
                         gradients in float64.
  config_inputs.npz      the inputs of the reduced benchmark configurations
                         (first rows of each; `--config-inputs` rewrites only
                         this file), so that their reference pin needs no
                         regeneration on the testing host.
  kat_kbar.json          the known answers the reference ships: the `kbar`
                         (mean kappa over 32 rows) of every (distribution,
                         sigma, K) in benchmarks/cpu_benchmarks/results/*.json,
                         with the generation parameters of
                         benchmarks/cpu_benchmarks/bench_cpu_e2e.py:7-41.
"""
import hashlib
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)
sys.path.insert(0, os.path.join(REPO, "tests"))
sys.path.insert(0, os.path.join(REPO, "fast-familywise-loss_b200"))
REF = os.environ.get("FW_REF_PATH") or os.path.join(os.path.dirname(REPO), "reference")
sys.path.insert(0, REF)

import torch  # noqa: E402

import cases  # noqa: E402
from fwloss_b200 import workloads  # noqa: E402
from oracle import ref_cpu  # noqa: E402
import reference_impl  # noqa: E402  (the reference's own module)

CONFIG_ROWS = {"cfg0": 256, "cfg1": 512, "cfg2": 64, "cfg3": 2048, "cfg4": 8}


def input_sha256(z, y):
    return np.array(hashlib.sha256(np.ascontiguousarray(z).tobytes() + np.ascontiguousarray(y).tobytes()).hexdigest())


def sparse(g):
    r, c = np.nonzero(g)
    return r.astype(np.int32), c.astype(np.int32), g[r, c].astype(np.float32)


def reference_outputs(z, y):
    B, C = z.shape
    zt = torch.from_numpy(z).clone().requires_grad_(True)
    yt = torch.from_numpy(y)
    H, losses, mean, kappas = reference_impl.FWLoss(C, reduction="mean")(zt, yt)
    mean.backward()
    L, G, K = ref_cpu.ref_loss_grad(z, y, 1.0 / B)
    out = {
        "kappa_ref32": kappas.numpy().astype(np.int64),
        "H_ref32": H.detach().numpy().astype(np.float32),
        "loss_ref32": losses.detach().numpy().astype(np.float32),
        "mean_ref32": np.float32(mean.item()),
        "kappa_cpu": K.astype(np.int64),
        "loss_cpu": L.astype(np.float64),
    }
    for tag, g in (("grad_ref32", zt.grad.numpy()), ("grad_cpu", G)):
        r, c, v = sparse(g)
        out[tag + "_r"], out[tag + "_c"], out[tag + "_v"] = r, c, v
    return out


def reference_outputs_f64(z, y):
    B, C = z.shape
    zt = torch.from_numpy(z).clone().requires_grad_(True)
    yt = torch.from_numpy(y)
    H, losses, mean, kappas = reference_impl.FWLoss(C, reduction="mean")(zt, yt)
    mean.backward()
    L, G, K = ref_cpu.ref_loss_grad64(z, y, 1.0 / B)
    out = {
        "kappa_ref64": kappas.numpy().astype(np.int64),
        "H_ref64": H.detach().numpy().astype(np.float64),
        "loss_ref64": losses.detach().numpy().astype(np.float64),
        "kappa_cpu64": K.astype(np.int64),
        "loss_cpu64": L.astype(np.float64),
    }
    for tag, g in (("grad_ref64", zt.grad.numpy()), ("grad_cpu64", G)):
        r, c = np.nonzero(g)
        out[tag + "_r"], out[tag + "_c"] = r.astype(np.int32), c.astype(np.int32)
        out[tag + "_v"] = g[r, c].astype(np.float64)
    return out


def all_cases():
    for name, gen in cases.parity_cases(full=False):
        yield name, gen
    for name, rows in CONFIG_ROWS.items():
        def g(name=name, rows=rows):
            z, y = workloads.make(name, rows=rows)
            return z.numpy(), y.numpy()
        yield name, g


def kat():
    res = os.path.join(REF, "benchmarks", "cpu_benchmarks", "results")
    out = {}
    for fname in ("gaussian.json", "gaussian_avx2_1thread.json", "laplace.json", "mixture.json"):
        d = json.load(open(os.path.join(res, fname)))
        stds = list(d["runs"].keys())
        entry = {"N": d["N"], "Ks": d["Ks"], "dist": d.get("dist", "gaussian"),
                 "mix_mean": d.get("mix_mean", 2.0), "stds": stds, "kbar": {}}
        for s in stds:
            runs = d["runs"][s]["FW (ours)"]
            assert [r["K"] for r in runs] == d["Ks"], fname
            entry["kbar"][s] = [r["kbar"] for r in runs]
        out[fname[:-5]] = entry
    return out


# Rows of each reduced configuration whose inputs are stored in
# config_inputs.npz (the first rows of the fixture cases above; fewer rows
# where the full case would be large).
STORED_ROWS = {"cfg0": 256, "cfg1": 512, "cfg2": 16, "cfg3": 2048, "cfg4": 4}


def write_config_inputs():
    """config_inputs.npz: the inputs of the reduced benchmark configurations
    (their first STORED_ROWS rows), so that the golden comparison of those
    cases does not depend on the host regenerating them with torch's CPU
    generator.  Checked against the fingerprint the fixtures recorded for the
    whole case."""
    golden = np.load(os.path.join(HERE, "reference_outputs.npz"))
    store = {}
    for name, rows in CONFIG_ROWS.items():
        z, y = workloads.make(name, rows=rows)
        z, y = z.numpy(), y.numpy()
        assert str(golden[f"{name}/input_sha256"]) == str(input_sha256(z, y)), \
            f"{name}: this host regenerates other inputs than the fixtures were made from"
        n = STORED_ROWS[name]
        store[f"{name}/z"] = np.ascontiguousarray(z[:n])
        store[f"{name}/y"] = np.ascontiguousarray(y[:n])
        store[f"{name}/case_rows"] = np.int64(rows)
    np.savez_compressed(os.path.join(HERE, "config_inputs.npz"), **store)


def main():
    if "--config-inputs" in sys.argv:  # only the stored inputs (fixtures unchanged)
        write_config_inputs()
        return
    store = {}
    for name, gen in all_cases():
        z, y = gen()
        for k, v in reference_outputs(z, y).items():
            store[f"{name}/{k}"] = v
        store[f"{name}/input_sha256"] = input_sha256(z, y)
        print(name, z.shape, flush=True)
    np.savez_compressed(os.path.join(HERE, "reference_outputs.npz"), **store)
    store64 = {}
    for name, gen in cases.f64_cases():
        z, y = gen()
        for k, v in reference_outputs_f64(z, y).items():
            store64[f"{name}/{k}"] = v
        store64[f"{name}/input_sha256"] = input_sha256(z, y)
        print(name, z.shape, flush=True)
    np.savez_compressed(os.path.join(HERE, "reference_outputs_f64.npz"), **store64)
    with open(os.path.join(HERE, "kat_kbar.json"), "w") as f:
        json.dump(kat(), f, indent=1)


if __name__ == "__main__":
    main()
