"""Loads the reference's CPU extension built by oracle/build.py, and the C
restatement -- TEST INFRASTRUCTURE ONLY (checker and timed CPU baseline).

ref_module() returns the module compiled from the reference's
src/cpu/fw_cpu.cpp for the best ISA this host supports; its functions are the
reference's own: familywise_loss(Z, y, reduction 0=sum/1=mean),
fw_loss_grad(Z, y, scale, flat_kmax, serial_below, use_chunked),
set_params, simd (src/cpu/fw_cpu.cpp:745-779).
"""
import ctypes
import importlib.machinery
import importlib.util
import os

import numpy as np

from . import build as _build

_mods = {}
_oracle = None


def host_isas():
    try:
        flags = open("/proc/cpuinfo").read()
    except OSError:
        flags = ""
    have = []
    if all(f" {f}" in flags for f in ("avx512f", "avx512dq", "avx512bw", "avx512vl")):
        have.append("avx512")
    if " avx2" in flags and " fma" in flags:
        have.append("avx2")
    return have


def ref_available():
    return any(os.path.exists(_build.ref_module_path(i)) for i in host_isas())


def ref_module(isa=None):
    """The reference CPU extension (raises if it was not built)."""
    import torch  # noqa: F401  (libtorch must be loaded first)

    isas = [isa] if isa else host_isas()
    for i in isas:
        path = _build.ref_module_path(i)
        if not os.path.exists(path):
            continue
        if i not in _mods:
            name = f"fw_cpu_ref_{i}"
            loader = importlib.machinery.ExtensionFileLoader(name, path)
            spec = importlib.util.spec_from_file_location(name, path, loader=loader)
            mod = importlib.util.module_from_spec(spec)
            loader.exec_module(mod)
            _mods[i] = mod
        return _mods[i]
    raise ImportError("reference CPU extension not built (run `python oracle/build.py` where the "
                      "reference checkout is present)")


def ref_loss_grad(z, y, scale):
    """(loss [B] f64, grad [B, C] f32 scaled, kappa [B] i64) from the
    reference CPU code (fw_loss_grad, src/cpu/fw_cpu.cpp:750-756)."""
    import torch

    m = ref_module()
    Z = torch.as_tensor(np.ascontiguousarray(z, dtype=np.float32))
    Y = torch.as_tensor(np.ascontiguousarray(y, dtype=np.int64))
    L, G, K = m.fw_loss_grad(Z, Y, float(scale), 2 ** 62, 100_000, True)
    return L.numpy(), G.numpy(), K.numpy()


def ref_loss_grad64(z, y, scale):
    """(loss [B] f64, grad [B, C] f64 scaled, kappa [B] i64) from the
    reference CPU code on float64 logits (fw_loss_grad, its float64 branch,
    src/cpu/fw_cpu.cpp:698-704)."""
    import torch

    m = ref_module()
    Z = torch.as_tensor(np.ascontiguousarray(z, dtype=np.float64))
    Y = torch.as_tensor(np.ascontiguousarray(y, dtype=np.int64))
    L, G, K = m.fw_loss_grad(Z, Y, float(scale), 2 ** 62, 100_000, True)
    return L.numpy(), G.numpy(), K.numpy()


def c_oracle():
    global _oracle
    if _oracle is None:
        path = _build.build_oracle()
        lib = ctypes.CDLL(path)
        P = ctypes.c_void_p
        lib.fwo_solve_rows.argtypes = [P, P, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                                       P, P, P, P, ctypes.c_int]
        lib.fwo_solve_rows.restype = None
        _oracle = lib
    return _oracle


def c_solve(z, y, threads=0):
    """C restatement: (tau, kappa, M, loss) as numpy arrays."""
    z = np.ascontiguousarray(z, dtype=np.float32)
    y = np.ascontiguousarray(y, dtype=np.int64)
    B, C = z.shape
    tau = np.empty(B)
    kap = np.empty(B, dtype=np.int64)
    M = np.empty(B)
    loss = np.empty(B)
    c_oracle().fwo_solve_rows(z.ctypes.data, y.ctypes.data, B, C, C, tau.ctypes.data,
                              kap.ctypes.data, M.ctypes.data, loss.ctypes.data, int(threads))
    return tau, kap, M, loss
