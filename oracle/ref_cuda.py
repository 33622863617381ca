"""Loads the reference's own CUDA extension built by oracle/build.py
(src/cuda/fw_radix_argmax.cu + src/cuda/binding.cpp for sm_100a, module
fw_radix_cuda_ref) -- TEST AND BASELINE INFRASTRUCTURE ONLY: the GPU baseline
bench.py times next to our kernels and a kappa parity check; nothing in the
product imports it.

forward_backward() is the reference benchmark's own dispatch
(benchmarks/cuda_benchmarks/CE_FW_perf.py:76-88): K < 10000 takes
fw_forward_small + fw_backward_small, larger K fw_forward + fw_backward.
"""
import importlib.machinery
import importlib.util
import os

from . import build as _build

_mod = None


def available():
    return os.path.exists(_build.ref_cuda_module_path())


def module():
    global _mod
    if _mod is None:
        import torch  # noqa: F401  (libtorch first)

        path = _build.ref_cuda_module_path()
        if not os.path.exists(path):
            raise ImportError("reference CUDA extension not built (run `python oracle/build.py` where the "
                              "reference checkout is present)")
        loader = importlib.machinery.ExtensionFileLoader("fw_radix_cuda_ref", path)
        spec = importlib.util.spec_from_file_location("fw_radix_cuda_ref", path, loader=loader)
        mod = importlib.util.module_from_spec(spec)
        loader.exec_module(mod)
        _mod = mod
    return _mod


def forward_backward(z, y):
    """(H, losses, mean, kappa, grad) of the reference CUDA path, as its
    benchmark calls it (the gradient carries the built-in 1/N)."""
    m = module()
    if z.shape[1] < 10000:
        H, losses, mean, kappa, sel = m.fw_forward_small(z, y)
        grad = m.fw_backward_small(y, sel, kappa)
    else:
        H, losses, mean, kappa, cb, ci, cc = m.fw_forward(z, y)
        grad = m.fw_backward(z, y, H, kappa, cb, ci, cc)
    return H, losses, mean, kappa, grad
