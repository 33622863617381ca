"""Loads the drop-in C++ module `fw_radix_cuda` built next to this package.

There is no fallback: if the module (or the CUDA library it links) is missing,
importing the operators raises, telling the user to build.
"""
import importlib
import os
import sys

import torch  # noqa: F401  (the extension links libtorch; load torch first)

_HERE = os.path.dirname(os.path.abspath(__file__))
_SRC_ROOT = os.path.dirname(_HERE)

_ext = None


def ext():
    global _ext
    if _ext is None:
        if _SRC_ROOT not in sys.path:
            sys.path.insert(0, _SRC_ROOT)
        try:
            _ext = importlib.import_module("fw_radix_cuda")
        except ImportError as e:  # no silent fallback to another implementation
            raise ImportError(
                "fwloss_b200: the native module fw_radix_cuda is not built or does not load "
                f"({e}); run `python build_native.py` in {_SRC_ROOT}") from e
    return _ext
