"""fwloss_b200: Familywise loss forward+backward on NVIDIA B200 (sm_100a).

Python API (drop-in for the reference's Python-facing entry points):
  familywise_loss(logits, target, reduction)  like fwcpp.familywise_loss
  FWLoss(num_classes, reduction, device)      like reference_impl.FWLoss
  fw_radix_cuda (sibling module)              like the reference's extension
C ABI: libfwloss_b200.so, declared in include/fwloss_b200.h; `capi` binds it
with ctypes.
"""
from .functional import familywise_loss, fw_rows, mean_of_rows  # noqa: F401
from .modules import FWLoss  # noqa: F401
from . import capi  # noqa: F401

__all__ = ["familywise_loss", "fw_rows", "mean_of_rows", "FWLoss", "capi"]
__version__ = "0.1.0"
