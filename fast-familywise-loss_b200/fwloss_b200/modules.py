"""`FWLoss` module with the constructor and outputs of the reference's
`reference_impl.FWLoss` (reference_impl.py:3-35), computed by the fused CUDA
kernels instead of sort + cumsum + max.

    fw = FWLoss(num_classes, reduction="mean", device="cuda")
    H, losses, mean, kappas = fw(logits, target)      # "mean"
    mean.backward()

Outputs for reduction "mean": H [N] fp32 (the threshold h*, rounded toward
-inf), per-row losses [N], their mean (0-d) and kappas [N] int64 (support
sizes, the reference's `max_result.indices + 1`).  "sum" returns
losses.sum(), "none" the per-row losses, as in the reference.
"""
import torch

from .functional import fw_rows, mean_of_rows, _REDUCTIONS


class FWLoss(torch.nn.Module):
    def __init__(self, num_classes, reduction="mean", device="cpu"):
        super().__init__()
        if reduction not in _REDUCTIONS:
            raise ValueError(f"Invalid reduction mode: {reduction}")
        self.num_classes = int(num_classes)
        self.reduction = reduction
        self.device = device

    def forward(self, input, target):
        if input.shape[-1] != self.num_classes:
            raise ValueError(f"FWLoss: expected {self.num_classes} classes, got {input.shape[-1]}")
        n = input.shape[0]
        if self.reduction == "mean":
            losses, H, kappa = fw_rows(input, target, 1.0 / n if n else 1.0)
            return H, losses, mean_of_rows(losses), kappa.to(torch.int64)
        losses, H, kappa = fw_rows(input, target, 1.0)
        if self.reduction == "sum":
            return losses.sum()
        return losses
