"""Autograd front-end of the fused FW-loss kernels.

    from fwloss_b200 import familywise_loss
    loss = familywise_loss(logits, target, reduction="mean")   # logits: [N, K] fp32 CUDA
    loss.backward()

Mirrors the CPU extension's `fwcpp.familywise_loss(logits, target,
reduction)` (src/cpu/fwcpp.py:18-19, src/cpu/fw_cpu.cpp:721-749): the
gradient is produced by the forward kernel (one read of the logits, one write
of the gradient) and saved; backward only applies the upstream gradient.
Unlike the CPU version, backward never synchronises with the host: the
upstream gradient is read on the device, and rows whose factor is exactly 1
(the usual `loss.backward()`) are left untouched.  "none" is supported in
addition to "mean" and "sum".

When no gradient can be asked for (under torch.no_grad(), or logits that do
not require grad -- evaluation with FWLoss), the forward-only kernel runs
instead: same H, losses and kappa, but the logits are read once and no
gradient is written (half the HBM bytes of the fused kernel).  The reference
computes the gradient in forward either way (src/cpu/fw_cpu.cpp:722-733).
"""
import torch

from ._native import ext

_REDUCTIONS = ("mean", "sum", "none")


def _wants_grad(logits):
    return torch.is_grad_enabled() and logits.requires_grad


def _forward_only(logits, target, status):
    """(losses in the logits' dtype, H, kappa) without a gradient."""
    H, losses, kappa = ext().forward_rows(logits.detach(), target, status)
    if logits.dtype not in (torch.float32, torch.float64):
        losses = losses.to(logits.dtype)
    return losses, H, kappa


def _check_inputs(logits, target):
    if not (isinstance(logits, torch.Tensor) and logits.is_cuda):
        raise TypeError("familywise_loss: logits must be a CUDA tensor (this build has no CPU path)")
    if logits.dim() != 2 or logits.dtype not in (torch.float32, torch.bfloat16, torch.float16, torch.float64):
        raise TypeError("familywise_loss: logits must be a 2-D float32, bfloat16, float16 or float64 tensor [N, K]")
    if target.dim() != 1 or target.shape[0] != logits.shape[0]:
        raise ValueError("familywise_loss: target must have shape [N]")
    if target.dtype != torch.int64:
        raise TypeError("familywise_loss: target must be int64")
    if target.device != logits.device:
        raise ValueError("familywise_loss: target must be on the logits' device")


class _FWRows(torch.autograd.Function):
    """Per-row losses [N] (differentiable), H [N] and kappa [N] (not).

    The gradient is computed in forward with scale `assumed`; backward
    multiplies row r by grad_losses[r] / assumed on the device.
    """

    @staticmethod
    def forward(ctx, logits, target, assumed, status):
        grad, H, losses, kappa = ext().fused_fwd_bwd(logits.detach(), target, float(assumed), status)
        ctx.grad = grad
        ctx.assumed = float(assumed)
        ctx.mark_non_differentiable(H, kappa)
        if logits.dtype != torch.float32:  # losses in the logits' dtype, like torch losses
            losses = losses.to(logits.dtype)
        return losses, H, kappa

    @staticmethod
    def backward(ctx, g_losses, g_H, g_kappa):
        grad = ctx.grad
        ctx.grad = None
        if g_losses is None:
            return None, None, None, None
        ext().scale_grad(grad, g_losses.contiguous(), True, ctx.assumed)
        return grad, None, None, None


SUPPORT_LIST = 8  # support columns listed per row for the per-row reduction
# Rows longer than this take the listed-support path for "none" (B200: cfg2
# shape forward+backward 278 -> 177 us); shorter rows stay in L2 and gain
# nothing from it (cfg1 shape: 19.0 vs 19.4 us).
LISTED_MIN_CLASSES = 2048


class _FWRowsListed(torch.autograd.Function):
    """_FWRows for float32/bfloat16/float16 logits with the support columns
    listed by the forward kernel: backward rewrites kappa + 1 entries per row
    (rows whose support is longer than the list are scaled whole)."""

    @staticmethod
    def forward(ctx, logits, target, status):
        grad, H, losses, kappa, cols = ext().fused_fwd_bwd_cols(logits.detach(), target, 1.0, SUPPORT_LIST, status)
        ctx.grad, ctx.cols, ctx.kappa, ctx.target = grad, cols, kappa, target
        ctx.mark_non_differentiable(H, kappa)
        if logits.dtype != torch.float32:
            losses = losses.to(logits.dtype)
        return losses, H, kappa

    @staticmethod
    def backward(ctx, g_losses, g_H, g_kappa):
        grad = ctx.grad
        ctx.grad = None
        if g_losses is None:
            return None, None, None
        ext().scale_grad_cols(grad, ctx.cols, ctx.kappa, ctx.target, g_losses.contiguous(), True, 1.0)
        return grad, None, None


class _FWReduced(torch.autograd.Function):
    """scale * sum of the per-row losses as a 0-d tensor ("mean"/"sum")."""

    @staticmethod
    def forward(ctx, logits, target, scale, status):
        grad, H, losses, kappa = ext().fused_fwd_bwd(logits.detach(), target, float(scale), status)
        ctx.grad = grad
        out = ext().loss_reduce(losses, float(scale))
        return out if logits.dtype == torch.float32 else out.to(logits.dtype)

    @staticmethod
    def backward(ctx, g):
        grad = ctx.grad
        ctx.grad = None
        ext().scale_grad(grad, g.reshape(1), False, 1.0)
        return grad, None, None, None


class _MeanOfRows(torch.autograd.Function):
    """Deterministic mean of a loss vector (fixed-order fp64 reduction)."""

    @staticmethod
    def forward(ctx, losses):
        ctx.n = losses.shape[0]
        wide = losses if losses.dtype == torch.float64 else losses.float()
        out = ext().loss_reduce(wide, 1.0 / ctx.n if ctx.n else float("nan"))
        return out if losses.dtype == torch.float32 else out.to(losses.dtype)

    @staticmethod
    def backward(ctx, g):
        return (g * (1.0 / ctx.n)).expand(ctx.n)


def familywise_loss(logits, target, reduction="mean", status=None):
    """FW loss of logits [N, K] (fp32, CUDA) against int64 targets [N].

    reduction "mean" / "sum" return a 0-d tensor, "none" the per-row losses.
    bfloat16 / float16 logits are accepted (fp32 arithmetic; gradient and loss
    in the logits' dtype), and float64 logits (fp64 arithmetic, gradient and
    loss; the reference CPU kernel's float64 path, src/cpu/fw_cpu.cpp:698-704).
    `status`, if given, is an int32 CUDA tensor whose first word receives the
    bit-or of FWB_STATUS_* flags (label out of range, non-finite row).
    """
    if reduction not in _REDUCTIONS:
        raise ValueError(f"Invalid reduction mode: {reduction}")
    _check_inputs(logits, target)
    n = logits.shape[0]
    scale = (1.0 / n if n else float("nan")) if reduction == "mean" else 1.0
    if not _wants_grad(logits):
        if reduction == "none":
            return _forward_only(logits, target, status)[0]
        _, losses, _ = ext().forward_rows(logits.detach(), target, status)  # fp32 (fp64) losses
        out = ext().loss_reduce(losses, scale)
        return out if out.dtype == logits.dtype else out.to(logits.dtype)
    if reduction == "none":
        if logits.dtype == torch.float64 or logits.shape[1] <= LISTED_MIN_CLASSES:
            return _FWRows.apply(logits, target, 1.0, status)[0]
        return _FWRowsListed.apply(logits, target, status)[0]
    return _FWReduced.apply(logits, target, scale, status)


def fw_rows(logits, target, assumed_scale=1.0, status=None):
    """(losses [N] differentiable, H [N] fp32 (fp64 for float64 logits), kappa [N] int32).
    Without a possible gradient (no_grad, or logits not requiring grad) the
    forward-only kernel runs and the losses are plain tensors."""
    _check_inputs(logits, target)
    if not _wants_grad(logits):
        return _forward_only(logits, target, status)
    return _FWRows.apply(logits, target, float(assumed_scale), status)


def mean_of_rows(losses):
    return _MeanOfRows.apply(losses)
