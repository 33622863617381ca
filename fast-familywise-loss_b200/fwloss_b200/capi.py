"""ctypes binding of the C ABI in libfwloss_b200.so (include/fwloss_b200.h).

Every wrapper takes CUDA tensors, passes raw device pointers, sizes and the
current torch stream of the tensors' device, and raises FWError on a non-zero
return code.  Nothing here computes anything: all work happens in the CUDA
kernels behind the C ABI.  This is the path the GPU parity tests use, and the
template for a binding from another host language (cgo, JNI, N-API): one
foreign-function prototype per declaration of the header, raw pointers in,
an int status out.
"""
import ctypes
import os

import torch

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libfwloss_b200.so")

FWB_OK = 0
FWB_STATUS_LABEL_RANGE = 1
FWB_STATUS_NONFINITE = 2

_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_SIGS = {
    "fw_version": ([], ctypes.c_char_p),
    "fw_error_string": ([ctypes.c_int], ctypes.c_char_p),
    "fw_fused_fwd_bwd": ([_P, _P, _I64, _I64, _I64, ctypes.c_float, _P, _P, _P, _P, _P, _P], ctypes.c_int),
    "fw_forward_mask": ([_P, _P, _I64, _I64, _I64, _P, _P, _P, _P, _P, _P], ctypes.c_int),
    "fw_backward_mask": ([_P, _P, _P, _I64, _I64, ctypes.c_float, _P, _P, _P], ctypes.c_int),
    "fw_forward_candidates": ([_P, _P, _I64, _I64, _I64, _P, _P, _P, _P, _P, _P, _P, _P], ctypes.c_int),
    "fw_backward_candidates": ([_P, _P, _P, _P, _P, _P, _I64, _I64, ctypes.c_float, _P, _P, _P], ctypes.c_int),
    "fw_scale_grad": ([_P, _P, ctypes.c_int, ctypes.c_float, _I64, _I64, _I64, _P], ctypes.c_int),
    "fw_loss_reduce": ([_P, _I64, ctypes.c_double, _P, _P], ctypes.c_int),
    "fw_fused_fwd_bwd_typed": ([ctypes.c_int, _P, _P, _I64, _I64, _I64, ctypes.c_float, _P, _P, _P, _P,
                                _P, _P], ctypes.c_int),
    "fw_scale_grad_typed": ([ctypes.c_int, _P, _P, ctypes.c_int, ctypes.c_float, _I64, _I64, _I64, _P],
                            ctypes.c_int),
}
_SIGS["fw_fused_fwd_bwd_cols"] = ([ctypes.c_int, _P, _P, _I64, _I64, _I64, ctypes.c_float, _P, _P, _P, _P, _P,
                                   ctypes.c_int, _P, _P], ctypes.c_int)
_SIGS["fw_scale_grad_cols"] = ([ctypes.c_int, _P, _I64, _P, ctypes.c_int, _P, _P, _P, ctypes.c_int, ctypes.c_float,
                                _I64, _I64, _P], ctypes.c_int)
_SIGS["fw_shard_scan"] = ([_P, _I64, _I64, _I64, ctypes.c_int, _P, _P, _P, _P], ctypes.c_int)
_SIGS["fw_shard_solve"] = ([_P, ctypes.c_int, ctypes.c_int, _P, _I64, ctypes.c_int, _P, _I64, _P,
                           ctypes.c_float, _P, _P, _P, _P, _P, _P, _P, _P, _P], ctypes.c_int)
_SIGS["fw_label_logits"] = ([_P, _I64, _I64, _I64, _P, _I64, _P, _P], ctypes.c_int)
_SIGS["fw_chunks_solve"] = ([_P, _P, ctypes.c_int, _P, _I64, ctypes.c_int, _P, _P, _P, _P, _P, _P, _P, _P, _P,
                            _P], ctypes.c_int)
_SIGS["fw_sparse_grad_hidden"] = ([ctypes.c_int, _P, _I64, _I64, _P, ctypes.c_int, _P, _P, _I64, ctypes.c_float,
                                  _P, ctypes.c_int, _P, _P], ctypes.c_int)
_SIGS["fw_sparse_grad_weight"] = ([ctypes.c_int, _P, _I64, _I64, _P, ctypes.c_int, _P, _P, _I64, ctypes.c_float,
                                  _P, ctypes.c_int, _P, _P], ctypes.c_int)
_SIGS["fw_weight_grad_keys"] = ([_P, ctypes.c_int, _P, _P, _I64, _I64, _P, _P], ctypes.c_int)
_SIGS["fw_segment_grad_weight"] = ([ctypes.c_int, _P, _I64, _I64, _P, _I64, _P, ctypes.c_float, _P,
                                   ctypes.c_int, _P, _P], ctypes.c_int)
_SIGS["fw_lmhead_fused_scan"] = ([ctypes.c_int, _P, _I64, _I64, _P, _I64, ctypes.c_int, _P, ctypes.c_int, _P, _P,
                                  _P, _P, _P, _P], ctypes.c_int)
_SIGS["fw_fused_fwd_bwd_f64"] = ([_P, _P, _I64, _I64, _I64, ctypes.c_double, _P, _P, _P, _P, _P, _P],
                                 ctypes.c_int)
_SIGS["fw_scale_grad_f64"] = ([_P, _P, ctypes.c_int, ctypes.c_double, _I64, _I64, _I64, _P], ctypes.c_int)
_SIGS["fw_loss_reduce_f64"] = ([_P, _I64, ctypes.c_double, _P, _P], ctypes.c_int)
_SIGS["fw_sparse_grad_hidden_shard"] = ([ctypes.c_int, _P, _I64, _I64, _I64, _P, ctypes.c_int, _P, _P, _I64,
                                         ctypes.c_float, _P, ctypes.c_int, _P, _P], ctypes.c_int)
_SIGS["fw_weight_grad_keys_shard"] = ([_P, ctypes.c_int, _P, _P, _I64, _I64, _I64, _P, _P], ctypes.c_int)
_SIGS["fw_forward_rows"] = ([ctypes.c_int, _P, _P, _I64, _I64, _I64, _P, _P, _P, _P, _P], ctypes.c_int)
_SIGS["fw_forward_rows_f64"] = ([_P, _P, _I64, _I64, _I64, _P, _P, _P, _P, _P], ctypes.c_int)
_SIGS["fw_lmhead_fused_loss_noalloc"] = ([ctypes.c_int, _P, _I64, _I64, _P, _I64, ctypes.c_int, _P, ctypes.c_int,
                                          _P, _P, _P, _P, _P, _P, _P, _P, _P], ctypes.c_int)
_SIGS["fw_peer_buffer_create"] = ([_P, _P], ctypes.c_int)
_SIGS["fw_peer_buffer_open"] = ([_P, _P], ctypes.c_int)
_SIGS["fw_peer_buffer_close"] = ([_P], ctypes.c_int)
_SIGS["fw_peer_buffer_destroy"] = ([_P], ctypes.c_int)
_SIGS["fw_loss_allreduce"] = ([_P, _I64, ctypes.c_double, _P, ctypes.c_int, ctypes.c_int, _P, _P,
                               ctypes.c_double, _P], ctypes.c_int)
_SIGS["fw_loss_allreduce_f64"] = ([_P, _I64, ctypes.c_double, _P, ctypes.c_int, ctypes.c_int, _P, _P,
                                   ctypes.c_double, _P], ctypes.c_int)
DTYPE_CODES = {torch.float32: 0, torch.bfloat16: 1, torch.float16: 2}
_ANY_FLOAT = (torch.float32, torch.bfloat16, torch.float16, torch.float64)

EXPORTED = tuple(_SIGS)

_lib = None


class FWError(RuntimeError):
    pass


def load():
    """Loads the library (once) and declares the prototypes."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise FWError(f"{LIB_PATH} is missing: run `python build_native.py` in the package directory")
        lib = ctypes.CDLL(LIB_PATH)
        for name, (args, res) in _SIGS.items():
            fn = getattr(lib, name)
            fn.argtypes = args
            fn.restype = res
        _lib = lib
    return _lib


def version():
    return load().fw_version().decode()


def _ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream(t):
    return ctypes.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


def _check(rc, what):
    if rc != FWB_OK:
        raise FWError(f"{what}: {load().fw_error_string(rc).decode()} (code {rc})")


def _rows(z, any_float=False):
    if z.dim() != 2 or not z.is_cuda or z.dtype not in (_ANY_FLOAT if any_float else (torch.float32,)):
        raise FWError("logits must be a 2-D float32 CUDA tensor" +
                      (" (or bfloat16 / float16 / float64)" if any_float else ""))
    if z.stride(1) != 1 or (z.size(0) > 1 and z.stride(0) < z.size(1)):
        z = z.contiguous()
    ld = z.stride(0) if z.size(0) > 1 else z.size(1)
    return z, max(ld, z.size(1))


def fused_fwd_bwd(z, y, grad_scale, grad=None, status=None):
    """(grad, H, loss, kappa) from the fused kernel; grad has z's row stride
    and dtype (float32 logits use fw_fused_fwd_bwd, 16-bit logits
    fw_fused_fwd_bwd_typed, float64 logits fw_fused_fwd_bwd_f64 with fp64 H
    and loss)."""
    z, ld = _rows(z, any_float=True)
    B, C = z.shape
    if grad is None:
        grad = torch.empty_strided((B, C), (ld, 1), dtype=z.dtype, device=z.device)
    f64 = z.dtype == torch.float64
    H = torch.empty(B, dtype=torch.float64 if f64 else torch.float32, device=z.device)
    loss = torch.empty(B, dtype=H.dtype, device=z.device)
    kappa = torch.empty(B, dtype=torch.int32, device=z.device)
    lib = load()
    with torch.cuda.device(z.device):
        if f64:
            rc = lib.fw_fused_fwd_bwd_f64(_ptr(z), _ptr(y), B, C, ld, float(grad_scale), _ptr(grad),
                                          _ptr(H), _ptr(loss), _ptr(kappa), _ptr(status), _stream(z))
        elif z.dtype == torch.float32:
            rc = lib.fw_fused_fwd_bwd(_ptr(z), _ptr(y), B, C, ld, float(grad_scale), _ptr(grad),
                                      _ptr(H), _ptr(loss), _ptr(kappa), _ptr(status), _stream(z))
        else:
            rc = lib.fw_fused_fwd_bwd_typed(DTYPE_CODES[z.dtype], _ptr(z), _ptr(y), B, C, ld,
                                            float(grad_scale), _ptr(grad), _ptr(H), _ptr(loss),
                                            _ptr(kappa), _ptr(status), _stream(z))
        _check(rc, "fw_fused_fwd_bwd")
    return grad, H, loss, kappa


def forward_rows(z, y, status=None):
    """(H, loss, kappa) without a gradient (fw_forward_rows; float64 logits:
    fw_forward_rows_f64 with fp64 H and loss)."""
    z, ld = _rows(z, any_float=True)
    B, C = z.shape
    f64 = z.dtype == torch.float64
    H = torch.empty(B, dtype=torch.float64 if f64 else torch.float32, device=z.device)
    loss = torch.empty(B, dtype=H.dtype, device=z.device)
    kappa = torch.empty(B, dtype=torch.int32, device=z.device)
    lib = load()
    with torch.cuda.device(z.device):
        if f64:
            rc = lib.fw_forward_rows_f64(_ptr(z), _ptr(y), B, C, ld, _ptr(H), _ptr(loss), _ptr(kappa),
                                         _ptr(status), _stream(z))
        else:
            rc = lib.fw_forward_rows(DTYPE_CODES[z.dtype], _ptr(z), _ptr(y), B, C, ld, _ptr(H), _ptr(loss),
                                     _ptr(kappa), _ptr(status), _stream(z))
        _check(rc, "fw_forward_rows")
    return H, loss, kappa


def forward_mask(z, y, status=None):
    z, ld = _rows(z)
    B, C = z.shape
    mask = torch.empty((B, C), dtype=torch.bool, device=z.device)
    H = torch.empty(B, dtype=torch.float32, device=z.device)
    loss = torch.empty(B, dtype=torch.float32, device=z.device)
    kappa = torch.empty(B, dtype=torch.int32, device=z.device)
    with torch.cuda.device(z.device):
        _check(load().fw_forward_mask(_ptr(z), _ptr(y), B, C, ld, _ptr(H), _ptr(loss), _ptr(kappa),
                                      _ptr(mask), _ptr(status), _stream(z)), "fw_forward_mask")
    return H, loss, kappa, mask


def backward_mask(y, mask, kappa, grad_scale, status=None):
    B, C = mask.shape
    grad = torch.empty((B, C), dtype=torch.float32, device=mask.device)
    with torch.cuda.device(mask.device):
        _check(load().fw_backward_mask(_ptr(y), _ptr(mask.contiguous()), _ptr(kappa), B, C,
                                       float(grad_scale), _ptr(grad), _ptr(status), _stream(mask)),
               "fw_backward_mask")
    return grad


def forward_candidates(z, y, status=None):
    z, ld = _rows(z)
    B, C = z.shape
    dev = z.device
    cv = torch.empty((B, C), dtype=torch.float32, device=dev)
    ci = torch.empty((B, C), dtype=torch.int32, device=dev)
    cc = torch.empty(B, dtype=torch.int32, device=dev)
    H = torch.empty(B, dtype=torch.float32, device=dev)
    loss = torch.empty(B, dtype=torch.float32, device=dev)
    kappa = torch.empty(B, dtype=torch.int32, device=dev)
    with torch.cuda.device(dev):
        _check(load().fw_forward_candidates(_ptr(z), _ptr(y), B, C, ld, _ptr(H), _ptr(loss),
                                            _ptr(kappa), _ptr(cv), _ptr(ci), _ptr(cc), _ptr(status),
                                            _stream(z)), "fw_forward_candidates")
    return H, loss, kappa, cv, ci, cc


def backward_candidates(cv, ci, cc, H, kappa, y, grad_scale, status=None):
    B, C = cv.shape
    grad = torch.empty((B, C), dtype=torch.float32, device=cv.device)
    with torch.cuda.device(cv.device):
        _check(load().fw_backward_candidates(_ptr(cv), _ptr(ci), _ptr(cc), _ptr(H), _ptr(kappa),
                                             _ptr(y), B, C, float(grad_scale), _ptr(grad),
                                             _ptr(status), _stream(cv)), "fw_backward_candidates")
    return grad


def scale_grad(grad, grad_output, per_row, assumed_scale):
    B, C = grad.shape
    ld = grad.stride(0) if B > 1 else C
    if grad.dtype == torch.float64:
        go = grad_output.to(torch.float64)
        with torch.cuda.device(grad.device):
            _check(load().fw_scale_grad_f64(_ptr(grad), _ptr(go), int(bool(per_row)), float(assumed_scale),
                                            B, C, ld, _stream(grad)), "fw_scale_grad_f64")
        return grad
    go = grad_output.to(torch.float32)
    with torch.cuda.device(grad.device):
        _check(load().fw_scale_grad_typed(DTYPE_CODES[grad.dtype], _ptr(grad), _ptr(go), int(bool(per_row)),
                                          float(assumed_scale), B, C, ld, _stream(grad)), "fw_scale_grad")
    return grad


def loss_reduce(loss, scale):
    """scale * sum(loss) for float32 or float64 losses (result of the same dtype)."""
    out = torch.empty((), dtype=loss.dtype, device=loss.device)
    fn = load().fw_loss_reduce_f64 if loss.dtype == torch.float64 else load().fw_loss_reduce
    with torch.cuda.device(loss.device):
        _check(fn(_ptr(loss), loss.numel(), float(scale), _ptr(out), _stream(loss)), "fw_loss_reduce")
    return out


def shard_scan(z, K):
    """Class-sharded step 1 on this rank's shard: (grad shard, summary, local_idx)."""
    z, ld = _rows(z)
    B, C = z.shape
    grad = torch.empty_strided((B, C), (ld, 1), dtype=torch.float32, device=z.device)
    summary = torch.empty((B, 4 + K), dtype=torch.int32, device=z.device)
    local_idx = torch.empty((B, K), dtype=torch.int32, device=z.device)
    with torch.cuda.device(z.device):
        _check(load().fw_shard_scan(_ptr(z), B, C, ld, int(K), _ptr(grad), _ptr(summary), _ptr(local_idx),
                                    _stream(z)), "fw_shard_scan")
    return grad, summary, local_idx


def shard_solve(gathered, rank, col_start, z, y, grad_scale, grad, local_idx, status=None):
    """Class-sharded step 3: (H, kappa, loss_part, fb_rows, fb_count); grad patched in place."""
    z, ld = _rows(z)
    B = z.shape[0]
    nranks = len(col_start) - 1
    K = gathered.shape[2] - 4
    cs = (ctypes.c_int64 * len(col_start))(*[int(c) for c in col_start])
    dev = z.device
    H = torch.empty(B, dtype=torch.float32, device=dev)
    kappa = torch.empty(B, dtype=torch.int32, device=dev)
    loss_part = torch.empty(B, dtype=torch.float32, device=dev)
    fb_rows = torch.empty(max(B, 1), dtype=torch.int32, device=dev)
    fb_count = torch.empty(1, dtype=torch.int32, device=dev)
    with torch.cuda.device(dev):
        _check(load().fw_shard_solve(_ptr(gathered.contiguous()), nranks, int(rank), cs, B, int(K), _ptr(z), ld,
                                     _ptr(y), float(grad_scale), _ptr(grad), _ptr(local_idx), _ptr(H),
                                     _ptr(kappa), _ptr(loss_part), _ptr(fb_rows), _ptr(fb_count),
                                     _ptr(status), _stream(z)), "fw_shard_solve")
    return H, kappa, loss_part, fb_rows, fb_count
