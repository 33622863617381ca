"""The C-ABI library and the drop-in module load and export what
include/fwloss_b200.h declares; host-side argument checks return their error
codes before any device work (CPU only)."""
import ctypes
import os
import re

import pytest

from fwloss_b200 import capi

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include",
                      "fwloss_b200.h")


def declared_symbols():
    text = open(HEADER).read()
    return re.findall(r"FWB_API\s+[\w\s\*]+?\b(fw_\w+)\s*\(", text)


def test_library_exports_every_declared_symbol():
    names = declared_symbols()
    assert len(names) >= 9
    lib = ctypes.CDLL(capi.LIB_PATH)
    for n in names:
        assert hasattr(lib, n), n
    assert set(names) == set(capi.EXPORTED)


def test_only_c_abi_is_exported():
    import subprocess

    out = subprocess.run(["nm", "-D", "--defined-only", capi.LIB_PATH], capture_output=True, text=True).stdout
    text_syms = {ln.split()[-1] for ln in out.splitlines() if " T " in ln}
    assert text_syms == set(declared_symbols())


def test_version_and_error_strings():
    assert capi.version() == "0.1.0"
    lib = capi.load()
    for code in range(7):
        assert lib.fw_error_string(code)
    assert b"unknown" in lib.fw_error_string(99)


def test_argument_checks_without_device():
    lib = capi.load()
    P = None
    dummy = ctypes.c_void_p(16)
    # C < 1, ld < C, B < 0 -> FWB_E_SHAPE
    assert lib.fw_fused_fwd_bwd(dummy, dummy, 4, 0, 0, 1.0, dummy, P, P, P, P, P) == 1
    assert lib.fw_fused_fwd_bwd(dummy, dummy, 4, 10, 9, 1.0, dummy, P, P, P, P, P) == 1
    assert lib.fw_fused_fwd_bwd(dummy, dummy, -1, 10, 10, 1.0, dummy, P, P, P, P, P) == 1
    assert lib.fw_forward_mask(dummy, dummy, 2, 2 ** 31, 2 ** 31, P, P, P, dummy, P, P) == 1
    # missing required pointers -> FWB_E_POINTER
    assert lib.fw_fused_fwd_bwd(P, dummy, 4, 10, 10, 1.0, dummy, P, P, P, P, P) == 2
    assert lib.fw_fused_fwd_bwd(dummy, dummy, 4, 10, 10, 1.0, P, P, P, P, P, P) == 2
    assert lib.fw_forward_candidates(dummy, dummy, 4, 10, 10, P, P, P, P, dummy, P, P, P) == 2
    assert lib.fw_backward_mask(P, dummy, dummy, 4, 10, 1.0, dummy, P, P) == 2
    assert lib.fw_loss_reduce(dummy, 4, 1.0, P, P) == 2
    # forward only: dtype, shape and pointer checks; an empty batch is a no-op
    assert lib.fw_forward_rows(7, dummy, dummy, 4, 10, 10, P, P, P, P, P) == 5
    assert lib.fw_forward_rows(0, dummy, dummy, 4, 10, 9, P, P, P, P, P) == 1
    assert lib.fw_forward_rows(1, P, dummy, 4, 10, 10, P, P, P, P, P) == 2
    assert lib.fw_forward_rows(2, dummy, P, 4, 10, 10, P, P, P, P, P) == 2
    assert lib.fw_forward_rows(0, P, P, 0, 10, 10, P, P, P, P, P) == 0
    assert lib.fw_forward_rows_f64(dummy, dummy, -1, 10, 10, P, P, P, P, P) == 1
    assert lib.fw_forward_rows_f64(P, dummy, 4, 10, 10, P, P, P, P, P) == 2
    assert lib.fw_forward_rows_f64(P, P, 0, 10, 10, P, P, P, P, P) == 0
    # an empty batch is a valid no-op (no launch)
    assert lib.fw_fused_fwd_bwd(P, P, 0, 10, 10, 1.0, P, P, P, P, P, P) == 0
    # float64 entry points: same checks
    assert lib.fw_fused_fwd_bwd_f64(dummy, dummy, 4, 10, 9, 1.0, dummy, P, P, P, P, P) == 1
    assert lib.fw_fused_fwd_bwd_f64(dummy, dummy, 4, 10, 10, 1.0, P, P, P, P, P, P) == 2
    assert lib.fw_fused_fwd_bwd_f64(P, P, 0, 10, 10, 1.0, P, P, P, P, P, P) == 0
    assert lib.fw_scale_grad_f64(dummy, P, 0, 1.0, 4, 10, 10, P) == 2
    assert lib.fw_loss_reduce_f64(dummy, 4, 1.0, P, P) == 2


def test_dropin_module_surface():
    import torch  # noqa: F401

    import fw_radix_cuda

    for fn in ("fw_forward", "fw_backward", "fw_forward_small", "fw_backward_small"):
        assert callable(getattr(fw_radix_cuda, fn))
    with pytest.raises(RuntimeError, match="CUDA"):
        fw_radix_cuda.fw_forward_small(torch.randn(2, 5), torch.zeros(2, dtype=torch.long))


def test_argument_checks_of_the_later_entry_points():
    """Shape, capacity, dtype and pointer checks that return before any device
    work: the listed-support forms, the vocabulary-parallel backward and the
    allocation-free LM-head forward."""
    lib = capi.load()
    P = None
    d = ctypes.c_void_p(256)
    # fw_fused_fwd_bwd_cols: dtype, shape, capacity (sup_k), pointers
    assert lib.fw_fused_fwd_bwd_cols(9, d, d, 4, 10, 10, 1.0, d, P, P, d, d, 8, P, P) == 5
    assert lib.fw_fused_fwd_bwd_cols(0, d, d, 4, 10, 9, 1.0, d, P, P, d, d, 8, P, P) == 1
    assert lib.fw_fused_fwd_bwd_cols(0, d, d, 4, 10, 10, 1.0, d, P, P, d, d, 0, P, P) == 4
    assert lib.fw_fused_fwd_bwd_cols(0, d, d, 4, 10, 10, 1.0, d, P, P, P, d, 8, P, P) == 2
    assert lib.fw_fused_fwd_bwd_cols(0, d, d, 4, 10, 10, 1.0, d, P, P, d, P, 8, P, P) == 2
    assert lib.fw_fused_fwd_bwd_cols(0, P, P, 0, 10, 10, 1.0, P, P, P, P, P, 8, P, P) == 0
    # fw_scale_grad_cols
    assert lib.fw_scale_grad_cols(0, d, 10, d, 0, d, d, d, 1, 1.0, 4, 10, P) == 4
    assert lib.fw_scale_grad_cols(0, P, 10, d, 8, d, d, d, 1, 1.0, 4, 10, P) == 2
    assert lib.fw_scale_grad_cols(0, d, 9, d, 8, d, d, d, 1, 1.0, 4, 10, P) == 1
    # vocabulary-parallel backward
    assert lib.fw_sparse_grad_hidden_shard(0, d, -1, 10, 8, d, 4, d, d, 4, 1.0, d, 0, d, P) == 1
    assert lib.fw_sparse_grad_hidden_shard(2, d, 0, 10, 8, d, 4, d, d, 4, 1.0, d, 0, d, P) == 5
    assert lib.fw_sparse_grad_hidden_shard(0, P, 0, 10, 8, d, 4, d, d, 4, 1.0, d, 0, d, P) == 2
    assert lib.fw_weight_grad_keys_shard(d, 4, d, d, 4, 0, 0, d, P) == 1
    assert lib.fw_weight_grad_keys_shard(P, 4, d, d, 4, 0, 10, d, P) == 2
    # allocation-free LM-head forward: chunk count and workspace limits
    cs = (ctypes.c_int64 * 3)(0, 256, 1000)
    assert lib.fw_lmhead_fused_loss_noalloc(1, d, 4, 64, d, 1000, 0, cs, 8, d, P, d, P, d, d, d, P, P) == 4
    assert lib.fw_lmhead_fused_loss_noalloc(1, d, 1 << 20, 64, d, 1000, 2, cs, 64, d, P, d, P, d, d, d, P, P) == 4
    assert lib.fw_lmhead_fused_loss_noalloc(1, d, -1, 64, d, 1000, 2, cs, 8, d, P, d, P, d, d, d, P, P) == 1
    # nchunks * K above the chunk solve's 256-entry list: refused before any kernel is queued
    cs16 = (ctypes.c_int64 * 17)(*[256 * i for i in range(17)])
    assert lib.fw_lmhead_fused_loss_noalloc(1, d, 4, 64, d, 4096, 16, cs16, 32, d, P, d, P, d, d, d, P, P) == 4


def test_argument_checks_of_the_cross_gpu_loss_sum():
    """fw_loss_allreduce refuses bad rank counts, ranks, pointers and timeouts
    before any device work; the exchange-buffer set-up refuses null
    pointers."""
    lib = capi.load()
    P = None
    d = ctypes.c_void_p(256)
    bufs = (ctypes.c_void_p * 9)(*([256] * 9))
    assert lib.fw_loss_allreduce(d, 4, 1.0, bufs, 9, 0, d, P, 1.0, P) == 4     # world > FWB_PEER_MAX
    assert lib.fw_loss_allreduce(d, 4, 1.0, bufs, 0, 0, d, P, 1.0, P) == 4     # world < 1
    assert lib.fw_loss_allreduce(d, 4, 1.0, bufs, 2, 2, d, P, 1.0, P) == 1     # rank outside [0, world)
    assert lib.fw_loss_allreduce(d, -1, 1.0, bufs, 2, 0, d, P, 1.0, P) == 1    # B < 0
    assert lib.fw_loss_allreduce(d, 4, 1.0, bufs, 2, 0, d, P, 0.0, P) == 1     # timeout must be > 0
    assert lib.fw_loss_allreduce(d, 4, 1.0, bufs, 2, 0, P, P, 1.0, P) == 2     # out
    assert lib.fw_loss_allreduce(P, 4, 1.0, bufs, 2, 0, d, P, 1.0, P) == 2     # losses
    holes = (ctypes.c_void_p * 2)(256, None)
    assert lib.fw_loss_allreduce_f64(d, 4, 1.0, holes, 2, 0, d, P, 1.0, P) == 2  # a missing buffer
    assert lib.fw_peer_buffer_create(P, d) == 2
    assert lib.fw_peer_buffer_open(P, d) == 2
    assert lib.fw_peer_buffer_close(P) == 2
    assert lib.fw_peer_buffer_destroy(P) == 2
