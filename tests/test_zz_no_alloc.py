"""fw_lmhead_fused_loss_noalloc: the LM-head FW-loss forward for callers that
cannot allocate device memory (a plugin whose host framework owns all device
memory, a server that forbids allocation after start-up, an FFI host that only
holds the buffers it is given).  It keeps its workspace in a fixed array inside
the library, so the caller passes only inputs and outputs.

The test calls it through the C ABI and compares every output with the
allocating pair fw_lmhead_fused_scan + fw_chunks_solve run on buffers from
torch.  Two calls in a row with different shapes and data check that nothing
left in the shared array by one call leaks into the next.  The file name sorts
last so that a run stopping at its first failure has run every other test."""
import ctypes

import numpy as np
import pytest
import torch

from fwloss_b200 import capi
from fwloss_b200.lm_head import tile_col_start

pytestmark = pytest.mark.gpu

FWB_OK = 0
FWB_E_CAPACITY = 4
DTYPE_BF16 = 1
SCRATCH_WORDS = 16 * 1024 * 1024 // 4  # FWB_NOALLOC_SCRATCH_BYTES / 4


def _p(t):
    return ctypes.c_void_p(t.data_ptr())


def _inputs(B, D, C, seed, zero_rows=(), bad_label=None):
    g = torch.Generator(device="cuda").manual_seed(seed)
    hidden = (torch.randn(B, D, generator=g, device="cuda") / D ** 0.5 * 4.0).to(torch.bfloat16)
    weight = torch.randn(C, D, generator=g, device="cuda").to(torch.bfloat16)
    target = torch.randint(0, C, (B,), generator=g, device="cuda")
    for r in zero_rows:
        hidden[r] = 0  # constant logits: the row goes to the caller's exact path
    if bad_label is not None:
        target[bad_label] = C + 3
    return hidden, weight, target


def _outputs(B, nchunks, K):
    return {
        "H": torch.full((B,), -7.0, device="cuda"),
        "kappa": torch.full((B,), -7, dtype=torch.int32, device="cuda"),
        "loss": torch.full((B,), -7.0, device="cuda"),
        "sup_cols": torch.full((B, nchunks * K), -7, dtype=torch.int32, device="cuda"),
        "fb_rows": torch.full((B,), -7, dtype=torch.int32, device="cuda"),
        "fb_count": torch.full((1,), -7, dtype=torch.int32, device="cuda"),
        "status": torch.zeros(1, dtype=torch.int32, device="cuda"),
    }


def _with_caller_workspace(lib, hidden, weight, target, cs, K, out, stream):
    B, D = hidden.shape
    C = weight.shape[0]
    n = len(cs) - 1
    summaries = torch.empty((n, B, 4 + K), dtype=torch.int32, device="cuda")
    local_idx = torch.empty((n, B, K), dtype=torch.int32, device="cuda")
    zy = torch.empty(B, device="cuda")
    col = (ctypes.c_int64 * len(cs))(*cs)
    rc = lib.fw_lmhead_fused_scan(DTYPE_BF16, _p(hidden), B, D, _p(weight), C, n, col, K, _p(target), _p(zy),
                                  _p(summaries), _p(local_idx), _p(out["status"]), stream)
    assert rc == FWB_OK
    rc = lib.fw_chunks_solve(_p(summaries), _p(local_idx), n, col, B, K, _p(zy), _p(target), _p(out["H"]),
                             _p(out["kappa"]), _p(out["loss"]), _p(out["sup_cols"]), _p(out["fb_rows"]),
                             _p(out["fb_count"]), _p(out["status"]), stream)
    assert rc == FWB_OK


def _no_alloc(lib, hidden, weight, target, cs, K, out, stream):
    B, D = hidden.shape
    C = weight.shape[0]
    n = len(cs) - 1
    col = (ctypes.c_int64 * len(cs))(*cs)
    return lib.fw_lmhead_fused_loss_noalloc(DTYPE_BF16, _p(hidden), B, D, _p(weight), C, n, col, K, _p(target),
                                            _p(out["H"]), _p(out["kappa"]), _p(out["loss"]), _p(out["sup_cols"]),
                                            _p(out["fb_rows"]), _p(out["fb_count"]), _p(out["status"]), stream)


def _host(out):
    return {k: v.cpu().numpy() for k, v in out.items()}


CALLS = [
    # (B, D, C, nchunks, K, seed, zero_rows, bad_label)
    (300, 256, 5000, 3, 16, 11, (), None),
    (130, 512, 12345, 5, 8, 12, (0, 1, 77), 5),
]


def test_no_alloc_matches_caller_workspace_on_two_calls_in_a_row():
    lib = capi.load()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    for B, D, C, nchunks, K, seed, zero_rows, bad_label in CALLS:
        hidden, weight, target = _inputs(B, D, C, seed, zero_rows, bad_label)
        cs = tile_col_start(C, nchunks)
        n = len(cs) - 1
        ref = _outputs(B, n, K)
        _with_caller_workspace(lib, hidden, weight, target, cs, K, ref, stream)
        got = _outputs(B, n, K)
        assert _no_alloc(lib, hidden, weight, target, cs, K, got, stream) == FWB_OK
        torch.cuda.synchronize()
        r, g = _host(ref), _host(got)
        assert g["status"][0] == r["status"][0]
        assert (g["status"][0] & 1) == (1 if bad_label is not None else 0)
        np.testing.assert_array_equal(g["kappa"], r["kappa"])
        np.testing.assert_array_equal(g["sup_cols"], r["sup_cols"])
        np.testing.assert_allclose(g["H"], r["H"], rtol=1e-5, atol=1e-6)
        np.testing.assert_allclose(g["loss"], r["loss"], rtol=1e-5, atol=1e-6)
        nfb = int(r["fb_count"][0])
        assert int(g["fb_count"][0]) == nfb == len(zero_rows)
        np.testing.assert_array_equal(np.sort(g["fb_rows"][:nfb]), np.sort(r["fb_rows"][:nfb]))
        if bad_label is not None:
            assert np.isnan(g["loss"][bad_label])


def test_no_alloc_rejects_problems_beyond_its_workspace():
    lib = capi.load()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    # nchunks * B * (4 + 2K) + B words must fit in the fixed workspace
    B, D, C, K = 8192, 64, 4096, 32
    cs = tile_col_start(C, 8)
    n = len(cs) - 1
    assert n * B * (4 + 2 * K) + B > SCRATCH_WORDS
    hidden, weight, target = _inputs(B, D, C, 3)
    out = _outputs(B, n, K)
    assert _no_alloc(lib, hidden, weight, target, cs, K, out, stream) == FWB_E_CAPACITY
    torch.cuda.synchronize()
    assert int(out["kappa"].min()) == -7 and int(out["kappa"].max()) == -7  # nothing was written
    # a small batch whose chunk lists exceed the solve's 256 entries per row
    # (nchunks * K = 16 * 32): refused before the scan touches the array
    B, C, K = 64, 16 * 256, 32
    cs = tile_col_start(C, 16)
    n = len(cs) - 1
    assert n * K > 256
    hidden, weight, target = _inputs(B, D, C, 4)
    out = _outputs(B, n, K)
    assert _no_alloc(lib, hidden, weight, target, cs, K, out, stream) == FWB_E_CAPACITY
    torch.cuda.synchronize()
    assert int(out["kappa"].min()) == -7 and int(out["kappa"].max()) == -7
    assert int(out["status"][0]) == 0
