"""The allocation-free backward scan, m4_scan_bwd_noalloc.

Some callers of this library may not allocate device memory while the
operator runs: an XLA FFI custom call or other framework plugin that must not
use the device allocator, code recorded into a CUDA graph, or a server that
reserves all device memory up front. For them the library offers one
backward scan that takes its scratch from a fixed 32 MiB array compiled into
the library instead of a caller-provided workspace.

This file runs last (pytest collects files in name order) so that, if it
fails, a run that stops at the first failure has already run every other test.
It checks the allocation-free entry point against the regular one
(m4_scan_bwd with a caller workspace) on the same inputs, bf16 and float32,
for two calls in a row after a call on another problem has left unrelated
values in the shared scratch (which keeps the last call's contents): the
results must be identical bit for bit. It also checks that a problem larger
than the fixed scratch is refused without launching anything.
"""

import ctypes

import pytest
import torch

from oracle import scan as S

pytestmark = pytest.mark.gpu


def _inputs(batch, time, heads, seed, dtype):
    cfg = S.config_inputs(batch, time, heads, 64, 64, seed=seed)
    dev = "cuda:0"
    t = {k: torch.tensor(v, device=dev) for k, v in cfg.items()}
    for k in ("c", "b", "x", "d_y"):
        t[k] = t[k].to(dtype).contiguous()
    t["q_bias"] = t["q_bias"].reshape(heads, 64).contiguous()
    t["k_bias"] = t["k_bias"].reshape(heads, 64).contiguous()
    return t


def _forward(lib, dims, t):
    """m4_scan_fwd into a fresh residual; returns the residual."""
    rbytes = lib.m4_scan_residual_bytes(ctypes.byref(dims))
    resid = torch.empty(rbytes, dtype=torch.uint8, device="cuda:0")
    y = torch.empty_like(t["x"])
    final = torch.empty(dims.batch, dims.heads, 64, 64, device="cuda:0")
    p = lambda x: x.data_ptr()  # noqa: E731
    status = lib.m4_scan_fwd(ctypes.byref(dims), *[p(t[k]) for k in ("c", "b", "x", "adt", "dt",
                                                                      "trap_logits", "angles",
                                                                      "q_bias", "k_bias")],
                             p(y), p(final), p(resid), rbytes, torch.cuda.current_stream().cuda_stream)
    assert status == 0, lib.m4_status_string(status)
    return resid


def _grads(lib, dims, t, resid, noalloc):
    outs = dict(
        dc=torch.empty_like(t["c"]), db=torch.empty_like(t["b"]), dx=torch.empty_like(t["x"]),
        d_adt=torch.empty_like(t["adt"]), d_dt=torch.empty_like(t["dt"]),
        d_trap=torch.empty_like(t["trap_logits"]), d_angles=torch.empty_like(t["angles"]),
        d_qb=torch.empty_like(t["q_bias"]), d_kb=torch.empty_like(t["k_bias"]),
    )
    p = lambda x: x.data_ptr()  # noqa: E731
    common = [ctypes.byref(dims)] + [p(t[k]) for k in ("c", "b", "x", "adt", "dt", "trap_logits",
                                                         "angles", "q_bias", "k_bias")]
    common += [p(resid), resid.numel(), p(t["d_y"]), p(t["d_final"])]
    common += [p(outs[k]) for k in ("dc", "db", "dx", "d_adt", "d_dt", "d_trap", "d_angles",
                                    "d_qb", "d_kb")]
    stream = torch.cuda.current_stream().cuda_stream
    if noalloc:
        status = lib.m4_scan_bwd_noalloc(*common, stream)
    else:
        wbytes = lib.m4_scan_workspace_bytes(ctypes.byref(dims))
        work = torch.empty(wbytes, dtype=torch.uint8, device="cuda:0")
        status = lib.m4_scan_bwd(*common, p(work), wbytes, stream)
    assert status == 0, lib.m4_status_string(status)
    torch.cuda.synchronize()
    return outs


@pytest.mark.parametrize("bf16", [1, 0])
def test_noalloc_backward_matches_workspace_backward_on_two_calls(bf16):
    from mamba4_b200 import _lib

    lib = _lib.load()
    dtype = torch.bfloat16 if bf16 else torch.float32
    batch, time, heads = 2, 300, 16
    t = _inputs(batch, time, heads, seed=21, dtype=dtype)
    dims = _lib.ScanDims(batch, time, heads, 64, 64, 32, 64, bf16, 0)
    resid = _forward(lib, dims, t)
    expected = _grads(lib, dims, t, resid, noalloc=False)
    # Leave unrelated values in the shared scratch first: another problem
    # (other inputs, another length, so every buffer inside the scratch sits
    # at another offset). A kernel that read scratch before writing it would
    # then see stale data.
    other = _inputs(3, 171, 16, seed=5, dtype=dtype)
    odims = _lib.ScanDims(3, 171, 16, 64, 64, 32, 64, bf16, 0)
    _grads(lib, odims, other, _forward(lib, odims, other), noalloc=True)
    for call in range(2):
        got = _grads(lib, dims, t, resid, noalloc=True)
        for name in expected:
            # Same kernels, same inputs: identical bits, whatever the scratch held.
            assert torch.equal(got[name], expected[name]), f"{name} (call {call + 1})"


def test_noalloc_backward_refuses_problems_beyond_its_scratch():
    from mamba4_b200 import _lib

    lib = _lib.load()
    # 64 x 1024 x 16 token-heads need about 690 MB of scratch, above the fixed
    # 32 MiB: the call returns M4_ERR_WORKSPACE before launching anything.
    dims = _lib.ScanDims(64, 1024, 16, 64, 64, 32, 64, 1, 0)
    assert lib.m4_scan_workspace_bytes(ctypes.byref(dims)) > (32 << 20)
    buf = torch.zeros(1024, dtype=torch.uint8, device="cuda:0")
    ptrs = [buf.data_ptr()] * 9
    resid_bytes = lib.m4_scan_residual_bytes(ctypes.byref(dims))
    status = lib.m4_scan_bwd_noalloc(ctypes.byref(dims), *ptrs, buf.data_ptr(), resid_bytes,
                                     buf.data_ptr(), None, *([buf.data_ptr()] * 9),
                                     torch.cuda.current_stream().cuda_stream)
    assert status == 6  # M4_ERR_WORKSPACE
