"""Parity at the benchmarked shapes.

Three checks that the shapes `bench.py` times compute the right thing:

* the memory read at configs[2]'s sequence length, heads and dims
  (T = 1024, sixteen 64-token chunks per sequence, H = 8, D = P = 64) against
  the float64 chunked oracle, at the north-star bars (rel 1e-4 forward,
  1e-3 gradients, absolute floor tol * max|expected|), with batch 2 so the
  oracle finishes in seconds;
* the full configs[2] problem (batch 128: a 9.7 GB factor residual whose
  offsets pass 4 GB): batch rows are independent, so rows 0, 63 and 127 of
  the full run must equal, bit for bit, the same operator run on that row
  alone; the floor gradient (a sum over the batch) must equal the sum of the
  128 single-row floor gradients within 1e-4 (float32 sums in another order);
* the bf16 scan at configs[1] (batch 16): rows 0 and 15 bit-exact against
  single-row runs, and the bias gradients (sums over the batch) against the
  sum of the 16 single-row bias gradients within 1e-4.

The reference pins the same operators at its own shapes
(`lm/tests/test_mamba4.py:382-404`, `lm/tests/test_flashmamba.py:98-168`).
"""

import math

import numpy as np
import pytest
import torch

from oracle import memread as M

pytestmark = pytest.mark.gpu

FWD_TOL = 1e-4
GRAD_TOL = 1e-3
MEM_NAMES = ("keys", "values", "queries", "beta", "log_decay")


def close(actual, expected, tol, name=""):
    actual = actual.detach().double().cpu().numpy()
    scale = float(np.abs(expected).max()) or 1.0
    np.testing.assert_allclose(actual, expected, rtol=tol, atol=tol * scale, err_msg=name)


def memread(inputs, floor, d_out, d_var):
    """Forward + backward through the public operator; returns outputs and the
    gradients of (keys, values, queries, beta, log_decay, floor)."""
    from mamba4_b200 import selective_memory_fused

    leaves = [inputs[n].detach().requires_grad_(True) for n in MEM_NAMES]
    fl = floor.detach().requires_grad_(True)
    res = selective_memory_fused(*leaves, fl)
    grads = torch.autograd.grad((res.output, res.variance), leaves + [fl], (d_out, d_var))
    outs = (res.output, res.variance, res.state.evidence, res.state.cross)
    return [o.detach() for o in outs], [g.detach() for g in grads]


def test_memory_read_config2_sequence_matches_oracle():
    # T = 1024 (16 chunks, 64 sub-chunks), H = 8, D = P = 64.
    cfg = M.config_inputs(2, 1024, 8, 64, 64, seed=0)
    dev = "cuda:0"
    t = {n: torch.tensor(cfg[n], device=dev) for n in cfg}
    outs, grads = memread(t, t["floor"], t["d_output"], t["d_variance"])
    args = [cfg[n] for n in (*MEM_NAMES, "floor")]
    fwd = M.chunked_forward(*args)
    for a, name in zip(outs, ("output", "variance", "evidence", "cross")):
        close(a, fwd[name], FWD_TOL, name)
    bwd = M.chunked_backward(*args, None, cfg["d_output"], cfg["d_variance"])
    for g, name in zip(grads, (*MEM_NAMES, "floor")):
        close(g, bwd[name], GRAD_TOL, name)


def config2_on_device(batch, seed, device):
    """configs[2] distributions generated on the device (the bench's recipe)."""
    g = torch.Generator(device=device).manual_seed(seed)
    T, H, D = 1024, 8, 64
    q = torch.randn(batch, T, H, D, device=device, generator=g) / 8
    k = torch.randn(batch, T, H, D, device=device, generator=g) / 8
    v = torch.randn(batch, T, H, D, device=device, generator=g)
    lam = torch.sigmoid(torch.randn(batch, T, H, device=device, generator=g) + 2.0)
    beta = torch.sigmoid(torch.randn(batch, T, H, device=device, generator=g))
    d_out = torch.randn(batch, T, H, D, device=device, generator=g)
    d_var = torch.randn(batch, T, H, device=device, generator=g)
    k = torch.cat((torch.zeros_like(k[:, :1]), k[:, :-1]), 1).contiguous()
    return dict(keys=k, values=v, queries=q, beta=beta, log_decay=torch.log(lam),
                d_output=d_out, d_variance=d_var)


def test_memory_read_full_config2_rows_equal_single_row_runs():
    dev = "cuda:0"
    batch = 128
    full = config2_on_device(batch, seed=5, device=dev)
    floor = torch.full((8, 64), 0.1, device=dev)
    outs, grads = memread(full, floor, full["d_output"], full["d_variance"])
    # The factor residual of this problem spans 9.7 GB: rows past 63 sit at
    # offsets beyond 2^32 bytes.
    from mamba4_b200 import _lib

    dims = _lib.MemDims(batch, 1024, 8, 64, 64)
    import ctypes

    assert _lib.load().m4_memread_residual_bytes(ctypes.byref(dims)) > 9 * 2**30
    floor_sum = torch.zeros(8, 64, dtype=torch.float64, device=dev)
    for row in range(batch):
        one = {n: v[row:row + 1].contiguous() for n, v in full.items()}
        o1, g1 = memread(one, floor, one["d_output"], one["d_variance"])
        floor_sum += g1[-1].double()
        if row in (0, 63, 127):
            for a, b, name in zip(outs[:2], o1[:2], ("output", "variance")):
                assert torch.equal(a[row:row + 1], b), (row, name)
            for a, b, name in zip(outs[2:], o1[2:], ("evidence", "cross")):
                assert torch.equal(a[row:row + 1], b), (row, name)
            for a, b, name in zip(grads[:-1], g1[:-1], MEM_NAMES):
                assert torch.equal(a[row:row + 1], b), (row, name)
    ref = floor_sum.cpu().numpy()
    close(grads[-1], ref, 1e-4, "floor (sum over the batch)")
    for t in (*outs, *grads):
        assert torch.isfinite(t).all()


SCAN_NAMES = ("c", "b", "x", "adt", "dt", "trap_logits", "angles", "q_bias", "k_bias")


def config1_on_device(batch, seed, device):
    """configs[1] distributions generated on the device (the bench's recipe)."""
    g = torch.Generator(device=device).manual_seed(seed)
    T, H, P, N = 1024, 16, 64, 64
    bf = torch.bfloat16
    x = (torch.randn(batch, T, H * P, device=device, generator=g) / 8).to(bf)
    b = (torch.randn(batch, T, N, device=device, generator=g) / 8).to(bf)
    c = (torch.randn(batch, T, N, device=device, generator=g) / 8).to(bf)
    dt = torch.nn.functional.softplus(torch.randn(batch, T, H, device=device, generator=g) * 0.5 - 3.0)
    a = -torch.exp(torch.rand(H, device=device, generator=g) * math.log(16.0))
    trap = torch.randn(batch, T, H, device=device, generator=g)
    angles = (torch.rand(batch, T, N // 2, device=device, generator=g) * 2 - 1) * math.pi
    d_y = torch.randn(batch, T, H * P, device=device, generator=g).to(bf)
    d_final = torch.randn(batch, H, N, P, device=device, generator=g)
    return dict(c=c, b=b, x=x, adt=a * dt, dt=dt, trap_logits=trap, angles=angles,
                q_bias=torch.ones(H, 1, N, device=device), k_bias=torch.ones(H, 1, N, device=device),
                d_y=d_y, d_final=d_final)


def scan(inputs):
    from mamba4_b200 import mamba3_fused

    leaves = [inputs[n].detach().requires_grad_(True) for n in SCAN_NAMES]
    y, final = mamba3_fused(*leaves[:7], q_bias=leaves[7], k_bias=leaves[8])
    grads = torch.autograd.grad((y, final), leaves, (inputs["d_y"], inputs["d_final"]))
    return y.detach(), final.detach(), [g.detach() for g in grads]


def test_scan_bf16_full_config1_rows_equal_single_row_runs():
    dev = "cuda:0"
    batch = 16
    full = config1_on_device(batch, seed=9, device=dev)
    y, final, grads = scan(full)
    bias_sum = [torch.zeros_like(full["q_bias"], dtype=torch.float64) for _ in range(2)]
    for row in range(batch):
        one = {n: (v if n in ("q_bias", "k_bias") else v[row:row + 1].contiguous()) for n, v in full.items()}
        y1, f1, g1 = scan(one)
        bias_sum[0] += g1[7].double()
        bias_sum[1] += g1[8].double()
        if row in (0, batch - 1):
            assert torch.equal(y[row:row + 1], y1), row
            assert torch.equal(final[row:row + 1], f1), row
            for a, b, name in zip(grads[:7], g1[:7], SCAN_NAMES):
                assert torch.equal(a[row:row + 1], b), (row, name)
    for g, ref, name in zip(grads[7:], bias_sum, ("q_bias", "k_bias")):
        close(g, ref.cpu().numpy(), 1e-4, name + " (sum over the batch)")
    for t in (y, final, *grads):
        assert torch.isfinite(t.float()).all()
