"""CUDA one-token decode kernels vs the float64 oracles (parity gate).

`selective_decode` (m4_memread_decode) follows lm/kernels/mamba4.py:341-355;
`mamba3_step` (m4_scan_step) the scan core of _Mamba3StepMixer,
lm/models/mamba4.py:412-481. Tolerances: float32 reads relative 1e-4 with an
absolute floor of 1e-4 x max|expected| (the north-star forward bar), the
reference's own decode-vs-prefill pin (rtol 3e-5, atol 3e-6,
lm/tests/test_mamba4.py:107-134) at its shapes, and bfloat16 steps within a
few bf16 units against the rounding-point oracle.
"""

import ctypes

import numpy as np
import pytest
import torch

from oracle import memread as M
from oracle import scan as S

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda:0")


def close(actual, expected, tol, name=""):
    actual = actual.detach().double().cpu().numpy() if torch.is_tensor(actual) else np.asarray(actual)
    expected = expected.detach().double().cpu().numpy() if torch.is_tensor(expected) else np.asarray(expected)
    scale = float(np.abs(expected).max()) or 1.0
    np.testing.assert_allclose(actual, expected, rtol=tol, atol=tol * scale, err_msg=name)


def _device_status_clear():
    from mamba4_b200 import _lib

    assert _lib.load().m4_device_status() == 0


def _random_state(batch, heads, dim, value_dim, seed):
    rng = np.random.default_rng(seed)
    s = rng.normal(size=(batch, heads, dim, dim)) * 0.3
    ev = (s @ np.swapaxes(s, -1, -2)).astype(np.float32)
    cr = (rng.normal(size=(batch, heads, value_dim, dim)) * 0.3).astype(np.float32)
    return ev, cr


@pytest.mark.parametrize("value_dim", [64, 128])
def test_memory_decode_matches_oracle(value_dim):
    from mamba4_b200 import SelectiveState, selective_decode

    batch, heads, dim = 3, 5, 64
    cfg = M.config_inputs(batch, 1, heads, dim, value_dim, seed=11)
    ev, cr = _random_state(batch, heads, dim, value_dim, seed=12)
    args = [cfg[n][:, 0] for n in ("keys", "values", "queries", "beta", "log_decay")]
    out, var, ev2, cr2 = M.decode_step(ev, cr, *args, cfg["floor"])
    t = lambda a: torch.tensor(a, device=DEV)  # noqa: E731
    res = selective_decode(SelectiveState(t(ev), t(cr)), *map(t, args), t(cfg["floor"]))
    close(res.output, out, 1e-4, "output")
    close(res.variance, var, 1e-4, "variance")
    close(res.state.evidence, ev2, 1e-5, "evidence")
    close(res.state.cross, cr2, 1e-5, "cross")
    _device_status_clear()


def test_memory_decode_steps_reproduce_prefill_at_reference_shapes():
    """The reference's decode-vs-prefill pin (lm/tests/test_mamba4.py:107-134):
    B 2, H 3, D 4, P 5 through the identity-block padding."""
    from mamba4_b200 import selective_decode, selective_initial_state, selective_memory_fused

    rng = np.random.default_rng(0)
    batch, time, heads, dim, value_dim = 2, 11, 3, 4, 5
    k = torch.tensor(rng.normal(size=(batch, time, heads, dim)).astype(np.float32), device=DEV)
    v = torch.tensor(rng.normal(size=(batch, time, heads, value_dim)).astype(np.float32), device=DEV)
    q = torch.tensor(rng.normal(size=(batch, time, heads, dim)).astype(np.float32), device=DEV)
    beta = torch.tensor(rng.uniform(0.2, 0.9, (batch, time, heads)).astype(np.float32), device=DEV)
    log_decay = torch.log(torch.tensor(rng.uniform(0.6, 0.99, (batch, time, heads)).astype(np.float32),
                                       device=DEV))
    floor = torch.tensor(rng.uniform(0.2, 0.8, (heads, dim)).astype(np.float32), device=DEV)
    full = selective_memory_fused(k, v, q, beta, log_decay, floor)
    state = selective_initial_state(batch, heads, dim, value_dim, device=DEV)
    for t in range(time):
        step = selective_decode(state, k[:, t], v[:, t], q[:, t], beta[:, t], log_decay[:, t], floor)
        state = step.state
        np.testing.assert_allclose(step.output.cpu().numpy(), full.output[:, t].cpu().numpy(),
                                   rtol=3e-5, atol=3e-6)
        np.testing.assert_allclose(step.variance.cpu().numpy(), full.variance[:, t].cpu().numpy(),
                                   rtol=3e-5, atol=3e-6)
    close(state.evidence, full.state.evidence, 1e-5, "evidence")
    close(state.cross, full.state.cross, 1e-5, "cross")


def test_memory_decode_in_place_through_the_c_abi():
    from mamba4_b200 import _lib

    lib = _lib.load()
    batch, heads, dim, value_dim = 2, 3, 64, 64
    cfg = M.config_inputs(batch, 1, heads, dim, value_dim, seed=21)
    ev, cr = _random_state(batch, heads, dim, value_dim, seed=22)
    args = [cfg[n][:, 0] for n in ("keys", "values", "queries", "beta", "log_decay")]
    out, var, ev2, cr2 = M.decode_step(ev, cr, *args, cfg["floor"])
    t = lambda a: torch.tensor(np.ascontiguousarray(a), device=DEV)  # noqa: E731
    e, c = t(ev), t(cr)
    k, v, qq, b, g = map(t, args)
    f = t(cfg["floor"])
    o = torch.empty(batch, heads, value_dim, device=DEV)
    s = torch.empty(batch, heads, device=DEV)
    dims = _lib.MemDims(batch, 1, heads, dim, value_dim)
    st = lib.m4_memread_decode(ctypes.byref(dims), *map(_lib.ptr, (e, c, k, v, qq, b, g, f, o, s, e, c)),
                               torch.cuda.current_stream().cuda_stream)
    assert st == 0
    close(o, out, 1e-4, "output")
    close(e, ev2, 1e-5, "evidence in place")
    close(c, cr2, 1e-5, "cross in place")


def _scan_inputs(batch, time, heads, state_dim, head_dim, seed):
    return S.config_inputs(batch, time, heads, head_dim, state_dim, seed=seed)


KEYS = ("c", "b", "x", "adt", "dt", "trap_logits", "angles")


@pytest.mark.parametrize("state_dim", [64, 128])
def test_scan_step_float32_reproduces_mamba3_fused(state_dim):
    from mamba4_b200 import mamba3_fused, mamba3_step, mamba3_step_cache

    batch, time, heads = 2, 70, 3
    sc = _scan_inputs(batch, time, heads, state_dim, 64, seed=5)
    t = lambda a: torch.tensor(a, device=DEV)  # noqa: E731
    args = [t(sc[n]) for n in KEYS]
    qb, kb = t(sc["q_bias"]), t(sc["k_bias"])
    y_full, final = mamba3_fused(*args, q_bias=qb, k_bias=kb)
    cache = mamba3_step_cache(batch, heads, state_dim, 64, sc["angles"].shape[-1], device=DEV)
    ys = []
    for i in range(time):
        y, cache = mamba3_step(cache, *[a[:, i] for a in args], q_bias=qb, k_bias=kb)
        ys.append(y)
    close(torch.stack(ys, 1), y_full, 1e-4, "y")
    close(cache.state, final, 1e-4, "final state")
    _device_status_clear()


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("state_dim,head_dim", [(64, 64), (16, 8), (96, 64), (128, 64)])
def test_scan_step_matches_oracle(dtype, state_dim, head_dim):
    from mamba4_b200 import Mamba3StepCache, mamba3_step

    batch, heads = 3, 4
    sc = _scan_inputs(batch, 1, heads, state_dim, head_dim, seed=7)
    rng = np.random.default_rng(8)
    angle_count = sc["angles"].shape[-1]
    cache = (rng.normal(size=(batch, heads, state_dim, head_dim)).astype(np.float32) * 0.1,
             rng.normal(size=(batch, heads, state_dim)).astype(np.float32) * 0.1,
             rng.normal(size=(batch, heads, head_dim)).astype(np.float32) * 0.1,
             rng.uniform(-3, 3, (batch, heads, angle_count)).astype(np.float32))
    step_in = [sc[n][:, 0] for n in KEYS]
    model = None if dtype == torch.float32 else torch.bfloat16
    if model is not None:  # c, b, x arrive in the model dtype
        step_in[:3] = [torch.tensor(a).to(model).float().numpy() for a in step_in[:3]]
    ey, (es, ek, ev, ep) = S.step_decode(cache, *step_in, sc["q_bias"], sc["k_bias"], model_dtype=model)
    t = lambda a: torch.tensor(a, device=DEV)  # noqa: E731
    args = [t(a) for a in step_in]
    args[0], args[1], args[2] = (a.to(dtype) for a in args[:3])
    y, new = mamba3_step(Mamba3StepCache(*map(t, cache)), *args, q_bias=t(sc["q_bias"]),
                         k_bias=t(sc["k_bias"]))
    assert y.dtype == dtype
    tol = 1e-4 if dtype == torch.float32 else 2e-2
    close(y, ey, tol, "y")
    close(new.state, es, 1e-4 if dtype == torch.float32 else 1e-2, "state")
    close(new.previous_keys, ek, 1e-5 if dtype == torch.float32 else 1e-2, "previous keys")
    close(new.previous_values, ev, 1e-6, "previous values")
    close(new.phase, ep, 1e-6, "phase")
    _device_status_clear()
