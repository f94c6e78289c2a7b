"""The CPU oracle against the reference's golden vectors and known answers.

The fixtures in tests/golden/ were produced by the reference's own NumPy
operator code (analysis/memory.py, analysis/gradients.py) with
tests/golden/make_golden.py. These tests pin the oracle before the CUDA
parity tests rely on it.
"""

from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import memread as M
from oracle import scan as S

GOLDEN = Path(__file__).resolve().parent / "golden"


def test_memory_oracle_matches_reference_evidence_reads():
    g = np.load(GOLDEN / "memory_reads.npz")
    time, dim = g["keys"].shape
    f = M.dense_forward(
        g["keys"][None, :, None],
        g["values"][None, :, None],
        g["queries"][None, :, None],
        g["beta"][None, :, None],
        np.log(g["decay"])[None, :, None],
        np.full((1, dim), float(g["ridge"])),
    )
    np.testing.assert_allclose(f["output"][0, :, 0], g["reads"], rtol=1e-12, atol=1e-12)
    np.testing.assert_allclose(f["variance"][0, :, 0], g["confidences"], rtol=1e-12)
    np.testing.assert_allclose(f["evidence"][0, 0], g["evidence"], atol=1e-12)
    np.testing.assert_allclose(f["cross"][0, 0], g["cross"], atol=1e-12)
    for chunk in (1, 4, 5, 16):
        c = M.chunked_forward(
            g["keys"][None, :, None], g["values"][None, :, None],
            g["queries"][None, :, None], g["beta"][None, :, None],
            np.log(g["decay"])[None, :, None], np.full((1, dim), float(g["ridge"])),
            chunk_size=chunk,
        )
        np.testing.assert_allclose(c["output"][0, :, 0], g["reads"], rtol=1e-10, atol=1e-12)


@pytest.mark.parametrize("form", ["dense", "chunked"])
def test_memory_oracle_gradients_match_reference_terminal_vjp(form):
    g = np.load(GOLDEN / "memory_terminal_vjp.npz")
    time, dim = g["keys"].shape
    value_dim = g["values"].shape[1]
    queries = np.zeros((time, dim))
    queries[-1] = g["query"]
    d_out = np.zeros((1, time, 1, value_dim))
    d_out[0, -1, 0] = g["upstream"]
    args = (
        g["keys"][None, :, None], g["values"][None, :, None], queries[None, :, None],
        g["beta"][None, :, None], np.log(g["decay"])[None, :, None],
        np.full((1, dim), float(g["ridge"])), None, d_out, np.zeros((1, time, 1)),
    )
    if form == "dense":
        grads = M.dense_backward(*args)
    else:
        grads = M.chunked_backward(*args, chunk_size=4)
    np.testing.assert_allclose(grads["keys"][0, :, 0], g["grad_keys"], rtol=1e-9, atol=1e-12)
    np.testing.assert_allclose(grads["values"][0, :, 0], g["grad_values"], rtol=1e-9, atol=1e-12)
    np.testing.assert_allclose(grads["beta"][0, :, 0], g["grad_beta"], rtol=1e-9, atol=1e-12)
    # The reference differentiates the decay itself; the operator takes its log.
    np.testing.assert_allclose(
        grads["log_decay"][0, :, 0], g["grad_decay"] * g["decay"], rtol=1e-9, atol=1e-12
    )
    np.testing.assert_allclose(grads["queries"][0, -1, 0], g["grad_query"], rtol=1e-9)


def _random_memory(batch=2, time=13, heads=3, dim=4, value_dim=5, seed=0):
    # Input recipe of lm/tests/test_mamba4.py:187-197.
    rng = np.random.default_rng(seed)
    k = rng.normal(size=(batch, time, heads, dim))
    q = rng.normal(size=k.shape)
    k /= np.linalg.norm(k, axis=-1, keepdims=True)
    q /= np.linalg.norm(q, axis=-1, keepdims=True)
    v = rng.normal(size=(batch, time, heads, value_dim))
    beta = rng.uniform(0.05, 1.0, size=k.shape[:-1])
    decay = rng.uniform(0.3, 0.999, size=k.shape[:-1])
    floor = rng.uniform(0.25, 1.5, size=(heads, dim))
    return k, v, q, beta, np.log(decay), floor


@pytest.mark.parametrize("chunk", [1, 4, 5, 13, 16])
def test_chunked_oracle_equals_dense_recurrence(chunk):
    # lm/tests/test_mamba4.py:32-43 (chunked reads vs sequential dense solves).
    args = _random_memory()
    dense = M.dense_forward(*args)
    chunked = M.chunked_forward(*args, chunk_size=chunk)
    for name in ("output", "variance", "evidence", "cross"):
        np.testing.assert_allclose(chunked[name], dense[name], rtol=1e-10, atol=1e-12)


def test_chunk_form_gradients_equal_torch_autograd():
    rng = np.random.default_rng(7)
    k, v, q, beta, log_decay, floor = _random_memory(time=11, seed=3)
    batch, time, heads, dim = k.shape
    p = v.shape[-1]
    s0 = rng.normal(size=(batch, heads, dim, dim))
    s0 = s0 @ np.swapaxes(s0, -1, -2) * 0.1
    c0 = rng.normal(size=(batch, heads, p, dim)) * 0.1
    cot = [rng.normal(size=s) for s in ((batch, time, heads, p), (batch, time, heads),
                                         (batch, heads, dim, dim), (batch, heads, p, dim))]
    leaves = [torch.tensor(a, requires_grad=True) for a in (k, v, q, beta, log_decay, floor, s0, c0)]
    kk, vv, qq, bb, gg, ff, ss, cc = leaves
    eye = torch.eye(dim, dtype=torch.float64)
    outs, var = [], []
    for t in range(time):
        lam = torch.exp(gg[:, t])[..., None, None]
        ss = lam * ss + bb[:, t, :, None, None] * kk[:, t, :, :, None] * kk[:, t, :, None, :]
        cc = lam * cc + bb[:, t, :, None, None] * vv[:, t, :, :, None] * kk[:, t, :, None, :]
        y = torch.linalg.solve(ss + ff[None, :, :, None] * eye, qq[:, t, ..., None])[..., 0]
        outs.append(torch.einsum("bhpd,bhd->bhp", cc, y))
        var.append((qq[:, t] * y).sum(-1))
    loss = sum((a * torch.tensor(c)).sum() for a, c in zip(
        (torch.stack(outs, 1), torch.stack(var, 1), ss, cc), cot))
    expected = torch.autograd.grad(loss, leaves)
    names = ["keys", "values", "queries", "beta", "log_decay", "floor", "evidence0", "cross0"]
    for chunk in (3, 8):
        got = M.chunked_backward(k, v, q, beta, log_decay, floor, (s0, c0), *cot, chunk_size=chunk)
        for name, want in zip(names, expected):
            np.testing.assert_allclose(got[name], want.numpy(), rtol=1e-9, atol=1e-11)


def test_exact_recall_of_independent_keys_as_floor_vanishes():
    # Known answer, lm/tests/test_mamba4.py:137-152: read(k_i) = v_i / (1 + floor/beta).
    dim, value_dim = 4, 3
    keys = np.eye(dim)[None, :, None, :]
    values = np.random.default_rng(1).normal(size=(1, dim, 1, value_dim))
    beta = np.full((1, dim, 1), 2.0)
    f = M.dense_forward(keys, values, keys, beta, np.zeros_like(beta), np.full((1, dim), 1e-3))
    precision = f["evidence"][0, 0] + 1e-3 * np.eye(dim)
    for i in range(dim):
        read = f["cross"][0, 0] @ np.linalg.solve(precision, keys[0, i, 0])
        np.testing.assert_allclose(read, values[0, i, 0] / (1 + 5e-4), rtol=1e-12)


def test_precision_respects_undiscounted_floor():
    # lm/tests/test_mamba4.py:46-58.
    k, v, q, beta, log_decay, floor = _random_memory(time=40)
    decay = np.exp(log_decay)
    decay[:, ::7] = 1e-4
    decay[:, 3::7] = 1.0
    f = M.chunked_forward(k, v, q, beta, np.log(decay), floor, chunk_size=8)
    precision = f["evidence"] + floor[None, :, :, None] * np.eye(4)
    assert np.all(np.linalg.eigvalsh(precision)[..., 0] >= floor.min(-1)[None] - 1e-9)
    assert np.all(f["variance"] <= 1 / floor.min() + 1e-9)


def test_scan_oracle_matches_reference_mamba3_core():
    g = np.load(GOLDEN / "mamba3_reads.npz")
    time = len(g["dt"])
    trap_logits = np.log(g["trap"] / (1 - g["trap"]))
    t = lambda a: torch.tensor(np.asarray(a, np.float64))  # noqa: E731
    for chunk in (1, 3, 16):
        y, _ = S.chunked_scan(
            t(g["q"])[None, :, None], t(g["b"])[None, :, None], t(g["x"])[None, :, None],
            t(g["real_a"] * g["dt"])[None, :, None], t(g["dt"])[None, :, None],
            t(trap_logits)[None, :, None], t(g["rates"])[None, :, None], chunk=chunk,
        )
        np.testing.assert_allclose(y[0, :, 0].numpy(), g["reads"], rtol=1e-10, atol=1e-12)
    lf, _ = S.local_frame_forward(
        g["q"][None, :, None, None], g["b"][None, :, None, None], g["x"][None, :, None, None],
        (g["real_a"] * g["dt"])[None, :, None], g["dt"][None, :, None],
        trap_logits[None, :, None], g["rates"][None, :, None],
    )
    np.testing.assert_allclose(lf[0, :, 0, 0], g["reads"], rtol=1e-10, atol=1e-12)
    assert time == g["reads"].shape[0]


@pytest.mark.parametrize("length, chunk", [(45, 16), (32, 8), (7, 16), (40, 128)])
def test_scan_oracle_chunked_equals_local_frame(length, chunk):
    # Input recipe of lm/tests/test_flashmamba.py:14-37.
    rng = np.random.default_rng(length)
    batch, heads, state, width = 2, 3, 8, 6
    q = rng.normal(size=(batch, length, heads, 1, state))
    k = rng.normal(size=q.shape)
    v = rng.normal(size=(batch, length, heads, 1, width))
    dt = np.log1p(np.exp(rng.normal(size=(batch, length, heads)) - 1))
    adt = -dt * rng.uniform(0.5, 2.0, dt.shape)
    trap = rng.normal(size=dt.shape)
    angles = rng.normal(size=(batch, length, heads, state // 4))
    qb = rng.normal(size=(heads, 1, state)) * 0.1
    kb = rng.normal(size=(heads, 1, state)) * 0.1
    ref, _ = S.local_frame_forward(q, k, v, adt, dt, trap, angles, qb, kb)
    t = lambda a: torch.tensor(a)  # noqa: E731
    y, _ = S.chunked_scan(t(q[..., 0, :]), t(k[..., 0, :]), t(v[..., 0, :]), t(adt), t(dt),
                          t(trap), t(angles), t(qb[:, 0]), t(kb[:, 0]), chunk=chunk)
    np.testing.assert_allclose(y.numpy(), ref[..., 0, :], rtol=1e-10, atol=1e-10)


@pytest.mark.parametrize("chunk", [1, 4, 16])
def test_scan_euler_limit_is_hebbian(chunk):
    # analysis/tests/test_memory.py:105-109: with the trapezoid entirely on the
    # current token (sigmoid(trap_logit) = 1), unit steps, no decay and no
    # rotation, the scan read is the Hebbian read y_t = sum_{s<=t} (q_t.k_s) v_s.
    rng = np.random.default_rng(24)
    batch, time, heads, state, width = 2, 9, 3, 8, 5
    q, k = rng.normal(size=(batch, time, heads, state)), rng.normal(size=(batch, time, heads, state))
    v = rng.normal(size=(batch, time, heads, width))
    ones = np.ones((batch, time, heads))
    t = lambda a: torch.tensor(a, dtype=torch.float64)  # noqa: E731
    y, _ = S.chunked_scan(t(q), t(k), t(v), t(0 * ones), t(ones), t(50 * ones),
                          t(np.zeros((batch, time, heads, 2))), chunk=chunk)
    scores = np.einsum("bthn,bshn->bhts", q, k) * np.tril(np.ones((time, time)))
    np.testing.assert_allclose(y.numpy(), np.einsum("bhts,bshp->bthp", scores, v), rtol=1e-10, atol=1e-10)


def test_scan_no_future_leakage():
    # lm/tests/test_mamba3_transformer.py:72-77: outputs before t ignore inputs after t.
    cfg = S.config_inputs(1, 40, 2, 8, 8, seed=5)
    args = [torch.tensor(cfg[n], dtype=torch.float64) for n in
            ("c", "b", "x", "adt", "dt", "trap_logits", "angles", "q_bias", "k_bias")]
    y, _ = S.fused_layout_scan(*args, chunk=16)
    changed = [a.clone() for a in args]
    for i in range(7):
        if changed[i].ndim >= 2 and changed[i].shape[1] == 40:
            changed[i][:, 25:] = changed[i][:, 25:] * 0.5 + 0.3
    y2, _ = S.fused_layout_scan(*changed, chunk=16)
    # scale_t = gamma_t + dt_(t+1)(1-trap_(t+1)): y_t depends on token t+1's dt/trap
    # only through the *source* weight of s=t, which affects outputs > t.
    np.testing.assert_allclose(y[:, :25].numpy(), y2[:, :25].numpy(), rtol=0, atol=0)


def test_decode_oracles_step_through_the_sequence_oracles():
    """One-token oracles (`selective_decode`, lm/kernels/mamba4.py:341-355;
    the scan core of `_Mamba3StepMixer`, lm/models/mamba4.py:412-481)
    stepped from a zero state reproduce the sequence oracles."""
    import torch

    from oracle import scan as S

    cfg = M.config_inputs(2, 20, 3, 8, 5, seed=3)
    names = ("keys", "values", "queries", "beta", "log_decay", "floor")
    fwd = M.dense_forward(*[cfg[n] for n in names])
    batch, time, heads, dim = cfg["keys"].shape
    ev = np.zeros((batch, heads, dim, dim))
    cr = np.zeros((batch, heads, cfg["values"].shape[-1], dim))
    for t in range(time):
        out, var, ev, cr = M.decode_step(ev, cr, cfg["keys"][:, t], cfg["values"][:, t],
                                         cfg["queries"][:, t], cfg["beta"][:, t],
                                         cfg["log_decay"][:, t], cfg["floor"])
        np.testing.assert_allclose(out, fwd["output"][:, t], rtol=1e-12, atol=1e-14)
        np.testing.assert_allclose(var, fwd["variance"][:, t], rtol=1e-12, atol=1e-14)
    np.testing.assert_allclose(ev, fwd["evidence"], rtol=1e-12, atol=1e-14)

    sc = S.config_inputs(2, 70, 3, 8, 8, seed=1)
    keys = ("c", "b", "x", "adt", "dt", "trap_logits", "angles", "q_bias", "k_bias")
    ey, ef = S.fused_layout_scan(*[torch.tensor(sc[n], dtype=torch.float64) for n in keys])
    batch, time = sc["c"].shape[:2]
    heads = sc["dt"].shape[-1]
    n_state, head_dim = sc["c"].shape[-1], sc["x"].shape[-1] // heads
    cache = (np.zeros((batch, heads, n_state, head_dim)), np.zeros((batch, heads, n_state)),
             np.zeros((batch, heads, head_dim)), np.zeros((batch, heads, sc["angles"].shape[-1])))
    ys = []
    for t in range(time):
        y, cache = S.step_decode(cache, *[sc[n][:, t] for n in keys[:7]], sc["q_bias"], sc["k_bias"])
        ys.append(y)
    scale = float(ey.abs().max())
    assert float((torch.stack(ys, 1) - ey).abs().max()) < 1e-12 * scale
    assert float((cache[0] - ef).abs().max()) < 1e-12 * float(ef.abs().max())


def test_spd_solve_vjp_is_the_derivative_along_symmetric_directions():
    # lm/kernels/mamba4.py:208-215: d rhs = z and dA = -sym(z y^T) give the
    # directional derivative of <g, y> along any symmetric perturbation of A
    # (the only directions the lower-triangle read sees) and along rhs.
    rng = np.random.default_rng(3)
    m = rng.normal(size=(4, 6, 6))
    a = m @ np.swapaxes(m, -1, -2) + 0.5 * np.eye(6)
    rhs = rng.normal(size=(4, 6))
    g = rng.normal(size=(4, 6))
    da, dr = M.spd_solve_vjp(a, rhs, g)
    e = rng.normal(size=(4, 6, 6))
    e = e + np.swapaxes(e, -1, -2)
    f = rng.normal(size=(4, 6))
    h = 1e-6
    fd = (np.sum(g * M.spd_solve(a + h * e, rhs + h * f)) - np.sum(g * M.spd_solve(a - h * e, rhs - h * f))) / (2 * h)
    np.testing.assert_allclose(np.sum(da * e) + np.sum(dr * f), fd, rtol=1e-6)
    # Only the lower triangle is read.
    upper = np.triu(rng.normal(size=(4, 6, 6)), 1)
    np.testing.assert_allclose(M.spd_solve(a + upper, rhs), M.spd_solve(a, rhs), rtol=1e-12)


def test_cpu_timing_path_equals_the_oracle():
    # oracle/cpu_path.py (the timed CPU baseline: the reference's XLA path
    # restated in PyTorch) computes the same operators as the float64 oracle.
    import torch

    from oracle import cpu_path as C
    from oracle import scan as S

    cfg = M.config_inputs(2, 100, 3, 64, 64, seed=4)
    names = ("keys", "values", "queries", "beta", "log_decay", "floor")
    t = {n: torch.tensor(cfg[n], dtype=torch.float64) for n in cfg}
    loss, grads = C.memory_step(t)
    fwd = M.chunked_forward(*[cfg[n] for n in names])
    ref_loss = np.sum(fwd["output"] * cfg["d_output"]) + np.sum(fwd["variance"] * cfg["d_variance"])
    np.testing.assert_allclose(float(loss), ref_loss, rtol=1e-9)
    bwd = M.chunked_backward(*[cfg[n] for n in names], None, cfg["d_output"], cfg["d_variance"])
    for g, n in zip(grads, names):
        np.testing.assert_allclose(g.numpy(), bwd[n], rtol=1e-7, atol=1e-9 * np.abs(bwd[n]).max())
    sc = S.config_inputs(2, 130, 3, 64, 64, seed=5)
    keys = ("c", "b", "x", "adt", "dt", "trap_logits", "angles", "q_bias", "k_bias")
    st = {n: torch.tensor(sc[n], dtype=torch.float64) for n in sc}
    y, final = C.mamba3_scan(*[st[n] for n in keys])
    ey, ef = S.fused_layout_scan(*[st[n] for n in keys])
    np.testing.assert_allclose(y.numpy(), ey.numpy(), rtol=1e-9, atol=1e-12)
    np.testing.assert_allclose(final.numpy(), ef.numpy(), rtol=1e-9, atol=1e-12)
    _, sg = C.scan_step(st)
    eg = S.fused_layout_grads([sc[n] for n in keys], sc["d_y"], sc["d_final"])
    for g, e, n in zip(sg, eg, keys):
        np.testing.assert_allclose(g.numpy(), e.numpy(), rtol=1e-7, atol=1e-9 * float(e.abs().max()), err_msg=n)
