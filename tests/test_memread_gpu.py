"""CUDA memory read vs the float64 oracle (parity gate).

Tolerances follow the north star: relative 1e-4 on float32 forward outputs
and 1e-3 on gradients, each with an absolute floor scaled to the tensor's
largest magnitude (assert_allclose(rtol=r, atol=r * max|expected|)).
"""

import numpy as np
import pytest
import torch

from oracle import memread as M

pytestmark = pytest.mark.gpu

FWD_TOL = 1e-4
GRAD_TOL = 1e-3


def close(actual, expected, tol, name=""):
    actual = actual.detach().double().cpu().numpy() if torch.is_tensor(actual) else actual
    scale = float(np.abs(expected).max()) or 1.0
    np.testing.assert_allclose(actual, expected, rtol=tol, atol=tol * scale, err_msg=name)


def inputs(batch, time, heads, dim, value_dim, seed=0, initial=False):
    cfg = M.config_inputs(batch, time, heads, dim, value_dim, seed)
    rng = np.random.default_rng(seed + 1)
    init = None
    if initial:
        s = rng.normal(size=(batch, heads, dim, dim)) * 0.3
        init = ((s @ np.swapaxes(s, -1, -2)).astype(np.float32),
                (rng.normal(size=(batch, heads, value_dim, dim)) * 0.3).astype(np.float32))
    cfg["d_evidence"] = rng.normal(size=(batch, heads, dim, dim)).astype(np.float32)
    cfg["d_cross"] = rng.normal(size=(batch, heads, value_dim, dim)).astype(np.float32)
    return cfg, init


def run_cuda(cfg, init):
    from mamba4_b200 import SelectiveState, selective_memory_fused

    dev = torch.device("cuda:0")
    names = ("keys", "values", "queries", "beta", "log_decay", "floor")
    leaves = [torch.tensor(cfg[n], device=dev, requires_grad=True) for n in names]
    initial = None
    if init is not None:
        s0 = torch.tensor(init[0], device=dev, requires_grad=True)
        c0 = torch.tensor(init[1], device=dev, requires_grad=True)
        leaves += [s0, c0]
        initial = SelectiveState(s0, c0)
    res = selective_memory_fused(*leaves[:6], initial=initial)
    loss = ((res.output * torch.tensor(cfg["d_output"], device=dev)).sum()
            + (res.variance * torch.tensor(cfg["d_variance"], device=dev)).sum()
            + (res.state.evidence * torch.tensor(cfg["d_evidence"], device=dev)).sum()
            + (res.state.cross * torch.tensor(cfg["d_cross"], device=dev)).sum())
    grads = torch.autograd.grad(loss, leaves)
    return res, grads


def check_against_oracle(cfg, init, chunk=64):
    res, grads = run_cuda(cfg, init)
    args = [cfg[n] for n in ("keys", "values", "queries", "beta", "log_decay", "floor")]
    fwd = M.chunked_forward(*args, init, chunk_size=chunk)
    close(res.output, fwd["output"], FWD_TOL, "output")
    close(res.variance, fwd["variance"], FWD_TOL, "variance")
    close(res.state.evidence, fwd["evidence"], FWD_TOL, "evidence")
    close(res.state.cross, fwd["cross"], FWD_TOL, "cross")
    bwd = M.chunked_backward(*args, init, cfg["d_output"], cfg["d_variance"], cfg["d_evidence"],
                             cfg["d_cross"], chunk_size=chunk)
    names = ["keys", "values", "queries", "beta", "log_decay", "floor"]
    if init is not None:
        names += ["evidence0", "cross0"]
    for name, g in zip(names, grads):
        close(g, bwd[name], GRAD_TOL, name)


@pytest.mark.parametrize("time, value_dim", [(100, 64), (64, 128), (1, 64), (131, 128)])
def test_memory_read_matches_oracle_ragged(time, value_dim):
    cfg, init = inputs(2, time, 3, 64, value_dim, seed=time)
    check_against_oracle(cfg, init)


def test_memory_read_with_initial_state_matches_oracle():
    cfg, init = inputs(2, 90, 2, 64, 64, seed=11, initial=True)
    check_against_oracle(cfg, init)


def test_memory_read_config0_matches_oracle():
    # batch 8, seq 256, 4 heads, D = P = 64, seed 0.
    cfg, _ = inputs(8, 256, 4, 64, 64, seed=0)
    check_against_oracle(cfg, None)


@pytest.mark.parametrize("chunk", [1, 4, 5, 13, 16])
def test_reference_small_shapes_through_padding(chunk):
    # lm/tests/test_mamba4.py:32-43 inputs (D = 4, P = 5): the host adapter
    # pads to D = 64 with an identity block; results equal the dense oracle.
    rng = np.random.default_rng(0)
    k = rng.normal(size=(2, 13, 3, 4)).astype(np.float32)
    q = rng.normal(size=k.shape).astype(np.float32)
    k /= np.linalg.norm(k, axis=-1, keepdims=True)
    q /= np.linalg.norm(q, axis=-1, keepdims=True)
    v = rng.normal(size=(2, 13, 3, 5)).astype(np.float32)
    beta = rng.uniform(0.05, 1.0, size=k.shape[:-1]).astype(np.float32)
    decay = rng.uniform(0.3, 0.999, size=k.shape[:-1]).astype(np.float32)
    floor = rng.uniform(0.25, 1.5, size=(3, 4)).astype(np.float32)
    from mamba4_b200 import selective_gaussian_memory

    t = lambda a: torch.tensor(a, device="cuda")  # noqa: E731
    res = selective_gaussian_memory(t(k), t(v), t(q), t(beta), t(np.log(decay)), t(floor),
                                    chunk_size=chunk, solver="fused")
    dense = M.dense_forward(k, v, q, beta, np.log(decay), floor)
    for a, name in ((res.output, "output"), (res.variance, "variance"),
                    (res.state.evidence, "evidence"), (res.state.cross, "cross")):
        np.testing.assert_allclose(a.double().cpu().numpy(), dense[name], rtol=3e-5, atol=3e-6)


def test_exact_recall_of_independent_keys_on_gpu():
    # Known answer, lm/tests/test_mamba4.py:137-152.
    from mamba4_b200 import selective_memory_fused

    dim, value_dim = 4, 3
    keys = torch.eye(dim, device="cuda")[None, :, None, :]
    values = torch.tensor(np.random.default_rng(1).normal(size=(1, dim, 1, value_dim)),
                          dtype=torch.float32, device="cuda")
    beta = torch.full((1, dim, 1), 2.0, device="cuda")
    res = selective_memory_fused(keys, values, keys, beta, torch.zeros_like(beta),
                                 torch.full((1, dim), 1e-3, device="cuda"), chunk_size=2)
    precision = res.state.evidence[0, 0].double().cpu().numpy() + 1e-3 * np.eye(dim)
    for i in range(dim):
        read = res.state.cross[0, 0].double().cpu().numpy() @ np.linalg.solve(precision, np.eye(dim)[i])
        np.testing.assert_allclose(read, values[0, i, 0].double().cpu().numpy() / (1 + 5e-4), rtol=1e-5)


def test_memory_read_is_deterministic():
    cfg, _ = inputs(2, 128, 2, 64, 64, seed=3)
    r1, g1 = run_cuda(cfg, None)
    r2, g2 = run_cuda(cfg, None)
    assert torch.equal(r1.output, r2.output)
    for a, b in zip(g1, g2):
        assert torch.equal(a, b)


def test_shape_errors_mirror_reference():
    from mamba4_b200 import selective_gaussian_memory

    k = torch.zeros(1, 4, 2, 8, device="cuda")
    with pytest.raises(ValueError, match="disagree"):
        selective_gaussian_memory(k, torch.zeros(1, 4, 3, 5, device="cuda"), k,
                                  torch.ones(1, 4, 2, device="cuda"), torch.zeros(1, 4, 2, device="cuda"),
                                  torch.ones(2, 8, device="cuda"))
    with pytest.raises(ValueError, match="Unknown SPD solve backend"):
        selective_gaussian_memory(k, torch.zeros(1, 4, 2, 5, device="cuda"), k,
                                  torch.ones(1, 4, 2, device="cuda"), torch.zeros(1, 4, 2, device="cuda"),
                                  torch.ones(2, 8, device="cuda"), solver="nope")


def test_ill_conditioned_evidence_stays_within_the_float32_bound():
    # The block LDL^T factors without pivoting (every diagonal block of an SPD
    # matrix's Schur complements is SPD). Keys near an 8-dimensional subspace,
    # a tiny floor, no decay and beta 1 give evidence with condition numbers
    # about 2e4 by the last token; a backward-stable float32 solve keeps the
    # forward error within a small multiple of kappa * 2^-24, and the
    # backward must stay finite.
    from mamba4_b200 import selective_memory_fused

    rng = np.random.default_rng(7)
    B, T, H, D, P = 1, 256, 2, 64, 64
    basis = np.linalg.qr(rng.normal(size=(D, 8)))[0]
    k = rng.normal(size=(B, T, H, 8)) @ basis.T + 1e-2 * rng.normal(size=(B, T, H, D))
    k /= np.linalg.norm(k, axis=-1, keepdims=True)
    q = rng.normal(size=(B, T, H, D))
    q /= np.linalg.norm(q, axis=-1, keepdims=True)
    v = rng.normal(size=(B, T, H, P))
    beta, log_decay = np.ones((B, T, H)), np.zeros((B, T, H))
    floor = np.full((H, D), 1e-3)
    k, q, v, beta, log_decay, floor = (a.astype(np.float32) for a in (k, q, v, beta, log_decay, floor))
    kappa = max(np.linalg.cond(np.einsum("td,te->de", k[0, :, h].astype(np.float64), k[0, :, h].astype(np.float64))
                               + np.diag(floor[h].astype(np.float64))) for h in range(H))
    assert kappa > 1e4
    tol = 20 * kappa * 2.0**-24
    ref = M.dense_forward(k, v, q, beta, log_decay, floor)
    dev = torch.device("cuda:0")
    leaves = [torch.tensor(a, device=dev, requires_grad=True) for a in (k, v, q, beta, log_decay, floor)]
    res = selective_memory_fused(*leaves)
    close(res.output, ref["output"], tol, "output")
    close(res.variance, ref["variance"], tol, "variance")
    grads = torch.autograd.grad((res.output.square().sum() + res.variance.sum()), leaves)
    for g in grads:
        assert torch.isfinite(g).all()
