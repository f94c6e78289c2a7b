"""Standalone SPD solve and the reference's solver names (parity gate).

`spd_solve` (reference `lm/kernels/mamba4.py:187-218`) against the float64
oracle: solution at rel 1e-4, the custom-VJP cotangents (d rhs = z,
dA = -sym(z y^T)) at rel 1e-3, each with an absolute floor tol * max|expected|.
Every solver name the reference accepts runs the CUDA path and gives the
same memory read as "cuda".
"""

import numpy as np
import pytest
import torch

from oracle import memread as M

pytestmark = pytest.mark.gpu


def close(actual, expected, tol, name=""):
    actual = actual.detach().double().cpu().numpy()
    if expected.size == 0:
        assert actual.size == 0
        return
    scale = float(np.abs(expected).max()) or 1.0
    np.testing.assert_allclose(actual, expected, rtol=tol, atol=tol * scale, err_msg=name)


def spd_inputs(batch_shape, dim, seed):
    rng = np.random.default_rng(seed)
    m = rng.normal(size=(*batch_shape, dim, dim)) / np.sqrt(dim)
    a = m @ np.swapaxes(m, -1, -2) + np.diag(rng.uniform(0.1, 1.0, size=dim))
    rhs = rng.normal(size=(*batch_shape, dim))
    g = rng.normal(size=(*batch_shape, dim))
    return a.astype(np.float32), rhs.astype(np.float32), g.astype(np.float32)


@pytest.mark.parametrize("batch_shape, dim", [((3, 5), 64), ((7,), 16), ((2, 3), 4), ((5,), 1),
                                              ((4,), 37), ((0,), 8)])
def test_spd_solve_matches_oracle(batch_shape, dim):
    from mamba4_b200 import spd_solve

    a, rhs, g = spd_inputs(batch_shape, dim, seed=dim)
    ta = torch.tensor(a, device="cuda", requires_grad=True)
    tr = torch.tensor(rhs, device="cuda", requires_grad=True)
    y = spd_solve(ta, tr, "blocked")
    close(y, M.spd_solve(a, rhs), 1e-4, "solution")
    if y.numel() == 0:
        return
    da, dr = torch.autograd.grad(y, (ta, tr), torch.tensor(g, device="cuda"))
    ea, er = M.spd_solve_vjp(a, rhs, g)
    close(da, ea, 1e-3, "d precision")
    close(dr, er, 1e-3, "d rhs")


def test_spd_solve_reads_only_the_lower_triangle():
    from mamba4_b200 import spd_solve

    a, rhs, _ = spd_inputs((6,), 64, seed=4)
    junk = a.copy()
    iu = np.triu_indices(64, 1)
    junk[:, iu[0], iu[1]] = np.nan  # never read
    y = spd_solve(torch.tensor(junk, device="cuda"), torch.tensor(rhs, device="cuda"))
    assert torch.isfinite(y).all()
    close(y, M.spd_solve(a, rhs), 1e-4, "solution")


def test_spd_solve_errors_mirror_reference():
    from mamba4_b200 import spd_solve

    a = torch.eye(4, device="cuda")[None]
    with pytest.raises(ValueError, match="Unknown SPD solve backend"):
        spd_solve(a, torch.ones(1, 4, device="cuda"), "nope")
    with pytest.raises(ValueError, match="does not match"):
        spd_solve(a, torch.ones(2, 4, device="cuda"))


def test_every_reference_solver_name_runs_the_cuda_path():
    # The 60M reference config selects "blocked" (lm/configs/mamba4-60m.json:40).
    from mamba4_b200 import selective_gaussian_memory

    cfg = M.config_inputs(2, 70, 2, 64, 64, seed=2)
    t = {n: torch.tensor(v, device="cuda") for n, v in cfg.items()}
    args = [t[n] for n in ("keys", "values", "queries", "beta", "log_decay", "floor")]
    base = selective_gaussian_memory(*args, solver="cuda")
    for name in (None, "fused", "loop", "blocked", "unrolled", "auto"):
        res = selective_gaussian_memory(*args, solver=name)
        assert torch.equal(res.output, base.output), name
        assert torch.equal(res.variance, base.variance), name
    fwd = M.chunked_forward(*[cfg[n] for n in ("keys", "values", "queries", "beta", "log_decay", "floor")])
    close(base.output, fwd["output"], 1e-4, "output")
