"""CUDA Mamba-3 scan vs the oracle (parity gate).

float32 operands: relative 1e-4 forward, 1e-3 gradients against the float64
oracle (absolute floor scaled to each tensor's max). bfloat16 operands (the
benchmark dtype): outputs and gradients against the oracle that applies the
reference kernels' own bf16 rounding points (forward `flashmamba.py:582-653`,
backward `:734-751`), within a few bf16 ulps elementwise (rtol 2e-2,
atol 2e-2 * max) and a relative Frobenius error below 5e-3. Against float64
the reference's bf16 arithmetic itself is up to ~3% off for the angle-rate
gradient (a suffix sum over the whole sequence), which is why bf16 parity is
pinned to the rounding-point restatement.
"""

import numpy as np
import pytest
import torch

from oracle import scan as S

pytestmark = pytest.mark.gpu

NAMES = ("c", "b", "x", "adt", "dt", "trap_logits", "angles", "q_bias", "k_bias")


def close(actual, expected, tol, name=""):
    a = actual.detach().double().cpu().numpy()
    e = expected.detach().double().cpu().numpy() if torch.is_tensor(expected) else expected
    if e.size == 0:
        assert a.size == 0
        return
    scale = float(np.abs(e).max()) or 1.0
    np.testing.assert_allclose(a, e, rtol=tol, atol=tol * scale, err_msg=name)


def rel_fro(actual, expected):
    a = actual.detach().double().cpu()
    e = expected.detach().double().cpu()
    return float((a - e).norm() / max(float(e.norm()), 1e-30))


def make(batch, time, heads, angle_count, seed, random_bias=True, state_dim=64):
    cfg = S.config_inputs(batch, time, heads, 64, state_dim, seed=seed)
    cfg["angles"] = cfg["angles"][..., :angle_count].copy()
    rng = np.random.default_rng(seed + 7)
    if random_bias:
        cfg["q_bias"] = (1 + 0.1 * rng.normal(size=cfg["q_bias"].shape)).astype(np.float32)
        cfg["k_bias"] = (1 + 0.1 * rng.normal(size=cfg["k_bias"].shape)).astype(np.float32)
    return cfg


def run_cuda(cfg, dtype):
    from mamba4_b200 import mamba3_fused

    dev = "cuda:0"
    leaves = []
    for n in NAMES:
        t = torch.tensor(cfg[n], device=dev)
        if n in ("c", "b", "x"):
            t = t.to(dtype)
        leaves.append(t.requires_grad_(True))
    y, final = mamba3_fused(*leaves[:7], q_bias=leaves[7], k_bias=leaves[8])
    loss = (y.float() * torch.tensor(cfg["d_y"], device=dev)).sum() + (
        final * torch.tensor(cfg["d_final"], device=dev)).sum()
    grads = torch.autograd.grad(loss, leaves)
    return y, final, grads


@pytest.mark.parametrize("time, angle_count", [(100, 32), (64, 16), (7, 32), (200, 0)])
def test_scan_fp32_matches_oracle(time, angle_count):
    cfg = make(2, time, 3, angle_count, seed=time)
    y, final, grads = run_cuda(cfg, torch.float32)
    args = [torch.tensor(cfg[n], dtype=torch.float64) for n in NAMES]
    ey, ef = S.fused_layout_scan(*args, chunk=64)
    close(y, ey, 1e-4, "y")
    close(final, ef, 1e-4, "final")
    eg = S.fused_layout_grads([cfg[n] for n in NAMES], cfg["d_y"], cfg["d_final"], chunk=64)
    for name, g, e in zip(NAMES, grads, eg):
        close(g, e, 1e-3, name)


def test_scan_bf16_config1_shape_matches_oracle():
    # BASELINE config 1 distributions (batch reduced to 2 for the oracle).
    cfg = make(2, 1024, 16, 32, seed=0, random_bias=False)
    y, final, grads = run_cuda(cfg, torch.bfloat16)
    args = [torch.tensor(cfg[n], dtype=torch.float32) for n in NAMES]
    for i in range(3):
        args[i] = args[i].to(torch.bfloat16).float()
    ey, ef = S.fused_layout_scan(*args, chunk=64, model_dtype=torch.bfloat16,
                                 compute_dtype=torch.float32)
    close(y, ey, 2e-2, "y")
    assert rel_fro(y, ey) < 5e-3
    close(final, ef, 2e-2, "final")
    assert rel_fro(final, ef) < 5e-3
    eg = S.fused_layout_grads_emulated(args, cfg["d_y"], cfg["d_final"], chunk=64,
                                       model_dtype=torch.bfloat16)
    for name, g, e in zip(NAMES, grads, eg):
        close(g, e, 2e-2, name)
        assert rel_fro(g, e) < 5e-3, (name, rel_fro(g, e))


@pytest.mark.parametrize("time, angle_count", [(100, 16), (7, 32), (200, 0), (130, 32)])
def test_scan_bf16_ragged_lengths_and_angle_counts(time, angle_count):
    # Partial last chunks (TMA and cp.async zero fill past T), 0 / 16 / 32
    # rotation pairs, random biases; same bars as the configs[1] shape.
    cfg = make(2, time, 3, angle_count, seed=time + angle_count)
    y, final, grads = run_cuda(cfg, torch.bfloat16)
    args = [torch.tensor(cfg[n], dtype=torch.float32) for n in NAMES]
    for i in range(3):
        args[i] = args[i].to(torch.bfloat16).float()
    ey, ef = S.fused_layout_scan(*args, chunk=64, model_dtype=torch.bfloat16,
                                 compute_dtype=torch.float32)
    close(y, ey, 2e-2, "y")
    assert rel_fro(y, ey) < 5e-3
    close(final, ef, 2e-2, "final")
    assert rel_fro(final, ef) < 5e-3
    eg = S.fused_layout_grads_emulated(args, cfg["d_y"], cfg["d_final"], chunk=64,
                                       model_dtype=torch.bfloat16)
    for name, g, e in zip(NAMES, grads, eg):
        if e.numel() == 0:
            continue
        close(g, e, 2e-2, name)
        assert rel_fro(g, e) < 5e-3, (name, rel_fro(g, e))


@pytest.mark.parametrize("state_dim, time, angle_count", [(96, 130, 24), (128, 100, 64), (128, 64, 32)])
def test_scan_fp32_reference_state_dims_match_oracle(state_dim, time, angle_count):
    # The reference models' state dims: 96 (lm/configs/mamba4-60m.json:10) and
    # 128 (lm/configs/mamba4-125m.json:10); same bars as N = 64.
    cfg = make(2, time, 3, angle_count, seed=state_dim + time, state_dim=state_dim)
    y, final, grads = run_cuda(cfg, torch.float32)
    args = [torch.tensor(cfg[n], dtype=torch.float64) for n in NAMES]
    ey, ef = S.fused_layout_scan(*args, chunk=64)
    close(y, ey, 1e-4, "y")
    close(final, ef, 1e-4, "final")
    eg = S.fused_layout_grads([cfg[n] for n in NAMES], cfg["d_y"], cfg["d_final"], chunk=64)
    for name, g, e in zip(NAMES, grads, eg):
        close(g, e, 1e-3, name)


@pytest.mark.parametrize("state_dim, time, angle_count", [(96, 200, 24), (128, 130, 32), (128, 64, 64)])
def test_scan_bf16_reference_state_dims_match_oracle(state_dim, time, angle_count):
    # bf16 at N = 96 / 128 against the rounding-point oracle, same bars as N = 64.
    cfg = make(2, time, 4, angle_count, seed=state_dim + time + 1, state_dim=state_dim)
    y, final, grads = run_cuda(cfg, torch.bfloat16)
    args = [torch.tensor(cfg[n], dtype=torch.float32) for n in NAMES]
    for i in range(3):
        args[i] = args[i].to(torch.bfloat16).float()
    ey, ef = S.fused_layout_scan(*args, chunk=64, model_dtype=torch.bfloat16,
                                 compute_dtype=torch.float32)
    close(y, ey, 2e-2, "y")
    assert rel_fro(y, ey) < 5e-3
    close(final, ef, 2e-2, "final")
    assert rel_fro(final, ef) < 5e-3
    eg = S.fused_layout_grads_emulated(args, cfg["d_y"], cfg["d_final"], chunk=64,
                                       model_dtype=torch.bfloat16)
    for name, g, e in zip(NAMES, grads, eg):
        close(g, e, 2e-2, name)
        assert rel_fro(g, e) < 5e-3, (name, rel_fro(g, e))


def test_scan_bf16_per_head_layout_matches_oracle():
    # mamba3_flash_heads with bf16 q/k/v and per-head angle rates.
    from mamba4_b200 import mamba3_flash_heads

    batch, time, heads = 2, 150, 3
    cfg = S.config_inputs(batch, time, heads, 64, 64, seed=31, per_head_angles=True)
    rng = np.random.default_rng(32)
    q = (rng.standard_normal((batch, time, heads, 64)) / 8).astype(np.float32)
    k = (rng.standard_normal((batch, time, heads, 64)) / 8).astype(np.float32)
    v = cfg["x"].reshape(batch, time, heads, 64)
    qb = (1 + 0.1 * rng.normal(size=(heads, 64))).astype(np.float32)
    kb = (1 + 0.1 * rng.normal(size=(heads, 64))).astype(np.float32)
    arrays = [q, k, v, cfg["adt"], cfg["dt"], cfg["trap_logits"], cfg["angles"], qb, kb]
    dev = "cuda:0"
    leaves = []
    for i, a in enumerate(arrays):
        t = torch.tensor(a, device=dev)
        if i < 3:
            t = t.to(torch.bfloat16)
        leaves.append(t.requires_grad_(True))
    y, final = mamba3_flash_heads(*leaves[:7], q_bias=leaves[7], k_bias=leaves[8])
    dy = torch.tensor(rng.standard_normal((batch, time, heads, 64)).astype(np.float32))
    dfin = torch.tensor(rng.standard_normal((batch, heads, 64, 64)).astype(np.float32))
    loss = (y.float() * dy.to(dev)).sum() + (final * dfin.to(dev)).sum()
    grads = torch.autograd.grad(loss, leaves)
    ref = [torch.tensor(a, dtype=torch.float32) for a in arrays]
    for i in range(3):
        ref[i] = ref[i].to(torch.bfloat16).float()
    ey, ef = S.chunked_scan(*ref, chunk=64, model_dtype=torch.bfloat16, compute_dtype=torch.float32)
    close(y, ey, 2e-2, "y")
    assert rel_fro(y, ey) < 5e-3
    close(final, ef, 2e-2, "final")
    eg = S.chunked_scan_backward_emulated(*ref, dy, dfin, chunk=64, model_dtype=torch.bfloat16)
    for i, (g, e) in enumerate(zip(grads, eg)):
        close(g, e, 2e-2, str(i))
        assert rel_fro(g, e) < 5e-3, (i, rel_fro(g, e))


@pytest.mark.parametrize("length, heads_per_step", [(45, 2), (40, 4), (7, 1)])
def test_reference_fused_test_shapes_through_padding(length, heads_per_step):
    # lm/tests/test_flashmamba.py:98-168 inputs: N = 8, P = 6, 2 angle pairs.
    from mamba4_b200 import mamba3_fused

    rng = np.random.default_rng(length + 16)
    batch, heads, state, width, count = 2, 4, 8, 6, 2
    c = rng.normal(size=(batch, length, state)).astype(np.float32)
    b = rng.normal(size=c.shape).astype(np.float32)
    x = rng.normal(size=(batch, length, heads * width)).astype(np.float32)
    dt = np.log1p(np.exp(rng.normal(size=(batch, length, heads)) - 1)).astype(np.float32)
    adt = (-dt * rng.uniform(0.5, 2.0, dt.shape)).astype(np.float32)
    trap = rng.normal(size=dt.shape).astype(np.float32)
    angles = rng.normal(size=(batch, length, count)).astype(np.float32)
    qb = (rng.normal(size=(heads, 1, state)) * 0.1).astype(np.float32)
    kb = (rng.normal(size=(heads, 1, state)) * 0.1).astype(np.float32)
    arrays = (c, b, x, adt, dt, trap, angles, qb, kb)
    leaves = [torch.tensor(a, device="cuda", requires_grad=True) for a in arrays]
    y, final = mamba3_fused(*leaves[:7], q_bias=leaves[7], k_bias=leaves[8],
                            chunk_size=16, heads_per_step=heads_per_step)
    wy = rng.normal(size=x.shape)
    wf = rng.normal(size=(batch, heads, state, width))
    ey, ef = S.fused_layout_scan(*[torch.tensor(a, dtype=torch.float64) for a in arrays], chunk=16)
    close(y, ey, 2e-5, "y")
    close(final, ef, 2e-5, "final")
    loss = (y * torch.tensor(wy, device="cuda", dtype=torch.float32)).sum() + (
        final * torch.tensor(wf, device="cuda", dtype=torch.float32)).sum()
    grads = torch.autograd.grad(loss, leaves)
    eg = S.fused_layout_grads(arrays, wy, wf, chunk=16)
    for name, g, e in zip(NAMES, grads, eg):
        close(g, e, 5e-5, name)


def test_per_head_layout_matches_oracle():
    # mamba3_flash surface (lm/tests/test_flashmamba.py:14-48 shapes, N = 8, P = 6).
    from mamba4_b200 import mamba3_flash

    rng = np.random.default_rng(45)
    batch, length, heads, state, width = 2, 45, 3, 8, 6
    q = rng.normal(size=(batch, length, heads, 1, state)).astype(np.float32)
    k = rng.normal(size=q.shape).astype(np.float32)
    v = rng.normal(size=(batch, length, heads, 1, width)).astype(np.float32)
    dt = np.log1p(np.exp(rng.normal(size=(batch, length, heads)) - 1)).astype(np.float32)
    adt = (-dt * rng.uniform(0.5, 2.0, dt.shape)).astype(np.float32)
    trap = rng.normal(size=dt.shape).astype(np.float32)
    angles = rng.normal(size=(batch, length, heads, state // 4)).astype(np.float32)
    qb = (rng.normal(size=(heads, 1, state)) * 0.1).astype(np.float32)
    kb = (rng.normal(size=(heads, 1, state)) * 0.1).astype(np.float32)
    arrays = (q, k, v, adt, dt, trap, angles, qb, kb)
    leaves = [torch.tensor(a, device="cuda", requires_grad=True) for a in arrays]
    y, final = mamba3_flash(*leaves[:7], q_bias=leaves[7], k_bias=leaves[8], chunk_size=16)
    t64 = [torch.tensor(a, dtype=torch.float64) for a in arrays]
    ey, ef = S.chunked_scan(t64[0][..., 0, :], t64[1][..., 0, :], t64[2][..., 0, :], *t64[3:7],
                            t64[7][:, 0], t64[8][:, 0], chunk=16)
    close(y[..., 0, :], ey, 2e-5, "y")
    close(final, ef, 2e-5, "final")
    wy = rng.normal(size=v.shape[:3] + (width,))
    wf = rng.normal(size=(batch, heads, state, width))
    loss = (y[..., 0, :] * torch.tensor(wy, device="cuda", dtype=torch.float32)).sum() + (
        final * torch.tensor(wf, device="cuda", dtype=torch.float32)).sum()
    grads = torch.autograd.grad(loss, leaves)
    per_head = (q[..., 0, :], k[..., 0, :], v[..., 0, :], adt, dt, trap, angles, qb[:, 0], kb[:, 0])
    eg = S.chunked_grads(per_head, wy, wf, chunk=16)
    for i, (g, e) in enumerate(zip(grads, eg)):
        if i in (0, 1, 2):
            g = g[..., 0, :]
        if i in (7, 8):
            g = g[:, 0]
        close(g, e, 5e-5, str(i))


def test_scan_errors_mirror_reference():
    from mamba4_b200 import mamba3_flash

    z = torch.zeros(1, 4, 2, 2, 8, device="cuda")
    with pytest.raises(ValueError, match="rank-one"):
        mamba3_flash(z, z, z, torch.zeros(1, 4, 2, device="cuda"), torch.zeros(1, 4, 2, device="cuda"),
                     torch.zeros(1, 4, 2, device="cuda"), torch.zeros(1, 4, 2, 2, device="cuda"))
