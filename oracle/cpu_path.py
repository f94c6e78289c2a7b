"""float32 PyTorch-CPU restatement of the reference's own CPU path, for timing.

TEST INFRASTRUCTURE ONLY (see `oracle/__init__.py`): used by `bench.py`'s
`cpu_baseline` and `--impl reference` legs as the timed CPU baseline, never
by the product package.

The reference's CPU path is its JAX/XLA code under `JAX_PLATFORMS=cpu`
(jax is not installed on these machines), run the way its kernel benchmark
runs it: value and gradient of a projected loss. This module restates that
path in float32 PyTorch on the host's cores, with the same algorithms and
the same precision as the reference:

* memory read: the XLA path of `selective_gaussian_memory`
  (`lm/kernels/mamba4.py:263-338`): chunked masked-decay evidence einsums,
  the chunk-boundary carry, materialised per-token precisions, `spd_solve`
  by Cholesky with the reference's custom VJP (`:187-218`: z = A^-1 g,
  d rhs = z, dA = -sym(z y^T)), and the within-chunk read einsums;
* scan: `mamba3_chunked` (`lm/kernels/mamba3.py:162-255`) on the
  projection layout of `mamba3_fused` (`lm/kernels/flashmamba.py:1114-1147`,
  shared C/B broadcast over heads, trapezoid weights from the trap logits),
  with the rotary frame of `_rotary_frame` (`lm/kernels/mamba3.py:43-55`).

Gradients come from torch autograd, as the reference's from jax autodiff.
"""

from __future__ import annotations

import torch

F32 = torch.float32


class _SpdSolve(torch.autograd.Function):
    """`spd_solve` with the reference's custom VJP (`lm/kernels/mamba4.py:187-218`)."""

    @staticmethod
    def forward(ctx, precision, rhs):
        lower = torch.linalg.cholesky(precision)  # reads the lower triangle
        y = torch.cholesky_solve(rhs[..., None], lower)[..., 0]
        ctx.save_for_backward(lower, y)
        return y

    @staticmethod
    def backward(ctx, gradient):
        lower, y = ctx.saved_tensors
        z = torch.cholesky_solve(gradient[..., None], lower)[..., 0]
        outer = z[..., :, None] * y[..., None, :]
        return -0.5 * (outer + outer.transpose(-1, -2)), z


def memory_read(keys, values, queries, beta, log_decay, floor, chunk_size=64):
    """XLA path of `selective_gaussian_memory` (`lm/kernels/mamba4.py:263-338`),
    zero initial state. keys/queries [B,T,H,D], values [B,T,H,P], beta and
    log_decay [B,T,H], floor [H,D]; returns (output [B,T,H,P], variance [B,T,H])."""
    batch, time, heads, dim = keys.shape
    value_dim = values.shape[-1]
    padding = (-time) % chunk_size
    count = (time + padding) // chunk_size

    def chunks(x):
        x = torch.nn.functional.pad(x, [0, 0] * (x.ndim - 2) + [0, padding])
        x = x.reshape(batch, count, chunk_size, *x.shape[2:])
        return x.transpose(2, 3)  # [B,n,H,c,...]

    k, v, q = chunks(keys), chunks(values), chunks(queries)
    b, g = chunks(beta), chunks(log_decay)
    prefix = torch.cumsum(g, dim=-1)
    causal = torch.tril(torch.ones(chunk_size, chunk_size, dtype=torch.bool))
    difference = prefix[..., :, None] - prefix[..., None, :]
    weights = torch.where(causal, torch.exp(torch.where(causal, difference, 0.0)), 0.0)
    weights = weights * b[..., None, :]
    outer = (k[..., :, None] * k[..., None, :]).reshape(*k.shape[:-1], dim * dim)
    local = torch.einsum("bnhts,bnhse->bnhte", weights, outer)
    chunk_evidence = local[..., -1, :].reshape(*local.shape[:3], dim, dim)
    chunk_cross = torch.einsum("bnhs,bnhsp,bnhsd->bnhpd", weights[..., -1, :], v, k)
    chunk_decay = torch.exp(prefix[..., -1])
    # Chunk-boundary carry (the reference's associative scan, as a running sum).
    s = torch.zeros(batch, heads, dim, dim, dtype=keys.dtype)
    c = torch.zeros(batch, heads, value_dim, dim, dtype=keys.dtype)
    starts_s, starts_c = [], []
    for n in range(count):
        starts_s.append(s)
        starts_c.append(c)
        d = chunk_decay[:, n, :, None, None]
        s = chunk_evidence[:, n] + d * s
        c = chunk_cross[:, n] + d * c
    starts_s = torch.stack(starts_s, 1)
    starts_c = torch.stack(starts_c, 1)
    carried = torch.exp(prefix)
    evidence = local.reshape(*local.shape[:-1], dim, dim)
    evidence = evidence + carried[..., None, None] * starts_s[:, :, :, None]
    diagonal = floor[:, :, None] * torch.eye(dim, dtype=keys.dtype)
    precision = evidence + diagonal[None, None, :, None]
    solved = _SpdSolve.apply(precision, q)
    variance = torch.sum(q * solved, dim=-1)
    scores = torch.einsum("bnhtd,bnhsd->bnhts", solved, k)
    within = torch.einsum("bnhts,bnhsp->bnhtp", scores * weights, v)
    inherited = torch.einsum("bnhtd,bnhpd->bnhtp", solved, starts_c)
    output = within + carried[..., None] * inherited

    def unchunk(x):
        x = x.transpose(2, 3)
        return x.reshape(batch, count * chunk_size, *x.shape[3:])[:, :time]

    return unchunk(output), unchunk(variance)


def _rotate(x, phase):
    """Pairwise rotation of coordinates (2i, 2i+1) by phase[i] (zero past the
    angle count), `lm/kernels/mamba3.py:43-55`."""
    half = x.shape[-1] // 2
    pad = half - phase.shape[-1]
    if pad:
        phase = torch.nn.functional.pad(phase, (0, pad))
    pairs = x.reshape(*x.shape[:-1], half, 2)
    cos, sin = torch.cos(phase), torch.sin(phase)
    left, right = pairs[..., 0], pairs[..., 1]
    return torch.stack((left * cos - right * sin, left * sin + right * cos), -1).reshape(x.shape)


def mamba3_scan(c, b, x, adt, dt, trap_logits, angles, q_bias, k_bias, chunk_size=64):
    """`mamba3_chunked` (`lm/kernels/mamba3.py:162-255`) on the projection
    layout of `mamba3_fused`: c, b [B,T,N], x [B,T,H*P], adt/dt/trap [B,T,H],
    angles [B,T,A], biases [H,1,N]. Returns (y [B,T,H*P], final [B,H,N,P])."""
    batch, length, state_dim = c.shape
    heads = dt.shape[-1]
    v = x.reshape(batch, length, heads, -1)
    q = c[:, :, None, :] + q_bias.reshape(heads, state_dim)
    k = b[:, :, None, :] + k_bias.reshape(heads, state_dim)
    phase = torch.cumsum(angles[:, :, None, :] * dt[..., None], dim=1)  # [B,T,H,A]
    q, k = _rotate(q, phase), _rotate(k, phase)
    trap = torch.sigmoid(trap_logits)
    gamma = dt * trap
    previous = dt * (1 - trap)
    scale = gamma + torch.cat((previous[:, 1:], torch.zeros_like(previous[:, :1])), 1)
    padding = (-length) % chunk_size

    def chunks(a):
        a = torch.nn.functional.pad(a, [0, 0] * (a.ndim - 2) + [0, padding])
        return a.reshape(batch, -1, chunk_size, *a.shape[2:])

    qc, kc, vc, log_decay, current, source = (chunks(a) for a in (q, k, v, adt, gamma, scale))
    prefix = torch.cumsum(log_decay, dim=2)  # [B,n,c,H]
    decay = torch.exp(torch.clamp(prefix[:, :, :, None, :] - prefix[:, :, None, :, :], max=0.0))
    score = torch.einsum("bcthn,bcshn->bchts", qc, kc)
    score = score * decay.permute(0, 1, 4, 2, 3) * source.permute(0, 1, 3, 2)[:, :, :, None, :]
    lower = torch.tril(torch.ones(chunk_size, chunk_size, dtype=torch.bool), -1)
    score = torch.where(lower, score, 0.0)
    within = torch.einsum("bchts,bcshp->bcthp", score, vc)
    diagonal = torch.einsum("bcthn,bcthn->bcth", qc, kc)[..., None] * vc * current[..., None]
    tail = torch.exp(prefix[:, :, -1:, :] - prefix)
    update = torch.einsum("bcthn,bcthp->bchnp", kc, vc * (source * tail)[..., None])
    chunk_decay = torch.exp(prefix[:, :, -1])[..., None, None]  # [B,n,H,1,1]
    state = torch.zeros(batch, heads, state_dim, v.shape[-1], dtype=c.dtype)
    starts = []
    for n in range(qc.shape[1]):
        starts.append(state)
        state = update[:, n] + chunk_decay[:, n] * state
    starts = torch.stack(starts, 1)
    inherited = torch.einsum("bcthn,bchnp->bcthp", qc, starts) * torch.exp(prefix)[..., None]
    y = (within + diagonal + inherited).reshape(batch, -1, heads * v.shape[-1])[:, :length]
    return y, state


def memory_step(inputs):
    """One timed step: value and gradient of the projected loss through the
    memory read (the reference benchmark's `value_and_grad(projected_loss)`)."""
    names = ("keys", "values", "queries", "beta", "log_decay")
    leaves = [inputs[n].detach().clone().requires_grad_(True) for n in names]
    out, var = memory_read(*leaves, inputs["floor"])
    loss = (out * inputs["d_output"]).sum() + (var * inputs["d_variance"]).sum()
    return loss.detach(), torch.autograd.grad(loss, leaves)


def scan_step(inputs):
    """One timed step of the scan: value and gradient of the projected loss."""
    names = ("c", "b", "x", "adt", "dt", "trap_logits", "angles", "q_bias", "k_bias")
    leaves = [inputs[n].detach().clone().requires_grad_(True) for n in names]
    y, final = mamba3_scan(*leaves)
    loss = (y * inputs["d_y"]).sum() + (final * inputs["d_final"]).sum()
    return loss.detach(), torch.autograd.grad(loss, leaves)
