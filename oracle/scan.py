"""CPU restatement of the Mamba-3 SISO chunked scan (oracle).

TEST INFRASTRUCTURE ONLY (see `oracle/__init__.py`): never imported by the
product package.

Three restatements of the reference recurrence:

* `local_frame_forward` - float64 NumPy, the independent local-frame
  recurrence of `lm/kernels/mamba3.py:286-340` (`numpy_reference`): it rotates
  the previous state each step instead of rotating B/C cumulatively, so it
  pins rotation signs and phase integration.
* `chunked_scan` - PyTorch-CPU restatement of the chunked scan in the rotated
  frame, `lm/kernels/mamba3.py:162-255` (`mamba3_chunked`) as reorganised by
  the FlashMamba kernels `lm/kernels/flashmamba.py:589-660`
  (`_fused_forward_kernel`) with the same model-dtype rounding points:
  bias add (`:582-583`), rotation (`:634`), masked scores (`:647`), carried
  state read (`:651`), weighted values (`:653`) and output (`:652`). In
  float64 with `model_dtype=None` it is the exact recurrence; autograd through
  it is the gradient oracle (`chunked_grads`).
* `fused_layout_*` - the projection-layout surface of `mamba3_fused`
  (`lm/kernels/flashmamba.py:1114-1162`): shared c, b [B,T,N], values
  x [B,T,H*P], shared angle rates [B,T,A], biases [H,1,N].
"""

from __future__ import annotations

import numpy as np
import torch

F64 = torch.float64


def _sigmoid(x):
    return 1.0 / (1.0 + np.exp(-x))


def local_frame_forward(
    q, k, v, adt, dt, trap_logits, angles, q_bias=None, k_bias=None
):
    """Float64 local-frame reference, `lm/kernels/mamba3.py:286-340`.

    q, k [B,T,H,R,N], v [B,T,H,R,P], adt/dt/trap_logits [B,T,H], angles
    [B,T,H,A] rates (A <= N/2, pairwise rotation), biases [H,R,N]. Returns the
    output [B,T,H,R,P] and the final state [B,H,N,P] (in the local frame,
    which equals the rotated-frame state of the chunked form rotated back by
    the total phase; only outputs are compared across frames).
    """
    q, k, v = (np.asarray(a, np.float64) for a in (q, k, v))
    if q_bias is not None:
        q = q + np.asarray(q_bias, np.float64)
    if k_bias is not None:
        k = k + np.asarray(k_bias, np.float64)
    batch, length, heads, _, state_dim = q.shape
    half = state_dim // 2
    state = np.zeros((batch, heads, state_dim, v.shape[-1]))
    previous = np.zeros_like(state)
    output = np.empty(v.shape)
    angles = np.asarray(angles, np.float64)
    dt = np.asarray(dt, np.float64)
    adt = np.asarray(adt, np.float64)
    trap_logits = np.asarray(trap_logits, np.float64)

    def rotate_state(array, increment):
        # Rotate state rows (2i, 2i+1) by `increment` (pairwise real form).
        inc = np.pad(increment, [(0, 0), (0, 0), (0, half - increment.shape[-1])])
        pairs = np.swapaxes(array, -1, -2).reshape(*array.shape[:2], -1, half, 2)
        left, right = pairs[..., 0], pairs[..., 1]
        cos, sin = np.cos(inc)[:, :, None, :], np.sin(inc)[:, :, None, :]
        left, right = left * cos - right * sin, left * sin + right * cos
        out = np.stack((left, right), -1).reshape(np.swapaxes(array, -1, -2).shape)
        return np.swapaxes(out, -1, -2)

    for t in range(length):
        delta = angles[:, t] * dt[:, t][..., None]
        alpha = np.exp(adt[:, t])[..., None, None]
        trap = _sigmoid(trap_logits[:, t])
        current = np.einsum("bhrn,bhrp->bhnp", k[:, t], v[:, t])
        state = alpha * rotate_state(state, -delta)
        state = state + (dt[:, t] * (1 - trap))[..., None, None] * alpha * rotate_state(
            previous, -delta
        )
        state = state + (dt[:, t] * trap)[..., None, None] * current
        output[:, t] = np.einsum("bhrn,bhnp->bhrp", q[:, t], state)
        previous = current
    return output, state


def _duplicate(angles, state_dim):
    """[...,A] rates onto both coordinates of each pair, zero beyond 2A.

    Restates `angle_rates` (`lm/kernels/flashmamba.py:1105-1111`).
    """
    count = angles.shape[-1]
    if 2 * count > state_dim:
        raise ValueError("Mamba-3 state dimension must be even and contain angles")
    rates = torch.repeat_interleave(angles, 2, dim=-1)
    pad = state_dim - 2 * count
    if pad:
        rates = torch.nn.functional.pad(rates, (0, pad))
    return rates


def _partner(x):
    """(-x[2i+1], x[2i]) on each pair (`lm/kernels/flashmamba.py:566-572`)."""
    pairs = x.reshape(*x.shape[:-1], -1, 2)
    return torch.stack((-pairs[..., 1], pairs[..., 0]), -1).reshape(x.shape)


def chunked_scan(
    q,
    k,
    v,
    adt,
    dt,
    trap_logits,
    angles,
    q_bias=None,
    k_bias=None,
    *,
    chunk=64,
    model_dtype=None,
    compute_dtype=F64,
):
    """Rotated-frame chunked SISO scan on per-head tensors (torch, CPU).

    q, k [B,T,H,N] (queries C and keys B per head), v [B,T,H,P], adt, dt,
    trap_logits [B,T,H], angles [B,T,H,A] rates, biases [H,N]. Returns
    y [B,T,H,P] and final [B,H,N,P]. With `model_dtype` (e.g. bfloat16) every
    rounding point of the reference kernel is applied; products of rounded
    operands accumulate in `compute_dtype`.
    """
    cd = compute_dtype

    def rd(x):
        return x if model_dtype is None else x.to(model_dtype).to(cd)

    q, k, v = (a.to(cd) for a in (q, k, v))
    batch, length, heads, state_dim = q.shape
    value_dim = v.shape[-1]
    if q_bias is not None:
        q = q + q_bias.to(cd)
    if k_bias is not None:
        k = k + k_bias.to(cd)
    q, k, v = rd(q), rd(k), rd(v)
    dt = dt.to(cd)
    rates = _duplicate(angles.to(cd), state_dim)
    theta = torch.cumsum(rates * dt[..., None], dim=1)
    cos, sin = torch.cos(theta), torch.sin(theta)
    q = rd(q * cos + _partner(q) * sin)
    k = rd(k * cos + _partner(k) * sin)
    trap = torch.sigmoid(trap_logits.to(cd))
    gamma = dt * trap
    previous = dt * (1 - trap)
    scale = gamma + torch.cat((previous[:, 1:], torch.zeros_like(previous[:, :1])), 1)
    padding = (-length) % chunk

    def pad_time(x):
        spec = [0, 0] * (x.ndim - 2) + [0, padding]
        return torch.nn.functional.pad(x, spec)

    qc, kc, vc = (pad_time(a).reshape(batch, -1, chunk, heads, a.shape[-1]) for a in (q, k, v))
    ac, gc, sc = (pad_time(a).reshape(batch, -1, chunk, heads) for a in (adt.to(cd), gamma, scale))
    count = qc.shape[1]
    lower = torch.tril(torch.ones(chunk, chunk, dtype=torch.bool), -1)
    diag = torch.eye(chunk, dtype=torch.bool)
    state = torch.zeros(batch, heads, state_dim, value_dim, dtype=cd)
    outputs = []
    for n in range(count):
        p = torch.cumsum(ac[:, n], dim=1)  # [B,c,H]
        diff = p[:, :, None, :] - p[:, None, :, :]  # [B,t,s,H]
        decay = torch.where(lower[None, :, :, None], torch.exp(torch.where(
            lower[None, :, :, None], diff, torch.zeros_like(diff))), torch.zeros_like(diff))
        weights = decay * sc[:, n][:, None, :, :] + torch.where(
            diag[None, :, :, None], gc[:, n][:, :, None, :], torch.zeros_like(diff)
        )
        scores = torch.einsum("bthn,bshn->btsh", qc[:, n], kc[:, n])
        mixed = rd(scores * weights)
        within = torch.einsum("btsh,bshp->bthp", mixed, vc[:, n])
        inherited = torch.einsum("bthn,bhnp->bthp", qc[:, n], rd(state))
        y = rd(within + torch.exp(p)[..., None] * inherited)
        outputs.append(y)
        tail = torch.exp(p[:, -1:, :] - p)
        weighted = rd(vc[:, n] * (sc[:, n] * tail)[..., None])
        update = torch.einsum("bshn,bshp->bhnp", kc[:, n], weighted)
        state = torch.exp(p[:, -1, :])[..., None, None] * state + update
    y = torch.stack(outputs, 1).reshape(batch, count * chunk, heads, value_dim)
    return y[:, :length], state


def chunked_grads(args, weights_y, weights_final, chunk=64):
    """Float64 autograd gradients of sum(y*wy) + sum(final*wf).

    `args` = (q, k, v, adt, dt, trap_logits, angles, q_bias, k_bias) per-head
    tensors; returns the 9 gradients in that order (the reference tests'
    loss, `lm/tests/test_flashmamba.py:41-48`).
    """
    leaves = [torch.as_tensor(a, dtype=F64).clone().requires_grad_(True) for a in args]
    y, final = chunked_scan(*leaves, chunk=chunk)
    loss = (y * torch.as_tensor(weights_y, dtype=F64)).sum() + (
        final * torch.as_tensor(weights_final, dtype=F64)
    ).sum()
    return [g.detach() for g in torch.autograd.grad(loss, leaves)]


def fused_to_heads(c, b, x, angles, q_bias, k_bias, heads):
    """Projection layout -> per-head tensors (`lm/kernels/flashmamba.py:1129-1134`)."""
    batch, length, state_dim = c.shape
    q = c[:, :, None, :].expand(batch, length, heads, state_dim)
    k = b[:, :, None, :].expand(batch, length, heads, state_dim)
    v = x.reshape(batch, length, heads, -1)
    per_head = angles[:, :, None, :].expand(batch, length, heads, angles.shape[-1])
    return q, k, v, per_head, q_bias.reshape(heads, state_dim), k_bias.reshape(heads, state_dim)


def fused_layout_scan(
    c, b, x, adt, dt, trap_logits, angles, q_bias, k_bias, *, chunk=64,
    model_dtype=None, compute_dtype=F64,
):
    """`mamba3_fused` surface: y [B,T,H*P], final [B,H,N,P]."""
    heads = dt.shape[-1]
    q, k, v, per_head, qb, kb = fused_to_heads(c, b, x, angles, q_bias, k_bias, heads)
    y, final = chunked_scan(
        q, k, v, adt, dt, trap_logits, per_head, qb, kb,
        chunk=chunk, model_dtype=model_dtype, compute_dtype=compute_dtype,
    )
    return y.reshape(*y.shape[:2], -1), final


def fused_layout_grads(args, weights_y, weights_final, chunk=64):
    """Float64 autograd of the fused-layout scan; args as `mamba3_fused`
    positional order (c, b, x, adt, dt, trap_logits, angles, q_bias, k_bias)."""
    leaves = [torch.as_tensor(a, dtype=F64).clone().requires_grad_(True) for a in args]
    y, final = fused_layout_scan(*leaves, chunk=chunk)
    loss = (y * torch.as_tensor(weights_y, dtype=F64)).sum() + (
        final * torch.as_tensor(weights_final, dtype=F64)
    ).sum()
    return [g.detach() for g in torch.autograd.grad(loss, leaves)]


def step_decode(cache, c, b, x, adt, dt, trap_logits, angles, q_bias, k_bias, model_dtype=None):
    """One cached token of the Mamba-3 SISO scan, float64 (rounded to
    `model_dtype` where the reference rounds).

    Restates the scan core of `_Mamba3StepMixer` (`lm/models/mamba4.py:412-481`):
    cache = (state [B,H,N,P], previous_keys [B,H,N], previous_values [B,H,P],
    phase [B,H,A]); c, b [B,N] shared by the heads (or [B,H,N]); x [B,H*P];
    adt, dt, trap_logits [B,H]; angles [B,A] (or [B,H,A]); biases [H,N] or
    [H,1,N]. Biased c/b are rounded to the model dtype (`:440-441`), rotated
    pairwise by the advanced phase and rounded again (`rotate`,
    `lm/kernels/mamba3.py:20-40`); the state update and the read run in
    float (`:447-462`). Returns (y [B,H*P], new cache).
    """
    state, prev_k, prev_v, phase = (torch.as_tensor(a, dtype=F64) for a in cache)
    batch, heads, n_state, head_dim = state.shape
    rd = (lambda t: t) if model_dtype is None else (lambda t: t.to(model_dtype).to(F64))
    c, b, x = (torch.as_tensor(a, dtype=F64) for a in (c, b, x))
    adt, dt, trap = (torch.as_tensor(a, dtype=F64) for a in (adt, dt, trap_logits))
    ang = torch.as_tensor(angles, dtype=F64)
    if c.dim() == 2:
        c, b = c[:, None, :].expand(batch, heads, n_state), b[:, None, :].expand(batch, heads, n_state)
    if ang.dim() == 2:
        ang = ang[:, None, :].expand(batch, heads, ang.shape[-1])
    qb = torch.as_tensor(q_bias, dtype=F64).reshape(heads, n_state)
    kb = torch.as_tensor(k_bias, dtype=F64).reshape(heads, n_state)
    phase = phase + ang * dt[..., None]
    pairs = n_state // 2
    theta = torch.nn.functional.pad(phase, (0, pairs - phase.shape[-1]))
    cos, sin = torch.cos(theta), torch.sin(theta)

    def rotate(u):
        left, right = u[..., 0::2], u[..., 1::2]
        out = torch.stack((left * cos - right * sin, left * sin + right * cos), dim=-1)
        return rd(out.reshape(u.shape))

    q = rotate(rd(c + qb))
    k = rotate(rd(b + kb))
    v = rd(x.reshape(batch, heads, head_dim))
    gate = 1.0 / (1.0 + torch.exp(-trap))
    alpha = torch.exp(adt)[..., None, None]
    previous = prev_k[..., :, None] * prev_v[..., None, :]
    current = k[..., :, None] * v[..., None, :]
    state = alpha * (state + (dt * (1 - gate))[..., None, None] * previous)
    state = state + (dt * gate)[..., None, None] * current
    y = rd(torch.einsum("bhn,bhnp->bhp", q, state))
    return y.reshape(batch, heads * head_dim), (state, k, v, phase)


def config_inputs(batch, time, heads, head_dim, state_dim, seed=0, per_head_angles=False):
    """Seeded inputs of BASELINE config 1 (numpy float32; c, b, x meant as bf16).

    Draw order (numpy default_rng(seed)): x [B,T,H*P], b [B,T,N], c [B,T,N]
    ~ N(0,1)/8; dt = softplus(N(-3, 0.5)) [B,T,H]; per-head A = -exp(U(log 1,
    log 16)) [H] and adt = A dt; trap_logits ~ N(0,1) [B,T,H]; angle rates
    ~ U(-pi, pi) on N/2 pairs ([B,T,N/2], or [B,T,H,N/2] per head); biases
    are ones (model init, `lm/models/mamba3.py:89-100`); cotangents
    dy ~ N(0,1) [B,T,H*P], d_final ~ N(0,1) [B,H,N,P].
    """
    rng = np.random.default_rng(seed)
    x = (rng.standard_normal((batch, time, heads * head_dim)) / 8).astype(np.float32)
    b = (rng.standard_normal((batch, time, state_dim)) / 8).astype(np.float32)
    c = (rng.standard_normal((batch, time, state_dim)) / 8).astype(np.float32)
    raw = rng.normal(-3.0, 0.5, (batch, time, heads))
    dt = np.log1p(np.exp(raw)).astype(np.float32)
    a = -np.exp(rng.uniform(np.log(1.0), np.log(16.0), heads))
    adt = (a[None, None, :] * dt).astype(np.float32)
    trap = rng.standard_normal((batch, time, heads)).astype(np.float32)
    shape = (batch, time, heads, state_dim // 2) if per_head_angles else (
        batch, time, state_dim // 2)
    angles = rng.uniform(-np.pi, np.pi, shape).astype(np.float32)
    ones = np.ones((heads, 1, state_dim), np.float32)
    dy = rng.standard_normal((batch, time, heads * head_dim)).astype(np.float32)
    d_final = rng.standard_normal((batch, heads, state_dim, head_dim)).astype(np.float32)
    return dict(
        c=c, b=b, x=x, adt=adt, dt=dt, trap_logits=trap, angles=angles,
        q_bias=ones, k_bias=ones.copy(), d_y=dy, d_final=d_final,
    )


def _chunk_weights(p, scl, gam, chunk):
    """decay [B,t,s,H] (strict lower), W = decay*scale + diag(gamma)."""
    lower = torch.tril(torch.ones(chunk, chunk, dtype=torch.bool), -1)
    diag = torch.eye(chunk, dtype=torch.bool)
    diff = p[:, :, None, :] - p[:, None, :, :]
    zero = torch.zeros_like(diff)
    decay = torch.where(lower[None, :, :, None], torch.exp(torch.where(lower[None, :, :, None], diff, zero)), zero)
    weights = decay * scl[:, None, :, :] + torch.where(diag[None, :, :, None], gam[:, :, None, :], zero)
    return decay, weights, lower, diag


def chunked_scan_backward_emulated(
    q, k, v, adt, dt, trap_logits, angles, q_bias, k_bias, d_y, d_final, *,
    chunk=64, model_dtype=torch.bfloat16,
):
    """Gradients with the reference backward kernel's own rounding points.

    Restates `_fused_backward_kernel` (`lm/kernels/flashmamba.py:663-786`) and
    its XLA epilogue (`:1081-1099`) on per-head tensors, in float32 with the
    model-dtype casts of the reference: the masked scores and their
    cotangent products (`:734-737`), dY scaled by e^p (`:740`), the chunk-
    start state (`:742`, `:744`) and the end-state cotangent (`:748`). The
    trapezoid gates and angle duplication are differentiated exactly (the
    reference leaves them to JAX autodiff, `:1142-1147`, `:1105-1111`).
    Inputs as `chunked_scan`; d_y [B,T,H,P], d_final [B,H,N,P]. Returns the
    9 input gradients (q, k, v, adt, dt, trap_logits, angles, q_bias, k_bias).
    """
    cd = torch.float32

    def rd(x):
        return x.to(model_dtype).to(cd)

    q, k, v = (a.to(cd) for a in (q, k, v))
    batch, length, heads, state_dim = q.shape
    value_dim = v.shape[-1]
    qb = torch.zeros(heads, state_dim, dtype=cd) if q_bias is None else q_bias.to(cd)
    kb = torch.zeros(heads, state_dim, dtype=cd) if k_bias is None else k_bias.to(cd)
    q0, k0 = rd(q + qb), rd(k + kb)
    dt = dt.to(cd)
    rates = _duplicate(angles.to(cd), state_dim)
    theta = torch.cumsum(rates * dt[..., None], dim=1)
    cos, sin = torch.cos(theta), torch.sin(theta)
    q_rot = q0 * cos + _partner(q0) * sin
    k_rot = k0 * cos + _partner(k0) * sin
    qr, kr = rd(q_rot), rd(k_rot)
    v = rd(v)
    dy = rd(d_y.to(cd))
    trap = torch.sigmoid(trap_logits.to(cd))
    gamma = dt * trap
    previous = dt * (1 - trap)
    scale = gamma + torch.cat((previous[:, 1:], torch.zeros_like(previous[:, :1])), 1)
    padding = (-length) % chunk

    def pad_time(x):
        return torch.nn.functional.pad(x, [0, 0] * (x.ndim - 2) + [0, padding])

    qc, kc, vc, dyc = (pad_time(a).reshape(batch, -1, chunk, heads, a.shape[-1]) for a in (qr, kr, v, dy))
    ac, gc, sc = (pad_time(a).reshape(batch, -1, chunk, heads) for a in (adt.to(cd), gamma, scale))
    count = qc.shape[1]
    # Forward pass for the chunk-start states (model-dtype rounding points).
    state = torch.zeros(batch, heads, state_dim, value_dim, dtype=cd)
    starts = []
    for n in range(count):
        starts.append(state)
        p = torch.cumsum(ac[:, n], dim=1)
        tail = torch.exp(p[:, -1:, :] - p)
        weighted = rd(vc[:, n] * (sc[:, n] * tail)[..., None])
        state = torch.exp(p[:, -1, :])[..., None, None] * state + torch.einsum(
            "bshn,bshp->bhnp", kc[:, n], weighted)
    carry = d_final.to(cd).clone()
    dq = torch.zeros_like(qc)
    dk = torch.zeros_like(kc)
    dv = torch.zeros_like(vc)
    dlog = torch.zeros_like(ac)
    dgam = torch.zeros_like(ac)
    dscl = torch.zeros_like(ac)
    for n in range(count - 1, -1, -1):
        qn, kn, vn, dyn = qc[:, n], kc[:, n], vc[:, n], dyc[:, n]
        p = torch.cumsum(ac[:, n], dim=1)
        tail = torch.exp(p[:, -1:, :] - p)
        decay, weights, lower, diag = _chunk_weights(p, sc[:, n], gc[:, n], chunk)
        source = sc[:, n] * tail
        start = starts[n]
        end_decay = torch.exp(p[:, -1, :])
        scores = torch.einsum("bthn,bshn->btsh", qn, kn)
        d_mixed = torch.einsum("bthp,bshp->btsh", dyn, vn)
        mixed = scores * weights
        dvn = torch.einsum("btsh,bthp->bshp", rd(mixed), dyn)
        d_scores = rd(d_mixed * weights)
        dqn = torch.einsum("btsh,bshn->bthn", d_scores, kn)
        dkn = torch.einsum("btsh,bthn->bshn", d_scores, qn)
        d_weights = d_mixed * scores
        carried = torch.exp(p)
        scaled_dy = rd(dyn * carried[..., None])
        start_low = rd(start)
        dqn = dqn + torch.einsum("bthp,bhnp->bthn", scaled_dy, start_low)
        inherited = torch.einsum("bthn,bhnp->bthp", qn, start_low)
        dp_col = carried * torch.sum(dyn * inherited, -1)
        d_start = torch.einsum("bthn,bthp->bhnp", qn, scaled_dy) + end_decay[..., None, None] * carry
        end_low = rd(carry)
        v_end = torch.einsum("bshp,bhnp->bshn", vn, end_low)
        dkn = dkn + source[..., None] * v_end
        dvn = dvn + source[..., None] * torch.einsum("bshn,bhnp->bshp", kn, end_low)
        d_source = torch.sum(kn * v_end, -1)
        flow = d_source * source
        off = torch.where(lower[None, :, :, None], d_weights * weights, torch.zeros_like(weights))
        dp = dp_col + off.sum(2) - flow - off.sum(1)
        dgam[:, n] = torch.diagonal(d_weights, dim1=1, dim2=2).permute(0, 2, 1)
        dscl[:, n] = d_source * tail + (d_weights * decay).sum(1)
        last = flow.sum(1) + end_decay * torch.sum(carry * start, (-1, -2))
        dp[:, -1] = dp[:, -1] + last
        dlog[:, n] = torch.flip(torch.cumsum(torch.flip(dp, [1]), 1), [1])
        dq[:, n], dk[:, n], dv[:, n] = dqn, dkn, dvn
        carry = d_start

    def unpad(x):
        return x.reshape(batch, count * chunk, *x.shape[3:])[:, :length]

    dq, dk, dv = unpad(dq), unpad(dk), rd(unpad(dv))
    dlog, dgam, dscl = unpad(dlog), unpad(dgam), unpad(dscl)
    # Rotation backward (fp32): dq_pre = R^T dq, d_theta = dq.J q_rot + dk.J k_rot.
    dq_pre = dq * cos - _partner(dq) * sin
    dk_pre = dk * cos - _partner(dk) * sin
    d_theta = dq * _partner(q_rot) + dk * _partner(k_rot)
    d_inc = torch.flip(torch.cumsum(torch.flip(d_theta, [1]), 1), [1])
    d_rates = d_inc * dt[..., None]
    count_a = angles.shape[-1]
    d_angles = d_rates[..., : 2 * count_a].reshape(*d_rates.shape[:-1], count_a, 2).sum(-1)
    d_dt_phase = torch.sum(d_inc * rates, -1)
    # Gates: gamma = dt s, prev = dt (1 - s), scale_t = gamma_t + prev_(t+1).
    g_total = dgam + dscl
    prev_bar = torch.cat((torch.zeros_like(dscl[:, :1]), dscl[:, :-1]), 1)
    d_dt = g_total * trap + prev_bar * (1 - trap) + d_dt_phase
    d_trap = (g_total - prev_bar) * dt * trap * (1 - trap)
    return [dq_pre, dk_pre, dv, dlog, d_dt, d_trap, d_angles,
            dq_pre.sum((0, 1)), dk_pre.sum((0, 1))]


def fused_layout_grads_emulated(args, d_y, d_final, *, chunk=64, model_dtype=torch.bfloat16):
    """`chunked_scan_backward_emulated` on the projection layout: shared c, b
    and angles sum their per-head gradients over heads; returns gradients in
    `mamba3_fused` argument order."""
    c, b, x, adt, dt, trap, angles, q_bias, k_bias = (torch.as_tensor(a, dtype=torch.float32) for a in args)
    heads = dt.shape[-1]
    q, k, v, per_head, qb, kb = fused_to_heads(c, b, x, angles, q_bias, k_bias, heads)
    dyh = torch.as_tensor(d_y, dtype=torch.float32).reshape(*x.shape[:2], heads, -1)
    g = chunked_scan_backward_emulated(q, k, v, adt, dt, trap, per_head, qb, kb, dyh,
                                       torch.as_tensor(d_final, dtype=torch.float32),
                                       chunk=chunk, model_dtype=model_dtype)
    return [g[0].sum(2), g[1].sum(2), g[2].reshape(x.shape), g[3], g[4], g[5], g[6].sum(2),
            g[7].reshape(q_bias.shape), g[8].reshape(k_bias.shape)]
