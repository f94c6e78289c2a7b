"""Mamba-3 SISO chunked scan on B200: the reference's FlashMamba surface.

Mirrors `lm/kernels/flashmamba.py`: `mamba3_fused` (projection layout,
:1114-1162), `mamba3_flash_heads` / `mamba3_flash` (per-head layout,
:467-540) and `angle_rates` (:1105-1111), with the same argument meaning,
shapes and ValueError messages. The scan runs in the CUDA library through the
C ABI (`m4_scan_fwd/bwd`); the trapezoid gates, the angle duplication and
their derivatives are folded into those kernels. No CPU path exists.
"""

from __future__ import annotations

import ctypes
from typing import NamedTuple

import torch
import torch.nn.functional as F

from . import _lib
from .remat import operator_results

STATE_DIMS = (64, 96, 128)   # state dims the kernels implement (smaller ones are padded)
STATE_DIM = STATE_DIMS[-1]
HEAD_DIM = 64
CHUNK = 64


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def kernel_state_dim(state_dim: int) -> int:
    """Smallest state dim the kernels implement that holds `state_dim`
    (zero-padded coordinates never interact)."""
    for n in STATE_DIMS:
        if state_dim <= n:
            return n
    raise ValueError(f"Scan supports state dims up to {STATE_DIM}")


def sequence_state_dim(state_dim: int, bf16: bool) -> int:
    """State dim a whole-sequence scan runs at: bfloat16 scans above 64 run
    the tensor-core kernels at 128 (96 is zero-padded: the padded state rows
    stay zero and every product with them is zero, so outputs and gradients
    are those of the unpadded scan); float32 runs 64, 96 or 128 natively."""
    n = kernel_state_dim(state_dim)
    return 128 if bf16 and n > 64 else n


def scan_forward(c, b, x, adt, dt, trap, angles, q_bias, k_bias, per_head):
    """m4_scan_fwd on padded, contiguous operands: returns y, final, residual
    (inside a block rematerialized under the "kernels" policy, the recompute
    returns the forward's results instead of relaunching: the reference's
    "ssd_scan" checkpoint name)."""
    return operator_results(lambda: _scan_forward(c, b, x, adt, dt, trap, angles, q_bias, k_bias, per_head))


def _scan_forward(c, b, x, adt, dt, trap, angles, q_bias, k_bias, per_head):
    lib = _lib.load()
    batch, time = c.shape[:2]
    heads = dt.shape[-1]
    bf16 = x.dtype == torch.bfloat16
    n = c.shape[-1]
    dims = _lib.ScanDims(batch, time, heads, HEAD_DIM, n, angles.shape[-1], CHUNK,
                         int(bf16), int(per_head))
    y = torch.empty_like(x)
    final = torch.empty(batch, heads, n, HEAD_DIM, device=x.device)
    nbytes = lib.m4_scan_residual_bytes(ctypes.byref(dims))
    resid = torch.empty(nbytes, dtype=torch.uint8, device=x.device)
    _lib.check(
        lib.m4_scan_fwd(ctypes.byref(dims), *map(_lib.ptr, (c, b, x, adt, dt, trap, angles, q_bias,
                                                             k_bias, y, final, resid)),
                        nbytes, _stream()),
        "m4_scan_fwd")
    return y, final, resid


def scan_backward(c, b, x, adt, dt, trap, angles, q_bias, k_bias, resid, d_y, d_final, per_head):
    """m4_scan_bwd: returns dc, db, dx, d_adt, d_dt, d_trap, d_angles, d_q_bias, d_k_bias."""
    lib = _lib.load()
    batch, time = c.shape[:2]
    heads = dt.shape[-1]
    bf16 = x.dtype == torch.bfloat16
    dims = _lib.ScanDims(batch, time, heads, HEAD_DIM, c.shape[-1], angles.shape[-1], CHUNK, int(bf16),
                         int(per_head))
    d_y = torch.zeros_like(x) if d_y is None else d_y.to(x.dtype).contiguous()
    d_final = None if d_final is None else d_final.float().contiguous()
    dc, db, dx = torch.empty_like(c), torch.empty_like(b), torch.empty_like(x)
    dadt, ddt, dtrap = torch.empty_like(adt), torch.empty_like(dt), torch.empty_like(trap)
    dang = torch.empty_like(angles)
    dqb = torch.empty_like(q_bias) if q_bias is not None else None
    dkb = torch.empty_like(k_bias) if k_bias is not None else None
    wbytes = lib.m4_scan_workspace_bytes(ctypes.byref(dims))
    work = torch.empty(wbytes, dtype=torch.uint8, device=x.device)
    _lib.check(
        lib.m4_scan_bwd(ctypes.byref(dims), *map(_lib.ptr, (c, b, x, adt, dt, trap, angles, q_bias,
                                                             k_bias, resid)),
                        resid.numel(),
                        *map(_lib.ptr, (d_y, d_final, dc, db, dx, dadt, ddt, dtrap, dang, dqb, dkb,
                                        work)),
                        wbytes, _stream()),
        "m4_scan_bwd")
    return dc, db, dx, dadt, ddt, dtrap, dang, dqb, dkb


class _Scan(torch.autograd.Function):
    """Forward/backward over padded operands (N in {64, 96, 128}, P = 64, chunk 64)."""

    @staticmethod
    def forward(ctx, c, b, x, adt, dt, trap, angles, q_bias, k_bias, per_head):
        y, final, resid = scan_forward(c, b, x, adt, dt, trap, angles, q_bias, k_bias, per_head)
        ctx.save_for_backward(c, b, x, adt, dt, trap, angles, q_bias, k_bias, resid)
        ctx.per_head = per_head
        ctx.set_materialize_grads(False)  # an unused final state passes no zero tensor
        return y, final

    @staticmethod
    def backward(ctx, d_y, d_final):
        return (*scan_backward(*ctx.saved_tensors, d_y, d_final, ctx.per_head), None)


def _pad(t, pads):
    """F.pad only when something is padded (a zero pad still copies)."""
    return F.pad(t, pads) if any(pads) else t


def _prepare(c, b, x, adt, dt, trap_logits, angles, q_bias, k_bias, heads, per_head):
    """Pad N to the next kernel state dim (64, 96 or 128) and P to 64 (zero
    coordinates do not interact) and fix dtypes."""
    state_dim = c.shape[-1]
    value_dim = x.shape[-1] // heads
    if state_dim % 2 or angles.shape[-1] > state_dim // 2:
        # Message of lm/kernels/mamba3.py:23-24.
        raise ValueError("Mamba-3 state dimension must be even and contain angles")
    if state_dim > STATE_DIM or value_dim > HEAD_DIM:
        raise ValueError(f"Scan supports state dims up to {STATE_DIM} and head dims up to {HEAD_DIM}")
    model = x.dtype if x.dtype in (torch.bfloat16, torch.float32) else torch.float32
    pn = (0, sequence_state_dim(state_dim, model == torch.bfloat16) - state_dim)
    c = _pad(c.to(model), pn).contiguous()
    b = _pad(b.to(model), pn).contiguous()
    lead = x.shape[:-1]
    if value_dim != HEAD_DIM:
        x = F.pad(x.to(model).reshape(*lead, heads, value_dim), (0, HEAD_DIM - value_dim))
    x = x.to(model).reshape(*lead, heads * HEAD_DIM).contiguous()
    f32 = lambda a: a.float().contiguous()  # noqa: E731
    qb = None if q_bias is None else _pad(f32(q_bias).reshape(heads, state_dim), pn).contiguous()
    kb = None if k_bias is None else _pad(f32(k_bias).reshape(heads, state_dim), pn).contiguous()
    return c, b, x, f32(adt), f32(dt), f32(trap_logits), f32(angles), qb, kb, value_dim, state_dim


def mamba3_fused(
    c, b, x, adt, dt, trap_logits, angles, *, q_bias, k_bias, chunk_size=CHUNK,
    interpret=None, heads_per_step=None,
):
    """SISO Mamba-3 with one shared query and key per token (one group).

    c, b [B,T,N]; x [B,T,H*P] (bfloat16 or float32); adt, dt, trap_logits
    [B,T,H]; angles [B,T,A] shared rates; q_bias, k_bias [H,1,N]. Returns
    y [B,T,H*P] and the final state [B,H,N,P] (`flashmamba.py:1129-1135`).
    `chunk_size`, `interpret` and `heads_per_step` are accepted for signature
    compatibility (TPU tiling knobs); the kernels tile by 64.
    """
    del chunk_size, interpret, heads_per_step
    if not x.is_cuda:
        raise RuntimeError("mamba3_fused runs on CUDA tensors only (no CPU path)")
    heads = dt.shape[-1]
    c, b, x, adt, dt, trap, ang, qb, kb, value_dim, state_dim = _prepare(
        c, b, x, adt, dt, trap_logits, angles, q_bias, k_bias, heads, False)
    y, final = _Scan.apply(c, b, x, adt, dt, trap, ang, qb, kb, False)
    if value_dim != HEAD_DIM:
        lead = y.shape[:-1]
        y = y.reshape(*lead, heads, HEAD_DIM)[..., :value_dim].reshape(*lead, heads * value_dim)
    if state_dim != final.shape[2] or value_dim != HEAD_DIM:
        final = final[:, :, :state_dim, :value_dim]
    return y, final


def mamba3_flash_heads(
    q, k, v, adt, dt, trap_logits, angles, *, q_bias=None, k_bias=None, chunk_size=CHUNK,
    interpret=None, heads_per_step=None,
):
    """Per-head layout (`flashmamba.py:467-502`): q, k [B,T,H,N], v [B,T,H,P],
    angles [B,T,H,A], biases [H,N]. Returns [B,T,H,P] and [B,H,N,P]."""
    del chunk_size, interpret, heads_per_step
    if not v.is_cuda:
        raise RuntimeError("mamba3_flash_heads runs on CUDA tensors only (no CPU path)")
    batch, time, heads, value_dim = v.shape
    x = v.reshape(batch, time, heads * value_dim)
    c, b, x, adt, dt, trap, ang, qb, kb, value_dim, state_dim = _prepare(
        q, k, x, adt, dt, trap_logits, angles, q_bias, k_bias, heads, True)
    y, final = _Scan.apply(c, b, x, adt, dt, trap, ang, qb, kb, True)
    y = y.reshape(batch, time, heads, HEAD_DIM)[..., :value_dim]
    return y, final[:, :, :state_dim, :value_dim]


def mamba3_flash(
    q, k, v, adt, dt, trap_logits, angles, *, chunk_size=CHUNK, q_bias=None, k_bias=None,
    pairwise=True, interpret=None, heads_per_step=None,
):
    """Drop-in for `mamba3_chunked` with rank-one heads (`flashmamba.py:505-540`)."""
    if q.shape[3] != 1:
        raise ValueError("mamba3_flash supports SISO (rank-one) heads only")
    if not pairwise:
        raise ValueError("mamba3_flash implements pairwise rotation")
    output, final = mamba3_flash_heads(
        q[..., 0, :], k[..., 0, :], v[..., 0, :], adt, dt, trap_logits, angles,
        q_bias=None if q_bias is None else q_bias[:, 0],
        k_bias=None if k_bias is None else k_bias[:, 0],
        chunk_size=chunk_size, interpret=interpret, heads_per_step=heads_per_step,
    )
    return output[..., None, :], final


def angle_rates(angles, state_dim):
    """[B,T,A] rates on both coordinates of their pair, zero on fixed ones
    (`flashmamba.py:1105-1111`). The kernels duplicate internally; this is the
    explicit form for callers that need it."""
    rates = torch.repeat_interleave(angles.float(), 2, dim=-1)
    return F.pad(rates, (0, state_dim - rates.shape[-1]))


class Mamba3StepCache(NamedTuple):
    """Constant-size decode cache of one Mamba-3 layer (the scan part of the
    reference's layer cache, `lm/models/mamba4.py:477-481`)."""

    state: torch.Tensor            # [B,H,N,P] float32
    previous_keys: torch.Tensor    # [B,H,N] rotated key of the last token
    previous_values: torch.Tensor  # [B,H,P] value of the last token
    phase: torch.Tensor            # [B,H,A] accumulated rotation phase


def mamba3_step_cache(batch, heads, state_dim, head_dim, angle_count, device=None):
    """Zero cache (`lm/models/mamba4.py:527-560`, scan fields)."""
    z = lambda *shape: torch.zeros(*shape, dtype=torch.float32, device=device)  # noqa: E731
    return Mamba3StepCache(z(batch, heads, state_dim, head_dim), z(batch, heads, state_dim),
                           z(batch, heads, head_dim), z(batch, heads, angle_count))


def mamba3_step(cache, c, b, x, adt, dt, trap_logits, angles, *, q_bias, k_bias, inplace=False):
    """One cached token of the SISO scan: the scan core of `_Mamba3StepMixer`
    (`lm/models/mamba4.py:412-481`) through `m4_scan_step`.

    cache: Mamba3StepCache; c, b [B,N] (shared by the heads, as mamba3_fused)
    or [B,H,N]; x [B,H*P] (bfloat16 or float32); adt, dt, trap_logits [B,H];
    angles [B,A] (or [B,H,A]) rates; q_bias, k_bias [H,1,N] or [H,N].
    Returns y [B,H*P] (dtype of x; before the D skip and gate) and the new
    cache. Stepping mamba3_step_cache(...) through a sequence gives
    mamba3_fused's y and final state (`test_decode_gpu.py`). With
    inplace=True the new cache is written over `cache`'s tensors (float32,
    contiguous, unpadded dims) instead of fresh ones.
    """
    if not x.is_cuda:
        raise RuntimeError("mamba3_step runs on CUDA tensors only (no CPU path)")
    heads = dt.shape[-1]
    per_head = c.dim() == 3
    batch = x.shape[0]
    state_dim = c.shape[-1]
    value_dim = x.shape[-1] // heads
    angle_count = angles.shape[-1]
    if state_dim % 2 or angle_count > state_dim // 2:
        raise ValueError("Mamba-3 state dimension must be even and contain angles")
    if state_dim > STATE_DIM or value_dim > HEAD_DIM:
        raise ValueError(f"Scan supports state dims up to {STATE_DIM} and head dims up to {HEAD_DIM}")
    model = x.dtype if x.dtype in (torch.bfloat16, torch.float32) else torch.float32
    kn = kernel_state_dim(state_dim)
    pad_n, pad_p = kn - state_dim, HEAD_DIM - value_dim
    c = _pad(c.to(model), (0, pad_n)).contiguous()
    b = _pad(b.to(model), (0, pad_n)).contiguous()
    xp = _pad(x.to(model).reshape(batch, heads, value_dim), (0, pad_p))
    xp = xp.reshape(batch, heads * HEAD_DIM).contiguous()
    f32 = lambda a: a.float().contiguous()  # noqa: E731
    qb = None if q_bias is None else _pad(f32(q_bias).reshape(heads, state_dim), (0, pad_n)).contiguous()
    kb = None if k_bias is None else _pad(f32(k_bias).reshape(heads, state_dim), (0, pad_n)).contiguous()
    st = _pad(f32(cache.state), (0, pad_p, 0, pad_n)).contiguous()
    pk = _pad(f32(cache.previous_keys), (0, pad_n)).contiguous()
    pv = _pad(f32(cache.previous_values), (0, pad_p)).contiguous()
    ph = f32(cache.phase)
    y = torch.empty_like(xp)
    if inplace:  # the kernel reads every cache value before it writes any
        st_out, pk_out, pv_out, ph_out = st, pk, pv, ph
    else:
        st_out, pk_out, pv_out, ph_out = (torch.empty_like(t) for t in (st, pk, pv, ph))
    dims = _lib.ScanDims(batch, 1, heads, HEAD_DIM, kn, angle_count, CHUNK,
                         int(model == torch.bfloat16), int(per_head))
    lib = _lib.load()
    _lib.check(
        lib.m4_scan_step(ctypes.byref(dims), *map(_lib.ptr, (st, pk, pv, ph, c, b, xp, f32(adt), f32(dt),
                                                              f32(trap_logits), f32(angles), qb, kb, y,
                                                              st_out, pk_out, pv_out, ph_out)),
                         _stream()),
        "m4_scan_step")
    y = y.reshape(batch, heads, HEAD_DIM)[..., :value_dim].reshape(batch, heads * value_dim)
    new = Mamba3StepCache(st_out[:, :, :state_dim, :value_dim], pk_out[..., :state_dim],
                          pv_out[..., :value_dim], ph_out)
    return y, new
