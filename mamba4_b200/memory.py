"""Selective conjugate memory read: the reference operator surface on B200.

Mirrors `lm/kernels/mamba4.py` (SelectiveState, SelectiveResult,
selective_initial_state, selective_gaussian_memory) and
`lm/kernels/mamba4_fused.py:372-454` (selective_memory_fused) with the same
argument meaning, shapes, broadcasting and ValueError messages. The compute
runs in the CUDA library through the C ABI (`m4_memread_fwd/bwd`); there is
no CPU path. Gradients come from the library's backward, wrapped as a
torch.autograd.Function (the reference's jax.custom_vjp).
"""

from __future__ import annotations

from typing import NamedTuple

import torch
import torch.nn.functional as F

from . import _lib
from .remat import operator_results

KEY_DIM = 64
VALUE_DIMS = (64, 128)


class SelectiveState(NamedTuple):
    """Evidence-only sufficient statistics (`lm/kernels/mamba4.py:18-22`)."""

    evidence: torch.Tensor
    cross: torch.Tensor


class SelectiveResult(NamedTuple):
    """Reads, variances and final state (`lm/kernels/mamba4.py:25-28`)."""

    output: torch.Tensor
    variance: torch.Tensor
    state: SelectiveState


def selective_initial_state(batch, heads, key_dim, value_dim, device=None):
    """Zero state (`lm/kernels/mamba4.py:221-225`)."""
    return SelectiveState(
        torch.zeros(batch, heads, key_dim, key_dim, dtype=torch.float32, device=device),
        torch.zeros(batch, heads, value_dim, key_dim, dtype=torch.float32, device=device),
    )


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _dims(batch, time, heads, value_dim):
    return _lib.MemDims(batch, time, heads, KEY_DIM, value_dim)


class _MemoryRead(torch.autograd.Function):
    """Forward/backward pair over padded operands (D = 64, P in {64, 128})."""

    @staticmethod
    def forward(ctx, keys, values, queries, beta, log_decay, floor, init_s, init_c):
        def launch():
            lib = _lib.load()
            batch, time, heads, _ = keys.shape
            value_dim = values.shape[-1]
            dims = _dims(batch, time, heads, value_dim)
            dev = keys.device
            out = torch.empty(batch, time, heads, value_dim, device=dev)
            var = torch.empty(batch, time, heads, device=dev)
            s_fin = torch.empty(batch, heads, KEY_DIM, KEY_DIM, device=dev)
            c_fin = torch.empty(batch, heads, value_dim, KEY_DIM, device=dev)
            nbytes = lib.m4_memread_residual_bytes(ctypes_ref(dims))
            resid = torch.empty(nbytes, dtype=torch.uint8, device=dev)
            _lib.check(
                lib.m4_memread_fwd(
                    ctypes_ref(dims), *map(_lib.ptr, (keys, values, queries, beta, log_decay, floor,
                                                       init_s, init_c, out, var, s_fin, c_fin, resid)),
                    nbytes, _stream()),
                "m4_memread_fwd")
            return out, var, s_fin, c_fin, resid

        # Inside a block rematerialized under the "kernels" policy the
        # recompute reuses these results (the reference's "memory_solve"
        # checkpoint name) instead of relaunching.
        out, var, s_fin, c_fin, resid = operator_results(launch)
        ctx.save_for_backward(keys, values, queries, beta, log_decay, floor, init_s, init_c, resid)
        ctx.set_materialize_grads(False)  # unused outputs (often the final states) pass no zero tensors
        ctx.has_initial = init_s is not None
        return out, var, s_fin, c_fin

    @staticmethod
    def backward(ctx, d_out, d_var, d_s, d_c):
        lib = _lib.load()
        keys, values, queries, beta, log_decay, floor, init_s, init_c, resid = ctx.saved_tensors
        batch, time, heads, _ = keys.shape
        value_dim = values.shape[-1]
        dims = _dims(batch, time, heads, value_dim)
        dev = keys.device
        d_out = torch.zeros_like(values) if d_out is None else d_out.float().contiguous()
        d_var = torch.zeros_like(beta) if d_var is None else d_var.float().contiguous()
        d_s = None if d_s is None else d_s.float().contiguous()
        d_c = None if d_c is None else d_c.float().contiguous()
        dk, dv, dq = torch.empty_like(keys), torch.empty_like(values), torch.empty_like(queries)
        dbeta, dlog = torch.empty_like(beta), torch.empty_like(log_decay)
        dfloor = torch.empty_like(floor)
        dis = torch.empty_like(init_s) if ctx.has_initial else None
        dic = torch.empty_like(init_c) if ctx.has_initial else None
        wbytes = lib.m4_memread_workspace_bytes(ctypes_ref(dims))
        work = torch.empty(wbytes, dtype=torch.uint8, device=dev)
        _lib.check(
            lib.m4_memread_bwd(
                ctypes_ref(dims), *map(_lib.ptr, (keys, values, queries, beta, log_decay, floor,
                                                   init_s, init_c, resid)),
                resid.numel(),
                *map(_lib.ptr, (d_out, d_var, d_s, d_c, dk, dv, dq, dbeta, dlog, dfloor, dis, dic,
                                work)),
                wbytes, _stream()),
            "m4_memread_bwd")
        return dk, dv, dq, dbeta, dlog, dfloor, dis, dic


def ctypes_ref(dims):
    import ctypes

    return ctypes.byref(dims)


def _pad_last(x, size, value=0.0):
    extra = size - x.shape[-1]
    return x if extra == 0 else F.pad(x, (0, extra), value=value)


def selective_memory_fused(
    keys, values, queries, beta, log_decay, floor, *, chunk_size=64, initial=None
):
    """Exact chunked reads of the fixed-floor selective Gaussian memory.

    Same contract as `selective_memory_fused` / `selective_gaussian_memory`
    (`lm/kernels/mamba4.py:240-248`): keys/queries [B,T,H,D], values [B,T,H,P],
    beta and log_decay [B,T,H] (log_decay <= 0), floor [H,D] positive,
    optional initial SelectiveState. Returns SelectiveResult(output [B,T,H,P],
    variance [B,T,H], final SelectiveState). `chunk_size` is accepted for
    signature compatibility; the kernels use their own tiling and results are
    chunk-independent up to float32 rounding.

    Key dims D < 64 are padded with an identity block (zero keys and queries,
    unit floor), which solves to zero and leaves the true coordinates
    unchanged, as `batched_solve` pads to 8 (`mamba4_fused.py:289-297`).
    """
    del chunk_size
    keys, values, queries = (torch.as_tensor(a).float() for a in (keys, values, queries))
    if not keys.is_cuda:
        raise RuntimeError("selective_memory_fused runs on CUDA tensors only (no CPU path)")
    batch, time, heads, dim = keys.shape
    value_dim = values.shape[-1]
    if queries.shape != keys.shape or values.shape[:3] != keys.shape[:3]:
        raise ValueError("Selective memory keys, values and queries disagree")
    if dim > KEY_DIM:
        raise ValueError(f"Selective memory key dimension {dim} exceeds {KEY_DIM}")
    if value_dim > VALUE_DIMS[-1]:
        raise ValueError(f"Selective memory value dimension {value_dim} exceeds {VALUE_DIMS[-1]}")
    shape = (batch, time, heads)
    dev = keys.device
    beta = torch.broadcast_to(torch.as_tensor(beta, dtype=torch.float32, device=dev), shape)
    log_decay = torch.broadcast_to(torch.as_tensor(log_decay, dtype=torch.float32, device=dev), shape)
    floor = torch.broadcast_to(torch.as_tensor(floor, dtype=torch.float32, device=dev), (heads, dim))
    pv = VALUE_DIMS[0] if value_dim <= VALUE_DIMS[0] else VALUE_DIMS[1]
    k = _pad_last(keys, KEY_DIM).contiguous()
    q = _pad_last(queries, KEY_DIM).contiguous()
    v = _pad_last(values, pv).contiguous()
    f = _pad_last(floor, KEY_DIM, 1.0).contiguous()
    init_s = init_c = None
    if initial is not None:
        s0 = torch.as_tensor(initial.evidence, dtype=torch.float32, device=dev)
        c0 = torch.as_tensor(initial.cross, dtype=torch.float32, device=dev)
        init_s = F.pad(s0, (0, KEY_DIM - dim, 0, KEY_DIM - dim)).contiguous()
        init_c = F.pad(c0, (0, KEY_DIM - dim, 0, pv - value_dim)).contiguous()
    out, var, s_fin, c_fin = _MemoryRead.apply(
        k, v, q, beta.contiguous(), log_decay.contiguous(), f, init_s, init_c
    )
    state = SelectiveState(s_fin[..., :dim, :dim], c_fin[..., :value_dim, :dim])
    return SelectiveResult(out[..., :value_dim], var, state)


def selective_decode(state, key, value, query, beta, log_decay, floor, solver=None, inplace=False):
    """One exact write/read against a carried state (`lm/kernels/mamba4.py:341-355`).

    state: SelectiveState(evidence [B,H,D,D], cross [B,H,P,D]); key, query
    [B,H,D]; value [B,H,P]; beta, log_decay [B,H]; floor [H,D]. Returns
    SelectiveResult(output [B,H,P], variance [B,H], SelectiveState(evidence',
    cross')) through `m4_memread_decode` (one warp per head: rank-one state
    update, 64x64 block LDL^T with the forward substitution interleaved,
    back-substitution).
    `solver` is accepted for signature compatibility ("cuda"/"fused"/None).
    Key dims below 64 are padded with an identity block as in
    `selective_memory_fused`. No gradient (the reference decodes without one).
    With inplace=True the new state is written over `state`'s tensors
    (float32, contiguous, unpadded dims) instead of fresh ones.
    """
    if solver not in (None, *SOLVERS):
        raise ValueError(f"Unknown SPD solve backend {solver}")
    key, value, query = (torch.as_tensor(a).float() for a in (key, value, query))
    if not key.is_cuda:
        raise RuntimeError("selective_decode runs on CUDA tensors only (no CPU path)")
    batch, heads, dim = key.shape
    value_dim = value.shape[-1]
    if query.shape != key.shape or value.shape[:2] != key.shape[:2]:
        raise ValueError("Selective memory keys, values and queries disagree")
    if dim > KEY_DIM:
        raise ValueError(f"Selective memory key dimension {dim} exceeds {KEY_DIM}")
    if value_dim > VALUE_DIMS[-1]:
        raise ValueError(f"Selective memory value dimension {value_dim} exceeds {VALUE_DIMS[-1]}")
    dev = key.device
    pv = VALUE_DIMS[0] if value_dim <= VALUE_DIMS[0] else VALUE_DIMS[1]
    shape = (batch, heads)
    beta = torch.broadcast_to(torch.as_tensor(beta, dtype=torch.float32, device=dev), shape).contiguous()
    log_decay = torch.broadcast_to(torch.as_tensor(log_decay, dtype=torch.float32, device=dev),
                                   shape).contiguous()
    floor = torch.broadcast_to(torch.as_tensor(floor, dtype=torch.float32, device=dev), (heads, dim))
    ev = torch.as_tensor(state.evidence, dtype=torch.float32, device=dev)
    cr = torch.as_tensor(state.cross, dtype=torch.float32, device=dev)
    if dim != KEY_DIM:
        ev = F.pad(ev, (0, KEY_DIM - dim, 0, KEY_DIM - dim))
    if dim != KEY_DIM or value_dim != pv:
        cr = F.pad(cr, (0, KEY_DIM - dim, 0, pv - value_dim))
    ev, cr = ev.contiguous(), cr.contiguous()
    k = _pad_last(key, KEY_DIM).contiguous()
    q = _pad_last(query, KEY_DIM).contiguous()
    v = _pad_last(value, pv).contiguous()
    f = _pad_last(floor, KEY_DIM, 1.0).contiguous()
    out = torch.empty(batch, heads, pv, device=dev)
    var = torch.empty(batch, heads, device=dev)
    # In place the kernel reads all of E before writing E' and each row of C
    # before writing that row.
    ev_out, cr_out = (ev, cr) if inplace else (torch.empty_like(ev), torch.empty_like(cr))
    dims = _dims(batch, 1, heads, pv)
    lib = _lib.load()
    _lib.check(
        lib.m4_memread_decode(ctypes_ref(dims), *map(_lib.ptr, (ev, cr, k, v, q, beta, log_decay, f, out,
                                                                var, ev_out, cr_out)), _stream()),
        "m4_memread_decode")
    new_state = SelectiveState(ev_out[..., :dim, :dim], cr_out[..., :value_dim, :dim])
    return SelectiveResult(out[..., :value_dim], var, new_state)


# Solver names the reference accepts (`lm/kernels/mamba4.py:167-184`,
# `:249-262`) plus "cuda". Every name selects the same mathematics (an exact
# solve of the same SPD system: Cholesky in the reference, a block LDL^T in
# this library's memory read; the reference's backends differ only in their
# arithmetic schedule), so all of them run the sm_100a kernels.
SOLVERS = ("cuda", "fused", "loop", "blocked", "unrolled", "auto")


class _SpdSolve(torch.autograd.Function):
    """precision @ y = rhs over [count, dim, dim] / [count, dim] float32."""

    @staticmethod
    def forward(ctx, precision, rhs):
        lib = _lib.load()
        count, dim = rhs.shape
        solution = torch.empty_like(rhs)
        nbytes = lib.m4_spd_solve_factor_bytes(count, dim)
        factor = torch.empty(max(nbytes, 16), dtype=torch.uint8, device=rhs.device)
        _lib.check(lib.m4_spd_solve_fwd(count, dim, _lib.ptr(precision), _lib.ptr(rhs), _lib.ptr(solution),
                                        _lib.ptr(factor), nbytes, _stream()), "m4_spd_solve_fwd")
        ctx.save_for_backward(factor, solution)
        return solution

    @staticmethod
    def backward(ctx, gradient):
        lib = _lib.load()
        factor, solution = ctx.saved_tensors
        count, dim = solution.shape
        gradient = gradient.float().contiguous()
        d_precision = torch.empty(count, dim, dim, dtype=torch.float32, device=solution.device)
        d_rhs = torch.empty_like(solution)
        nbytes = lib.m4_spd_solve_factor_bytes(count, dim)
        _lib.check(lib.m4_spd_solve_bwd(count, dim, _lib.ptr(factor), nbytes, _lib.ptr(solution),
                                        _lib.ptr(gradient), _lib.ptr(d_precision), _lib.ptr(d_rhs),
                                        _stream()), "m4_spd_solve_bwd")
        return d_precision, d_rhs


def spd_solve(precision, rhs, backend=None):
    """Solve precision @ y = rhs for SPD [...,d,d] precision and [...,d] rhs.

    Mirrors `spd_solve` (`lm/kernels/mamba4.py:187-218`): float32, only the
    lower triangle of `precision` is read, d <= 64; the backward reuses the
    stored LDL^T factor, z = A^-1 g, d rhs = z and d A = -sym(z y^T)
    (`:208-215`). `backend` takes the reference's names (None, "loop",
    "blocked", "unrolled", "auto", "fused") and "cuda"; they change only the
    reference's arithmetic schedule, and all run the `m4_spd_solve_*` kernels.
    """
    if backend not in (None, *SOLVERS):
        raise ValueError(f"Unknown SPD solve backend {backend}")
    precision = torch.as_tensor(precision).float()
    rhs = torch.as_tensor(rhs).float()
    if not rhs.is_cuda or not precision.is_cuda:
        raise RuntimeError("spd_solve runs on CUDA tensors only (no CPU path)")
    dim = rhs.shape[-1]
    if precision.shape != rhs.shape + (dim,):
        raise ValueError(f"SPD solve precision {tuple(precision.shape)} does not match rhs {tuple(rhs.shape)}")
    if dim > KEY_DIM:
        raise ValueError(f"SPD solve dimension {dim} exceeds {KEY_DIM}")
    count = rhs.numel() // dim if dim else 0
    solution = _SpdSolve.apply(precision.reshape(count, dim, dim).contiguous(),
                               rhs.reshape(count, dim).contiguous())
    return solution.reshape(rhs.shape)


def selective_gaussian_memory(
    keys, values, queries, beta, log_decay, floor, *, chunk_size=64, initial=None, solver=None
):
    """`lm/kernels/mamba4.py:228-338` dispatcher with the B200 solver.

    Every solver name the reference accepts ("fused", "loop", "blocked",
    "unrolled", "auto", or None) and "cuda" runs the sm_100a kernels: they
    solve the same system, so a reference config (the 60M model's "blocked",
    `lm/configs/mamba4-60m.json:40`) runs unchanged. Unknown names raise the
    reference's ValueError.
    """
    if solver not in (None, *SOLVERS):
        raise ValueError(f"Unknown SPD solve backend {solver}")
    return selective_memory_fused(
        keys, values, queries, beta, log_decay, floor, chunk_size=chunk_size, initial=initial
    )
