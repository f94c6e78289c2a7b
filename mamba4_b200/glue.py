"""Fused model glue around the hot operators (CUDA, through the C ABI).

`mamba_mixer_core` replaces the XLA elementwise code of the Mamba-3 mixer's
flash branch (`lm/models/mamba3.py:74-117`): the projection split, B/C
RMSNorm, dt softplus, heavy-tail decay, the scan, the D skip and the SiLU
gate, with one kernel before the scan, one after it, and their hand-written
backward kernels. `rms_norm_bf16` is `RMSNorm` (`lm/models/common.py:25-45`)
on bfloat16 rows. Parameter gradients are reduced in a fixed order.
"""

from __future__ import annotations

import ctypes

import torch

from . import _lib
from .flashmamba import scan_backward, scan_forward


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _mix_dims(rows, inner, heads, angles, eps, stride):
    return _lib.MixerDims(rows, inner, heads, angles, eps, stride)


class _MambaMixerCore(torch.autograd.Function):
    @staticmethod
    def forward(ctx, proj, b_scale, c_scale, dt_bias, D, q_bias, k_bias, inner, heads, angles, eps):
        lib = _lib.load()
        batch, time, width = proj.shape
        rows = batch * time
        dims = _mix_dims(rows, inner, heads, angles, eps, width)
        dev = proj.device
        c = torch.empty(batch, time, 64, dtype=torch.bfloat16, device=dev)
        b = torch.empty_like(c)
        x = torch.empty(batch, time, inner, dtype=torch.bfloat16, device=dev)
        adt = torch.empty(batch, time, heads, device=dev)
        dt, trap = torch.empty_like(adt), torch.empty_like(adt)
        ang = torch.empty(batch, time, angles, device=dev)
        _lib.check(lib.m4_mixer_prep_fwd(ctypes.byref(dims), *map(_lib.ptr, (
            proj, b_scale, c_scale, dt_bias, c, b, x, adt, dt, trap, ang)), _stream()),
            "m4_mixer_prep_fwd")
        qb = q_bias.reshape(heads, 64)
        kb = k_bias.reshape(heads, 64)
        y, _, resid = scan_forward(c, b, x, adt, dt, trap, ang, qb, kb, False)
        out = torch.empty(batch, time, inner, dtype=torch.bfloat16, device=dev)
        _lib.check(lib.m4_mixer_post_fwd(ctypes.byref(dims), *map(_lib.ptr, (proj, y, D, out)), _stream()),
                   "m4_mixer_post_fwd")
        ctx.save_for_backward(proj, b_scale, c_scale, dt_bias, D, c, b, x, adt, dt, trap, ang, qb, kb,
                              resid, y)
        ctx.cfg = (inner, heads, angles, eps)
        return out

    @staticmethod
    def backward(ctx, g_out):
        lib = _lib.load()
        (proj, b_scale, c_scale, dt_bias, D, c, b, x, adt, dt, trap, ang, qb, kb, resid,
         y) = ctx.saved_tensors
        inner, heads, angles, eps = ctx.cfg
        batch, time, width = proj.shape
        dims = _mix_dims(batch * time, inner, heads, angles, eps, width)
        g_out = g_out.to(torch.bfloat16).contiguous()
        nw = lib.m4_mixer_partial_rows(ctypes.byref(dims))
        part = torch.empty(nw * (128 + heads), device=proj.device)
        d_proj = torch.empty_like(proj)
        d_y = torch.empty_like(y)
        dD = torch.empty_like(D)
        _lib.check(lib.m4_mixer_post_bwd(ctypes.byref(dims), *map(_lib.ptr, (
            proj, y, D, g_out, d_y, d_proj, part, dD)), _stream()), "m4_mixer_post_bwd")
        dc, db, dx, dadt, ddt, dtrap, dang, dqb, dkb = scan_backward(
            c, b, x, adt, dt, trap, ang, qb, kb, resid, d_y, None, False)
        d_bs, d_cs, d_dtb = torch.empty_like(b_scale), torch.empty_like(c_scale), torch.empty_like(dt_bias)
        _lib.check(lib.m4_mixer_prep_bwd(ctypes.byref(dims), *map(_lib.ptr, (
            proj, b_scale, c_scale, dt_bias, D, g_out, dc, db, dx, dadt, ddt, dtrap, dang, d_proj, part,
            d_bs, d_cs, d_dtb)), _stream()), "m4_mixer_prep_bwd")
        return (d_proj, d_bs, d_cs, d_dtb, dD, dqb.reshape(heads, 1, 64), dkb.reshape(heads, 1, 64),
                None, None, None, None)


def mamba_mixer_core(proj, b_scale, c_scale, dt_bias, D, q_bias, k_bias, *, inner, heads, angles, eps):
    """proj [B,T,2 inner + 128 + 3 heads + angles] bf16 -> gated scan output
    [B,T,inner] bf16 (input of the mixer's out projection)."""
    if not proj.is_cuda:
        raise RuntimeError("mamba_mixer_core runs on CUDA tensors only (no CPU path)")
    if proj.dtype != torch.bfloat16:
        raise ValueError("mamba_mixer_core expects a bfloat16 projection")
    f32 = lambda t: t.float().contiguous()  # noqa: E731
    width = 2 * inner + 128 + 3 * heads + angles
    if proj.shape[-1] != width:
        raise ValueError(f"projection width {proj.shape[-1]} != 2 inner + 128 + 3 heads + angles = {width}")
    if width % 8:
        # Rows are read with 16-byte loads: pad the row stride to a multiple of 8.
        proj = torch.nn.functional.pad(proj, (0, -width % 8))
    return _MambaMixerCore.apply(proj.contiguous(), f32(b_scale), f32(c_scale), f32(dt_bias), f32(D),
                                 f32(q_bias), f32(k_bias), inner, heads, angles, eps)


class _RMSNormBF16(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, scale, eps):
        lib = _lib.load()
        features = x.shape[-1]
        rows = x.numel() // features
        y = torch.empty_like(x)
        rstd = torch.empty(rows, device=x.device)
        _lib.check(lib.m4_rmsnorm_fwd(rows, features, eps, *map(_lib.ptr, (x, scale, y, rstd)), _stream()),
                   "m4_rmsnorm_fwd")
        ctx.save_for_backward(x, scale, rstd)
        return y

    @staticmethod
    def backward(ctx, gy):
        lib = _lib.load()
        x, scale, rstd = ctx.saved_tensors
        features = x.shape[-1]
        rows = x.numel() // features
        gy = gy.to(torch.bfloat16).contiguous()
        gx = torch.empty_like(x)
        part = torch.empty(lib.m4_rmsnorm_partial_rows(rows) * features, device=x.device)
        gscale = torch.empty_like(scale)
        _lib.check(lib.m4_rmsnorm_bwd(rows, features, *map(_lib.ptr, (x, scale, rstd, gy, gx, part, gscale)),
                                      _stream()), "m4_rmsnorm_bwd")
        return gx, gscale, None


def rms_norm_bf16(x, scale, eps):
    """bf16 rows -> bf16 rows, float32 statistics; features in {256, 512, 768, 1024}."""
    if not x.is_cuda:
        raise RuntimeError("rms_norm_bf16 runs on CUDA tensors only (no CPU path)")
    return _RMSNormBF16.apply(x.to(torch.bfloat16).contiguous(), scale.float().contiguous(), eps)
