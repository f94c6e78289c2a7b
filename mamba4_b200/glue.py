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
import torch.nn.functional as F

from . import _lib
from .flashmamba import mamba3_step, scan_backward, scan_forward, sequence_state_dim


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _mix_dims(rows, inner, heads, angles, eps, stride, state):
    return _lib.MixerDims(rows, inner, heads, angles, eps, stride, state)


class _MambaMixerCore(torch.autograd.Function):
    @staticmethod
    def forward(ctx, proj, b_scale, c_scale, dt_bias, D, q_bias, k_bias, inner, heads, angles, eps, state):
        lib = _lib.load()
        batch, time, width = proj.shape
        rows = batch * time
        dims = _mix_dims(rows, inner, heads, angles, eps, width, state)
        dev = proj.device
        c = torch.empty(batch, time, state, dtype=torch.bfloat16, device=dev)
        b = torch.empty_like(c)
        x = torch.empty(batch, time, inner, dtype=torch.bfloat16, device=dev)
        adt = torch.empty(batch, time, heads, device=dev)
        dt, trap = torch.empty_like(adt), torch.empty_like(adt)
        ang = torch.empty(batch, time, angles, device=dev)
        _lib.check(lib.m4_mixer_prep_fwd(ctypes.byref(dims), *map(_lib.ptr, (
            proj, b_scale, c_scale, dt_bias, c, b, x, adt, dt, trap, ang)), _stream()),
            "m4_mixer_prep_fwd")
        qb = q_bias.reshape(heads, state)
        kb = k_bias.reshape(heads, state)
        # The scan's state dim (96 runs the tensor-core kernels zero-padded to 128).
        pad = sequence_state_dim(state, True) - state
        if pad:
            c, b = F.pad(c, (0, pad)), F.pad(b, (0, pad))
            qb, kb = F.pad(qb, (0, pad)), F.pad(kb, (0, pad))
        y, _, resid = scan_forward(c, b, x, adt, dt, trap, ang, qb, kb, False)
        out = torch.empty(batch, time, inner, dtype=torch.bfloat16, device=dev)
        _lib.check(lib.m4_mixer_post_fwd(ctypes.byref(dims), *map(_lib.ptr, (proj, y, D, out)), _stream()),
                   "m4_mixer_post_fwd")
        ctx.save_for_backward(proj, b_scale, c_scale, dt_bias, D, c, b, x, adt, dt, trap, ang, qb, kb,
                              resid, y)
        ctx.cfg = (inner, heads, angles, eps, state)
        return out

    @staticmethod
    def backward(ctx, g_out):
        lib = _lib.load()
        (proj, b_scale, c_scale, dt_bias, D, c, b, x, adt, dt, trap, ang, qb, kb, resid,
         y) = ctx.saved_tensors
        inner, heads, angles, eps, state = ctx.cfg
        batch, time, width = proj.shape
        dims = _mix_dims(batch * time, inner, heads, angles, eps, width, state)
        g_out = g_out.to(torch.bfloat16).contiguous()
        nw = lib.m4_mixer_partial_rows(ctypes.byref(dims))
        part = torch.empty(nw * (2 * state + heads), device=proj.device)
        d_proj = torch.empty_like(proj)
        d_y = torch.empty_like(y)
        dD = torch.empty_like(D)
        _lib.check(lib.m4_mixer_post_bwd(ctypes.byref(dims), *map(_lib.ptr, (
            proj, y, D, g_out, d_y, d_proj, part, dD)), _stream()), "m4_mixer_post_bwd")
        dc, db, dx, dadt, ddt, dtrap, dang, dqb, dkb = scan_backward(
            c, b, x, adt, dt, trap, ang, qb, kb, resid, d_y, None, False)
        if c.shape[-1] != state:  # drop the zero-padded state coordinates
            dc, db = dc[..., :state].contiguous(), db[..., :state].contiguous()
            dqb, dkb = dqb[..., :state].contiguous(), dkb[..., :state].contiguous()
        d_bs, d_cs, d_dtb = torch.empty_like(b_scale), torch.empty_like(c_scale), torch.empty_like(dt_bias)
        _lib.check(lib.m4_mixer_prep_bwd(ctypes.byref(dims), *map(_lib.ptr, (
            proj, b_scale, c_scale, dt_bias, D, g_out, dc, db, dx, dadt, ddt, dtrap, dang, d_proj, part,
            d_bs, d_cs, d_dtb)), _stream()), "m4_mixer_prep_bwd")
        return (d_proj, d_bs, d_cs, d_dtb, dD, dqb.reshape(heads, 1, state), dkb.reshape(heads, 1, state),
                None, None, None, None, None)


def mamba_mixer_core(proj, b_scale, c_scale, dt_bias, D, q_bias, k_bias, *, inner, heads, angles, eps,
                     state=64):
    """proj [B,T,2 inner + 2 state + 3 heads + angles] bf16 -> gated scan
    output [B,T,inner] bf16 (input of the mixer's out projection); `state`
    is the scan state dim N (64, 96 or 128), the width of the B and C slices."""
    if not proj.is_cuda:
        raise RuntimeError("mamba_mixer_core runs on CUDA tensors only (no CPU path)")
    if proj.dtype != torch.bfloat16:
        raise ValueError("mamba_mixer_core expects a bfloat16 projection")
    f32 = lambda t: t.float().contiguous()  # noqa: E731
    width = 2 * inner + 2 * state + 3 * heads + angles
    if proj.shape[-1] != width:
        raise ValueError(f"projection width {proj.shape[-1]} != 2 inner + 2 state + 3 heads + angles = {width}")
    if width % 8:
        # Rows are read with 16-byte loads: pad the row stride to a multiple of 8.
        proj = torch.nn.functional.pad(proj, (0, -width % 8))
    return _MambaMixerCore.apply(proj.contiguous(), f32(b_scale), f32(c_scale), f32(dt_bias), f32(D),
                                 f32(q_bias), f32(k_bias), inner, heads, angles, eps, state)


@torch.no_grad()
def mamba_mixer_step(proj, b_scale, c_scale, dt_bias, D, q_bias, k_bias, cache, *, inner, heads, angles, eps,
                     inplace=False, state=64):
    """One cached token of the mixer core (`_Mamba3StepMixer`,
    `lm/models/mamba4.py:412-481`): proj [B, width] bf16 and the scan cache
    -> (gated output [B, inner] bf16, new cache), through the training
    glue's kernels at one row per sequence (`m4_mixer_prep_fwd`, the scan
    step `m4_scan_step`, `m4_mixer_post_fwd`): three launches, the same
    rounding points as `mamba_mixer_core`. inplace=True writes the new scan
    cache over `cache`'s tensors (see `mamba3_step`)."""
    if not proj.is_cuda:
        raise RuntimeError("mamba_mixer_step runs on CUDA tensors only (no CPU path)")
    if proj.dtype != torch.bfloat16:
        raise ValueError("mamba_mixer_step expects a bfloat16 projection")
    width = 2 * inner + 2 * state + 3 * heads + angles
    if proj.shape[-1] != width:
        raise ValueError(f"projection width {proj.shape[-1]} != 2 inner + 2 state + 3 heads + angles = {width}")
    if width % 8:
        proj = torch.nn.functional.pad(proj, (0, -width % 8))
    proj = proj.contiguous()
    lib = _lib.load()
    batch = proj.shape[0]
    dims = _mix_dims(batch, inner, heads, angles, eps, proj.shape[-1], state)
    dev = proj.device
    c = torch.empty(batch, state, dtype=torch.bfloat16, device=dev)
    b = torch.empty_like(c)
    x = torch.empty(batch, inner, dtype=torch.bfloat16, device=dev)
    adt = torch.empty(batch, heads, device=dev)
    dt, trap = torch.empty_like(adt), torch.empty_like(adt)
    ang = torch.empty(batch, angles, device=dev)
    f32 = lambda t: t.float().contiguous()  # noqa: E731
    _lib.check(lib.m4_mixer_prep_fwd(ctypes.byref(dims), *map(_lib.ptr, (
        proj, f32(b_scale), f32(c_scale), f32(dt_bias), c, b, x, adt, dt, trap, ang)), _stream()),
        "m4_mixer_prep_fwd")
    y, cache = mamba3_step(cache, c, b, x, adt, dt, trap, ang, q_bias=q_bias, k_bias=k_bias, inplace=inplace)
    out = torch.empty(batch, inner, dtype=torch.bfloat16, device=dev)
    _lib.check(lib.m4_mixer_post_fwd(ctypes.byref(dims), *map(_lib.ptr, (proj, y, f32(D), out)), _stream()),
               "m4_mixer_post_fwd")
    return out, cache


ADD_RMS_FEATURES = (256, 512, 768, 1024)


@torch.no_grad()
def add_rms_norm_bf16(x, delta, scale, eps):
    """Residual add fused with the next RMSNorm, for decode (no gradient):
    returns (x + delta, rmsnorm(x + delta) * scale), both bf16 [rows, F] with
    F in ADD_RMS_FEATURES; the same rounding as the residual add followed by
    `rms_norm_bf16` (the decode blocks' residual, lm/models/mamba4.py:358,
    :404, then the next block's norm)."""
    if not x.is_cuda:
        raise RuntimeError("add_rms_norm_bf16 runs on CUDA tensors only (no CPU path)")
    features = x.shape[-1]
    if x.dtype != torch.bfloat16 or delta.dtype != torch.bfloat16 or features not in ADD_RMS_FEATURES:
        raise ValueError(f"add_rms_norm_bf16 expects bf16 rows of {ADD_RMS_FEATURES} features")
    x, delta = x.contiguous(), delta.contiguous()
    x_out, y = torch.empty_like(x), torch.empty_like(x)
    lib = _lib.load()
    _lib.check(lib.m4_add_rmsnorm_fwd(x.numel() // features, features, float(eps), *map(_lib.ptr, (
        x, delta, scale.float().contiguous(), x_out, y)), _stream()), "m4_add_rmsnorm_fwd")
    return x_out, y


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


# ---------------------------------------------------------------------------
# Selective-memory mixer glue (lm/models/mamba4.py:155-260)
# ---------------------------------------------------------------------------
def _row_stride(view):
    """Row stride (elements) of a [B,T,F] view whose rows are uniformly spaced."""
    b, t, f = view.shape
    if view.stride(2) != 1 or (b > 1 and view.stride(0) != t * view.stride(1)):
        raise ValueError("expected a [B,T,F] view with unit last stride and uniform row stride")
    return view.stride(1)


def _memmix_dims(batch, time, heads, stride, gate_stride, beta_max):
    return _lib.MemMixDims(batch, time, heads, stride, gate_stride, beta_max)


class GradSlab:
    """One gradient buffer for a projection whose column slices feed several
    glue kernels (the memory mixer's gate and rest columns): each backward
    kernel writes its columns straight into it (the kernels store gradients
    with the row stride of their input view), and the split returns it whole,
    so autograd never builds the projection gradient from zero-filled
    slice-sized pieces and an add."""

    def __init__(self):
        self.shape = None
        self.buf = None

    def attach(self, proj, used):
        self.shape, self.dtype, self.device, self.used = proj.shape, proj.dtype, proj.device, used
        self.buf = None

    def buffer(self):
        if self.buf is None:
            self.buf = torch.empty(self.shape, dtype=self.dtype, device=self.device)
            if self.used < self.shape[-1]:
                self.buf[..., self.used:].zero_()  # columns no kernel reads get no gradient
        return self.buf


def _is_slice_of(base, t, col):
    return (t is not None and t.dim() == base.dim() and t.data_ptr() == base.data_ptr() + col * base.element_size()
            and t.stride()[:-1] == base.stride()[:-1] and t.stride(-1) == 1)


class _SplitProjection(torch.autograd.Function):
    """proj [B,T,W] -> (proj[..., :inner], proj[..., inner:inner + rest]) as views."""

    @staticmethod
    def forward(ctx, proj, inner, rest, slab):
        slab.attach(proj, inner + rest)
        ctx.slab, ctx.inner, ctx.rest = slab, inner, rest
        return proj[..., :inner], proj[..., inner: inner + rest]

    @staticmethod
    def backward(ctx, d_gate, d_rest):
        slab, inner, rest = ctx.slab, ctx.inner, ctx.rest
        buf = slab.buf
        slab.buf = None
        if buf is not None and _is_slice_of(buf, d_gate, 0) and _is_slice_of(buf, d_rest, inner):
            return buf, None, None, None
        out = torch.zeros(slab.shape, dtype=slab.dtype, device=slab.device)
        if d_gate is not None:
            out[..., :inner] = d_gate
        if d_rest is not None:
            out[..., inner: inner + rest] = d_rest
        return out, None, None, None


def split_projection(proj, inner, rest, slab):
    """Gate and rest column views of the memory mixer's projection that share
    one gradient buffer (`slab`, passed on to the prep and post glue)."""
    return _SplitProjection.apply(proj, inner, rest, slab)


def _grad_view(slab, col, like, stride):
    """Gradient buffer for a [B,T,F] view with row stride `stride`: a column
    slice of the slab when there is one, else a fresh buffer of that stride."""
    if slab is not None and slab.shape is not None:
        return slab.buffer()[..., col: col + like.shape[-1]]
    batch, time, width = like.shape
    return torch.empty(batch, time, stride, dtype=torch.bfloat16, device=like.device)[..., :width]


class _MemPrep(torch.autograd.Function):
    @staticmethod
    def forward(ctx, rest, conv_w, conv_b, beta_bias, dt_bias, a_log, heads, bound, beta_max, slab, col):
        lib = _lib.load()
        batch, time, _ = rest.shape
        dims = _memmix_dims(batch, time, heads, _row_stride(rest), 0 + 128 * heads, beta_max)
        dev = rest.device
        values = torch.empty(batch, time, heads, 128, device=dev)
        keys = torch.empty(batch, time, heads, 64, device=dev)
        queries = torch.empty_like(keys)
        beta = torch.empty(batch, time, heads, device=dev)
        log_decay, order_logit = torch.empty_like(beta), torch.empty_like(beta)
        _lib.check(lib.m4_memmix_prep_fwd(ctypes.byref(dims), _lib.ptr(rest), _lib.ptr(conv_w), _lib.ptr(conv_b),
                                          bound, *map(_lib.ptr, (beta_bias, dt_bias, a_log, values, keys, queries,
                                                                 beta, log_decay, order_logit)), _stream()),
                   "m4_memmix_prep_fwd")
        ctx.save_for_backward(rest, conv_w, conv_b, beta_bias, dt_bias, a_log)
        ctx.cfg = (heads, bound, beta_max)
        ctx.slab, ctx.col = slab, col
        return values, keys, queries, beta, log_decay, order_logit

    @staticmethod
    def backward(ctx, d_values, d_keys, d_queries, d_beta, d_log_decay, d_order):
        lib = _lib.load()
        rest, conv_w, conv_b, beta_bias, dt_bias, a_log = ctx.saved_tensors
        heads, bound, beta_max = ctx.cfg
        batch, time, _ = rest.shape
        dims = _memmix_dims(batch, time, heads, _row_stride(rest), 128 * heads, beta_max)
        dev = rest.device

        def g(t, shape):
            return torch.zeros(shape, device=dev) if t is None else t.float().contiguous()

        d_values = g(d_values, (batch, time, heads, 128))
        d_keys = g(d_keys, (batch, time, heads, 64))
        d_queries = g(d_queries, (batch, time, heads, 64))
        d_beta = g(d_beta, (batch, time, heads))
        d_log_decay = g(d_log_decay, (batch, time, heads))
        d_order = g(d_order, (batch, time, heads))
        channels = 256 * heads
        d_conv = torch.empty(batch, time, channels, device=dev)
        d_rest = _grad_view(ctx.slab, ctx.col, rest, _row_stride(rest))
        part = torch.empty(lib.m4_memmix_partial_floats(ctypes.byref(dims)), device=dev)
        d_w, d_b = torch.empty_like(conv_w), torch.empty_like(conv_b)
        d_bb, d_dtb, d_al = torch.empty_like(beta_bias), torch.empty_like(dt_bias), torch.empty_like(a_log)
        _lib.check(lib.m4_memmix_prep_bwd(ctypes.byref(dims), _lib.ptr(rest), _lib.ptr(conv_w), _lib.ptr(conv_b),
                                          bound, *map(_lib.ptr, (beta_bias, dt_bias, a_log, d_values, d_keys,
                                                                 d_queries, d_beta, d_log_decay, d_order, d_conv,
                                                                 d_rest, part, d_w, d_b, d_bb, d_dtb, d_al)),
                                          _stream()), "m4_memmix_prep_bwd")
        return d_rest, d_w, d_b, d_bb, d_dtb, d_al, None, None, None, None, None


class _OrderScan(torch.autograd.Function):
    @staticmethod
    def forward(ctx, values, logit):
        lib = _lib.load()
        batch, time, heads, _ = values.shape
        dims = _memmix_dims(batch, time, heads, 259 * heads + (-259 * heads) % 8, 128 * heads, 1.0)
        ordered = torch.empty_like(values)
        scratch = torch.empty(lib.m4_memmix_order_scratch_floats(ctypes.byref(dims)), device=values.device)
        _lib.check(lib.m4_memmix_order_fwd(ctypes.byref(dims), *map(_lib.ptr, (values, logit, ordered, scratch)),
                                           _stream()), "m4_memmix_order_fwd")
        ctx.save_for_backward(values, logit, ordered)
        return ordered

    @staticmethod
    def backward(ctx, g):
        lib = _lib.load()
        values, logit, ordered = ctx.saved_tensors
        batch, time, heads, _ = values.shape
        dims = _memmix_dims(batch, time, heads, 259 * heads + (-259 * heads) % 8, 128 * heads, 1.0)
        d_values = torch.empty_like(values)
        d_logit4 = torch.empty(batch, time, heads, 4, device=values.device)
        scratch = torch.empty(lib.m4_memmix_order_scratch_floats(ctypes.byref(dims)), device=values.device)
        _lib.check(lib.m4_memmix_order_bwd(ctypes.byref(dims), *map(_lib.ptr, (
            values, logit, ordered, g.float().contiguous(), d_values, d_logit4, scratch)), _stream()),
            "m4_memmix_order_bwd")
        return d_values, d_logit4.sum(-1)


class _MemPost(torch.autograd.Function):
    @staticmethod
    def forward(ctx, out, var, values, ordered, gate, conf_scale, D, order_mix, scale, eps, slab):
        lib = _lib.load()
        batch, time, heads, _ = values.shape
        dims = _memmix_dims(batch, time, heads, 259 * heads + (-259 * heads) % 8, _row_stride(gate), 1.0)
        y = torch.empty(batch, time, heads * 128, dtype=torch.bfloat16, device=values.device)
        rstd = torch.empty(batch, time, heads, device=values.device)
        _lib.check(lib.m4_memmix_post_fwd(ctypes.byref(dims), eps, *map(_lib.ptr, (
            out, var, values, ordered, gate, conf_scale, D, order_mix, scale, y, rstd)), _stream()),
            "m4_memmix_post_fwd")
        ctx.save_for_backward(out, var, values, ordered, gate, conf_scale, D, order_mix, scale, rstd)
        ctx.slab = slab
        return y

    @staticmethod
    def backward(ctx, g):
        lib = _lib.load()
        out, var, values, ordered, gate, conf_scale, D, order_mix, scale, rstd = ctx.saved_tensors
        batch, time, heads, _ = values.shape
        dims = _memmix_dims(batch, time, heads, 259 * heads + (-259 * heads) % 8, _row_stride(gate), 1.0)
        dev = values.device
        d_out, d_values, d_ordered = (torch.empty_like(values) for _ in range(3))
        d_var = torch.empty_like(var)
        d_gate = _grad_view(ctx.slab, 0, gate, _row_stride(gate))
        part = torch.empty(lib.m4_memmix_partial_floats(ctypes.byref(dims)), device=dev)
        d_cs, d_D, d_om, d_scale = (torch.empty_like(t) for t in (conf_scale, D, order_mix, scale))
        _lib.check(lib.m4_memmix_post_bwd(ctypes.byref(dims), *map(_lib.ptr, (
            out, var, values, ordered, gate, conf_scale, D, order_mix, scale, rstd,
            g.to(torch.bfloat16).contiguous(), d_out, d_var, d_values, d_ordered, d_gate, part, d_cs, d_D, d_om,
            d_scale)), _stream()), "m4_memmix_post_bwd")
        return d_out, d_var, d_values, d_ordered, d_gate, d_cs, d_D, d_om, d_scale, None, None


def memory_mixer_prep(rest, conv_w, conv_b, beta_bias, dt_bias, a_log, *, heads, bound, beta_max, slab=None,
                      col=0):
    """rest [B,T,259h] bf16 view (value|key|query|beta|dt|order columns) ->
    values [B,T,h,128], unit keys (shifted one token) and queries [B,T,h,64],
    beta, log_decay, order logit [B,T,h] (float32). With `slab` (from
    split_projection) the gradient of `rest` is written into its columns
    starting at `col`."""
    if not rest.is_cuda:
        raise RuntimeError("memory_mixer_prep runs on CUDA tensors only (no CPU path)")
    if rest.dtype != torch.bfloat16 or rest.shape[-1] != 259 * heads:
        raise ValueError("memory_mixer_prep expects bf16 rows of 259 * heads columns")
    f32 = lambda t: t.float().contiguous()  # noqa: E731
    return _MemPrep.apply(rest, f32(conv_w), f32(conv_b), f32(beta_bias), f32(dt_bias), f32(a_log), heads,
                          float(bound), float(beta_max), slab, col)


def order_scan(values, logit):
    """Order head of the memory mixer: h_t = s h_(t-1) + (1 - s) v_t, s = sigmoid(logit)."""
    return _OrderScan.apply(values.float().contiguous(), logit.float().contiguous())


def memory_mixer_post(out, var, values, ordered, gate, conf_scale, D, order_mix, scale, eps, slab=None):
    """Confidence gate, D skip, order mix, read RMSNorm and SiLU gate -> bf16 [B,T,128h].
    With `slab` (from split_projection) the gradient of `gate` is written into
    its first columns."""
    f32 = lambda t: t.float().contiguous()  # noqa: E731
    return _MemPost.apply(f32(out), f32(var), f32(values), f32(ordered), gate, f32(conf_scale), f32(D),
                          f32(order_mix), f32(scale), float(eps), slab)


@torch.no_grad()
def memory_mixer_step(proj, cache, conv_w, conv_b, beta_bias, dt_bias, a_log, floor, conf_scale, D, order_mix,
                      scale, *, heads, bound, beta_max, eps, order_head=True, inplace=False):
    """One cached token of the memory mixer (`lm/models/mamba4.py:127-337`
    with a cache) in three launches: `m4_memmix_prep_step` (conv over the
    history rows and the current one, SiLU, unit key and query, gates),
    `m4_memread_decode` (the read with the key carried from the previous
    token: the key shift) and `m4_memmix_post_step` (order-head step,
    confidence gate, D skip, read RMSNorm, SiLU gate).

    proj [B, width] bf16: gate [128h] | rest [259h] columns (width a multiple
    of 8). cache: dict(history [B, 3, width] bf16 (the previous three
    projection rows, zero before the sequence start), shifted [B,h,64] (the
    previous token's unit key, zero at the first token), memory
    (SelectiveState), order [B,h,128]). Returns (y [B, 128h] bf16, new cache).
    inplace=True writes the new memory state over the cached one (see
    `selective_decode`); the other cache entries are always fresh tensors.
    """
    from .memory import selective_decode

    if not proj.is_cuda:
        raise RuntimeError("memory_mixer_step runs on CUDA tensors only (no CPU path)")
    batch, width = proj.shape
    inner = 128 * heads
    if proj.dtype != torch.bfloat16 or width % 8 or width < inner + 259 * heads:
        raise ValueError("memory_mixer_step expects bf16 rows of gate and rest columns, width a multiple of 8")
    lib = _lib.load()
    dev = proj.device
    window = torch.cat((cache["history"], proj[:, None]), dim=1)         # [B, 4, width]
    dims = _memmix_dims(batch, window.shape[1], heads, width, width, beta_max)
    values = torch.empty(batch, heads, 128, device=dev)
    keys, queries = torch.empty(batch, heads, 64, device=dev), torch.empty(batch, heads, 64, device=dev)
    beta, log_decay, order_logit = (torch.empty(batch, heads, device=dev) for _ in range(3))
    f32 = lambda t: t.float().contiguous()  # noqa: E731
    _lib.check(lib.m4_memmix_prep_step(
        ctypes.byref(dims), window[..., inner:].data_ptr(), *map(_lib.ptr, (f32(conv_w), f32(conv_b))),
        float(bound), *map(_lib.ptr, (f32(beta_bias), f32(dt_bias), f32(a_log), values, keys, queries, beta,
                                      log_decay, order_logit)), _stream()), "m4_memmix_prep_step")
    res = selective_decode(cache["memory"], cache["shifted"], values, queries, beta, log_decay, floor,
                           inplace=inplace)
    y = torch.empty(batch, inner, dtype=torch.bfloat16, device=dev)
    order = torch.empty_like(values) if order_head else None
    pdims = _memmix_dims(batch, 1, heads, width, width, beta_max)
    _lib.check(lib.m4_memmix_post_step(
        ctypes.byref(pdims), float(eps), *map(_lib.ptr, (
            res.output, res.variance, values, order_logit, f32(cache["order"]) if order_head else None, order,
            proj, f32(conf_scale), f32(D), f32(order_mix), f32(scale), y)), _stream()), "m4_memmix_post_step")
    new = dict(history=window[:, 1:], shifted=keys, memory=res.state,
               order=order if order_head else cache["order"])
    return y, new


# ---------------------------------------------------------------------------
# Tied output head + cross-entropy (lm/models/mamba4.py:499-504, lm/train.py:81-87)
# ---------------------------------------------------------------------------
class _HeadCrossEntropy(torch.autograd.Function):
    """loss[r] = logsumexp(l_r) - l_r[target_r] with l = rd_bf16(x W^T): the
    bf16 logits are kept (not widened to float32) and overwritten in place by
    their gradient in the backward."""

    @staticmethod
    def forward(ctx, x, weight, targets):
        lib = _lib.load()
        rows, vocab = x.shape[0], weight.shape[0]
        w16 = weight.to(torch.bfloat16)
        if vocab % 8:
            # Rows of 16-byte multiples: zero weight rows give ignored logits.
            w16 = torch.nn.functional.pad(w16, (0, 0, 0, -vocab % 8))
        ld = w16.shape[0]
        logits = torch.matmul(x, w16.t())
        loss = torch.empty(rows, device=x.device)
        lse = torch.empty(rows, device=x.device)
        _lib.check(lib.m4_cross_entropy_fwd(rows, vocab, ld, *map(_lib.ptr, (logits, targets, loss, lse)),
                                            _stream()), "m4_cross_entropy_fwd")
        ctx.save_for_backward(x, w16, targets, logits, lse)
        ctx.vocab = vocab
        return loss

    @staticmethod
    def backward(ctx, g):
        lib = _lib.load()
        x, w16, targets, logits, lse = ctx.saved_tensors
        rows, ld = logits.shape
        vocab = ctx.vocab
        _lib.check(lib.m4_cross_entropy_bwd(rows, vocab, ld, *map(_lib.ptr, (logits, targets, lse,
                                                                             g.float().contiguous())), _stream()),
                   "m4_cross_entropy_bwd")
        dx = torch.matmul(logits, w16)
        dw = torch.matmul(logits.t(), x)[:vocab].float()
        return dx, dw, None


def head_cross_entropy(x, weight, targets):
    """Per-token loss of the tied head: x [..., D] bf16, weight [V, D] (the
    embedding), targets [...] int64 -> float32 loss [...]."""
    if not x.is_cuda:
        raise RuntimeError("head_cross_entropy runs on CUDA tensors only (no CPU path)")
    lead = x.shape[:-1]
    loss = _HeadCrossEntropy.apply(x.reshape(-1, x.shape[-1]).to(torch.bfloat16).contiguous(), weight,
                                   targets.reshape(-1).to(torch.int64).contiguous())
    return loss.reshape(lead)
