"""CPU restatement of the model glue around the hot-path operators (oracle).

TEST INFRASTRUCTURE ONLY (see `oracle/__init__.py`): the fused glue kernels
of the product package are checked against compositions built from these
functions, never the other way round.

* `causal_conv`: the memory mixer's depthwise causal convolution
  (`lm/models/mamba4.py:98-108`).
* `order_memory_chunked`: the order head h_t = lam_t h_(t-1) + (1 - lam_t) v_t
  in the reference's chunked form (`lm/models/mamba4.py:59-95`).
* `EmulatedScan`: the Mamba-3 scan of `mamba3_fused` as an autograd function
  whose forward and backward are the bf16 rounding-point restatements of the
  reference kernels (`oracle/scan.py`: `fused_layout_scan` with
  `model_dtype=bfloat16`, `fused_layout_grads_emulated`), so a float64 glue
  composition around it sees the scan the reference computes.
* `memory_read`: the memory read in float64 with autograd (the XLA path of
  `selective_gaussian_memory` restated in `oracle/cpu_path.py`).

All functions run on CPU tensors of any float dtype.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

from . import cpu_path
from . import scan as S


def causal_conv(x, weight, bias):
    """Depthwise causal convolution over time (`lm/models/mamba4.py:98-108`):
    x [B,T,C], weight [taps, C], bias [C]; output_t = bias + sum_j
    weight[j] x_(t - taps + 1 + j) with zeros before the sequence."""
    taps = weight.shape[0]
    xt = F.pad(x.transpose(1, 2), (taps - 1, 0))
    w = weight.t().unsqueeze(1)  # [channels, 1, taps]
    return F.conv1d(xt, w, bias, groups=x.shape[-1]).transpose(1, 2)


def order_memory_chunked(values, log_decay, chunk_size=64):
    """h_t = lam_t h_(t-1) + (1 - lam_t) v_t, lam = exp(log_decay), in the
    reference's chunked form (`lm/models/mamba4.py:59-95`): values [B,T,H,P],
    log_decay [B,T,H]."""
    x = values
    batch, time, heads, width = x.shape
    pad = (-time) % chunk_size
    count = (time + pad) // chunk_size

    def chunks(a):
        a = F.pad(a, [0, 0] * (a.ndim - 2) + [0, pad])
        return a.reshape(batch, count, chunk_size, *a.shape[2:]).transpose(2, 3)

    value, logs = chunks(x), chunks(log_decay)   # [B,n,H,c,P], [B,n,H,c]
    inflow = -torch.expm1(logs)
    prefix = torch.cumsum(logs, dim=-1)
    causal = torch.tril(torch.ones(chunk_size, chunk_size, dtype=torch.bool))
    diff = prefix[..., :, None] - prefix[..., None, :]
    weights = torch.where(causal, torch.exp(torch.where(causal, diff, torch.zeros_like(diff))),
                          torch.zeros_like(diff))
    local = torch.einsum("bnhts,bnhsp->bnhtp", weights * inflow[..., None, :], value)
    ends = local[..., -1, :]                               # [B,n,H,P]
    decay = torch.exp(prefix[..., -1])                     # [B,n,H]
    carries, state = [], torch.zeros_like(ends[:, 0])
    for n in range(count):
        carries.append(state)
        state = decay[:, n, :, None] * state + ends[:, n]
    starts = torch.stack(carries, 1)
    out = local + torch.exp(prefix)[..., None] * starts[..., None, :]
    return out.transpose(2, 3).reshape(batch, count * chunk_size, heads, width)[:, :time]


class EmulatedScan(torch.autograd.Function):
    """`mamba3_fused(c, b, x, adt, dt, trap_logits, angles, q_bias, k_bias)` with
    the reference kernels' bf16 rounding points in both directions; returns
    (y [B,T,H*P], final [B,H,N,P]) in the input dtype."""

    @staticmethod
    def forward(ctx, c, b, x, adt, dt, trap_logits, angles, q_bias, k_bias):
        args = [a.detach().float() for a in (c, b, x, adt, dt, trap_logits, angles, q_bias, k_bias)]
        for i in range(3):
            args[i] = args[i].to(torch.bfloat16).float()
        ctx.args = args
        ctx.dtype = x.dtype
        y, final = S.fused_layout_scan(*args, chunk=64, model_dtype=torch.bfloat16,
                                       compute_dtype=torch.float32)
        return y.to(x.dtype), final.to(x.dtype)

    @staticmethod
    def backward(ctx, d_y, d_final):
        grads = S.fused_layout_grads_emulated(ctx.args, d_y.float(), d_final.float(), chunk=64,
                                              model_dtype=torch.bfloat16)
        return tuple(g.to(ctx.dtype) for g in grads)


def memory_read(keys, values, queries, beta, log_decay, floor):
    """Memory read (output, variance) with autograd in the inputs' dtype."""
    return cpu_path.memory_read(keys, values, queries, beta, log_decay, floor)
