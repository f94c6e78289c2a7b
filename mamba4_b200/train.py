"""Data-parallel Mamba 4 training step (one process per GPU, NCCL).

Restates `lm/train.py` (`optimizer` :57-78, `local_loss` :81-87, `make_steps`
:90-114) for torch.distributed: every rank computes the summed token loss of
its shard; the gradient sums, the target count and the loss numerator cross
the ranks in ONE all-reduce per step, DDP's bucketed NCCL all-reduce
(overlapped with the backward) with a communication hook that sums instead
of averaging and carries the two scalars in the last bucket (the reference's
psum of count, gradients and loss, `:95-99`). The summed gradients are then
divided by the global count, clipped to global norm 1.0 as
optax.clip_by_global_norm does, and applied with AdamW (b1 0.9, b2 0.95,
eps 1e-8, weight decay 0.1 on parameters with ndim >= 2) under a warmup +
cosine schedule (optax warmup_cosine_decay).
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.distributed as dist
import torch.nn.functional as F


@dataclass(frozen=True)
class TrainSettings:
    """Subset of the reference `TrainConfig` (`lm/config.py:91-121`)."""

    learning_rate: float = 6e-4
    min_lr_ratio: float = 0.1
    warmup_steps: int = 200
    total_steps: int = 7630
    weight_decay: float = 0.1
    beta1: float = 0.9
    beta2: float = 0.95
    adam_epsilon: float = 1e-8
    clip_norm: float = 1.0


def learning_rate(settings: TrainSettings, step: int) -> float:
    """optax.warmup_cosine_decay_schedule as configured at `lm/train.py:57-65`."""
    warmup = min(settings.warmup_steps, max(1, settings.total_steps // 10))
    peak = settings.learning_rate
    init = peak / warmup
    end = peak * settings.min_lr_ratio
    decay_steps = max(settings.total_steps, warmup + 1)
    if step < warmup:
        return init + (peak - init) * step / warmup
    progress = min(1.0, (step - warmup) / max(1, decay_steps - warmup))
    return end + (peak - end) * 0.5 * (1 + math.cos(math.pi * progress))


def param_groups(model: torch.nn.Module, weight_decay: float):
    """Weight decay only on parameters with ndim >= 2 (`lm/train.py:66`)."""
    decay = [p for p in model.parameters() if p.ndim >= 2]
    other = [p for p in model.parameters() if p.ndim < 2]
    return [{"params": decay, "weight_decay": weight_decay}, {"params": other, "weight_decay": 0.0}]


class _Totals:
    """Communication-hook state: the (target count, loss numerator) pair this
    rank contributes, and the global sums the last bucket brings back."""

    def __init__(self, device):
        self.local = torch.zeros(2, dtype=torch.float32, device=device)
        self.total = torch.zeros(2, dtype=torch.float32, device=device)


def _sum_with_totals(state: _Totals, bucket):
    """DDP communication hook: all-reduce (sum) each gradient bucket; the last
    bucket also carries the target count and loss numerator, so a step makes
    one all-reduce per bucket and no other collective."""
    buf = bucket.buffer()
    if not bucket.is_last():
        return dist.all_reduce(buf, async_op=True).get_future().then(lambda f: f.value()[0])
    combined = torch.cat((buf, state.local.to(buf.dtype)))
    fut = dist.all_reduce(combined, async_op=True).get_future()

    def unpack(f):
        out = f.value()[0]
        buf.copy_(out[:-2])
        state.total.copy_(out[-2:])
        return buf

    return fut.then(unpack)


class DataParallelTrainer:
    """One optimizer step per call on this rank's shard of the global batch.

    `world` > 1 requires an initialised process group; gradients, the target
    count and the loss numerator are summed by DDP's bucketed all-reduce with
    `_sum_with_totals` as the communication hook (one NCCL all-reduce per
    bucket, overlapped with the backward; nothing else crosses ranks).
    """

    def __init__(self, model: torch.nn.Module, settings: TrainSettings, world: int = 1,
                 device_id: int | None = None, bucket_mb: int = 64):
        self.settings = settings
        self.world = world
        self.model = model
        device = next(model.parameters()).device
        self.totals = _Totals(device)
        if world > 1:
            self.net = torch.nn.parallel.DistributedDataParallel(
                model, device_ids=None if device_id is None else [device_id],
                bucket_cap_mb=bucket_mb, gradient_as_bucket_view=True, static_graph=True,
                broadcast_buffers=False)
            self.net.register_comm_hook(self.totals, _sum_with_totals)
        else:
            self.net = model
        fused = device.type == "cuda"
        self.optimizer = torch.optim.AdamW(
            param_groups(model, settings.weight_decay), lr=settings.learning_rate,
            betas=(settings.beta1, settings.beta2), eps=settings.adam_epsilon, fused=fused)
        self.step_index = 0

    def step(self, tokens: torch.Tensor, targets: torch.Tensor, mask: torch.Tensor):
        """Returns (global mean loss, global target count, grad norm) as tensors."""
        count = mask.sum().to(torch.float32)
        with torch.autocast(tokens.device.type, dtype=torch.bfloat16, enabled=tokens.is_cuda):
            if getattr(self.model, "fused_loss", False) and tokens.is_cuda:
                # Per-token losses from the fused head (the model takes targets).
                losses = self.net(tokens, targets).reshape(-1)
            else:
                logits = self.net(tokens)
                losses = F.cross_entropy(logits.float().reshape(-1, logits.shape[-1]), targets.reshape(-1),
                                         reduction="none")
        numerator = (losses * mask.reshape(-1).float()).sum()
        if self.world > 1:
            self.totals.local.copy_(torch.stack((count, numerator.detach().float())))
        numerator.backward()  # gradient sums (the hook sums over ranks, no averaging)
        if self.world > 1:
            count, total_numerator = self.totals.total[0], self.totals.total[1]
        else:
            total_numerator = numerator.detach().float()
        total = torch.clamp(count, min=1.0)
        grads = [p.grad for p in self.model.parameters() if p.grad is not None]
        # Gradients are sums over the global batch; the reference divides by
        # the global count and clips the global norm (lm/train.py:97-100,
        # optax.clip_by_global_norm): one scale covers both.
        norm_sum = torch.linalg.vector_norm(torch.stack(torch._foreach_norm(grads)))
        norm = norm_sum / total
        clip = self.settings.clip_norm
        scale = torch.where(norm < clip, 1.0 / total, clip / norm_sum)
        torch._foreach_mul_(grads, scale)
        for group in self.optimizer.param_groups:
            group["lr"] = learning_rate(self.settings, self.step_index)
        self.optimizer.step()
        self.optimizer.zero_grad(set_to_none=True)  # fresh gradients next step: no fill, no accumulate
        self.step_index += 1
        return total_numerator / total, count, norm


def synthetic_batch(batch: int, seq: int, vocab: int, seed: int, device):
    """Uniform-random token ids: inputs, next-token
    targets, unit loss mask."""
    g = torch.Generator(device="cpu").manual_seed(seed)
    ids = torch.randint(0, vocab, (batch, seq + 1), generator=g)
    tokens = ids[:, :-1].contiguous()
    targets = ids[:, 1:].contiguous()
    mask = torch.ones(batch, seq, dtype=torch.float32)
    return tokens.to(device), targets.to(device), mask.to(device)
