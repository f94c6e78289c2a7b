"""Data-parallel Mamba 4 training step (one process per GPU, NCCL).

Restates `lm/train.py` (`optimizer` :57-78, `local_loss` :81-87, `make_steps`
:90-114) for torch.distributed: every rank computes the summed token loss of
its shard, the global target count is all-reduced first, gradients are summed
over ranks by DDP's bucketed NCCL all-reduce (overlapped with the backward)
and divided by the global count, then clipped to global norm 1.0 and applied
with AdamW (b1 0.9, b2 0.95, eps 1e-8, weight decay 0.1 on parameters with
ndim >= 2) under a warmup + cosine schedule (optax warmup_cosine_decay).
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


class DataParallelTrainer:
    """One optimizer step per call on this rank's shard of the global batch.

    `world` > 1 requires an initialised process group; gradients are summed by
    DDP (one NCCL all-reduce per bucket, overlapped with the backward).
    """

    def __init__(self, model: torch.nn.Module, settings: TrainSettings, world: int = 1,
                 device_id: int | None = None, bucket_mb: int = 64):
        self.settings = settings
        self.world = world
        self.model = model
        if world > 1:
            self.net = torch.nn.parallel.DistributedDataParallel(
                model, device_ids=None if device_id is None else [device_id],
                bucket_cap_mb=bucket_mb, gradient_as_bucket_view=True, static_graph=True)
        else:
            self.net = model
        fused = next(model.parameters()).is_cuda
        self.optimizer = torch.optim.AdamW(
            param_groups(model, settings.weight_decay), lr=settings.learning_rate,
            betas=(settings.beta1, settings.beta2), eps=settings.adam_epsilon, fused=fused)
        self.step_index = 0

    def _all_reduce(self, t: torch.Tensor) -> torch.Tensor:
        if self.world > 1:
            dist.all_reduce(t)
        return t

    def step(self, tokens: torch.Tensor, targets: torch.Tensor, mask: torch.Tensor):
        """Returns (global mean loss, global target count, grad norm) as tensors."""
        count = self._all_reduce(mask.sum().to(torch.float32))
        total = torch.clamp(count, min=1.0)
        with torch.autocast(tokens.device.type, dtype=torch.bfloat16, enabled=tokens.is_cuda):
            if getattr(self.model, "fused_loss", False) and tokens.is_cuda:
                # Per-token losses from the fused head (the model takes targets).
                losses = self.net(tokens, targets).reshape(-1)
            else:
                logits = self.net(tokens)
                losses = F.cross_entropy(logits.float().reshape(-1, logits.shape[-1]), targets.reshape(-1),
                                         reduction="none")
        numerator = (losses * mask.reshape(-1).float()).sum()
        # DDP averages over ranks; scaling by world / global count turns the
        # average into sum-over-ranks / global count (`lm/train.py:95-99`).
        (numerator * (self.world / total)).backward()
        norm = torch.nn.utils.clip_grad_norm_(self.model.parameters(), self.settings.clip_norm)
        for group in self.optimizer.param_groups:
            group["lr"] = learning_rate(self.settings, self.step_index)
        self.optimizer.step()
        self.optimizer.zero_grad(set_to_none=True)  # fresh gradients next step: no fill, no accumulate
        self.step_index += 1
        loss = self._all_reduce(numerator.detach().clone()) / total
        return loss, count, norm


def synthetic_batch(batch: int, seq: int, vocab: int, seed: int, device):
    """Uniform-random token ids: inputs, next-token
    targets, unit loss mask."""
    g = torch.Generator(device="cpu").manual_seed(seed)
    ids = torch.randint(0, vocab, (batch, seq + 1), generator=g)
    tokens = ids[:, :-1].contiguous()
    targets = ids[:, 1:].contiguous()
    mask = torch.ones(batch, seq, dtype=torch.float32)
    return tokens.to(device), targets.to(device), mask.to(device)
