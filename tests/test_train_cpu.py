"""Data-parallel training logic on CPU ranks (gloo, world size 2).

The multi-device check of the reference (`lm/tests/test_training.py:18-56`):
uneven loss masks across ranks, gradients summed over ranks and divided by
the global target count, must equal a single process on the whole batch.
A small CPU model stands in for the CUDA operators; the trainer code under
test is the one the GPU training step uses.
"""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from mamba4_b200.train import DataParallelTrainer, TrainSettings, learning_rate


class Tiny(torch.nn.Module):
    def __init__(self, vocab=17, width=8):
        super().__init__()
        g = torch.Generator().manual_seed(0)
        self.embedding = torch.nn.Embedding(vocab, width)
        self.proj = torch.nn.Linear(width, width, bias=False)
        self.scale = torch.nn.Parameter(torch.ones(width))
        with torch.no_grad():
            self.embedding.weight.copy_(torch.randn(vocab, width, generator=g) * 0.5)
            self.proj.weight.copy_(torch.randn(width, width, generator=g) * 0.5)

    def forward(self, tokens):
        x = torch.tanh(self.proj(self.embedding(tokens))) * self.scale
        return x @ self.embedding.weight.t()


def batch():
    g = torch.Generator().manual_seed(1)
    tokens = torch.randint(0, 17, (4, 6), generator=g)
    targets = torch.randint(0, 17, (4, 6), generator=g)
    mask = torch.zeros(4, 6)
    for row, n in enumerate([6, 4, 1, 0]):  # uneven masks, as the reference test
        mask[row, :n] = 1
    return tokens, targets, mask


SETTINGS = TrainSettings(learning_rate=0.1, warmup_steps=1, total_steps=10)


def _worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        tokens, targets, mask = batch()
        rows = slice(rank * 2, rank * 2 + 2)
        trainer = DataParallelTrainer(Tiny(), SETTINGS, world=world)
        calls = []
        plain = dist.all_reduce

        def counting(*args, **kwargs):
            calls.append(args[0].numel())
            return plain(*args, **kwargs)

        dist.all_reduce = counting
        try:
            loss, count, norm = trainer.step(tokens[rows], targets[rows], mask[rows])
        finally:
            dist.all_reduce = plain
        if rank == 0:
            out.put({"loss": float(loss), "count": float(count), "norm": float(norm),
                     "params": [p.detach().tolist() for p in trainer.model.parameters()],
                     "all_reduce_sizes": calls})
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.timeout(120)
def test_two_rank_step_equals_single_process_with_uneven_masks():
    tokens, targets, mask = batch()
    single = DataParallelTrainer(Tiny(), SETTINGS, world=1)
    loss1, count1, norm1 = single.step(tokens, targets, mask)
    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, out)) for r in range(2)]
    for p in procs:
        p.start()
    result = out.get(timeout=100)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    # One collective per step: the tiny model's gradients fit one bucket, which
    # also carries the target count and loss numerator (2 extra floats).
    n_params = sum(p.numel() for p in single.model.parameters())
    assert result["all_reduce_sizes"] == [n_params + 2]
    assert result["count"] == float(count1) == 11.0
    assert abs(result["loss"] - float(loss1)) < 1e-6
    assert abs(result["norm"] - float(norm1)) < 1e-5
    for a, b in zip(result["params"], single.model.parameters()):
        torch.testing.assert_close(torch.tensor(a), b.detach(), rtol=1e-6, atol=1e-7)


def test_weight_decay_mask_and_schedule():
    from mamba4_b200.train import param_groups

    groups = param_groups(Tiny(), 0.1)
    assert all(p.ndim >= 2 for p in groups[0]["params"]) and groups[0]["weight_decay"] == 0.1
    assert all(p.ndim < 2 for p in groups[1]["params"]) and groups[1]["weight_decay"] == 0.0
    s = TrainSettings(learning_rate=1.0, warmup_steps=10, total_steps=100, min_lr_ratio=0.1)
    assert learning_rate(s, 0) == pytest.approx(0.1)          # init = peak / warmup
    assert learning_rate(s, 10) == pytest.approx(1.0)         # peak after warmup
    assert learning_rate(s, 100) == pytest.approx(0.1)        # end = peak * min ratio


def test_model_parameter_counts_match_the_baseline_configs():
    from mamba4_b200.model import CONFIGS, Mamba4LM, parameter_count

    n60 = parameter_count(Mamba4LM(CONFIGS["60m"]))
    n125 = parameter_count(Mamba4LM(CONFIGS["125m"]))
    assert 50e6 < n60 < 60e6
    assert 110e6 < n125 < 130e6
    assert CONFIGS["60m"].layer_pattern.count("M") == 4 and CONFIGS["60m"].n_layers == 16
    assert CONFIGS["125m"].layer_pattern.count("M") == 4 and CONFIGS["125m"].n_layers == 21
