"""The Mamba 4 LM around the CUDA operators: it trains, it is causal, and the
memory layer's parameters all receive gradient (the model-level checks of
`lm/tests/test_mamba4.py:347-402`)."""

import pytest
import torch

from mamba4_b200.model import Mamba4Config, Mamba4LM
from mamba4_b200.train import DataParallelTrainer, TrainSettings

pytestmark = pytest.mark.gpu

TINY = Mamba4Config(vocab_size=97, d_model=128, layer_pattern="SMSM")


def test_lm_step_reduces_loss_on_a_learnable_sequence():
    torch.manual_seed(0)
    model = Mamba4LM(TINY).cuda()
    trainer = DataParallelTrainer(model, TrainSettings(learning_rate=3e-3, warmup_steps=2, total_steps=200))
    ids = (torch.arange(4 * 129, device="cuda").reshape(4, 129) * 7) % TINY.vocab_size
    tokens, targets = ids[:, :-1].contiguous(), ids[:, 1:].contiguous()
    mask = torch.ones_like(tokens, dtype=torch.float32)
    losses = []
    for _ in range(40):
        loss, count, norm = trainer.step(tokens, targets, mask)
        losses.append(float(loss))
        assert torch.isfinite(norm)
    assert count.item() == tokens.numel()
    assert losses[-1] < 0.5 * losses[0], losses


def test_lm_is_causal_and_gradients_reach_memory_parameters():
    torch.manual_seed(1)
    model = Mamba4LM(TINY).cuda()
    tokens = (torch.arange(80, device="cuda")[None] * 7) % TINY.vocab_size
    with torch.autocast("cuda", dtype=torch.bfloat16):
        logits = model(tokens)
        changed = tokens.clone()
        changed[:, 50:] = 3
        logits2 = model(changed)
    torch.testing.assert_close(logits[:, :50], logits2[:, :50], rtol=0, atol=1e-4)
    assert (logits[:, 60:] - logits2[:, 60:]).abs().max() > 1e-3
    with torch.autocast("cuda", dtype=torch.bfloat16):
        loss = torch.nn.functional.cross_entropy(model(tokens)[0, :-1].float(), tokens[0, 1:])
    loss.backward()
    memory = model.blocks[1].mixer
    for name in ("floor", "a_log", "dt_bias", "beta_bias", "conv_weight", "D", "confidence_scale",
                 "order_mix"):
        grad = getattr(memory, name).grad
        assert grad is not None and torch.isfinite(grad).all() and grad.norm() > 1e-9, name
    for p in model.parameters():
        assert p.grad is not None and torch.isfinite(p.grad).all()


def test_cached_decode_matches_prefill_logits():
    """Token-by-token cached decode (`Mamba4LM.decode_step`, the reference's
    `decode_step`, lm/models/mamba4.py:507-560) reproduces the prefill
    logits (lm/tests/test_mamba4.py:407-419). The prefill scan rounds its
    chunk products to bfloat16 where the one-token step does not, so the bar
    is a bfloat16-level relative error rather than the reference's float32
    2e-5."""
    torch.manual_seed(3)
    model = Mamba4LM(TINY).cuda().eval()
    tokens = (torch.arange(2 * 11, device="cuda").reshape(2, 11) * 5) % TINY.vocab_size
    with torch.no_grad(), torch.autocast("cuda", dtype=torch.bfloat16):
        logits = model(tokens)
        cache = model.init_cache(2, device="cuda")
        steps = []
        for i in range(tokens.shape[1]):
            out, cache = model.decode_step(tokens[:, i], cache)
            steps.append(out)
    decoded = torch.stack(steps, 1)
    err = (decoded - logits).norm() / logits.norm()
    assert err < 2e-2, float(err)
    assert (decoded - logits).abs().max() < 0.05 * logits.abs().max()
    assert (decoded.argmax(-1) == logits.argmax(-1)).float().mean() > 0.9


def test_graphed_decode_matches_eager_decode():
    """The CUDA-graph decoder replays exactly the eager decode's kernels:
    logits and cache agree bit for bit over a sequence, and reset() returns
    to the empty cache."""
    from mamba4_b200.model import GraphedDecoder, _cache_tensors

    torch.manual_seed(5)
    model = Mamba4LM(TINY).cuda().eval()
    tokens = (torch.arange(3 * 9, device="cuda").reshape(3, 9) * 7) % TINY.vocab_size
    dec = GraphedDecoder(model, 3)
    for _ in range(2):
        cache = model.init_cache(3, device="cuda")
        for i in range(tokens.shape[1]):
            with torch.no_grad(), torch.autocast("cuda", dtype=torch.bfloat16):
                ref, cache = model.decode_step(tokens[:, i], cache)
            got = dec.step(tokens[:, i])
            assert torch.equal(got, ref), i
        for a, b in zip(_cache_tensors(dec.cache), _cache_tensors(cache)):
            assert torch.equal(a, b)
        dec.reset()
    # The graph's bf16 weight copies follow the model after refresh_weights().
    with torch.no_grad():
        for p in model.parameters():
            p.mul_(1.01)
    dec.refresh_weights()
    cache = model.init_cache(3, device="cuda")
    for i in range(3):
        with torch.no_grad(), torch.autocast("cuda", dtype=torch.bfloat16):
            ref, cache = model.decode_step(tokens[:, i], cache)
        assert torch.equal(dec.step(tokens[:, i]), ref), i


@pytest.mark.parametrize("policy", ["full", "kernels", "mixers", "mixers-1"])
def test_remat_policies_reproduce_the_gradients(policy, monkeypatch):
    """Every rematerialization policy of the reference (`remat_block`,
    lm/models/common.py:97-122) gives the loss and gradients of the model
    without remat (the recomputed forward is deterministic); "kernels"
    recomputes the blocks without relaunching the scan."""
    import dataclasses

    from mamba4_b200 import flashmamba

    torch.manual_seed(3)
    base = Mamba4LM(TINY).cuda()
    model = Mamba4LM(dataclasses.replace(TINY, remat=True, remat_policy=policy)).cuda()
    model.load_state_dict(base.state_dict())
    ids = (torch.arange(2 * 201, device="cuda").reshape(2, 201) * 5) % TINY.vocab_size
    tokens, targets = ids[:, :-1].contiguous(), ids[:, 1:].contiguous()
    calls = [0]
    inner = flashmamba._scan_forward

    def counted(*args):
        calls[0] += 1
        return inner(*args)

    monkeypatch.setattr(flashmamba, "_scan_forward", counted)
    results = []
    for m in (base, model):
        calls[0] = 0
        with torch.autocast("cuda", dtype=torch.bfloat16):
            loss = m(tokens, targets).sum()
        loss.backward()
        results.append((loss.detach(), [p.grad.clone() for p in m.parameters()], calls[0]))
    (l0, g0, n0), (l1, g1, n1) = results
    torch.testing.assert_close(l1, l0, rtol=0, atol=0)
    for a, b in zip(g1, g0):
        torch.testing.assert_close(a, b, rtol=1e-6, atol=1e-7)
    scans = TINY.layer_pattern.count("S")
    assert n0 == scans
    expected = {"full": 2 * scans, "kernels": scans, "mixers": 2 * scans, "mixers-1": scans + 1}[policy]
    assert n1 == expected
