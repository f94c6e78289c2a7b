"""Rematerialization policies (`remat_block`, lm/models/common.py:97-122):
which blocks each policy name recomputes, and the record/replay of operator
results under "kernels" (CPU; the GPU test runs the LM under every policy)."""

import pytest
import torch

from mamba4_b200.remat import block_modes, operator_results, run_block


def test_policy_names_select_blocks_as_the_reference():
    # lm/configs/mamba4-125m.json: "remat_policy": "mixers-3" on this pattern.
    pattern = "SSSMSSSSMSSSSMSSSSMSS"
    modes = block_modes(pattern, "mixers-3")
    assert modes[:3] == ["full"] * 3 and all(m is None for m in modes[3:])
    # "mixers": every non-memory block, no memory block.
    assert block_modes("SSSM" * 2, "mixers") == ["full", "full", "full", None] * 2
    # position counts non-memory blocks only.
    assert block_modes("SMSMS", "mixers-2") == ["full", None, "full", None, None]
    assert block_modes("SMS", "full") == ["full"] * 3
    assert block_modes("SMS", "kernels") == ["kernels"] * 3
    with pytest.raises(ValueError, match="Unknown remat_policy: other"):
        block_modes("SM", "other")


class _Block(torch.nn.Module):
    """A block whose middle step stands for a library operator: an autograd
    function that counts its launches and goes through operator_results."""

    launches = 0

    class _Op(torch.autograd.Function):
        @staticmethod
        def forward(ctx, x):
            def launch():
                _Block.launches += 1
                return (torch.tanh(x), torch.cosh(x))  # output and a "residual"
            y, resid = operator_results(launch)
            ctx.save_for_backward(resid)
            return y

        @staticmethod
        def backward(ctx, g):
            (resid,) = ctx.saved_tensors
            return g / resid ** 2

    def __init__(self):
        super().__init__()
        self.lin = torch.nn.Linear(8, 8)

    def forward(self, x):
        return x + self.lin(self._Op.apply(self.lin(x)))


@pytest.mark.parametrize("mode, launches", [(None, 1), ("full", 2), ("kernels", 1)])
def test_kernels_mode_replays_operator_results(mode, launches):
    torch.manual_seed(0)
    block = _Block()
    x = torch.randn(4, 8, requires_grad=True)
    ref = torch.autograd.grad(block(x).square().sum(), [x, *block.parameters()])
    _Block.launches = 0
    out = run_block(block, x, mode)
    grads = torch.autograd.grad(out.square().sum(), [x, *block.parameters()])
    assert _Block.launches == launches
    for a, b in zip(grads, ref):
        torch.testing.assert_close(a, b, rtol=0, atol=0)
