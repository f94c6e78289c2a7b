"""Rematerialization policies of the reference's `remat_block`
(`lm/models/common.py:97-122`), on `torch.utils.checkpoint`.

* ``"full"``: every block is recomputed in the backward pass.
* ``"kernels"``: every block is recomputed except the library operators'
  results: the memory read's outputs and stored factors (the reference's
  ``"memory_solve"`` checkpoint name) and the scan's outputs and residuals
  (``"ssd_scan"``) are kept from the forward and replayed, not relaunched.
* ``"mixers"``: every non-memory block is recomputed; memory blocks keep all
  their activations (including the stored factors their backward reuses).
* ``"mixers-N"``: only the first N non-memory blocks are recomputed.

Unknown names raise the reference's ``ValueError``.
"""

from __future__ import annotations

import threading
from contextlib import contextmanager

from torch.utils.checkpoint import checkpoint

_local = threading.local()


def block_modes(layer_pattern: str, policy: str) -> list:
    """Per block of `layer_pattern` ("M" = memory block): None (kept),
    "full" (recomputed) or "kernels" (recomputed, operator results kept),
    as `remat_block` decides (`lm/models/common.py:109-122`)."""
    modes, position = [], 0
    for kind in layer_pattern:
        memory = kind == "M"
        if policy == "full":
            mode = "full"
        elif policy == "kernels":
            mode = "kernels"
        elif policy.startswith("mixers"):
            _, _, count = policy.partition("-")
            mode = None if memory or (count and position >= int(count)) else "full"
        else:
            raise ValueError(f"Unknown remat_policy: {policy}")
        modes.append(mode)
        position += not memory
    return modes


class _KernelStore:
    """Results of the library operators called inside one rematerialized
    block: recorded in order on the block's forward, returned in the same
    order when the backward recomputes the block."""

    def __init__(self):
        self.items = []
        self.replay = False
        self.pos = 0


@contextmanager
def _active(store):
    prev = getattr(_local, "store", None)
    _local.store = store
    try:
        yield
    finally:
        _local.store = prev


def operator_results(compute):
    """`compute()` (a tuple of tensors: an operator's outputs and residuals),
    or, while a ``"kernels"`` block is being recomputed, the tuple that call
    produced on the block's forward (outputs detached, so the recomputed
    graph gets its own nodes)."""
    store = getattr(_local, "store", None)
    if store is None:
        return compute()
    if store.replay:
        item = store.items[store.pos]
        store.pos += 1
        return tuple(t.detach() if t is not None else None for t in item)
    item = compute()
    store.items.append(item)
    return item


def run_block(block, x, mode):
    """`block(x)` under a mode of `block_modes`."""
    if mode is None:
        return block(x)
    if mode == "full":
        return checkpoint(block, x, use_reentrant=False)
    store = _KernelStore()
    calls = [0]

    def run(inp):
        store.replay = calls[0] > 0
        store.pos = 0
        calls[0] += 1
        with _active(store):
            return block(inp)

    return checkpoint(run, x, use_reentrant=False)
