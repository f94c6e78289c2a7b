"""CPU oracle for the Mamba 4 hot path.

TEST INFRASTRUCTURE ONLY. Nothing in the product package (`mamba4_b200`)
imports this package: only `tests/`, `__graft_entry__.smoke()` and the
`cpu_baseline` / `--impl reference` legs of `bench.py` use it, and only as the
checker or the timed CPU baseline.

The reference (tasmaikeni13/mamba4) is JAX/Pallas code whose runtime (jax,
jaxlib, flax, optax) is not installed here, so these modules restate its
algorithms in float64 NumPy (and float64/bfloat16 PyTorch-CPU where the
reference's bfloat16 rounding points must be reproduced). Every function cites
the reference file:line it follows. The restatements are pinned against golden
vectors produced by the reference's own importable NumPy code
(`analysis/memory.py`, `analysis/gradients.py`) and against the known-answer
tests of `lm/tests/test_mamba4.py`; see `tests/golden/make_golden.py`.
"""
