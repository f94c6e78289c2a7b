"""Generate the golden vectors that pin the CPU oracle to the reference.

Run with MAMBA4_REFERENCE set to a checkout of the reference tree
(tasmaikeni13/mamba4):

    MAMBA4_REFERENCE=<reference checkout> python tests/golden/make_golden.py

It imports the reference's own NumPy operator code, which runs without JAX:
`analysis/memory.py` (EvidenceState.write/read/confidence, mamba3_core) and
`analysis/gradients.py` (terminal_stream_vjp), and writes small .npz fixtures
beside this script. Tests compare the oracle (and through it the CUDA path)
against these files; nothing at test or bench time reads the reference tree.
"""

import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def _reference():
    root = os.environ.get("MAMBA4_REFERENCE")
    if not root:
        raise SystemExit("set MAMBA4_REFERENCE to the reference checkout (tasmaikeni13/mamba4)")
    sys.path.insert(0, root)
    from analysis.gradients import terminal_stream_vjp
    from analysis.memory import EvidenceState, mamba3_core

    return EvidenceState, terminal_stream_vjp, mamba3_core


def memory_reads(EvidenceState):
    """Per-token exact reads of one head with an isotropic floor (ridge)."""
    rng = np.random.default_rng(101)
    time, dim, value_dim, ridge = 12, 6, 5, 0.3
    keys = rng.normal(size=(time, dim))
    keys /= np.linalg.norm(keys, axis=-1, keepdims=True)
    queries = rng.normal(size=(time, dim))
    queries /= np.linalg.norm(queries, axis=-1, keepdims=True)
    values = rng.normal(size=(time, value_dim))
    beta = rng.uniform(0.05, 1.0, time)
    decay = rng.uniform(0.3, 0.999, time)
    state = EvidenceState.zeros(dim, value_dim)
    reads, confidences = [], []
    for t in range(time):
        state.write(keys[t], values[t], beta[t], decay[t])
        reads.append(state.read(queries[t], ridge)[0])
        confidences.append(state.confidence(queries[t], ridge)[0])
    np.savez(
        HERE / "memory_reads.npz",
        keys=keys, values=values, queries=queries, beta=beta, decay=decay,
        ridge=ridge, reads=np.array(reads), confidences=np.array(confidences),
        evidence=state.s, cross=state.c,
    )


def memory_terminal_vjp(terminal_stream_vjp):
    """Analytic gradients of a terminal read (upstream . read(query))."""
    rng = np.random.default_rng(102)
    time, dim, value_dim, ridge = 9, 5, 3, 0.2
    keys = rng.normal(size=(time, dim))
    values = rng.normal(size=(time, value_dim))
    beta = rng.uniform(0.2, 2.0, time)
    decay = rng.uniform(0.5, 0.95, time)
    query = rng.normal(size=dim)
    upstream = rng.normal(size=value_dim)
    grads = terminal_stream_vjp(keys, values, beta, decay, query, upstream, ridge)
    np.savez(
        HERE / "memory_terminal_vjp.npz",
        keys=keys, values=values, beta=beta, decay=decay, query=query,
        upstream=upstream, ridge=ridge,
        **{f"grad_{name}": value for name, value in grads.items()},
    )


def mamba3_reads(mamba3_core):
    """Per-token reads of the local-frame Mamba-3 SISO recurrence."""
    rng = np.random.default_rng(103)
    time, state_dim, value_dim = 10, 8, 3
    b = rng.normal(size=(time, state_dim, 1))
    x = rng.normal(size=(time, value_dim, 1))
    q = rng.normal(size=(time, state_dim, 1))
    dt = rng.uniform(0.1, 1.0, time)
    real_a = -rng.uniform(0.05, 1.5, time)
    rates = rng.normal(size=(time, state_dim // 2))
    trap = rng.uniform(0.2, 0.8, time)
    reads = []
    for t in range(1, time + 1):
        # angles passed to mamba3_core are already dt-integrated increments
        out, final = mamba3_core(
            b[:t], x[:t], q[t - 1 : t], dt[:t], real_a[:t],
            rates[:t] * dt[:t, None], trap[:t],
        )
        reads.append(out[0, :, 0])
    np.savez(
        HERE / "mamba3_reads.npz",
        b=b[..., 0], x=x[..., 0], q=q[..., 0], dt=dt, real_a=real_a,
        rates=rates, trap=trap, reads=np.array(reads), final=final,
    )


def main():
    EvidenceState, terminal_stream_vjp, mamba3_core = _reference()
    memory_reads(EvidenceState)
    memory_terminal_vjp(terminal_stream_vjp)
    mamba3_reads(mamba3_core)
    print("wrote", sorted(p.name for p in HERE.glob("*.npz")))


if __name__ == "__main__":
    main()
