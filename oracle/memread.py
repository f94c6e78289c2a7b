"""Float64 CPU restatement of the selective conjugate memory read (oracle).

TEST INFRASTRUCTURE ONLY (see `oracle/__init__.py`): never imported by the
product package.

Operator contract (reference `lm/kernels/mamba4.py:228-338`, fused variant
`lm/kernels/mamba4_fused.py:372-454`): keys/queries [B,T,H,D], values
[B,T,H,P], beta and log_decay [B,T,H], floor [H,D], optional initial state
(evidence [B,H,D,D], cross [B,H,P,D]). Per head, with lam_t = exp(log_decay_t),

    S_t = lam_t S_(t-1) + beta_t k_t k_t^T,   C_t = lam_t C_(t-1) + beta_t v_t k_t^T,
    A_t = S_t + diag(floor),   y_t = A_t^-1 q_t,
    output_t = C_t y_t,   variance_t = q_t^T y_t,

and the final state is (S_(T-1), C_(T-1)).

`dense_forward` follows the sequential oracle `lm/kernels/mamba4_reference.py:6-32`.
`dense_backward` is the exact reverse recurrence of that forward: the
generalisation to every token of `analysis/gradients.py:9-36`
(`terminal_stream_vjp`) with the solve derivative of `lm/kernels/mamba4.py:208-215`
(z = A^-1 g, dA = -z y^T, d rhs = z). `chunked_forward` / `chunked_backward`
restate the chunked algebra of `lm/kernels/mamba4_fused.py:372-454` and
`:340-366` extended to every input (the part the reference leaves to JAX
autodiff); they are the formulas the CUDA kernels implement and are checked
here against the dense recurrence.
"""

from __future__ import annotations

import numpy as np

F64 = np.float64


def _prepare(keys, values, queries, beta, log_decay, floor, initial):
    k, v, q = (np.asarray(a, F64) for a in (keys, values, queries))
    batch, time, heads, dim = k.shape
    value_dim = v.shape[-1]
    if q.shape != k.shape or v.shape[:3] != k.shape[:3]:
        # Same check and message as lm/kernels/mamba4.py:268-269.
        raise ValueError("Selective memory keys, values and queries disagree")
    shape = (batch, time, heads)
    b = np.broadcast_to(np.asarray(beta, F64), shape)
    g = np.broadcast_to(np.asarray(log_decay, F64), shape)
    f = np.broadcast_to(np.asarray(floor, F64), (heads, dim))
    if initial is None:
        s0 = np.zeros((batch, heads, dim, dim))
        c0 = np.zeros((batch, heads, value_dim, dim))
    else:
        s0 = np.asarray(initial[0], F64)
        c0 = np.asarray(initial[1], F64)
    return k, v, q, b, g, f, s0, c0


def dense_forward(keys, values, queries, beta, log_decay, floor, initial=None):
    """Sequential fixed-floor recurrence with dense solves, float64.

    Follows `lm/kernels/mamba4_reference.py:6-32` with decay = exp(log_decay)
    and an optional initial state (`lm/kernels/mamba4.py:274-278`).
    Returns a dict with output, variance, evidence, cross and solved (y).
    """
    k, v, q, b, g, f, s, c = _prepare(
        keys, values, queries, beta, log_decay, floor, initial
    )
    batch, time, heads, dim = k.shape
    eye = np.eye(dim)
    lam = np.exp(g)
    outputs, variances, solved = [], [], []
    for t in range(time):
        kt, vt, qt = k[:, t], v[:, t], q[:, t]
        s = lam[:, t, :, None, None] * s + b[:, t, :, None, None] * (
            kt[..., :, None] * kt[..., None, :]
        )
        c = lam[:, t, :, None, None] * c + b[:, t, :, None, None] * (
            vt[..., :, None] * kt[..., None, :]
        )
        precision = s + f[None, :, :, None] * eye
        y = np.linalg.solve(precision, qt[..., None])[..., 0]
        solved.append(y)
        outputs.append(np.einsum("bhpd,bhd->bhp", c, y))
        variances.append(np.sum(qt * y, axis=-1))
    return dict(
        output=np.stack(outputs, 1),
        variance=np.stack(variances, 1),
        evidence=s,
        cross=c,
        solved=np.stack(solved, 1),
    )


def dense_backward(
    keys,
    values,
    queries,
    beta,
    log_decay,
    floor,
    initial,
    d_output,
    d_variance,
    d_evidence=None,
    d_cross=None,
):
    """Exact reverse-mode gradients of `dense_forward`, float64.

    Reverse recurrence over the adjoint statistics (S_bar, C_bar), as
    `analysis/gradients.py:19-36` does for a terminal read, applied to a read
    at every token. Per token (descending t):
        g_t = C_t^T d_out_t + d_var_t q_t,  z_t = A_t^-1 g_t,
        d q_t = z_t + d_var_t y_t,  S_bar += -z_t y_t^T,  C_bar += d_out_t y_t^T,
        d k_t = beta_t ((S_bar + S_bar^T) k_t + C_bar^T v_t),
        d v_t = beta_t C_bar k_t,  d beta_t = k^T S_bar k + v^T C_bar k,
        d log_decay_t = lam_t (<S_bar, S_(t-1)> + <C_bar, C_(t-1)>),
        then S_bar, C_bar *= lam_t.
    d floor = -sum_t z_t * y_t. Returns a dict keyed like the inputs plus
    `evidence0` / `cross0` (gradient of the initial state).
    """
    k, v, q, b, g, f, s_init, c_init = _prepare(
        keys, values, queries, beta, log_decay, floor, initial
    )
    batch, time, heads, dim = k.shape
    eye = np.eye(dim)
    lam = np.exp(g)
    d_out = np.asarray(d_output, F64)
    d_var = np.asarray(d_variance, F64)
    # Forward states S_t, C_t for every t, and S_(-1), C_(-1).
    states_s, states_c = [s_init], [c_init]
    s, c = s_init, c_init
    for t in range(time):
        kt, vt = k[:, t], v[:, t]
        s = lam[:, t, :, None, None] * s + b[:, t, :, None, None] * (
            kt[..., :, None] * kt[..., None, :]
        )
        c = lam[:, t, :, None, None] * c + b[:, t, :, None, None] * (
            vt[..., :, None] * kt[..., None, :]
        )
        states_s.append(s)
        states_c.append(c)
    s_bar = (
        np.zeros_like(s) if d_evidence is None else np.asarray(d_evidence, F64).copy()
    )
    c_bar = np.zeros_like(c) if d_cross is None else np.asarray(d_cross, F64).copy()
    grads = {
        name: np.zeros(shape)
        for name, shape in (
            ("keys", k.shape),
            ("values", v.shape),
            ("queries", q.shape),
            ("beta", b.shape),
            ("log_decay", g.shape),
        )
    }
    d_floor = np.zeros((heads, dim))
    for t in range(time - 1, -1, -1):
        kt, vt, qt = k[:, t], v[:, t], q[:, t]
        s_t, c_t = states_s[t + 1], states_c[t + 1]
        precision = s_t + f[None, :, :, None] * eye
        y = np.linalg.solve(precision, qt[..., None])[..., 0]
        rhs = np.einsum("bhpd,bhp->bhd", c_t, d_out[:, t]) + d_var[:, t, :, None] * qt
        z = np.linalg.solve(precision, rhs[..., None])[..., 0]
        grads["queries"][:, t] = z + d_var[:, t, :, None] * y
        s_bar = s_bar - z[..., :, None] * y[..., None, :]
        c_bar = c_bar + d_out[:, t][..., :, None] * y[..., None, :]
        d_floor -= np.sum(z * y, axis=0)
        bt = b[:, t, :, None]
        sym = s_bar + np.swapaxes(s_bar, -1, -2)
        grads["keys"][:, t] = bt * (
            np.einsum("bhde,bhe->bhd", sym, kt) + np.einsum("bhpd,bhp->bhd", c_bar, vt)
        )
        grads["values"][:, t] = bt * np.einsum("bhpd,bhd->bhp", c_bar, kt)
        grads["beta"][:, t] = np.einsum("bhd,bhde,bhe->bh", kt, s_bar, kt) + np.einsum(
            "bhp,bhpd,bhd->bh", vt, c_bar, kt
        )
        d_lam = np.sum(s_bar * states_s[t], axis=(-1, -2)) + np.sum(
            c_bar * states_c[t], axis=(-1, -2)
        )
        grads["log_decay"][:, t] = lam[:, t] * d_lam
        s_bar = lam[:, t, :, None, None] * s_bar
        c_bar = lam[:, t, :, None, None] * c_bar
    grads["floor"] = d_floor
    grads["evidence0"] = s_bar
    grads["cross0"] = c_bar
    return grads


def _chunks(x, chunk, padding):
    """[B,T,...] -> [B,n,c,...] padded with zeros (writes nothing, no decay)."""
    x = np.pad(x, [(0, 0), (0, padding)] + [(0, 0)] * (x.ndim - 2))
    return x.reshape(x.shape[0], -1, chunk, *x.shape[2:])


def chunked_forward(
    keys, values, queries, beta, log_decay, floor, initial=None, chunk_size=64
):
    """Chunked exact reads, float64 restatement of `mamba4_fused.py:372-454`.

    Per chunk: P = inclusive prefix of log_decay, W[t,s] = beta_s e^(P_t-P_s)
    (s <= t), A_t = e^(P_t) S0 + sum_s W[t,s] k_s k_s^T + diag(floor), reads
    output_t = e^(P_t) C0 y_t + sum_s W[t,s] (k_s . y_t) v_s. Chunk-start
    states come from the decayed carry of `lm/kernels/prefix.py:27-44`.
    Returns the dense_forward dict plus per-chunk starts (s0, c0).
    """
    k, v, q, b, g, f, s, c = _prepare(
        keys, values, queries, beta, log_decay, floor, initial
    )
    batch, time, heads, dim = k.shape
    padding = (-time) % chunk_size
    kc, vc, qc = (_chunks(a, chunk_size, padding) for a in (k, v, q))
    bc, gc = (_chunks(a, chunk_size, padding) for a in (b, g))
    count = kc.shape[1]
    prefix = np.cumsum(gc, axis=2)  # [B,n,c,H]
    causal = np.tril(np.ones((chunk_size, chunk_size), bool))
    diff = prefix[:, :, :, None, :] - prefix[:, :, None, :, :]  # [B,n,t,s,H]
    decay = np.where(causal[None, None, :, :, None], np.exp(np.where(
        causal[None, None, :, :, None], diff, 0.0)), 0.0)
    weights = decay * bc[:, :, None, :, :]
    tail = bc * np.exp(prefix[:, :, -1:, :] - prefix)  # [B,n,c,H]
    end = np.exp(prefix[:, :, -1, :])  # [B,n,H]
    starts_s, starts_c = [], []
    for n in range(count):
        starts_s.append(s)
        starts_c.append(c)
        s = end[:, n, :, None, None] * s + np.einsum(
            "bsh,bshd,bshe->bhde", tail[:, n], kc[:, n], kc[:, n]
        )
        c = end[:, n, :, None, None] * c + np.einsum(
            "bsh,bshp,bshd->bhpd", tail[:, n], vc[:, n], kc[:, n]
        )
    s0 = np.stack(starts_s, 1)  # [B,n,H,D,D]
    c0 = np.stack(starts_c, 1)
    eye = np.eye(dim)
    carried = np.exp(prefix)  # [B,n,c,H]
    precision = (
        carried[..., None, None] * s0[:, :, None]
        + np.einsum("bntsh,bnshd,bnshe->bnthde", weights, kc, kc)
        + f[None, None, None, :, :, None] * eye
    )
    y = np.linalg.solve(precision, qc[..., None])[..., 0]  # [B,n,c,H,D]
    scores = np.einsum("bnthd,bnshd->bntsh", y, kc)
    within = np.einsum("bntsh,bnshp->bnthp", scores * weights, vc)
    inherited = np.einsum("bnthd,bnhpd->bnthp", y, c0)
    output = within + carried[..., None] * inherited
    variance = np.sum(qc * y, axis=-1)

    def unchunk(x):
        return x.reshape(batch, count * chunk_size, *x.shape[3:])[:, :time]

    return dict(
        output=unchunk(output),
        variance=unchunk(variance),
        evidence=s,
        cross=c,
        solved=unchunk(y),
        s0=s0,
        c0=c0,
    )


def chunked_backward(
    keys,
    values,
    queries,
    beta,
    log_decay,
    floor,
    initial,
    d_output,
    d_variance,
    d_evidence=None,
    d_cross=None,
    chunk_size=64,
):
    """Chunk-form gradients of every input (the algebra of the CUDA backward).

    Extends `_chunk_solve_backward` (`lm/kernels/mamba4_fused.py:340-366`),
    which covers the solve, to the chunk reads and the chunk-start carry that
    the reference differentiates with JAX autodiff (`:410-447`). Per chunk,
    with GY = Y K^T, GZ = Z K^T, OV = dO V^T (all [t,s]) and the end weights
    w_s = beta_s e^(P_L - P_s):
        g_t  = e^(P_t) C0^T dO_t + ((W o OV) K)_t + dvar_t q_t,  z_t = A_t^-1 g_t
        dS0  = -sum_t e^(P_t) z_t y_t^T + e^(P_L) dS_end      (carried backwards)
        dC0  =  sum_t e^(P_t) dO_t y_t^T + e^(P_L) dC_end
        dK   = -(W o GY)^T Z - (W o GZ)^T Y + (W o OV)^T Y
               + diag(w) (K (dS_end + dS_end^T) + V dC_end)
        dV   = (W o GY)^T dO + diag(w) K dC_end^T
        dW   = GY o (OV - GZ) (s <= t),  dw_s = k^T dS_end k + v^T dC_end k
        dbeta_s = sum_t dW[t,s] e^(P_t-P_s) + dw_s e^(P_L-P_s)
        dP_t = sum_s dW W [t,.] - sum_t' dW W [.,t] - dw_t w_t
               + e^(P_t) (-z_t^T S0 y_t + dO_t^T C0 y_t)
               + [t = L] (sum_s dw_s w_s + e^(P_L) (<dS_end,S0> + <dC_end,C0>))
        dlog_decay = reverse cumulative sum of dP within the chunk
        dq_t = z_t + dvar_t y_t,  dfloor = -sum_t z_t o y_t.
    """
    k, v, q, b, g, f, s_init, c_init = _prepare(
        keys, values, queries, beta, log_decay, floor, initial
    )
    batch, time, heads, dim = k.shape
    fwd = chunked_forward(k, v, q, b, g, f, (s_init, c_init), chunk_size)
    padding = (-time) % chunk_size
    kc, vc, qc = (_chunks(a, chunk_size, padding) for a in (k, v, q))
    bc, gc = (_chunks(a, chunk_size, padding) for a in (b, g))
    yc = _chunks(fwd["solved"], chunk_size, padding)
    doc = _chunks(np.asarray(d_output, F64), chunk_size, padding)
    dvc = _chunks(np.asarray(d_variance, F64), chunk_size, padding)
    s0, c0 = fwd["s0"], fwd["c0"]
    count = kc.shape[1]
    prefix = np.cumsum(gc, axis=2)
    causal = np.tril(np.ones((chunk_size, chunk_size), bool))
    diff = prefix[:, :, :, None, :] - prefix[:, :, None, :, :]
    decay = np.where(causal[None, None, :, :, None], np.exp(np.where(
        causal[None, None, :, :, None], diff, 0.0)), 0.0)
    weights = decay * bc[:, :, None, :, :]  # [B,n,t,s,H]
    carried = np.exp(prefix)  # [B,n,c,H]
    tail = np.exp(prefix[:, :, -1:, :] - prefix)
    end_w = bc * tail  # w_s
    end = np.exp(prefix[:, :, -1, :])
    eye = np.eye(dim)
    ov = np.einsum("bnthp,bnshp->bntsh", doc, vc)
    rhs = (
        carried[..., None] * np.einsum("bnhpd,bnthp->bnthd", c0, doc)
        + np.einsum("bntsh,bnshd->bnthd", weights * ov, kc)
        + dvc[..., None] * qc
    )
    precision = (
        carried[..., None, None] * s0[:, :, None]
        + np.einsum("bntsh,bnshd,bnshe->bnthde", weights, kc, kc)
        + f[None, None, None, :, :, None] * eye
    )
    z = np.linalg.solve(precision, rhs[..., None])[..., 0]
    # Local adjoint summaries and the reverse carry over chunks.
    x_s = -np.einsum("bnth,bnthd,bnthe->bnhde", carried, z, yc)
    x_c = np.einsum("bnth,bnthp,bnthd->bnhpd", carried, doc, yc)
    s_end = np.zeros((batch, count, heads, dim, dim))
    c_end = np.zeros((batch, count, heads, v.shape[-1], dim))
    s_bar = (
        np.zeros((batch, heads, dim, dim))
        if d_evidence is None
        else np.asarray(d_evidence, F64)
    )
    c_bar = (
        np.zeros((batch, heads, v.shape[-1], dim))
        if d_cross is None
        else np.asarray(d_cross, F64)
    )
    for n in range(count - 1, -1, -1):
        s_end[:, n], c_end[:, n] = s_bar, c_bar
        s_bar = x_s[:, n] + end[:, n, :, None, None] * s_bar
        c_bar = x_c[:, n] + end[:, n, :, None, None] * c_bar
    gy = np.einsum("bnthd,bnshd->bntsh", yc, kc)
    gz = np.einsum("bnthd,bnshd->bntsh", z, kc)
    sym_end = s_end + np.swapaxes(s_end, -1, -2)
    dk = (
        -np.einsum("bntsh,bnthd->bnshd", weights * gy, z)
        - np.einsum("bntsh,bnthd->bnshd", weights * gz, yc)
        + np.einsum("bntsh,bnthd->bnshd", weights * ov, yc)
        + end_w[..., None]
        * (
            np.einsum("bnhde,bnshe->bnshd", sym_end, kc)
            + np.einsum("bnhpd,bnshp->bnshd", c_end, vc)
        )
    )
    dv = np.einsum("bntsh,bnthp->bnshp", weights * gy, doc) + end_w[
        ..., None
    ] * np.einsum("bnhpd,bnshd->bnshp", c_end, kc)
    dw = np.where(causal[None, None, :, :, None], gy * (ov - gz), 0.0)
    dw_end = np.einsum("bnshd,bnhde,bnshe->bnsh", kc, s_end, kc) + np.einsum(
        "bnshp,bnhpd,bnshd->bnsh", vc, c_end, kc
    )
    dbeta = np.sum(dw * decay, axis=2) + dw_end * tail
    weighted = dw * weights
    s0y = np.einsum("bnhde,bnthe->bnthd", s0, yc)
    c0y = np.einsum("bnhpd,bnthd->bnthp", c0, yc)
    dp = (
        np.sum(weighted, axis=3)
        - np.sum(weighted, axis=2)
        - dw_end * end_w
        + carried * (-np.sum(z * s0y, -1) + np.sum(doc * c0y, -1))
    )
    last = np.sum(dw_end * end_w, axis=2) + end * (
        np.sum(s_end * s0, axis=(-1, -2)) + np.sum(c_end * c0, axis=(-1, -2))
    )
    dp[:, :, -1] += last
    dg = np.cumsum(dp[:, :, ::-1], axis=2)[:, :, ::-1]
    dq = z + dvc[..., None] * yc
    dfloor = -np.sum(z * yc, axis=(0, 1, 2))

    def unchunk(x):
        return x.reshape(batch, count * chunk_size, *x.shape[3:])[:, :time]

    return dict(
        keys=unchunk(dk),
        values=unchunk(dv),
        queries=unchunk(dq),
        beta=unchunk(dbeta),
        log_decay=unchunk(dg),
        floor=dfloor,
        evidence0=s_bar,
        cross0=c_bar,
    )


def decode_step(evidence, cross, key, value, query, beta, log_decay, floor):
    """One exact write/read against a carried state, float64.

    Follows `selective_decode` (`lm/kernels/mamba4.py:341-355`): evidence
    [B,H,D,D], cross [B,H,P,D], key/query [B,H,D], value [B,H,P], beta and
    log_decay [B,H], floor [H,D]. Returns (output [B,H,P], variance [B,H],
    evidence', cross').
    """
    s, c = np.asarray(evidence, F64), np.asarray(cross, F64)
    k, v, q = (np.asarray(a, F64) for a in (key, value, query))
    lam = np.exp(np.asarray(log_decay, F64))[..., None, None]
    b = np.asarray(beta, F64)[..., None, None]
    s = lam * s + b * (k[..., :, None] * k[..., None, :])
    c = lam * c + b * (v[..., :, None] * k[..., None, :])
    dim = k.shape[-1]
    precision = s + np.asarray(floor, F64)[None, :, :, None] * np.eye(dim)
    y = np.linalg.solve(precision, q[..., None])[..., 0]
    return np.einsum("bhpd,bhd->bhp", c, y), np.sum(q * y, axis=-1), s, c


def spd_solve(precision, rhs):
    """Float64 solve of precision @ y = rhs, reading only the lower triangle.

    Restates `spd_solve` (`lm/kernels/mamba4.py:187-206`): precision
    [...,d,d] SPD, rhs [...,d]; the Cholesky backends there read the lower
    triangle only, so the matrix solved is tril(A) + tril(A, -1)^T.
    """
    a = np.asarray(precision, F64)
    a = np.tril(a) + np.swapaxes(np.tril(a, -1), -1, -2)
    return np.linalg.solve(a, np.asarray(rhs, F64)[..., None])[..., 0]


def spd_solve_vjp(precision, rhs, gradient):
    """`_spd_solve_backward` (`lm/kernels/mamba4.py:208-215`), float64:
    z = A^-1 g, d rhs = z, d precision = -(z y^T + y z^T) / 2.
    Returns (d_precision, d_rhs)."""
    y = spd_solve(precision, rhs)
    z = spd_solve(precision, gradient)
    outer = z[..., :, None] * y[..., None, :]
    return -0.5 * (outer + np.swapaxes(outer, -1, -2)), z


def config_inputs(batch, time, heads, dim, value_dim, seed=0):
    """Seeded inputs of BASELINE configs 0 and 2 (float32 arrays).

    Draw order (numpy default_rng(seed)): q, k ~ N(0,1)/8 [B,T,H,D];
    v ~ N(0,1) [B,T,H,P]; lam = sigmoid(N(2,1)); beta = sigmoid(N(0,1));
    cotangents d_out ~ N(0,1) [B,T,H,P], d_var ~ N(0,1) [B,T,H]. Keys are then
    shifted one token (each v_t is written under k_(t-1), k_(-1) = 0), as the
    model does at `lm/models/mamba4.py:183-194`. Floor 0.1, zero initial state.
    """
    rng = np.random.default_rng(seed)
    q = (rng.standard_normal((batch, time, heads, dim)) / 8).astype(np.float32)
    k = (rng.standard_normal((batch, time, heads, dim)) / 8).astype(np.float32)
    v = rng.standard_normal((batch, time, heads, value_dim)).astype(np.float32)
    lam = 1 / (1 + np.exp(-rng.normal(2.0, 1.0, (batch, time, heads))))
    beta = 1 / (1 + np.exp(-rng.standard_normal((batch, time, heads))))
    d_out = rng.standard_normal((batch, time, heads, value_dim)).astype(np.float32)
    d_var = rng.standard_normal((batch, time, heads)).astype(np.float32)
    shifted = np.concatenate((np.zeros_like(k[:, :1]), k[:, :-1]), axis=1)
    floor = np.full((heads, dim), 0.1, np.float32)
    return dict(
        keys=shifted,
        values=v,
        queries=q,
        beta=beta.astype(np.float32),
        log_decay=np.log(lam).astype(np.float32),
        floor=floor,
        d_output=d_out,
        d_variance=d_var,
    )
