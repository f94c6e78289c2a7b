"""Fused model glue against compositions of the reference model code.

The compositions restate the reference glue (`lm/models/mamba3.py:74-117`,
`lm/models/mamba4.py:155-260`, `lm/models/common.py:25-45`) in float64 on
the CPU around the oracle operators (`oracle/glue.py`): the scan with the
reference kernels' bf16 rounding points in both directions, the memory read
in float64, the order head and causal convolution in the reference's chunked
forms. They keep the model's bf16 rounding points (norm outputs, the mixer
output). Fused outputs and every gradient must agree elementwise within a
few bf16 steps: rtol 2e-2 with an absolute floor of 2e-2 * max|expected|
(the bar of the bf16 scan tests).
"""

import pytest
import torch
import torch.nn.functional as F

from mamba4_b200.glue import mamba_mixer_core, rms_norm_bf16
from oracle import glue as G

pytestmark = pytest.mark.gpu
F64 = torch.float64
TOL = 2e-2


def close(actual, expected, name="", tol=TOL):
    """Elementwise |a - e| <= tol |e| + tol max|e|."""
    a = actual.detach().to(F64).cpu()
    e = expected.detach().to(F64).cpu()
    scale = float(e.abs().max()) or 1.0
    torch.testing.assert_close(a, e, rtol=tol, atol=tol * scale, msg=lambda m: f"{name}: {m}")


def bf16_round(x):
    """Round to bfloat16 inside a float64 composition (gradient passes through)."""
    return x.to(torch.bfloat16).to(x.dtype)


def rel(a, b):
    a, b = a.float(), b.float()
    return ((a - b).norm() / b.norm().clamp_min(1e-30)).item()


def composite_rms(x, scale, eps):
    x32 = x.float()
    return (x32 * torch.rsqrt(x32.square().mean(-1, keepdim=True) + eps) * scale).to(torch.bfloat16)


def heavy_tail(x):
    return torch.clamp(x, min=0) + torch.reciprocal(1 - torch.clamp(x, max=0))


def composite_core64(proj, bs, cs, dtb, D, qb, kb, inner, heads, angles, eps):
    """Mamba-3 mixer glue (`lm/models/mamba3.py:74-117`) in float64 around the
    rounding-point scan oracle; bf16 rounding at the B/C norms and output."""
    n = bs.shape[0]
    z, x, b, c, raw_dt, raw_a, trap, ang = torch.split(proj, (inner, inner, n, n, heads, heads, heads, angles), -1)

    def rms(v, scale):
        return bf16_round(v * torch.rsqrt(v.square().mean(-1, keepdim=True) + eps) * scale)

    b, c = rms(b, bs), rms(c, cs)
    dt = F.softplus(raw_dt + dtb)
    a = -torch.clamp(heavy_tail(raw_a), min=1e-4)
    y, _ = G.EmulatedScan.apply(c, b, x, a * dt, dt, trap, ang, qb, kb)
    y = y + x * torch.repeat_interleave(D, 64)
    return bf16_round(y * F.silu(z))


@pytest.mark.parametrize("batch,time,state", [(2, 160, 64), (1, 64, 64), (2, 100, 96), (1, 130, 128)])
def test_mixer_core_matches_composition(batch, time, state):
    torch.manual_seed(0)
    inner, heads, angles, eps = 256, 4, state // 4, 1e-5  # row width 668 at N = 64: padded to 672
    width = 2 * inner + 2 * state + 3 * heads + angles
    dev = "cuda"
    proj = torch.randn(batch, time, width, device=dev)
    proj[..., 2 * inner + 2 * state: 2 * inner + 2 * state + heads] -= 3.0  # dt around softplus(-3)
    proj = proj.to(torch.bfloat16)
    params = [torch.rand(state, device=dev) + 0.5, torch.rand(state, device=dev) + 0.5,
              torch.randn(heads, device=dev) - 2.0, torch.randn(heads, device=dev),
              torch.randn(heads, 1, state, device=dev) * 0.5 + 1.0,
              torch.randn(heads, 1, state, device=dev) * 0.5 + 1.0]
    g = torch.randn(batch, time, inner, device=dev).to(torch.bfloat16)
    p = proj.clone().requires_grad_()
    ps = [t.clone().requires_grad_() for t in params]
    out_f = mamba_mixer_core(p, *ps, inner=inner, heads=heads, angles=angles, eps=eps, state=state)
    g_f = torch.autograd.grad(out_f, [p, *ps], g)
    p64 = proj.to(F64).cpu().requires_grad_()
    ps64 = [t.to(F64).cpu().requires_grad_() for t in params]
    out_c = composite_core64(p64, *ps64, inner, heads, angles, eps)
    g_c = torch.autograd.grad(out_c, [p64, *ps64], g.to(F64).cpu())
    close(out_f, out_c, "output")
    names = ["proj", "B_norm.scale", "C_norm.scale", "dt_bias", "D", "C_bias", "B_bias"]
    for name, a, b in zip(names, g_f, g_c):
        assert torch.isfinite(a.float()).all(), name
        close(a, b, name)


@pytest.mark.parametrize("features", [512, 768])
def test_rms_norm_bf16_matches_composition(features):
    torch.manual_seed(1)
    x = (torch.randn(300, features, device="cuda") * 3).to(torch.bfloat16)
    scale = torch.rand(features, device="cuda") + 0.5
    g = torch.randn(300, features, device="cuda").to(torch.bfloat16)
    xa, sa = x.clone().requires_grad_(), scale.clone().requires_grad_()
    xb, sb = x.clone().requires_grad_(), scale.clone().requires_grad_()
    ya = rms_norm_bf16(xa, sa, 1e-5)
    yb = composite_rms(xb, sb, 1e-5)
    assert rel(ya, yb) < 4e-3
    ga = torch.autograd.grad(ya, (xa, sa), g)
    gb = torch.autograd.grad(yb, (xb, sb), g)
    assert rel(ga[0], gb[0]) < 1e-2
    assert rel(ga[1], gb[1]) < 1e-3


def composite_memory_mixer64(m, proj, p):
    """The memory mixer (`lm/models/mamba4.py:155-260`) in float64 on the CPU
    from the bf16 projection `proj` and float64 parameter copies `p`, around
    the float64 memory-read oracle; bf16 rounding at the read norm and the
    output, as the model."""
    cfg = m.cfg
    h, d, pd = cfg.memory_heads, cfg.key_dim, cfg.memory_head_dim
    batch, time, _ = proj.shape
    gate, value, key, query, beta_raw, dt_raw, order_raw = torch.split(proj, m.sizes, dim=-1)
    mixed = torch.cat((value, key, query), -1)
    mixed = F.silu(G.causal_conv(mixed, p["conv_weight"] - m.bound, p["conv_bias"]))
    value = mixed[..., : cfg.inner].reshape(batch, time, h, pd)
    key = mixed[..., cfg.inner: cfg.inner + h * d].reshape(batch, time, h, d)
    query = mixed[..., cfg.inner + h * d:].reshape(batch, time, h, d)
    key = torch.cat((torch.zeros_like(key[:, :1]), key[:, :-1]), 1)
    key, query = _unit(key), _unit(query)
    beta = cfg.memory_beta_max * torch.sigmoid(beta_raw + p["beta_bias"])
    log_decay = -torch.exp(p["a_log"]) * F.softplus(dt_raw + p["dt_bias"])
    floor = cfg.floor_min + F.softplus(p["floor"])
    output, variance = G.memory_read(key, value, query, beta, log_decay, floor)
    read = output * torch.sigmoid(1 - p["confidence_scale"] * torch.log1p(variance))[..., None]
    read = read + p["D"][:, None] * value
    ordered = G.order_memory_chunked(value, F.logsigmoid(order_raw + 2), 64)
    read = read + torch.sigmoid(p["order_mix"])[:, None] * ordered
    read = bf16_round(read * torch.rsqrt(read.square().mean(-1, keepdim=True) + cfg.norm_eps)
                      * p["read_norm.scale"])
    read = bf16_round(read * F.silu(gate.reshape(read.shape)))
    return read.reshape(batch, time, cfg.inner)


@pytest.mark.parametrize("time,d_model", [(160, 512), (64, 512), (100, 128)])
def test_memory_mixer_glue_matches_composition(time, d_model):
    from mamba4_b200.model import Mamba4Config, SelectiveMemoryMixer

    torch.manual_seed(2)
    cfg = Mamba4Config(d_model=d_model, layer_pattern="M")
    m = SelectiveMemoryMixer(cfg).cuda()
    with torch.no_grad():  # non-trivial values for the scalar parameters
        m.confidence_scale.uniform_(0.05, 0.3)
        m.D.uniform_(0.5, 1.5)
        m.order_mix.uniform_(-1.5, 0.5)
        m.read_norm.scale.uniform_(0.5, 1.5)
        m.conv_bias.uniform_(-0.1, 0.1)
    u = (torch.randn(2, time, d_model, device="cuda")).to(torch.bfloat16)
    g = torch.randn(2, time, cfg.inner, device="cuda").to(torch.bfloat16)
    m.out_proj = torch.nn.Identity()
    named = [(n, q) for n, q in m.named_parameters() if n != "in_proj.weight"]
    # Fused path, from the model's own bf16 projection (autocast in_proj).
    uu = u.clone().requires_grad_()
    with torch.autocast("cuda", dtype=torch.bfloat16):
        proj = m.in_proj(uu)
        y_f = m(uu)
    grads = torch.autograd.grad(y_f, [uu, m.in_proj.weight, *[q for _, q in named]], g)
    # float64 composition from the same bf16 projection values; the input and
    # projection-weight gradients follow by the chain rule through in_proj.
    p64 = proj.detach().to(F64).cpu().requires_grad_()
    params64 = {n: q.detach().to(F64).cpu().requires_grad_() for n, q in named}
    y_c = composite_memory_mixer64(m, p64, params64)
    g64 = torch.autograd.grad(y_c, [p64, *params64.values()], g.to(F64).cpu())
    d_proj = g64[0].reshape(-1, p64.shape[-1])
    w64 = m.in_proj.weight.detach().to(torch.bfloat16).to(F64).cpu()
    d_u = (d_proj @ w64).reshape(u.shape)
    d_w = d_proj.t() @ u.to(F64).cpu().reshape(-1, d_model)
    close(y_f, y_c, "output")
    close(grads[0], d_u, "u")
    close(grads[1], d_w, "in_proj.weight")
    for (name, _), a, b in zip(named, grads[2:], g64[1:]):
        assert a is not None and torch.isfinite(a.float()).all(), name
        close(a, b, name)


def test_head_cross_entropy_matches_composition():
    from mamba4_b200.glue import head_cross_entropy

    torch.manual_seed(3)
    rows, dim, vocab = 300, 256, 997  # not a multiple of 8: padded row stride
    x = (torch.randn(rows, dim, device="cuda")).to(torch.bfloat16)
    w = torch.randn(vocab, dim, device="cuda") * 0.05
    t = torch.randint(0, vocab, (rows,), device="cuda")
    g = torch.rand(rows, device="cuda")
    g[::7] = 0.0  # masked tokens
    xa, wa = x.clone().requires_grad_(), w.clone().requires_grad_()
    xb, wb = x.clone().requires_grad_(), w.clone().requires_grad_()
    la = head_cross_entropy(xa, wa, t)
    lb = F.cross_entropy(F.linear(xb, wb.to(torch.bfloat16)).float(), t, reduction="none")
    torch.testing.assert_close(la, lb, rtol=1e-5, atol=1e-5)
    ga = torch.autograd.grad(la, (xa, wa), g)
    gb = torch.autograd.grad(lb, (xb, wb), g)
    assert rel(ga[0], gb[0]) < 1e-2
    assert rel(ga[1], gb[1]) < 1e-2


def test_memory_mixer_shared_gradient_buffer_is_exact():
    """split_projection + GradSlab (the glue kernels write the gate / rest
    gradients straight into one projection-gradient buffer) gives bitwise the
    gradients of plain slicing (autograd assembling the projection gradient)."""
    from mamba4_b200.glue import GradSlab, memory_mixer_post, memory_mixer_prep, split_projection

    torch.manual_seed(5)
    heads, inner, batch, time = 2, 256, 2, 96
    width = inner + 259 * heads + 10  # trailing columns no kernel reads (row stride a multiple of 8)
    proj0 = (torch.randn(batch, time, width, device="cuda") * 0.5).to(torch.bfloat16)
    conv_w = torch.rand(4, 256 * heads, device="cuda")
    conv_b = torch.randn(256 * heads, device="cuda") * 0.1
    beta_bias, dt_bias, a_log = (torch.randn(heads, device="cuda") * 0.1 for _ in range(3))
    cs, D, om = torch.full((heads,), 0.1, device="cuda"), torch.ones(heads, device="cuda"), torch.zeros(heads, device="cuda")
    scale = torch.ones(128, device="cuda")
    g_vals = torch.randn(batch, time, heads, 128, device="cuda")
    g_y = torch.randn(batch, time, inner, device="cuda").to(torch.bfloat16)
    out = torch.randn(batch, time, heads, 128, device="cuda")
    var = torch.rand(batch, time, heads, device="cuda")

    def run(use_slab):
        proj = proj0.clone().requires_grad_()
        if use_slab:
            slab = GradSlab()
            gate, rest = split_projection(proj, inner, 259 * heads, slab)
        else:
            slab = None
            gate, rest = proj[..., :inner], proj[..., inner: inner + 259 * heads]
        vals, keys, queries, beta, log_decay, order = memory_mixer_prep(
            rest, conv_w, conv_b, beta_bias, dt_bias, a_log, heads=heads, bound=0.5, beta_max=1.0,
            slab=slab, col=inner)
        y = memory_mixer_post(out, var, vals, vals, gate, cs, D, om, scale, 1e-5, slab=slab)
        loss = (vals * g_vals).sum() + (y.float() * g_y.float()).sum() + keys.sum() + beta.sum() + log_decay.sum()
        return torch.autograd.grad(loss, proj)[0]

    a, b = run(True), run(False)
    assert torch.equal(a, b)
    assert (a[..., inner + 259 * heads:] == 0).all()


def _unit(x):
    return x * torch.rsqrt((x * x).sum(-1, keepdim=True) + 1e-6)


def composite_memory_step(proj, cache, p, heads, bound, beta_max, eps, floor):
    """The cached memory mixer restated in PyTorch (fp32 between the bf16
    projection and output; `lm/models/mamba4.py:127-337` with a cache)
    around the CUDA one-token read."""
    from mamba4_b200.memory import selective_decode

    inner, d = 128 * heads, 64
    batch = proj.shape[0]
    gate, value, key, query, beta_raw, dt_raw, order_raw = torch.split(
        proj[:, : inner + 259 * heads], (inner, inner, heads * d, heads * d, heads, heads, heads), -1)
    window = torch.cat((cache["history"], proj[:, None]), 1)[..., inner: inner + 256 * heads]
    conv = p["conv_b"] + (window.float() * (p["conv_w"] - bound)[None]).sum(1)
    act = conv * torch.sigmoid(conv)
    v = act[:, :inner].reshape(batch, heads, 128)
    k = _unit(act[:, inner: inner + heads * d].reshape(batch, heads, d))
    q = _unit(act[:, inner + heads * d:].reshape(batch, heads, d))
    beta = beta_max * torch.sigmoid(beta_raw.float() + p["beta_bias"])
    log_decay = -torch.exp(p["a_log"]) * F.softplus(dt_raw.float() + p["dt_bias"])
    res = selective_decode(cache["memory"], cache["shifted"], v, q, beta, log_decay, floor)
    read = res.output * torch.sigmoid(1 - p["conf"] * torch.log1p(res.variance))[..., None] + p["D"][:, None] * v
    lam = torch.sigmoid(order_raw.float() + 2)[..., None]
    order = lam * cache["order"] + (1 - lam) * v
    read = read + torch.sigmoid(p["order_mix"])[:, None] * order
    rs = torch.rsqrt(read.square().mean(-1, keepdim=True) + eps)
    normed = (read * rs * p["scale"]).to(torch.bfloat16).float()
    g = gate.float().reshape(batch, heads, 128)
    y = (normed * (g * torch.sigmoid(g))).to(torch.bfloat16).reshape(batch, inner)
    return y, dict(history=torch.cat((cache["history"], proj[:, None]), 1)[:, 1:], shifted=k, memory=res.state,
                   order=order)


def test_memory_mixer_step_matches_composite():
    """Three-launch cached memory mixer (`memory_mixer_step`) against the
    PyTorch composition over several tokens: same outputs up to bf16
    rounding, same carried state."""
    from mamba4_b200.glue import memory_mixer_step
    from mamba4_b200.memory import selective_initial_state

    torch.manual_seed(11)
    heads, batch, steps = 4, 3, 6
    inner = 128 * heads
    width = inner + 259 * heads + (-(inner + 259 * heads)) % 8
    C = 256 * heads
    dev = "cuda"
    p = dict(conv_w=torch.rand(4, C, device=dev), conv_b=0.1 * torch.randn(C, device=dev),
             beta_bias=torch.randn(heads, device=dev), dt_bias=torch.randn(heads, device=dev),
             a_log=torch.rand(heads, device=dev) * 2, conf=torch.full((heads,), 0.1, device=dev),
             D=torch.randn(heads, device=dev), order_mix=torch.randn(heads, device=dev),
             scale=1 + 0.1 * torch.randn(128, device=dev))
    floor = 0.25 + F.softplus(torch.randn(heads, 64, device=dev))
    zero = lambda: dict(history=torch.zeros(batch, 3, width, dtype=torch.bfloat16, device=dev),  # noqa: E731
                        shifted=torch.zeros(batch, heads, 64, device=dev),
                        memory=selective_initial_state(batch, heads, 64, 128, device=dev),
                        order=torch.zeros(batch, heads, 128, device=dev))
    ca, cb = zero(), zero()
    for _ in range(steps):
        proj = torch.randn(batch, width, device=dev).to(torch.bfloat16)
        ya, ca = memory_mixer_step(proj, ca, p["conv_w"], p["conv_b"], p["beta_bias"], p["dt_bias"], p["a_log"],
                                   floor, p["conf"], p["D"], p["order_mix"], p["scale"], heads=heads, bound=0.5,
                                   beta_max=1.0, eps=1e-5)
        yb, cb = composite_memory_step(proj, cb, p, heads, 0.5, 1.0, 1e-5, floor)
        assert rel(ya, yb) < 1e-2
        assert rel(ca["shifted"], cb["shifted"]) < 1e-5
        assert rel(ca["order"], cb["order"]) < 1e-5
        assert rel(ca["memory"].evidence, cb["memory"].evidence) < 1e-5
        assert rel(ca["memory"].cross, cb["memory"].cross) < 1e-5
        assert torch.equal(ca["history"], cb["history"])


def test_add_rms_norm_matches_add_then_norm():
    """The decode path's fused residual add + RMSNorm gives exactly the
    residual add followed by the RMSNorm kernel."""
    from mamba4_b200.glue import add_rms_norm_bf16

    torch.manual_seed(12)
    for features in (256, 512, 768, 1024):
        x = torch.randn(37, features, device="cuda").to(torch.bfloat16)
        d = torch.randn(37, features, device="cuda").to(torch.bfloat16)
        scale = 1 + 0.1 * torch.randn(features, device="cuda")
        xo, y = add_rms_norm_bf16(x, d, scale, 1e-5)
        ref = x + d
        assert torch.equal(xo, ref)
        assert torch.equal(y, rms_norm_bf16(ref, scale, 1e-5))
        assert rel(y, composite_rms(ref, scale, 1e-5)) < 1e-2


def test_single_shifted_token_leaves_only_the_floor():
    """lm/tests/test_mamba4.py:364-376: with the key shift the first token
    writes a zero key, so after one token the evidence is exactly zero and
    the precision is the floor itself."""
    from mamba4_b200.glue import memory_mixer_prep
    from mamba4_b200.memory import selective_memory_fused

    torch.manual_seed(13)
    heads, C = 4, 256 * 4
    rest = torch.randn(3, 1, 259 * heads + (-259 * heads) % 8, device="cuda").to(torch.bfloat16)
    rest = rest[..., : 259 * heads]
    value, key, query, beta, log_decay, _ = memory_mixer_prep(
        rest, torch.rand(4, C, device="cuda"), torch.randn(C, device="cuda"), torch.randn(heads, device="cuda"),
        torch.randn(heads, device="cuda"), torch.rand(heads, device="cuda"), heads=heads, bound=0.5, beta_max=1.0)
    assert torch.count_nonzero(key) == 0
    floor = 0.25 + torch.rand(heads, 64, device="cuda")
    res = selective_memory_fused(key, value, query, beta, log_decay, floor)
    assert torch.count_nonzero(res.state.evidence) == 0
    precision = res.state.evidence + torch.diag_embed(floor)[None]
    eig = torch.linalg.eigvalsh(precision.double())
    assert torch.allclose(eig[..., -1], floor.double().max(-1).values[None].expand_as(eig[..., -1]), rtol=1e-6)


def test_mamba_mixer_step_matches_composite():
    """Three-launch cached Mamba-3 mixer core (`mamba_mixer_step`) against the
    PyTorch composition of the same token (B/C RMSNorm, dt softplus,
    heavy-tail decay around `mamba3_step`, D skip and SiLU gate) over several
    tokens: outputs to bf16 rounding, caches to float32 rounding."""
    from mamba4_b200.flashmamba import mamba3_step, mamba3_step_cache
    from mamba4_b200.glue import mamba_mixer_step

    torch.manual_seed(14)
    batch, heads, angles, eps = 3, 4, 16, 1e-5
    inner = 64 * heads
    width = 2 * inner + 128 + 3 * heads + angles
    bs, cs = 1 + 0.1 * torch.randn(64, device="cuda"), 1 + 0.1 * torch.randn(64, device="cuda")
    dtb, D = torch.randn(heads, device="cuda") - 3, torch.randn(heads, device="cuda")
    qb, kb = torch.ones(heads, 1, 64, device="cuda"), torch.ones(heads, 1, 64, device="cuda")
    ca = mamba3_step_cache(batch, heads, 64, 64, angles, device="cuda")
    cb = mamba3_step_cache(batch, heads, 64, 64, angles, device="cuda")
    for _ in range(5):
        proj = torch.randn(batch, width, device="cuda").to(torch.bfloat16)
        ya, ca = mamba_mixer_step(proj, bs, cs, dtb, D, qb, kb, ca, inner=inner, heads=heads, angles=angles,
                                  eps=eps)
        z, x, b, c, raw_dt, raw_a, trap, ang = torch.split(
            proj, (inner, inner, 64, 64, heads, heads, heads, angles), -1)
        dt = F.softplus(raw_dt.float() + dtb)
        adt = -torch.clamp(heavy_tail(raw_a.float()), min=1e-4) * dt
        y, cb = mamba3_step(cb, composite_rms(c, cs, eps), composite_rms(b, bs, eps), x.contiguous(), adt, dt,
                            trap.float(), ang.float(), q_bias=qb, k_bias=kb)
        yh = y.float().reshape(batch, heads, 64) + x.float().reshape(batch, heads, 64) * D[:, None]
        zf = z.float().reshape(batch, heads, 64)
        yb = (yh * (zf * torch.sigmoid(zf))).to(torch.bfloat16).reshape(batch, inner)
        assert rel(ya, yb) < 1e-2
        for ta, tb in zip(ca, cb):
            assert rel(ta, tb) < 1e-2
