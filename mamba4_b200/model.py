"""Mamba 4 language model around the B200 operators (PyTorch modules).

Restates the reference model (`lm/models/mamba4.py`, `lm/models/mamba3.py`,
`lm/models/common.py`) with the same parameter tree, initialisation and
forward arithmetic, using this package's CUDA operators for the two hot
ops: the memory read (`selective_memory_fused`) and the Mamba-3 scan
(`mamba3_fused`). Linear layers run in bfloat16 (torch autocast), norms,
gates and the memory statistics in float32, as the reference's
`dtype="bfloat16"`, `param_dtype="float32"` configuration does.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.nn as nn
import torch.nn.functional as F

from .flashmamba import Mamba3StepCache, mamba3_step_cache
from .glue import (ADD_RMS_FEATURES, GradSlab, add_rms_norm_bf16, head_cross_entropy, mamba_mixer_core,
                   mamba_mixer_step, memory_mixer_post, memory_mixer_prep, memory_mixer_step, order_scan,
                   rms_norm_bf16, split_projection)
from .memory import selective_initial_state, selective_memory_fused
from .remat import block_modes, run_block


@dataclass(frozen=True)
class Mamba4Config:
    """Subset of the reference `ModelConfig` (`lm/config.py:6-89`) the
    Mamba 4 model reads. Defaults: BASELINE config 3 (60M)."""

    vocab_size: int = 50304
    d_model: int = 512
    layer_pattern: str = "SSSM" * 4
    expand: int = 2
    head_dim: int = 64          # Mamba-3 head dim (16 heads at d_model 512)
    d_state: int = 96           # Mamba-3 state dim N (the kernels run 64, 96 and 128)
    rope_fraction: float = 0.5  # angle pairs = d_state * rope_fraction / 2
    key_dim: int = 64           # memory key dim
    memory_head_dim: int = 128  # memory value dim (8 heads at d_model 512)
    conv_kernel: int = 4
    floor_min: float = 0.25
    floor_init: float = 1.0
    order_head: bool = True
    memory_beta_max: float = 1.0
    memory_key_shift: bool = True
    norm_eps: float = 1e-5
    chunk_size: int = 64
    # Activation rematerialization (`lm/config.py:26-34`, `remat_block` in
    # lm/models/common.py:97-122): off by default here (a B200 holds the
    # configs' activations: 180 GB of HBM); the reference's policy names are
    # accepted ("full", "kernels", "mixers", "mixers-N").
    remat: bool = False
    remat_policy: str = "full"

    @property
    def n_layers(self) -> int:
        return len(self.layer_pattern)

    @property
    def inner(self) -> int:
        return self.d_model * self.expand

    @property
    def num_heads(self) -> int:
        return self.inner // self.head_dim

    @property
    def memory_heads(self) -> int:
        return self.inner // self.memory_head_dim


CONFIGS = {
    # d_model 512, 16 blocks (12 Mamba-3 + 4 memory, one
    # every 4th block), memory 8 heads x key 64 (value 128, forced by
    # d_model * expand = heads * value_dim), vocab 50304; Mamba-3 state 96
    # as the reference 60M model (lm/configs/mamba4-60m.json:10).
    "60m": Mamba4Config(d_state=96),
    # d_model 768, 17 Mamba-3 + 4 memory layers
    # (pattern of lm/configs/mamba4-125m.json), memory 12 heads x 128,
    # Mamba-3 state 128 (lm/configs/mamba4-125m.json:10).
    "125m": Mamba4Config(d_model=768, layer_pattern="SSSMSSSSMSSSSMSSSSMSS", d_state=128,
                         remat_policy="mixers-3"),
}


class RMSNorm(nn.Module):
    """`lm/models/common.py:25-45`: fp32 statistics, output in the model dtype."""

    def __init__(self, features: int, eps: float, out_dtype=torch.bfloat16):
        super().__init__()
        self.scale = nn.Parameter(torch.ones(features))
        self.eps = eps
        self.out_dtype = out_dtype

    def forward(self, x):
        if (x.is_cuda and x.dtype == torch.bfloat16 and self.out_dtype == torch.bfloat16
                and x.shape[-1] in (256, 512, 768, 1024)):
            return rms_norm_bf16(x, self.scale, self.eps)
        x32 = x.float()
        var = x32.square().mean(-1, keepdim=True)
        return (x32 * torch.rsqrt(var + self.eps) * self.scale).to(self.out_dtype)


def _dense(din, dout, std):
    layer = nn.Linear(din, dout, bias=False)
    nn.init.normal_(layer.weight, 0.0, std)
    return layer


def heavy_tail_activation(x):
    """`lm/models/mamba3.py:28-29`."""
    return torch.clamp(x, min=0) + torch.reciprocal(1 - torch.clamp(x, max=0))


def timestep_bias_init(shape, generator=None):
    """`lm/models/mamba3.py:32-36`: inverse softplus of log-uniform dt."""
    u = torch.rand(shape, generator=generator)
    dt = torch.exp(u * (math.log(0.1) - math.log(0.001)) + math.log(0.001))
    return dt + torch.log(-torch.expm1(-dt))


class Mamba3Mixer(nn.Module):
    """Flash branch of `Mamba3Mixer` (`lm/models/mamba3.py:43-132`)."""

    def __init__(self, cfg: Mamba4Config):
        super().__init__()
        self.cfg = cfg
        h, n = cfg.num_heads, cfg.d_state
        self.angles = int(cfg.d_state * cfg.rope_fraction) // 2
        self.sizes = (cfg.inner, cfg.inner, n, n, h, h, h, self.angles)
        self.in_proj = _dense(cfg.d_model, sum(self.sizes), 0.02)
        self.B_norm = RMSNorm(n, cfg.norm_eps)
        self.C_norm = RMSNorm(n, cfg.norm_eps)
        self.B_bias = nn.Parameter(torch.ones(h, 1, n))
        self.C_bias = nn.Parameter(torch.ones(h, 1, n))
        self.dt_bias = nn.Parameter(timestep_bias_init((h,)))
        self.D = nn.Parameter(torch.ones(h))
        self.out_proj = _dense(cfg.inner, cfg.d_model, 0.02 / math.sqrt(2 * cfg.n_layers))

    def forward(self, u):
        cfg = self.cfg
        proj = self.in_proj(u)
        with torch.autocast("cuda", enabled=False):
            y = mamba_mixer_core(proj.to(torch.bfloat16), self.B_norm.scale, self.C_norm.scale, self.dt_bias,
                                 self.D, self.C_bias, self.B_bias, inner=cfg.inner, heads=cfg.num_heads,
                                 angles=self.angles, eps=cfg.norm_eps, state=cfg.d_state)
        return self.out_proj(y)

    def init_cache(self, batch, device=None):
        cfg = self.cfg
        return mamba3_step_cache(batch, cfg.num_heads, cfg.d_state, cfg.head_dim, self.angles, device=device)

    def decode(self, u, cache: Mamba3StepCache, inplace=False):
        """One token (`_Mamba3StepMixer`, `lm/models/mamba4.py:412-481`):
        u [B, d_model] bf16 -> ([B, d_model], new cache) through the
        training glue's prep and post kernels around the scan step (same
        rounding points: B/C RMSNorm to bf16, scan output bf16,
        out = bf16((y + x D) silu(z)))."""
        cfg = self.cfg
        proj = self.in_proj(u)
        with torch.autocast("cuda", enabled=False):
            out, cache = mamba_mixer_step(proj.to(torch.bfloat16), self.B_norm.scale, self.C_norm.scale,
                                          self.dt_bias, self.D, self.C_bias, self.B_bias, cache,
                                          inner=cfg.inner, heads=cfg.num_heads, angles=self.angles,
                                          eps=cfg.norm_eps, inplace=inplace, state=cfg.d_state)
        return self.out_proj(out), cache


class SelectiveMemoryMixer(nn.Module):
    """`SelectiveMemoryMixer` (`lm/models/mamba4.py:115-337`), training path."""

    def __init__(self, cfg: Mamba4Config):
        super().__init__()
        self.cfg = cfg
        h, d, p = cfg.memory_heads, cfg.key_dim, cfg.memory_head_dim
        if h * p != cfg.inner:
            raise ValueError("Expanded dimension must divide exactly into memory heads")
        if cfg.floor_min <= 0 or cfg.floor_init <= cfg.floor_min:
            raise ValueError("Selective floor must be positive and above its minimum")
        self.sizes = (cfg.inner, cfg.inner, h * d, h * d, h, h, h)
        self.in_proj = _dense(cfg.d_model, sum(self.sizes), 0.02)
        channels = cfg.inner + 2 * h * d
        bound = 1 / math.sqrt(cfg.conv_kernel)
        self.conv_weight = nn.Parameter(torch.empty(cfg.conv_kernel, channels).uniform_(0.0, 2 * bound))
        self.conv_bias = nn.Parameter(torch.zeros(channels))
        self.bound = bound
        start = 0.5 / max(cfg.memory_beta_max, 1.0)
        self.beta_bias = nn.Parameter(torch.full((h,), math.log(start / (1 - start))))
        self.dt_bias = nn.Parameter(timestep_bias_init((h,)))
        self.a_log = nn.Parameter(torch.log(torch.empty(h).uniform_(1.0, 16.0)))
        self.floor = nn.Parameter(torch.full((h, d), math.log(math.expm1(cfg.floor_init - cfg.floor_min))))
        self.confidence_scale = nn.Parameter(torch.full((h,), 0.1))
        self.D = nn.Parameter(torch.ones(h))
        self.order_mix = nn.Parameter(torch.full((h,), -1.0))
        self.read_norm = RMSNorm(p, cfg.norm_eps)
        self.out_proj = _dense(cfg.inner, cfg.d_model, 0.02 / math.sqrt(2 * cfg.n_layers))

    def forward(self, u):
        cfg = self.cfg
        h = cfg.memory_heads
        if cfg.key_dim != 64 or cfg.memory_head_dim != 128 or not cfg.memory_key_shift or cfg.conv_kernel != 4:
            raise ValueError("the fused memory mixer supports key_dim 64, memory_head_dim 128, "
                             "conv_kernel 4 and the key shift")
        proj = self.in_proj(u)
        with torch.autocast("cuda", enabled=False):
            proj = proj.to(torch.bfloat16)
            if proj.shape[-1] % 8:
                # The fused glue reads rows with 16-byte loads.
                proj = F.pad(proj, (0, -proj.shape[-1] % 8))
            slab = GradSlab()
            gate, rest = split_projection(proj, cfg.inner, 259 * h, slab)
            value, key, query, beta, log_decay, order_logit = memory_mixer_prep(
                rest, self.conv_weight, self.conv_bias, self.beta_bias, self.dt_bias, self.a_log, heads=h,
                bound=self.bound, beta_max=cfg.memory_beta_max, slab=slab, col=cfg.inner)
            floor = cfg.floor_min + F.softplus(self.floor)
            res = selective_memory_fused(key, value, query, beta, log_decay, floor, chunk_size=cfg.chunk_size)
            ordered = order_scan(value, order_logit) if cfg.order_head else torch.zeros_like(value)
            read = memory_mixer_post(res.output, res.variance, value, ordered, gate, self.confidence_scale,
                                     self.D, self.order_mix, self.read_norm.scale, cfg.norm_eps, slab=slab)
        return self.out_proj(read)

    def init_cache(self, batch, device=None):
        """Constant-size decode cache (`lm/models/mamba4.py:527-560`): the
        previous three projection rows (the conv history), the previous
        token's unit key (the key shift), the memory state and the order
        state."""
        cfg = self.cfg
        h, d, p = cfg.memory_heads, cfg.key_dim, cfg.memory_head_dim
        width = sum(self.sizes) + (-sum(self.sizes)) % 8
        return dict(memory=selective_initial_state(batch, h, d, p, device=device),
                    history=torch.zeros(batch, cfg.conv_kernel - 1, width, dtype=torch.bfloat16, device=device),
                    order=torch.zeros(batch, h, p, device=device),
                    shifted=torch.zeros(batch, h, d, device=device))

    def decode(self, u, cache, inplace=False):
        """One token of the cached memory mixer (`lm/models/mamba4.py:127-337`
        with `cache`) through `memory_mixer_step`: the training glue's
        kernels at one token (same rounding points) around the one-token
        read `m4_memread_decode`."""
        cfg = self.cfg
        if cfg.key_dim != 64 or cfg.memory_head_dim != 128 or not cfg.memory_key_shift or cfg.conv_kernel != 4:
            raise ValueError("the fused memory mixer supports key_dim 64, memory_head_dim 128, "
                             "conv_kernel 4 and the key shift")
        proj = self.in_proj(u)
        with torch.autocast("cuda", enabled=False):
            proj = proj.to(torch.bfloat16)
            if proj.shape[-1] % 8:
                proj = F.pad(proj, (0, -proj.shape[-1] % 8))
            floor = cfg.floor_min + F.softplus(self.floor)
            out, cache = memory_mixer_step(
                proj, cache, self.conv_weight, self.conv_bias, self.beta_bias, self.dt_bias, self.a_log, floor,
                self.confidence_scale, self.D, self.order_mix, self.read_norm.scale, heads=cfg.memory_heads,
                bound=self.bound, beta_max=cfg.memory_beta_max, eps=cfg.norm_eps, order_head=cfg.order_head,
                inplace=inplace)
        return self.out_proj(out), cache


class Block(nn.Module):
    """Pre-norm residual block (`Mamba3Block`, `SelectiveMemoryBlock`)."""

    def __init__(self, cfg: Mamba4Config, kind: str):
        super().__init__()
        self.norm = RMSNorm(cfg.d_model, cfg.norm_eps)
        self.mixer = SelectiveMemoryMixer(cfg) if kind == "M" else Mamba3Mixer(cfg)

    def forward(self, x):
        return x + self.mixer(self.norm(x)).to(x.dtype)


class Mamba4LM(nn.Module):
    """`Mamba4LM` (`lm/models/mamba4.py:484-504`): embedding, blocks per the
    layer pattern, final RMSNorm, tied output head with float32 logits."""

    def __init__(self, cfg: Mamba4Config):
        super().__init__()
        if set(cfg.layer_pattern) - {"M", "S"}:
            raise ValueError("layer_pattern must contain n_layers M/S characters")
        self.cfg = cfg
        self.embedding = nn.Embedding(cfg.vocab_size, cfg.d_model)
        nn.init.normal_(self.embedding.weight, 0.0, 0.02)
        self.blocks = nn.ModuleList(Block(cfg, k) for k in cfg.layer_pattern)
        self.final_norm = RMSNorm(cfg.d_model, cfg.norm_eps)
        self.remat_modes = block_modes(cfg.layer_pattern, cfg.remat_policy)  # validates the name
        self.fused_loss = True  # forward(tokens, targets) returns per-token losses

    def hidden(self, tokens):
        # bfloat16 residual stream and final norm (Embed dtype bf16).
        x = self.embedding(tokens).to(torch.bfloat16)
        remat = self.cfg.remat and torch.is_grad_enabled()
        for block, mode in zip(self.blocks, self.remat_modes):
            x = run_block(block, x, mode) if remat else block(x)
        return self.final_norm(x)

    def forward(self, tokens, targets=None):
        """Logits [B,T,V] float32 (tied head, attend().astype(f32)); with
        `targets`, the per-token cross-entropy [B,T] from the fused head."""
        x = self.hidden(tokens)
        if targets is not None:
            return head_cross_entropy(x, self.embedding.weight, targets)
        return F.linear(x, self.embedding.weight.to(x.dtype)).float()

    def init_cache(self, batch, device=None):
        """Constant-size decode cache of every layer (`lm/models/mamba4.py:527-560`)."""
        return [block.mixer.init_cache(batch, device=device) for block in self.blocks]

    @torch.no_grad()
    def decode_step(self, tokens, cache, inplace=False):
        """One cached decode step (`lm/models/mamba4.py:507-524`): tokens [B]
        -> (logits [B, V] float32, new cache). Run under the same autocast as
        the forward. inplace=True writes the layers' scan states and memory
        states over `cache`'s tensors (the graph decoder's static cache)
        instead of fresh ones."""
        x = self.embedding(tokens).to(torch.bfloat16)
        new = []
        fused = x.shape[-1] in ADD_RMS_FEATURES
        h = self.blocks[0].norm(x)
        for i, (block, layer) in enumerate(zip(self.blocks, cache)):
            out, layer = block.mixer.decode(h, layer, inplace=inplace)
            new.append(layer)
            norm = self.blocks[i + 1].norm if i + 1 < len(self.blocks) else self.final_norm
            if fused:
                # The block's residual add and the next norm in one launch.
                x, h = add_rms_norm_bf16(x, out.to(x.dtype), norm.scale, norm.eps)
            else:
                x = x + out.to(x.dtype)
                h = norm(x)
        return F.linear(h, self.embedding.weight.to(h.dtype)).float(), new


def _cache_tensors(cache):
    """The tensors of a layer-cache tree (lists, dicts and named tuples) in a
    fixed order."""
    if isinstance(cache, torch.Tensor):
        return [cache]
    if isinstance(cache, dict):
        return [t for k in sorted(cache) for t in _cache_tensors(cache[k])]
    return [t for item in cache for t in _cache_tensors(item)]


class GraphedDecoder:
    """`Mamba4LM.decode_step` captured once as a CUDA graph (the B200
    counterpart of the reference's jitted decode, `lm/models/mamba4.py:507-524`).

    A decode step is about a hundred small launches (block norms,
    projections, the glue kernels, `m4_scan_step`, `m4_memread_decode`);
    replaying them as one graph removes the per-launch host cost. The cache
    lives in static buffers that the graph reads and then overwrites with the
    next cache, so `step(tokens)` returns the same logits as eager
    `decode_step` calls from `model.init_cache(batch)` (the graph runs the
    same kernels on the same operands). `logits` is a static buffer,
    overwritten by the next step.

    The linear and embedding weights enter the graph as bfloat16 copies (the
    casts autocast would otherwise repeat at every token, one launch and a
    full weight read each); call `refresh_weights()` after changing the
    model's parameters. Every other parameter is read in place at each replay.
    """

    def __init__(self, model: Mamba4LM, batch: int, device=None, dtype=torch.bfloat16):
        self.model, self.batch, self.dtype = model, batch, dtype
        device = torch.device("cuda" if device is None else device)
        self._shadow = [(mod, mod.weight, nn.Parameter(mod.weight.detach().to(dtype), requires_grad=False))
                        for mod in model.modules() if isinstance(mod, (nn.Linear, nn.Embedding))]
        self._initial = model.init_cache(batch, device=device)
        self.cache = model.init_cache(batch, device=device)
        self._static = _cache_tensors(self.cache)
        self.tokens = torch.zeros(batch, dtype=torch.long, device=device)
        current = torch.cuda.current_stream(device)
        side = torch.cuda.Stream(device)
        side.wait_stream(current)
        self._install(True)
        try:
            with torch.cuda.stream(side):
                for _ in range(2):
                    self._body()
            current.wait_stream(side)
            self.graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(self.graph):
                self.logits = self._body()
        finally:
            self._install(False)
        self.reset()

    def _install(self, shadow: bool):
        for mod, full, low in self._shadow:
            mod._parameters["weight"] = low if shadow else full

    @torch.no_grad()
    def _body(self):
        with torch.autocast("cuda", dtype=self.dtype):
            logits, new = self.model.decode_step(self.tokens, self.cache, inplace=True)
        for dst, src in zip(self._static, _cache_tensors(new)):
            if dst.data_ptr() != src.data_ptr():
                dst.copy_(src)
        return logits

    @torch.no_grad()
    def refresh_weights(self):
        """Copy the model's current linear and embedding weights into the
        graph's bfloat16 copies."""
        for _, full, low in self._shadow:
            low.copy_(full)

    def reset(self):
        """Back to the empty cache (a new batch of sequences)."""
        for dst, src in zip(self._static, _cache_tensors(self._initial)):
            dst.copy_(src)

    def step(self, tokens: torch.Tensor) -> torch.Tensor:
        """tokens [batch] -> logits [batch, vocab] float32 (static buffer)."""
        self.tokens.copy_(tokens, non_blocking=True)
        self.graph.replay()
        return self.logits


def parameter_count(model: nn.Module) -> int:
    return sum(p.numel() for p in model.parameters())
