"""Benchmark of the Mamba 4 FlashMamba hot path on B200.

Default workload ("hotpath", BASELINE configs[1] + configs[2]): one step is
  * one Mamba-3 SISO scan layer forward+backward on config 1
    (batch 16 x seq 1024, 16 heads, P = N = 64, chunk 64, bf16 operands), and
  * one memory-read layer forward+backward on config 2
    (batch 128 x seq 1024, 8 heads, D = P = 64, fp32, factors stored),
on seeded synthetic inputs already resident in HBM. The metric is the
baseline's "memory-read+scan tokens/s fwd+bwd": tokens through the two layers
(16,384 + 131,072 per GPU per step) per second. Under torchrun every rank
runs its own batch (no data-path exchange; weak scaling) and the value is the
job total. `e2e` is the same metric through the public operator API with the
inputs copied from pinned host memory and every output and gradient copied
back inside the timed region.

`--impl reference` times the reference's CPU path for the same workload
(its XLA algorithms restated in float32 PyTorch, `oracle/cpu_path.py`; the
reference's JAX runtime is not installed) on all host cores: K whole steps,
each a bounded sample of whole sequences in the workload's token mix.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

MEM_CFG = dict(batch=128, time=1024, heads=8, dim=64, value_dim=64)      # configs[2]
SCAN_CFG = dict(batch=16, time=1024, heads=16, head_dim=64, state_dim=64)  # configs[1]
SMALL_MEM_CFG = dict(batch=16, time=1024, heads=8, dim=64, value_dim=64)
# ncu-sized case of the same kernels (stored factors 302 MB, still above L2).
PROFILE_MEM_CFG = dict(batch=4, time=1024, heads=8, dim=64, value_dim=64)
PROFILE_SCAN_CFG = dict(batch=4, time=1024, heads=16, head_dim=64, state_dim=64)
# Algorithmic work per unit (per token-head for the memory read, per token for
# the scan at H = 16, P = N = 64, c = 64): the figures of the hot-path survey.
MEM_FWD_BYTES, MEM_BWD_BYTES = 9356, 10132
MEM_FWD_FLOPS, MEM_BWD_FLOPS = 122421, 80160
SCAN_BYTES, SCAN_FLOPS = 11776, 1835008
L2_BYTES = 126 * 2**20


def peaks():
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        p = json.loads(path.read_text())
        return dict(hbm=p["hbm_gbs"], bf16=p["bf16_tflops"], bf16_sust=p["bf16_tflops_sustained"],
                    source="measured")
    return dict(hbm=6650.0, bf16=1590.0, bf16_sust=1400.0, source="fallback")


class ClockSampler:
    """nvidia-smi clocks and throttle reasons during the timed region."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
             "clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.samples = []
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.QUERY}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) == 8:
                self.samples.append(parts)

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(s[1]) for s in self.samples if s[1].replace(".", "").isdigit()]
        mx = [float(s[2]) for s in self.samples if s[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for s in self.samples for n, v in zip(names, s[4:]) if v == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons,
                "samples": len(self.samples)}


def setup_dist(n_gpus):
    import torch

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist

        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def max_over_ranks(value, world):
    if world == 1:
        return value
    import torch
    import torch.distributed as dist

    t = torch.tensor([value], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def make_mem(cfg, seed, device):
    """Seeded config-2 inputs generated on the device (torch RNG; same
    distributions as the oracle's config_inputs)."""
    import torch

    g = torch.Generator(device=device).manual_seed(seed)
    B, T, H, D, P = cfg["batch"], cfg["time"], cfg["heads"], cfg["dim"], cfg["value_dim"]
    q = torch.randn(B, T, H, D, device=device, generator=g) / 8
    k = torch.randn(B, T, H, D, device=device, generator=g) / 8
    v = torch.randn(B, T, H, P, device=device, generator=g)
    lam = torch.sigmoid(torch.randn(B, T, H, device=device, generator=g) + 2.0)
    beta = torch.sigmoid(torch.randn(B, T, H, device=device, generator=g))
    d_out = torch.randn(B, T, H, P, device=device, generator=g)
    d_var = torch.randn(B, T, H, device=device, generator=g)
    k = torch.cat((torch.zeros_like(k[:, :1]), k[:, :-1]), 1).contiguous()
    floor = torch.full((H, D), 0.1, device=device)
    return dict(keys=k, values=v, queries=q, beta=beta, log_decay=torch.log(lam), floor=floor,
                d_output=d_out, d_variance=d_var)


def make_scan(cfg, seed, device):
    import math

    import torch

    g = torch.Generator(device=device).manual_seed(seed)
    B, T, H, P, N = cfg["batch"], cfg["time"], cfg["heads"], cfg["head_dim"], cfg["state_dim"]
    bf = torch.bfloat16
    x = (torch.randn(B, T, H * P, device=device, generator=g) / 8).to(bf)
    b = (torch.randn(B, T, N, device=device, generator=g) / 8).to(bf)
    c = (torch.randn(B, T, N, device=device, generator=g) / 8).to(bf)
    dt = torch.nn.functional.softplus(torch.randn(B, T, H, device=device, generator=g) * 0.5 - 3.0)
    a = -torch.exp(torch.rand(H, device=device, generator=g) * math.log(16.0))
    adt = a * dt
    trap = torch.randn(B, T, H, device=device, generator=g)
    angles = (torch.rand(B, T, N // 2, device=device, generator=g) * 2 - 1) * math.pi
    ones = torch.ones(H, 1, N, device=device)
    d_y = torch.randn(B, T, H * P, device=device, generator=g).to(bf)
    d_final = torch.randn(B, H, N, P, device=device, generator=g)
    return dict(c=c, b=b, x=x, adt=adt, dt=dt, trap_logits=trap, angles=angles, q_bias=ones,
                k_bias=ones.clone(), d_y=d_y, d_final=d_final)


def memread_step(m, requires=True):
    import torch

    from mamba4_b200 import selective_memory_fused

    leaves = [m[n].requires_grad_(requires) for n in ("keys", "values", "queries", "beta", "log_decay")]
    res = selective_memory_fused(*leaves, m["floor"])
    grads = torch.autograd.grad((res.output, res.variance), leaves,
                                (m["d_output"], m["d_variance"]))
    return res, grads


def scan_step(s):
    import torch

    from mamba4_b200 import mamba3_fused

    names = ("c", "b", "x", "adt", "dt", "trap_logits", "angles", "q_bias", "k_bias")
    leaves = [s[n].requires_grad_(True) for n in names]
    y, final = mamba3_fused(*leaves[:7], q_bias=leaves[7], k_bias=leaves[8])
    grads = torch.autograd.grad((y, final), leaves, (s["d_y"], s["d_final"]))
    return y, final, grads


def count_launches(fn):
    """Kernels of this library (names in namespace m4::) launched by one call
    of fn, counted by the CUDA profiler outside the timed region."""
    import torch
    from torch.profiler import ProfilerActivity, profile

    torch.cuda.synchronize()
    try:
        with profile(activities=[ProfilerActivity.CUDA]) as prof:
            fn()
            torch.cuda.synchronize()
    except RuntimeError:  # the profiler is unavailable (e.g. under another profiler)
        return None
    return sum(e.count for e in prof.key_averages() if "m4::" in e.key)


def launches(fn, steps):
    n = count_launches(fn)
    return None if n is None else n * steps


def time_region(fn, steps, warmup, world, streams=()):
    """Device time (ms) of `steps` calls of fn on the current stream. Work
    that fn issues on side `streams` (pipelined copies) is bracketed too: the
    streams wait for the start event and the stop event waits for them."""
    import torch

    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    cur = torch.cuda.current_stream()
    start.record()
    for st in streams:
        st.wait_stream(cur)
    for _ in range(steps):
        fn()
    for st in streams:
        cur.wait_stream(st)
    stop.record()
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    return start.elapsed_time(stop)


def op_times(fn_fwd, fn_bwd, reps=5):
    """Average device time (ms) of a forward and a backward call, CUDA events."""
    import torch

    fwd_ms, bwd_ms = [], []
    for _ in range(reps):
        e0, e1, e2 = (torch.cuda.Event(enable_timing=True) for _ in range(3))
        e0.record()
        ctx = fn_fwd()
        e1.record()
        fn_bwd(ctx)
        e2.record()
        torch.cuda.synchronize()
        fwd_ms.append(e0.elapsed_time(e1))
        bwd_ms.append(e1.elapsed_time(e2))
    return statistics.median(fwd_ms), statistics.median(bwd_ms)


CPU_SAMPLE_MEM_SEQS = 8   # memory-read sequences per CPU sample step (of configs[2])
CPU_SAMPLE_SCAN_SEQS = 1  # scan sequences per CPU sample step (of configs[1]): the 8:1 token mix


def cpu_sample_inputs(mem_cfg, scan_cfg):
    """One bounded sample of the hot-path workload for the CPU baseline:
    CPU_SAMPLE_MEM_SEQS whole sequences of the memory-read config and
    CPU_SAMPLE_SCAN_SEQS of the scan config (full length, all heads, the
    workload's own mix of memory-read to scan tokens), float32 host tensors
    from the oracle's seeded generators (the scan's c, b, x rounded to bf16
    as the GPU step's inputs are)."""
    import torch

    from oracle import memread as M
    from oracle import scan as S

    mseq = min(CPU_SAMPLE_MEM_SEQS, mem_cfg["batch"])
    sseq = min(CPU_SAMPLE_SCAN_SEQS, scan_cfg["batch"])
    cfg = M.config_inputs(mseq, mem_cfg["time"], mem_cfg["heads"], mem_cfg["dim"], mem_cfg["value_dim"], seed=0)
    mem = {n: torch.tensor(v) for n, v in cfg.items()}
    sc = S.config_inputs(sseq, scan_cfg["time"], scan_cfg["heads"], scan_cfg["head_dim"],
                         scan_cfg["state_dim"], seed=1)
    scan = {n: torch.tensor(v) for n, v in sc.items()}
    for n in ("c", "b", "x", "d_y"):
        scan[n] = scan[n].to(torch.bfloat16).float()
    tokens = mseq * mem_cfg["time"] + sseq * scan_cfg["time"]
    desc = (f"reference CPU path restated in float32 PyTorch (oracle/cpu_path.py: the XLA memory read of "
            f"selective_gaussian_memory with the spd_solve VJP, and mamba3_chunked), value and gradient of "
            f"the projected loss; one step = {mseq} x {mem_cfg['time']} tokens x {mem_cfg['heads']} heads of "
            f"the memory read + {sseq} x {scan_cfg['time']} tokens x {scan_cfg['heads']} heads of the scan "
            f"({tokens} tokens, the workload's token mix)")
    return mem, scan, tokens, desc


def cpu_sample_step(mem, scan):
    from oracle import cpu_path as C

    C.memory_step(mem)
    C.scan_step(scan)


def cpu_baseline_sample(mem_cfg, scan_cfg, threads):
    """The CPU restatement of the reference path on the host's cores: one
    warm-up and one timed sample step (whole sequences, not extrapolated).
    Returns (tokens/s, seconds per sample step, description)."""
    import torch

    torch.set_num_threads(threads)
    mem, scan, tokens, desc = cpu_sample_inputs(mem_cfg, scan_cfg)
    cpu_sample_step(mem, scan)
    t0 = time.perf_counter()
    cpu_sample_step(mem, scan)
    dt = time.perf_counter() - t0
    return tokens / dt, dt, desc


def host_threads():
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def hotpath_config(workload, mem_cfg, scan_cfg):
    """The `config` object of the hot-path line (both arms)."""
    tokens = mem_cfg["batch"] * mem_cfg["time"] + scan_cfg["batch"] * scan_cfg["time"]
    return {"workload": {"hotpath": "configs[1]+configs[2] (hotpath)",
                         "small": "small memory read (16x1024x8) + configs[1] scan",
                         "profile": "ncu-sized memory read (4x1024x8) + scan (4x1024x16)"}[workload],
            "memread": mem_cfg, "scan": dict(scan_cfg, chunk=64, dtype="bf16"),
            "tokens_per_step_per_gpu": tokens, "l2": "inputs larger than L2 (memory-read "
            "operands 268 MB each, stored factors 9.7 GB)"}


def run_reference(args):
    """The reference arm: rank 0 times K steps (after W warm-up steps) of the
    reference's CPU path, restated in float32 PyTorch, on all host threads.
    Each step is one bounded sample of the workload (see cpu_sample_inputs);
    ms_per_step is the measured time of that sample step and value its tokens
    per second. Other ranks exit without work."""
    import torch

    if int(os.environ.get("RANK", "0")) != 0:
        return
    threads = host_threads()
    torch.set_num_threads(threads)
    mem, scan, tokens, desc = cpu_sample_inputs(MEM_CFG, SCAN_CFG)
    for _ in range(args.warmup):
        cpu_sample_step(mem, scan)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        cpu_sample_step(mem, scan)
    ms_per_step = 1000.0 * (time.perf_counter() - t0) / args.steps
    value = tokens / (ms_per_step / 1000.0)
    line = {
        "impl": "reference", "metric": "memory-read+scan tokens/s fwd+bwd", "value": value,
        "unit": "tokens/s", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": hotpath_config("hotpath", MEM_CFG, SCAN_CFG),
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": threads, "kind": "port",
                         "sample": desc},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def measure_e2e_hotpath(m, s, dev, world, tokens, args):
    """The hot-path step through the public operators with every input copied
    in from pinned host memory and every output and gradient copied back,
    pipelined over two device input slots and two pinned output slots: step
    i+1's inputs cross on one copy stream and step i's results on another
    while step i computes. Times the same K steps as the device-timed line
    (max over ranks); returns the `e2e` JSON object."""
    import torch

    pin = [{k: v.detach().cpu().pin_memory() for k, v in src.items()} for src in (m, s)]
    h2d = sum(t.numel() * t.element_size() for d in pin for t in d.values())
    slots = [[{k: torch.empty_like(v, device=dev) for k, v in d.items()} for d in pin] for _ in range(2)]
    copy_in, copy_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    freed = [torch.cuda.Event(), torch.cuda.Event()]
    out_host = [None, None]
    state = {"i": 0, "d2h": 0}
    compute = torch.cuda.current_stream(dev)

    def e2e_step():
        slot = state["i"] % 2
        state["i"] += 1
        dm, ds = slots[slot]
        with torch.cuda.stream(copy_in):
            copy_in.wait_event(freed[slot])
            for dst, src in zip((dm, ds), pin):
                for k, v in src.items():
                    dst[k].copy_(v, non_blocking=True)
            ready = torch.cuda.Event()
            ready.record(copy_in)
        compute.wait_event(ready)
        leaves_m = {k: v.detach() for k, v in dm.items()}
        leaves_s = {k: v.detach() for k, v in ds.items()}
        res, mg = memread_step(leaves_m)
        y, fin, sg = scan_step(leaves_s)
        outs = [t.detach() for t in (res.output, res.variance, res.state.evidence, res.state.cross,
                                     *mg, y, fin, *sg)]
        freed[slot].record(compute)
        if out_host[slot] is None:
            out_host[slot] = [torch.empty(t.shape, dtype=t.dtype, pin_memory=True) for t in outs]
            state["d2h"] = sum(t.numel() * t.element_size() for t in outs)
        done = torch.cuda.Event()
        done.record(compute)
        with torch.cuda.stream(copy_out):
            copy_out.wait_event(done)
            for h, t in zip(out_host[slot], outs):
                t.record_stream(copy_out)
                h.copy_(t, non_blocking=True)

    n = args.steps
    e2e_ms = max_over_ranks(time_region(e2e_step, n, args.warmup, world, streams=(copy_in, copy_out)),
                            world) / n
    return {"value": world * tokens / (e2e_ms / 1000.0), "unit": "tokens/s",
            "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": state["d2h"], "ms_per_step": e2e_ms,
            "pipelined": "inputs of step i+1 copied in and results of step i copied out "
                         "while step i computes (two slots, two copy streams)",
            "host_link": f"bound by PCIe / host memory, shared by the {world} rank(s) of this node "
                         "(about 50 GB/s per direction for one GPU, about 130 GB/s aggregate measured "
                         "with 8): per-GPU e2e falls as ranks are added; the device-timed value is the "
                         "kernels' claim"}


def measure_decode(world, rank, local, batch=64, tokens=64, warmup=8):
    """Cached decode of the 60M LM (`Mamba4LM.decode_step`, the reference's
    decode_step): `batch` sequences on each rank, one token per call, as one
    CUDA-graph replay (`GraphedDecoder`) and as eager launches. Returns
    generated tokens/s over all ranks (max-over-ranks device time) and the
    one-token latency of each."""
    import torch

    from mamba4_b200.model import CONFIGS, GraphedDecoder, Mamba4LM

    dev = torch.device("cuda", local)
    cfg = CONFIGS["60m"]
    torch.manual_seed(4321)
    model = Mamba4LM(cfg).to(dev).eval()
    g = torch.Generator(device=dev).manual_seed(77 + rank)
    ids = torch.randint(0, cfg.vocab_size, (tokens + warmup, batch), device=dev, generator=g)

    dec = GraphedDecoder(model, batch, device=dev)
    it = iter(range(tokens + warmup))
    graph_ms = max_over_ranks(time_region(lambda: dec.step(ids[next(it)]), tokens, warmup, world),
                              world) / tokens
    with torch.no_grad(), torch.autocast("cuda", dtype=torch.bfloat16):
        cache = model.init_cache(batch, device=dev)
        it = iter(range(tokens + warmup))

        def eager():
            nonlocal cache
            _, cache = model.decode_step(ids[next(it)], cache)

        eager_ms = max_over_ranks(time_region(eager, tokens, warmup, world), world) / tokens
    del model, cache, dec
    torch.cuda.empty_cache()
    return {"metric": "Mamba 4 60M cached decode tokens/s", "value": world * batch / (graph_ms / 1000.0),
            "unit": "tokens/s", "ms_per_token": graph_ms, "batch_per_gpu": batch, "tokens": tokens,
            "warmup": warmup, "launch": "one CUDA graph per token (GraphedDecoder)",
            "eager": {"value": world * batch / (eager_ms / 1000.0), "ms_per_token": eager_ms}}


def run_ours(args):
    import torch

    world, rank, local = setup_dist(args.gpus)
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    mem_cfg = {"small": SMALL_MEM_CFG, "profile": PROFILE_MEM_CFG}.get(args.workload, MEM_CFG)
    scan_cfg = PROFILE_SCAN_CFG if args.workload == "profile" else SCAN_CFG
    m = make_mem(mem_cfg, seed=1000 + rank, device=dev)
    s = make_scan(scan_cfg, seed=2000 + rank, device=dev)

    def step():
        memread_step(m)
        scan_step(s)

    with ClockSampler(local) as clocks:
        total_ms = time_region(step, args.steps, args.warmup, world)
    total_ms = max_over_ranks(total_ms, world)
    ms_per_step = total_ms / args.steps
    mem_tokens = mem_cfg["batch"] * mem_cfg["time"]
    scan_tokens = scan_cfg["batch"] * scan_cfg["time"]
    tokens = mem_tokens + scan_tokens
    value = world * tokens / (ms_per_step / 1000.0)

    # Per-op device times (rank-local) for the roofline and the components.
    from mamba4_b200 import selective_memory_fused

    mleaves = [m[n].detach().requires_grad_(True) for n in ("keys", "values", "queries", "beta", "log_decay")]

    def mfwd():
        return selective_memory_fused(*mleaves, m["floor"])

    def mbwd(res):
        torch.autograd.grad((res.output, res.variance), mleaves, (m["d_output"], m["d_variance"]))

    mem_fwd_ms, mem_bwd_ms = op_times(mfwd, mbwd)
    from mamba4_b200 import mamba3_fused

    names = ("c", "b", "x", "adt", "dt", "trap_logits", "angles", "q_bias", "k_bias")
    sleaves = [s[n].detach().requires_grad_(True) for n in names]

    def sfwd():
        return mamba3_fused(*sleaves[:7], q_bias=sleaves[7], k_bias=sleaves[8])

    def sbwd(out):
        torch.autograd.grad(out, sleaves, (s["d_y"], s["d_final"]))

    scan_fwd_ms, scan_bwd_ms = op_times(sfwd, sbwd)

    # End to end through the public API with host buffers, pipelined: step
    # i+1's inputs cross PCIe on a copy stream while step i computes, and
    # step i's results come back on a second copy stream (two device input
    # slots, two pinned output slots). Every step still copies all of its
    # inputs in and all of its results out inside the timed region.
    e2e = None
    if not args.no_e2e:
        e2e = measure_e2e_hotpath(m, s, dev, world, tokens, args)
    pk = peaks()
    token_heads = mem_tokens * mem_cfg["heads"]
    fwd_bytes = MEM_FWD_BYTES * token_heads
    achieved = fwd_bytes / (mem_fwd_ms / 1000.0) / 1e9
    mem_total_bytes = (MEM_FWD_BYTES + MEM_BWD_BYTES) * token_heads
    mem_flops = (MEM_FWD_FLOPS + MEM_BWD_FLOPS) * token_heads
    scan_ms = scan_fwd_ms + scan_bwd_ms
    traffic = None
    tpath = ROOT / "profiles" / "memread_traffic.json"
    if tpath.exists():
        traffic = json.loads(tpath.read_text()).get("memread_fwd_bytes_per_launch_c2")
    roofline = {
        "bound": "hbm", "kernel": "m4_memread_fwd (states + solve + output kernels)",
        "achieved": achieved, "peak": pk["hbm"], "unit": "GB/s", "frac": achieved / pk["hbm"],
        "traffic": traffic, "peak_source": pk["source"],
        "algorithmic_bytes": fwd_bytes,
        "fp32": {"tflops": MEM_FWD_FLOPS * token_heads / (mem_fwd_ms / 1000.0) / 1e12,
                 "nominal_peak_tflops": 74.4},
    }
    components = {
        "memread_c2": {"fwd_ms": mem_fwd_ms, "bwd_ms": mem_bwd_ms,
                       "tokens_per_s": mem_tokens / ((mem_fwd_ms + mem_bwd_ms) / 1000.0),
                       "hbm_frac": mem_total_bytes / ((mem_fwd_ms + mem_bwd_ms) / 1000.0) / 1e9 / pk["hbm"],
                       "fp32_tflops": mem_flops / ((mem_fwd_ms + mem_bwd_ms) / 1000.0) / 1e12},
        "scan_c1": {"fwd_ms": scan_fwd_ms, "bwd_ms": scan_bwd_ms,
                    "tokens_per_s": scan_tokens / (scan_ms / 1000.0),
                    "hbm_frac": SCAN_BYTES * scan_tokens / (scan_ms / 1000.0) / 1e9 / pk["hbm"],
                    "tensor_tflops": SCAN_FLOPS * scan_tokens / (scan_ms / 1000.0) / 1e12},
    }
    line = {
        "metric": "memory-read+scan tokens/s fwd+bwd", "value": value, "unit": "tokens/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_per_step,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32+bf16",
        "data": "synthetic",
        "config": hotpath_config(args.workload, mem_cfg, scan_cfg),
        "roofline": roofline, "components": components, "e2e": e2e,
        "gpu_launches": launches(step, args.steps), "clocks": clocks.summary(),
    }
    if rank == 0 and world == 1 and not args.no_cpu:
        rate, step_s, desc = cpu_baseline_sample(mem_cfg, scan_cfg, host_threads())
        line["cpu_baseline"] = {"value": rate, "unit": "tokens/s", "cores": host_threads(),
                                "kind": "port", "sample": f"{desc}; one timed step of {step_s:.2f} s"}
    if not args.no_lm and args.workload == "hotpath":
        # The second half of the metric: the data-parallel 60M LM training
        # step on the same ranks (one NCCL gradient all-reduce per step).
        del m, s
        step = e2e_step = None
        torch.cuda.empty_cache()
        line["lm60m"] = measure_lm(args, "lm60m", world, rank, local)
        # the 125M step (64 sequences per GPU) on the same ranks.
        line["lm125m"] = measure_lm(args, "lm125m", world, rank, local)
    if not args.no_decode and args.workload == "hotpath":
        line["decode"] = measure_decode(world, rank, local)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()


LM_PER_GPU = {"lm60m": 32, "lm125m": 64}
LM_SEQ = 1024


def lm_flops_per_token(cfg):
    """Model FLOPs per token for one training step (fwd + bwd): 6 x matmul
    parameters (in/out projections and the tied head) plus the two hot
    operators' survey figures (memory read 202,581 per token-head; scan
    1,835,008 per token at 16 heads, scaled by heads)."""
    s_layers = cfg.layer_pattern.count("S")
    m_layers = cfg.layer_pattern.count("M")
    h, n = cfg.num_heads, cfg.d_state
    angles = int(cfg.d_state * cfg.rope_fraction) // 2
    s_proj = cfg.d_model * (2 * cfg.inner + 2 * n + 3 * h + angles) + cfg.inner * cfg.d_model
    mh, d = cfg.memory_heads, cfg.key_dim
    m_proj = cfg.d_model * (2 * cfg.inner + 2 * mh * d + 3 * mh) + cfg.inner * cfg.d_model
    matmul = s_layers * s_proj + m_layers * m_proj + cfg.vocab_size * cfg.d_model
    # The scan's chunk products per token and head: 2 c N + 2 c P + 4 N P
    # (c = P = 64), i.e. the survey figure (N = 64) scaled by (192 N + 4096) / 16384.
    scan = SCAN_FLOPS * (h / 16) * (192 * n + 4096) / 16384
    return 6 * matmul + m_layers * mh * (MEM_FWD_FLOPS + MEM_BWD_FLOPS) + s_layers * scan


def measure_lm(args, workload, world, rank, local):
    """One data-parallel LM training step per iteration on this rank's shard;
    returns the JSON object (global tokens/s, max over ranks)."""
    import torch

    from mamba4_b200.model import CONFIGS, Mamba4LM
    from mamba4_b200.train import DataParallelTrainer, TrainSettings, synthetic_batch

    dev = torch.device("cuda", local)
    name = workload[2:]
    cfg = CONFIGS[name]
    per_gpu = args.lm_batch or LM_PER_GPU[workload]
    torch.manual_seed(1234)
    model = Mamba4LM(cfg).to(dev)
    trainer = DataParallelTrainer(model, TrainSettings(), world=world, device_id=local)
    tokens, targets, mask = synthetic_batch(per_gpu, LM_SEQ, cfg.vocab_size, seed=100 + rank, device=dev)

    def step():
        trainer.step(tokens, targets, mask)

    with ClockSampler(local) as clocks:
        total_ms = time_region(step, args.steps, args.warmup, world)
    total_ms = max_over_ranks(total_ms, world)
    ms_per_step = total_ms / args.steps
    tokens_per_step = world * per_gpu * LM_SEQ
    value = tokens_per_step / (ms_per_step / 1000.0)
    e2e = None
    if not args.no_e2e:
        host = [t.cpu().pin_memory() for t in (tokens, targets, mask)]
        loss_host = torch.empty((), dtype=torch.float32, pin_memory=True)

        def e2e_step():
            t, y, m = (h.to(dev, non_blocking=True) for h in host)
            loss, _, _ = trainer.step(t, y, m)
            loss_host.copy_(loss, non_blocking=True)

        e_ms = max_over_ranks(time_region(e2e_step, args.steps, args.warmup, world), world) / args.steps
        e2e = {"value": tokens_per_step / (e_ms / 1000.0), "unit": "tokens/s",
               "h2d_bytes_per_step": sum(h.numel() * h.element_size() for h in host),
               "d2h_bytes_per_step": 4, "ms_per_step": e_ms}
    pk = peaks()
    flops = lm_flops_per_token(cfg) * per_gpu * LM_SEQ / (ms_per_step / 1000.0) / 1e12
    line = {
        "metric": f"Mamba 4 {name.upper()} train tokens/s", "value": value, "unit": "tokens/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_per_step,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (uniform-random token ids)",
        "config": {"workload": "configs[3]" if name == "60m" else "configs[4]", "model": f"mamba4-{name}",
                   "global_batch": world * per_gpu, "seq_len": LM_SEQ, "parallelism": f"dp{world}",
                   "layer_pattern": cfg.layer_pattern, "d_model": cfg.d_model, "vocab": cfg.vocab_size,
                   "l2": "activations and stored factors far exceed L2"},
        "roofline": {"bound": "tensor", "kernel": "whole training step (model FLOPs utilisation)",
                     "achieved": flops, "peak": pk["bf16_sust"], "unit": "TFLOP/s",
                     "frac": flops / pk["bf16_sust"], "traffic": None, "peak_source": pk["source"]},
        "e2e": e2e, "clocks": clocks.summary(),
        "gpu_launches": launches(step, args.steps),
    }
    del trainer, model
    torch.cuda.empty_cache()
    return line


def run_lm(args):
    import torch

    world, rank, local = setup_dist(args.gpus)
    torch.cuda.set_device(local)
    line = measure_lm(args, args.workload, world, rank, local)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()


def run_decode(args):
    import torch

    world, rank, local = setup_dist(args.gpus)
    torch.cuda.set_device(local)
    line = measure_decode(world, rank, local, batch=args.lm_batch or 64)
    line.update(n_gpus=world, higher_is_better=True, scaling="weak", vs_baseline=None, dtype="bf16",
                data="synthetic (uniform-random token ids)", config={"workload": "60M cached decode"})
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()


def main():
    p = argparse.ArgumentParser(description=__doc__)
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=10)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--workload", choices=["hotpath", "small", "profile", "lm60m", "lm125m", "decode"], default="hotpath")
    p.add_argument("--lm-batch", type=int, default=0,
                   help="LM workloads: sequences per GPU (default: the configuration's; smaller for ncu captures)")
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--no-cpu", action="store_true")
    p.add_argument("--no-decode", action="store_true",
                   help="hot-path workload: skip the cached-decode measurement of the 60M LM")
    p.add_argument("--no-lm", action="store_true",
                   help="hot-path workload: skip the nested data-parallel 60M and 125M LM step measurements")
    args = p.parse_args()
    if args.impl == "reference":
        run_reference(args)
    elif args.workload.startswith("lm"):
        run_lm(args)
    elif args.workload == "decode":
        run_decode(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
