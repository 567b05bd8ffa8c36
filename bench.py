#!/usr/bin/env python
"""Fused optimizer-step benchmark: Gparams/s and fraction of the HBM roofline on B200.

Workload (BASELINE.json metric): a Llama-7B-shaped parameter set (hidden 4096, 32 layers, MLP 11008,
vocab 32000, untied: 291 tensors, 6,738,415,616 parameters), bf16 weights with an fp32 master, AdamW with
bf16 moments (stochastic rounding on), bf16 gradients.  One step = one optimizer step over every parameter:
the fused update kernels (20 algorithmic bytes per parameter: master r/w 8, grad 2, m r/w 4, v r/w 4, bf16
weight 2) plus, on N > 1 GPUs, the NCCL all-gather of the new bf16 weights (ZeRO-1, fixed model: strong
scaling).  Synthetic data: weights ~ N(0, 0.02), gradients ~ N(0, 1e-3) from seeded generators.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl abx|reference]

``--impl reference`` times the reference's own CPU kernel library (oracle/_ref, compiled from the
reference sources) on the host cores, on a bounded sample of the same workload.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

LLAMA7B = dict(hidden=4096, layers=32, mlp=11008, vocab=32000, kv=4096)
BYTES_PER_PARAM = {("adamw", "bf16"): 20, ("adamw", "fp32"): 28, ("adamw", "fp8"): 16.125,
                   ("lion", "bf16"): 16, ("lion", "fp32"): 20, ("lion", "fp8"): 14.0625}
# DRAM bytes (read + write) per parameter of the update kernel, from one ncu capture of the small Llama case
# (1 layer, vocab 8000: 267,923,456 parameters); the traffic of a launch grows with its parameters, so the
# full-size figure is this times the parameters a step updates.
MEASURED_DRAM_BYTES_PER_PARAM = {("adamw", "bf16"): (2.679388e9 + 2.622009e9) / 267923456,
                                 ("adamw", "fp8"): (2.160363e9 + 2.111521e9) / 267923456}
# How the new weights reach the other ranks (ZeroAdamBridge.gather), as the bench line names it.
GATHER_LABELS = {None: None, "p2p": "fused peer stores", "ce": "copy-engine peer copies", "nccl": "nccl"}


def llama_shapes(hidden, layers, mlp, vocab, kv, tied=False):
    """Parameter shapes in the optimizer order of a Llama decoder (embedding, layers, final norm, lm_head)."""
    shapes = [(vocab, hidden)]
    for _ in range(layers):
        shapes += [(hidden, hidden), (kv, hidden), (kv, hidden), (hidden, hidden), (mlp, hidden), (mlp, hidden),
                   (hidden, mlp), (hidden,), (hidden,)]
    shapes.append((hidden,))
    if not tied:
        shapes.append((vocab, hidden))
    return shapes


def numel(shape):
    n = 1
    for d in shape:
        n *= d
    return n


# --------------------------------------------------------------------------- clocks

class ClockSampler:
    """SM clock and clock-event (throttle) reasons of one GPU, sampled through NVML every 10 ms on a thread
    while the timed region runs (read-only queries; nothing is set)."""

    REASONS = {"hw_slowdown": "nvmlClocksEventReasonHwSlowdown",
               "hw_thermal_slowdown": "nvmlClocksEventReasonHwThermalSlowdown",
               "sw_thermal_slowdown": "nvmlClocksEventReasonSwThermalSlowdown",
               "sw_power_cap": "nvmlClocksEventReasonSwPowerCap"}

    def __init__(self, index: int, period: float = 0.01):
        self.index, self.period = index, period
        self.mhz, self.reasons, self.max_mhz = [], set(), None

    def _loop(self):
        import pynvml
        h = pynvml.nvmlDeviceGetHandleByIndex(self.index)
        self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM)
        bits = {name: getattr(pynvml, attr) for name, attr in self.REASONS.items()}
        while not self._stop.is_set():
            self.mhz.append(pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM))
            active = pynvml.nvmlDeviceGetCurrentClocksEventReasons(h)
            self.reasons.update(name for name, bit in bits.items() if active & bit)
            self._ready.set()
            self._stop.wait(self.period)

    def __enter__(self):
        import threading
        self._stop = threading.Event()
        self._ready = threading.Event()
        self._thread = None
        try:
            import pynvml
            pynvml.nvmlInit()
            self._thread = threading.Thread(target=self._loop, daemon=True)
            self._thread.start()
            self._ready.wait(5.0)   # the sampler is running before the timed region starts
            self.mhz.clear()        # ... and only samples taken inside it are kept
            self.reasons.clear()
        except Exception:  # noqa: BLE001 -- no NVML: the line reports no samples
            self._thread = None
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._thread is not None:
            self._thread.join(timeout=2)

    def summary(self) -> dict:
        return {"sm_mhz": statistics.median(self.mhz) if self.mhz else None, "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.mhz)}


# --------------------------------------------------------------------------- CPU baseline

def metric_name(algo: str, prec: str) -> str:
    """The metric string of a bench line (the same on the repo's arm and the reference arm)."""
    if (algo, prec) == ("adamw", "bf16"):
        return "fused step Gparams/s and % of HBM roofline (7B, bf16 moments)"
    return f"fused step Gparams/s ({algo}, {prec} moments)"


def workload_name(dims: dict, algo: str, prec: str, clip: float | None) -> str:
    name = (f"llama7b-{algo}-{prec}-moments" if dims == LLAMA7B else
            f"llama-{dims['layers']}L-v{dims['vocab']}-{algo}-{prec}-moments")
    return name + ("" if clip is None else f"-clip{clip:g}")


def default_reference_threads() -> int:
    """The reference's default pool size: two thirds of the usable cores, at most 32 (adambridge/engine.py:635)."""
    return max(1, min(32, (2 * len(os.sched_getaffinity(0))) // 3))


def cpu_reference_sample(seconds: float = 10.0, steps: int | None = None, warmup: int = 1, algo: str = "adamw",
                         prec: str = "bf16", threads: int | None = None, simd: str | None = None):
    """Time the reference's own kernel library (oracle/_ref) -- or, where it was not built, the oracle port --
    on one Llama-7B decoder layer's seven matrices (202,375,168 params; moments in ``prec``, bf16 grad and
    weights, fp32 master), on ``threads`` host threads (default: every usable core) at SIMD level ``simd``
    (default: the best this CPU runs).  Returns (Gparams/s, threads, kind, sample description, ms per step)."""
    import numpy as np

    from oracle import oracle as O

    ref = O.load_reference()
    kind = "reference" if ref is not None else "port"
    if ref is None:
        threads = 1
    elif threads is None:
        threads = len(os.sched_getaffinity(0))
    h, mlp = LLAMA7B["hidden"], LLAMA7B["mlp"]
    shapes = [(h, h)] * 4 + [(mlp, h)] * 3
    if ref is None:
        shapes = [(h, h)]   # the single-threaded port gets a smaller sample
    mv = {"fp32": O.DT_F32, "bf16": O.DT_BF16, "fp8": O.DT_FP8}[prec]
    alg = O.LION if algo == "lion" else O.ADAMW
    rng = np.random.default_rng(0)
    segs, keep = [], []
    group = (O.Group(lr=1e-5, beta1=0.9, beta2=0.99, eps=0.0, weight_decay=0.1, seed=0, stochastic=1) if alg == O.LION
             else O.Group(lr=1e-4, beta1=0.9, beta2=0.999, eps=1e-8, weight_decay=0.01, seed=0, stochastic=1))
    for i, shp in enumerate(shapes):
        n = numel(shp)
        hs = O.HostSegment(n, O.DT_BF16, mv, O.DT_BF16, O.DT_F32, alg, index=i)
        mlen = hs.moment_len()
        mdt = {O.DT_F32: np.float32, O.DT_BF16: np.uint16, O.DT_FP8: np.uint8}[mv]
        hs.buffers = {"p": (rng.standard_normal(n, dtype=np.float32) * 0.02),
                      "g": O.bf16_bits(rng.standard_normal(n, dtype=np.float32) * 1e-3),
                      "m": np.zeros(mlen, mdt), "out": np.zeros(n, np.uint16)}
        if alg == O.ADAMW:
            hs.buffers["v"] = np.zeros(mlen, mdt)
        if mv == O.DT_FP8:
            hs.buffers["m_scale"] = np.ones(hs.nblocks, np.float32)
            if alg == O.ADAMW:
                hs.buffers["v_scale"] = np.ones(hs.nblocks, np.float32)
        keep.append(hs)
        segs.append(hs.ctype(group))
    total = sum(s.n for s in segs)
    arr = O.seg_array(segs)
    orc = None if ref is not None else O.load_oracle()
    level = None
    if ref is not None:
        saved_level = ref.simd_level
        if simd is not None:
            ref.set_simd_level({v: k for k, v in O.SIMD_NAMES.items()}[simd])
        level = O.SIMD_NAMES[ref.simd_level]

    def one(step):
        for s in segs:
            s.step = step
        rc = ref.multi_step_array(arr, threads) if ref is not None else orc.multi_step(segs, O.SIMD_AVX512)
        if rc != 0:
            raise RuntimeError(f"CPU baseline update failed ({rc})")

    try:
        step = 0
        for _ in range(warmup):
            step += 1
            one(step)
        times = []
        t_end = time.perf_counter() + seconds
        while (steps is None and time.perf_counter() < t_end) or (steps is not None and len(times) < steps):
            step += 1
            t0 = time.perf_counter()
            one(step)
            times.append(time.perf_counter() - t0)
    finally:
        if ref is not None:
            ref.set_simd_level(saved_level)
    med = statistics.median(times)
    del keep
    desc = (f"{len(shapes)} tensors of one Llama-7B layer ({total:,} params), {algo} {prec} moments, bf16 grad/out, "
            f"{len(times)} steps, median; simd={level or 'port'}")
    return total / med / 1e9, threads, kind, desc, med * 1e3


def cpu_baseline_block(args) -> dict:
    """The reference's CPU path on this host for the bench line: the headline sample on every usable core, plus
    the variants a reference user would run -- its default pool (2/3 of the cores, at most 32), the same mode at
    the forced AVX2 level, and the FP8 mode -- each bounded to a few seconds."""
    algo, prec = args.algorithm, args.precision
    gps, threads, kind, desc, _ = cpu_reference_sample(seconds=args.cpu_seconds, algo=algo, prec=prec)
    block = {"value": round(gps, 4), "unit": "Gparams/s", "cores": threads, "kind": kind, "sample": desc}
    if kind != "reference" or args.cpu_variant_seconds <= 0:
        return block
    variants = []
    wanted = [dict(threads=default_reference_threads(), algo=algo, prec=prec, simd=None, why="reference default pool"),
              dict(threads=None, algo=algo, prec=prec, simd="avx2", why="forced avx2")]
    if prec != "fp8":
        wanted += [dict(threads=None, algo=algo, prec="fp8", simd=None, why="fp8 moments"),
                   dict(threads=None, algo=algo, prec="fp8", simd="avx2", why="fp8 moments, forced avx2")]
    for w in wanted:
        try:
            v_gps, v_threads, _, v_desc, _ = cpu_reference_sample(seconds=args.cpu_variant_seconds, algo=w["algo"],
                                                                 prec=w["prec"], threads=w["threads"], simd=w["simd"])
        except Exception as exc:  # noqa: BLE001 -- a variant this CPU cannot run (no AVX2) is reported, not fatal
            variants.append({"variant": w["why"], "error": str(exc)})
            continue
        variants.append({"variant": w["why"], "value": round(v_gps, 4), "unit": "Gparams/s", "cores": v_threads,
                         "sample": v_desc})
    block["variants"] = variants
    return block


def reference_arm(args, rank: int, world: int) -> None:
    """--impl reference: the reference's CPU implementation on this host, rank 0 only, on the same metric,
    workload and unit as the repo's arm."""
    if rank != 0:
        return
    algo, prec = args.algorithm, args.precision
    gps, threads, kind, desc, ms = cpu_reference_sample(steps=args.steps, warmup=args.warmup, algo=algo, prec=prec)
    dims = dict(LLAMA7B)
    line = {"impl": "reference", "metric": metric_name(algo, prec), "value": round(gps, 4),
            "unit": "Gparams/s", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms, 3), "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "f32", "data": "synthetic",
            "config": {"workload": workload_name(dims, algo, prec, None), "parallelism": "host threads",
                       "sample": "each step updates one Llama-7B decoder layer's matrices; Gparams/s is its rate"},
            "cpu_baseline": {"value": round(gps, 4), "unit": "Gparams/s", "cores": threads, "kind": kind,
                             "sample": desc},
            "e2e": {"value": round(gps, 4), "unit": "Gparams/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def torch_fused_adamw_rate(dims: dict, steps: int, warmup: int, dev) -> dict:
    """The reference's only GPU update, its gpu_state_budget path (adambridge/optimizer.py:364-430, _step_gpu), on
    the parameter set ``dims``: FP32 master weights and moments on the GPU, each bf16 gradient converted with
    grad.to(float32), torch.optim.AdamW(fused=True), then torch._foreach_copy_ of the masters into the bf16
    weights.  CUDA events; returns the rate, the time and the roofline of the bytes that path moves."""
    import torch
    shapes = llama_shapes(**dims)
    n_params = sum(numel(sh) for sh in shapes)
    gen = torch.Generator(device=dev).manual_seed(1234)
    weights, masters, grads = [], [], []
    with torch.no_grad():
        for sh in shapes:
            w = torch.empty(sh, dtype=torch.bfloat16, device=dev).normal_(0.0, 0.02, generator=gen)
            weights.append(w)
            masters.append(torch.nn.Parameter(w.float()))
            grads.append(torch.empty(sh, dtype=torch.bfloat16, device=dev).normal_(0.0, 1e-3, generator=gen))
    inner = torch.optim.AdamW(masters, lr=2e-5, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.01, fused=True)

    def step():
        for mp, g in zip(masters, grads):
            mp.grad = g.to(torch.float32)
        inner.step()
        torch._foreach_copy_(weights, masters)
        for mp in masters:
            mp.grad = None

    for _ in range(warmup):
        step()
    torch.cuda.synchronize(dev)
    cur = torch.cuda.current_stream(dev)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(dev.index or 0) as clocks:
        t0.record(cur)
        for _ in range(steps):
            step()
        t1.record(cur)
        torch.cuda.synchronize(dev)
    ms = t0.elapsed_time(t1) / steps
    del inner, masters, grads, weights
    torch.cuda.empty_cache()
    # bytes the path moves: grad bf16 read + fp32 write, fused AdamW (p, g, m, v read; p, m, v written, fp32),
    # master read + bf16 weight write
    bpp = 2 + 4 + 7 * 4 + 4 + 2
    peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()) if (ROOT / "MEASURED_PEAKS.json").exists() else {}
    peak = peaks.get("hbm_gbs", 6650.0)
    achieved = bpp * n_params / (ms / 1e3) / 1e9
    return {"value": round(n_params / (ms / 1e3) / 1e9, 4), "unit": "Gparams/s", "ms_per_step": round(ms, 3),
            "steps": steps, "params": n_params,
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4),
                         "basis": f"{bpp} B/param moved by grad.to(fp32) + fused AdamW + _foreach_copy_"},
            "clocks": clocks.summary(),
            "path": "the reference's gpu_state_budget update: fp32 state on the GPU, grad.to(float32), "
                    "torch.optim.AdamW(fused=True), torch._foreach_copy_ into the bf16 weights"}


def reference_gpu_arm(args, rank: int) -> None:
    """--impl reference-gpu: torch_fused_adamw_rate on the 7B set as its own line (rank 0 only).  The default
    N = 1 run of the repo's arm also reports it, as ``reference_gpu_update``."""
    if rank != 0:
        return
    import torch
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    dims = dict(LLAMA7B)
    if args.layers is not None:
        dims["layers"] = args.layers
    if args.vocab is not None:
        dims["vocab"] = args.vocab
    r = torch_fused_adamw_rate(dims, args.steps, args.warmup, dev)
    line = {"impl": "reference-gpu", "metric": "fused step Gparams/s (7B, the reference's GPU update)",
            "value": r["value"], "unit": "Gparams/s", "n_gpus": 1, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": r["ms_per_step"], "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": "llama7b-adamw-fp32-state-torch-fused (gpu_state_budget path)",
                       "params": r["params"]},
            "roofline": r["roofline"], "clocks": r["clocks"]}
    print(json.dumps(line), flush=True)


# --------------------------------------------------------------------------- training workload (config 5)

def train_arm(args, rank: int, world: int, local_rank: int) -> dict | None:
    """--workload train: the end-to-end training step of the reference's config 5 (with ``--delay``, its
    delayed-update variant) -- a random-init Llama-7B
    decoder (bf16 weights, activation checkpointing per layer), batch 8 x sequence 512 of uniform token ids per
    rank, ZeroAdamBridge (AdamW, bf16 moments) with its backward hooks reduce-scattering each round of
    gradients while backward runs, then the fused update + all-gather.  Prints tokens/s for the whole job and
    the update kernels' share of the step."""
    import torch
    import torch.distributed as dist
    import torch.nn.functional as F
    from torch.utils.checkpoint import checkpoint

    from adambridge_b200 import native
    from adambridge_b200.zero import ZeroAdamBridge

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    kern = native.load()
    dims = dict(LLAMA7B)
    if args.layers is not None:
        dims["layers"] = args.layers
    if args.vocab is not None:
        dims["vocab"] = args.vocab
    hidden, vocab, heads = dims["hidden"], dims["vocab"], 32
    hd = hidden // heads
    batch, seq = 8, 512

    class RMSNorm(torch.nn.Module):
        def __init__(self):
            super().__init__()
            self.weight = torch.nn.Parameter(torch.ones(hidden))

        def forward(self, x):
            xf = x.float()
            return (xf * torch.rsqrt(xf.square().mean(-1, keepdim=True) + 1e-5)).to(x.dtype) * self.weight

    class Block(torch.nn.Module):
        def __init__(self):
            super().__init__()
            lin = lambda o, i: torch.nn.Linear(i, o, bias=False)   # noqa: E731
            self.q, self.k, self.v, self.o = lin(hidden, hidden), lin(dims["kv"], hidden), lin(dims["kv"], hidden), lin(hidden, hidden)
            self.gate, self.up, self.down = lin(dims["mlp"], hidden), lin(dims["mlp"], hidden), lin(hidden, dims["mlp"])
            self.norm1, self.norm2 = RMSNorm(), RMSNorm()

        def forward(self, x, cos, sin):
            b, t, _ = x.shape
            h = self.norm1(x)

            def rope(z):
                z = z.view(b, t, -1, hd).transpose(1, 2)
                z1, z2 = z[..., : hd // 2], z[..., hd // 2:]
                return torch.cat((z1 * cos - z2 * sin, z2 * cos + z1 * sin), dim=-1)

            att = F.scaled_dot_product_attention(rope(self.q(h)), rope(self.k(h)),
                                                 self.v(h).view(b, t, -1, hd).transpose(1, 2), is_causal=True)
            x = x + self.o(att.transpose(1, 2).reshape(b, t, hidden))
            h = self.norm2(x)
            return x + self.down(F.silu(self.gate(h)) * self.up(h))

    class Decoder(torch.nn.Module):
        def __init__(self):
            super().__init__()
            self.emb = torch.nn.Embedding(vocab, hidden)
            self.blocks = torch.nn.ModuleList(Block() for _ in range(dims["layers"]))
            self.norm = RMSNorm()
            self.lm_head = torch.nn.Linear(hidden, vocab, bias=False)

        def forward(self, tokens):
            pos = torch.arange(tokens.shape[1], device=tokens.device, dtype=torch.float32)
            inv = 1.0 / (10000.0 ** (torch.arange(0, hd, 2, device=tokens.device, dtype=torch.float32) / hd))
            ang = torch.outer(pos, inv)
            cos, sin = ang.cos().to(torch.bfloat16), ang.sin().to(torch.bfloat16)
            x = self.emb(tokens)
            for blk in self.blocks:
                x = checkpoint(blk, x, cos, sin, use_reentrant=False)
            return self.lm_head(self.norm(x))

    torch.manual_seed(0)   # the same initial weights on every rank
    with torch.device(dev):
        model = Decoder().to(torch.bfloat16)
    n_params = sum(p.numel() for p in model.parameters())
    opt = ZeroAdamBridge(list(model.parameters()), lr=2e-5, precision="bf16", rounds=args.rounds or 32,
                         gather=args.gather, delay_updates=args.delay, max_ctas=args.max_ctas)
    opt.attach_hooks(model, update_in_backward=not args.update_at_step,
                     backward_max_ctas=args.max_ctas if args.max_ctas > 0 else None)
    gen = torch.Generator(device=dev).manual_seed(1000 + rank)
    tokens = torch.randint(0, vocab, (batch, seq + 1), device=dev, generator=gen)
    marks = []   # (backward's GPU work done, step done) events of every timed step

    def step():
        logits = model(tokens[:, :-1])
        loss = F.cross_entropy(logits.float().reshape(-1, vocab), tokens[:, 1:].reshape(-1))
        loss.backward()
        b = torch.cuda.Event(enable_timing=True)
        b.record(torch.cuda.current_stream(dev))
        opt.step()
        e = torch.cuda.Event(enable_timing=True)
        e.record(torch.cuda.current_stream(dev))
        marks.append((b, e))
        return loss

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    launches0 = kern.launch_count()
    opt.trace = []
    marks.clear()
    cur = torch.cuda.current_stream(dev)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local_rank) as clocks:
        t0.record(cur)
        for _ in range(args.steps):
            loss = step()
        t1.record(cur)
        torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    ms = t0.elapsed_time(t1) / args.steps
    upd_ms = sum(a.elapsed_time(b) for a, b in opt.trace) / args.steps
    exposed_ms = sum(b.elapsed_time(e) for b, e in marks) / args.steps
    opt.trace = None
    t = torch.tensor([ms, upd_ms, exposed_ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms, upd_ms, exposed_ms = t.tolist()
    loss_host = float(loss.detach().float().item())
    if rank != 0:
        return None
    tokens_per_step = batch * seq * world
    line = {"metric": "training step tokens/s (Llama-7B decoder, ZeRO-1 AdamW bf16 moments, hooks)",
            "value": round(tokens_per_step / (ms / 1e3), 1), "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 2), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": "llama-train-c5" if dims == LLAMA7B else f"llama-{dims['layers']}L-train",
                       "params": n_params, "batch_per_rank": batch, "seq_len": seq, "activation_checkpointing": True,
                       "hooks": True, "delay_updates": args.delay, "parallelism": f"zero1-dp{world}",
                       "rounds": opt.layout.rounds,
                       "all_gather": GATHER_LABELS[opt.gather]},
            "update_kernels_ms": round(upd_ms, 3),
            "exposed_update_ms": round(exposed_ms, 3),
            "exposed_basis": "per step, from the end of backward's GPU work (an event after loss.backward()) to the "
                             "end of opt.step() on the compute stream: the part of the update and all-gather the "
                             "step waits for; max over ranks",
            "update_in_backward": not args.update_at_step and not args.delay,
            "loss": round(loss_host, 4),
            "gpu_launches": kern.launch_count() - launches0, "clocks": clocks.summary()}
    return line


# --------------------------------------------------------------------------- state conversion

CONVERT_BYTES = {"fp32": 4.0, "bf16": 2.0, "fp8": 1.0 + 4.0 / 128, "fp24": 3.0}


def convert_arm(args, rank: int, world: int, local_rank: int) -> dict | None:
    """--workload convert: libabx's state-format conversion kernel (abx_convert) re-encoding the second moment of
    the 7B parameter set -- 6,738,415,616 values -- from ``--convert-from`` to ``--precision`` (what
    ``set_precision`` does to every moment), one launch per tensor, CUDA events.  Algorithmic bytes: the source
    read plus the destination written (fp32 4, bf16 2, fp8 1 + 4/128 per value)."""
    import torch

    from adambridge_b200 import native
    from adambridge_b200.precision import StateBuffer

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    kern = native.load()
    dims = dict(LLAMA7B)
    if args.layers is not None:
        dims["layers"] = args.layers
    if args.vocab is not None:
        dims["vocab"] = args.vocab
    sizes = [numel(s) for s in llama_shapes(**dims)]
    total = sum(sizes)
    src_fmt, dst_fmt = args.convert_from, args.precision
    gen = torch.Generator(device=dev).manual_seed(77)
    srcs, dsts = [], []
    with torch.no_grad():
        for n in sizes:
            v = torch.empty(n, device=dev).exponential_(generator=gen).mul_(1e-6)   # v >= 0, like a second moment
            srcs.append(StateBuffer.converted(v, src_fmt, "v", dev))
            del v
            dsts.append(StateBuffer.allocate(dst_fmt, "v", n, dev))
    cur = torch.cuda.current_stream(dev)

    def once():
        for s, d in zip(srcs, dsts):
            d.assign(s)

    for _ in range(args.warmup):
        once()
    torch.cuda.synchronize()
    launches0 = kern.launch_count()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local_rank) as clocks:
        a.record(cur)
        for _ in range(args.steps):
            once()
        b.record(cur)
        torch.cuda.synchronize()
    ms = a.elapsed_time(b) / args.steps
    launches = kern.launch_count() - launches0
    if rank != 0:
        return None
    bpv = CONVERT_BYTES[src_fmt] + CONVERT_BYTES[dst_fmt]
    peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()) if (ROOT / "MEASURED_PEAKS.json").exists() else {}
    peak = peaks.get("hbm_gbs", 6650.0)
    achieved = bpv * total / (ms / 1e3) / 1e9
    return {"metric": f"state conversion Gvalues/s ({src_fmt} -> {dst_fmt} moments)",
            "value": round(total / (ms / 1e3) / 1e9, 3), "unit": "Gvalues/s", "n_gpus": 1, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms, 3), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": f"llama7b-second-moment-{src_fmt}-to-{dst_fmt}", "values": total,
                       "tensors": len(sizes), "l2": "no flush: %.1f GB per step >> 126 MB L2" % (bpv * total / 1e9)},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4),
                         "basis": f"{bpv:g} B/value (source read + destination written) x {total:,} values / "
                                  "conversion time (CUDA events), one abx_convert launch per tensor; peak = "
                                  + ("MEASURED_PEAKS.json hbm_gbs (of measured)" if "hbm_gbs" in peaks
                                     else "6650 GB/s (of fallback)")},
            "gpu_launches": launches, "clocks": clocks.summary()}


# --------------------------------------------------------------------------- multi-GPU checks

def sharded_parity(args, world: int, rank: int, dev) -> dict:
    """After the timed region: is the sharded step the unsharded one, bit for bit, on this node?

    A sample of the 7B set's tensors -- the embedding and the lm_head (each split over ranks), a 4096^2 and
    both MLP shapes, two norms -- gets two optimizer steps from a ZeroAdamBridge / ZeroLionBridge of this
    world (the bench's gather mode and precision; gradients handed in as each rank's shard) and from a
    world-1 AdamBridge / LionBridge on a copy of the same tensors (the same gradients, whole).  Every rank
    then compares the weights it holds after the all-gather (every element of every sampled tensor, so
    every peer's stores into this rank are checked) and its own shard of the master and the moments with the
    unsharded optimizer's.  Mismatch counts are summed over the ranks."""
    import torch
    import torch.distributed as dist

    from adambridge_b200 import AdamBridge, LionBridge
    from adambridge_b200.zero import ZeroAdamBridge, ZeroLionBridge

    h, mlp, vocab = LLAMA7B["hidden"], LLAMA7B["mlp"], LLAMA7B["vocab"]
    shapes = [(vocab, h), (h, h), (h,), (mlp, h), (h, mlp), (h,), (vocab, h)]
    algo, prec = args.algorithm, args.precision
    kw = dict(lr=1e-5, betas=(0.9, 0.99), weight_decay=0.1) if algo == "lion" else \
        dict(lr=2e-5, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.01)
    gen = torch.Generator(device=dev).manual_seed(4321)      # the same tensors on every rank
    with torch.no_grad():
        init = [torch.empty(s, dtype=torch.bfloat16, device=dev).normal_(0.0, 0.02, generator=gen) for s in shapes]
    zparams = [torch.nn.Parameter(w.clone()) for w in init]
    aparams = [torch.nn.Parameter(w.clone()) for w in init]
    del init
    zcls, acls = (ZeroLionBridge, LionBridge) if algo == "lion" else (ZeroAdamBridge, AdamBridge)
    zopt = zcls(zparams, precision=prec, gather=args.gather, max_ctas=args.max_ctas, **kw)
    aopt = acls(aparams, precision=prec, **kw)
    L = zopt.layout
    pieces = [pc for rnd in zopt._pieces for pc in rnd]
    for step in range(2):
        gen = torch.Generator(device=dev).manual_seed(9000 + step)
        with torch.no_grad():
            grads = [torch.empty(s, dtype=torch.bfloat16, device=dev).normal_(0.0, 1e-3, generator=gen)
                     for s in shapes]
            for pc in pieces:
                zopt.grad_shard[pc.local_lo:pc.local_lo + pc.n].copy_(grads[pc.index].view(-1)[pc.t_lo:pc.t_hi])
        zopt.step_shard()
        for p, g in zip(aparams, grads):
            p.grad = g
        aopt.step()
        aopt.zero_grad(set_to_none=True)
    torch.cuda.synchronize(dev)

    def bits(t):
        return t.view({1: torch.uint8, 2: torch.int16, 4: torch.int32}[t.element_size()])

    checked = torch.zeros(2, dtype=torch.int64, device=dev)    # (elements compared, mismatches)
    with torch.no_grad():
        for zp, ap in zip(zparams, aparams):
            checked[0] += zp.numel()
            checked[1] += (bits(zp.detach()) != bits(ap.detach())).sum()
        zstores = [("master", zopt.master), ("m", zopt.m)] + ([] if zopt.v is None else [("v", zopt.v)])
        for pc in pieces:
            slot = aopt.slots[pc.index]
            for name, zst in zstores:
                ast = getattr(slot, name)
                zbuf, zsc = zst.operands
                abuf, asc = ast.operands
                for a, b in ((zbuf[pc.local_lo:pc.local_lo + pc.n], abuf[pc.t_lo:pc.t_hi]),
                             (zsc[pc.local_lo // 128:-(-(pc.local_lo + pc.n) // 128)] if zsc is not None else None,
                              asc[pc.t_lo // 128:-(-pc.t_hi // 128)] if asc is not None else None)):
                    if a is None:
                        continue
                    checked[0] += a.numel()
                    checked[1] += (bits(a) != bits(b)).sum()
    if world > 1:
        dist.all_reduce(checked)
    straddling = sum(1 for i in range(len(shapes))
                     if len({r for r in range(world) for rnd in L.pieces(r) for pc in rnd if pc.index == i}) > 1)
    n_checked, n_bad = (int(x) for x in checked.tolist())
    gather = GATHER_LABELS[zopt.gather]
    del zopt, aopt, zparams, aparams
    torch.cuda.empty_cache()
    return {"checked": n_checked, "mismatches": n_bad, "tensors": len(shapes), "split_over_ranks": straddling,
            "steps": 2, "against": f"world-1 {acls.__name__} on the same tensors and gradients",
            "gather": gather}


def host_link_gbs(host_g, host_w, opt, world: int, dev, iters: int = 3) -> dict:
    """What the host link alone moves for this rank, every rank copying at once (the same pinned buffers and
    bytes as the end-to-end step, no update): host->device, device->host, and both directions together.  GB/s
    per rank, the slowest rank's time; the end-to-end step cannot beat the 'both' figure."""
    import torch
    import torch.distributed as dist

    h2d_s, d2h_s = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    src_w = opt.flat_weights[:host_w.numel()]

    def timed(up: bool, down: bool) -> float:
        torch.cuda.synchronize(dev)
        if world > 1:
            dist.barrier()
        cur = torch.cuda.current_stream(dev)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(cur)
        for s in (h2d_s, d2h_s):
            s.wait_event(a)
        for _ in range(iters):
            if up:
                with torch.cuda.stream(h2d_s):
                    opt.grad_shard.copy_(host_g, non_blocking=True)
            if down:
                with torch.cuda.stream(d2h_s):
                    host_w.copy_(src_w, non_blocking=True)
        cur.wait_stream(h2d_s)
        cur.wait_stream(d2h_s)
        b.record(cur)
        torch.cuda.synchronize(dev)
        ms = torch.tensor([a.elapsed_time(b) / iters], dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(ms, op=dist.ReduceOp.MAX)
        return ms.item()

    gb = host_g.numel() * host_g.element_size() / 1e9
    up, down, both = timed(True, False), timed(False, True), timed(True, True)
    return {"h2d_gbs": round(gb / (up / 1e3), 1), "d2h_gbs": round(gb / (down / 1e3), 1),
            "both_directions_gbs_each": round(gb / (both / 1e3), 1), "ranks_copying": world,
            "basis": f"{gb:.2f} GB each way per rank from/to pinned host memory, CUDA events, max over ranks"}


def nccl_allgather_gbs(opt, world: int, dev, iters: int = 5) -> float:
    """NVLink ingress per rank (GB/s) that NCCL's in-place all-gather reaches on the step's own weight buffer
    (every rank receives (world - 1) x its shard): the reference rate for the fused all-gather."""
    import torch
    import torch.distributed as dist

    L = opt.layout
    buf = opt.flat_weights
    mine = [buf[slice(*L.rank_range(r, opt.rank))] for r in range(L.rounds)]
    outs = [buf[slice(*L.round_range(r))] for r in range(L.rounds)]
    cur = torch.cuda.current_stream(dev)

    def once():
        for out, m in zip(outs, mine):
            dist.all_gather_into_tensor(out, m)

    once()
    torch.cuda.synchronize(dev)
    dist.barrier()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(cur)
    for _ in range(iters):
        once()
    b.record(cur)
    torch.cuda.synchronize(dev)
    ms = torch.tensor([a.elapsed_time(b) / iters], dtype=torch.float64, device=dev)
    dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    received = (world - 1) * L.chunk * L.rounds * buf.element_size()
    return received / (ms.item() / 1e3) / 1e9


# --------------------------------------------------------------------------- GPU arm

def gpu_arm(args, rank: int, world: int, local_rank: int) -> dict | None:
    import torch
    import torch.distributed as dist

    from adambridge_b200 import native
    from adambridge_b200.zero import ZeroAdamBridge, ZeroLionBridge

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    kern = native.load()
    dims = dict(LLAMA7B)
    if args.layers is not None:
        dims["layers"] = args.layers
    if args.vocab is not None:
        dims["vocab"] = args.vocab
    shapes = llama_shapes(**dims)
    n_params = sum(numel(s) for s in shapes)
    algo, prec = args.algorithm, args.precision
    bpp = BYTES_PER_PARAM[(algo, prec)]

    gen = torch.Generator(device=dev).manual_seed(1234)
    params = []
    with torch.no_grad():
        for shp in shapes:
            p = torch.empty(shp, dtype=torch.bfloat16, device=dev)
            p.normal_(0.0, 0.02, generator=gen)
            params.append(torch.nn.Parameter(p))
    cls = ZeroLionBridge if algo == "lion" else ZeroAdamBridge
    kw = dict(lr=1e-5, betas=(0.9, 0.99), weight_decay=0.1) if algo == "lion" else \
        dict(lr=2e-5, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.01)
    opt = cls(params, precision=prec, rounds=args.rounds or 8, max_ctas=args.max_ctas, gather=args.gather, **kw)
    L = opt.layout
    shard_params = sum(pc.n for r in opt._pieces for pc in r)
    with torch.no_grad():
        opt.grad_shard.normal_(0.0, 1e-3, generator=gen)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()

    def step():
        if args.clip is not None:
            opt.clip_shard_grad_norm_(args.clip)
        opt.step_shard()

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()

    launches0 = kern.launch_count()
    opt.trace = []
    cur = torch.cuda.current_stream(dev)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local_rank) as clocks:
        torch.cuda.synchronize()
        t0.record(cur)
        for _ in range(args.steps):
            step()
        t1.record(cur)
        torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    launches = kern.launch_count() - launches0
    ms = t0.elapsed_time(t1) / args.steps
    kernel_ms = sum(s.elapsed_time(e) for s, e in opt.trace) / args.steps
    norm_ms = sum(s.elapsed_time(e) for s, e in opt.norm_trace) / args.steps
    n_launches_trace = len(opt.trace)
    opt.trace = None
    ms_t = torch.tensor([ms, kernel_ms, norm_ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(ms_t, op=dist.ReduceOp.MAX)
    ms_max, kernel_ms_max, norm_ms_max = ms_t.tolist()

    # ---- e2e: host buffers through the public API (pinned grad shard in, updated weight shard out)
    e2e = None
    if not args.no_e2e:
        e2e_steps = max(1, min(args.steps, args.e2e_steps))
        host_g = torch.empty(L.shard_numel, dtype=opt.grad_dtype, pin_memory=True)
        host_g.copy_(opt.grad_shard.cpu())
        host_w = torch.empty(L.shard_numel, dtype=opt.dtype, pin_memory=True)

        def e2e_step():
            if args.clip is not None:
                opt.grad_shard.copy_(host_g, non_blocking=True)
                opt.clip_shard_grad_norm_(args.clip)
                opt.step_shard(weights_out=host_w)
            else:
                opt.step_shard(host_g, weights_out=host_w)   # copies in and out overlap the rounds' updates

        e2e_step()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(cur)
        for _ in range(e2e_steps):
            e2e_step()
        b.record(cur)
        torch.cuda.synchronize()
        e_ms = torch.tensor([a.elapsed_time(b) / e2e_steps], dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(e_ms, op=dist.ReduceOp.MAX)
        e_ms = e_ms.item()
        link = host_link_gbs(host_g, host_w, opt, world, dev)
        e2e = {"value": round(n_params / (e_ms / 1e3) / 1e9, 4), "unit": "Gparams/s", "host_link": link,
               "h2d_bytes_per_step": host_g.numel() * host_g.element_size(),
               "d2h_bytes_per_step": host_w.numel() * host_w.element_size(), "ms_per_step": round(e_ms, 3),
               "path": "ZeroAdamBridge.step_shard(host gradient shard, weights_out=host weight shard): every step "
                       "copies the gradient shard in from pinned host memory and the updated weight shard out, "
                       f"round by round ({L.rounds} rounds) overlapping the updates"}
        del host_g, host_w

    # ---- N > 1: the NVLink reference rate (NCCL's all-gather of the same bytes), then the parity check
    nccl_gbs = nccl_allgather_gbs(opt, world, dev) if world > 1 else None
    gather_mode = opt.gather
    fused_gather = gather_mode == "p2p"
    del opt
    torch.cuda.empty_cache()
    parity = None if args.no_parity else sharded_parity(args, world, rank, dev)
    ref_gpu = None
    if world == 1 and not args.no_reference_gpu and (algo, prec) == ("adamw", "bf16"):
        # the reference's own GPU update on the same parameter set, with this run's state freed first
        del params
        torch.cuda.empty_cache()
        ref_gpu = torch_fused_adamw_rate(dims, max(2, min(args.steps, 5)), 2, dev)

    if rank != 0:
        return None
    peaks = {}
    pk = ROOT / "MEASURED_PEAKS.json"
    if pk.exists():
        peaks = json.loads(pk.read_text())
    peak = peaks.get("hbm_gbs", 6650.0)
    peak_note = "MEASURED_PEAKS.json hbm_gbs (of measured)" if "hbm_gbs" in peaks else "6650 GB/s (of fallback)"
    hbm_bytes = bpp * shard_params
    nvl_bytes = 0
    if fused_gather:
        # the kernel also stores its new bf16 weights into the world - 1 peers (NVLink egress) and receives the
        # peers' (NVLink ingress, written into this GPU's HBM): per direction, (world - 1) x its shard
        nvl_bytes = (world - 1) * shard_params * 2
        hbm_bytes += nvl_bytes
    bound = "nvlink" if fused_gather and nvl_bytes / nccl_gbs > hbm_bytes / peak else "hbm"
    if bound == "nvlink":
        achieved = nvl_bytes / (kernel_ms_max / 1e3) / 1e9
        peak, peak_note = round(nccl_gbs, 1), (f"{nccl_gbs:.0f} GB/s NVLink ingress per rank of NCCL's all-gather of "
                                               "the same weight buffer, measured in this run (of measured)")
    else:
        achieved = hbm_bytes / (kernel_ms_max / 1e3) / 1e9
    line = {
        "metric": metric_name(algo, prec),
        "value": round(n_params / (ms_max / 1e3) / 1e9, 4), "unit": "Gparams/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_max, 3), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": workload_name(dims, algo, prec, args.clip), "params": n_params, "tensors": len(shapes),
                   "weights": "bf16", "grads": "bf16", "master": "fp32", "stochastic_rounding": True,
                   "parallelism": f"zero1-dp{world}", "rounds": L.rounds, "max_ctas": args.max_ctas,
                   "all_gather": GATHER_LABELS[gather_mode],
                   "l2": "no flush: each step streams %.1f GB >> 126 MB L2" % (bpp * shard_params / 1e9)},
        "roofline": {"bound": bound, "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4),
                     "traffic": (round(MEASURED_DRAM_BYTES_PER_PARAM[(algo, prec)] * shard_params)
                                 if (algo, prec) in MEASURED_DRAM_BYTES_PER_PARAM else None),
                     "traffic_basis": "dram__bytes_read.sum + dram__bytes_write.sum per parameter from ncu on the "
                                      "1-layer case, times the parameters of one step (all of its launches)",
                     "basis": (f"{bpp} B/param x {shard_params:,} params per rank per step"
                               + (f" + {nvl_bytes / 1e9:.2f} GB of peers' weights received" if fused_gather else "")
                               + (f"; NVLink: {nvl_bytes / 1e9:.2f} GB per direction per rank" if fused_gather else "")
                               + f" / update-kernel time {kernel_ms_max:.3f} ms (CUDA events on the update stream, "
                               f"{n_launches_trace // args.steps} multi-segment calls per step); peak = {peak_note}")},
        "gpu_launches": launches,
        "clocks": clocks.summary(),
        "e2e": e2e,
    }
    if args.clip is not None:
        g_bytes = shard_params * opt.grad_shard.element_size()
        line["clip"] = {"max_norm": args.clip, "norm_kernels_ms": round(norm_ms_max, 3),
                        "norm_gbs": round(g_bytes / (norm_ms_max / 1e3) / 1e9, 1),
                        "basis": "clip_shard_grad_norm_ before every step: one read of the bf16 gradient shard "
                                 "(per-tensor sums of squares), the coefficient applied inside the update kernel"}
    if world > 1:
        received = (world - 1) * L.chunk * L.rounds * 2
        line["allgather"] = {"bytes_received_per_rank": int(received), "step_ms": round(ms_max, 3),
                             "update_kernel_ms": round(kernel_ms_max, 3),
                             "nccl_allgather_gbs": round(nccl_gbs, 1),
                             "ingress_gbs_over_step": round(received / (ms_max / 1e3) / 1e9, 1),
                             "limited_by": ("NVLink ingress of the update kernel's peer stores" if bound == "nvlink"
                                            else "NVLink ingress of the copy engines' peer copies"
                                            if gather_mode == "ce" and received / (ms_max / 1e3) / 1e9 > 0.5 * nccl_gbs
                                            else "HBM traffic of the update kernel")}
    if parity is not None:
        line["parity"] = parity
    if ref_gpu is not None:
        line["reference_gpu_update"] = ref_gpu
    if world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline_block(args)
    return line


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="abx", choices=["abx", "reference", "reference-gpu"])
    ap.add_argument("--workload", default="update", choices=["update", "train", "convert"],
                    help="update: the fused optimizer step (the headline); train: config 5's training step; "
                         "convert: the state-format conversion kernel on the 7B set's second moment")
    ap.add_argument("--convert-from", default="fp32", choices=["fp32", "bf16", "fp8"],
                    help="--workload convert: the source format (the destination is --precision)")
    ap.add_argument("--algorithm", default="adamw", choices=["adamw", "lion"])
    ap.add_argument("--precision", default="bf16", choices=["fp32", "bf16", "fp8"])
    ap.add_argument("--rounds", type=int, default=None,
                    help="rounds of the ZeRO layout (default: 8 for the update, whose end-to-end host copies "
                         "overlap round by round; 32 for the training step, whose last round's update is what "
                         "the step still waits for after backward)")
    ap.add_argument("--max-ctas", type=int, default=0, help="cap the update kernel's CTAs (0: every SM)")
    ap.add_argument("--gather", default="auto", choices=["auto", "p2p", "ce", "nccl"],
                    help="N > 1: all-gather fused into the update as peer stores (p2p), copy-engine copies into "
                         "the peers' buffers (ce), or NCCL's")
    ap.add_argument("--layers", type=int, default=None, help="override the decoder depth (small profiling cases)")
    ap.add_argument("--vocab", type=int, default=None, help="override the vocabulary (small profiling cases)")
    ap.add_argument("--clip", type=float, default=None,
                    help="clip_grad_norm_ to this max norm before every step (norm kernels + scaled update)")
    ap.add_argument("--delay", action="store_true",
                    help="--workload train: delayed updates (each update overlaps the next forward)")
    ap.add_argument("--update-at-step", action="store_true",
                    help="--workload train: the hooks only reduce-scatter; every round is updated at step()")
    ap.add_argument("--e2e-steps", type=int, default=3)
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--cpu-variant-seconds", type=float, default=3.0,
                    help="seconds per extra CPU-baseline variant (default pool, forced avx2, fp8); 0 skips them")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-parity", action="store_true", help="skip the sharded-vs-unsharded check after timing")
    ap.add_argument("--no-reference-gpu", action="store_true",
                    help="N = 1: skip timing the reference's own GPU update (torch fused AdamW) after the step")
    args = ap.parse_args()
    if args.warmup < 3 and args.impl == "abx":
        print("warning: fewer than 3 warm-up steps", file=sys.stderr)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        reference_arm(args, rank, world)
        return 0
    if args.impl == "reference-gpu":
        reference_gpu_arm(args, rank)
        return 0
    import datetime

    import torch
    import torch.distributed as dist
    result_fd = None
    if world > 1:
        # NCCL logs its communicators (INFO: ranks, devices, transports) to standard output.  Everything this
        # process writes to standard output from here on goes to standard error instead, so the result line,
        # written to the saved descriptor, is the only line on standard output.
        if os.environ.get("NCCL_DEBUG", "").upper() in ("", "NONE", "VERSION", "WARN"):
            os.environ["NCCL_DEBUG"] = "INFO"          # communicator size and transports, on standard error
            os.environ.setdefault("NCCL_DEBUG_SUBSYS", "INIT,ENV")
        sys.stdout.flush()
        result_fd = os.dup(1)
        os.dup2(2, 1)
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local_rank))
    line = None
    try:
        if args.workload == "train":
            line = train_arm(args, rank, world, local_rank)
        elif args.workload == "convert":
            line = convert_arm(args, rank, world, local_rank)
        else:
            line = gpu_arm(args, rank, world, local_rank)
    finally:
        if world > 1:
            dist.destroy_process_group()
    if line is not None:
        text = json.dumps(line) + "\n"
        if result_fd is None:
            sys.stdout.write(text)
            sys.stdout.flush()
        else:
            os.write(result_fd, text.encode())
    return 0


if __name__ == "__main__":
    sys.exit(main())
