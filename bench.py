"""Benchmark of MORPH's optimizer-step hot path on B200 (one JSON line).

Workload: the dense 5B-shaped AdamW step — 42 layers of
{3 x [3072, 6144], 4 x [3072, 3072], 4 x [3072]} plus a [65536, 3072] tied
embedding = 4,165,459,968 FP32 masters with FP32 m and v, BF16 gradients
N(0, 1e-4), global-norm clip at 1.0 (torch clip_grad_norm_ rule), AdamW
lr 3e-4, betas (.9, .95), eps 1e-8, weight decay .1, BF16 compute copy written
by the update. Parameters are flat-sharded ZeRO-1 style over the ranks; each
step all-reduces the 16-byte {sum of squares, nonfinite} record and, with N > 1,
all-gathers the updated BF16 shards.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl morph|reference]

``value`` is params/s of the whole job (device-timed with CUDA events, max over
ranks, inputs resident in HBM; 116.6 GB of algorithmic traffic per step is far
larger than the 126 MB L2, so no flush is needed). ``e2e`` is the same metric
through the public ``morph_b200.AdamW.step()`` with the BF16 gradients copied
from pinned host memory every step and the step record (norm, skip) read back.
``--impl reference`` times the reference's CPU step (torch.optim.AdamW with
foreach=False after clip_grad_norm_, morph/training/runner.py:100-101) on the
host cores over a bounded sample of the same workload.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

import numpy as np
import torch

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

METRIC = "AdamW step params/s & HBM GB/s (% of ~8 TB/s) at 4.2B params, 1/2/4/8 B200"
LR, BETAS, EPS, WD, MAX_NORM = 3e-4, (0.9, 0.95), 1e-8, 0.1, 1.0
APPLY_BYTES = 28   # kernel 1: g 2 R + w,m,v 12 R + w,m,v 12 W + BF16 copy 2 W
STATS_BYTES = 2    # kernel 2: g 2 R
# Kernel 1's DRAM traffic per parameter, dram__bytes_read.sum + dram__bytes_write.sum
# from one ncu capture of a one-layer launch (1.321516 GB + 1.262883 GB over
# 94,384,128 params); traffic grows in proportion to the parameters processed.
NVLINK_GBS = 770.0  # measured peer copy per direction per GPU on this pool (B200, NVLink 5)
APPLY_TRAFFIC_PER_PARAM = (1.321516e9 + 1.262883e9) / 94384128  # ncu, k_adamw_apply_bulk, one layer
FALLBACK_HBM_GBS = 6650.0


def config2_shapes(layers=42, embedding=True):
    """Config 2's tensors; ``layers``/``embedding`` shrink it for profiling captures."""
    shapes = []
    for layer in range(layers):
        shapes += [(f"blocks.{layer}.ffn.{n}", (3072, 6144)) for n in ("gate", "up", "down")]
        shapes += [(f"blocks.{layer}.ssm.{n}", (3072, 3072)) for n in ("in", "x", "z", "out")]
        shapes += [(f"blocks.{layer}.vec.{n}", (3072,)) for n in ("norm", "bias", "dt_bias", "skip")]
    if embedding:
        shapes.append(("embedding.weight", (65536, 3072)))
    return shapes


def numel(shape):
    n = 1
    for s in shape:
        n *= s
    return n


def measured_peaks():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during the timed region."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index):
        # nvidia-smi addresses GPUs by physical index or UUID; CUDA_VISIBLE_DEVICES
        # may renumber, so use the UUID of the torch device.
        try:
            self.index = "GPU-" + str(torch.cuda.get_device_properties(device_index).uuid)
        except Exception:
            self.index = str(device_index)
        self.proc = None

    def __enter__(self):
        """Start sampling every 50 ms and wait (up to 5 s) for the first sample,
        so that even a short timed region is covered."""
        import threading
        self.first = []
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.QUERY}",
                                          "--format=csv,noheader,nounits", "-lms", "50"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            reader = threading.Thread(target=lambda: self.first.append(self.proc.stdout.readline()), daemon=True)
            reader.start()
            reader.join(timeout=5.0)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *exc):
        self.lines = [l for l in self.first if l and l.strip()]
        if self.proc is not None:
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=10)
            except Exception:
                self.proc.kill()
                out = ""
            self.lines += [l for l in out.splitlines() if l.strip()]

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in getattr(self, "lines", []):
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for name, val in zip(names, f[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


# ----------------------------------------------------------------- CPU side --

def cpu_threads():
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


REF_DIR = os.path.join(REPO, "baseline", "_ref")


def installed_reference_optimizer():
    """The reference's streamtrain.optimizer as installed (unmodified) in
    baseline/_ref by __graft_entry__.install_reference(), or None."""
    if not os.path.isdir(os.path.join(REF_DIR, "streamtrain")):
        return None
    if REF_DIR not in sys.path:
        sys.path.append(REF_DIR)
    try:
        import streamtrain.optimizer as ref_opt
    except Exception:
        return None
    return ref_opt


def reference_muon_cpu_time(shape, seed=0):
    """Seconds of one Muon matrix step of the reference on the host cores, and
    how it was run: the installed reference's HybridMuonAdamW.step
    (streamtrain/optimizer.py:48-62) on a one-matrix model when baseline/_ref
    holds it ("reference"), else the same arithmetic restated here ("port").
    One warm-up, one timed step."""
    threads = cpu_threads()
    torch.set_num_threads(threads)
    g = torch.Generator().manual_seed(seed)
    lr, wd = 3e-4, .1
    ref = installed_reference_optimizer()
    if ref is not None:
        # the Linear weight is [rows, cols] = shape; the LayerNorm gives the AdamW group a parameter
        model = torch.nn.Sequential(torch.nn.Linear(shape[1], shape[0], bias=False), torch.nn.LayerNorm(8))
        grad = (torch.randn(shape, generator=g) * 1e-4).bfloat16().float()
        opt = ref.HybridMuonAdamW(model, lr=lr, weight_decay=wd)

        def ref_step():
            model[0].weight.grad = grad
            for q in model[1].parameters():
                q.grad = torch.zeros_like(q)
            opt.step()

        ref_step()
        t0 = time.perf_counter()
        ref_step()
        return time.perf_counter() - t0, threads, "reference"
    p = torch.randn(shape, generator=g) * .02
    mom = torch.zeros(shape)
    grad = (torch.randn(shape, generator=g) * 1e-4).bfloat16()

    def step():
        gf = grad.float()
        mom.lerp_(gf, .05)
        u = gf.lerp(mom, .95)
        x = u.float()
        tall = x.shape[0] > x.shape[1]
        if tall:
            x = x.T
        x = x / (x.norm() + 1e-7)
        for _ in range(5):
            a = x @ x.T
            x = 3.4445 * x + (-4.775 * a + 2.0315 * (a @ a)) @ x
        o = x.T if tall else x
        o = o * max(1, shape[0] / shape[1]) ** .5
        p.mul_(1 - lr * wd).add_(o, alpha=-lr)

    step()
    t0 = time.perf_counter()
    step()
    return time.perf_counter() - t0, threads, "port"


def reference_cpu_step_time(layers=1, steps=3, warmup=1, seed=0):
    """Time the reference's CPU step on a bounded sample of config 2: ``layers``
    layers (94,384,128 params each) through torch.nn.utils.clip_grad_norm_
    (max_norm 1.0) and torch.optim.AdamW(foreach=False) — the calls at
    morph/training/runner.py:100-101 with the optimizer of
    streamtrain/optimizer.py:40 — on every host thread. Returns
    (params per step, seconds per step list, threads)."""
    threads = cpu_threads()
    torch.set_num_threads(threads)
    g = torch.Generator().manual_seed(seed)
    shapes = [s for _, s in config2_shapes()[: 11 * layers]]
    params = [torch.nn.Parameter(torch.randn(s, generator=g) * 0.02) for s in shapes]
    grads = [(torch.randn(s, generator=g) * 1e-4).to(torch.bfloat16) for s in shapes]
    opt = torch.optim.AdamW(params, lr=LR, betas=BETAS, eps=EPS, weight_decay=WD, foreach=False)
    times = []
    for i in range(warmup + steps):
        for p, gr in zip(params, grads):
            p.grad = gr.float()
        t0 = time.perf_counter()
        torch.nn.utils.clip_grad_norm_(params, MAX_NORM)
        opt.step()
        dt = time.perf_counter() - t0
        if i >= warmup:
            times.append(dt)
    return sum(numel(s) for s in shapes), times, threads


def run_reference(args, rank):
    """``--impl reference``: the reference's CPU step on host cores, rank 0 only."""
    if rank != 0:
        return
    n, times, threads = reference_cpu_step_time(layers=1, steps=args.steps, warmup=args.warmup)
    sec = sum(times) / len(times)
    value = n / sec
    sample = (f"1 of 42 layers of config 2 ({n:,} params: 3x[3072,6144], 4x[3072,3072], 4x[3072]) per step; "
              "clip_grad_norm_(1.0) + torch.optim.AdamW(foreach=False), FP32 grads from BF16")
    line = {"metric": METRIC, "value": value, "unit": "params/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": sec * 1e3, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic", "impl": "reference",
            "config": {"workload": "config2: dense 5B-shaped AdamW step, CPU sample", "params_per_step": n},
            "cpu_baseline": {"value": value, "unit": "params/s", "cores": threads, "kind": "reference",
                             "sample": sample},
            "e2e": {"value": value, "unit": "params/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------- GPU side --

def shard_bounds(total, world, rank, align=16):
    per = -(-total // world)
    per = -(-per // align) * align
    lo = min(total, rank * per)
    hi = min(total, lo + per)
    return lo, hi


def run_morph(args, rank, world, local_rank):
    import torch.distributed as dist
    from morph_b200 import AdamW, _lib
    from morph_b200.optim import StepEngine

    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    shapes = config2_shapes(args.layers, not args.no_embedding)
    sizes = [numel(s) for _, s in shapes]
    total = sum(sizes)
    lo, hi = shard_bounds(total, world, rank)
    n_local = hi - lo
    per = shard_bounds(total, world, 0)[1]  # padded shard length; every rank allocates it

    # Flat shard buffers: FP32 w, m, v; BF16 gradient shard; the full BF16 weights
    # (this rank's slice of it is where the update writes its BF16 copy).
    gen = torch.Generator(device=device).manual_seed(1234 + rank)
    w = torch.empty(per, dtype=torch.float32, device=device)
    chunk = 1 << 28
    for s in range(0, per, chunk):
        e = min(per, s + chunk)
        w[s:e].normal_(0.0, 0.02, generator=gen)
    m = torch.zeros_like(w)
    v = torch.zeros_like(w)
    g = torch.empty(per, dtype=torch.bfloat16, device=device)
    for s in range(0, per, chunk):
        e = min(per, s + chunk)
        g[s:e] = torch.empty(e - s, device=device).normal_(0.0, 1e-4, generator=gen).to(torch.bfloat16)
    full16 = torch.zeros(per * world, dtype=torch.bfloat16, device=device)
    out = full16[rank * per:(rank + 1) * per]

    # Segments: pieces of the model's tensors inside this rank's shard.
    pieces = []
    off = 0
    for (name, shape), n in zip(shapes, sizes):
        a, b = max(off, lo), min(off + n, hi)
        if a < b:
            pieces.append((a - lo, b - a))
        off += n
    eng = StepEngine(device)
    views = [(w[o:o + n], m[o:o + n], v[o:o + n], g[o:o + n], out[o:o + n]) for o, n in pieces]
    for vw in views:
        eng.slot(vw[0], 0)
    entries = [(vw[0], vw[1], vw[2], vw[3], vw[4], 0) for vw in views]
    groups = [(LR, BETAS[0], BETAS[1], EPS, WD, "torch")]
    plan = eng.prepare(entries, groups, _lib.MB_BF16, _lib.MB_BF16)
    fin = eng.finalize_opts(_lib.MB_FIN_CLIP_TORCH | _lib.MB_FIN_GATE, MAX_NORM)
    lib = eng.lib
    import ctypes
    pp, pf = ctypes.byref(plan), ctypes.byref(fin)
    record = eng.state_buf[:16].view(torch.float64)

    def one_step(evs=None):
        s = _lib.stream_handle()
        if evs is not None:
            evs[0].record()
        if world == 1:
            _lib.check(lib.mb_grad_stats(pp, pf, s))
        else:
            _lib.check(lib.mb_grad_stats(pp, None, s))
            dist.all_reduce(record)
            _lib.check(lib.mb_step_finalize(pp, pf, s))
        if evs is not None:
            evs[1].record()
        _lib.check(lib.mb_adamw_apply(pp, s))
        eng.max_clock += 1
        if evs is not None:
            evs[2].record()
        if world > 1:
            dist.all_gather_into_tensor(full16, out)
        if evs is not None:
            evs[3].record()

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local_rank])
        torch.cuda.synchronize()

    for _ in range(args.warmup):
        one_step()
    barrier()
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(args.steps)]
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local_rank) as clk:
        barrier()
        start.record()
        for i in range(args.steps):
            one_step(evs[i])
        stop.record()
        barrier()
    total_ms = start.elapsed_time(stop)
    stats_ms = sum(e[0].elapsed_time(e[1]) for e in evs) / args.steps
    apply_ms = sum(e[1].elapsed_time(e[2]) for e in evs) / args.steps
    gather_ms = sum(e[2].elapsed_time(e[3]) for e in evs) / args.steps
    st = eng.read_state()
    if st.status or st.skip:
        raise RuntimeError(f"bench step refused: status {st.status} skip {st.skip}")
    t = torch.tensor([total_ms, stats_ms, apply_ms, gather_ms], dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    total_ms, stats_ms, apply_ms, gather_ms = t.tolist()
    ms_per_step = total_ms / args.steps
    value = total / (ms_per_step / 1e3)
    clocks = clk.summary()
    del views, entries, plan

    # e2e through the public API: AdamW.step() (1 GPU) or ZeroAdamW.step()
    # (N GPUs) on the model's tensors, gradients copied from pinned host memory
    # each step, the step record read back.
    e2e = None
    if not args.no_e2e and world == 1:
        e2e = run_e2e(args, device, shapes, sizes, w[:total], m[:total], v[:total], g[:total], out[:total])


    hbm, peak_kind = measured_peaks()
    achieved = APPLY_BYTES * n_local / (apply_ms / 1e3) / 1e9
    line = {
        "metric": METRIC, "value": value, "unit": "params/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": ("config2: dense 5B-shaped AdamW step (4,165,459,968 params, BF16 grads, "
                                "clip 1.0, BF16 compute copy)") if total == 4165459968 else
                               f"config2 reduced for profiling: {args.layers} layers"
                               f"{'' if not args.no_embedding else ', no embedding'} ({total:,} params)",
                   "params": total, "grad_dtype": "bf16", "parallelism": f"zero1-dp{world}",
                   "l2": "inputs larger than L2 (116.6 GB of traffic per step vs 126 MB L2); no flush"},
        "hbm_gbs": (APPLY_BYTES + STATS_BYTES) * total / (ms_per_step / 1e3) / 1e9,
        "kernels_ms": {"grad_stats": stats_ms, "adamw_apply": apply_ms, "all_gather": gather_ms},
        "roofline": {"bound": "hbm", "kernel": "mb_adamw_apply", "achieved": achieved, "peak": hbm,
                     "peak_kind": peak_kind, "unit": "GB/s", "frac": achieved / hbm,
                     "algorithmic_bytes_per_launch": APPLY_BYTES * n_local,
                     "traffic": APPLY_TRAFFIC_PER_PARAM * n_local,
                     "traffic_basis": "ncu one-layer capture scaled by params per launch"},
        "gpu_launches": 2 * args.steps if world == 1 else 3 * args.steps,
        "clocks": clocks,
    }
    if e2e is not None:
        line["e2e"] = e2e
    if rank == 0 and not args.no_cpu_baseline and world == 1:
        n, times, threads = reference_cpu_step_time(layers=1, steps=3, warmup=1)
        line["cpu_baseline"] = {"value": n / (sum(times) / len(times)), "unit": "params/s", "cores": threads,
                                "kind": "reference",
                                "sample": f"1 of 42 layers ({n:,} params), clip_grad_norm_ + "
                                          "torch.optim.AdamW(foreach=False), 3 timed steps"}
    return line


def ns_flops(rows, cols, steps=5):
    """Algorithmic FLOPs of orthogonalize on [rows, cols] (m <= n after the
    transpose): per iteration X X^T (2 m^2 n), A A (2 m^3), B X (2 m^2 n)."""
    m, n = min(rows, cols), max(rows, cols)
    return steps * (4 * m * m * n + 2 * m ** 3)


def ns_flops_executed(rows, cols, steps=5):
    """FLOPs the kernels execute: X X^T and the M polynomial compute only the
    128x256 tiles not entirely below the diagonal (of the 256-padded m)."""
    m, n = min(rows, cols), max(rows, cols)
    mp = -(-m // 256) * 256
    np_ = -(-n // 256) * 256
    mt, nt = mp // 128, mp // 256
    frac = sum(min(mt, 2 * bn + 2) for bn in range(nt)) / (mt * nt)
    return steps * (frac * 2 * mp * mp * np_ + frac * 2 * mp ** 3 + 2 * mp * mp * np_)


def run_ns_only(args):
    """Profiling case: orthogonalize one [rows, cols] matrix (BF16 operands)
    ``steps`` times after ``warmup`` runs; prints its time and TFLOP/s."""
    from morph_b200 import orthogonalize
    rows, cols = (int(x) for x in args.ns_shape.split("x"))
    device = torch.device("cuda", 0)
    g = torch.randn(rows, cols, device=device, generator=torch.Generator(device=device).manual_seed(0))
    for _ in range(args.warmup):
        orthogonalize(g, ns_dtype="bf16")
    torch.cuda.synchronize()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(args.steps):
        orthogonalize(g, ns_dtype="bf16")
    stop.record()
    torch.cuda.synchronize()
    ms = start.elapsed_time(stop) / args.steps
    print(json.dumps({"workload": f"orthogonalize {rows}x{cols} bf16", "ms": ms,
                      "tflops": ns_flops(rows, cols) / (ms / 1e3) / 1e12,
                      "tflops_executed": ns_flops_executed(rows, cols) / (ms / 1e3) / 1e12}), flush=True)


def config4_model(device, layers=32):
    """Config 4's parameters (random init) with seeded BF16 gradients N(0, 1e-4):
    32 layers x {3 x [4096, 11008], 4 x [4096, 4096]} Linear weights, a
    [65536, 4096] embedding and 64 vectors [4096]. Every rank builds the same."""

    n_layers = layers

    class Model(torch.nn.Module):
        def __init__(self):
            super().__init__()
            layers = []
            for _ in range(n_layers):
                layers += [torch.nn.Linear(11008, 4096, bias=False, device=device) for _ in range(3)]
                layers += [torch.nn.Linear(4096, 4096, bias=False, device=device) for _ in range(4)]
            self.layers = torch.nn.ModuleList(layers)
            self.embedding = torch.nn.Embedding(65536, 4096, device=device)
            self.norms = torch.nn.ParameterList([torch.nn.Parameter(torch.ones(4096, device=device))
                                                 for _ in range(64)])

    with torch.no_grad():
        model = Model()
    gen = torch.Generator(device=device).manual_seed(4)
    for p in model.parameters():
        p.grad_dtype = None
        p.grad = (torch.randn(p.shape, device=device, generator=gen) * 1e-4).to(torch.bfloat16)
    return model


CONFIG4_WORKLOAD = ("config4: Muon 32 x {3 x [4096,11008], 4 x [4096,4096]} + AdamW [65536,4096] + 64 x [4096]")


def config4_workload(args):
    if args.c4_layers == 32:
        return CONFIG4_WORKLOAD
    return f"config4 reduced for profiling: {args.c4_layers} layers"


def run_config4_zero(args, rank, world, local_rank, emit=True):
    """Config 4 on N GPUs: ZeroHybridMuonAdamW (whole Muon matrices dealt over
    the ranks, AdamW group flat-sharded, BF16 weights all-gathered per round).
    Time per step = max over ranks of the device-timed step."""
    import torch.distributed as dist
    from morph_b200.zero import ZeroHybridMuonAdamW
    device = torch.device("cuda", local_rank)
    model = config4_model(device, args.c4_layers)
    opt = ZeroHybridMuonAdamW(model, lr=3e-4, weight_decay=.1, ns_dtype="bf16", device=device, sync=False)
    grads = [p.grad for p in model.parameters()]
    for _ in range(args.warmup):
        opt.step(grads)
    opt.check()
    torch.cuda.synchronize()
    dist.barrier()
    torch.cuda.synchronize()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local_rank) as clk:
        start.record()
        for _ in range(args.steps):
            opt.step(grads)
        stop.record()
        torch.cuda.synchronize()
    opt.check()  # the device gate's verdict on the last step (every rank reads the same record)
    dist.barrier()
    t = torch.tensor([start.elapsed_time(stop) / args.steps], device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    step_ms = float(t.item())
    opt.close()
    total_flop = sum(ns_flops(*q.shape) for q in opt.muon)
    peaks = {}
    try:
        with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as f:
            peaks = json.load(f)
    except Exception:
        pass
    peak = float(peaks.get("bf16_tflops_sustained", 1400.0))
    if rank == 0:
        achieved = total_flop / (step_ms / 1e3) / 1e12
        line = {"metric": "Hybrid Muon+AdamW step (config 4, 7B shape)", "value": step_ms / 1e3, "unit": "s/step",
                "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": step_ms,
                "higher_is_better": False, "scaling": "strong", "dtype": "bf16 NS operands, f32 state",
                "data": "synthetic",
                "config": {"workload": config4_workload(args), "parallelism": f"muon-matrix-shard + zero1-dp{world}",
                           "muon_matrices_per_rank": len(opt.owned), "rounds": len(opt.rounds)},
                "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak * world,
                             "peak_kind": "measured sustained x n_gpus" if peaks else "fallback x n_gpus",
                             "unit": "TFLOP/s", "frac": achieved / (peak * world),
                             "basis": "whole step time, algorithmic NS FLOPs"},
                "clocks": clk.summary()}
        if emit:
            print(json.dumps(line), flush=True)
        return line
    return None


def run_config4(args, emit=True):
    """Config 4: hybrid Muon + AdamW at the 7B shape, one GPU. Muon: 32 layers x
    {3 x [4096, 11008], 4 x [4096, 4096]} FP32 masters and momentum, BF16 grads
    N(0, 1e-4), Newton-Schulz 5 iterations on BF16 tcgen05 GEMMs. AdamW: a
    [65536, 4096] embedding and 64 vectors [4096]. Prints one JSON line with the
    step time and the Newton-Schulz tensor throughput per matrix shape."""
    import ctypes
    from morph_b200 import HybridMuonAdamW, _lib
    from morph_b200.muon import NS_COEFFS
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)

    model = config4_model(device, args.c4_layers)
    # sync=False: step() only enqueues (the gate is read on the device); checked after the timed region
    opt = HybridMuonAdamW(model, lr=3e-4, weight_decay=.1, ns_dtype="bf16", sync=False)
    muon_params = sum(p.numel() for p in opt.muon)
    adam_params = sum(p.numel() for g in opt.adam.param_groups for p in g["params"])
    for _ in range(args.warmup):
        opt.step()
    torch.cuda.synchronize()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(0) as clk:
        start.record()
        for _ in range(args.steps):
            opt.step()
        stop.record()
        torch.cuda.synchronize()
    opt.check()  # every timed step was applied
    step_ms = start.elapsed_time(stop) / args.steps
    # Muon step of one matrix, and of the batch the optimizer launches for the
    # shape (momentum + normalise + 5 NS iterations + update), timed alone
    per_shape = {}
    for shape in ((4096, 11008), (4096, 4096)):
        idxs = [i for i, q in enumerate(opt.muon) if tuple(q.shape) == shape]
        rows, cols = shape
        per = _lib.lib().mb_muon_batch_workspace_bytes(1, rows, cols)
        cap = max(1, min(_lib.MB_MUON_MAX_BATCH, opt.workspace_limit // per))
        size = -(-len(idxs) // -(-len(idxs) // cap))
        err = torch.zeros(1, dtype=torch.int32, device=device)
        a = _lib.MuonArgs(.05, .95, *NS_COEFFS, 5, max(1, rows / cols) ** .5, 1 - 3e-4 * .1, -3e-4, _lib.MB_BF16)
        entry = {}
        for batch in (1, size):
            sel = idxs[:batch]
            nbytes = _lib.lib().mb_muon_batch_workspace_bytes(batch, rows, cols)
            ws = torch.empty(nbytes, dtype=torch.uint8, device=device)
            table = ctypes.c_void_p * batch
            w_t = table(*[_lib.ptr(opt.muon[i]) for i in sel])
            m_t = table(*[_lib.ptr(opt.momentum[i]) for i in sel])
            g_t = table(*[_lib.ptr(opt.muon[i].grad) for i in sel])
            evs = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
            reps = 10 if batch == 1 else 3
            for i in range(3 + reps):
                if i == 3:
                    evs[0].record()
                _lib.check(_lib.lib().mb_muon_step_batched(w_t, m_t, g_t, _lib.MB_BF16, None, _lib.MB_NONE, batch,
                                                           rows, cols, ctypes.byref(a), _lib.ptr(ws), nbytes,
                                                           _lib.ptr(err), _lib.stream_handle()))
            evs[1].record()
            torch.cuda.synchronize()
            del ws
            ms = evs[0].elapsed_time(evs[1]) / reps / batch  # per matrix
            fl = ns_flops(rows, cols)
            fe = ns_flops_executed(rows, cols)
            entry["single" if batch == 1 else f"batch{batch}"] = {
                "ms_per_matrix": ms, "ns_tflops": fl / (ms / 1e3) / 1e12, "ns_flop": fl,
                "ns_tflops_executed": fe / (ms / 1e3) / 1e12}
        per_shape[f"{rows}x{cols}"] = entry
    total_flop = sum(ns_flops(*q.shape) for q in opt.muon)
    exec_flop = sum(ns_flops_executed(*q.shape) for q in opt.muon)
    peaks = {}
    try:
        with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as f:
            peaks = json.load(f)
    except Exception:
        pass
    peak = float(peaks.get("bf16_tflops_sustained", 1400.0))
    achieved = total_flop / (step_ms / 1e3) / 1e12
    line = {"metric": "Hybrid Muon+AdamW step (config 4, 7B shape)", "value": step_ms / 1e3, "unit": "s/step",
            "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": step_ms,
            "higher_is_better": False, "dtype": "bf16 NS operands, f32 state", "data": "synthetic",
            "config": {"workload": config4_workload(args), "muon_params": muon_params,
                       "adam_params": adam_params, "ns_flop_per_step": total_flop},
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak,
                         "peak_kind": "measured sustained" if peaks else "fallback", "unit": "TFLOP/s",
                         "frac": achieved / peak, "basis": "whole step time, algorithmic NS FLOPs",
                         "achieved_executed": exec_flop / (step_ms / 1e3) / 1e12,
                         "frac_executed": exec_flop / (step_ms / 1e3) / 1e12 / peak,
                         "note": "symmetric GEMMs skip lower tiles, so algorithmic FLOP/s can exceed the peak"},
            "per_matrix": per_shape, "clocks": clk.summary()}
    if not args.no_cpu_baseline:
        counts = {}
        for q in opt.muon:
            counts[tuple(q.shape)] = counts.get(tuple(q.shape), 0) + 1
        est, threads, sample, kind = 0.0, 1, {}, "port"
        for shape, cnt in counts.items():
            sec, threads, kind = reference_muon_cpu_time(shape)
            sample[f"{shape[0]}x{shape[1]}"] = sec
            est += sec * cnt
        how = ("the installed reference's HybridMuonAdamW.step on a one-matrix model" if kind == "reference"
               else "optimizer.py:52-61 with FP32 orthogonalize, restated")
        line["cpu_baseline"] = {"value": est, "unit": "s/step", "cores": threads, "kind": kind,
                                "sample": f"one Muon step ({how}) of each matrix shape on the host cores, scaled "
                                          "by the shape counts; the AdamW group (4% of the parameters, <1% of the "
                                          "work) is not included",
                                "per_matrix_s": sample}
    if emit:
        print(json.dumps(line), flush=True)
    return line


def host_link_gbs(device, nbytes=1 << 30):
    """Measured pinned-host <-> device copy bandwidth (H2D, D2H, both at once), GB/s."""
    host = torch.empty(nbytes, dtype=torch.uint8, pin_memory=True)
    host2 = torch.empty(nbytes, dtype=torch.uint8, pin_memory=True)
    dev = torch.empty(nbytes, dtype=torch.uint8, device=device)
    dev2 = torch.empty(nbytes, dtype=torch.uint8, device=device)
    s1, s2 = torch.cuda.Stream(device), torch.cuda.Stream(device)
    out = {}
    for name in ("h2d", "d2h", "both"):
        best = 0.0
        for _ in range(3):
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            if name in ("h2d", "both"):
                with torch.cuda.stream(s1):
                    dev.copy_(host, non_blocking=True)
            if name in ("d2h", "both"):
                with torch.cuda.stream(s2):
                    host2.copy_(dev2, non_blocking=True)
            torch.cuda.synchronize()
            dt = time.perf_counter() - t0
            best = max(best, (2 if name == "both" else 1) * nbytes / dt / 1e9)
        out[name] = best
    return out


def reference_rows_cpu_time(rows_k, cols, steps=2):
    """DiskState.update's arithmetic (streamtrain/disk.py:210-215) on the gathered
    [k, cols] rows in RAM, the reference's CPU work for one config-5 step."""
    import math
    threads = cpu_threads()
    torch.set_num_threads(threads)
    g = torch.Generator().manual_seed(5)
    w = torch.randn(rows_k, cols, generator=g) * .02
    m = torch.zeros_like(w)
    v = torch.zeros_like(w)
    grad = (torch.randn(rows_k, cols, generator=g) * 1e-3).half()
    times = []
    for step in range(1, steps + 2):
        t0 = time.perf_counter()
        gg = grad.float() * 1.0
        m.lerp_(gg, .1)
        v.mul_(.999).addcmul_(gg, gg, value=.001)
        d = v.sqrt().div_(math.sqrt(1 - .999 ** step)).add_(1e-8)
        w.mul_(1 - 1e-4 * .01).addcdiv_(m, d, value=-1e-4 / (1 - .9 ** step))
        if step > 1:
            times.append(time.perf_counter() - t0)
    return times, threads


def reference_disk_update(path, size, gradient, step, lr, clip, chunk_elements=1048576):
    """streamtrain/disk.py:203-223 restated literally (memmap chunks, torch CPU
    ops, write back, flush, fsync): the reference arm of the file-backed update."""
    import math
    mapped = np.memmap(path, dtype="float32", mode="r+", shape=(3, size))
    for start in range(0, size, chunk_elements):
        end = min(start + chunk_elements, size)
        weight, first, second = [torch.from_numpy(mapped[i, start:end].copy()) for i in range(3)]
        g = gradient.flatten()[start:end] * clip
        first.lerp_(g, .1)
        second.mul_(.999).addcmul_(g, g, value=.001)
        denominator = second.sqrt().div_(math.sqrt(1 - .999 ** step)).add_(1e-8)
        weight.mul_(1 - lr * .01).addcdiv_(first, denominator, value=-lr / (1 - .9 ** step))
        mapped[:, start:end] = np.stack((weight.numpy(), first.numpy(), second.numpy()))
    mapped.flush()
    del mapped
    fd = os.open(path, os.O_RDWR)
    try:
        os.fsync(fd)
    finally:
        os.close(fd)


def run_extra(args):
    """Measurements of the paths beside the configs' step (one GPU):
    rows: kernel 3 (lazy row-sparse update) on a device-resident config-5 table;
    disk: DiskState.update on a 64M-parameter (3, size) state file, GPU arithmetic
          (morph_b200.disk_io) vs the reference's CPU loop, wall clock incl. file I/O;
    accum: microbatch gradient accumulation (512M FP32 window, BF16 grads), HBM roofline;
    export: FP16 export of 256M FP32 masters into pinned host buffers, host-link roofline."""
    import shutil
    import tempfile
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    peaks = {}
    try:
        with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as f:
            peaks = json.load(f)
    except Exception:
        pass
    hbm = float(peaks.get("hbm_gbs", 6650.0))
    out = {"metric": "beside-the-step paths", "n_gpus": 1, "data": "synthetic"}
    if args.extra in ("disk", "all"):
        from morph_b200.disk_io import install
        size = 64 << 20
        root = tempfile.mkdtemp(prefix="mb_disk_")
        try:
            gen = torch.Generator().manual_seed(1)
            planes = torch.empty(3, size)
            planes[0].normal_(0, .02, generator=gen)
            planes[1].zero_()
            planes[2].zero_()
            planes.numpy().tofile(os.path.join(root, "ref.bin"))
            planes.numpy().tofile(os.path.join(root, "gpu.bin"))
            del planes
            grad = torch.empty(size, pin_memory=True)
            grad.normal_(0, 1e-3, generator=gen)

            class Store:
                pass
            store = Store()
            store.root, store.entries = root, {"gpu": {"file": "gpu.bin", "size": size}}
            install(store, device)
            store.update("gpu", grad, 1, 1e-4, 1.0)  # warm-up: buffers, page cache
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            for step in (2, 3, 4):
                store.update("gpu", grad, step, 1e-4, 1.0)
            torch.cuda.synchronize()
            gpu_s = (time.perf_counter() - t0) / 3
            threads = cpu_threads()
            torch.set_num_threads(threads)
            reference_disk_update(os.path.join(root, "ref.bin"), size, grad, 1, 1e-4, 1.0)
            t0 = time.perf_counter()
            for step in (2, 3, 4):
                reference_disk_update(os.path.join(root, "ref.bin"), size, grad, step, 1e-4, 1.0)
            ref_s = (time.perf_counter() - t0) / 3
            a = np.fromfile(os.path.join(root, "ref.bin"), dtype=np.float32).reshape(3, size)[:, : 1 << 20]
            b = np.fromfile(os.path.join(root, "gpu.bin"), dtype=np.float32).reshape(3, size)[:, : 1 << 20]
            agree = {"w_max_abs_diff": float(np.abs(a[0] - b[0]).max()),
                     "m_bit_equal": bool(np.array_equal(a[1], b[1])),
                     "v_bit_equal": bool(np.array_equal(a[2], b[2])),
                     "w_bit_equal_frac": float((a[0] == b[0]).mean())}
        finally:
            shutil.rmtree(root, ignore_errors=True)
        out["disk"] = {"workload": "DiskState.update, one (3, 67108864) FP32 state file, FP32 host gradient, "
                                   "chunk 1048576, 4 steps",
                       "value": size / gpu_s, "unit": "params/s", "s_per_update": gpu_s,
                       "reference_cpu": {"value": size / ref_s, "s_per_update": ref_s, "cores": threads,
                                         "kind": "reference (disk.py:203-223 restated in bench.py)"},
                       "speedup": ref_s / gpu_s, "file_bytes_rw_per_update": 24 * size,
                       "agreement_first_1M_after_4_steps": agree,
                       "note": "wall clock incl. page-cache file reads/writes and fsync on the box's /tmp; "
                               "torch's CPU sqrt (vectorised) differs from IEEE sqrt by <= 1 ulp on some "
                               "elements, so w agrees within 1e-6 relative, not bit for bit"}
    if args.extra in ("rows", "all"):
        # kernel 3 on a device-resident table: DeviceDiskState.update_rows
        from morph_b200.disk import DeviceDiskState
        rows, cols = args.rows, 3072
        k = rows // 10
        gen = torch.Generator(device=device).manual_seed(3)
        planes = torch.zeros(3, rows * cols, device=device)
        planes[0].normal_(0, .02, generator=gen)
        store = DeviceDiskState({"t": planes}, {"t": (rows, cols)})
        idxs = [torch.randperm(rows, device=device, generator=gen)[:k].sort().values for _ in range(4)]
        grads = (torch.randn(k, cols, device=device, generator=gen) * 1e-3).half()
        for i in range(3):
            store.update_rows("t", idxs[i % 4], grads, i + 1, 1e-4, 1.0, check=False)
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
        reps = 10
        ev[0].record()
        for i in range(reps):
            store.update_rows("t", idxs[i % 4], grads, i + 4, 1e-4, 1.0, check=False)
        ev[1].record()
        torch.cuda.synchronize()
        store.errors()
        ms = ev[0].elapsed_time(ev[1]) / reps
        algo = (26 * cols + 8) * k  # w, m, v read + written, f16 grad read, int64 index
        out["rows"] = {"workload": f"update_rows on a device table [{rows},{cols}] (w, m, v planes), "
                                   f"{k} sorted unique rows per launch, f16 grads (config-5 shapes, device-resident)",
                       "ms": ms, "touched_params_per_s": k * cols / (ms / 1e3),
                       "GB/s": algo / (ms / 1e3) / 1e9, "frac": algo / (ms / 1e3) / 1e9 / hbm,
                       "algorithmic_bytes_per_launch": algo, "peak_hbm_gbs": hbm}
        del planes, store, grads
        torch.cuda.empty_cache()
    if args.extra in ("accum", "all"):
        from morph_b200.disk import accumulate_, norm_record
        n = 512 << 20
        acc = torch.zeros(n, device=device)
        g = (torch.randn(n, device=device) * 1e-3).to(torch.bfloat16)
        rec = norm_record(device)
        res = {}
        for label, kw in (("accumulate", {}), ("accumulate+norm", {"record": rec})):
            for _ in range(3):
                accumulate_(acc, g, 1024.0, **kw)
            ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
            ev[0].record()
            for _ in range(10):
                accumulate_(acc, g, 1024.0, **kw)
            ev[1].record()
            torch.cuda.synchronize()
            ms = ev[0].elapsed_time(ev[1]) / 10
            gbs = 10 * n / (ms / 1e3) / 1e9
            res[label] = {"ms": ms, "GB/s": gbs, "frac": gbs / hbm}
        out["accum"] = {"workload": "acc (512M FP32) += bf16 grad / 1024, 10 B/elem (inputs > L2)",
                        "peak_hbm_gbs": hbm, **res}
    if args.extra in ("export", "all"):
        from morph_b200.export import export_fp16
        import hashlib
        n = 256 << 20
        src = torch.randn(n, device=device) * .02

        class Null:
            def write(self, b):
                return len(b)
        export_fp16(src, Null(), staging_elements=1 << 25)
        res = {}
        for label, dig in (("no digest", None), ("sha256", hashlib.sha256())):
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            export_fp16(src, Null(), digest=dig, staging_elements=1 << 25)
            torch.cuda.synchronize()
            sec = time.perf_counter() - t0
            res[label] = {"s": sec, "GB/s_fp16_out": 2 * n / sec / 1e9}
        host = src[: 1 << 25].cpu().numpy()
        t0 = time.perf_counter()
        for start in range(0, host.size, 1048576):  # export.py:31-34 per chunk, without the file write
            value = host[start:start + 1048576]
            if not np.isfinite(value).all() or np.abs(value).max(initial=0) > 65504:
                raise ValueError("unexpected")
            value.astype("<f2").tobytes()
        ref_rate = host.size / (time.perf_counter() - t0)
        out["export"] = {"workload": "FP16 export of 256M FP32 device masters (512 MB out), null sink",
                         **res, "host_link": host_link_gbs(device),
                         "reference_cast_elems_per_s": ref_rate}
    print(json.dumps(out), flush=True)


def run_config1(args, emit=True):
    """Config 1 (and the latency side of config 3): 64 x [128, 128] FP32 masters,
    FP16 grads x 2^16 with the device loss scale (2^16, growth 2000), lr 3e-4,
    betas (.9, .95), eps 1e-8, wd .1, FP16 copy of the weights every step.
    Launch-bound: times the eager AdamW.step and the same step replayed from a
    CUDA graph, next to the reference's CPU step (unscale + torch AdamW)."""
    from morph_b200 import AdamW, DynamicLossScale
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    gen = torch.Generator(device=device).manual_seed(1234)
    ps = [torch.nn.Parameter(torch.randn(128, 128, device=device, generator=gen) * .02) for _ in range(64)]
    for p in ps:
        p.grad_dtype = None
        p.grad = (torch.randn(128, 128, device=device, generator=gen) * 1e-3 * 65536.0).half()
    scaler = DynamicLossScale(scale=65536.0, growth_interval=2000, device=device)
    opt = AdamW(ps, lr=3e-4, betas=(.9, .95), eps=1e-8, weight_decay=.1, loss_scale=scaler,
                low_precision=torch.float16)
    reps = 200
    for _ in range(max(3, args.warmup)):
        opt.step()
    torch.cuda.synchronize()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
    t0 = time.perf_counter()
    ev[0].record()
    for _ in range(reps):
        opt.step()
    ev[1].record()
    torch.cuda.synchronize()
    eager_us = (time.perf_counter() - t0) / reps * 1e6
    eager_dev_us = ev[0].elapsed_time(ev[1]) / reps * 1e3
    side = torch.cuda.Stream(device)
    side.wait_stream(torch.cuda.current_stream(device))
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(side), torch.cuda.graph(graph, stream=side):
        opt.step()
    torch.cuda.current_stream(device).wait_stream(side)
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize()
    # Three windows of reps * 10 replays (~60 ms each); the median is reported and
    # every window is listed, so one window disturbed by the host (a fresh box's
    # first seconds) does not set the figure.
    trials, dev_trials = [], []
    with ClockSampler(0) as clk:
        for _ in range(3):
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            ev[0].record()
            for _ in range(reps * 10):
                graph.replay()
            ev[1].record()
            torch.cuda.synchronize()
            trials.append((time.perf_counter() - t0) / (reps * 10) * 1e6)
            dev_trials.append(ev[0].elapsed_time(ev[1]) / (reps * 10) * 1e3)
    graph_us = sorted(trials)[1]
    graph_dev_us = sorted(dev_trials)[1]
    # the reference's CPU step on the same shapes: unscale the FP16 grads, torch AdamW
    threads = cpu_threads()
    torch.set_num_threads(threads)
    cp = [torch.nn.Parameter(p.detach().cpu().clone()) for p in ps]
    cg = [p.grad.cpu() for p in ps]
    copt = torch.optim.AdamW(cp, lr=3e-4, betas=(.9, .95), eps=1e-8, weight_decay=.1, foreach=False)

    def cpu_step():
        for q, g in zip(cp, cg):
            q.grad = g.float() / 65536.0
        copt.step()
        [q.detach().half() for q in cp]  # the FP16 weights of each step

    for _ in range(3):
        cpu_step()
    t0 = time.perf_counter()
    for _ in range(20):
        cpu_step()
    cpu_us = (time.perf_counter() - t0) / 20 * 1e6
    n = 64 * 128 * 128
    hbm, peak_kind = measured_peaks()
    achieved = (APPLY_BYTES + STATS_BYTES) * n / (graph_dev_us / 1e6) / 1e9
    line = {"metric": "AdamW step latency, config 1 (64 x [128,128], FP16 grads, loss scale 2^16, FP16 copy)",
            "value": graph_us, "unit": "us/step", "n_gpus": 1, "steps": reps, "warmup": max(3, args.warmup),
            "higher_is_better": False, "dtype": "f32", "data": "synthetic",
            "config": {"workload": "config1: 1,048,576 params", "params": n},
            "eager_us_per_step": eager_us, "eager_device_us_per_step": eager_dev_us,
            "graph_replay_us_per_step": graph_us, "ms_per_step": graph_us / 1e3,
            "graph_replay_trials_us": trials, "graph_replay_device_us_per_step": graph_dev_us,
            "roofline": {"bound": "latency", "achieved": achieved, "peak": hbm, "peak_kind": peak_kind,
                         "unit": "GB/s", "frac": achieved / hbm,
                         "algorithmic_bytes_per_step": (APPLY_BYTES + STATS_BYTES) * n,
                         "note": "31.5 MB per step moves in a few microseconds; the two kernels' latency "
                                 "(one or two tiles per CTA, then the last CTA's finalize) bounds the "
                                 "graph replay"},
            "clocks": clk.summary(),
            "cpu_baseline": {"value": cpu_us, "unit": "us/step", "cores": threads, "kind": "reference",
                             "sample": "unscale + torch.optim.AdamW(foreach=False) + FP16 copy on the same shapes"},
            "gpu_launches_per_step": 2}
    if emit:
        print(json.dumps(line), flush=True)
    return line


def run_config5(args, rank=0, world=1, local_rank=0, emit=True):
    """Config 5: lazy row-sparse AdamW with the [262144, 3072] table's w, m, v in
    pinned host memory, 10% of rows (sorted unique int64) touched per step with
    FP16 grads N(0, 1e-3), DiskState.update hyperparameters (lr 1e-4, clip 1.0),
    256 MiB ping-pong windows. Metric: touched params/s; roofline: host link.
    N > 1: the rows are sharded in contiguous blocks (ShardedRowTable), each GPU
    streams its block over its own host link; time = max over ranks."""
    from morph_b200.offload import OffloadedRowTable, ShardedRowTable
    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    rows, cols, k = 262144, 3072, 26214
    if world > 1:
        import torch.distributed as dist
        table = ShardedRowTable(rows, cols, device=device)
        local = table.local
    else:
        table = local = OffloadedRowTable(rows, cols, device=device)
    window_rows = local.window_rows
    # masters N(0, 0.02), drawn on the device and copied into the pinned planes
    gen = torch.Generator(device=device).manual_seed(1234 + rank)
    for r0 in range(0, local.rows, 8192):
        r1 = min(local.rows, r0 + 8192)
        local.w[r0:r1].copy_(torch.empty(r1 - r0, cols, device=device).normal_(0.0, 0.02, generator=gen))
    steps = args.warmup + args.steps
    idxs, grads = [], []
    gdev = torch.Generator(device=device).manual_seed(99)
    for step in range(steps):
        gi = torch.Generator().manual_seed(1234 + step)
        idxs.append(torch.randperm(rows, generator=gi)[:k].sort().values.to(device))
        grads.append((torch.randn(k, cols, device=device, generator=gdev) * 1e-3).half())
    for step in range(args.warmup):
        table.step(idxs[step], grads[step], step + 1, 1e-4, 1.0)
    table.synchronize()
    if world > 1:
        dist.barrier()
        torch.cuda.synchronize()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local_rank) as clk:
        start.record()
        for step in range(args.warmup, steps):
            table.step(idxs[step], grads[step], step + 1, 1e-4, 1.0)
        stop.record()
        table.synchronize()
    ms = start.elapsed_time(stop) / args.steps
    if world > 1:
        t = torch.tensor([ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
        dist.barrier()
    link_bytes = 24 * k * cols
    link = host_link_gbs(device)  # every rank at once: the links' aggregate
    if world > 1:
        agg = torch.tensor([link["h2d"], link["d2h"], link["both"]], device=device, dtype=torch.float64)
        dist.all_reduce(agg)
        link = {"h2d": float(agg[0]), "d2h": float(agg[1]), "both": float(agg[2]), "ranks_concurrent": world}
    achieved = link_bytes / (ms / 1e3) / 1e9
    if rank != 0:
        return
    line = {"metric": "lazy row-sparse AdamW on pinned-host state (config 5)", "value": k * cols / (ms / 1e3),
            "unit": "touched params/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": ms, "higher_is_better": True, "scaling": "strong", "dtype": "f32 state, f16 grads",
            "data": "synthetic",
            "config": {"workload": "config5: [262144,3072] table, 26214 rows/step, 256 MiB windows",
                       "window_rows": window_rows, "touched_params": k * cols,
                       "parallelism": "single GPU" if world == 1 else f"row-block shard over {world} GPUs"},
            "roofline": {"bound": "host link", "achieved": achieved, "peak": link["both"],
                         "unit": "GB/s", "frac": achieved / link["both"],
                         "algorithmic_link_bytes_per_step": link_bytes, "link_measured": link},
            "clocks": clk.summary()}
    if world == 1:
        ref_times, threads = reference_rows_cpu_time(k, cols)
        line["cpu_baseline"] = {"value": k * cols / (sum(ref_times) / len(ref_times)), "unit": "touched params/s",
                                "cores": threads, "kind": "reference",
                                "sample": "the torch calls of streamtrain/disk.py:210-215 (DiskState.update "
                                          "without its memmap and fsync) on the gathered [26214, 3072] rows in RAM"}
    if emit:
        print(json.dumps(line), flush=True)
    return line


def zero_parity_check(opt, grads, shapes, sizes, rank, world, local_rank):
    """Correctness of the sharded step inside the measured run (N > 1).

    * replicas: per-chunk sums of the 32-bit words of every rank's full
      low-precision weight buffer are all-gathered and must be identical;
    * sampled pieces: the first and last ZeRO piece of each rank (the first one
      of every rank but 0 starts mid-tensor), up to 1M elements each, are
      snapshotted before one more fused step and recomputed on the same GPU as
      a stand-alone one-GPU AdamW step (mb_step_finalize from the all-reduced
      {sum of squares, nonfinite} record, then mb_adamw_apply); w, m, v, the
      BF16 copy at the piece's place in the gathered weights and the clip
      coefficient must be bit-identical. The one-GPU kernels are the ones the
      GPU parity tests hold bit-exact to the CPU oracle."""
    import ctypes
    import torch.distributed as dist
    from morph_b200 import _lib
    from morph_b200.optim import StepEngine
    device = opt.device
    offsets = np.concatenate([[0], np.cumsum(sizes)]).astype(np.int64).tolist()
    flat_g = [g.reshape(-1) for g in grads]
    eng0 = opt.backend.engine
    owned = [j for j, pc in enumerate(opt.pieces) if pc[3] > 0]
    picks = []
    for j in sorted({owned[0], owned[-1]}) if owned else []:
        i, t_off, s_off, n, _ = opt.pieces[j]
        n = min(n, 1 << 20)
        picks.append(dict(i=i, t_off=t_off, s_off=s_off, n=n, w=opt.master[s_off:s_off + n].clone(),
                          m=opt.exp_avg[s_off:s_off + n].clone(), v=opt.exp_avg_sq[s_off:s_off + n].clone(),
                          g=flat_g[i][t_off:t_off + n].clone(),
                          clock=int(eng0.clocks[eng0.slots[id(opt._keys[j])]])))
    torch.cuda.synchronize(device)
    opt.step(grads)
    torch.cuda.synchronize(device)
    info = opt.last_step()
    ok = info["status"] == 0 and not info["skipped"]
    record = opt.backend.record().clone()
    lib = _lib.lib()
    for pk in picks:
        eng = StepEngine(device)
        key = object()
        eng.slot(key, pk["clock"])
        out = torch.empty(pk["n"], dtype=opt.low_precision, device=device)
        plan = eng.prepare([(pk["w"], pk["m"], pk["v"], pk["g"], out, 0)],
                           [(opt.lr, opt.betas[0], opt.betas[1], opt.eps, opt.weight_decay, "torch")],
                           _lib.dtype_code(pk["g"].dtype), _lib.dtype_code(opt.low_precision), keys=[key])
        eng.state_buf[:16].copy_(record.view(torch.uint8))
        fin = eng.finalize_opts(opt._fin_flags(), opt.max_norm)
        with torch.cuda.device(device):
            _lib.check(lib.mb_step_finalize(ctypes.byref(plan), ctypes.byref(fin), _lib.stream_handle()))
            _lib.check(lib.mb_adamw_apply(ctypes.byref(plan), _lib.stream_handle()))
        torch.cuda.synchronize(device)
        s_off, n = pk["s_off"], pk["n"]
        f_off = offsets[pk["i"]] + pk["t_off"]
        ok = ok and torch.equal(pk["w"], opt.master[s_off:s_off + n])
        ok = ok and torch.equal(pk["m"], opt.exp_avg[s_off:s_off + n])
        ok = ok and torch.equal(pk["v"], opt.exp_avg_sq[s_off:s_off + n])
        ok = ok and torch.equal(out.view(torch.int16), opt.flat_weights[f_off:f_off + n].view(torch.int16))
        ok = ok and np.float32(eng.read_state().clip_coef) == np.float32(info["clip_coef"])
    total = sum(sizes)
    words = opt.flat_weights[:total - total % 2].view(torch.int32)
    chunk = 1 << 22
    sums = torch.stack([words[a:a + chunk].sum(dtype=torch.int64) for a in range(0, words.numel(), chunk)])
    gathered = [torch.empty_like(sums) for _ in range(world)]
    dist.all_gather(gathered, sums)
    replicas = all(torch.equal(gathered[0], x) for x in gathered[1:])
    flags = torch.tensor([int(ok), len(picks), sum(int(p["t_off"] > 0) for p in picks),
                          sum(p["n"] for p in picks)], dtype=torch.int64, device=device)
    low = flags.clone()
    dist.all_reduce(low, op=dist.ReduceOp.MIN)
    dist.all_reduce(flags)
    return {"replicas_identical": bool(replicas), "sampled_bit_exact": bool(low[0]),
            "pieces_checked": int(flags[1]), "pieces_starting_mid_tensor": int(flags[2]),
            "elements_checked": int(flags[3]),
            "method": "per-chunk word sums of every rank's gathered BF16 weights compared across ranks; the first "
                      "and last ZeRO piece of each rank recomputed as a one-GPU AdamW step from the all-reduced "
                      "norm record (w, m, v, BF16 copy in the gathered buffer, clip coefficient bit-identical)"}


def run_update_only(args, rank, world, local_rank, shapes, sizes):
    """The update alone at N > 1: each rank runs a complete AdamW step over its
    own contiguous 1/N shard of config 2 (fresh FP32 w, m, v, BF16 gradients and
    a BF16 copy of the shard) with the global norm all-reduced, and no
    all-gather of the copies. Separate buffers from the sharded optimizer, so
    its state is untouched. Time per step = max over ranks."""
    import ctypes
    import torch.distributed as dist
    from morph_b200 import _lib
    from morph_b200.optim import StepEngine
    device = torch.device("cuda", local_rank)
    total = sum(sizes)
    lo, hi = shard_bounds(total, world, rank)
    n_local = hi - lo
    gen = torch.Generator(device=device).manual_seed(4321 + rank)
    w = torch.empty(n_local, dtype=torch.float32, device=device)
    g = torch.empty(n_local, dtype=torch.bfloat16, device=device)
    for s0 in range(0, n_local, 1 << 28):
        e0 = min(n_local, s0 + (1 << 28))
        w[s0:e0].normal_(0.0, 0.02, generator=gen)
        g[s0:e0] = torch.empty(e0 - s0, device=device).normal_(0.0, 1e-4, generator=gen).to(torch.bfloat16)
    m, v = torch.zeros_like(w), torch.zeros_like(w)
    out = torch.empty(n_local, dtype=torch.bfloat16, device=device)
    eng = StepEngine(device)
    entries, off = [], 0
    for n in sizes:
        a, b = max(off, lo), min(off + n, hi)
        if a < b:
            o, k = a - lo, b - a
            piece = w[o:o + k]  # the clock slot is keyed by this view object: keep it in the entry
            eng.slot(piece, 0)
            entries.append((piece, m[o:o + k], v[o:o + k], g[o:o + k], out[o:o + k], 0))
        off += n
    plan = eng.prepare(entries, [(LR, BETAS[0], BETAS[1], EPS, WD, "torch")], _lib.MB_BF16, _lib.MB_BF16)
    fin = eng.finalize_opts(_lib.MB_FIN_CLIP_TORCH | _lib.MB_FIN_GATE, MAX_NORM)
    pp, pf = ctypes.byref(plan), ctypes.byref(fin)
    record = eng.state_buf[:16].view(torch.float64)
    lib = eng.lib
    steps = max(1, min(args.steps, 5))

    def one_step(evs=None):
        s = _lib.stream_handle()
        _lib.check(lib.mb_grad_stats(pp, None, s))
        dist.all_reduce(record)
        _lib.check(lib.mb_step_finalize(pp, pf, s))
        if evs is not None:
            evs[0].record()
        _lib.check(lib.mb_adamw_apply(pp, s))
        if evs is not None:
            evs[1].record()

    for _ in range(3):
        one_step()
    dist.barrier(device_ids=[local_rank])
    torch.cuda.synchronize()
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(2)] for _ in range(steps)]
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for i in range(steps):
        one_step(evs[i])
    stop.record()
    torch.cuda.synchronize()
    st = eng.read_state()
    t = torch.tensor([start.elapsed_time(stop) / steps, sum(e[0].elapsed_time(e[1]) for e in evs) / steps,
                      float(st.status or st.skip)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms, apply_ms, bad = t.tolist()
    if bad:
        raise RuntimeError("update-only step refused")
    hbm, peak_kind = measured_peaks()
    owned = torch.tensor([n_local], dtype=torch.int64, device=device)
    dist.all_reduce(owned, op=dist.ReduceOp.MAX)
    achieved = APPLY_BYTES * int(owned) / (apply_ms / 1e3) / 1e9
    return {"value": total / (ms / 1e3), "unit": "params/s", "ms_per_step": ms, "steps": steps,
            "kernels_ms": {"adamw_apply": apply_ms},
            "roofline": {"bound": "hbm", "kernel": "mb_adamw_apply", "achieved": achieved, "peak": hbm,
                         "peak_kind": peak_kind, "unit": "GB/s", "frac": achieved / hbm,
                         "algorithmic_bytes_per_launch": APPLY_BYTES * int(owned)},
            "workload": f"each rank's contiguous 1/{world} of config 2: kernel 2, all-reduce of the norm record, "
                        "finalize, kernel 1 with the BF16 copy of the shard; no all-gather"}


def run_morph_zero(args, rank, world, local_rank):
    """N > 1: config 2 through morph_b200.zero.ZeroAdamW (round-robin chunks,
    8 update/all-gather rounds). ``value``: device-timed steps with the BF16
    gradients resident; ``e2e``: each rank also copies its gradient chunks from
    pinned host memory and reads the 16-byte record back every step."""
    import torch.distributed as dist
    from morph_b200.zero import ZeroAdamW
    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    shapes = config2_shapes(args.layers, not args.no_embedding)
    sizes = [numel(s) for _, s in shapes]
    total = sum(sizes)
    full = torch.empty(total, dtype=torch.float32, device=device)
    gen = torch.Generator(device=device).manual_seed(1234)
    for s0 in range(0, total, 1 << 28):
        full[s0:min(total, s0 + (1 << 28))].normal_(0.0, 0.02, generator=gen)
    params, off = [], 0
    for (_, shape), n in zip(shapes, sizes):
        params.append(full[off:off + n].view(shape))
        off += n
    # sync=False: step() only enqueues, as the one-GPU run's AdamW does; a refused
    # step is reported by last_step() after the timed region
    opt = ZeroAdamW(params, LR, BETAS, EPS, WD, max_norm=MAX_NORM, gate=True, device=device, rounds=args.rounds,
                    reserve_sms=args.reserve_sms, peer_writes=False if args.no_peer_writes else "auto", sync=False)
    del params, full
    torch.cuda.empty_cache()
    gflat = torch.empty(total, dtype=torch.bfloat16, device=device)
    for s0 in range(0, total, 1 << 28):
        e0 = min(total, s0 + (1 << 28))
        gflat[s0:e0] = torch.empty(e0 - s0, device=device).normal_(0.0, 1e-4, generator=gen).to(torch.bfloat16)
    grads, off = [], 0
    for (_, shape), n in zip(shapes, sizes):
        grads.append(gflat[off:off + n].view(shape))
        off += n
    owned = sum(hi - lo for _, lo, hi in opt.chunks)

    def barrier():
        dist.barrier(device_ids=[local_rank])
        torch.cuda.synchronize()

    for _ in range(args.warmup):
        opt.step(grads)
    barrier()
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(args.steps)]
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local_rank) as clk:
        barrier()
        start.record()
        for i in range(args.steps):
            opt.step(grads, events=evs[i])
        stop.record()
        barrier()
    info = opt.last_step()
    if info["status"] or info["skipped"]:
        raise RuntimeError(f"bench step refused: {info}")
    k = args.steps
    t = torch.tensor([start.elapsed_time(stop),
                      sum(e[0].elapsed_time(e[1]) for e in evs) / k,
                      sum(e[1].elapsed_time(e[2]) for e in evs) / k,
                      sum(e[2].elapsed_time(e[3]) for e in evs) / k], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    total_ms, stats_ms, apply_ms, tail_ms = t.tolist()
    ms_per_step = total_ms / k
    clocks = clk.summary()

    e2e = None
    if not args.no_e2e:
        # Each rank uploads the gradient chunks it owns from pinned host memory every
        # step; step k+1's upload (copy stream) overlaps step k's update, through two
        # device gradient buffers.
        chunks = [(lo, hi) for _, lo, hi in opt.chunks if hi > lo]
        hosts = [torch.empty(hi - lo, dtype=torch.bfloat16, pin_memory=True).copy_(gflat[lo:hi]) for lo, hi in chunks]
        gbufs = [gflat, torch.empty_like(gflat)]
        gviews = []
        for b in gbufs:
            vs, off = [], 0
            for (_, shape), n in zip(shapes, sizes):
                vs.append(b[off:off + n].view(shape))
                off += n
            gviews.append(vs)
        rec = torch.empty(2, dtype=torch.float64, pin_memory=True)
        steps = max(1, min(k, 5))
        copy_stream = torch.cuda.Stream(device)
        compute = torch.cuda.current_stream(device)
        ready = [torch.cuda.Event() for _ in range(2)]
        done = [torch.cuda.Event() for _ in range(2)]
        cursor = [0]

        def upload(j):
            b = j % 2
            with torch.cuda.stream(copy_stream):
                if j >= 2:
                    copy_stream.wait_event(done[b])
                for (lo, hi), h in zip(chunks, hosts):
                    gbufs[b][lo:hi].copy_(h, non_blocking=True)
                ready[b].record(copy_stream)

        def run(n):
            copy_stream.wait_stream(compute)
            upload(cursor[0])
            for i in range(n):
                j = cursor[0]
                if i + 1 < n:
                    upload(j + 1)
                compute.wait_event(ready[j % 2])
                opt.step(gviews[j % 2])
                done[j % 2].record(compute)
                rec.copy_(opt.backend.record(), non_blocking=True)
                cursor[0] += 1

        run(2)
        barrier()
        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s0.record()
        run(steps)
        s1.record()
        barrier()
        te = torch.tensor([s0.elapsed_time(s1) / steps], dtype=torch.float64, device=device)
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
        ms = float(te.item())
        e2e = {"value": total / (ms / 1e3), "unit": "params/s", "ms_per_step": ms, "steps": steps,
               "h2d_bytes_per_step": 2 * total, "d2h_bytes_per_step": 16 * world,
               "path": f"morph_b200.zero.ZeroAdamW.step() on {world} GPUs, each rank's gradient chunks H2D "
                       "from pinned host; step k+1's upload overlaps step k's update"}
        del gbufs, gviews

    hbm, peak_kind = measured_peaks()
    achieved = APPLY_BYTES * owned / (apply_ms / 1e3) / 1e9
    roofline = {"bound": "hbm", "kernel": "mb_adamw_apply_tiles", "achieved": achieved, "peak": hbm,
                "peak_kind": peak_kind, "unit": "GB/s", "frac": achieved / hbm,
                "algorithmic_bytes_per_launch": APPLY_BYTES * owned,
                "traffic": APPLY_TRAFFIC_PER_PARAM * owned,
                "traffic_basis": "ncu one-layer capture scaled by params per launch",
                "note": "update rounds overlap the BF16 all-gather, which shares SMs and HBM"}
    if opt.peer_writes:
        # fused update + all-gather: the slower of the HBM work and the NVLink sends bounds the launch
        link_bytes = 2 * owned * (world - 1)
        # this rank's own 28 B/param plus the other ranks' BF16 copies landing in its HBM
        hbm_bytes = APPLY_BYTES * owned + 2 * (total - owned)
        t_hbm = hbm_bytes / (hbm * 1e9)
        t_link = link_bytes / (NVLINK_GBS * 1e9)
        roofline = {"bound": "nvlink" if t_link > t_hbm else "hbm", "kernel": "mb_adamw_apply_tiles_peers",
                    "achieved": (max(t_hbm, t_link) / (apply_ms / 1e3)), "peak": 1.0, "unit": "of target time",
                    "frac": max(t_hbm, t_link) / (apply_ms / 1e3),
                    "target_ms": 1e3 * max(t_hbm, t_link), "hbm_ms": 1e3 * t_hbm, "nvlink_ms": 1e3 * t_link,
                    "nvlink_bytes_per_rank": link_bytes, "nvlink_peak_gbs": NVLINK_GBS,
                    "nvlink_achieved_gbs": link_bytes / (apply_ms / 1e3) / 1e9,
                    "hbm_achieved_gbs": hbm_bytes / (apply_ms / 1e3) / 1e9, "hbm_bytes_per_rank": hbm_bytes,
                    "hbm_peak": hbm, "peak_kind": peak_kind,
                    "algorithmic_bytes_per_launch": APPLY_BYTES * owned,
                    "traffic": APPLY_TRAFFIC_PER_PARAM * owned,
                    "traffic_basis": "ncu one-layer capture scaled by params per launch (HBM side)",
                    "note": "kernel 1 stores each BF16 copy into every rank's buffer over NVLink (peer "
                            "pointers); target = max(HBM bytes (own 28 B/param + 2 B/param received from "
                            "the other ranks) / measured HBM peak, NVLink bytes / measured 770 GB/s peer copy)"}
    line = {
        "metric": METRIC, "value": total / (ms_per_step / 1e3), "unit": "params/s", "n_gpus": world,
        "steps": k, "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "config2: dense 5B-shaped AdamW step (4,165,459,968 params, BF16 grads, "
                               "clip 1.0, BF16 compute copy)" if total == 4165459968 else
                               f"config2 reduced: {args.layers} layers ({total:,} params)",
                   "params": total, "grad_dtype": "bf16", "parallelism": f"zero1-dp{world}",
                   "rounds": opt.rounds, "reserve_sms": args.reserve_sms,
                   "l2": "inputs larger than L2; no flush"},
        "hbm_gbs": (APPLY_BYTES + STATS_BYTES) * total / (ms_per_step / 1e3) / 1e9,
        "phases_ms": {"stats_allreduce_finalize": stats_ms, "update_rounds": apply_ms,
                      "allgather_tail": tail_ms},
        "all_gather": "fused into kernel 1 (peer stores over NVLink)" if opt.peer_writes else "NCCL, per round",
        "roofline": roofline,
        "gpu_launches": (2 + opt.rounds) * k,
        "clocks": clocks,
    }
    if e2e is not None:
        line["e2e"] = e2e
    line["parity"] = zero_parity_check(opt, grads, shapes, sizes, rank, world, local_rank)
    opt.close()
    return line


def run_e2e(args, device, shapes, sizes, w, m, v, g, out):
    from morph_b200 import AdamW
    params, off = [], 0
    for (name, shape), n in zip(shapes, sizes):
        p = torch.nn.Parameter(w[off:off + n].view(shape))
        p.grad_dtype = None  # BF16 gradients on FP32 masters
        p.grad = g[off:off + n].view(shape)
        params.append((p, off, n))
        off += n
    opt = AdamW([p for p, _, _ in params], lr=LR, betas=BETAS, eps=EPS, weight_decay=WD, foreach=False,
                max_norm=MAX_NORM, gate=True, sync=False, low_precision=torch.bfloat16)
    for p, o, n in params:
        st = opt.state[p]
        st["exp_avg"] = m[o:o + n].view(p.shape)
        st["exp_avg_sq"] = v[o:o + n].view(p.shape)
        opt.low_precision_copies[p] = out[o:o + n].view(p.shape)
    host = torch.empty(g.numel(), dtype=torch.bfloat16, pin_memory=True)
    host.copy_(g)
    rec_host = torch.empty(96, dtype=torch.uint8, pin_memory=True)
    eng_state = None
    steps = max(1, min(args.steps, 5))
    # Two device gradient buffers: step k+1's upload (copy stream) runs while
    # step k updates (compute stream); a buffer is refilled only after the step
    # that read it is done.
    bufs = [g, torch.empty_like(g)]
    views = [[b[o:o + n].view(p.shape) for p, o, n in params] for b in bufs]
    copy_stream = torch.cuda.Stream(device)
    compute = torch.cuda.current_stream(device)
    ready = [torch.cuda.Event() for _ in range(2)]
    done = [torch.cuda.Event() for _ in range(2)]
    k = 0

    def upload(j):
        b = j % 2
        with torch.cuda.stream(copy_stream):
            if j >= 2:
                copy_stream.wait_event(done[b])
            bufs[b].copy_(host, non_blocking=True)
            ready[b].record(copy_stream)

    def run(n):
        """n steps; all n uploads are issued here, each (but the first) while
        the previous step updates."""
        nonlocal eng_state, k
        copy_stream.wait_stream(compute)  # nothing of these steps starts before the caller's marker
        upload(k)
        for i in range(n):
            b = k % 2
            if i + 1 < n:
                upload(k + 1)
            compute.wait_event(ready[b])
            for (p, _, _), gv in zip(params, views[b]):
                p.grad = gv
            opt.step()
            done[b].record(compute)
            if eng_state is None:
                eng_state = opt._engine.state_buf
            rec_host.copy_(eng_state, non_blocking=True)
            k += 1

    run(2)
    torch.cuda.synchronize()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    run(steps)
    stop.record()
    torch.cuda.synchronize()
    ms = start.elapsed_time(stop) / steps
    total = g.numel()
    return {"value": total / (ms / 1e3), "unit": "params/s", "ms_per_step": ms, "steps": steps,
            "h2d_bytes_per_step": total * 2, "d2h_bytes_per_step": 96,
            "path": "morph_b200.AdamW.step(), 463 tensors, grads H2D from pinned host; step k+1's upload "
                    "overlaps step k's update (two device gradient buffers)"}


def _summary(line):
    """The fields of a config's own line kept in the headline line's ``configs``."""
    keep = ("metric", "value", "unit", "ms_per_step", "higher_is_better", "n_gpus", "steps", "warmup", "dtype",
            "roofline", "clocks", "cpu_baseline", "eager_us_per_step", "eager_device_us_per_step",
            "graph_replay_us_per_step", "graph_replay_trials_us", "graph_replay_device_us_per_step", "per_matrix")
    out = {k: line[k] for k in keep if k in line}
    out["workload"] = line.get("config", {}).get("workload")
    out["parallelism"] = line.get("config", {}).get("parallelism")
    return out


def run_sub_configs(args, rank, world, local_rank):
    """BASELINE configs 1, 4 and 5 measured in the same run as the headline
    (one GPU), and configs 4 and 5 sharded at N > 1 (config 1 is a single-GPU
    latency case). Each keeps its own metric, roofline and clock record."""
    import gc
    sub = argparse.Namespace(**vars(args))
    sub.warmup = 3
    out = {}

    def fresh():
        gc.collect()
        torch.cuda.empty_cache()

    fresh()
    if world == 1:
        out["config1"] = _summary(run_config1(sub, emit=False))
        fresh()
        sub.steps = min(args.steps, 5)
        out["config4"] = _summary(run_config4(sub, emit=False))
        fresh()
        sub.steps = min(args.steps, 10)
        out["config5"] = _summary(run_config5(sub, emit=False))
    else:
        sub.steps = min(args.steps, 5)
        line = run_config4_zero(sub, rank, world, local_rank, emit=False)
        if line is not None:
            out["config4"] = _summary(line)
        fresh()
        sub.steps = min(args.steps, 10)
        line = run_config5(sub, rank, world, local_rank, emit=False)
        if line is not None:
            out["config5"] = _summary(line)
    fresh()
    return out


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["morph", "reference"], default="morph")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--layers", type=int, default=42, help="profiling only: fewer layers than config 2")
    ap.add_argument("--no-embedding", action="store_true", help="profiling only: drop the embedding")
    ap.add_argument("--config", type=int, default=2, choices=[1, 2, 4, 5],
                    help="2 (default): the dense AdamW step; 1: the launch-bound small step; "
                         "4: the hybrid Muon+AdamW step; 5: row-sparse AdamW on pinned-host state")
    ap.add_argument("--rounds", type=int, default=8, help="N > 1: update/all-gather rounds per step")
    ap.add_argument("--reserve-sms", type=int, default=24, help="N > 1: SMs left to NCCL during the update")
    ap.add_argument("--no-peer-writes", action="store_true",
                    help="N > 1: NCCL all-gather rounds instead of kernel 1's peer stores")
    ap.add_argument("--c4-layers", type=int, default=32, help="profiling only: fewer layers than config 4")
    ap.add_argument("--ns-shape", default=None, help="profiling only, with --config 4: one matrix, e.g. 4096x4096")
    ap.add_argument("--rows", type=int, default=262144, help="--extra rows: table rows (profiling: fewer)")
    ap.add_argument("--no-configs", action="store_true",
                    help="config 2 only: skip the configs 1/4/5 records measured after the headline")
    ap.add_argument("--extra", choices=["disk", "rows", "accum", "export", "all"], default=None,
                    help="measure a path beside the configs' step instead (one GPU)")
    args = ap.parse_args()
    if args.warmup < 3 and args.impl == "morph":
        print("warning: fewer than 3 warm-up steps", file=sys.stderr)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank)
        return
    if args.extra:
        run_extra(args)
        return
    if args.config == 1:
        run_config1(args)
        return
    if args.config == 4 and (args.ns_shape or world == 1):
        run_ns_only(args) if args.ns_shape else run_config4(args)
        return
    if args.config == 5 and world == 1:
        run_config5(args)
        return
    if world > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    try:
        if world > 1 and args.config == 4:
            run_config4_zero(args, rank, world, local_rank)
        elif world > 1 and args.config == 5:
            run_config5(args, rank, world, local_rank)
        else:
            full = args.layers == 42 and not args.no_embedding
            if world > 1:
                line = run_morph_zero(args, rank, world, local_rank)
                torch.cuda.empty_cache()
                shapes = config2_shapes(args.layers, not args.no_embedding)
                line["update_only"] = run_update_only(args, rank, world, local_rank, shapes,
                                                      [numel(s) for _, s in shapes])
            else:
                line = run_morph(args, rank, world, local_rank)
            if full and not args.no_configs:
                line["configs"] = run_sub_configs(args, rank, world, local_rank)
            if rank == 0:
                print(json.dumps(line), flush=True)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
