#!/usr/bin/env python3
"""Benchmark of the WeDLM block-parallel decode step on B200.

``python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]
[--workload entropy_select|decode_8b]`` prints ONE JSON line (rank 0).

Workloads (seeded synthetic inputs; no dataset is involved):

* ``entropy_select`` -- the fused entropy-select stage at 8B vocabulary: bf16 logits
  ``[64 x 96, 151936]`` (1.867 GB, larger than L2) drawn N(0, 2.5^2) plus one
  N(8, 1) spike per row; tau 0.8, lambda 0.05, cap 8, T 0.  A step is one
  ``wedlm_entropy_select`` over the whole batch.  Multi-GPU: every rank runs its own
  batch (weak scaling, no collective on the data path).
* ``decode_8b`` (default) -- streaming block decode of the 8B-shape random-init bf16
  model (36 layers, hidden 4096, 32/8 heads, head_dim 128, SwiGLU 12288, vocab 151936,
  N(0, 0.02^2) weights, norm weights 1): a 512-token uniform random prompt, then 512
  tokens generated with window 96 and the balanced preset (tau 0.8, lambda 0.05, cap 8
  with the entropy-EMA rule), temperature 0.  A step is one iteration of the streaming
  loop: one forward of the 96-token window against the KV cache, the fused
  entropy-select pass and the commit.  Multi-GPU: one independent sequence per rank
  (data-parallel replicas, weak scaling, no collective on the data path).

For N > 1 launch with ``torchrun --nproc-per-node N bench.py --gpus N``.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "wedlm-rs_b200"))
sys.path.insert(0, ROOT)

METRIC = "committed tok/s at 8B shape, block 96; fused entropy-select GB/s vs HBM peak"
V_8B = 151936
FALLBACK_HBM_GBS = 6650.0
FALLBACK_BF16_TFLOPS = 1590.0


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        d = json.load(open(p))
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, FALLBACK_BF16_TFLOPS, "fallback"


def profile_traffic(name: str):
    """DRAM bytes of one ncu capture (dram__bytes_read.sum + dram__bytes_write.sum), from
    the machine-readable record profiles/dram_traffic.json; None when absent."""
    try:
        return float(json.load(open(os.path.join(ROOT, "profiles", "dram_traffic.json")))[name]["bytes"])
    except (OSError, KeyError, ValueError, TypeError):
        return None


class ClockSampler:
    """nvidia-smi clock / throttle sampling in the background."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device = device
        self.samples = []
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.device), f"--query-gpu={self.Q}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.samples.append((time.time(), line.strip()))

    def stop(self, t0: float, t1: float):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = [s for (t, s) in self.samples if t0 - 0.15 <= t <= t1 + 0.15] or \
               [s for (_, s) in self.samples]
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            f = [x.strip() for x in r.split(",")]
            try:
                sm.append(float(f[1]))
                smax = float(f[2])
            except (ValueError, IndexError):
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        sm.sort()
        return {"sm_mhz": sm[len(sm) // 2] if sm else None, "sm_max_mhz": smax,
                "reasons": sorted(reasons), "samples": len(sm)}


# ----------------------------------------------------------------------------------
def dist_setup(gpus: int):
    import torch
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if ws > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    return rank, ws, local


def barrier(ws):
    if ws > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(x: float, ws: int) -> float:
    if ws == 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def make_c2_logits(rows: int, V: int, seed: int):
    import torch
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    x = torch.randn(rows, V, generator=g, device="cuda", dtype=torch.float32).mul_(2.5)
    cols = torch.randint(0, V, (rows,), generator=g, device="cuda")
    spike = torch.randn(rows, generator=g, device="cuda").add_(8.0)
    x[torch.arange(rows, device="cuda"), cols] += spike
    return x.to(torch.bfloat16)


# ----------------------------------------------------------------------------------
def bench_entropy_sharded(args, rank, ws, local):
    """Vocabulary-sharded entropy-select over `ws` GPUs: every rank holds the columns
    [r V/ws, (r+1) V/ws) of the same 64 x 96-row bf16 logits, computes per-row partials
    (max, sum 2^(x-m), sum 2^(x-m)(x-m), argmax) on its shard, the partials (16 B per row)
    are all-gathered over NCCL, and every rank combines them and applies the commit rule.
    Strong scaling: the whole job processes the full logits once per step."""
    import torch
    import torch.distributed as dist
    from wedlm_b200 import Context
    rows_per_seq, nseq = 96, args.nseq
    rows, V = rows_per_seq * nseq, V_8B
    assert V % ws == 0 and (V // ws) % 8 == 0
    Vr = V // ws
    ctx = Context(None, device=local)
    full = make_c2_logits(rows, V, seed=1234)
    shard = full[:, rank * Vr:(rank + 1) * Vr].contiguous()
    del full
    torch.cuda.empty_cache()
    seq_rows = torch.arange(0, rows + 1, rows_per_seq, dtype=torch.int32, device="cuda")
    mask_pos = torch.arange(rows, dtype=torch.int32, device="cuda") % rows_per_seq
    caps = torch.full((nseq,), 8, dtype=torch.int32, device="cuda")
    part = torch.empty(rows, 4, dtype=torch.float32, device="cuda")
    gath = torch.empty(ws, rows, 4, dtype=torch.float32, device="cuda")
    stream = torch.cuda.current_stream()

    def step(src):
        ctx.entropy_partials(src, rank * Vr, 0.0, out=part, stream=stream)
        dist.all_gather_into_tensor(gath, part)
        return ctx.entropy_combine(gath, 0.8, 0.05, seq_rows, mask_pos, caps, stream=stream)

    hbm, _, peak_kind = peaks()
    clk = ClockSampler(local)
    clk.start()
    for _ in range(args.warmup):
        step(shard)
    torch.cuda.synchronize()
    barrier(ws)
    t0 = time.time()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        step(shard)
    e1.record(stream)
    torch.cuda.synchronize()
    barrier(ws)
    clocks = clk.stop(t0, time.time())
    ms = max_over_ranks(e0.elapsed_time(e1) / args.steps, ws)
    total = rows * V * 2
    # partials kernel alone (this rank's shard), for the roofline
    k0, k1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    k0.record(stream)
    for _ in range(args.steps):
        ctx.entropy_partials(shard, rank * Vr, 0.0, out=part, stream=stream)
    k1.record(stream)
    torch.cuda.synchronize()
    kms = k0.elapsed_time(k1) / args.steps
    achieved = rows * Vr * 2 / (kms * 1e-3) / 1e9
    # end to end: the shard from pinned host memory, results back to the host
    host = shard.cpu().pin_memory()
    dev = torch.empty_like(shard)
    h_out = {k: torch.empty(rows if k != "n_selected" else nseq,
                            dtype=torch.float32 if k in ("H", "maxprob") else torch.int32,
                            pin_memory=True) for k in ("H", "argmax", "maxprob", "selected", "n_selected")}
    barrier(ws)
    x0, x1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ne2e = max(3, min(args.steps, 10))
    x0.record(stream)
    for _ in range(ne2e):
        dev.copy_(host, non_blocking=True)
        out = step(dev)
        for k in h_out:
            h_out[k].copy_(out[k], non_blocking=True)
    x1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks(x0.elapsed_time(x1) / ne2e, ws)
    d2h = sum(t.numel() * t.element_size() for t in h_out.values())
    ctx.close()
    return {"metric": METRIC, "value": round(total / (ms * 1e-3) / 1e9, 1), "unit": "GB/s",
            "n_gpus": ws, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic: seeded N(0,2.5^2) bf16 logits + one N(8,1) spike per row",
            "config": {"workload": f"entropy_select vocab-sharded: {nseq} seqs x 96 mask rows x "
                                   f"151936 vocab over {ws} GPUs ({Vr} columns each), NCCL "
                                   "all-gather of 16 B per row, combine + commit rule on every rank",
                       "rows": rows, "vocab": V, "bytes_per_step_total": total,
                       "l2": f"inputs larger than L2 ({rows * Vr * 2 / 1e9:.2f} GB per GPU)",
                       "parallelism": f"vocab{ws}"},
            "clocks": clocks,
            "e2e": {"value": round(total / (e2e_ms * 1e-3) / 1e9, 1), "unit": "GB/s",
                    "h2d_bytes_per_step": rows * Vr * 2, "d2h_bytes_per_step": d2h},
            "gpu_launches": args.steps * 2,
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm,
                         "peak_kind": peak_kind, "unit": "GB/s", "frac": round(achieved / hbm, 4),
                         "traffic": None, "kernel": "entropy_partials_kernel<bf16> (per rank)"}}


def bench_entropy_select(args, rank, ws, local):
    if ws > 1 and args.shard == "vocab":
        return bench_entropy_sharded(args, rank, ws, local)
    import torch
    from wedlm_b200 import Context
    rows_per_seq, nseq = 96, args.nseq
    rows, V = rows_per_seq * nseq, V_8B
    ctx = Context(None, device=local)
    logits = make_c2_logits(rows, V, seed=1234 + rank)
    nbytes = rows * V * 2
    # inputs larger than L2: small batches cycle over copies that together exceed it
    ncopy = max(1, -(-300_000_000 // nbytes))
    bufs = [logits] + [logits.clone() for _ in range(ncopy - 1)]
    seq_rows = torch.arange(0, rows + 1, rows_per_seq, dtype=torch.int32, device="cuda")
    mask_pos = torch.arange(rows, dtype=torch.int32, device="cuda") % rows_per_seq
    caps = torch.full((nseq,), 8, dtype=torch.int32, device="cuda")
    outs = {"H": torch.empty(rows, dtype=torch.float32, device="cuda"),
            "argmax": torch.empty(rows, dtype=torch.int32, device="cuda"),
            "maxprob": torch.empty(rows, dtype=torch.float32, device="cuda"),
            "selected": torch.empty(rows, dtype=torch.int32, device="cuda"),
            "n_selected": torch.empty(nseq, dtype=torch.int32, device="cuda")}
    stream = torch.cuda.current_stream()
    it = [0]

    def step(s=None):
        x = bufs[it[0] % ncopy]
        it[0] += 1
        return ctx.entropy_select(x, 0.0, 0.8, 0.05, seq_rows, mask_pos, caps, out=outs,
                                  stream=s if s is not None else stream)

    hbm, _, peak_kind = peaks()
    clk = ClockSampler(local)
    clk.start()
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    # hold the GPU under load for a while so the clock record covers a loaded period
    t_end = time.time() + args.hold_seconds
    while time.time() < t_end:
        for _ in range(50):
            step()
        torch.cuda.synchronize()
    # the timed launches replay from a CUDA graph, so that the host's launch rate does not
    # gap them at small batches
    side = torch.cuda.Stream()
    side.wait_stream(stream)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(side):
        with torch.cuda.graph(graph, stream=side):
            for _ in range(args.steps):
                step(side)
    stream.wait_stream(side)
    graph.replay()
    torch.cuda.synchronize()
    barrier(ws)
    torch.cuda.synchronize()
    t0 = time.time()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    graph.replay()
    ev1.record(stream)
    torch.cuda.synchronize()
    barrier(ws)
    t1 = time.time()
    ms = ev0.elapsed_time(ev1) / args.steps
    clocks = clk.stop(t0, t1)
    ms_max = max_over_ranks(ms, ws)
    value = nbytes * ws / (ms_max * 1e-3) / 1e9
    del graph

    achieved = nbytes / (ms * 1e-3) / 1e9
    if args.profile:
        ctx.close()
        return {"metric": METRIC, "value": round(value, 1), "unit": "GB/s", "n_gpus": ws,
                "ms_per_step": round(ms_max, 4), "note": "profiling run (no e2e, no clocks)"}

    # end to end through the C ABI with host buffers: pinned H2D of the logits, the
    # kernel, D2H of every per-row and per-sequence result
    host = torch.empty((rows, V), dtype=torch.bfloat16, pin_memory=True)
    host.copy_(logits)
    dev = torch.empty_like(logits)
    outs = {k: torch.empty(rows if k != "n_selected" else nseq,
                           dtype=torch.float32 if k in ("H", "maxprob") else torch.int32,
                           device="cuda") for k in ("H", "argmax", "maxprob", "selected", "n_selected")}
    houts = {k: torch.empty(v.shape, dtype=v.dtype, pin_memory=True) for k, v in outs.items()}
    d2h = sum(v.numel() * v.element_size() for v in outs.values())

    def e2e_step():
        dev.copy_(host, non_blocking=True)
        ctx.entropy_select(dev, 0.0, 0.8, 0.05, seq_rows, mask_pos, caps, out=outs, stream=stream)
        for k in outs:
            houts[k].copy_(outs[k], non_blocking=True)

    for _ in range(2):
        e2e_step()
    torch.cuda.synchronize()
    barrier(ws)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ne2e = max(3, min(args.steps, 10))
    e0.record(stream)
    for _ in range(ne2e):
        e2e_step()
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1) / ne2e, ws)
    del host, dev

    line = {
        "metric": METRIC, "value": round(value, 1), "unit": "GB/s", "n_gpus": ws,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_max, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic: seeded N(0,2.5^2) bf16 logits + one N(8,1) spike per row",
        "config": {"workload": f"entropy_select: {nseq} seqs x 96 mask rows x 151936 vocab, "
                               "bf16 logits, tau 0.8, lambda 0.05, cap 8, T 0",
                   "rows_per_gpu": rows, "vocab": V, "bytes_per_step_per_gpu": nbytes,
                   "l2": (f"inputs larger than L2 ({nbytes / 1e9:.2f} GB per GPU)" if ncopy == 1 else
                          f"launches cycle over {ncopy} copies of the logits ({ncopy * nbytes / 1e6:.0f} MB > L2)"),
                   "timing": "CUDA-graph replay of the timed launches",
                   "parallelism": f"dp{ws}"},
        "clocks": clocks,
        "e2e": {"value": round(nbytes * ws / (e2e_ms * 1e-3) / 1e9, 2), "unit": "GB/s",
                "h2d_bytes_per_step": nbytes, "d2h_bytes_per_step": d2h},
        "gpu_launches": args.steps,
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm,
                     "peak_kind": peak_kind, "unit": "GB/s", "frac": round(achieved / hbm, 4),
                     "traffic": profile_traffic("entropy_select_c2") if nseq == 64 else None,
                     "kernel": "entropy_select_kernel<bf16>"},
    }
    if rank == 0 and ws == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline_entropy(logits, budget_s=args.cpu_seconds)
    ctx.close()
    return line


def cpu_baseline_entropy(logits_dev, budget_s: float, nthreads: int = 0):
    """The C restatement of the reference's CPU path on a bounded sample (96-row
    batches of the same logits) for about `budget_s` seconds."""
    import numpy as np
    import torch
    from oracle import cbind
    sample = logits_dev[:96].contiguous().view(torch.int16).cpu().numpy().view(np.uint16)
    nthreads = nthreads or os.cpu_count()
    seq_rows, mask_pos, caps = [0, 96], list(range(96)), [8]
    cbind.entropy_select(sample, "bf16", 0.0, 0.8, 0.05, seq_rows, mask_pos, caps, nthreads)
    n, t0 = 0, time.time()
    while True:
        cbind.entropy_select(sample, "bf16", 0.0, 0.8, 0.05, seq_rows, mask_pos, caps, nthreads)
        n += 1
        if time.time() - t0 >= budget_s:
            break
    dt = time.time() - t0
    return {"value": round(n * sample.nbytes / dt / 1e9, 3), "unit": "GB/s", "cores": nthreads,
            "kind": "port",
            "sample": f"{n} x 96 rows x 151936 bf16 logits (the C restatement of "
                      f"compute_entropies_with_probs + select + greedy argmax), {dt:.1f} s"}


def reference_entropy(args, rank, ws):
    """--impl reference: the reference's CPU algorithm (C restatement; the Rust crate
    cannot be built without cargo/candle) on the host cores, same metric."""
    import numpy as np
    from oracle import cbind
    from oracle.model import f32_to_bf16_bits
    rows, V = 768, V_8B
    rng = np.random.default_rng(1234)
    x = rng.standard_normal((rows, V), dtype=np.float32) * np.float32(2.5)
    x[np.arange(rows), rng.integers(0, V, rows)] += rng.normal(8, 1, rows).astype(np.float32)
    b = f32_to_bf16_bits(x)
    nth = os.cpu_count()
    sr = list(range(0, rows + 1, 96))
    mp = [i % 96 for i in range(rows)]
    caps = [8] * (rows // 96)
    for _ in range(args.warmup):
        cbind.entropy_select(b, "bf16", 0.0, 0.8, 0.05, sr, mp, caps, nth)
    t0 = time.time()
    for _ in range(args.steps):
        cbind.entropy_select(b, "bf16", 0.0, 0.8, 0.05, sr, mp, caps, nth)
    dt = (time.time() - t0) / args.steps
    v = b.nbytes / dt / 1e9
    return {"metric": METRIC, "value": round(v, 3), "unit": "GB/s", "impl": "reference",
            "n_gpus": ws, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(dt * 1e3, 2), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": "entropy_select: bounded sample of 8 seqs x 96 rows x 151936 "
                                   "bf16 logits per step (same per-row work as the B200 arm)"},
            "cpu_baseline": {"value": round(v, 3), "unit": "GB/s", "cores": nth, "kind": "port",
                             "sample": "768 rows per step"},
            "e2e": {"value": round(v, 3), "unit": "GB/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}


# ----------------------------------------------------------------------------------
# The projection GEMMs of one 8B decode step (M = 96 window rows), bf16, weights N x K.
GEMM_SHAPES_8B = [("qkv", 6144, 4096, 0), ("o_resid", 4096, 4096, 2), ("gate_up_swiglu", 12288, 4096, 3),
                  ("down_resid", 4096, 12288, 2), ("lm_head", 151936, 4096, 0)]


def bench_gemm_shapes(args, rank, ws, local):
    """The decode-step GEMM shapes on their own through wedlm_kernel_gemm: each step
    runs every shape once; weights rotate over enough copies to exceed L2, so every
    launch streams its weights from HBM.  At the decode's 96 rows the shapes are
    HBM-bound and report GB/s (algorithmic bytes); with --gemm-rows >= 512 (the 6144 rows
    of batched serving) they are tensor-bound and report TFLOP/s."""
    import torch
    from wedlm_b200 import Context
    hbm, tflops, peak_kind = peaks()
    ctx = Context(None, device=local)
    M = args.gemm_rows
    tensor = M >= 512
    X = torch.randn(M, 12288, device="cuda").to(torch.bfloat16)
    res = {}
    total_bytes, total_flops, total_ms = 0.0, 0.0, 0.0
    only = set(args.gemm_only.split(",")) if args.gemm_only else None
    for name, N, K, epi in GEMM_SHAPES_8B:
        if only and name not in only:
            continue
        nW = 2 if epi == 3 else 1
        wbytes = nW * N * K * 2
        R = max(1, -(-300_000_000 // wbytes)) if not args.profile else 1
        Ws = [[ctx.pack_weight(torch.randn(N, K, device="cuda").mul_(K ** -0.5).to(torch.bfloat16))
               for _ in range(nW)] for _ in range(R)]
        out = torch.zeros(M, N, device="cuda", dtype=torch.bfloat16)
        Xs = X[:, :K]
        def f(i):
            W = Ws[i % R]
            ctx.gemm(Xs, W[0], out, epi, W2=W[1] if nW == 2 else None, N=N,
                     resid=out if epi == 2 else None)
        for i in range(max(args.warmup, R)):
            f(i)
        torch.cuda.synchronize()
        n = args.steps if args.profile else max(args.steps, 2 * R)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        if args.profile:
            e0.record()
            for i in range(n):
                f(i)
            e1.record()
        else:
            # replay the launches from a CUDA graph so host overhead does not gap them
            side = torch.cuda.Stream()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.stream(side):
                with torch.cuda.graph(g, stream=side):
                    for i in range(n):
                        f(i)
            g.replay()
            torch.cuda.synchronize()
            e0.record()
            g.replay()
            e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / n
        byt = wbytes + M * K * 2 + M * N * 2 * (2 if epi == 2 else 1)
        flo = 2.0 * nW * M * N * K
        res[name] = {"N": N, "K": K, "us": round(ms * 1e3, 2), "GBps": round(byt / ms / 1e6, 1),
                     "TFLOPs": round(flo / ms / 1e9, 1),
                     "frac": round(flo / ms / 1e9 / tflops, 4) if tensor else
                             round(byt / ms / 1e6 / hbm, 4)}
        total_bytes += byt
        total_flops += flo
        total_ms += ms
        del Ws
        torch.cuda.empty_cache()
    ctx.check_device_error()
    ctx.close()
    if tensor:
        achieved, unit, bound, peak = total_flops / total_ms / 1e9, "TFLOP/s", "tensor", tflops
    else:
        achieved, unit, bound, peak = total_bytes / total_ms / 1e6, "GB/s", "hbm", hbm
    return {"metric": METRIC, "value": round(achieved, 1), "unit": unit, "n_gpus": ws,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(total_ms, 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic", "config": {"workload": "gemm_shapes: the five projection GEMMs "
                                                        f"of one 8B step at M = {M}", "shapes": res,
                                            "l2": "weights rotated over > 300 MB of copies"},
            "roofline": {"bound": bound, "achieved": round(achieved, 1), "peak": peak,
                         "peak_kind": peak_kind, "unit": unit, "frac": round(achieved / peak, 4)}}


# ----------------------------------------------------------------------------------
ATT_PREFIXES = (512, 2048, 8192)


def attention_flops(L: int, S: int = 96, nh: int = 32) -> float:
    """QK^T and PV over the visible pairs: every query sees the L cached keys and, causal
    over explicit positions, S(S+1)/2 window pairs in total."""
    return 4.0 * nh * 128 * (S * L + S * (S + 1) / 2)


def bench_block_attention(args, rank, ws, local):
    """8B-shape block attention alone (32/8 heads, head_dim 128, 96-row window, N(0,1)
    inputs, ranks = a seeded permutation of the window positions) at prefixes of 512,
    2048 and 8192 cached tokens.  Each timed launch is bracketed by CUDA events; a
    256 MB write between launches flushes L2, so K/V come from HBM every time."""
    import torch
    from wedlm_b200 import Context
    hbm, tflops_peak, peak_kind = peaks()
    ctx = Context(None, device=local)
    flush = torch.empty(64 * 1024 * 1024, dtype=torch.float32, device="cuda")
    stream = torch.cuda.current_stream()
    res = {}
    for L in ATT_PREFIXES:
        g = torch.Generator(device="cpu").manual_seed(L + rank)
        S, nh, nkv = 96, 32, 8
        q = torch.randn(S, nh, 128, generator=g).to(torch.bfloat16).cuda()
        k = torch.randn(L + S, nkv, 128, generator=g).to(torch.bfloat16).cuda()
        v = torch.randn(L + S, nkv, 128, generator=g).to(torch.bfloat16).cuda()
        rk = (L + torch.randperm(S, generator=g)).to(torch.int32).cuda()
        ctx.attention_prepare(q, k, v, L, rk, stream=stream)
        out = torch.empty(S, nh * 128, dtype=torch.bfloat16, device="cuda")
        for _ in range(args.warmup):
            ctx.attention_run(out, stream=stream)
        torch.cuda.synchronize()
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
               for _ in range(args.steps)]
        for e0, e1 in evs:
            flush.fill_(1.0)
            e0.record(stream)
            ctx.attention_run(out, stream=stream)
            e1.record(stream)
        torch.cuda.synchronize()
        ctx.check_device_error()
        ms = sorted(e0.elapsed_time(e1) for e0, e1 in evs)[len(evs) // 2]
        ms = max_over_ranks(ms, ws)
        fl = attention_flops(L)
        byts = (L + S) * nkv * 128 * 2 * 2 + 2 * S * nh * 128 * 2
        # end to end: host q/k/v in, prepare (layout copy) + attention, host out back
        hq, hk, hv = q.cpu().pin_memory(), k.cpu().pin_memory(), v.cpu().pin_memory()
        hout = torch.empty(out.shape, dtype=out.dtype, pin_memory=True)
        dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
        x0, x1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        x0.record(stream)
        for t_dev, t_host in ((dq, hq), (dk, hk), (dv, hv)):
            t_dev.copy_(t_host, non_blocking=True)
        ctx.attention_prepare(dq, dk, dv, L, rk, stream=stream)
        ctx.attention_run(out, stream=stream)
        hout.copy_(out, non_blocking=True)
        x1.record(stream)
        torch.cuda.synchronize()
        e2e_ms = max_over_ranks(x0.elapsed_time(x1), ws)
        res[L] = {"us": round(ms * 1e3, 2), "TFLOPs": round(fl / (ms * 1e-3) / 1e12, 1),
                  "GBps": round(byts / (ms * 1e-3) / 1e9, 1),
                  "frac_tensor": round(fl / (ms * 1e-3) / 1e12 / tflops_peak, 4),
                  "e2e_TFLOPs": round(fl / (e2e_ms * 1e-3) / 1e12, 3),
                  "h2d_bytes": int((hq.numel() + hk.numel() + hv.numel()) * 2),
                  "d2h_bytes": int(hout.numel() * 2)}
        del q, k, v, dq, dk, dv
    ctx.close()
    top = res[ATT_PREFIXES[-1]]
    return {"metric": METRIC, "value": top["TFLOPs"] * ws, "unit": "TFLOP/s", "n_gpus": ws,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": top["us"] / 1e3,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic: N(0,1) bf16 q/k/v, ranks = seeded permutation of the window positions",
            "config": {"workload": "block_attention: 8B-shape GQA (32/8 heads, head_dim 128), "
                                   "96-row window, causal over explicit positions",
                       "prefixes": {str(k2): v2 for k2, v2 in res.items()},
                       "l2": "256 MB written between timed launches", "parallelism": f"dp{ws}"},
            "e2e": {"value": top["e2e_TFLOPs"] * ws, "unit": "TFLOP/s",
                    "h2d_bytes_per_step": top["h2d_bytes"], "d2h_bytes_per_step": top["d2h_bytes"]},
            "gpu_launches": args.steps * 2,
            "roofline": {"bound": "tensor", "achieved": top["TFLOPs"], "peak": tflops_peak,
                         "peak_kind": peak_kind, "unit": "TFLOP/s", "frac": top["frac_tensor"],
                         "traffic": profile_traffic("attention_tc_block_8192"),
                         "kernel": "attention_tc_kernel + attention_combine_kernel"}}


# ----------------------------------------------------------------------------------
SERVE_SEQS, SERVE_PROMPT, SERVE_NEW = 64, 4096, 1024


def bench_serve_8b(args, rank, ws, local):
    """Batched serving at the 8B shape: 64 sequences in total, split over the GPUs
    (data parallel, 64 / N per GPU), each a 4096-token uniform random prompt, then
    streaming decode with window 96 and the fast preset (tau 1.0, lambda 0.05, cap 6),
    T 0.  One step = one forward over every live window of the GPU (64 / N x 96 rows) +
    entropy-select + commit.  `value`: committed tokens per second over K timed steps,
    summed over GPUs; `e2e`: the same including the prompt prefill from host ids."""
    import numpy as np
    import torch
    from wedlm_b200 import Context, ModelConfig, SamplingParams
    hbm, tflops, peak_kind = peaks()
    nloc = args.serve_seqs // ws
    assert nloc >= 1 and args.serve_seqs % ws == 0
    cfg = ModelConfig.wedlm_8b(max_block_tokens=WINDOW_8B)
    max_ctx = SERVE_PROMPT + SERVE_NEW + WINDOW_8B + 64
    ctx = Context(cfg, device=local, max_seqs=nloc, max_ctx=max_ctx)
    ctx.init_random(seed=0, std=0.02)
    prompts = np.stack([make_prompt(SERVE_PROMPT, seed=1000 + rank * nloc + b) for b in range(nloc)])
    params = SamplingParams.preset("fast", temperature=0.0)
    stream = torch.cuda.current_stream()
    barrier(ws)
    torch.cuda.synchronize()
    p0, p1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    p0.record(stream)
    ctx.decode_begin(list(range(nloc)), prompts, SERVE_NEW, WINDOW_8B, params)
    p1.record(stream)
    torch.cuda.synchronize()
    prefill_ms = max_over_ranks(p0.elapsed_time(p1), ws)
    ctx.decode_step(args.warmup)
    tok0 = sum(ctx.decode_result(b)[1]["tokens_generated"] for b in range(nloc))
    n0, h0, d0 = ctx.decode_io_bytes()
    launches0 = ctx.launch_count()
    clk = ClockSampler(local)
    clk.start()
    time.sleep(0.2)
    barrier(ws)
    torch.cuda.synchronize()
    t0 = time.time()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        ctx.decode_step(1)
    e1.record(stream)
    torch.cuda.synchronize()
    barrier(ws)
    clocks = clk.stop(t0, time.time())
    ms = max_over_ranks(e0.elapsed_time(e1) / args.steps, ws)
    tok1 = sum(ctx.decode_result(b)[1]["tokens_generated"] for b in range(nloc))
    n1, h1, d1 = ctx.decode_io_bytes()
    launches = ctx.launch_count() - launches0
    toks = float(tok1 - tok0)
    steps_here = args.warmup + args.steps
    if ws > 1:
        import torch.distributed as dist
        t = torch.tensor([toks], dtype=torch.float64, device="cuda")
        dist.all_reduce(t)
        toks = float(t.item())
    value = toks / (ms * args.steps * 1e-3)
    # prompt prefill + the measured steps, prompts from host ids, ids back to host
    e2e_s = (prefill_ms + ms * steps_here) * 1e-3
    e2e_tok = toks * steps_here / args.steps
    ctx.decode_end()
    rows = nloc * WINDOW_8B
    flops = 2.0 * rows * 7.568e9
    ctx.close()
    return {"metric": METRIC, "value": round(value, 2), "unit": "committed tok/s", "n_gpus": ws,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 3),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic: random-init N(0,0.02^2) 8B-shape weights, uniform random prompt ids",
            "config": {"workload": f"serve_8b: {args.serve_seqs} sequences ({nloc} per GPU), "
                                   f"{SERVE_PROMPT}-token prompts, window 96, fast preset "
                                   "(tau 1.0, lambda 0.05, cap 6), T 0",
                       "rows_per_step_per_gpu": rows, "prefill_ms": round(prefill_ms, 1),
                       "prefill_tok_s": round(ws * nloc * SERVE_PROMPT / (prefill_ms * 1e-3), 1),
                       "tokens_per_step": round(toks / args.steps, 2),
                       "l2": "inputs larger than L2 (15.1 GB of weights per step)",
                       "parallelism": f"dp{ws}"},
            "clocks": clocks,
            "e2e": {"value": round(e2e_tok / e2e_s, 2), "unit": "committed tok/s",
                    "h2d_bytes_per_step": int((h1 - h0) / max(n1 - n0, 1)),
                    "d2h_bytes_per_step": int((d1 - d0) / max(n1 - n0, 1)),
                    "scope": "prompt prefill from host ids + warm-up and timed steps"},
            "gpu_launches": int(launches),
            "roofline": {"bound": "tensor", "achieved": round(flops / (ms * 1e-3) / 1e12, 1),
                         "peak": tflops, "peak_kind": peak_kind, "unit": "TFLOP/s",
                         "frac": round(flops / (ms * 1e-3) / 1e12 / tflops, 4), "traffic": None,
                         "kernel": "whole step (GEMM flops 2 x rows x 7.57 G parameters)"}}


# ----------------------------------------------------------------------------------
PROMPT_8B, NEW_8B, WINDOW_8B = 512, 512, 96
E2E_CALLS = 5  # end-to-end generate calls per run; the median is reported
DECODE_8B_WORKLOAD = ("decode_8b: 8B-shape WeDLM, 512-token prompt, 512 new tokens, window 96, "
                      "balanced preset (tau 0.8, lambda 0.05, cap 8), T 0")


def decode_8b_config(layers: int = 36) -> dict:
    """The decode_8b workload, the ``config`` of both arms' lines: the model shape, the
    prompt, the window and the preset.  How an arm runs it (decode loop, parallelism)
    goes in top-level keys of its line."""
    workload = DECODE_8B_WORKLOAD if layers == 36 else \
        DECODE_8B_WORKLOAD + f" [reduced to {layers} layers]"
    return {"workload": workload, "layers": layers, "hidden": 4096, "heads": "32/8",
            "head_dim": 128, "ffn": 12288, "vocab": 151936, "window": WINDOW_8B,
            "l2": "inputs larger than L2: every step streams all weights (15.1 GB in bf16)"}


def balanced_params():
    from wedlm_b200 import SamplingParams
    return SamplingParams.preset("balanced", temperature=0.0)


def make_prompt(n: int, seed: int, vocab_hi: int = 151643):
    import numpy as np
    # uniform ids below the special-token range (eos 151643, mask 151665)
    return np.random.default_rng(seed).integers(0, vocab_hi, size=n).astype(np.int32)


def bench_decode_8b(args, rank, ws, local):
    import torch
    from wedlm_b200 import Context, ModelConfig
    hbm, tflops, peak_kind = peaks()
    if args.layers != 36 and not args.profile:
        raise SystemExit("--layers only applies to --profile runs (captures of a reduced model)")
    cfg = ModelConfig.wedlm_8b(max_block_tokens=WINDOW_8B, num_hidden_layers=args.layers)
    # vocabulary-sharded LM head + entropy pass over the ranks (NCCL all-gathers of the
    # final-normed rows and of the per-row partials), or plain data parallelism
    sharded = ws > 1 and args.lm_head == "vocab"
    if sharded:
        V = cfg.vocab_size
        cfg.vocab_shard_begin, cfg.vocab_shard_end = rank * V // ws, (rank + 1) * V // ws
    max_ctx = PROMPT_8B + NEW_8B + WINDOW_8B + 64
    ctx = Context(cfg, device=local, max_seqs=1, max_ctx=max_ctx)
    ctx.init_random(seed=0, std=0.02)
    if sharded:
        import torch.distributed as dist
        from wedlm_b200 import comm_unique_id
        uid = [comm_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        ctx.comm_init(uid[0], rank, ws, timeout_ms=120000)
    prompt = make_prompt(PROMPT_8B, seed=rank)
    params = balanced_params()
    stream = torch.cuda.current_stream()
    if not args.profile:
        # warm the kernels, tensor maps and scratch on a short run
        ctx.generate_streaming(prompt[:64], 8, WINDOW_8B, params)
        torch.cuda.synchronize()

    need = args.warmup + args.steps + args.profile_steps
    assert need < NEW_8B, "steps exceed one 512-token generation"
    ctx.decode_begin([0], prompt, NEW_8B, WINDOW_8B, params)
    ctx.decode_step(args.warmup)
    _, st0 = ctx.decode_result(0)
    n0, h0, d0 = ctx.decode_io_bytes()
    launches0 = ctx.launch_count()
    clk = ClockSampler(local)
    clk.start()
    time.sleep(0.3)
    barrier(ws)
    torch.cuda.synchronize()
    t0 = time.time()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    for _ in range(args.steps):
        ctx.decode_step(1)
    ev1.record(stream)
    torch.cuda.synchronize()
    barrier(ws)
    t1 = time.time()
    clocks = clk.stop(t0, t1)
    ms = ev0.elapsed_time(ev1) / args.steps
    _, st1 = ctx.decode_result(0)
    n1, h1, d1 = ctx.decode_io_bytes()
    launches = ctx.launch_count() - launches0
    toks = st1["tokens_generated"] - st0["tokens_generated"]
    ms_max = max_over_ranks(ms, ws)
    tok_total = toks
    if ws > 1:
        import torch.distributed as dist
        t = torch.tensor([float(toks)], dtype=torch.float64, device="cuda")
        dist.all_reduce(t)
        tok_total = float(t.item())
    value = tok_total / (ms_max * args.steps * 1e-3)

    # per-kernel-class device time over a further measured region
    ctx.profile_enable(True)
    ctx.decode_step(args.profile_steps)
    prof = ctx.profile_read()
    ctx.profile_enable(False)
    ctx.decode_end()

    if args.profile:
        ctx.close()
        return {"metric": METRIC, "value": round(value, 2), "unit": "committed tok/s",
                "ms_per_step": round(ms_max, 3), "kernel_classes": prof,
                "note": "profiling run (no e2e)"}
    # end to end through the public generate call: prompt from host, ids back to host.
    # Five calls; the median is reported and every call's time is kept.  One call spans
    # 513 host round trips, and on a shared machine a host-side stall of 0.4-1.3 s lands
    # in some calls (one to two of three were seen), not in all of them.
    runs = []
    eclk = ClockSampler(local)
    eclk.start()
    time.sleep(0.3)
    et0 = time.time()
    for _ in range(E2E_CALLS):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        barrier(ws)
        e0.record(stream)
        ids, est = ctx.generate_streaming(prompt, NEW_8B, WINDOW_8B, params)
        e1.record(stream)
        torch.cuda.synchronize()
        runs.append(max_over_ranks(e0.elapsed_time(e1) / 1e3, ws))
    e2e_clocks = eclk.stop(et0, time.time())
    e2e_s = sorted(runs)[len(runs) // 2]
    e2e_tok = float(est["tokens_generated"])
    e2e_steps = float(est["steps"])
    if ws > 1:
        import torch.distributed as dist
        t = torch.tensor([e2e_tok, e2e_steps], dtype=torch.float64, device="cuda")
        dist.all_reduce(t)
        e2e_tok, e2e_steps = float(t[0].item()), float(t[1].item()) / ws
    steps_timed = max(n1 - n0, 1)
    # the e2e call's own host<->device copies, counted by the session: the begin / step /
    # result sequence that wedlm_generate_streaming runs, once more with its counters read
    # (prompt ids and the loop's set-up in, one flag per step and the ids out)
    ctx.decode_begin([0], prompt, NEW_8B, WINDOW_8B, params)
    while ctx.decode_step(1 << 30) > 0:
        pass
    ctx.decode_result(0)
    call_steps, call_h2d, call_d2h = ctx.decode_io_bytes()
    ctx.decode_end()
    call_steps = max(call_steps, 1)

    # the reference benchmark's comparison: autoregressive decoding on the same model
    # (engine.rs:160-217), one token per forward at the cached prompt (it needs the whole
    # vocabulary on the context, so the vocabulary-sharded run leaves it out)
    n_ar = 64
    ar = None
    if not sharded:
        ctx.reset_sequence(0)
        ctx.generate_autoregressive(prompt[:64], 4)
        torch.cuda.synchronize()
        a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ctx.reset_sequence(0)
        a0.record(stream)
        ar_ids = ctx.generate_autoregressive(prompt, n_ar)
        a1.record(stream)
        torch.cuda.synchronize()
        ar_s = a0.elapsed_time(a1) / 1e3
        ar = {"value": round(len(ar_ids) / ar_s, 2), "unit": "tok/s", "tokens": len(ar_ids),
              "scope": "wedlm_generate_autoregressive: 512-token prompt prefill + "
                       f"{n_ar} tokens, one per forward",
              "note": "random-init entropy >> tau, so WeDLM commits one token per "
                      "96-row step here; with a trained model it commits several"}
    g = prof["gemm"]
    gemm_gbs = g["bytes"] / (g["ms"] * 1e-3) / 1e9 if g["ms"] > 0 else None
    a = prof["attention"]
    e = prof["entropy"]
    step_ms_prof = sum(v["ms"] for v in prof.values()) / max(args.profile_steps, 1)
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": "committed tok/s",
        "n_gpus": ws, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms_max, 3), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic: random-init N(0,0.02^2) 8B-shape weights, uniform random prompt ids",
        "config": decode_8b_config(),
        # a communicator keeps the host loop (its NCCL steps)
        "decode_loop": "host" if sharded else args.decode_loop,
        "parallelism": (f"dp{ws} sequences + LM head and entropy pass vocabulary-sharded "
                        f"over {ws} GPUs (NCCL all-gathers)" if sharded else
                        f"dp{ws} (one independent sequence per GPU)"),
        "tokens_per_step": round(toks / args.steps, 3),
        "clocks": clocks,
        "e2e": {"value": round(e2e_tok / e2e_s, 2), "unit": "committed tok/s",
                "h2d_bytes_per_step": round(call_h2d / call_steps, 1),
                "d2h_bytes_per_step": round(call_d2h / call_steps, 1),
                "bytes_per_call": {"h2d": int(call_h2d), "d2h": int(call_d2h),
                                   "steps": int(call_steps)},
                "timed_loop_bytes_per_step": {"h2d": round((h1 - h0) / steps_timed, 1),
                                              "d2h": round((d1 - d0) / steps_timed, 1)},
                "tokens": int(e2e_tok), "steps_per_sequence": round(e2e_steps, 1),
                "runs_s": [round(r, 4) for r in runs], "of_runs": f"median of {E2E_CALLS} calls",
                "clocks": e2e_clocks,
                "scope": "wedlm_generate_streaming: 512-token prompt prefill + up to 512 "
                         "tokens (fewer when EOS is generated), host ids in and out"},
        "gpu_launches": int(launches),
        "roofline": {"bound": "hbm", "achieved": round(gemm_gbs, 1) if gemm_gbs else None,
                     "peak": hbm, "peak_kind": peak_kind, "unit": "GB/s",
                     "frac": round(gemm_gbs / hbm, 4) if gemm_gbs else None,
                     "traffic": profile_traffic("gemm_tc_decode_8b"),
                     "per": "decode step (all GEMM-class launches of one step)",
                     "kernel": "gemm_tc_kernel (+ shared-tile reduce): QKV/O/gate-up/down/LM head",
                     "launches_per_step": round(g["launches"] / max(args.profile_steps, 1), 1),
                     "share_of_step": round(g["ms"] / max(sum(v["ms"] for v in prof.values()), 1e-9), 3)},
        "kernel_classes": {k: {"ms_per_step": round(v["ms"] / max(args.profile_steps, 1), 4),
                               "GBps": round(v["bytes"] / (v["ms"] * 1e-3) / 1e9, 1) if v["ms"] > 0 else None,
                               "TFLOPs": round(v["flops"] / (v["ms"] * 1e-3) / 1e12, 1) if v["ms"] > 0 and v["flops"] > 0 else None,
                               "launches_per_step": round(v["launches"] / max(args.profile_steps, 1), 1)}
                           for k, v in prof.items()},
        "profiled_step_ms": round(step_ms_prof, 3),
        "ar_baseline": ar,
    }
    ctx.close()
    del ctx
    torch.cuda.empty_cache()
    if not args.no_entropy:
        args2 = argparse.Namespace(**vars(args))
        args2.profile, args2.no_cpu_baseline, args2.hold_seconds = False, True, 0.5
        es = bench_entropy_select(args2, rank, ws, local)
        line["entropy_select"] = {
            "workload": es["config"]["workload"], "value": es["value"], "unit": "GB/s",
            "ms_per_step": es["ms_per_step"], "roofline": es["roofline"], "e2e": es["e2e"],
            "clocks": es["clocks"]}
    if rank == 0 and ws == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline_decode(args.cpu_seconds)
    return line


def _host_normal(shape, std: float, seed: int, threads: int):
    """N(0, std^2) f32 array drawn on `threads` host threads (numpy's generators release
    the GIL while filling `out`), one independent stream per thread."""
    import numpy as np
    from concurrent.futures import ThreadPoolExecutor
    out = np.empty(shape, np.float32)
    flat = out.reshape(-1)
    n = flat.size
    ss = np.random.SeedSequence(seed).spawn(threads)
    step = (n + threads - 1) // threads

    def fill(i):
        lo, hi = i * step, min(n, (i + 1) * step)
        if lo < hi:
            np.random.Generator(np.random.PCG64(ss[i])).standard_normal(
                out=flat[lo:hi], dtype=np.float32)
            flat[lo:hi] *= np.float32(std)

    with ThreadPoolExecutor(threads) as ex:
        list(ex.map(fill, range(threads)))
    return out


class HostDecodeRun:
    """The reference's streaming decode step on the host cores, measured whole.

    The oracle port of the reference path: the f32 forward of the full 8B-shape model
    (``layers`` decoder layers, hidden 4096, 32/8 heads, SwiGLU 12288, vocabulary
    151936, N(0, 0.02^2) weights, norm weights 1) with the LM head over all window rows
    as ``causal_lm.rs:68-79`` computes it, the entropy / selection / greedy argmax of
    ``sampler.rs`` and the loop of ``wedlm.rs:336-590`` (``oracle/decoder.py``), after
    caching the 512-token prompt.  Every timed step is one real iteration of the loop
    at the bench's cache lengths: nothing is sampled or extrapolated.  A step's time is
    the interval between the starts of consecutive window forwards, which holds the
    forward, the entropy pass, the selection and the commit / refill bookkeeping."""

    def __init__(self, layers: int = 36, seed: int = 0):
        import os as _os
        import numpy as np
        from oracle.model import OracleModel, WeDLMConfig, weight_names
        cfg = WeDLMConfig(**{**WeDLMConfig.wedlm_8b().to_dict(), "num_hidden_layers": layers,
                             "max_position_embeddings": 4096, "dtype": "float32"})
        self.cfg = cfg
        self.threads = _os.cpu_count() or 1
        t0 = time.time()
        w = {}
        for i, (name, shape) in enumerate(weight_names(cfg)):
            w[name] = (np.ones(shape, np.float32) if name.endswith("norm.weight")
                       else _host_normal(shape, 0.02, seed * 1000 + i, self.threads))
        self.model = OracleModel(cfg, w, "f32")
        self.setup_s = time.time() - t0
        self.starts = []
        self.model_forward = self.model.forward_with_positions
        self.model.forward_with_positions = self._timed_forward

    def _timed_forward(self, *a, **k):
        self.starts.append(time.time())
        return self.model_forward(*a, **k)

    def run(self, steps: int, warmup: int):
        """Cache the prompt, run the loop for warmup + steps iterations (and one more to
        close the last interval); returns the seconds of each timed step."""
        from oracle.decoder import OracleDecoder
        from oracle.sampler import SamplingParams as OSP
        prompt = make_prompt(PROMPT_8B, seed=0).tolist()
        dec = OracleDecoder(self.model, self.cfg.mask_token_id, self.cfg.eos_token_id)
        self.starts = []
        t0 = time.time()
        # one committed token per step here (random-init entropy >> tau): max_new tokens
        # take at least max_new + 1 iterations
        _, stats = dec.generate_streaming(prompt, warmup + steps + 1, WINDOW_8B,
                                          OSP(temperature=0.0, entropy_threshold=0.8,
                                              distance_penalty=0.05, max_tokens_per_step=8))
        self.total_s = time.time() - t0
        self.tokens_per_step = stats.tokens_generated / max(stats.steps, 1)
        st = self.starts
        n = min(steps, len(st) - 1 - warmup)
        return [st[warmup + i + 1] - st[warmup + i] for i in range(n)]


def cpu_baseline_decode(budget_s: float):
    """The reference arm's measurement as the GPU line's cpu_baseline: whole 36-layer
    steps of the port (``HostDecodeRun``) after a one-step warm-up, about 2 s each on 16
    cores: 3 of them, or fewer when the budget is below 6 s."""
    run = HostDecodeRun()
    n = 3 if budget_s >= 6.0 else 2
    steps = run.run(steps=n, warmup=1)
    step = sum(steps) / len(steps)
    return {"value": round(1.0 / step, 4), "unit": "committed tok/s", "cores": run.threads,
            "kind": "port",
            "sample": f"{len(steps)} whole streaming steps of the 36-layer f32 port after a "
                      f"512-token prompt (one window forward of 96 rows incl. the LM head over "
                      f"all rows, entropy, selection, commit; {step:.2f} s per step), numpy with "
                      f"{run.threads} BLAS threads; 1 committed token per step (random-init "
                      f"entropy >> tau)"}


def reference_attention(args, rank, ws):
    """--impl reference for block_attention: the reference's attention (attention.rs:188-221:
    scores, additive mask, softmax, weighted sum, GQA by repeating K/V) restated in numpy
    f32 on the host cores, at the largest prefix (8192), same metric (TFLOP/s)."""
    import os as _os
    import numpy as np
    L, S, nh, nkv, d = ATT_PREFIXES[-1], 96, 32, 8, 128
    rng = np.random.default_rng(L)
    q = rng.standard_normal((nh, S, d), dtype=np.float32)
    k = rng.standard_normal((nkv, L + S, d), dtype=np.float32)
    v = rng.standard_normal((nkv, L + S, d), dtype=np.float32)
    rank_ = L + rng.permutation(S)
    mask = np.zeros((S, L + S), np.float32)
    mask[:, L:] = np.where(rank_[None, :] <= rank_[:, None], 0.0, -np.inf)

    def step():
        g = nh // nkv
        kk, vv = np.repeat(k, g, axis=0), np.repeat(v, g, axis=0)
        sc = q @ kk.transpose(0, 2, 1) / np.sqrt(d) + mask[None]
        sc -= sc.max(axis=-1, keepdims=True)
        p = np.exp(sc)
        p /= p.sum(axis=-1, keepdims=True)
        return p @ vv

    for _ in range(max(1, args.warmup // 3)):
        step()
    n = max(2, min(args.steps, 5))
    t0 = time.time()
    for _ in range(n):
        step()
    s_per = (time.time() - t0) / n
    val = attention_flops(L) / s_per / 1e12
    return {"metric": METRIC, "value": round(val, 4), "unit": "TFLOP/s", "n_gpus": 1, "steps": n,
            "warmup": args.warmup, "ms_per_step": round(s_per * 1e3, 2), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic", "impl": "reference",
            "config": {"workload": "block_attention: 8B-shape GQA, 96-row window, prefix 8192, "
                                   "causal over explicit positions"},
            "cpu_baseline": {"value": round(val, 4), "unit": "TFLOP/s", "cores": _os.cpu_count(),
                             "kind": "port", "sample": f"{n} full launches at prefix {L}, numpy f32 with BLAS threads"},
            "e2e": {"value": round(val, 4), "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}


def reference_decode(args, rank, ws):
    """--impl reference for decode_8b: the reference's algorithm on the host cores (the
    oracle port; the Rust crate cannot be built without cargo and candle).  Every step
    is a whole streaming step of the 36-layer model (``HostDecodeRun``), timed as is.
    ``--layers`` shrinks the model for quick contract checks only."""
    layers = args.layers
    run = HostDecodeRun(layers=layers)
    steps = run.run(steps=args.steps, warmup=args.warmup)
    step = sum(steps) / len(steps)
    v = 1.0 / step
    sample = (f"{len(steps)} whole streaming steps after {args.warmup} warm-up steps and the "
              f"512-token prompt: {layers}-layer f32 port, one 96-row window forward incl. the "
              f"LM head over all rows + entropy + selection + commit per step; numpy with "
              f"{run.threads} BLAS threads (weights drawn in {run.setup_s:.1f} s, loop "
              f"{run.total_s:.1f} s)")
    return {"metric": METRIC, "value": round(v, 4), "unit": "committed tok/s",
            "impl": "reference", "n_gpus": ws, "steps": len(steps), "warmup": args.warmup,
            "ms_per_step": round(step * 1e3, 1), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": decode_8b_config(layers),
            "parallelism": f"one host process, {run.threads} BLAS threads",
            "tokens_per_step": round(run.tokens_per_step, 3),
            "cpu_baseline": {"value": round(v, 4), "unit": "committed tok/s",
                             "cores": run.threads, "kind": "port", "sample": sample},
            "e2e": {"value": round(v, 4), "unit": "committed tok/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}


# ----------------------------------------------------------------------------------
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--workload", default="decode_8b",
                    choices=["decode_8b", "entropy_select", "gemm_shapes", "block_attention",
                             "serve_8b"])
    ap.add_argument("--gemm-only", default="", help="comma list of gemm_shapes names")
    ap.add_argument("--gemm-rows", type=int, default=96,
                    help="gemm_shapes: token rows (96 = one decode window; 6144 = serve_8b)")
    ap.add_argument("--profile-steps", type=int, default=10,
                    help="decode steps timed per kernel class after the headline region")
    ap.add_argument("--no-entropy", action="store_true",
                    help="skip the entropy-select sub-measurement of decode_8b")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--nseq", type=int, default=64, help="sequences of 96 mask rows per GPU")
    ap.add_argument("--serve-seqs", type=int, default=SERVE_SEQS,
                    help="serve_8b: sequences in total over all GPUs")
    ap.add_argument("--shard", default="vocab", choices=["vocab", "dp"],
                    help="entropy_select on N > 1 GPUs: shard the vocabulary (NCCL combine of "
                         "per-row partials) or run independent batches")
    ap.add_argument("--lm-head", default="dp", choices=["vocab", "dp"],
                    help="decode_8b on N > 1 GPUs: vocabulary-shard the LM head and the "
                         "entropy pass over the ranks, or keep a whole LM head per GPU")
    ap.add_argument("--hold-seconds", type=float, default=1.0)
    ap.add_argument("--layers", type=int, default=36,
                    help="decoder layers of the decode_8b model (only with --profile: small "
                         "captures of the same kernels)")
    ap.add_argument("--profile", action="store_true",
                    help="short run for ncu: no load hold, no e2e, no CPU baseline")
    ap.add_argument("--decode-loop", default="graph", choices=["graph", "device", "host"],
                    help="decode session bookkeeping: on the device with one CUDA graph per "
                         "step (default), on the device without the graph, or on the host")
    args = ap.parse_args()
    os.environ["WEDLM_DEVICE_LOOP"] = "0" if args.decode_loop == "host" else "1"
    os.environ["WEDLM_STEP_GRAPH"] = "1" if args.decode_loop == "graph" else "0"
    args.warmup = max(args.warmup, 3)
    if args.profile:
        args.hold_seconds, args.no_cpu_baseline = 0.0, True

    if args.impl == "reference":
        rank = int(os.environ.get("RANK", "0"))
        ws = int(os.environ.get("WORLD_SIZE", "1"))
        if rank != 0:
            return
        fn = {"decode_8b": reference_decode, "serve_8b": reference_decode,
              "entropy_select": reference_entropy,
              "block_attention": reference_attention}.get(args.workload)
        if fn is None:
            print(json.dumps({"impl": "reference", "unavailable": "gemm_shapes times single "
                              "kernels of this implementation; the reference has no such unit"}),
                  flush=True)
            return
        print(json.dumps(fn(args, rank, ws)), flush=True)
        return

    rank, ws, local = dist_setup(args.gpus)
    if args.workload == "decode_8b":
        line = bench_decode_8b(args, rank, ws, local)
    elif args.workload == "gemm_shapes":
        line = bench_gemm_shapes(args, rank, ws, local)
    elif args.workload == "block_attention":
        line = bench_block_attention(args, rank, ws, local)
    elif args.workload == "serve_8b":
        line = bench_serve_8b(args, rank, ws, local)
    else:
        line = bench_entropy_select(args, rank, ws, local)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if ws > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
