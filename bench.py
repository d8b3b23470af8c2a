"""Benchmark of the quantized-linear hot path (one JSON line on rank 0).

Default workload = BASELINE config 1: AWQ W4A16 linear, K=4096, N=14336,
group 128, swept over M in {1, 16, 128, 1024, 4096} (decode GEMV through
prefill GEMM).  One *step* = one call of the AWQ linear at every M of the
sweep (5 launches).  ``value`` = sweep FLOPs / device time (TFLOP/s), inputs
resident in HBM, each timed step's five calls back to back as a serving step
runs them (programmatic dependent launch between consecutive kernels), the
dominant M=4096 call between an event pair of its own for the roofline;
``sweep`` gives each call's device time chained (``us``: a CUDA graph of
back-to-back calls of one M) and with a launch of its own (``us_event``: an event
pair around every call, a separate pass); ``e2e`` = the same metric through the public
API with host (pinned) activations copied in and outputs copied back inside the
timed region (copies on their own streams, overlapping the neighbouring calls'
compute, as a serving loop pipelines them).

L2 hygiene: the timed loop rotates over enough weight copies that the set
streamed between two uses of a copy exceeds 2x the 126 MB L2.

The line also carries ``fp8_sweep``: BASELINE config 2 (FP8 W8A8, (K, N) in
{(4096,4096), (4096,28672), (14336,4096)} x M in {1, 32, 512, 8192}), device
time per quant+GEMM call, as context (``--no-fp8`` skips it).  ``--case`` runs
a few launches of one shape for ncu captures.

``--impl reference`` times the reference side on the same workload: the
reference has no CPU implementation of this path, so the CPU restatement in
oracle/ (OpenMP, all host threads) is timed on a bounded sample; where the
reference's own linear_fwd was compiled (oracle/_ref) its GPU time on the
dequantised weights is reported next to it.

The line also carries ``decode``: BASELINE configs 3 and 4, one decode step of
the Llama-3-8B AWQ and Llama-3-70B FP8 decoders (random weights, KV cache filled
to the context) on this package's kernels, captured as one CUDA graph, tok/s per
batch; ``--no-decode`` skips it, ``--decode 8b-awq|70b-fp8`` runs one of them
alone (``--batch``, ``--ctx``).

Multi-GPU (torchrun, one process per GPU): the config-1 sweep runs on every rank
with its own weights (replicas, weak scaling, no collective on the data path);
the decode blocks run tensor parallel over all ranks (column-parallel q/k/v and
gate/up, row-parallel o and down with the one-shot NVLink all-reduce), so their
tok/s at N GPUs is strong scaling of a fixed batch.  Timing is the max over ranks.
"""
from __future__ import annotations

import argparse
import json
import os
import pathlib
import statistics
import subprocess
import sys
import threading
import time

import numpy as np
import torch

ROOT = pathlib.Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}

AWQ_K, AWQ_N, AWQ_G = 4096, 14336, 128
AWQ_MS = [1, 16, 128, 1024, 4096]
AWQ_WORKLOAD = "config1: AWQ W4A16 K=4096 N=14336 g=128, M in {1,16,128,1024,4096}"
FP8_K, FP8_N = 4096, 28672
FP8_MS = [1, 32, 512, 8192]
# DRAM bytes (read + write) of one awq_gemm_tmem_kernel<256> launch at M=4096 and
# how they were captured (ncu cannot run inside the timed bench; the figure is
# re-captured whenever the kernel changes and printed with its source).
AWQ_GEMM_M4096_DRAM_BYTES = 93_518_848 + 74_575_360
AWQ_GEMM_M4096_TRAFFIC_SOURCE = (
    "ncu --metrics dram__bytes_read.sum,dram__bytes_write.sum,gpu__time_duration.sum "
    "--clock-control none -k regex:awq_gemm_tmem -s 1 -c 1 python bench.py --case awq:4096 "
    "(93.52 MB read + 74.58 MB written; awq_gemm_tmem_kernel<256, 128, __half>, 128-deep "
    "K-blocks, 374.0 us cold-cache under ncu)")


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d, "measured"
    return dict(FALLBACK_PEAKS), "fallback"


# ------------------------------------------------------------------ clocks
class ClockSampler:
    """nvidia-smi sampling during the timed region (SM clock, throttle reasons)."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []
        self.t = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (OSError, ValueError):
            self.proc = None
            return
        self.t = threading.Thread(target=self._read, daemon=True)
        self.t.start()

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        if self.t:
            self.t.join(timeout=2)
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax = float(parts[2])
            except ValueError:
                continue
            for nm, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax,
                "reasons": sorted(reasons), "samples": len(sm)}


# --------------------------------------------------------------- workloads
def awq_weights(device, copies, seed=0):
    """Seeded config-1 AWQ weights (draw order q, z, s), `copies` independent copies
    made by rotating the packed words so every copy is distinct memory."""
    rng = np.random.default_rng(seed)
    K, N, g = AWQ_K, AWQ_N, AWQ_G
    q = rng.integers(0, 16, size=(K, N), dtype=np.int64).astype(np.uint32)
    z = rng.integers(0, 16, size=(K // g, N), dtype=np.int64).astype(np.uint32)
    s = rng.uniform(0.001, 0.02, size=(K // g, N)).astype(np.float16)
    order = np.array([0, 2, 4, 6, 1, 3, 5, 7])
    sh = (4 * np.arange(8, dtype=np.uint32))

    def pack(a):
        a = a.reshape(a.shape[0], -1, 8)[:, :, order]
        return (a << sh).sum(axis=2, dtype=np.uint64).astype(np.uint32).view(np.int32)

    qw = torch.from_numpy(pack(q)).to(device)
    qz = torch.from_numpy(pack(z)).to(device)
    sc = torch.from_numpy(s).to(device)
    out = []
    for c in range(copies):
        out.append((qw.roll(c, 0).contiguous() if c else qw, qz, sc))
    return out


def awq_flops(M):
    return 2.0 * M * AWQ_K * AWQ_N


def awq_bytes(M):
    K, N, g = AWQ_K, AWQ_N, AWQ_G
    return K * N / 2 + (K // g) * (N // 8) * 4 + (K // g) * N * 2 + 2 * M * K + 2 * M * N


def fp8_flops(M):
    return 2.0 * M * FP8_K * FP8_N


def fp8_bytes(M):
    return 2 * M * FP8_K + FP8_N * FP8_K + 4 * FP8_N + 2 * M * FP8_N


# ------------------------------------------------------------------ timing
def time_sweep(calls, steps, warmup, stream, timed=None, barrier=None):
    """calls: list of (name, fn).  Returns (total_ms, per-call mean ms).  Calls
    whose index is in `timed` (all when None) get an event pair of their own;
    the others run back to back with their neighbours (programmatic dependent
    launch between consecutive kernels), and their per-call entry is None."""
    timed = set(range(len(calls))) if timed is None else set(timed)
    for _ in range(warmup):
        for _, fn in calls:
            fn(0)
    torch.cuda.synchronize()
    if barrier is not None:  # every rank starts the timed steps together
        barrier()
    ev = [[(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in calls] for _ in range(steps)]
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for i in range(steps):
        for j, (_, fn) in enumerate(calls):
            if j in timed:
                ev[i][j][0].record(stream)
            fn(i + 1)
            if j in timed:
                ev[i][j][1].record(stream)
    t1.record(stream)
    torch.cuda.synchronize()
    total = t0.elapsed_time(t1)
    per = [sum(ev[i][j][0].elapsed_time(ev[i][j][1]) for i in range(steps)) / steps
           if j in timed else None for j in range(len(calls))]
    return total, per


def max_over_ranks(v, dist_on, device):
    if not dist_on:
        return v
    import torch.distributed as dist
    t = torch.tensor([v], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def run_awq(args, device, dist_on, world, rank):
    import lmrs_b200 as L
    copies = 8
    W = awq_weights(device, copies)
    K, N, g = AWQ_K, AWQ_N, AWQ_G
    gen = torch.Generator(device="cpu").manual_seed(1)
    xs = {M: torch.randn(M, K, generator=gen).half().to(device) for M in AWQ_MS}
    ys = {M: torch.empty(M, N, dtype=torch.float16, device=device) for M in AWQ_MS}
    stream = torch.cuda.current_stream(device)

    def mk(M):
        def f(i):
            qw, qz, sc = W[i % copies]
            L.awq_linear(xs[M], qw, qz, sc, None, g, out=ys[M])
        return f

    calls = [(f"M={M}", mk(M)) for M in AWQ_MS]

    # per-call device time chained as in a decode / serving step (a graph of
    # back-to-back calls with programmatic dependent launch between them)
    chain_us = [graph_time(fn, 24) for _, fn in calls]
    if dist_on:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    clk = ClockSampler(torch.cuda.current_device() if "CUDA_VISIBLE_DEVICES" not in os.environ
                       else int(os.environ["CUDA_VISIBLE_DEVICES"].split(",")[torch.cuda.current_device()]))
    clk.start()
    # the timed steps: the five calls back to back as a serving step runs them
    # (programmatic dependent launch between consecutive kernels); the dominant
    # call (M=4096, ~2/3 of the step) has an event pair of its own for the roofline
    dom = AWQ_MS.index(4096)
    total_ms, per_dom = time_sweep(calls, args.steps, args.warmup, stream, timed=[dom],
                                   barrier=torch.distributed.barrier if dist_on else None)
    clocks = clk.stop()
    # per-call device time with a launch of its own (event pair around every call),
    # a separate pass outside the headline: `us_event` in the sweep
    _, per_ms = time_sweep(calls, args.steps, 1, stream)
    if dist_on:
        torch.distributed.barrier()
    total_ms = max_over_ranks(total_ms, dist_on, device)
    flops_step = sum(awq_flops(M) for M in AWQ_MS)
    ms_step = total_ms / args.steps
    value = world * flops_step / (ms_step * 1e-3) / 1e12

    # ---- e2e: host activations in (pinned), outputs back, through the public API.
    # Three streams pipeline the calls as a serving loop would: a call's input is
    # copied in and the previous call's output copied out while it computes
    # (double-buffered device tensors; every call's copies are inside the timed
    # region, and a buffer is refilled only after its last reader finished).
    hx = {M: xs[M].cpu().pin_memory() for M in AWQ_MS}
    hy = {M: torch.empty(M, N, dtype=torch.float16).pin_memory() for M in AWQ_MS}
    xdb = {M: [torch.empty_like(xs[M]) for _ in range(2)] for M in AWQ_MS}
    ydb = {M: [torch.empty_like(ys[M]) for _ in range(2)] for M in AWQ_MS}
    s_in, s_out = torch.cuda.Stream(device), torch.cuda.Stream(device)
    ev_done, ev_out = {}, {}

    def e2e_step(i):
        bi = i & 1
        for M in AWQ_MS:
            qw, qz, sc = W[i % copies]
            key = (M, bi)
            with torch.cuda.stream(s_in):
                if key in ev_done:
                    s_in.wait_event(ev_done[key])      # the call that read this buffer is done
                xdb[M][bi].copy_(hx[M], non_blocking=True)
                ev_in = torch.cuda.Event()
                ev_in.record(s_in)
            stream.wait_event(ev_in)
            if key in ev_out:
                stream.wait_event(ev_out[key])         # this output buffer was copied out
            L.awq_linear(xdb[M][bi], qw, qz, sc, None, g, out=ydb[M][bi])
            ev_done[key] = torch.cuda.Event()
            ev_done[key].record(stream)
            with torch.cuda.stream(s_out):
                s_out.wait_event(ev_done[key])
                hy[M].copy_(ydb[M][bi], non_blocking=True)
                ev_out[key] = torch.cuda.Event()
                ev_out[key].record(s_out)

    for i in range(args.warmup):
        e2e_step(i)
    torch.cuda.synchronize()
    if dist_on:
        torch.distributed.barrier()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    s_in.wait_stream(stream)
    s_out.wait_stream(stream)
    for i in range(args.steps):
        e2e_step(i + 1)
    stream.wait_stream(s_in)
    stream.wait_stream(s_out)
    b.record(stream)
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks(a.elapsed_time(b) / args.steps, dist_on, device)
    h2d = sum(2 * M * K for M in AWQ_MS)
    d2h = sum(2 * M * N for M in AWQ_MS)

    pk, pk_kind = peaks()
    sweep = []
    for M, t, tc in zip(AWQ_MS, per_ms, chain_us):
        bound = "hbm" if M <= 64 else "tensor"
        gbs = awq_bytes(M) / (tc * 1e-6) / 1e9
        tfl = awq_flops(M) / (tc * 1e-6) / 1e12
        frac = gbs / pk["hbm_gbs"] if bound == "hbm" else tfl / pk["bf16_tflops"]
        ev_frac = (awq_bytes(M) / (t * 1e-3) / 1e9 / pk["hbm_gbs"] if bound == "hbm"
                   else awq_flops(M) / (t * 1e-3) / 1e12 / pk["bf16_tflops"])
        sweep.append({"M": M, "us": round(tc, 2), "GB_s": round(gbs, 1),
                      "TFLOP_s": round(tfl, 2), "bound": bound, "frac": round(frac, 4),
                      "us_event": round(t * 1e3, 2), "frac_event": round(ev_frac, 4)})
    # dominant kernel (M=4096), timed inside the headline's steps
    Md = AWQ_MS[dom]
    ach = awq_flops(Md) / (per_dom[dom] * 1e-3) / 1e12
    roof = {"bound": "tensor", "kernel": f"awq_gemm_tmem_kernel<256> (M={Md})", "achieved": round(ach, 2),
            "peak": pk["bf16_tflops"], "unit": "TFLOP/s", "frac": round(ach / pk["bf16_tflops"], 4),
            "peak_source": f"{pk_kind} bf16 dense (burst)",
            "traffic": AWQ_GEMM_M4096_DRAM_BYTES if Md == 4096 else None,
            "traffic_source": AWQ_GEMM_M4096_TRAFFIC_SOURCE if Md == 4096 else None,
            "traffic_unit": "bytes per launch (ncu dram__bytes_read.sum + dram__bytes_write.sum)",
            "algorithmic_bytes": awq_bytes(Md), "algorithmic_flops": awq_flops(Md)}
    return dict(
        metric="awq_w4a16_linear_throughput_config1_sweep", value=round(value, 3), unit="TFLOP/s",
        ms_per_step=round(ms_step, 4), dtype="f16 (int4 weights, fp32 accumulate)",
        config={"workload": AWQ_WORKLOAD,
                "global_batch": sum(AWQ_MS), "parallelism": f"replicas{world}",
                "timing": "each timed step's five calls back to back (programmatic dependent launch), the M=4096 call between an event pair of its own",
                "l2": f"rotating {copies} weight copies ({copies * awq_bytes(0) / 1e6:.0f} MB > 2x L2)"},
        roofline=roof, sweep=sweep, clocks=clocks,
        e2e={"value": round(world * flops_step / (e2e_ms * 1e-3) / 1e12, 3), "unit": "TFLOP/s",
             "ms_per_step": round(e2e_ms, 4), "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
        gpu_launches=args.steps * len(AWQ_MS),
        _peaks=pk, _weights=W)


# Columns of the config-1 weight the CPU arm computes per step: every M of the
# sweep, full K, this many of the N = 14336 output channels (the work per output
# is the same K-long dot product, so the TFLOP/s of the slice is the sweep's).
CPU_SAMPLE_COLS = 1024


def cpu_sweep(nthreads, steps, warmup, ncols=CPU_SAMPLE_COLS):
    """The config-1 sweep on the host cores through the oracle's OpenMP C
    restatement (dequant + fp32-FMA linear, the reference's linear_kernel
    arithmetic): each step is one call at every M in the sweep on the first
    `ncols` output channels of the seeded config-1 weights.  Returns the
    cpu_baseline dict (value in TFLOP/s)."""
    from oracle import oracle as O
    K, N, g = AWQ_K, AWQ_N, AWQ_G
    d = O.awq_inputs(max(AWQ_MS), K, N, g, seed=0)
    qw = np.ascontiguousarray(d["qweight"][:, :ncols // 8])
    qz = np.ascontiguousarray(d["qzeros"][:, :ncols // 8])
    sc = np.ascontiguousarray(d["scales"][:, :ncols])
    xs = {M: np.ascontiguousarray(d["x"][:M]) for M in AWQ_MS}

    def step():
        for M in AWQ_MS:
            O.c_awq_linear(xs[M], qw, qz, sc, None, M, K, ncols, g, nthreads=nthreads)

    for _ in range(warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(steps):
        step()
    t = time.perf_counter() - t0
    fl = steps * sum(2.0 * M * K * ncols for M in AWQ_MS)
    # config 0 (M=8, K=N=4096, g=128), the reference's CPU-runnable case, whole
    d0 = O.awq_inputs(8, 4096, 4096, 128, seed=0)
    reps, t0c = 5, time.perf_counter()
    for _ in range(reps):
        O.c_awq_linear(d0["x"], d0["qweight"], d0["qzeros"], d0["scales"], None, 8, 4096, 4096,
                       128, nthreads=nthreads)
    c0_ms = (time.perf_counter() - t0c) / reps * 1e3
    return {"value": round(fl / t / 1e12, 5), "unit": "TFLOP/s", "cores": nthreads, "kind": "port",
            "steps": steps, "warmup": warmup, "ms_per_step": round(t / steps * 1e3, 2),
            "sample": f"every M in {AWQ_MS} of the config-1 sweep, K=4096, the first {ncols} of "
                      f"the 14336 output channels per step (dequant + fp32-FMA linear, "
                      f"oracle/lmrs_oracle.c, OpenMP over {nthreads} host threads)",
            "config0": {"M": 8, "K": 4096, "N": 4096, "group": 128, "ms": round(c0_ms, 2),
                        "TFLOP_s": round(2.0 * 8 * 4096 * 4096 / (c0_ms * 1e-3) / 1e12, 5),
                        "what": "whole config-0 AWQ linear, median-free mean of 5 calls"}}


def ref_gpu_linear_fwd(device, steps=2):
    """The reference's own linear_fwd (oracle/_ref, its kernels/ffi/tensor_ffi.cu
    built unchanged) on the config-1 weights dequantised on the host by the
    oracle; loads nothing of this package."""
    import ctypes
    so = ROOT / "oracle" / "_ref" / "libref_ffi.so"
    if not so.exists():
        return None
    from oracle import oracle as O
    lib = ctypes.CDLL(str(so))
    P, I = ctypes.c_void_p, ctypes.c_int
    lib.linear_fwd.argtypes = [P, P, P, P, I, I, I, I, P]
    d = O.awq_inputs(max(AWQ_MS), AWQ_K, AWQ_N, AWQ_G, seed=0)
    w_kn = O.c_awq_dequant(d["qweight"], d["qzeros"], d["scales"], AWQ_K, AWQ_N, AWQ_G)
    w_nk = torch.from_numpy(np.ascontiguousarray(w_kn.T)).to(device)
    xall = torch.from_numpy(d["x"]).to(device)
    stream = torch.cuda.current_stream(device)
    res = []
    tot_fl, tot_ms = 0.0, 0.0
    for M in AWQ_MS:
        x = xall[:M].contiguous()
        y = torch.empty(M, AWQ_N, dtype=torch.float16, device=device)
        call = lambda: lib.linear_fwd(P(y.data_ptr()), P(x.data_ptr()), P(w_nk.data_ptr()), None,
                                      M, AWQ_K, AWQ_N, 1, P(stream.cuda_stream))
        call()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(steps):
            call()
        b.record(stream)
        torch.cuda.synchronize()
        ms = a.elapsed_time(b) / steps
        tot_fl += awq_flops(M)
        tot_ms += ms
        res.append({"M": M, "us": round(ms * 1e3, 1), "TFLOP_s": round(awq_flops(M) / ms / 1e9, 3)})
    return {"kernel": "reference linear_fwd (kernels/ffi/tensor_ffi.cu, sm_100a, fp16, "
                      "on dequantised weights)",
            "value": round(tot_fl / (tot_ms * 1e-3) / 1e12, 4), "unit": "TFLOP/s", "sweep": res}


def run_case(case, launches=3):
    """A handful of launches of one kernel shape, for ncu captures."""
    import lmrs_b200 as L
    dev = torch.device("cuda", 0)
    kind, *dims = case.split(":")
    if kind == "awq":
        M = int(dims[0])
        W = awq_weights(dev, 1)
        x = torch.randn(M, AWQ_K, device=dev).half()
        for _ in range(launches):
            L.awq_linear(x, *W[0], None, AWQ_G)
    elif kind == "fp8":
        M, K, N = (int(v) for v in dims)
        w = (torch.randn(N, K, device=dev) * 0.02).bfloat16()
        wq, sw = L.quantize_fp8_weight(w)
        x = torch.randn(M, K, device=dev).bfloat16()
        ws = L.Workspace()
        for _ in range(launches):
            L.fp8_linear(x, wq, sw, None, ws)
    elif kind == "attn":
        # paged decode attention: batch, q heads, KV heads, context (grouped heads)
        import math
        from lmrs_b200 import decode_ops as DO
        B, hq, hkv, ctx = (int(v) for v in dims)
        kc = torch.randn(B, hkv, ctx, 128, device=dev).bfloat16()
        vc = torch.randn_like(kc)
        q = torch.randn(B, hq, 128, device=dev).bfloat16()
        tables = torch.arange(B, dtype=torch.int32, device=dev).view(B, 1)
        lens = torch.full((B,), ctx, dtype=torch.int32, device=dev)
        ws = DO.AttentionWorkspace()
        for _ in range(launches):
            DO.paged_attention_decode(q, kc, vc, tables, lens, ctx, 1 / math.sqrt(128), 1, ws)
    elif kind == "decode":
        # eager decode steps of a config-3/4 decoder cut to `layers` layers:
        # decode:<8b-awq|70b-fp8>:<batch>:<layers>[:tp<N>]; tp<N>: the shapes one
        # of N tensor-parallel ranks holds (heads, KV heads, intermediate and
        # vocabulary divided by N), on this one GPU with no collective
        import dataclasses
        from lmrs_b200 import decoder as D
        preset, B, nl = dims[0], int(dims[1]), int(dims[2])
        attr, ctx, _, _ = DECODE_PRESETS[preset]
        cfg = dataclasses.replace(getattr(D, attr), layers=nl)
        if len(dims) > 3 and dims[3].startswith("tp"):
            n = int(dims[3][2:])
            cfg = dataclasses.replace(cfg, heads=cfg.heads // n, kv_heads=cfg.kv_heads // n,
                                      intermediate=cfg.intermediate // n, vocab=cfg.vocab // n)
        dec = D.QuantDecoder(cfg, batch=B, ctx=ctx, device=dev, seed=0)
        for _ in range(launches):
            dec.logits()
    else:
        raise SystemExit(f"unknown case {case}")
    torch.cuda.synchronize()
    print(f"case {case}: ok, device error word {L.read_device_error()}")


def graph_time(fn, steps):
    """Device time per call with host launch overhead removed: `steps` calls are
    captured into one CUDA graph after 3 eager warm-up calls and replayed."""
    for i in range(3):
        fn(i)
    torch.cuda.synchronize()
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            for i in range(steps):
                fn(i)
    torch.cuda.synchronize()
    g.replay()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    g.replay()
    b.record()
    torch.cuda.synchronize()
    del g
    return a.elapsed_time(b) / steps * 1e3


def measure_fp8_peak(device, n=8192, reps=10):
    """FP8 dense denominator measured in this run, the way the driver measures
    the bf16 one: a library e4m3 GEMM (torch._scaled_mm, cuBLASLt) at n^3, best
    of `reps` event-timed calls.  MEASURED_PEAKS.json holds no FP8 figure."""
    try:
        a = torch.randn(n, n, device=device).to(torch.float8_e4m3fn)
        b = torch.randn(n, n, device=device).to(torch.float8_e4m3fn).t()
        one = torch.ones((), device=device)
        for _ in range(3):
            torch._scaled_mm(a, b, scale_a=one, scale_b=one, out_dtype=torch.bfloat16)
        torch.cuda.synchronize()
        best = None
        for _ in range(reps):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            torch._scaled_mm(a, b, scale_a=one, scale_b=one, out_dtype=torch.bfloat16)
            e1.record()
            torch.cuda.synchronize()
            ms = e0.elapsed_time(e1)
            best = ms if best is None else min(best, ms)
        del a, b
        torch.cuda.empty_cache()
        return (round(2.0 * n ** 3 / (best * 1e-3) / 1e12, 1),
                f"measured in this run: torch._scaled_mm e4m3 {n}^3 -> bf16, best of {reps}")
    except Exception as e:  # an older torch without this signature
        return None, f"unavailable: {type(e).__name__}"


def fp8_sweep(device, steps=5):
    """Config 2: FP8 W8A8 (K, N) x M, device time per call (context for the line)."""
    import lmrs_b200 as L
    out = []
    pk, _ = peaks()
    fp8_peak, fp8_src = measure_fp8_peak(device)
    if fp8_peak is None:
        fp8_peak, fp8_src = 2 * pk["bf16_tflops"], "2 x the bf16 dense burst (scaled_mm unavailable)"
    for K, N in ((4096, 4096), (4096, 28672), (14336, 4096)):
        copies = max(2, int(3e8 // (N * K)))
        w = (torch.randn(N, K, device=device) * 0.02).bfloat16()
        wqs = [L.quantize_fp8_weight(w.roll(i, 0).contiguous()) for i in range(copies)]
        del w
        for M in FP8_MS:
            x = torch.randn(M, K, device=device).bfloat16()
            y = torch.empty(M, N, dtype=torch.bfloat16, device=device)
            ws = L.Workspace()
            ws.get(L.load_library().lmrs_fp8_linear_workspace_bytes(M, K, N), device)
            us = graph_time(lambda i: L.fp8_linear(x, *wqs[i % copies], None, ws, out=y), steps)
            byts = 2 * M * K + N * K + 4 * N + 2 * M * N
            tfl = 2.0 * M * K * N / us / 1e6
            gbs = byts / us / 1e3
            bound = "hbm" if M <= 256 else "tensor"
            frac = gbs / pk["hbm_gbs"] if bound == "hbm" else tfl / fp8_peak
            out.append({"K": K, "N": N, "M": M, "us": round(us, 2), "GB_s": round(gbs, 1),
                        "TFLOP_s": round(tfl, 2), "bound": bound, "frac": round(frac, 4)})
        del wqs
        torch.cuda.empty_cache()
    return {"config": "config2: FP8 W8A8, quant + GEMM per call, bf16 in/out; device time per "
                      "call from a CUDA-graph replay (host launch overhead excluded)",
            "fp8_peak_tflops": fp8_peak, "fp8_peak_source": fp8_src,
            "fp8_peak_2x_bf16": 2 * pk["bf16_tflops"],
            "points": out}


# ----------------------------------------------------------- decode (configs 3/4)
DECODE_PRESETS = {
    # name: (config attribute, context, batches, BASELINE config)
    "8b-awq": ("LLAMA3_8B_AWQ", 2048, (1, 16, 64), "config3"),
    "70b-fp8": ("LLAMA3_70B_FP8", 4096, (1, 32, 256), "config4"),
}


def _graph_ms(g, steps, warmup, stream, dist_on, device):
    """Per-replay device time of a captured graph: `warmup` untimed replays, then
    `steps` replays each bracketed by events; barrier + synchronize on both sides;
    returns (mean ms, median ms), each the max over ranks."""
    for _ in range(warmup):
        g.replay()
    torch.cuda.synchronize()
    if dist_on:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(steps)]
    for a, b in ev:
        a.record(stream)
        g.replay()
        b.record(stream)
    torch.cuda.synchronize()
    if dist_on:
        torch.distributed.barrier()
    ts = [a.elapsed_time(b) for a, b in ev]
    return (max_over_ranks(sum(ts) / len(ts), dist_on, device),
            max_over_ranks(statistics.median(ts), dist_on, device))


def run_decode(args, device, dist_on, world, rank, preset=None, batches=None, ctx=None):
    """Configs 3/4: one decode step of the Llama-shaped decoder (tensor parallel
    over the ranks), captured as one CUDA graph (all-reduces included) and
    replayed.  tok/s = batch / step time; the linear share replays the step's
    quantized projections alone."""
    from lmrs_b200 import decoder as D
    preset = preset or args.decode
    attr, ctx0, batches0, cname = DECODE_PRESETS[preset]
    cfg = getattr(D, attr)
    if getattr(args, "act", None) and cfg.quant == "awq":
        import dataclasses
        cfg = dataclasses.replace(cfg, act=args.act)
    ctx = ctx or args.ctx or ctx0
    if batches is None:
        batches = tuple(int(b) for b in args.batch.split(",")) if args.batch else batches0
    pg = torch.distributed.group.WORLD if dist_on else None
    stream = torch.cuda.current_stream(device)
    total = torch.cuda.get_device_properties(device).total_memory
    act_bytes = 2
    lin_b = cfg.linear_bytes(world)
    head_b = cfg.vocab // world * cfg.hidden * act_bytes
    embed_b = cfg.vocab * cfg.hidden * act_bytes
    pk, pk_kind = peaks()
    dec, points = None, []
    t_init = time.perf_counter()
    clk = ClockSampler(torch.cuda.current_device() if "CUDA_VISIBLE_DEVICES" not in os.environ
                       else int(os.environ["CUDA_VISIBLE_DEVICES"].split(",")[torch.cuda.current_device()]))
    clk_started = False
    for B in batches:
        kv_b = D.QuantDecoder.kv_bytes(cfg, B, ctx, world)
        need = lin_b + head_b + embed_b + kv_b
        if need > total - (8 << 30):  # same decision on every rank (all shapes are equal)
            points.append({"batch": B, "status": "does not fit",
                           "need_gb_per_gpu": round(need / 1e9, 1),
                           "hbm_gb_per_gpu": round(total / 1e9, 1)})
            continue
        if dec is None:
            dec = D.QuantDecoder(cfg, B, ctx, device, rank, world, seed=0, group=pg)
            torch.cuda.synchronize()
            init_s = time.perf_counter() - t_init
        else:
            dec.set_batch(B)
        g, out = D.graph_step(dec)
        gl, _ = D.graph_step(dec, dec.linears_only)
        if not clk_started:
            clk.start()
            clk_started = True
        step_ms, step_med = _graph_ms(g, args.steps, args.warmup, stream, dist_on, device)
        lin_ms, _ = _graph_ms(gl, args.steps, args.warmup, stream, dist_on, device)
        del gl
        ar_ms = None
        if dist_on:
            y = torch.zeros(B, cfg.hidden, dtype=dec.act, device=device)
            sg = torch.cuda.Stream(device)
            sg.wait_stream(stream)
            with torch.cuda.stream(sg):
                dec._all_reduce(y)
            stream.wait_stream(sg)
            torch.cuda.synchronize()
            ga = torch.cuda.CUDAGraph()
            with torch.cuda.graph(ga):
                for _ in range(2 * cfg.layers):
                    dec._all_reduce(y)   # the step's own all-reduce path (peer or NCCL)
            ar_ms, _ = _graph_ms(ga, args.steps, args.warmup, stream, dist_on, device)
            del ga
        # e2e: token ids in from pinned host memory, next tokens back, every step
        htok = dec.tokens.cpu().pin_memory()
        hout = torch.empty_like(out, device="cpu").pin_memory()
        for _ in range(args.warmup):
            dec.tokens.copy_(htok, non_blocking=True)
            g.replay()
            hout.copy_(out, non_blocking=True)
        torch.cuda.synchronize()
        if dist_on:
            torch.distributed.barrier()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(args.steps):
            dec.tokens.copy_(htok, non_blocking=True)
            g.replay()
            hout.copy_(out, non_blocking=True)
        b.record(stream)
        torch.cuda.synchronize()
        e2e_ms = max_over_ranks(a.elapsed_time(b) / args.steps, dist_on, device)
        del g
        byts = lin_b + head_b + kv_b   # per rank, per step (weights + LM head + KV read)
        gbs = byts / (step_med * 1e-3) / 1e9
        points.append({
            "batch": B, "ms_per_step": round(step_ms, 4), "ms_median": round(step_med, 4),
            "tok_s": round(B / (step_med * 1e-3), 1),
            "e2e_tok_s": round(B / (e2e_ms * 1e-3), 1), "e2e_ms_per_step": round(e2e_ms, 4),
            "own_launches_per_step": dec.own_launches_per_step(),
            "linear_ms": round(lin_ms, 4), "linear_share": round(lin_ms / step_med, 4),
            "linear_GB_s": round(lin_b / (lin_ms * 1e-3) / 1e9, 1),
            "linear_frac_hbm": round(lin_b / (lin_ms * 1e-3) / 1e9 / pk["hbm_gbs"], 4),
            "allreduce_ms": None if ar_ms is None else round(ar_ms, 4),
            "bytes_per_step_per_gpu": byts, "GB_s_per_gpu": round(gbs, 1),
            "frac_hbm": round(gbs / pk["hbm_gbs"], 4),
            "h2d_bytes_per_step": B * 8, "d2h_bytes_per_step": B * 8})
    clocks = clk.stop() if clk_started else None
    ok = [p for p in points if "tok_s" in p]
    best = max(ok, key=lambda p: p["batch"]) if ok else None
    line = {"metric": f"decode_tok_s_{cname}", "value": best["tok_s"] if best else None,
            "unit": "tok/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": best["ms_median"] if best else None, "higher_is_better": True,
            "scaling": "strong" if world > 1 else "weak", "vs_baseline": None,
            "dtype": f"{cfg.act} act, int4 weights" if cfg.quant == "awq" else "bf16 act, e4m3 W8A8",
            "data": "synthetic (random-init weights, random KV cache and token ids)",
            "config": {"workload": f"{cname}: {preset} decoder, one decode step at ctx {ctx}, "
                                   f"value = largest batch that fits",
                       "layers": cfg.layers, "hidden": cfg.hidden, "ctx": ctx,
                       "parallelism": f"tp{world}", "l2": "weights + KV per step >> L2"},
            "points": points, "clocks": clocks, "peak_hbm_gbs": pk["hbm_gbs"],
            "peak_source": pk_kind,
            "init_s": round(init_s, 1) if dec is not None else None}
    if dec is not None:
        dec.close()
    del dec
    return line


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["lmrs", "reference"], default="lmrs")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-fp8", action="store_true", help="skip the config-2 FP8 context sweep")
    ap.add_argument("--case", default=None,
                    help="profiling mode: run a few launches of one case and exit, e.g. "
                         "awq:4096 (config-1 shape, M=4096), fp8:8192:4096:28672 (M:K:N) or "
                         "attn:64:32:8:2048 (paged decode attention B:q heads:KV heads:ctx) or "
                         "decode:8b-awq:16:2 (eager decode steps, preset:batch:layers)")
    ap.add_argument("--decode", choices=sorted(DECODE_PRESETS), default=None,
                    help="configs 3/4: decode tok/s of the 8B AWQ or 70B FP8 decoder "
                         "(tensor parallel over the torchrun ranks)")
    ap.add_argument("--batch", default=None, help="decode batches, comma separated")
    ap.add_argument("--ctx", type=int, default=None, help="decode context length")
    ap.add_argument("--act", choices=["bf16", "f16"], default=None,
                    help="activation dtype of the AWQ decoder (default bf16, config 3's)")
    ap.add_argument("--no-decode", action="store_true",
                    help="skip the configs 3/4 decode blocks of the default line")
    args = ap.parse_args()
    if args.case:
        run_case(args.case)
        return
    args.warmup = max(args.warmup, 3)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dist_on = world > 1
    if dist_on:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    nthreads = os.cpu_count() or 1

    if args.impl == "reference":
        if rank != 0:
            if dist_on:
                torch.distributed.destroy_process_group()
            return
        cb = cpu_sweep(nthreads, args.steps, args.warmup)
        rg = ref_gpu_linear_fwd(device)
        line = {"metric": "awq_w4a16_linear_throughput_config1_sweep", "value": cb["value"],
                "unit": "TFLOP/s", "impl": "reference", "n_gpus": args.gpus,
                "steps": args.steps, "warmup": args.warmup,
                "ms_per_step": cb["ms_per_step"], "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "f16 (int4 weights, fp32 accumulate)",
                "data": "synthetic (seeded AWQ weights/activations, config-1 distributions)",
                "config": {"workload": AWQ_WORKLOAD, "global_batch": sum(AWQ_MS),
                           "parallelism": f"host threads ({nthreads})",
                           "sample": cb["sample"]},
                "cpu_baseline": cb,
                "e2e": {"value": cb["value"], "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0},
                "note": "the reference has no CPU implementation of this path (no Candle in "
                        "Cargo.lock); the CPU restatement in oracle/ stands in for it",
                "reference_gpu": rg}
        print(json.dumps(line), flush=True)
        if dist_on:
            torch.distributed.destroy_process_group()
        return

    if args.decode:
        line = run_decode(args, device, dist_on, world, rank)
        if rank == 0:
            print(json.dumps(line), flush=True)
        if dist_on:
            torch.distributed.barrier()
            torch.distributed.destroy_process_group()
        return

    res = run_awq(args, device, dist_on, world, rank)
    W = res.pop("_weights")
    res.pop("_peaks")
    del W
    torch.cuda.empty_cache()
    # decode tok/s (configs 3 and 4), tensor parallel over all ranks: every rank
    # takes part; the blocks land in rank 0's line
    decode = {}
    if not args.no_decode:
        import argparse as _ap
        dargs = _ap.Namespace(steps=min(args.steps, 20), warmup=args.warmup, ctx=None, batch=None,
                              decode=None)
        for preset in ("8b-awq", "70b-fp8"):
            blk = run_decode(dargs, device, dist_on, world, rank, preset=preset)
            torch.cuda.empty_cache()
            decode[blk["metric"]] = {k: blk[k] for k in ("value", "unit", "ms_per_step", "config",
                                                          "points", "dtype", "scaling")}
            decode[blk["metric"]]["clocks"] = blk["clocks"]
    if rank == 0:
        line = {"metric": res.pop("metric"), "value": res.pop("value"), "unit": res.pop("unit"),
                "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
                "ms_per_step": res.pop("ms_per_step"), "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": res.pop("dtype"),
                "data": "synthetic (seeded AWQ weights/activations, config-1 distributions)"}
        line.update(res)
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_sweep(nthreads, steps=3, warmup=1)
        if world == 1 and not args.no_fp8:
            line["fp8_sweep"] = fp8_sweep(device)
        if decode:
            line["decode"] = decode
        c4 = decode.get("decode_tok_s_config4", {})
        p1 = next((p for p in c4.get("points", []) if p.get("batch") == 1 and "tok_s" in p), None)
        if world == 1 and p1 is not None:
            # the N > 1 lines' headline (tensor-parallel config-4 decode at batch
            # 1) measured here at N = 1, so scaling can be read against it
            line["tp_headline"] = {"metric": "decode_tok_s_config4_batch1", "value": p1["tok_s"],
                                   "unit": "tok/s", "ms_per_step": p1["ms_median"],
                                   "parallelism": "tp1"}
        if world > 1 and p1 is not None:
            # N > 1: the headline is the tensor-parallel config-4 decode at batch 1
            # (strong scaling of one fixed step over the N GPUs); the per-rank
            # config-1 replicas move to `replica_sweep`.  The TP=1 figure is the
            # same point of the N=1 line's decode block.
            keys = ("metric", "value", "unit", "ms_per_step", "scaling", "dtype", "config",
                    "e2e", "roofline", "sweep")
            line["replica_sweep"] = {k: line.pop(k) for k in keys if k in line}
            line.update(
                metric="decode_tok_s_config4_batch1", value=p1["tok_s"], unit="tok/s",
                ms_per_step=p1["ms_median"], scaling="strong",
                dtype="bf16 act, e4m3 W8A8 (fp32 accumulate)",
                data="synthetic (random-init Llama-3-70B-shaped FP8 weights, random KV cache "
                     "and token ids)",
                config={"workload": "config4: Llama-3-70B FP8 decoder, one decode step at batch 1, "
                                    "ctx 4096, tensor parallel", "global_batch": 1,
                        "seq_len": 4096, "parallelism": f"tp{world}",
                        "l2": "weights + KV per step >> L2"},
                e2e={"value": p1["e2e_tok_s"], "unit": "tok/s",
                     "ms_per_step": p1["e2e_ms_per_step"],
                     "h2d_bytes_per_step": p1["h2d_bytes_per_step"],
                     "d2h_bytes_per_step": p1["d2h_bytes_per_step"]},
                allreduce_ms=p1.get("allreduce_ms"), clocks=c4.get("clocks"),
                gpu_launches=args.steps * p1["own_launches_per_step"])
        print(json.dumps(line), flush=True)
    if dist_on:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
