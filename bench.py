"""Benchmark of the B200 W4A8 mid-group linear layer.

Headline (N=1): the reference's decode configuration -- the four QwQ-32B
projections (qkv, o, gate_up, down) at M in {1,4,8,16,32,64}, int4 group-128
symmetric weights with fp32 per-group scales, bf16 activations quantised per
(token, group) inside the op.  One step = those 24 linear calls (quantiser +
GEMM each), shapes interleaved so every weight matrix is evicted from L2
before its next use (244 MB of weights per step > 126 MB L2).  The metric is
algorithmic HBM GB/s: sum over calls of N*K/2 + G*N*4 + M*K*2 + M*N*2 bytes,
divided by the step time.

  value          device time of K CUDA-graph replays of the step (inputs resident)
  e2e            the same step through the public op with host buffers: per step one
                 pinned host->device copy of the 24 inputs, the 24 eager op calls and
                 one device->host copy of the 24 outputs, copies overlapped with
                 neighbouring steps' compute on their own streams
  roofline       the GEMM kernel alone, each launch timed with CUDA events after an
                 L2 flush; achieved = algorithmic bytes / kernel time.  Timed alone
                 and cold, a launch pays the pipeline fill that the chained step
                 overlaps with the previous call, so the per-call sum can exceed the
                 step time
  prefill        the prefill configuration, M = 1024 ... 8192: GEMM int8 TOP/s against
                 cuBLAS int8 (torch._int_mm) measured in the same run; `value` over
                 M >= 2048, the regime of the target
  config3        group size {64, 128, 256} x {sym, asym} on gate_up / down: GB/s at
                 M = 16, TOP/s at M = 4096
  cpu_baseline   the reference's own C++ CPU GEMM (oracle/_ref, compiled from the
                 reference sources) plus the C port of its activation quantiser,
                 on a 1/8-of-N sample of the same sweep, all host threads
  tp_stack       the tensor-parallel configuration: 4 QwQ-32B decoder-layer linear
                 stacks, tensor-parallel over the N GPUs (tp = 1 at N = 1) with NCCL
                 and with the one-shot peer-memory all-reduce; layer tokens/s per M
                 and, at N > 1, the output's distance from the tp = 1 stack

Multi-GPU: one process per GPU (torchrun).  Every rank runs its own replica of
the sweep (weak scaling; the sweep has no exchange step) and the step time is
the max over ranks; the tensor-parallel layer stack, the configuration with an
exchange step, is reported beside it.

``--impl reference`` times the reference's CPU implementation instead.
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

REPO = os.path.dirname(os.path.abspath(__file__))
for _p in (REPO, os.path.join(REPO, "vllm-ascend910_b200")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

GK = 128
SHAPES = ["qkv", "o", "gate_up", "down"]
DECODE_MS = (1, 4, 8, 16, 32, 64)
PREFILL_MS = (1024, 2048, 4096, 8192)
METRIC = "W4A8 GEMM HBM GB/s (decode)"


def alg_bytes(M, N, K, gk=GK, scale_bytes=4, asym=False):
    G = -(-K // gk)
    return N * K // 2 + G * N * scale_bytes + (G * N * 2 if asym else 0) + M * K * 2 + M * N * 2


def sweep_configs(ms=DECODE_MS):
    return [(shape, M) for M in ms for shape in SHAPES]


def peaks():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        d = json.load(open(path))
        return d.get("hbm_gbs", 6650.0), "measured"
    return 6650.0, "fallback"


# ------------------------------------------------------------------ clocks

class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100", "-i", str(self.gpu)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except FileNotFoundError:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        out, _ = self.proc.communicate(timeout=10)
        rows = [r.split(",") for r in out.strip().splitlines() if r.strip()]
        sm = [float(r[1]) for r in rows if len(r) >= 9 and r[1].strip().replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if len(r) >= 9 and r[2].strip().replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = set()
        for r in rows:
            if len(r) < 9:
                continue
            for name, v in zip(names, r[5:9]):
                if v.strip().lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(sm)}


# ------------------------------------------------------------------ CPU baseline

def cpu_sample(n_div=8, ms=DECODE_MS, seed=0):
    """The reference C++ GEMM (+ the C port of its quantiser) on a 1/n_div-of-N
    sample of the sweep.  Returns (GB/s, seconds, threads, kind, description)."""
    import oracle
    from w4a8_b200 import synthetic as syn
    from w4a8_b200.synthetic import QWQ_SHAPES
    use_ref = oracle.ref_available()
    data = []
    for shape, M in sweep_configs(ms):
        K, N = QWQ_SHAPES[shape]
        Ns = N // n_div
        xb = syn.activation_np(M, K, seed + M)
        w = syn.weight_np(Ns, K, GK, seed + 7 + K)
        data.append((M, Ns, K, xb, w, oracle.f32_to_bf16(w.scale)))
    # every host thread, whatever OMP_NUM_THREADS the launcher exported (torchrun sets 1)
    threads = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)
    oracle.set_threads(threads)
    t0 = time.perf_counter()
    tot = 0
    for M, Ns, K, xb, w, wsb in data:
        q, s, _ = oracle.quant_act(xb, GK)
        if use_ref:
            oracle.ref_midgroup_gemm(q, s, w.codes, wsb, None, GK)
        else:
            oracle.gemm_kernel_order(q, oracle.bf16_to_f32(s), w.codes, w.scale, None, GK)
        tot += alg_bytes(M, Ns, K)
    dt = time.perf_counter() - t0
    kind = "reference" if use_ref else "port"
    desc = (f"decode sweep (24 calls) with N/{n_div} weight rows per call (the CPU GEMM's time is linear "
            f"in N, so GB/s over the sampled bytes stands for the whole sweep); "
            + ("ReferenceMidGroupGemm (int4_cube_lab/host/gemm_ref.cpp, -O3 -fopenmp) after the C port of "
               "fakequant_lab's activation quantiser" if use_ref else "C port of the reference CPU path"))
    return tot / dt / 1e9, dt, threads, kind, desc


def run_reference(args, rank, world):
    if rank != 0:
        return
    vals = []
    for _ in range(args.warmup):
        cpu_sample()
    for _ in range(args.steps):
        v, dt, threads, kind, desc = cpu_sample()
        vals.append((v, dt))
    v = statistics.median(x[0] for x in vals)
    line = {"impl": "reference", "metric": METRIC, "value": v, "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": 1e3 * statistics.median(x[1] for x in vals), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "i8", "data": "synthetic",
            "config": {"workload": "decode sweep, QwQ-32B qkv/o/gate_up/down x M in {1,4,8,16,32,64}, "
                                   "GK=128 sym int4, per-step sample of N/8 weight rows"},
            "cpu_baseline": {"value": v, "unit": "GB/s", "cores": threads, "kind": kind, "sample": desc},
            "e2e": {"value": v, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line))


# ------------------------------------------------------------------ GPU arm

def build_weights(torch, dev, seed=0):
    from w4a8_b200 import ops
    from w4a8_b200.synthetic import QWQ_SHAPES, weight_torch
    W = {}
    for i, shape in enumerate(SHAPES):
        K, N = QWQ_SHAPES[shape]
        codes, scale, _ = weight_torch(N, K, GK, seed + i, dev)
        packed = ops.pack_int4_grouped(codes, GK)
        del codes
        scale = scale.contiguous()
        # prepared once at load, like process_weights_after_loading; the raw
        # layout stays resident for the raw-layout comparison line
        W[shape] = (packed, scale, K, N, ops.prepare_weights(packed, scale, None, K, GK))
    return W


def l2_flush(torch, flush):
    """Evict L2 by READING a buffer twice its size (a write would leave dirty
    lines that the next kernel pays to write back)."""
    return flush.view(torch.int64).sum()


def time_kernels_cold(torch, ops, W, cfgs, xs, ys, flush, reps=4, gk=GK):
    """Per call: the GEMM (with its stream-K fix-up) on prepared weights, the L2
    flushed by a read before each launch.  Two CUDA graphs per call -- reps x
    [flush, GEMM] and reps x [flush] -- timed with events on the replay stream;
    the difference is the GEMMs' time without launch gaps."""
    out = []
    for (shape, M) in cfgs:
        packed, scale, K, N, pw = W[shape]
        ops.linear_quant(xs[(shape, M)], N, gk)
        y = ys[(shape, M)]
        ops.linear_gemm_prepared(M, pw, y)            # workspace exists before capture
        torch.cuda.synchronize()
        times = []
        for with_gemm in (True, False):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                for _ in range(reps):
                    l2_flush(torch, flush)
                    if with_gemm:
                        ops.linear_gemm_prepared(M, pw, y)
            g.replay()
            torch.cuda.synchronize()
            best = 1e9
            for _ in range(3):
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                g.replay()
                e1.record()
                e1.synchronize()
                best = min(best, e0.elapsed_time(e1) * 1e-3)
            times.append(best)
            del g
        out.append((shape, M, K, N, max(times[0] - times[1], 1e-9) / reps))
    return out


def e2e_run(torch, ops, W, cfgs, xs, ys, steps, dev, world, step_bytes):
    """The decode sweep end to end through the public op with host buffers.

    Per step: one host->device copy of the step's 24 inputs from a pinned host
    slab, the 24 ``ops.linear_prepared`` calls (eager, as a user makes them),
    and one device->host copy of the 24 outputs into a pinned host slab.  Steps
    are pipelined the way a serving loop overlaps transfers with compute: the
    copies run on their own streams with two device slabs, so step s+1's
    inputs travel while step s computes and step s's outputs travel back while
    step s+1 computes.  The time runs from the first input copy's start to the
    last output copy's end (events on the copy streams)."""
    import torch.distributed as dist
    bf16 = torch.bfloat16
    xsz = [xs[c].numel() for c in cfgs]
    ysz = [ys[c].numel() for c in cfgs]
    xo = [0]
    for n in xsz:
        xo.append(xo[-1] + (n + 7) // 8 * 8)             # 16-byte aligned slices
    yo = [0]
    for n in ysz:
        yo.append(yo[-1] + (n + 7) // 8 * 8)
    xh = torch.empty(xo[-1], dtype=bf16).pin_memory()
    for i, c in enumerate(cfgs):
        xh[xo[i]:xo[i] + xsz[i]].copy_(xs[c].reshape(-1).cpu())
    yh = [torch.empty(yo[-1], dtype=bf16).pin_memory() for _ in range(2)]
    xd = [torch.empty(xo[-1], dtype=bf16, device=dev) for _ in range(2)]
    yd = [torch.empty(yo[-1], dtype=bf16, device=dev) for _ in range(2)]
    xv = [[xd[b][xo[i]:xo[i] + xsz[i]].view(xs[c].shape) for i, c in enumerate(cfgs)] for b in range(2)]
    yv = [[yd[b][yo[i]:yo[i] + ysz[i]].view(ys[c].shape) for i, c in enumerate(cfgs)] for b in range(2)]
    comp = torch.cuda.current_stream(dev)
    h2d, d2h = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    ev = {k: [torch.cuda.Event() for _ in range(2)] for k in ("h2d", "comp", "d2h")}
    pws = [W[c[0]][4] for c in cfgs]

    def step(s):
        b = s & 1
        with torch.cuda.stream(h2d):
            if s >= 2:
                h2d.wait_event(ev["comp"][b])          # step s-2 is done reading this slab
            xd[b].copy_(xh, non_blocking=True)
            ev["h2d"][b].record(h2d)
        comp.wait_event(ev["h2d"][b])
        if s >= 2:
            comp.wait_event(ev["d2h"][b])              # step s-2's outputs have left this slab
        for x, pw, y in zip(xv[b], pws, yv[b]):
            ops.linear_prepared(x, pw, out=y)
        ev["comp"][b].record(comp)
        with torch.cuda.stream(d2h):
            d2h.wait_event(ev["comp"][b])
            yh[b].copy_(yd[b], non_blocking=True)
            ev["d2h"][b].record(d2h)

    for s in range(4):
        step(s)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record(h2d)
    for s in range(steps):
        step(s)
    t1.record(d2h)
    torch.cuda.synchronize()
    t = t0.elapsed_time(t1) * 1e-3 / steps
    if world > 1:
        tt = torch.tensor([t], device=dev, dtype=torch.float64)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        t = float(tt.item())
    last = yh[(steps - 1) & 1]
    same = all(torch.equal(last[yo[i]:yo[i] + ysz[i]], ys[c].reshape(-1).cpu()) for i, c in enumerate(cfgs))
    return {"value": world * step_bytes / t / 1e9, "unit": "GB/s", "h2d_bytes_per_step": xo[-1] * 2,
            "d2h_bytes_per_step": yo[-1] * 2, "ms_per_step": 1e3 * t, "steps": steps,
            "matches_graph_outputs": bool(same),
            "how": "per step one pinned H2D copy of the 24 inputs, 24 eager ops.linear_prepared calls, one "
                   "D2H copy of the 24 outputs; copies on their own streams, double-buffered, so transfers "
                   "of neighbouring steps overlap compute"}


def time_config3(torch, ops, syn, dev, flush, hbm_peak, i8_peak):
    """gate_up / down x GK {64, 128, 256} x {sym int4, asym
    uint4 + zero point}: GEMM GB/s at M = 16 and int8 TOP/s at M = 4096 (the
    cold-L2 graph-difference timing of the roofline line)."""
    from w4a8_b200.synthetic import QWQ_SHAPES
    rows = []
    for shape in ("gate_up", "down"):
        K, N = QWQ_SHAPES[shape]
        for gk in (64, 128, 256):
            for asym in (False, True):
                codes, scale, zero = syn.weight_torch(N, K, gk, 300 + gk, dev, asym=asym)
                packed = ops.pack_int4_grouped(codes, gk)
                del codes
                pw = ops.prepare_weights(packed, scale, zero, K, gk)
                Wc = {shape: (packed, scale, K, N, pw)}
                for M in (16, 4096):
                    x = syn.activation_torch(M, K, 310 + M, dev)
                    y = torch.empty(M, N, dtype=torch.bfloat16, device=dev)
                    (_, _, _, _, t), = time_kernels_cold(torch, ops, Wc, [(shape, M)], {(shape, M): x},
                                                         {(shape, M): y}, flush, reps=2, gk=gk)
                    by = alg_bytes(M, N, K, gk, 4, asym)
                    r = {"shape": shape, "gk": gk, "weights": "asym" if asym else "sym", "M": M,
                         "us": round(t * 1e6, 2)}
                    if M == 16:
                        r.update(GBps=round(by / t / 1e9, 1), frac_hbm=round(by / t / 1e9 / hbm_peak, 3))
                    else:
                        tops = 2 * M * N * K / t / 1e12
                        r.update(TOPS=round(tops, 1), frac_int8=round(tops / i8_peak, 3) if i8_peak else None)
                    rows.append(r)
                del Wc, pw, packed
    return rows


def int8_peak_tops(torch, dev):
    a = torch.randint(-128, 127, (8192, 8192), dtype=torch.int8, device=dev)
    b = torch.randint(-128, 127, (8192, 8192), dtype=torch.int8, device=dev).t()
    try:
        for _ in range(3):
            torch._int_mm(a, b)
        torch.cuda.synchronize()
        best = 1e9
        for _ in range(5):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            torch._int_mm(a, b)
            e1.record()
            e1.synchronize()
            best = min(best, e0.elapsed_time(e1) * 1e-3)
        return 2 * 8192 ** 3 / best / 1e12
    except Exception:
        return None


def run_gpu(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist

    from w4a8_b200 import ops
    from w4a8_b200 import synthetic as syn

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    hbm_peak, peak_src = peaks()
    sampler = ClockSampler(local_rank)
    W = build_weights(torch, dev, seed=rank)
    cfgs = sweep_configs()
    xs = {(s, M): syn.activation_torch(M, W[s][2], 100 + M, dev) for (s, M) in cfgs}
    ys = {(s, M): torch.empty(M, W[s][3], dtype=torch.bfloat16, device=dev) for (s, M) in cfgs}
    step_bytes = sum(alg_bytes(M, W[s][3], W[s][2]) for (s, M) in cfgs)

    def step():
        for (s, M) in cfgs:
            ops.linear_prepared(xs[(s, M)], W[s][4], out=ys[(s, M)])

    def step_raw():
        for (s, M) in cfgs:
            packed, scale, K, N, _ = W[s]
            ops.linear(xs[(s, M)], packed, scale, None, GK, out=ys[(s, M)])

    def timed_graph(fn, steps, warmup):
        fn()                                   # allocates the workspace
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            fn()
        for _ in range(max(3, warmup)):
            g.replay()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            g.replay()
        e1.record()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        t = e0.elapsed_time(e1) * 1e-3 / steps
        if world > 1:
            tt = torch.tensor([t], device=dev, dtype=torch.float64)
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
            t = float(tt.item())
        del g
        return t

    sampler.start()
    t_step = timed_graph(step, args.steps, args.warmup)
    value = world * step_bytes / t_step / 1e9
    t_raw = timed_graph(step_raw, max(3, min(args.steps, 50)), 3)
    raw_value = world * step_bytes / t_raw / 1e9
    # the same sweep with the quantiser fused into the GEMM for the calls with
    # M <= 16 (W4A8_OPT_FUSED_QUANT; off by default because it measures slower)
    from w4a8_b200 import _lib
    old_opt = _lib.lib().w4a8_set_options(_lib.OPT_FUSED_QUANT)
    try:
        t_fq = timed_graph(step, max(3, min(args.steps, 50)), 3)
    finally:
        _lib.lib().w4a8_set_options(old_opt)
    fq_value = world * step_bytes / t_fq / 1e9
    status = ops.workspace_status(dev)

    # ---- end to end through the public op, host buffers ----
    e2e = e2e_run(torch, ops, W, cfgs, xs, ys, max(3, min(args.steps, 20)), dev, world, step_bytes)

    # ---- dominant kernel alone (GEMM), cold L2, events per launch ----
    flush = torch.ones(512 << 20, dtype=torch.uint8, device=dev)
    kt = time_kernels_cold(torch, ops, W, cfgs, xs, ys, flush)
    k_bytes = sum(alg_bytes(M, N, K) for (_, M, K, N, _) in kt)
    k_time = sum(t for *_, t in kt)
    achieved = k_bytes / k_time / 1e9
    per_shape = [{"shape": s, "M": M, "us": round(t * 1e6, 2),
                  "GBps": round(alg_bytes(M, N, K) / t / 1e9, 1),
                  "frac": round(alg_bytes(M, N, K) / t / 1e9 / hbm_peak, 3)} for (s, M, K, N, t) in kt]
    traffic = None
    tfile = os.path.join(REPO, "profiles", "gemm_decode_traffic.json")
    if os.path.exists(tfile):
        tj = json.load(open(tfile))
        traffic = tj.get("bytes_per_launch")

    # ---- prefill subset: GEMM int8 TOP/s ----
    pre = []
    big = {}
    for M in PREFILL_MS:
        for s in SHAPES:
            K, N = W[s][2], W[s][3]
            x = syn.activation_torch(M, K, 200 + M, dev)
            y = torch.empty(M, N, dtype=torch.bfloat16, device=dev)
            big[(s, M)] = (x, y)
    pk = time_kernels_cold(torch, ops, W, list(big.keys()), {k: v[0] for k, v in big.items()},
                           {k: v[1] for k, v in big.items()}, flush, reps=2)
    for (s, M, K, N, t) in pk:
        pre.append({"shape": s, "M": M, "us": round(t * 1e6, 1), "TOPS": round(2 * M * N * K / t / 1e12, 1)})
    del big
    i8_peak = int8_peak_tops(torch, dev)
    pk2 = [r for r in pk if r[1] >= 2048]
    pre_tops = sum(2 * M * N * K for (_, M, K, N, _) in pk2) / sum(t for *_, t in pk2) / 1e12
    cfg3 = None if args.no_config3 else time_config3(torch, ops, syn, dev, flush, hbm_peak, i8_peak)
    status = status or ops.workspace_status(dev)
    clocks = sampler.stop()

    # ---- tensor-parallel layer stack (config 4), tp = N ----
    tp = None
    if not args.no_tp_stack:
        from w4a8_b200 import tp as tpmod
        tp = tpmod.bench_stack(world, rank, dev, ms=(16, 256, 4096), layers=4, iters=max(3, min(args.steps, 20)),
                               hbm_gbs=hbm_peak, i8_tops=i8_peak, allreduces=("nccl", "custom", "fused", "fused_push"))

    if rank != 0:
        return
    cpu = None
    if world == 1 and not args.no_cpu_baseline:
        v, dt, threads, kind, desc = cpu_sample()
        cpu = {"value": v, "unit": "GB/s", "cores": threads, "kind": kind, "sample": desc,
               "seconds": round(dt, 2)}
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    launches = args.steps * sum(kernels_per_call(M, W[s][3], W[s][2], sms) for (s, M) in cfgs)
    line = {
        "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": 1e3 * t_step, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "i8", "data": "synthetic",
        "config": {"workload": "decode sweep (BASELINE config 1): QwQ-32B qkv/o/gate_up/down x M in "
                               "{1,4,8,16,32,64}, int4 sym GK=128, fp32 lognormal scales, bf16 N(0,1) "
                               "activations with 0.5% x20 outlier channels, quantised per (token, group) in-op",
                   "calls_per_step": len(cfgs), "alg_bytes_per_step": step_bytes,
                   "l2": "inputs larger than L2: 244 MB of weights per step, shapes interleaved",
                   "timing": "CUDA graph of the step, events on the replay stream, max over ranks",
                   "parallelism": f"replicas x{world}" if world > 1 else "single GPU",
                   "reference_arm": "the reference's C++ CPU GEMM on all host cores of the box (whatever N), "
                                    "on an N/8 sample of each call's weight rows; its time is linear in N"},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm_peak, "unit": "GB/s",
                     "frac": achieved / hbm_peak, "traffic": traffic,
                     "kernel": "w4a8_gemm_kernel + its stream-K fix-up, prepared weights, L2 flushed by a "
                               "512 MB read before each launch; graph [flush, GEMM] minus graph [flush]; "
                               "timed alone and cold, so each launch pays the pipeline fill the chained "
                               "step overlaps with the previous call",
                     "traffic_source": "profiles/gemm_decode_traffic.json (ncu, the same 24 calls, per launch)",
                     "peak_source": f"{peak_src} (MEASURED_PEAKS.json hbm_gbs)" if peak_src == "measured" else peak_src},
        "e2e": e2e,
        "raw_layout": {"value": raw_value, "unit": "GB/s", "ms_per_step": 1e3 * t_raw,
                       "note": "same sweep on the reference row-major weight layout (2-D tensor copies)"},
        "fused_quant": {"value": fq_value, "unit": "GB/s", "ms_per_step": 1e3 * t_fq,
                        "note": "same sweep with the 16 calls of M <= 16 quantising their activation inside the "
                                "GEMM (W4A8_OPT_FUSED_QUANT) instead of in the standalone quantiser kernel that "
                                "the headline uses"},
        "gpu_launches": launches,
        "clocks": clocks,
        "prefill": {"metric": "W4A8 GEMM int8 TOP/s (prefill)", "value": pre_tops, "unit": "TOP/s",
                    "int8_peak_measured_cublas": i8_peak,
                    "frac_of_measured_int8": (pre_tops / i8_peak) if i8_peak else None,
                    "frac_of_nominal_4500": pre_tops / 4500.0, "per_shape": pre},
        "per_shape": per_shape,
        "cpu_baseline": cpu,
        "status_word": status,
    }
    if tp is not None:
        line["tp_stack"] = tp
    if cfg3 is not None:
        line["config3"] = cfg3
    print(json.dumps(line))


def kernels_per_call(M, N, K, sms, gk=GK):
    """Kernels one linear call launches: the quantiser, the GEMM and, when the
    GEMM's stream-K split leaves a tile divided between CTAs, the fix-up kernel
    (the host plan in csrc/w4a8_capi.cu)."""
    tt = 16 if M <= 16 else (32 if M <= 32 else (64 if M <= 64 else 128))
    G = -(-K // gk)
    last = K - (G - 1) * gk
    kpad = (G - 1) * (-(-gk // 64) * 64) + -(-last // 64) * 64
    kb_total = -(-kpad // 256)
    upt = -(-kb_total // (2 if tt <= 16 else 1)) if gk <= 256 else G
    units = -(-N // 128) * -(-M // tt) * upt
    grid = max(1, min(sms, units))
    split = any((c * units // grid) % upt for c in range(1, grid))
    return 2 + (1 if split else 0)


def profile_sweep():
    """The decode sweep's 24 calls once each after a warm-up pass, L2 flushed
    (by reading) before each: the target of the traffic capture (profiles/)."""
    import torch
    from w4a8_b200 import ops
    from w4a8_b200 import synthetic as syn
    dev = torch.device("cuda", 0)
    W = build_weights(torch, dev)
    cfgs = sweep_configs()
    xs = {(s, M): syn.activation_torch(M, W[s][2], 100 + M, dev) for (s, M) in cfgs}
    ys = {(s, M): torch.empty(M, W[s][3], dtype=torch.bfloat16, device=dev) for (s, M) in cfgs}
    flush = torch.ones(512 << 20, dtype=torch.uint8, device=dev)
    for _ in range(2):
        for (s, M) in cfgs:
            l2_flush(torch, flush)
            ops.linear_prepared(xs[(s, M)], W[s][4], out=ys[(s, M)])
    torch.cuda.synchronize()
    assert ops.workspace_status(dev) == 0
    print("profile sweep: " + " ".join(f"{s}:{M}" for (s, M) in cfgs))


def profile_case(spec: str):
    """One shape, a few launches: the target of the ncu captures (profiles/)."""
    import torch
    from w4a8_b200 import ops
    from w4a8_b200 import synthetic as syn
    from w4a8_b200.synthetic import QWQ_SHAPES
    shape, M = spec.split(":")
    M = int(M)
    K, N = QWQ_SHAPES[shape]
    dev = torch.device("cuda", 0)
    codes, scale, _ = syn.weight_torch(N, K, GK, 1, dev)
    packed = ops.pack_int4_grouped(codes, GK)
    pw = ops.prepare_weights(packed, scale, None, K, GK)
    x = syn.activation_torch(M, K, 2, dev)
    y = torch.empty(M, N, dtype=torch.bfloat16, device=dev)
    for _ in range(8):
        ops.linear_prepared(x, pw, out=y)
    torch.cuda.synchronize()
    assert ops.workspace_status(dev) == 0
    print(f"profile case {shape} M={M} K={K} N={N}: ok")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--no-tp-stack", action="store_true", help="skip the tensor-parallel layer stack")
    ap.add_argument("--no-config3", action="store_true", help="skip the group-size / asymmetry lines")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--profile-case", default=None, help="SHAPE:M, e.g. qkv:16 (ncu target)")
    ap.add_argument("--profile-sweep", action="store_true", help="each decode call once, cold (ncu target)")
    args = ap.parse_args()
    if args.profile_case:
        profile_case(args.profile_case)
        return
    if args.profile_sweep:
        profile_sweep()
        return
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local_rank)
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local_rank))
    try:
        run_gpu(args, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
