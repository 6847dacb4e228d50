#!/usr/bin/env python3
"""Benchmark of the B200 fixed-point simulator kernels (
the op-level sweep) — one JSON line on rank 0.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

A step is one pass of the MatMul sweep: M in {1, 8, 128, 2048} x K in {64, 512,
1024, 4096} x N in {32, 256, 1024, 4096} x batch in {1, 16} (A and B both
batched), int16 Q8.8 inputs uniform in [-1, 1), every product bit-exact
(sat16(floor(sum / 2^8))).  ``value`` = sum of the sweep's int16 MACs / device
time (GMAC/s, whole job over all ranks; each rank runs its own instance of the
sweep: weak scaling).  The VectorOP (Add / Mul / Div with broadcast, fused SiLU /
GELU-erf / GELU-tanh, 4M elements) and Softmax (rows 128 / 1024 / 4096, row and
column mode) sweeps of the same config are measured after it and reported under
``sweeps``.

Timing: inputs resident in HBM, the sweep replayed as one CUDA graph, CUDA
events on the launching stream, L2 flushed (256 MB write) between steps, max
over ranks.  ``e2e`` repeats the sweep through the public per-op API with
pinned host buffers (H2D of A and B, D2H of C inside the timed region).
``roofline``: the tcgen05 GEMM kernel's int8 tensor ops (8 per int16 MAC: four
int8 products, 2 ops each) over its event-timed duration, against int8 dense
peak measured live with cuBLASLt (torch._int_mm).  ``cpu_baseline``: the CPU
oracle (numpy float64 BLAS + floor / saturate, the reference simulator's own
method, _simulate.py:631) on the batch-1 half of the sweep, all host threads.
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

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

MS = (1, 8, 128, 2048)
KS = (64, 512, 1024, 4096)
NS = (32, 256, 1024, 4096)
BATCHES = (1, 16)


# the timed sweep runs the jobs of at most SMALL_MACS MACs concurrently on LANES streams
SMALL_MACS = 1 << 31
LANES = 4


def sweep_problems(batches=BATCHES):
    return [(b, m, k, n) for b in batches for m in MS for k in KS for n in NS]


def macs_of(problems):
    return sum(b * m * k * n for b, m, k, n in problems)


# ---------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms while running."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int):
        self.dev = device_index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.dev}", f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, mx, reasons = [], None, set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for nm, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# ---------------------------------------------------------------- CPU side (oracle)
def cpu_sweep_data(problems, seed=0):
    """The sweep's operands on the host (int16 Q8.8 in [-1, 1))."""
    rng = np.random.default_rng(seed)
    return [(rng.integers(-256, 256, size=(b, m, k), dtype=np.int16),
             rng.integers(-256, 256, size=(b, k, n), dtype=np.int16)) for b, m, k, n in problems]


def cpu_matmul_rate(problems, min_seconds=10.0, seed=0, data=None):
    """GMAC/s of the CPU oracle (numpy float64 matmul + floor + saturate) over
    ``problems`` repeated until ``min_seconds`` elapsed."""
    from oracle import spec
    if data is None:
        data = cpu_sweep_data(problems, seed)
    macs, t0 = 0, time.perf_counter()
    while True:
        for (A, B), (b, m, k, n) in zip(data, problems):
            spec.matmul_raw(A, B)
            macs += b * m * k * n
        el = time.perf_counter() - t0
        if el >= min_seconds:
            return macs / el / 1e9, el, macs


def run_reference(args):
    """--impl reference: the reference's CPU algorithm (the oracle port; the
    reference is Python and does not travel to the GPU box) on rank 0."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    cores = os.cpu_count() or 1
    os.environ.setdefault("OMP_NUM_THREADS", str(cores))
    os.environ.setdefault("OPENBLAS_NUM_THREADS", str(cores))
    sample = sweep_problems()  # the whole sweep, as the GPU arm times it
    data = cpu_sweep_data(sample)
    half = sweep_problems(batches=(1,))
    for _ in range(args.warmup):  # warm-up (untimed): the batch-1 half, threads and caches started
        cpu_matmul_rate(half, min_seconds=0.0, data=data[:len(half)])
    rates, secs = [], []
    for _ in range(args.steps):
        r, el, _ = cpu_matmul_rate(sample, min_seconds=0.0, data=data)
        rates.append(r)
        secs.append(el)
    value = macs_of(sample) * args.steps / sum(secs) / 1e9
    line = {"metric": "bit-exact fixed-point sim GMAC/s (op-level MatMul sweep)", "value": round(value, 3),
            "unit": "GMAC/s", "impl": "reference", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(1e3 * sum(secs) / args.steps, 3), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "int16 (exact int64 sums)", "data": "synthetic, seeded",
            "config": {"workload": "configs[1] op-level MatMul sweep: M{1,8,128,2048} x K{64,512,1024,4096} x "
                                   "N{32,256,1024,4096} x batch{1,16}", "problems": len(sample),
                       "gmac_per_step_per_gpu": round(macs_of(sample) / 1e9, 3)},
            "cpu_baseline": {"value": round(value, 3), "unit": "GMAC/s", "cores": cores, "kind": "port",
                             "sample": "the whole MatMul sweep (128 problems, %.1f GMAC) per step"
                                       % (macs_of(sample) / 1e9)},
            "e2e": {"value": round(value, 3), "unit": "GMAC/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------- GPU side
def measure_int8_peak(torch, device):
    """Dense int8 tensor throughput (TOPS) of cuBLASLt via torch._int_mm, burst."""
    try:
        a = torch.randint(-128, 127, (8192, 8192), dtype=torch.int8, device=device)
        b = torch.randint(-128, 127, (8192, 8192), dtype=torch.int8, device=device)
        for _ in range(3):
            torch._int_mm(a, b)
        torch.cuda.synchronize()
        best = 1e9
        for _ in range(10):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            torch._int_mm(a, b)
            e1.record()
            e1.synchronize()
            best = min(best, e0.elapsed_time(e1))
        return 2 * 8192 ** 3 / (best * 1e-3) / 1e12, "measured live: torch._int_mm int8 8192^3 (cuBLASLt), best of 10"
    except Exception as e:  # pragma: no cover
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            pk = json.load(f)
        return 2 * pk["bf16_tflops"], f"2 x measured bf16 ({e.__class__.__name__} from torch._int_mm)"


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-models", action="store_true", help="skip the MNIST / MobileNetV2 / BERT forward passes")
    ap.add_argument("--models", help="comma list of model cases to run (default: all)")
    ap.add_argument("--detail", help="write per-problem kernel times of one profiled step to this JSON file")
    ap.add_argument("--case", choices=["gemm", "gemm_small", "gemm_int16", "vectorop", "softmax", "softmax128",
                                       "softmax_col",
                                       "layernorm", "rmsnorm32", "dwconv", "dwconv14", "pwconv", "maxpool",
                                       "addxnorm", "mulact", "conv",
                                       "llama_prefill", "llama_decode"],
                    help="run one job a few times (a small case for ncu captures) and exit")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.impl == "reference":
        return run_reference(args)
    if args.case:
        return run_case(args)

    import torch

    from cormorant_b200 import ops
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    pg = None
    if world > 1:
        import datetime

        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
        pg = dist

    stream = torch.cuda.Stream(device=dev)
    gen = torch.Generator(device=dev)
    gen.manual_seed(1234 + rank)
    problems = sweep_problems()
    bufs = []
    with torch.cuda.stream(stream):
        for b, m, k, n in problems:
            A = torch.randint(-256, 256, (b * m * k,), dtype=torch.int16, device=dev, generator=gen)
            B = torch.randint(-256, 256, (b * k * n,), dtype=torch.int16, device=dev, generator=gen)
            Cc = torch.empty(b * m * n, dtype=torch.int16, device=dev)
            bufs.append((A, B, Cc))
        ws_bytes = 0
        import ctypes as Ct

        from cormorant_b200 import _lib
        for (b, m, k, n) in problems:
            d = _lib.MatmulDesc(0, 0, 0, m, k, n, b, m * k, k * n, m * n, 0, 0, 0, None, 0)
            need = Ct.c_size_t(0)
            _lib.check(_lib.lib().corm_matmul_workspace_size(Ct.byref(d), Ct.byref(need)))
            ws_bytes = max(ws_bytes, need.value)
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
        flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
        # the problems are independent jobs: the small ones (at most SMALL_MACS
        # MACs — a few output tiles, latency-bound) run first, spread over
        # LANES streams so that they share the SMs, then the rest in order on
        # the step's stream, each lane with a workspace of its own
        small = sorted((i for i, (b, m, k, n) in enumerate(problems) if b * m * k * n <= SMALL_MACS),
                       key=lambda i: -macs_of([problems[i]]))
        large = [i for i in range(len(problems)) if i not in set(small)]
        lane_of = {i: j % LANES for j, i in enumerate(small)}
        lane_ws = []
        for ln in range(LANES):
            need_l = 0
            for i in small:
                if lane_of[i] == ln:
                    b, m, k, n = problems[i]
                    d = _lib.MatmulDesc(0, 0, 0, m, k, n, b, m * k, k * n, m * n, 0, 0, 0, None, 0)
                    need = Ct.c_size_t(0)
                    _lib.check(_lib.lib().corm_matmul_workspace_size(Ct.byref(d), Ct.byref(need)))
                    need_l = max(need_l, need.value)
            lane_ws.append(torch.empty(max(need_l, 256), dtype=torch.uint8, device=dev))
    lanes = [torch.cuda.Stream(device=dev) for _ in range(LANES)]

    def one(i, w):
        (b, m, k, n), (A, B, Cc) = problems[i], bufs[i]
        ops.matmul(A, B, Cc, n=m, k=k, m=n, batch=b, a_batch_stride=m * k, b_batch_stride=k * n,
                   c_batch_stride=m * n, workspace=w)

    def run_sweep():  # one stream, problems in order (the profiled step)
        for i in range(len(problems)):
            one(i, ws)

    def run_sweep_lanes():  # the timed step (captured as one CUDA graph: fork, small jobs, join, large jobs)
        cur = torch.cuda.current_stream()
        for s_ in lanes:
            s_.wait_stream(cur)
        for i in small:
            with torch.cuda.stream(lanes[lane_of[i]]):
                one(i, lane_ws[lane_of[i]])
        for s_ in lanes:
            cur.wait_stream(s_)
        for i in large:
            one(i, ws)

    # eager warm-up (tensor maps, kernel attributes), count launches per step
    with torch.cuda.stream(stream):
        l0 = ops.launch_count()
        run_sweep_lanes()
        launches_per_step = ops.launch_count() - l0
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        run_sweep_lanes()
    torch.cuda.synchronize()

    def timed_steps(nsteps, fn):
        times = []
        for _ in range(nsteps):
            with torch.cuda.stream(stream):
                flush.zero_()
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(stream)
                fn()
                e1.record(stream)
            e1.synchronize()
            times.append(e0.elapsed_time(e1))
        return times

    timed_steps(args.warmup, graph.replay)
    if pg:
        pg.barrier()
    torch.cuda.synchronize()
    clocks = ClockSampler(local)
    clocks.start()
    time.sleep(0.5)
    times = timed_steps(args.steps, graph.replay)
    torch.cuda.synchronize()
    clk = clocks.stop()
    total_ms = sum(times)
    if pg:
        t = torch.tensor([total_ms], dtype=torch.float64, device=dev)
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
        total_ms = float(t.item())
    ms_per_step = total_ms / args.steps
    macs_step = macs_of(problems)
    value = world * macs_step * args.steps / (total_ms * 1e-3) / 1e9

    # per-kernel times of one eager step (events around every launch), queued
    # behind a gate so that the GPU runs them back to back, as in the graph,
    # and no event interval holds host submission time
    gated = profiled_step(torch, ops, stream, flush, run_sweep)
    prof = ops.profile_read()
    if args.detail and rank == 0:
        per = []
        with torch.cuda.stream(stream):
            ops.profile_enable(True)
            for (b, m, k, n), (A, B, Cc) in zip(problems, bufs):
                ops.matmul(A, B, Cc, n=m, k=k, m=n, batch=b, a_batch_stride=m * k, b_batch_stride=k * n,
                           c_batch_stride=m * n, workspace=ws)
                torch.cuda.synchronize()
                pr = ops.profile_read()
                per.append({"b": b, "m": m, "k": k, "n": n, "gmac": b * m * k * n / 1e9,
                            "kernels": {kk: round(v[1], 4) for kk, v in pr.items()}})
            ops.profile_enable(False)
        with open(args.detail, "w") as fh:
            json.dump(per, fh, indent=1)
    tensor_probs = [(b, m, k, n) for b, m, k, n in problems if m > 2]
    tensor_macs = sum(b * m * k * n for b, m, k, n in tensor_probs)
    # DRAM traffic of the GEMM kernel per launch: algorithmic bytes (A and B read
    # once — as int8 planes or as int16, the same bytes — and C written once)
    # times the DRAM / algorithmic ratio ncu measured for the launch's form: the
    # split-plane form 0.946 (4 x 2048 x 4096 x 4096: 201.43 MB read + 52.52 MB
    # written of 268.4 MB), the int16-operand form 1.11 (16 x 2048 x 4096 x 256:
    # 324.4 + 13.6 MB of 304 MB; A's second read per column-tile pair partly misses L2).
    def int16_form(m, k, n):  # the library's rule (csrc/matmul.cu tensor_path)
        return k % 8 == 0 and n % 8 == 0 and (m + n) * 500 > m * n
    ratio = {False: (201.43e6 + 52.52e6) / 268.4e6, True: (324.4e6 + 13.6e6) / 304e6}
    alg_bytes = sum(b * (2 * m * k + 2 * k * n + 2 * m * n) for b, m, k, n in tensor_probs)
    dram_bytes = sum(b * (2 * m * k + 2 * k * n + 2 * m * n) * ratio[int16_form(m, k, n)]
                     for b, m, k, n in tensor_probs)
    n_int16 = sum(1 for b, m, k, n in tensor_probs if int16_form(m, k, n))
    g_launches, g_ms, _ = prof.get("gemm_i8x4_kernel", (0, 0.0, 0.0))
    live_peak, live_src = measure_int8_peak(torch, dev)
    with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as fh:
        bf16 = float(json.load(fh)["bf16_tflops"])
    peak = 2 * bf16  # dense int8 = 2 x dense bf16 on B200; the pool's measured bf16 burst
    achieved = 8 * tensor_macs / (g_ms * 1e-3) / 1e12 if g_ms else None
    step_kernel_ms = sum(v[1] for v in prof.values())

    # VectorOP and Softmax sweeps of the same config
    sweeps = vector_sweeps(torch, ops, dev, stream, flush, args, rank, world)
    models = None if args.no_models else bench_models(torch, dev, stream, flush, args, world, rank, pg)

    # verification of the timed sweep's own outputs (after the timed region):
    # every rank's sampled grids gathered to rank 0 over NCCL and checked there
    parity = sweep_parity(torch, problems, bufs, dev, rank, world, pg)

    e2e = None
    if not args.no_e2e:
        e2e = run_e2e(torch, ops, dev, stream, problems, bufs, ws, args, pg, world)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        r, el, macs = cpu_matmul_rate(problems, min_seconds=5.0)
        cpu = {"value": round(r, 3), "unit": "GMAC/s", "cores": os.cpu_count(), "kind": "port",
               "sample": "the whole MatMul sweep (128 problems), repeated to %.1f s" % el}

    if rank == 0:
        line = {
            "metric": "bit-exact fixed-point sim GMAC/s (op-level MatMul sweep)",
            "value": round(value, 1), "unit": "GMAC/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_per_step, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "int16 (int8 x4 tensor split, int64 recombine)",
            "data": "synthetic int16 Q8.8 uniform [-1,1), seeded per rank",
            "config": {"workload": "configs[1] op-level MatMul sweep: M{1,8,128,2048} x K{64,512,1024,4096} x "
                                   "N{32,256,1024,4096} x batch{1,16}", "problems": len(problems),
                       "gmac_per_step_per_gpu": round(macs_step / 1e9, 3), "parallelism": f"dp{world} (replicas)",
                       "l2": "256 MB flush between steps; 7.6 GB of distinct operands per step",
                       "launch": "CUDA graph replay of the sweep: the %d jobs of at most 2^31 MACs first, spread "
                                 "over %d streams, then the other %d in order" % (len(small), LANES, len(large))},
            "gpu_launches": int(launches_per_step * args.steps),
            "roofline": {"bound": "tensor", "kernel": "gemm_i8x4_kernel", "achieved": round(achieved, 1) if achieved else None,
                         "peak": round(peak, 1), "unit": "TFLOP/s", "frac": round(achieved / peak, 4) if achieved else None,
                         "traffic": round(dram_bytes / max(g_launches, 1)),
                         "alg_bytes_per_launch": round(alg_bytes / max(g_launches, 1)),
                         "traffic_note": "DRAM bytes per GEMM launch, sweep average: each launch's algorithmic bytes x "
                                         "the DRAM/algorithmic ratio ncu measured for its form (split planes 0.946, "
                                         "int16 operands 1.11; %d of %d launches in the int16 form)"
                                         % (n_int16, len(tensor_probs)),
                         "peak_source": "of measured: 2 x MEASURED_PEAKS bf16_tflops burst (%.1f; B200 dense int8 = "
                                        "2 x dense bf16)" % bf16,
                         "live_int8_probe": {"peak": round(live_peak, 1), "frac": round(achieved / live_peak, 4)
                                             if achieved else None, "source": live_src},
                         "work": "8 int8 tensor ops per int16 MAC (4 int8 products); tensor-path problems (M > 2)",
                         "gemm_launches_per_step": g_launches, "gemm_ms_per_step": round(g_ms, 4),
                         "all_kernels_ms_per_step": round(step_kernel_ms, 4),
                         "timing": "CUDA events around every launch of one eager step queued behind a sleep kernel "
                                   "(launches back to back on the GPU, no host time inside an interval: %s)"
                                   % ("held" if gated else "gate ran out"),
                         "kernels": {k: {"launches": v[0], "ms": round(v[1], 4)} for k, v in sorted(prof.items())}},
            "clocks": clk,
            "parity": parity,
            "sweeps": sweeps,
        }
        if models:
            line["models"] = models
        if cpu:
            line["cpu_baseline"] = cpu
        if e2e:
            line["e2e"] = e2e
        print(json.dumps(line), flush=True)
    if pg:
        pg.barrier()
        pg.destroy_process_group()
    return 0


def profiled_step(torch, ops, stream, flush, fn, gate_ms=40.0):
    """One eager pass of ``fn`` with the library's per-launch events on,
    queued behind a bounded sleep kernel (``gate_ms`` of clock cycles) so that
    every launch is on the stream before the GPU reaches it: the events then
    time the kernels alone, back to back.  Returns whether the gate held (the
    GPU was still in the sleep when the host had queued the whole pass); if
    not, the pass is repeated once with a longer gate."""
    for _ in range(2):
        with torch.cuda.stream(stream):
            flush.zero_()
            ops.profile_read()
            torch.cuda._sleep(int(gate_ms * 1e-3 * 2.1e9))
            gate_end = torch.cuda.Event()
            gate_end.record(stream)
            ops.profile_enable(True)
            fn()
            ops.profile_enable(False)
            held = not gate_end.query()
        torch.cuda.synchronize()
        if held:
            return True
        gate_ms *= 4
    return False


def _gather_to_root(torch, pg, world, rank, t):
    """All ranks' equally sized 1-D tensors on rank 0 (all-gather: the
    verification step, after the timed regions); [t] when running alone."""
    if not pg:
        return [t]
    out = torch.empty(world * t.numel(), dtype=t.dtype, device=t.device)
    pg.all_gather_into_tensor(out, t)
    return list(out.split(t.numel())) if rank == 0 else []


def sweep_parity(torch, problems, bufs, dev, rank, world, pg):
    """Every problem of the timed sweep checked exactly at a seeded grid of
    >= 4096 outputs (its rows of A, columns of B and outputs, gathered on the
    device; oracle.sampled), on every rank: each rank's grids go to rank 0,
    which recomputes them with the CPU oracle.  Verification only: it runs
    after the timed region on the outputs the last timed step wrote."""
    from oracle import sampled
    parts, shapes = [], []
    for i, ((b, m, k, n), (A, B, Cc)) in enumerate(zip(problems, bufs)):
        idx = sampled.plan(b, m, k, n, seed=i, full_macs=None)
        subs = sampled.gather_t(A, B, Cc, b, m, k, n, idx)
        parts += [t.reshape(-1) for t in subs]
        shapes.append(tuple(tuple(t.shape) for t in subs))
    got = _gather_to_root(torch, pg, world, rank, torch.cat(parts).to(torch.int32))  # no int16 collectives
    if rank != 0:
        return None
    checked = bad = 0
    for fl in got:
        v = fl.cpu().numpy()
        off = 0
        for shs in shapes:
            seg = []
            for sh in shs:
                cnt = int(np.prod(sh))
                seg.append(v[off:off + cnt].reshape(sh))
                off += cnt
            c_n, c_bad = sampled.check(*seg)
            checked += c_n
            bad += c_bad
    return {"checked": checked, "mismatches": bad, "ranks": len(got), "problems": len(problems),
            "method": "per problem and rank, >= 4096 outputs (or all) at a seeded grid, recomputed exactly from "
                      "their rows of A and columns of B by the CPU oracle; grids gathered to rank 0"}


def _time_job(torch, stream, flush, fn, args):
    """Median device time (ms) of one job captured as a CUDA graph, the L2
    flushed before every replay (inputs come from HBM)."""
    with torch.cuda.stream(stream):
        fn()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        fn()
    return _time_graph(torch, stream, flush, g, args)


def cpu_vectorop_rate(jobs, size, outer, min_seconds=2.0):
    """Elements/s of the reference's VectorOP method on the host (the op on
    the raw operands, then its activation in float64 with the C library's
    exp / erf / tanh and host_quantize: _simulate.py:721-765,
    vectorop_act.py:60-79, as the oracle restates them), over ``jobs``."""
    from oracle import spec
    rng = np.random.default_rng(7)
    a = rng.integers(-256, 256, size=(outer, size)).astype(np.int64)
    b = rng.integers(-256, 256, size=(1, size)).astype(np.int64)
    b = np.where(b == 0, 1, b)
    n, t0 = 0, time.perf_counter()
    while True:
        for op, act in jobs:
            if op == 0:
                r = a + b
            elif op == 2:
                r = (a * b) >> 8
            else:
                num = a * 256
                q = np.abs(num) // np.abs(b)
                r = np.where((num < 0) ^ (b < 0), -q, q)
            r = spec.sat16(r)
            spec.host_quantize_raw(spec.act_real(act, r / 256.0))
            n += a.size
        el = time.perf_counter() - t0
        if el >= min_seconds:
            return n / el, el


def cpu_softmax_rate(cases, min_seconds=1.0):
    """Elements/s of the reference's softmax unit model on the host
    (vectorop_smx.softmax_raw / softmax_cols, as oracle.spec restates them),
    over (n, mode) cases of 2^20 elements each."""
    from oracle import spec
    rng = np.random.default_rng(8)
    cm, cs = spec.smx_scale_regs(8, 1.0)
    data = {n: rng.integers(-2048, 2048, size=((1 << 20) // n, n)).astype(np.int64) for n, _ in cases}
    cnt, t0 = 0, time.perf_counter()
    while True:
        for n, mode in cases:
            x = data[n] if mode == "row" else np.ascontiguousarray(data[n].T).T  # keys-major storage
            spec.softmax_rows(x, n, cm, cs, 8)
            cnt += x.size
        el = time.perf_counter() - t0
        if el >= min_seconds:
            return cnt / el, el


def cpu_pool_rate(min_seconds=1.0):
    """Input elements/s of the reference's pooling model on the host (the
    oracle's restatement of _pool2d_ref, _simulate.py:230-358) on the two
    pools of the sweep, a sample of each."""
    from oracle import spec
    rng = np.random.default_rng(9)
    xm = rng.integers(-256, 256, size=(64, 16, 28, 28)).astype(np.int64)
    xg = rng.integers(-256, 256, size=(8, 1280, 7, 7)).astype(np.int64)
    cnt, t0 = 0, time.perf_counter()
    while True:
        spec.pool_raw(xm, 2, 2, 2, 2, 0, 0, 1, 1, 14, 14, 0, 0, 0)
        spec.pool_raw(xg, 7, 7, 1, 1, 0, 0, 1, 1, 1, 1, 1, 0, 0)
        cnt += xm.size + xg.size
        el = time.perf_counter() - t0
        if el >= min_seconds:
            return cnt / el, el


def vector_sweeps(torch, ops, dev, stream, flush, args, rank=0, world=1):
    """configs[1] (b) VectorOP Add / Mul / Div with a broadcast operand
    (outer x size, stride 0) and fused SiLU / GELU-erf / GELU-tanh, and (c)
    the softmax unit on rows of 128 / 1024 / 4096 in row and keys-major
    modes; plus the pooling unit on the configs' pools.  Every job is timed
    alone (a CUDA graph of the one job, the L2 flushed before each replay,
    median of the steps); GB/s over the algorithmic bytes (operands read
    once, outputs written once, a stride-0 operand counted once).  The
    config's 4M-element VectorOP jobs last a few microseconds, so the same
    jobs on 64M elements (inputs far above L2) give the HBM roofline; the
    softmax and pool jobs run on inputs above 100 MB.  The CPU rate of the
    reference's method on a bounded sample is reported beside each."""
    with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as fh:
        hbm = float(json.load(fh).get("hbm_gbs") or 6650.0)
    gen = torch.Generator(device=dev)
    gen.manual_seed(99)
    jobs = [(op, act) for op in (0, 2, 3) for act in (4, 5, 6)]
    out = {"hbm_peak_gbs": hbm}
    for tag, N in (("vectorop", 1 << 22), ("vectorop_64M", 1 << 26)):
        size, outer = 1024, N // 1024
        with torch.cuda.stream(stream):
            a = torch.randint(-256, 256, (N,), dtype=torch.int16, device=dev, generator=gen)
            b = torch.randint(-256, 256, (size,), dtype=torch.int16, device=dev, generator=gen)
            b = torch.where(b == 0, torch.ones_like(b), b)
            c = torch.empty(N, dtype=torch.int16, device=dev)
        per = {}
        for op, act in jobs:
            nm = f"{('add', '', 'mul', 'div')[op]}_{('', '', '', '', 'silu', 'gelu', 'gelu_tanh')[act]}"
            per[nm] = _time_job(torch, stream, flush, lambda op=op, act=act: ops.vectorop(
                a, b, c, size=size, op=op, outer=outer, a_inc=size, b_inc=0, act=act), args)
        t = sum(per.values())
        vbytes = len(jobs) * (4 * N + 2 * size)
        gbs = vbytes / (t * 1e-3) / 1e9
        out[tag] = {"jobs": f"ADD/MUL/DIV x SiLU/GELU/GELU-tanh, {N >> 20}M elem, b broadcast "
                            f"(outer {outer} x size {size}, b_inc 0)",
                    "ms": round(t, 4), "GB/s": round(gbs, 1), "frac_of_measured_hbm": round(gbs / hbm, 3),
                    "bytes_per_elem": 4, "G_elem/s": round(len(jobs) * N / (t * 1e-3) / 1e9, 2),
                    "ms_per_job": {k: round(v, 4) for k, v in per.items()}}
        del a, b, c
    cm, cs = 12102203, 19
    smx = {}
    N = 1 << 26
    with torch.cuda.stream(stream):
        x = torch.randint(-2048, 2048, (N,), dtype=torch.int16, device=dev, generator=gen)
        p = torch.empty(N, dtype=torch.int16, device=dev)
    for n in (128, 1024, 4096):
        rows = N // n
        for mode in ("row", "col"):
            if mode == "row":
                fn = lambda n=n, rows=rows: ops.vectorop(x, None, p, size=n, op=10, outer=rows, a_inc=n, b_inc=n,  # noqa
                                                         smx_cm=cm, smx_cfg=cs | (8 << 8), smx_mask=n)
            else:  # keys-major: n keys x rows queries
                fn = lambda n=n, rows=rows: ops.vectorop(x, None, p, size=n, op=11, outer=rows, a_inc=rows,  # noqa
                                                         b_inc=n, smx_cm=cm, smx_cfg=cs | (8 << 8), smx_mask=n)
            t2 = _time_job(torch, stream, flush, fn, args)
            gbs = 4 * N / (t2 * 1e-3) / 1e9
            smx[f"{mode}{n}"] = {"ms": round(t2, 4), "GB/s": round(gbs, 1), "frac_of_measured_hbm": round(gbs / hbm, 3)}
    out["softmax"] = {"elements_per_job": N, "bytes_per_elem": 4, "jobs": smx}
    del x, p
    pools = {}
    for tag, (B, C, H, W, ph, st, oh, pt) in (("maxpool2x2_s2_16x28x28_b4096", (4096, 16, 28, 28, 2, 2, 14, 0)),
                                               ("gap_1280x7x7_b256", (256, 1280, 7, 7, 7, 1, 1, 1))):
        with torch.cuda.stream(stream):
            xin = torch.randint(-256, 256, (B * C * H * W,), dtype=torch.int16, device=dev, generator=gen)
            y = torch.empty(B * C * oh * oh + 8, dtype=torch.int16, device=dev)
        fn = lambda xin=xin, y=y, B=B, C=C, H=H, W=W, ph=ph, st=st, oh=oh, pt=pt: ops.pool(  # noqa
            xin, y, batch=B, channels=C, in_h=H, in_w=W, out_h=oh, out_w=oh, pool_h=ph, pool_w=ph, stride_h=st,
            stride_w=st, pool_type=pt)
        tp = _time_job(torch, stream, flush, fn, args)
        pb = 2 * B * C * (H * W + oh * oh)
        gbs = pb / (tp * 1e-3) / 1e9
        pools[tag] = {"ms": round(tp, 4), "GB/s": round(gbs, 1), "frac_of_measured_hbm": round(gbs / hbm, 3),
                      "bytes": pb}
        del xin, y
    out["pool"] = pools
    if rank == 0 and world == 1 and not args.no_cpu:
        r, el = cpu_vectorop_rate(jobs, 1024, 512)
        out["vectorop"]["cpu_baseline"] = {"value": round(r * 4 / 1e9, 4), "unit": "GB/s", "G_elem/s": round(r / 1e9, 5),
                                           "cores": 1, "kind": "port",
                                           "sample": "the 9 jobs on 512 x 1024 elements, repeated to %.1f s" % el}
        r, el = cpu_softmax_rate([(n, md) for n in (128, 1024, 4096) for md in ("row", "col")])
        out["softmax"]["cpu_baseline"] = {"value": round(r * 4 / 1e9, 4), "unit": "GB/s", "G_elem/s": round(r / 1e9, 5),
                                          "cores": 1, "kind": "port",
                                          "sample": "the 6 cases on 2^20 elements each, repeated to %.1f s" % el}
        r, el = cpu_pool_rate()
        out["pool"]["cpu_baseline"] = {"value": round(r * 2 / 1e9, 4), "unit": "GB/s (input bytes)",
                                       "G_elem/s": round(r / 1e9, 5), "cores": 1, "kind": "port",
                                       "sample": "64 x 16 x 28 x 28 MaxPool and 8 x 1280 x 7 x 7 GAP, repeated to "
                                                 "%.1f s" % el}
    return out


LLAMA_GOLDEN = os.path.join(ROOT, "tests", "golden", "llama_full_s{}.npz")


def _crc16(a) -> int:
    import zlib
    return zlib.crc32(np.ascontiguousarray(np.asarray(a, np.int64).astype("<i2")).tobytes())


def _verify_units(torch, pg, world, rank, unit_out, check):
    """Each rank's first unit (its raw outputs on the device, as int32)
    gathered to rank 0, where ``check(r, raw)`` compares it with the CPU
    oracle's output for that rank's unit (True / False, or None when not
    checked)."""
    got = _gather_to_root(torch, pg, world, rank, unit_out.to(torch.int32).reshape(-1).contiguous())
    if rank != 0:
        return None
    res = [check(r, g.cpu().numpy().astype(np.int64)) for r, g in enumerate(got)]
    done = [x for x in res if x is not None]
    return {"units_checked": len(done), "mismatching_units": sum(1 for x in done if not x),
            "ranks_checked": [r for r, x in enumerate(res) if x is not None]}


def bench_models(torch, dev, stream, flush, args, world, rank, pg):
    """configs[0] (MNIST CNN), configs[2] (MobileNetV2-1.0, 224x224, batch 256
    sharded over the ranks) and configs[3] (BERT-base encoder, 64 sequences of
    384 tokens sharded over the ranks), and configs[4]'s prefill: GpuSimulator
    forward passes on raw int16 inputs, replayed as CUDA graphs; images/s or
    tokens/s over all ranks, int16 GMAC/s.  Rank r runs units [r B, (r + 1) B)
    of the configuration's seeded input set.  After timing, every rank's first
    unit is gathered to rank 0 and compared with the CPU oracle's output for
    that unit (the Llama prefill with the oracle's committed golden); on rank
    0 at N = 1 the oracle's forward pass of one unit is timed too."""
    from cormorant_b200 import workloads as WL
    from cormorant_b200.simulator import GpuSimulator
    from oracle import graph as og
    out = {}
    cases = [("mnist_b1", "images", lambda b, f: WL.mnist(seed=1, batch=b, first=f), 1),
             ("mnist_b4096", "images", lambda b, f: WL.mnist(seed=1, batch=b, first=f), 4096),
             ("mobilenet_v2_224", "images", lambda b, f: WL.mobilenet_v2(seed=3, batch=b, res=224, first=f),
              max(1, 256 // world)),
             ("bert_base_384", "tokens", lambda b, f: WL.bert_base(seed=4, batch=b, seq=384, first=f),
              max(1, 64 // world)),
             ("llama360m_prefill512", "tokens", lambda b, f: WL.llama_prefill(seed=5, batch=b, seq=512, first=f),
              max(1, 64 // world))]
    seq_of = {"bert_base_384": 384, "llama360m_prefill512": 512}
    if not args.models or "llama360m_decode128" in args.models.split(","):
        out["llama360m_decode128"] = bench_llama_decode(torch, dev, stream, flush, args, world, rank, pg)
    for name, unit, build, batch in cases:
        if args.models and name not in args.models.split(","):
            continue
        g, feeds, macs_unit = build(batch, rank * batch)
        units = batch * seq_of.get(name, 1)
        sim = GpuSimulator(g, device=dev)
        keep = [t.onnx_name for t in g.output_tensors]
        with torch.cuda.stream(stream):
            raw = {t.onnx_name: (np.asarray(feeds[t.onnx_name]).astype(np.int64).reshape(-1) if t.host
                                 else sim._to_raw(t, feeds[t.onnx_name])) for t in g.input_tensors}
            dev_states = sim.states_to_device() if g.state_tensors else None
            sim.forward_raw(raw, keep=keep, states=dev_states)  # weights uploaded, workspaces sized
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            res, _ = sim.forward_raw(raw, keep=keep, states=dev_states)
        ms = _time_graph(torch, stream, flush, graph, args)
        if pg:
            t = torch.tensor([ms], dtype=torch.float64, device=dev)
            pg.all_reduce(t, op=pg.ReduceOp.MAX)
            ms = float(t.item())
        rate = world * units / (ms * 1e-3)
        out[name] = {"batch_per_gpu": batch, "ms_per_batch": round(ms, 4), f"{unit}_per_s": round(rate, 1),
                     "GMAC/s": round(rate * macs_unit / 1e9, 1), f"mmac_per_{unit[:-1]}": round(macs_unit / 1e6, 2),
                     "nodes": len(g.nodes), "units_per_rank": f"[rank * {batch}, (rank + 1) * {batch})"}
        if args.detail:  # per-kernel device time of one eager pass (events around each launch, gated)
            from cormorant_b200 import ops
            profiled_step(torch, ops, stream, flush, lambda: sim.forward_raw(raw, keep=keep, states=dev_states))
            prof = ops.profile_read()
            out[name]["kernels"] = {k: {"launches": v[0], "ms": round(v[1], 4)}
                                    for k, v in sorted(prof.items(), key=lambda kv: -kv[1][1])}
        # verification: each rank's first unit against the CPU oracle on rank 0
        ot = g.output_tensors[0]
        per_unit = ot.numel // batch
        unit_out = res[ot.onnx_name][:per_unit]
        cpu_s = {}

        def check(r, got, name=name, build=build, batch=batch):
            first = r * batch
            if name.startswith("llama"):
                path = LLAMA_GOLDEN.format(first)
                if not os.path.exists(path):
                    return None
                return _crc16(got) == int(np.load(path)["crc_prefill_logits"][0])
            if name == "bert_base_384" and r not in (0, world - 1):
                return None  # seconds of CPU per sequence: the first and the last rank's units
            if name == "mnist_b4096" and r:
                return None
            g1, f1, _ = build(1, first)
            t0 = time.perf_counter()
            ref = og.forward(g1, {k: np.asarray(v) for k, v in f1.items()})
            cpu_s.setdefault(r, time.perf_counter() - t0)
            return bool(np.array_equal(got, ref[g1.output_tensors[0].onnx_name].reshape(-1)))
        out[name]["parity"] = _verify_units(torch, pg, world, rank, unit_out, check)
        if rank == 0 and world == 1 and not args.no_cpu and 0 in cpu_s and name != "mnist_b4096":
            out[name][f"cpu_oracle_{unit}_per_s"] = round(seq_of.get(name, 1) / cpu_s[0], 3)
        del graph, res, sim, raw, dev_states
        torch.cuda.empty_cache()
        if rank == 0 and world == 1 and not args.no_cpu and name.startswith("llama"):
            # the CPU oracle on one layer of one 64-token sequence, scaled to the
            # full depth (extrapolated: the per-token work of a layer at 64 keys)
            from oracle import llm
            g1, f1, _ = WL.llama_prefill(seed=5, batch=1, seq=64, layers=1, vocab=1000)
            tm = {t.onnx_name: t for t in g1.input_tensors}
            r1 = {k: (np.asarray(v) if tm[k].host else np.rint(np.asarray(v) * 2.0 ** float(tm[k].exp)).astype(np.int64))
                  for k, v in f1.items()}
            t0 = time.perf_counter()
            llm.forward(g1, r1, {t.onnx_name: np.zeros(t.shape, np.int64) for t in g1.state_tensors})
            el = (time.perf_counter() - t0) * 32
            out[name]["cpu_oracle_tokens_per_s"] = round(64 / el, 4)
            out[name]["cpu_oracle_sample"] = "1 layer x 64 tokens, x32 layers (extrapolated)"
    return out


def bench_llama_decode(torch, dev, stream, flush, args, world, rank, pg, steps=128):
    """configs[4]'s decode: after the 512-token prefill of 64 / N sequences
    (rank r: sequences [r B, (r + 1) B)), ``steps`` greedy decode steps (pos
    512 .. 639): per step the device greedy step (argmax + embedding row) and
    one decode-step pass (the host softmax on the device), each captured as
    its own CUDA graph (the key count and the cache row are registers of the
    step); a timed step replays all of them.  Tokens/s over all ranks.  After
    timing, each rank's first sequence (its greedy ids and last logits) is
    gathered to rank 0 and compared with the CPU oracle's golden for that
    sequence."""
    from cormorant_b200 import workloads as WL
    from cormorant_b200.llm_runner import LlamaRunner
    B = max(1, 64 // world)
    m = WL.LlamaModel(seed=5, batch=B, seq=512, first=rank * B)
    r = LlamaRunner(m, device=dev)
    ids = torch.empty((steps, B), dtype=torch.int32, device=dev)
    with torch.cuda.stream(stream):
        lg0 = r.prefill()
        r.decode_step(lg0, steps - 1)  # the largest key count: workspaces and tables sized before capture
    torch.cuda.synchronize()
    pool = torch.cuda.graph_pool_handle()
    graphs, lg = [], lg0
    for i in range(steps):
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr, stream=stream, pool=pool):
            lg = r.decode_step(lg, i, ids[i])
        graphs.append(gr)

    class _Seq:
        def replay(self):
            for gr in graphs:
                gr.replay()
    ms = _time_graph(torch, stream, flush, _Seq(), args)
    if pg:
        t = torch.tensor([ms], dtype=torch.float64, device=dev)
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
        ms = float(t.item())
    keys_avg = float(np.mean([-(-(512 + i + 1) // 16) * 16 for i in range(steps)]))
    macs = m.macs_per_token(keys_avg, prefill=False)
    rate = world * B * steps / (ms * 1e-3)
    # HBM roofline of a step: every weight read once (int16, or its two int8
    # planes: 2 B either way) and the K / V cache rows the attention reads (the
    # key count of each step, 2 B per element), per rank
    D, H, KVh, HD = m.D, m.H, m.KV, m.HD
    w_elems = m.L * (D * (H * HD + 2 * KVh * HD) + H * HD * D + 3 * D * m.ffn) + D * m.vocab
    kv_bytes = float(np.mean([2 * 2 * m.L * B * KVh * HD * (512 + i + 1) for i in range(steps)]))
    step_bytes = 2.0 * w_elems + kv_bytes
    with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as fh:
        hbm = float(json.load(fh).get("hbm_gbs") or 6650.0)
    gbs = world * step_bytes / (ms / steps * 1e-3) / 1e9
    out = {"batch_per_gpu": B, "steps": steps, "ms_per_decode_run": round(ms, 3),
           "ms_per_token_step": round(ms / steps, 4), "tokens_per_s": round(rate, 1),
           "GMAC/s": round(rate * macs / 1e9, 1), "mmac_per_token": round(macs / 1e6, 2),
           "graph_nodes_per_step": len(m.decode_graph.nodes),
           "roofline": {"bound": "hbm", "alg_bytes_per_step_per_gpu": round(step_bytes),
                        "GB/s": round(gbs, 1), "frac_of_measured_hbm": round(gbs / (world * hbm), 4),
                        "bytes": "weights once (2 B each) + the K / V cache rows read (keys 513 .. 640)"},
           "first_ids": ids[0, :4].cpu().tolist()}
    # verification: every replay runs the same steps over the caches the prefill
    # left (a step's cache row is written before it is read), so the ids and the
    # last logits are those of a prefill and 128 greedy steps
    torch.cuda.synchronize()
    mine = torch.cat([ids[:, 0].to(torch.int64), lg[:m.vocab].to(torch.int64)])

    def check(rr, got):
        path = LLAMA_GOLDEN.format(rr * B)
        if not os.path.exists(path):
            return None
        z = np.load(path)
        return bool(np.array_equal(got[:steps], z["ids"][:steps]) and
                    _crc16(got[steps:]) == int(z["crc_step_logits"][steps - 1]))
    out["parity"] = _verify_units(torch, pg, world, rank, mine, check)
    if args.detail:  # per-kernel device time of one eager decode step (events around each launch, gated)
        from cormorant_b200 import ops
        profiled_step(torch, ops, stream, flush, lambda: r.decode_step(lg0, 0))
        prof = ops.profile_read()
        out["kernels"] = {k: {"launches": v[0], "ms": round(v[1], 4)}
                          for k, v in sorted(prof.items(), key=lambda kv: -kv[1][1])}
    del graphs, r
    torch.cuda.empty_cache()
    return out


def _time_graph(torch, stream, flush, g, args):
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    ts = []
    for _ in range(max(3, args.steps)):
        with torch.cuda.stream(stream):
            flush.zero_()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            g.replay()
            e1.record(stream)
        e1.synchronize()
        ts.append(e0.elapsed_time(e1))
    return statistics.median(ts)


def run_e2e(torch, ops, dev, stream, problems, bufs, ws, args, pg, world):
    """The sweep through the public per-op API with host buffers: H2D of A
    and B from pinned memory, the job, D2H of C, every step — pipelined over
    four streams (A and B in on two, jobs, copies out; events per job between
    them), so that job i's result travels back while job i + 1's operands arrive."""
    host = []
    for A, B, Cc in bufs:
        host.append((A.cpu().pin_memory(), B.cpu().pin_memory(), torch.empty(Cc.numel(), dtype=torch.int16).pin_memory()))
    h2d = sum((a.numel() + b.numel()) * 2 for a, b, _ in host)
    d2h = sum(c.numel() * 2 for _, _, c in host)
    nsteps = max(1, min(args.steps, 3))
    s_in, s_in2, s_out = (torch.cuda.Stream(device=dev) for _ in range(3))

    def step():
        s_in.wait_stream(stream)
        s_in2.wait_stream(stream)
        s_out.wait_stream(stream)
        for (b, m, k, n), (A, B, Cc), (hA, hB, hC) in zip(problems, bufs, host):
            with torch.cuda.stream(s_in):  # A and B on two copy streams at once
                A.copy_(hA, non_blocking=True)
                landed = torch.cuda.Event()
                landed.record(s_in)
            with torch.cuda.stream(s_in2):
                B.copy_(hB, non_blocking=True)
                landed2 = torch.cuda.Event()
                landed2.record(s_in2)
            stream.wait_event(landed)
            stream.wait_event(landed2)
            with torch.cuda.stream(stream):
                ops.matmul(A, B, Cc, n=m, k=k, m=n, batch=b, a_batch_stride=m * k, b_batch_stride=k * n,
                           c_batch_stride=m * n, workspace=ws)
                done = torch.cuda.Event()
                done.record(stream)
            s_out.wait_event(done)
            with torch.cuda.stream(s_out):
                hC.copy_(Cc, non_blocking=True)
        stream.wait_stream(s_in)
        stream.wait_stream(s_in2)
        stream.wait_stream(s_out)
    step()
    torch.cuda.synchronize()
    ts = []
    for _ in range(nsteps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        step()
        e1.record(stream)
        e1.synchronize()
        ts.append(e0.elapsed_time(e1))
    total = sum(ts)
    if pg:
        t = torch.tensor([total], dtype=torch.float64, device=dev)
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
        total = float(t.item())
    return {"value": round(world * macs_of(problems) * nsteps / (total * 1e-3) / 1e9, 1), "unit": "GMAC/s",
            "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "steps": nsteps,
            "ms_per_step": round(total / nsteps, 3),
            "path": "cormorant_b200.ops.matmul (C ABI) per problem; H2D (A, B), jobs and D2H on four streams, pipelined"}


def run_case(args):
    """One job, warmup + steps launches, for profiler captures of a single
    kernel on a small case (inputs above L2, a few hundred MB on the device)."""
    import torch

    from cormorant_b200 import ops
    torch.cuda.set_device(0)
    g = torch.Generator(device="cuda")
    g.manual_seed(5)
    ri = lambda n, lo=-256, hi=256: torch.randint(lo, hi, (n,), dtype=torch.int16, device="cuda", generator=g)  # noqa
    if args.case in ("gemm", "gemm_small", "gemm_int16"):
        # the split-plane form, the int16 form with 8 rows, the int16 form with A
        # in TMEM on a compute-heavy job (the sweep's 16 x 2048 x 4096 x 256)
        b, m, k, n = {"gemm": (4, 2048, 4096, 4096), "gemm_small": (16, 8, 4096, 4096),
                      "gemm_int16": (16, 2048, 4096, 256)}[args.case]
        A, B, C = ri(b * m * k), ri(b * k * n), torch.empty(b * m * n, dtype=torch.int16, device="cuda")
        fn = lambda: ops.matmul(A, B, C, n=m, k=k, m=n, batch=b, a_batch_stride=m * k, b_batch_stride=k * n,  # noqa
                                c_batch_stride=m * n)
    elif args.case == "vectorop":
        N = 1 << 26
        a, bb, c = ri(N), ri(1024), torch.empty(N, dtype=torch.int16, device="cuda")
        fn = lambda: ops.vectorop(a, bb, c, size=1024, op=2, outer=N // 1024, a_inc=1024, b_inc=0, act=5)  # noqa
    elif args.case == "softmax":
        N = 1 << 26
        x, p = ri(N, -2048, 2048), torch.empty(N, dtype=torch.int16, device="cuda")
        fn = lambda: ops.vectorop(x, None, p, size=1024, op=10, outer=N // 1024, a_inc=1024, b_inc=1024,  # noqa
                                  smx_cm=12102203, smx_cfg=19 | (8 << 8), smx_mask=1024)
    elif args.case == "softmax128":  # rows of 128 (the short-row form: 16 lanes a row)
        N = 1 << 26
        x, p = ri(N, -2048, 2048), torch.empty(N, dtype=torch.int16, device="cuda")
        fn = lambda: ops.vectorop(x, None, p, size=128, op=10, outer=N // 128, a_inc=128, b_inc=128,  # noqa
                                  smx_cm=12102203, smx_cfg=19 | (8 << 8), smx_mask=128)
    elif args.case == "softmax_col":  # keys-major, 512 keys x 64K queries (a prefill head group's scores)
        N = 1 << 25
        x, p = ri(N, -2048, 2048), torch.empty(N, dtype=torch.int16, device="cuda")
        fn = lambda: ops.vectorop(x, None, p, size=512, op=11, outer=N // 512, a_inc=N // 512, b_inc=512,  # noqa
                                  smx_cm=12102203, smx_cfg=19 | (8 << 8), smx_mask=512)
    elif args.case in ("layernorm", "rmsnorm32"):
        # BERT's LayerNorm (24576 rows x 768 int16) / Llama's RMSNorm of the
        # int32 residual (32768 rows x 960), the parameter blocks as the graphs build them
        import numpy as np

        from cormorant_b200 import rowops_host as RH
        if args.case == "layernorm":
            R_, n = 24576, 768
            words, g_, bb, E = RH.layernorm_job(np.ones(n), np.zeros(n), n, 1e-12)
            x = ri(R_ * n)
            op = RH.opword(RH.OP_NORM, ln=True)
            regs = dict(eps=int(E), bq_sh=RH.P1_BITS + g_ - bb, a_s1=2 * n)
        else:
            R_, n = 32768, 960
            words, bc, g_, E = RH.rmsnorm_job(np.ones(n), 1e-5, 15, np.full(n, 12))
            x = torch.randint(-(1 << 24), 1 << 24, (R_ * n,), dtype=torch.int32, device="cuda", generator=g)
            op = RH.opword(RH.OP_NORM, RH.K_I32, RH.K_I16, RH.K_I16, p_bcast=bool(bc))
            regs = dict(eps=int(E), bq_sh=0, a_s1=4 * n)
        pw = torch.from_numpy(np.asarray(words, np.int16)).cuda()
        y = torch.empty(R_ * n + 8, dtype=torch.int16, device="cuda")
        fn = lambda: ops.rowops(x, None, y, pw, op=op, n=n, rows=R_, blocks=1, c_s1=2 * n, win_lo=0,  # noqa
                                win_hi=RH.NO_WINDOW, **regs)
    elif args.case in ("dwconv", "dwconv14", "pwconv"):
        # MobileNetV2 at batch 64: the 3x3 stride-2 depthwise over 96 x 112 x
        # 112 (second block), the 3x3 depthwise over 576 x 14 x 14 (fifth
        # block), and the 1 x 1 expand 24 -> 144 over 56 x 56
        if args.case == "dwconv":
            N_, C_, H_, M_, k, s_, oh = 64, 96, 112, 96, 3, 2, 56
        elif args.case == "dwconv14":
            N_, C_, H_, M_, k, s_, oh = 64, 576, 14, 576, 3, 1, 14
        else:
            N_, C_, H_, M_, k, s_, oh = 64, 24, 56, 144, 1, 1, 56
        x = ri(N_ * C_ * H_ * H_)
        w = ri(M_ * (1 if args.case != "pwconv" else C_) * k * k, -64, 64)
        b = ri(M_, -64, 64)
        y = torch.empty(N_ * M_ * oh * oh, dtype=torch.int16, device="cuda")
        fn = lambda: ops.conv(x, w, b, y, batch=N_, in_ch=C_, in_h=H_, in_w=H_, out_ch=M_, out_h=oh, out_w=oh,  # noqa
                              kh=k, kw=k, stride_h=s_, stride_w=s_, pad_top=k // 2, pad_left=k // 2, has_bias=1,
                              is_depthwise=int(args.case != "pwconv"), flags=2 | 8)
    elif args.case == "maxpool":  # MNIST's first pool at batch 8192
        x = ri(8192 * 16 * 28 * 28)
        y = torch.empty(8192 * 16 * 14 * 14 + 8, dtype=torch.int16, device="cuda")
        fn = lambda: ops.pool(x, y, batch=8192, channels=16, in_h=28, in_w=28, out_h=14, out_w=14, pool_h=2,  # noqa
                              pool_w=2, stride_h=2, stride_w=2)
    elif args.case == "addxnorm":
        # a Llama layer's residual add + RMSNorm as one chain (the fused row
        # pass), prefill-sized: 32768 rows of 960, the residual int32 at 2^-15
        import numpy as np

        from cormorant_b200 import rowops_host as RH
        R_, n = 32768, 960
        wx, bx = RH.resadd_job(15, np.full(n, 13), n)
        wn, bn, g_, E = RH.rmsnorm_job(np.ones(n), 1e-5, 15, np.full(n, 12))
        h = torch.randint(-(1 << 24), 1 << 24, (R_ * n,), dtype=torch.int32, device="cuda", generator=g)
        d = ri(R_ * n)
        h2 = torch.empty(R_ * n, dtype=torch.int32, device="cuda")
        y = torch.empty(R_ * n + 8, dtype=torch.int16, device="cuda")
        px = torch.from_numpy(np.asarray(wx, np.int16)).cuda()
        pn = torch.from_numpy(np.asarray(wn, np.int16)).cuda()
        jobs = [dict(a=h, b=d, c=h2, p=px, n=n, rows=R_, op=RH.opword(RH.OP_ADDX, RH.K_I32, RH.K_I16, RH.K_I32,
                                                                       b_en=True, p_bcast=bool(bx)),
                     a_s1=4 * n, b_s1=2 * n, c_s1=4 * n, win_hi=RH.NO_WINDOW),
                dict(a=h2, c=y, p=pn, n=n, rows=R_, op=RH.opword(RH.OP_NORM, RH.K_I32, RH.K_I16, RH.K_I16,
                                                                 p_bcast=bool(bn)),
                     a_s1=4 * n, c_s1=2 * n, eps=int(E), win_hi=RH.NO_WINDOW)]
        fn = lambda: ops.rowops_chain(jobs)  # noqa
    elif args.case == "mulact":
        # a Llama prefill layer's gate / up pair with SiLU(g) u in its epilogue:
        # 32768 rows x 960 @ [960 x 2 x 2560], the output 32768 x 2560
        R_, k, ffn = 32768, 960, 2560
        A = ri(R_ * k)
        W = ri(k * 2 * ffn, -64, 64)
        y = torch.empty(R_ * ffn, dtype=torch.int16, device="cuda")
        fn = lambda: ops.matmul_groups(A, W, [y], [ffn], n=R_, k=k, flags=1, mulact=(1, 23))  # noqa
    elif args.case in ("llama_prefill", "llama_decode"):
        # two layers of the config-5 model (every kernel of a layer, a layer's
        # shapes): the prefill of 16 sequences x 512 tokens, or the prefill of
        # 64 and after it one decode step of the 64 (the decode bench's batch;
        # lean passes, as the bench runs them)
        from cormorant_b200 import workloads as WL
        from cormorant_b200.llm_runner import LlamaRunner
        m = WL.LlamaModel(seed=5, batch=64 if args.case == "llama_decode" else 16, seq=512, layers=2)
        r = LlamaRunner(m)
        lg = r.prefill()
        fn = (lambda: r.prefill()) if args.case == "llama_prefill" else (lambda: r.decode_step(lg, 0))  # noqa
    else:
        x = ri(64 * 144 * 56 * 56)
        w = ri(24 * 144, -64, 64)
        y = torch.empty(64 * 24 * 56 * 56, dtype=torch.int16, device="cuda")
        fn = lambda: ops.conv(x, w, None, y, batch=64, in_ch=144, in_h=56, in_w=56, out_ch=24, out_h=56,  # noqa
                              out_w=56, kh=1, kw=1, flags=2)
    for _ in range(args.warmup + args.steps):
        fn()
    torch.cuda.synchronize()
    assert ops.device_status() == 0
    print(f"case {args.case}: {args.warmup + args.steps} launches done")
    return 0


if __name__ == "__main__":
    sys.exit(main())
