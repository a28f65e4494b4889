"""Benchmark: fused NF4 GEMV on the reference's headline configuration.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--m M] [--impl ours|reference]

Workload: W (N=4096, K=14336) with N(0, 0.02^2)
entries, NF4 blocksize 64, double-quantized (8-bit dynamic map, blocksize 256,
around the float32 mean); x bf16 (M, 14336) of N(0, 1); y = x @ W.T.
Synthetic, seeded data (torch Philox on the device). Eight independent weight
copies (8 x 30.3 MB = 242 MB, more than the 126 MB L2) are rotated so every
call reads its weight from HBM.

A step is one GEMV call. `value` is the whole job's effective bandwidth
(algorithmic bytes: weight 30,292,996 B + x M*K*2 + y M*N*2, per call) with
inputs resident in HBM, timed with CUDA events around the replay of a CUDA
graph that holds the K timed calls. `e2e` is the same metric through the
public API (bnb_b200.matmul) with x copied from pinned host memory and y read
back every step; on one GPU the steps alternate between two streams (each
with its own buffers), so one step's copies overlap the other's call, and the
one-stream time per step is reported beside it. `m_sweep` repeats the device
timing at M = 2..20.

Multi-GPU (torchrun, one process per GPU): the north star's split. The
weight is partitioned by output rows (row_partition, whole nested blocks per
rank); a step is every rank's fused GEMV on its rows followed by the NVLink
all-gather of y (PeerGather: one kernel that stores {value, epoch} words into
every peer's inbox over NVLink and polls its own inbox, bounded), so
every rank holds the full (M, 4096) product when the step ends -- strong
scaling of one call. Each rank rotates 8 x N copies of its shard (242 MB per
rank whatever N is, more than L2). Before timing, every rank checks the
gathered y bitwise against the one-GPU product of the whole weight. The timed
region is bracketed by barriers and the max over ranks is reported.

Timing: after the barrier and a synchronize, a ~50 us spin kernel is queued
ahead of the start event so that the graph launch is already queued when the
clock starts (NVBench's blocking-kernel method); the K timed calls are one
graph replay.

Extra keys of the default line (N=1): `config1` (NF4 quantize and dequantize
of a 4096x4096 bf16 tensor), `config3` (8-bit blockwise of 2^28+37 elements,
f32/f16/bf16, blocksizes 256 and 4096), `config5` (the fused GEMM on the
Llama-3-70B MLP shapes at M=2048 beside dequantize+matmul), `next_rows`
(the config-2 weight shape through the fused 8-bit-weight GEMV and the fused
backward g @ W, each beside the reference's dequantize route) and, at every N,
`config4` (one pass over a Llama-3-8B decode stack with every GEMV
row-sharded and its y all-gathered). `config1` also times the single-launch
NF4 + double quantization beside the three-launch chain.

`--workload quant` and `--workload gemm` (not read by the driver) measure the
other configurations the same way: config 1 (NF4 quantize + dequantize round
trip of a 4096x4096 bf16 tensor, 8 rotated copies), config 3 (8-bit blockwise
quantize and dequantize of 2^28+37 elements, f32/f16/bf16, blocksizes 256 and
4096, 90% N(0,1) + 10% Laplace(0,8)) and config 5 (the fused tcgen05 GEMM on
the Llama-3-70B MLP shapes at M = 64, 512, 2048, beside dequantize + matmul).
`--workload llama` is config 4: a Llama-3-8B decode stack (32 layers x q, k,
v, o, gate, up, down; NF4 bs 64 double-quantized) with every GEMV sharded by
output rows across the torchrun ranks and its y all-gathered (PeerGather, or
NCCL with --gather nccl); one
step is one pass over the 224 matrices, captured in a CUDA graph.

`--impl reference` times the reference's arithmetic on the host cores: the
reference has no CPU kernel path of its own (its kernels are GPU-only CuTe DSL)
and cannot be installed here, so its GEMV is the oracle's C restatement
(oracle/bnbq_oracle.c, OpenMP on every core), on the same configuration.
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
sys.path.insert(0, str(ROOT / "bitsandbytes-jax_b200"))
sys.path.insert(0, str(ROOT))

N_ROWS, K_COLS, BS, BS2, ROTATE = 4096, 14336, 64, 256, 8
W_BYTES = N_ROWS * K_COLS // 2 + N_ROWS * K_COLS // BS + (N_ROWS * K_COLS // BS // BS2) * 4 + 256 * 4 + 4
METRIC = "NF4 GEMV effective HBM GB/s & µs at M=1..20 (4096×14336), % of B200 peak"
WORKLOAD = ("fused NF4 GEMV y = x @ W.T, W 4096x14336 NF4 bs64 double-quantized (bs2 256), "
            "x bf16 M x 14336, 8 rotated weight copies")


def algo_bytes(m: int) -> int:
    return W_BYTES + m * K_COLS * 2 + m * N_ROWS * 2


def measured_peaks() -> tuple[float, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
        except Exception:
            pass
    return 6650.0, "fallback"


def profiled_traffic(m: int):
    """DRAM bytes per launch from the committed ncu summary, if one exists."""
    p = ROOT / "profiles" / "gemv_nf4_traffic.json"
    if p.exists():
        try:
            return json.loads(p.read_text()).get(f"m{m}")
        except Exception:
            return None
    return None


# --------------------------------------------------------------- clocks

class ClockSampler:
    """nvidia-smi clocks and throttle reasons while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines: list[str] = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
            time.sleep(0.25)
        except FileNotFoundError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc is not None:
            time.sleep(0.2)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        sms, maxes, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sms.append(float(parts[1]))
                maxes.append(float(parts[2]))
            except ValueError:
                continue
            for name, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(name)
        if not sms:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sms), "sm_max_mhz": max(maxes),
                "reasons": sorted(reasons), "samples": len(sms)}


# ------------------------------------------------------------------ ours

def spin_ahead(torch, stream, us: float = 50.0) -> None:
    """Queue a ~`us` spin kernel on `stream`, so the work enqueued right after
    it is already queued when the GPU reaches the next event (untimed)."""
    with torch.cuda.stream(stream):
        torch.cuda._sleep(int(us * 1e-6 * 1.965e9))


class Shard:
    """One rotation copy as the timed call takes it: the rank's rows of the
    weight (the whole weight on one GPU)."""

    def __init__(self, rs, full=None):
        self.rs = rs        # bnb_b200.parallel.RowShard
        self.full = full    # the whole QuantizedArray (kept for copy 0 only)


def make_shards(torch, bnb, device, copies: int, rank: int, world: int):
    """`copies` independent weights (the same on every rank), each cut to this
    rank's rows; the full weight of copy 0 is kept for the bitwise check."""
    from bnb_b200.parallel import row_partition, shard_rows
    ranges = row_partition(N_ROWS, K_COLS, BS * BS2, world)
    a, b = ranges[rank]
    shards = []
    for i in range(copies):
        g = torch.Generator(device).manual_seed(100 + i)
        w = bnb.quantize((torch.randn(N_ROWS, K_COLS, device=device, generator=g) * 0.02).to(torch.bfloat16),
                         "nf4", BS, double_quant=True)
        rs = shard_rows(w, a, b)
        if world > 1:  # own copies of the rank's slices; the full weight is dropped
            rs.data, rs.absmax = rs.data.clone(), rs.absmax.clone()
        shards.append(Shard(rs, w if (i == 0 or world == 1) else None))
        del w
    torch.cuda.synchronize()
    return shards, ranges


def time_device(torch, step, steps: int, warmup: int, device, dist=None):
    """Device time (ms) of `steps` calls step(i) replayed from one CUDA graph."""
    for i in range(max(warmup, 3)):  # eager warm-up (also primes per-device setup)
        step(i)
    torch.cuda.synchronize()
    stream = torch.cuda.Stream(device=device)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(stream):
        with torch.cuda.graph(graph, stream=stream):
            for i in range(steps):
                step(i)
    for _ in range(2):  # graph warm-up replays
        with torch.cuda.stream(stream):
            graph.replay()
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    spin_ahead(torch, stream)
    start.record(stream)
    with torch.cuda.stream(stream):
        graph.replay()
    end.record(stream)
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    ms = start.elapsed_time(end)
    del graph
    return ms


def make_step(torch, shards, x, ranges, rank, world, pg):
    """One call: the fused GEMV on this rank's rows (+ the all-gather of y)."""
    from bnb_b200.kernels import gemv_nf4
    m = x.shape[0]
    copies = len(shards)
    if world == 1:
        ys = [torch.empty(m, N_ROWS, dtype=torch.bfloat16, device=x.device) for _ in range(copies)]
        args = []
        for sh in shards:
            a = sh.full.absmax
            args.append((sh.full.data, a.data, (a.absmax, a.code, a.offset, a.blocksize)))

        def step(i):
            d, aq, nested = args[i % copies]
            gemv_nf4(x, d, aq, N_ROWS, BS, nested=nested, out=ys[i % copies])
            return ys[i % copies]
        return step
    def step(i):  # the rank's rows and the exchange in one call
        return pg.matmul(x, shards[i % copies].rs)
    return step


def time_e2e(torch, step_fn, device, m: int, steps: int, warmup: int, dist=None, lanes: int = 1):
    """The public API with host buffers: pinned x -> device, the call, y -> host.

    lanes = 1: every step on one stream, so a step's copies and call run
    strictly after the previous step's (per-step latency). lanes = 2: steps
    alternate between two streams with their own pinned and device buffers,
    so the copies of one step overlap the call of the other (throughput of a
    pipelined caller); every step still copies its x in and its y out."""
    g = torch.Generator().manual_seed(7)
    xh = [torch.randn(m, K_COLS, generator=g).to(torch.bfloat16).pin_memory() for _ in range(lanes)]
    yh = [torch.empty(m, N_ROWS, dtype=torch.bfloat16).pin_memory() for _ in range(lanes)]
    xd = [torch.empty(m, K_COLS, dtype=torch.bfloat16, device=device) for _ in range(lanes)]
    main = torch.cuda.current_stream(device)
    streams = [main] if lanes == 1 else [torch.cuda.Stream(device) for _ in range(lanes)]

    def one(i):
        j = i % lanes
        if lanes > 1:
            torch.cuda.set_stream(streams[j])
        xd[j].copy_(xh[j], non_blocking=True)
        y = step_fn(xd[j], i)
        yh[j].copy_(y, non_blocking=True)

    for i in range(max(warmup, 3)):
        one(i)
    torch.cuda.set_stream(main)
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(main)
    for s in streams:
        s.wait_event(start)
    for i in range(steps):
        one(i)
    torch.cuda.set_stream(main)
    for s in streams:
        main.wait_stream(s)
    end.record(main)
    torch.cuda.synchronize()
    ms = start.elapsed_time(end)
    if dist is not None:
        t = torch.tensor([ms], device=device, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    return ms, m * K_COLS * 2, m * N_ROWS * 2


def cpu_baseline_gemv(seconds: float = 12.0):
    """The oracle's C restatement of the reference GEMV (its float32
    numerics), M=1 on the full 4096x14336 weight, OpenMP on every host core."""
    import numpy as np
    from oracle import oracle as O
    O.set_threads(os.cpu_count() or 1)
    rng = np.random.default_rng(0)
    w = (rng.standard_normal(N_ROWS * K_COLS) * 0.02).astype(np.float32)
    q, am = O.quantize_nf4(w, O.F32, BS)
    off = O.mean_f32(am)
    code = O.create_dynamic_map()
    q2, am2 = O.quantize_8bit(am, O.F32, BS2, code, offset=off)
    scales = O.nested_absmax(q2, am2, code, off, BS2)  # decoded per call below
    x = O.f32_to_bf16(rng.standard_normal((1, K_COLS)).astype(np.float32)).reshape(1, K_COLS)
    cores = O.num_threads()
    O.gemv_ref(x, O.BF16, q, N_ROWS, BS, scales)  # warm-up
    calls, t0 = 0, time.perf_counter()
    while True:
        scales = O.nested_absmax(q2, am2, code, off, BS2)
        O.gemv_ref(x, O.BF16, q, N_ROWS, BS, scales)
        calls += 1
        el = time.perf_counter() - t0
        if el >= seconds:
            break
    gbs = algo_bytes(1) * calls / el / 1e9
    return {"value": round(gbs, 3), "unit": "GB/s", "cores": cores, "kind": "port",
            "sample": f"{calls} full M=1 GEMV calls (4096x14336, double-quantized) in {el:.1f} s"}


def bench_config(m: int, world: int) -> dict:
    """The `config` object both arms print (identical keys and values)."""
    return {"workload": WORKLOAD, "m": m, "n": N_ROWS, "k": K_COLS, "blocksize": BS,
            "blocksize2": BS2, "weight_bytes": W_BYTES, "algorithmic_bytes_per_call": algo_bytes(m),
            "l2": "rotated weight copies: 242 MB per GPU (8 x N shards of 30.3/N MB), more than the 126 MB L2",
            "timing": "CUDA graph of the K calls, queued behind a spin kernel",
            "parallelism": f"tp{world} (rows) + NVLink all-gather of y" if world > 1 else "1 GPU"}


def run_ours(args, dist, rank, world, local_rank):
    import torch
    import bnb_b200 as bnb
    from bnb_b200.parallel import PeerGather

    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    copies = ROTATE * world
    shards, ranges = make_shards(torch, bnb, device, copies, rank, world)
    g = torch.Generator(device).manual_seed(1234)
    x = torch.randn(args.m, K_COLS, device=device, generator=g).to(torch.bfloat16)
    pg = PeerGather(GEMV_MAX_ROWS, N_ROWS, torch.bfloat16, device) if world > 1 else None
    step = make_step(torch, shards, x, ranges, rank, world, pg)

    # every rank: the gathered (or single-GPU) y of copy 0 equals the one-GPU product bitwise
    want = bnb.matmul(x, shards[0].full)
    ok = torch.equal(step(0), want)
    torch.cuda.synchronize()
    if dist is not None:
        flag = torch.tensor([0 if ok else 1], device=device, dtype=torch.int32)
        dist.all_reduce(flag, op=dist.ReduceOp.MAX)
        ok = int(flag.item()) == 0
    if not ok:
        raise RuntimeError("the gathered product differs from the one-GPU product")
    del want

    with ClockSampler(local_rank) as clocks:
        ms = time_device(torch, step, args.steps, args.warmup, device, dist)
    ms_t = torch.tensor([ms], device=device, dtype=torch.float64)
    if dist is not None:
        dist.all_reduce(ms_t, op=dist.ReduceOp.MAX)
    ms_max = float(ms_t.item())

    sweep = {}
    for m in ([2, 4, 8, 16, 20] if (args.sweep and world == 1) else []):
        xm = torch.randn(m, K_COLS, device=device, generator=g).to(torch.bfloat16)
        sm = make_step(torch, shards, xm, ranges, rank, world, pg)
        k = max(args.steps // 4, 64)
        per = time_device(torch, sm, k, args.warmup, device) / k
        sweep[f"m{m}"] = {"us": round(per * 1e3, 3), "gbs": round(algo_bytes(m) / (per * 1e-3) / 1e9, 1)}

    e2e_steps = min(args.steps, 500)
    if world == 1:
        def e2e_call(xd, i):
            return bnb.matmul(xd, shards[i % copies].full)
    else:
        def e2e_call(xd, i):
            return pg.matmul(xd, shards[i % copies].rs)
    # one GPU: two streams, steps overlapped (the throughput e2e), and one
    # stream (per-step latency, reported beside it); several GPUs: one stream
    # per rank (the peer exchange orders a rank's calls on its stream)
    e2e_lanes = 2 if world == 1 else 1
    e2e_ms, h2d, d2h = time_e2e(torch, e2e_call, device, args.m, e2e_steps, args.warmup, dist, e2e_lanes)
    e2e_serial_ms = (time_e2e(torch, e2e_call, device, args.m, e2e_steps, args.warmup, dist, 1)[0]
                     if e2e_lanes > 1 else e2e_ms)

    extras = {}
    if not args.no_extras:
        extras["config4"] = llama_pass(args, dist, rank, world, local_rank)
        if world == 1:
            extras["config1"], extras["config3"] = quant_cases(torch, device, args.warmup)
            extras["config5"] = gemm_cases(torch, bnb, device)
            try:  # an extension's failure is recorded in its key, not lost with the whole line
                extras["next_rows"] = next_rows_cases(torch, bnb, device, args.warmup)
            except (NotImplementedError, ValueError, RuntimeError) as e:
                extras["next_rows"] = {"error": f"{type(e).__name__}: {e}"[:300]}
    if pg is not None:
        torch.cuda.synchronize()
        dist.barrier()
        pg.close()

    # which kernels the timed call ran (the table GEMV unless it does not apply)
    from bnb_b200 import _lib
    nb = _lib.gemv_workspace_bytes(args.m, K_COLS, ranges[rank][1] - ranges[rank][0])
    wsp = _lib.workspace(device, torch._C._cuda_getCurrentRawStream(device.index), nb) if nb else None
    route = _lib.gemv_route(args.m, K_COLS, ranges[rank][1] - ranges[rank][0], BS,
                            shards[0].rs.absmax.data_ptr(), BS2, _lib.ptr(wsp), 0 if wsp is None else wsp.numel())
    kernel = {_lib.ROUTE_TABLE_GEMV: "gemv_xtab_kernel", _lib.ROUTE_GEMV: "gemv_bulk_kernel / gemm_kernel (precise)",
              _lib.ROUTE_GEMM: "gemm_kernel"}[route]
    if rank != 0:
        return None
    per_call_ms = ms_max / args.steps
    value = algo_bytes(args.m) * args.steps / (ms_max * 1e-3) / 1e9
    peak, peak_kind = measured_peaks()
    achieved = algo_bytes(args.m) / (per_call_ms * 1e-3) / 1e9
    line = {
        "metric": METRIC,
        "value": round(value, 2),
        "unit": "GB/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(per_call_ms, 6),
        "us_per_call": round(per_call_ms * 1e3, 3),
        "higher_is_better": True,
        "scaling": "strong" if world > 1 else "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (seeded torch Philox: W ~ N(0, 0.02^2), x ~ N(0, 1))",
        "config": bench_config(args.m, world),
        "verified": "gathered y == one-GPU product, bitwise, every rank" if world > 1 else "y == bnb.matmul(x, w)",
        "roofline": roofline_entry(args.m, per_call_ms, peak, peak_kind, world, kernel),
        "e2e": {"value": round(algo_bytes(args.m) * e2e_steps / (e2e_ms * 1e-3) / 1e9, 2), "unit": "GB/s",
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "us_per_step": round(e2e_ms / e2e_steps * 1e3, 3), "streams": e2e_lanes,
                "one_stream_us_per_step": round(e2e_serial_ms / e2e_steps * 1e3, 3)},
        "gpu_launches": args.steps * launches_per_call(args.m, route, world),
        "clocks": clocks.summary(),
    }
    if sweep:
        line["m_sweep"] = sweep
    line.update(extras)
    if world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline_gemv()
    return line


GEMV_MAX_ROWS = 20


def launches_per_call(m: int, route: int, world: int) -> int:
    """Kernels one timed call launches: the table GEMV is two (partials, then
    their reduction), the streaming GEMV and the GEMM one; M = 3, 4 take two
    passes; at N > 1 the exchange rides in the GEMV's epilogue for M <= 2 and
    is one more kernel otherwise."""
    from bnb_b200 import _lib
    per = 2 if route == _lib.ROUTE_TABLE_GEMV else 1
    if route != _lib.ROUTE_GEMM and 3 <= m <= 4:
        per *= 2
    return per + (1 if world > 1 and m > 2 else 0)


def roofline_entry(m, per_call_ms, peak, peak_kind, world, kernel):
    """The dominant kernel: the GEMV (the whole call at N=1)."""
    achieved = algo_bytes(m) / (per_call_ms * 1e-3) / 1e9
    entry = {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
             "frac": round(achieved / peak, 4), "peak_source": peak_kind,
             "traffic": profiled_traffic(m), "kernel": kernel}
    if world > 1:
        entry["note"] = "whole-call rate (GEMV on 1/N of the rows + all-gather) against one GPU's peak"
    return entry


def time_graph(torch, call, steps: int, warmup: int, device):
    """Device time of `steps` calls call(i) replayed from one CUDA graph (ms)."""
    for i in range(max(warmup, 3)):
        call(i)
    torch.cuda.synchronize()
    stream = torch.cuda.Stream(device=device)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(stream):
        with torch.cuda.graph(graph, stream=stream):
            for i in range(steps):
                call(i)
    graph.replay()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    with torch.cuda.stream(stream):
        graph.replay()
    end.record(stream)
    torch.cuda.synchronize()
    ms = start.elapsed_time(end)
    del graph
    return ms


def quant_cases(torch, device, warmup: int, steps: int = 8):
    """Configs 1 and 3: blockwise quantize / dequantize bandwidth (device time
    per call, CUDA graph of `steps` calls); returns (config1, config3) dicts."""
    from bnb_b200.kernels import (absmax_mean, create_dynamic_map, dequantize_blockwise, dequantize_nf4,
                                  quantize_blockwise, quantize_nf4, quantize_nf4_dq)
    peak, _ = measured_peaks()
    # config 1: 4096 x 4096 bf16, NF4 bs 64, 8 rotated copies (256 MiB)
    n1 = 4096 * 4096
    g = torch.Generator(device).manual_seed(0)
    xs = [(torch.randn(n1, device=device, generator=g) * 0.02).to(torch.bfloat16) for _ in range(8)]
    qs = [quantize_nf4(x, 64) for x in xs]
    b1 = n1 * 2 + n1 // 2 + 4 * (n1 // 64)
    s1 = max(steps, 16)
    tq = time_graph(torch, lambda i: quantize_nf4(xs[i % 8], 64), s1, warmup, device) / s1
    td = time_graph(torch, lambda i: dequantize_nf4(qs[i % 8][0], qs[i % 8][1], 64, torch.bfloat16),
                    s1, warmup, device) / s1
    c1 = {"workload": "NF4 bs64 of one 4096x4096 bf16 tensor (8 rotated copies)", "bytes_per_call": b1,
          "quantize_us": round(tq * 1e3, 2), "quantize_gbs": round(b1 / (tq * 1e-3) / 1e9, 1),
          "quantize_frac": round(b1 / (tq * 1e-3) / 1e9 / peak, 3),
          "dequantize_us": round(td * 1e3, 2), "dequantize_gbs": round(b1 / (td * 1e-3) / 1e9, 1),
          "dequantize_frac": round(b1 / (td * 1e-3) / 1e9 / peak, 3)}
    # double quantization (the weight format of config 2): one launch against the three-call chain
    code2 = create_dynamic_map(device=device)

    def dq_chain(i):
        q, a = quantize_nf4(xs[i % 8], 64)
        quantize_blockwise(a, code2, 256, offset=absmax_mean(a))

    try:  # an extension's failure is recorded in its key, not lost with the whole line
        tdq = time_graph(torch, lambda i: quantize_nf4_dq(xs[i % 8], 64, code2), s1, warmup, device) / s1
        tch = time_graph(torch, dq_chain, s1, warmup, device) / s1
        c1["double_quant_us"] = round(tdq * 1e3, 2)
        c1["double_quant_chain_us"] = round(tch * 1e3, 2)
    except (NotImplementedError, ValueError, RuntimeError) as e:
        c1["double_quant_error"] = f"{type(e).__name__}: {e}"[:300]
    del xs, qs
    # config 3: 2^28 + 37 elements, 90% N(0,1) + 10% Laplace(0,8), 8-bit dynamic map
    n3 = (1 << 28) + 37
    code = create_dynamic_map().to(device)
    base = torch.randn(n3, device=device, generator=g)
    mask = torch.rand(n3, device=device, generator=g) < 0.1
    u = torch.rand(n3, device=device, generator=g) - 0.5  # Laplace(0, 8) by inverse CDF
    lap = -8.0 * torch.sign(u) * torch.log1p(-2.0 * u.abs())
    del u
    base = torch.where(mask, lap, base)
    del mask, lap
    c3 = {"workload": "8-bit dynamic map, 2^28+37 elements, 90% N(0,1) + 10% Laplace(0,8)"}
    for dt, name in [(torch.float32, "f32"), (torch.float16, "f16"), (torch.bfloat16, "bf16")]:
        x = base.to(dt)
        for bs in (256, 4096):
            q, a = quantize_blockwise(x, code, bs)
            b3 = n3 * x.element_size() + n3 + 4 * (-(-n3 // bs))
            s3 = 3
            tq = time_graph(torch, lambda i: quantize_blockwise(x, code, bs), s3, 1, device) / s3
            td = time_graph(torch, lambda i: dequantize_blockwise(q, a, code, bs, dt), s3, 1, device) / s3
            c3[f"{name}_bs{bs}"] = {
                "bytes_per_call": b3,
                "quantize_us": round(tq * 1e3, 1), "quantize_gbs": round(b3 / (tq * 1e-3) / 1e9, 1),
                "quantize_frac": round(b3 / (tq * 1e-3) / 1e9 / peak, 3),
                "dequantize_us": round(td * 1e3, 1), "dequantize_gbs": round(b3 / (td * 1e-3) / 1e9, 1),
                "dequantize_frac": round(b3 / (td * 1e-3) / 1e9 / peak, 3)}
            del q, a
        del x
    del base
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    return c1, c3


def run_quant_workload(args, local_rank):
    import torch
    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    with ClockSampler(local_rank) as clocks:
        c1, c3 = quant_cases(torch, device, args.warmup, max(args.steps // 100, 8))
    rt_us = c1["quantize_us"] + c1["dequantize_us"]
    value = 2 * c1["bytes_per_call"] / (rt_us * 1e-6) / 1e9
    return {"metric": "blockwise quantize/dequantize effective HBM GB/s (configs 1 and 3)",
            "value": round(value, 1), "unit": "GB/s", "n_gpus": 1, "higher_is_better": True,
            "dtype": "bf16/f16/f32", "data": "synthetic (seeded torch Philox)",
            "config": {"workload": "config 1 NF4 round trip (value) + config 3 8-bit blockwise (details)"},
            "config1": c1, "config3": c3, "clocks": clocks.summary()}


def run_quant_profile(args, local_rank):
    """The driver of a quantize profile (an ncu target, not a measurement):
    four eager calls on 2^27 N(0, 1) values of --qdtype at --qbs --
    quantize_blockwise with the dynamic map (--qtype 8bit), or quantize_nf4
    on the 4096 x 4096 N(0, 0.02^2) tensor of config 1 (--qtype nf4), or the
    single-launch NF4 + double quantization of that tensor (--qtype nf4dq).
    Captured with, e.g.,
    ncu --set full --clock-control none -k regex:quant_8bit -s 2 -c 1 ...
    python bench.py --workload quant-profile --qdtype f16 --qbs 256"""
    import torch
    from bnb_b200.kernels import create_dynamic_map, quantize_blockwise, quantize_nf4, quantize_nf4_dq
    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    dt = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}[args.qdtype]
    g = torch.Generator(device).manual_seed(0)
    if args.qtype == "nf4dq":
        x = (torch.randn(4096 * 4096, device=device, generator=g) * 0.02).to(dt)
        for _ in range(4):
            q = quantize_nf4_dq(x, args.qbs)[0]
    elif args.qtype == "nf4":
        x = (torch.randn(4096 * 4096, device=device, generator=g) * 0.02).to(dt)
        for _ in range(4):
            q, a = quantize_nf4(x, args.qbs)
    else:
        x = torch.randn(1 << 27, device=device, generator=g).to(dt)
        code = create_dynamic_map().to(device)
        for _ in range(4):
            q, a = quantize_blockwise(x, code, args.qbs)
    torch.cuda.synchronize()
    return {"workload": "quant-profile", "qtype": args.qtype, "dtype": args.qdtype, "blocksize": args.qbs,
            "n": x.numel(),
            "calls": 4, "codes_checksum": int(q[:4096].to(torch.int64).sum().item())}


def run_matmul_profile(args, local_rank):
    """The driver of a matmul profile (an ncu target, not a measurement): four
    eager bnb.matmul calls at M = --rows on one (--pn, --pk) NF4 (--wq nf4) or
    8-bit (--wq 8bit) bs64 double-quantized weight of N(0, 0.02^2) entries,
    with the kernels the router picks (reported as "route"), or four calls of
    the fused backward g @ W with g of M x --pn (--backward)."""
    import torch
    import bnb_b200 as bnb
    from bnb_b200 import _lib
    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    g = torch.Generator(device).manual_seed(0)
    w = bnb.quantize((torch.randn(args.pn, args.pk, device=device, generator=g) * 0.02).to(torch.bfloat16), args.wq,
                     BS, double_quant=True)
    x = torch.randn(args.m, args.pk, device=device, generator=g).to(torch.bfloat16)
    if args.backward:  # the fused backward g @ W, g of M x --pn
        x = torch.randn(args.m, args.pn, device=device, generator=g).to(torch.bfloat16)
        from bnb_b200.kernels import gemv_t_nf4
        a = w.absmax
        for _ in range(4):
            y = gemv_t_nf4(x, w.data, a.data, args.pn, args.pk, BS, nested=(a.absmax, a.code, a.offset, a.blocksize))
        torch.cuda.synchronize()
        return {"workload": "matmul-profile", "backward": True, "n": args.pn, "k": args.pk, "m": args.m,
                "calls": 4, "y_checksum": float(y.float().sum().item())}
    for _ in range(4):
        y = bnb.matmul(x, w)
    torch.cuda.synchronize()
    nb = _lib.gemv_workspace_bytes(args.m, args.pk, args.pn) if args.m <= 20 else 0
    ws = torch.empty(max(nb, 16), dtype=torch.uint8, device=device)
    route = (_lib.gemv_route(args.m, args.pk, args.pn, BS, w.absmax.data.data_ptr(), BS2, ws.data_ptr(), nb)
             if args.wq == "nf4" else "8-bit GEMV" if args.m <= _lib.GEMV8_MAX_M else "dequantize + matmul")
    return {"workload": "matmul-profile", "weight": args.wq, "n": args.pn, "k": args.pk, "m": args.m, "calls": 4,
            "route": route,
            "y_checksum": float(y.float().sum().item())}


def next_rows_cases(torch, bnb, device, warmup: int):
    """The config-2 weight shape through the two extensions beyond the
    reference's kernels: the fused GEMV of an 8-bit weight (dynamic map, bs 64,
    double-quantized) and the fused backward g @ W of the NF4 weight, each
    beside the reference's own route (x @ w.dequantize().T; g @ w.dequantize()).
    Device time per call, CUDA graph over rotated weights (more than L2)."""
    from bnb_b200.kernels import gemv_t_nf4
    g0 = torch.Generator(device).manual_seed(5)
    out = {}
    w8 = [bnb.quantize((torch.randn(N_ROWS, K_COLS, device=device, generator=g0) * 0.02).to(torch.bfloat16), "8bit",
                       BS, double_quant=True) for _ in range(4)]
    b8 = N_ROWS * K_COLS + N_ROWS * K_COLS // BS
    for m in (1, 4):
        x = torch.randn(m, K_COLS, device=device, generator=g0).to(torch.bfloat16)
        t = time_graph(torch, lambda i: bnb.matmul(x, w8[i % 4]), 64, warmup, device) / 64
        tr = time_graph(torch, lambda i: x @ w8[i % 4].dequantize(x.dtype).T, 16, warmup, device) / 16
        out[f"gemv_8bit_m{m}"] = {"us": round(t * 1e3, 2), "weight_gbs": round(b8 / (t * 1e-3) / 1e9, 1),
                                  "dequantize_matmul_us": round(tr * 1e3, 2)}
    del w8
    w4 = [bnb.quantize((torch.randn(N_ROWS, K_COLS, device=device, generator=g0) * 0.02).to(torch.bfloat16), "nf4",
                       BS, double_quant=True) for _ in range(8)]

    def fused(w, gm):
        a = w.absmax
        return gemv_t_nf4(gm, w.data, a.data, N_ROWS, K_COLS, BS, nested=(a.absmax, a.code, a.offset, a.blocksize))

    for m in (1, 4):
        gm = torch.randn(m, N_ROWS, device=device, generator=g0).to(torch.bfloat16)
        t = time_graph(torch, lambda i: fused(w4[i % 8], gm), 64, warmup, device) / 64
        tr = time_graph(torch, lambda i: gm @ w4[i % 8].dequantize(gm.dtype), 16, warmup, device) / 16
        out[f"backward_m{m}"] = {"us": round(t * 1e3, 2), "weight_gbs": round(W_BYTES / (t * 1e-3) / 1e9, 1),
                                 "dequantize_matmul_us": round(tr * 1e3, 2)}
    del w4
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    return out


def gemm_cases(torch, bnb, device, ms=(64, 512, 2048)):
    """Config 5: the fused NF4 dequantize-GEMM on the Llama-3-70B MLP shapes,
    beside the reference's fallback (dequantize + matmul) and bnb_b200.matmul
    (the router: fused up to 512 rows of x, the fallback above)."""
    from bnb_b200.kernels.gemv import matmul_nf4
    out = {}
    peak_tf = 1669.8
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        peak_tf = float(json.loads(p.read_text()).get("bf16_tflops", peak_tf))
    for (n, k) in [(28672, 8192), (8192, 28672)]:
        g = torch.Generator(device).manual_seed(n)
        w = bnb.quantize((torch.randn(n, k, device=device, generator=g) * 0.015).to(torch.bfloat16),
                         "nf4", 64, double_quant=True)
        a = w.absmax
        nested = (a.absmax, a.code, a.offset, a.blocksize)
        for m in ms:
            x = torch.randn(m, k, device=device, generator=g).to(torch.bfloat16)
            s5 = 5 if m == 2048 else 10
            tf = time_graph(torch, lambda i: matmul_nf4(x, w.data, a.data, n, 64, nested=nested),
                            s5, 2, device) / s5
            tr = time_graph(torch, lambda i: x @ w.dequantize(torch.bfloat16).T, s5, 2, device) / s5
            tm = time_graph(torch, lambda i: bnb.matmul(x, w), s5, 2, device) / s5  # the router's choice
            fl = 2.0 * m * n * k
            out[f"{n}x{k}_m{m}"] = {"matmul_us": round(tm * 1e3, 1), "fused_us": round(tf * 1e3, 1),
                                    "fused_tflops": round(fl / (tf * 1e-3) / 1e12, 1),
                                    "dequant_matmul_us": round(tr * 1e3, 1),
                                    "speedup_vs_dequant_matmul": round(tr / tf, 2),
                                    "frac_of_bf16_peak": round(fl / (tf * 1e-3) / 1e12 / peak_tf, 3)}
        del w, a
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    out["peak_tflops"] = peak_tf
    return out


def run_gemm_workload(args, local_rank):
    import torch
    import bnb_b200 as bnb
    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    with ClockSampler(local_rank) as clocks:
        out = gemm_cases(torch, bnb, device)
    return {"metric": "fused NF4 dequantize-GEMM TFLOP/s (config 5)", "value": out["28672x8192_m2048"]["fused_tflops"],
            "unit": "TFLOP/s", "n_gpus": 1, "higher_is_better": True, "dtype": "bf16",
            "data": "synthetic (seeded torch Philox)",
            "config": {"workload": "config 5: Llama-3-70B MLP gate/up 28672x8192 and down 8192x28672, NF4 bs64 nested"},
            "config5": out, "clocks": clocks.summary()}


LLAMA8B = [(4096, 4096), (1024, 4096), (1024, 4096), (4096, 4096), (14336, 4096), (14336, 4096), (4096, 14336)]
# the same weights with q/k/v stacked into one matrix and gate/up into another
# (one GEMV and one exchange for each group): 4 matrices a layer
LLAMA8B_GROUPED = [(6144, 4096), (4096, 4096), (28672, 4096), (4096, 14336)]


def llama_pass(args, dist, rank, world, local_rank, m: int = 1, gather: str = "peer", grouped: bool = True):
    """Config 4: device time of one pass over a Llama-3-8B decode stack (32
    layers of q, k, v, o, gate, up, down; q/k/v and gate/up stacked into one
    NF4 matrix each when `grouped`), every GEMV row-sharded over the ranks and
    its y all-gathered. Max over ranks; every rank returns the same dict."""
    import torch
    from bnb_b200.parallel import PeerGather, all_gather_rows, matmul_rows, quantize_shard, row_partition, shard_rows
    device = torch.device("cuda", local_rank)
    layers = 32
    shards, plans = [], []
    weight_bytes = 0
    mats = LLAMA8B_GROUPED if grouped else LLAMA8B
    for i in range(layers * len(mats)):
        n, k = mats[i % len(mats)]
        ranges = row_partition(n, k, BS * BS2, world)  # whole nested blocks per rank
        a, b = ranges[rank]
        g = torch.Generator(device).manual_seed(1000 + i)  # the same full weight on every rank
        w_rows = (torch.randn(n, k, device=device, generator=g)[a:b] * 0.02).to(torch.bfloat16)
        qa = quantize_shard(w_rows, "nf4", BS, double_quant=True, group=None if dist is None else dist.group.WORLD)
        qa = type(qa)(qa.data, qa.absmax, qa.code, qa.offset, qa.qtype, qa.blocksize, (b - a, k), qa.dtype)
        sh = shard_rows(qa, 0, b - a)  # local arrays (own absmax2, block0 0); global row range below
        sh.start, sh.stop, sh.n_rows_total = a, b, n
        shards.append(sh)
        plans.append(ranges)
        weight_bytes += n * k // 2 + n * k // BS + 4 * (n * k // BS // BS2)
        del w_rows
    torch.cuda.synchronize()
    g = torch.Generator(device).manual_seed(5)
    xs = {k: torch.randn(m, k, device=device, generator=g).to(torch.bfloat16) for k in (4096, 14336)}
    peer = gather == "peer" and world > 1
    pgs = {n: PeerGather(m, n, torch.bfloat16, device) for n in sorted({n for n, _ in mats})} if peer else {}

    def step():
        for sh, ranges in zip(shards, plans):
            if peer:  # the rank's rows and the exchange in one call
                pgs[sh.n_rows_total].matmul(xs[sh.k], sh)
                continue
            y = matmul_rows(xs[sh.k], sh)
            if world > 1:
                all_gather_rows(y, ranges)

    for _ in range(3):
        step()
    torch.cuda.synchronize()
    stream = torch.cuda.Stream(device=device)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(stream):
        with torch.cuda.graph(graph, stream=stream):
            step()
    with torch.cuda.stream(stream):
        graph.replay()
    torch.cuda.synchronize()
    steps = 5
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    spin_ahead(torch, stream)
    start.record(stream)
    with torch.cuda.stream(stream):
        for _ in range(steps):
            graph.replay()
    end.record(stream)
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    ms = start.elapsed_time(end)
    del graph
    torch.cuda.synchronize()
    ms_t = torch.tensor([ms], device=device, dtype=torch.float64)
    if dist is not None:
        dist.all_reduce(ms_t, op=dist.ReduceOp.MAX)
    for pg in pgs.values():
        pg.close()
    if dist is not None:
        dist.barrier()
    per = float(ms_t.item()) / steps
    del shards, xs
    torch.cuda.empty_cache()
    shape = ("4 NF4 matrices (q|k|v and gate|up stacked)" if grouped else "7 NF4 matrices")
    return {"workload": f"Llama-3-8B decode stack, 32 layers x {shape} (bs64 nested), M={m}",
            "ms_per_pass": round(per, 4), "weight_gbs": round(weight_bytes / (per * 1e-3) / 1e9, 1),
            "weight_bytes_per_pass": weight_bytes, "n_gpus": world,
            "exchange": "NVLink peer stores" if peer else ("NCCL" if world > 1 else "none"),
            "parallelism": f"tp{world} (rows), y all-gathered after every GEMV" if world > 1 else "1 GPU"}


def run_llama_workload(args, dist, rank, world, local_rank):
    import torch
    torch.cuda.set_device(local_rank)
    with ClockSampler(local_rank) as clocks:
        c4 = llama_pass(args, dist, rank, world, local_rank, args.m, args.gather, not args.ungrouped)
    if rank != 0:
        return None
    return {"metric": "Llama-3-8B NF4 decode stack: effective weight GB/s, every GEMV row-sharded + all-gathered (config 4)",
            "value": c4["weight_gbs"], "unit": "GB/s", "n_gpus": world, "ms_per_step": c4["ms_per_pass"],
            "higher_is_better": True, "scaling": "strong", "dtype": "bf16", "data": "synthetic (seeded torch Philox)",
            "config": c4, "clocks": clocks.summary()}


def run_reference(args, rank):
    """The reference's arithmetic on the host cores (see module docstring), on
    every core of the host (torchrun's OMP_NUM_THREADS=1 is overridden)."""
    if rank != 0:
        return None
    import numpy as np
    from oracle import oracle as O
    O.set_threads(os.cpu_count() or 1)
    rng = np.random.default_rng(0)
    w = (rng.standard_normal(N_ROWS * K_COLS) * 0.02).astype(np.float32)
    q, am = O.quantize_nf4(w, O.F32, BS)
    off = O.mean_f32(am)
    code = O.create_dynamic_map()
    q2, am2 = O.quantize_8bit(am, O.F32, BS2, code, offset=off)
    x = O.f32_to_bf16(rng.standard_normal((args.m, K_COLS)).astype(np.float32)).reshape(args.m, K_COLS)
    cores = O.num_threads()

    def step():
        scales = O.nested_absmax(q2, am2, code, off, BS2)
        O.gemv_ref(x, O.BF16, q, N_ROWS, BS, scales)

    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    el = time.perf_counter() - t0
    value = algo_bytes(args.m) * args.steps / el / 1e9
    world = int(os.environ.get("WORLD_SIZE", "1"))
    return {
        "impl": "reference",
        "metric": METRIC, "value": round(value, 3), "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(el / args.steps * 1e3, 4),
        "higher_is_better": True, "scaling": "strong" if world > 1 else "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (numpy default_rng(0): W ~ N(0, 0.02^2), x ~ N(0, 1), the GPU arm's distributions)",
        "config": bench_config(args.m, world),
        "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": cores, "kind": "port",
                         "sample": f"{args.steps} full GEMV calls at M={args.m} on the host "
                                   f"(numpy default_rng(0) data of the same distributions)"},
        "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=16)
    ap.add_argument("--rows", "--m", dest="m", type=int, default=1)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-sweep", dest="sweep", action="store_false")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extras", action="store_true", help="skip the config 1/3/4/5 keys")
    ap.add_argument("--workload", choices=["gemv", "quant", "gemm", "llama", "quant-profile", "matmul-profile"],
                    default="gemv")
    ap.add_argument("--pn", type=int, default=14336, help="matmul-profile weight rows")
    ap.add_argument("--pk", type=int, default=4096, help="matmul-profile weight columns (K)")
    ap.add_argument("--qdtype", choices=["f32", "f16", "bf16"], default="f16", help="quant-profile input type")
    ap.add_argument("--qbs", type=int, default=256, help="quant-profile blocksize")
    ap.add_argument("--qtype", choices=["8bit", "nf4", "nf4dq"], default="8bit",
                    help="quant-profile quantization (nf4dq: NF4 with double quantization, one launch)")
    ap.add_argument("--wq", choices=["nf4", "8bit"], default="nf4", help="matmul-profile weight quantization")
    ap.add_argument("--backward", action="store_true", help="matmul-profile: the fused backward g @ W (NF4)")
    ap.add_argument("--gather", choices=["peer", "nccl"], default="peer", help="config 4 all-gather")
    ap.add_argument("--ungrouped", action="store_true", help="config 4 with q/k/v and gate/up as separate GEMVs")
    args = ap.parse_args()

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        if args.steps > 50:
            args.steps = 50  # each host step is a full GEMV: keep the run to seconds
        line = run_reference(args, rank)
        if line is not None:
            print(json.dumps(line), flush=True)
        return

    if args.workload in ("quant-profile", "matmul-profile"):
        if rank == 0:
            fn = run_quant_profile if args.workload == "quant-profile" else run_matmul_profile
            print(json.dumps(fn(args, local_rank)), flush=True)
        return

    if args.workload in ("quant", "gemm"):
        if rank == 0:
            fn = run_quant_workload if args.workload == "quant" else run_gemm_workload
            print(json.dumps(fn(args, local_rank)), flush=True)
        return

    dist = None
    if world > 1:
        import datetime
        import torch
        import torch.distributed as td
        torch.cuda.set_device(local_rank)
        td.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                              device_id=torch.device("cuda", local_rank))
        dist = td
    try:
        if args.workload == "llama":
            line = run_llama_workload(args, dist, rank, world, local_rank)
        else:
            line = run_ours(args, dist, rank, world, local_rank)
        if line is not None:
            print(json.dumps(line), flush=True)
    finally:
        if dist is not None:
            dist.barrier()
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
