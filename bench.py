#!/usr/bin/env python3
"""Benchmark of the W4A16 GEMM hot path on B200 -- one JSON line on rank 0.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload (the config the headline metric is quoted on):
the decode sweep M in {1, 4, 8, 16} x Llama-3-8B projections (N x K) 4096x4096,
1024x4096, 14336x4096, 4096x14336, G = 128.  One *step* runs all 16 GEMMs once,
each on its own weight copy (286 MB of packed weights per step, > 2x the 126 MB
L2, so nothing is served from L2 between uses).  Inputs are seeded synthetic
data with BASELINE's distributions (x ~ N(0,1) fp16, q ~ U{0..15}, scales ~
U[0.002, 0.02] fp16), resident in HBM before the timed region.

* value       -- algorithmic bytes (packed weights + scales + x + y) of all GEMMs
                 per second, device-timed (CUDA events around K CUDA-graph replays).
* e2e         -- the same metric through the public API (w4a16_opt.w4a16_gemm_out),
                 eager calls, with each step's activations copied host->device from
                 pinned memory and its outputs read back device->host (copies on a copy
                 stream, overlapping the neighbouring steps, as a serving loop does).
* roofline    -- achieved bytes/s of the decode kernel vs the measured HBM copy
                 bandwidth (MEASURED_PEAKS.json), plus the ncu DRAM traffic per launch
                 from profiles/ when a capture of this workload is committed.
* prefill     -- BASELINE configs[2] (M in {128, 512, 2048, 8192} x 14336x4096 /
                 4096x14336 x G in {64, 128}) in TFLOP/s against the measured dense
                 fp16/bf16 tensor peak (N = 1 only).
* cpu_baseline -- the reference's CPU path (fp16 dequant + fp32 matmul, torch CPU,
                 all host threads) over one pass of the same 16 GEMMs.

* tp70b       -- BASELINE configs[4] at this N (N = 1 included): Llama-3-70B gate/up
                 split along N (all-gather) and down split along K (fp32 all-reduce),
                 M in {1, 16} (GB/s) and M = 4096 (TFLOP/s), strong scaling, with the
                 collectives' share of the step.

With N > 1 (torchrun, one rank per GPU, NCCL) every rank serves its own decode sweep
(replicas of an 8B model: weak scaling; `value` is the sum over ranks, time the max
over ranks), and the tensor-parallel split is measured in tp70b.  ``--impl reference``
times the CPU reference path alone (rank 0).
"""
from __future__ import annotations

import argparse
import csv
import io
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "w4a16-gemm_b200")
for _p in (ROOT, PKG):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import torch  # noqa: E402

METRIC = "HBM GB/s at M≤16 & TFLOP/s at M≥128, 1–8 B200, % of roofline"
DECODE_SHAPES = (("q/o", 4096, 4096), ("k/v", 1024, 4096), ("gate/up", 14336, 4096), ("down", 4096, 14336))
DECODE_M = (1, 4, 8, 16)
DECODE_G = 128
PREFILL_M = (128, 512, 2048, 8192)
PREFILL_SHAPES = ((14336, 4096), (4096, 14336))
PREFILL_G = (64, 128)
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def alg_bytes(M, N, K, G):
    """Bytes a W4A16 GEMM must move at least once: packed weights, scales, x, y."""
    return N * K // 2 + 2 * N * (K // G) + 2 * M * K + 2 * M * N


def make_inputs(M, N, K, G, seed, device):
    """Seeded BASELINE inputs: x fp16 [M,K], q uint8 [N,K] (CPU), scales fp16, packed Wp.

    On "cpu" (the reference arm) nothing of this package is imported: the reference's CPU
    path takes the codes q directly and Wp is None."""
    gen = torch.Generator().manual_seed(seed)
    x = torch.randn(M, K, generator=gen).half()
    q = torch.randint(0, 16, (N, K), generator=gen, dtype=torch.uint8)
    scales = (torch.rand(K // G, N, generator=gen) * 0.018 + 0.002).half()
    if device == "cpu":
        return x, q, scales, None
    from w4a16_opt import pack_int4
    Wp = pack_int4(q.to(device))
    return x.to(device), q, scales.to(device), Wp


def bench_config(world):
    """The workload description both arms print (same dict, so the lines compare like for like)."""
    return {"workload": "configs[1] decode sweep: M in {1,4,8,16} x Llama-3-8B (N x K) "
                        "4096x4096, 1024x4096, 14336x4096, 4096x14336, G=128",
            "gemms_per_step": len(DECODE_SHAPES) * len(DECODE_M),
            "algorithmic_bytes_per_step": sum(alg_bytes(M, N, K, DECODE_G) for _, N, K in DECODE_SHAPES
                                              for M in DECODE_M),
            "l2": "inputs larger than L2: 16 distinct weight copies per step vs 126 MB L2",
            "parallelism": "single GPU" if world == 1 else f"{world} replicas (a sweep per GPU); tp{world} in tp70b"}


def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            d = json.load(f)
        return d, "measured"
    return dict(FALLBACK_PEAKS), "fallback"


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms while running."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        self.file = None

    def __enter__(self):
        self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=self.file, stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        self.file.flush()

    def summary(self):
        rows = []
        try:
            with open(self.file.name) as f:
                for r in csv.reader(f):
                    if len(r) >= 9:
                        rows.append([c.strip() for c in r])
        finally:
            os.unlink(self.file.name)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no nvidia-smi samples"], "samples": 0}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        smax = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(smax) if smax else None,
                "reasons": reasons, "samples": len(rows)}


def smi_index(local):
    """nvidia-smi index of this process's CUDA device (honours CUDA_VISIBLE_DEVICES)."""
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis:
        ids = [v.strip() for v in vis.split(",") if v.strip()]
        if local < len(ids):
            return ids[local]
    return str(local)


def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def max_over_ranks(v, world):
    if world == 1:
        return v
    import torch.distributed as dist
    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def graph_time_ms(step_fn, steps, warmup, world):
    """Capture one step in a CUDA graph, replay W untimed then K timed; device ms (max over ranks)."""
    from w4a16_opt.timing import GraphStep
    g = GraphStep(step_fn)
    g.warm(warmup)
    barrier(world)
    torch.cuda.synchronize()
    ms = g.total_ms(steps)
    torch.cuda.synchronize()
    barrier(world)
    ms = max_over_ranks(ms, world)
    g.close()
    return ms


def profile_traffic(name):
    """Per-launch DRAM bytes of a kernel from a committed ncu summary (profiles/<name>.json)."""
    path = os.path.join(ROOT, "profiles", name + ".json")
    if not os.path.exists(path):
        return None
    with open(path) as f:
        return json.load(f)


def cpu_reference_pass(units, threads):
    """One pass of the reference's CPU path over the given (x, q, scales, G) units; seconds."""
    from oracle import cpu_reference
    torch.set_num_threads(threads)
    t0 = time.perf_counter()
    for x, q, s, G in units:
        cpu_reference.ref_gemm(x, q, s, G)
    return time.perf_counter() - t0


# ---------------------------------------------------------------------------------------------- ours

def run_ours(args):
    world, rank, local = dist_env()
    torch.cuda.set_device(local)
    if world > 1:
        # rank 0's stdout carries exactly one JSON line: NCCL's own messages (its version
        # banner, debug output) go to stderr unless the caller chose a destination
        os.environ.setdefault("NCCL_DEBUG_FILE", "/dev/stderr")
        import datetime

        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    import w4a16_opt
    from w4a16_opt import tp

    # ---- decode sweep units.  With N ranks every rank serves its own full sweep (replicas of
    # an 8B model, which fits one GPU: weak scaling); the tensor-parallel split of the path is
    # measured on Llama-3-70B shapes below (tp70b).
    units, step_bytes, in_bytes, out_bytes = [], 0, 0, 0
    seed = 1000
    for name, N, K in DECODE_SHAPES:
        for M in DECODE_M:
            x, q, s, Wp = make_inputs(M, N, K, DECODE_G, seed, "cuda")
            seed += 1
            units.append({"name": name, "M": M, "N": N, "K": K, "x": x, "q": q, "s": s, "Wp": Wp,
                          "y": torch.empty(M, N, dtype=torch.float16, device="cuda")})
            step_bytes += alg_bytes(M, N, K, DECODE_G)
            in_bytes += 2 * M * K
            out_bytes += 2 * M * N
    # one workspace shared by every GEMM of the step (they run in stream order)
    ws = w4a16_opt.make_workspace(max(w4a16_opt.workspace_bytes(u["M"], u["N"], u["K"], u["K"] // DECODE_G)
                                      for u in units))
    torch.cuda.synchronize()

    def make_step(resident, fp32_scale=False):
        def step():
            for u in units:
                w4a16_opt.w4a16_gemm_out(u["Wp"], u["x"], u["s"], u["y"], workspace=ws, weights_resident=resident,
                                         fp32_scale=fp32_scale)
        return step

    # kernels of ours per step: one decode_kernel per GEMM (+ its combine kernel when a column
    # group is split across CTAs), as the route query reports
    launches_per_step = sum(w4a16_opt.query_route(u["M"], u["N"], u["K"], u["K"] // DECODE_G)["launches"]
                            for u in units)

    # headline: weights resident (loaded once, as in serving); the GEMMs stream them while
    # the previous GEMM finishes.  The default stream-ordered mode is measured right after.
    with ClockSampler(smi_index(local)) as clocks:
        ms = graph_time_ms(make_step(True), args.steps, args.warmup, world)
    ms_step = ms / args.steps
    value = world * step_bytes * args.steps / (ms / 1e3) / 1e9
    ms_default = graph_time_ms(make_step(False), args.steps, args.warmup, world)
    default_mode = {"value": round(world * step_bytes * args.steps / (ms_default / 1e3) / 1e9, 2), "unit": "GB/s",
                    "ms_per_step": round(ms_default / args.steps, 5),
                    "mode": "plain stream order: each GEMM reads its weights only after the previous kernel "
                            "on the stream has completed (w4a16_gemm default)"}
    ms_fs = graph_time_ms(make_step(True, True), args.steps, args.warmup, world)
    fp32_scale_mode = {"value": round(world * step_bytes * args.steps / (ms_fs / 1e3) / 1e9, 2), "unit": "GB/s",
                       "ms_per_step": round(ms_fs / args.steps, 5),
                       "mode": "weights resident + W4A16_FLAG_FP32_SCALE: for M <= 8 the group scales are applied "
                               "in fp32 after the tensor-core products (not the reference's bit-identical fp16 "
                               "dequantised weights; opt-in)"}

    # ---- e2e through the public API: every step copies its activations in from pinned host
    # memory (one transfer), makes the 16 calls into one output buffer and reads it back (one
    # transfer), as a serving loop does: the copies run on their own streams (one per
    # direction) and overlap the neighbouring steps' GEMMs (two buffer sets), and the host
    # waits for each step's result one step later.  Host wall time.
    e2e, host_us = None, None
    if world == 1:
        x_off, y_off = [0], [0]
        for u in units:
            x_off.append(x_off[-1] + u["x"].numel())
            y_off.append(y_off[-1] + u["M"] * u["N"])
        host_x = torch.cat([u["x"].flatten() for u in units]).cpu().pin_memory()
        dev_x = [torch.empty(x_off[-1], dtype=torch.float16, device="cuda") for _ in range(2)]
        host_y = [torch.empty(y_off[-1], dtype=torch.float16).pin_memory() for _ in range(2)]
        dev_y = [torch.empty(y_off[-1], dtype=torch.float16, device="cuda") for _ in range(2)]
        views = [[(u, dev_x[b][x_off[i]:x_off[i + 1]].view(u["M"], u["K"]),
                   dev_y[b][y_off[i]:y_off[i + 1]].view(u["M"], u["N"])) for i, u in enumerate(units)]
                 for b in range(2)]
        comp, h2d, d2h = torch.cuda.current_stream(), torch.cuda.Stream(), torch.cuda.Stream()
        h2d_done = [torch.cuda.Event() for _ in range(2)]
        comp_done = [torch.cuda.Event() for _ in range(2)]
        d2h_done = [torch.cuda.Event() for _ in range(2)]
        for b in range(2):
            comp_done[b].record(comp)
            d2h_done[b].record(comp)

        def e2e_step(i):
            b = i % 2
            h2d.wait_event(comp_done[b])              # buffer set b is free (step i - 2 computed)
            with torch.cuda.stream(h2d):
                dev_x[b].copy_(host_x, non_blocking=True)
                h2d_done[b].record(h2d)
            comp.wait_event(h2d_done[b])
            comp.wait_event(d2h_done[b])              # step i - 2's outputs have left dev_y[b]
            for u, xv, yv in views[b]:
                w4a16_opt.w4a16_gemm_out(u["Wp"], xv, u["s"], yv, weights_resident=True)
            comp_done[b].record(comp)
            d2h.wait_event(comp_done[b])
            with torch.cuda.stream(d2h):
                host_y[b].copy_(dev_y[b], non_blocking=True)
                d2h_done[b].record(d2h)
            if i > 0:
                d2h_done[(i - 1) % 2].synchronize()  # the previous step's result is on the host

        e2e_steps = max(3, min(args.steps, 2000))
        for i in range(max(3, min(args.warmup, 50))):
            e2e_step(i)
        d2h_done[0].synchronize()
        d2h_done[1].synchronize()
        t0 = time.perf_counter()
        for i in range(e2e_steps):
            e2e_step(i)
        d2h_done[(e2e_steps - 1) % 2].synchronize()
        e2e_s = time.perf_counter() - t0
        e2e = {"value": round(step_bytes * e2e_steps / e2e_s / 1e9, 2), "unit": "GB/s",
               "h2d_bytes_per_step": in_bytes, "d2h_bytes_per_step": out_bytes, "steps": e2e_steps,
               "ms_per_step": round(e2e_s * 1e3 / e2e_steps, 4),
               "api": "w4a16_opt.w4a16_gemm_out(weights_resident=True), eager, current stream; per step one "
                      "H2D copy of its activations and one D2H copy of its outputs on copy streams, "
                      "overlapping the neighbouring steps' GEMMs; each step's result waited for one step later"}
        # host cost of one eager call (Python + binding + C ABI + launch): bursts of 200 calls
        # from an idle GPU, short enough that the launch queue never fills (a full queue would
        # make the host wait for the GPU); median over bursts
        u0 = units[0]
        for _ in range(200):
            w4a16_opt.w4a16_gemm_out(u0["Wp"], u0["x"], u0["s"], u0["y"], weights_resident=True)
        torch.cuda.synchronize()
        bursts = []
        for _ in range(15):
            t0 = time.perf_counter()
            for _ in range(200):
                w4a16_opt.w4a16_gemm_out(u0["Wp"], u0["x"], u0["s"], u0["y"], weights_resident=True)
            bursts.append((time.perf_counter() - t0) / 200 * 1e6)
            torch.cuda.synchronize()
        host_us = round(sorted(bursts)[len(bursts) // 2], 2)
        torch.cuda.synchronize()
        del host_x, dev_x, host_y, dev_y, views, h2d, d2h

    peaks, peak_kind = load_peaks()
    traffic = profile_traffic("decode_sweep_traffic")
    roofline = {"bound": "hbm", "kernel": "w4a16::decode_kernel", "achieved": round(value / world, 1),
                "peak": peaks["hbm_gbs"], "unit": "GB/s", "frac": round(value / world / peaks["hbm_gbs"], 4),
                "peak_source": f"hbm_gbs ({peak_kind})",
                "traffic": None if traffic is None else traffic.get("decode_kernel_dram_bytes_per_step"),
                "algorithmic_bytes_per_step": step_bytes,
                "timing": "CUDA events around the step graph's replays: every GEMM of the step is one "
                          "decode_kernel launch, so this is the kernel time including the gaps between launches"}
    if world > 1:
        roofline["note"] = "per GPU: every rank streams its own sweep"

    # ---- prefill per shape, N = 1: one CUDA graph per (M, N, K, G) over distinct
    # weight copies (>= 256 MB of weights per graph, twice the L2)
    prefill = None
    if world == 1 and not args.no_prefill:
        rows, tot_flops, tot_ms = [], 0.0, 0.0
        for (N, K) in PREFILL_SHAPES:
            for G in PREFILL_G:
                for M in PREFILL_M:
                    x, q, s, Wp = make_inputs(M, N, K, G, seed, "cuda")
                    seed += 1
                    copies = max(2, -(-(256 << 20) // (Wp.numel() * 4)))
                    ws_list = [(Wp, s)] + [(Wp.clone(), s.clone()) for _ in range(copies - 1)]
                    y = torch.empty(M, N, dtype=torch.float16, device="cuda")

                    def pstep(ws_list=ws_list, x=x, y=y):
                        for w, sc in ws_list:
                            w4a16_opt.w4a16_gemm_out(w, x, sc, y, weights_resident=True)

                    reps = max(2, args.prefill_steps // 8)
                    pms = graph_time_ms(pstep, reps, 2, world) / (reps * copies)
                    flops = 2.0 * M * N * K
                    tf = flops / (pms / 1e3) / 1e12
                    route = w4a16_opt.query_route(M, N, K, K // G)
                    rows.append({"M": M, "N": N, "K": K, "G": G, "us": round(pms * 1e3, 2), "tflops": round(tf, 1),
                                 "frac": round(tf / peaks["bf16_tflops"], 4),
                                 "hbm_gbs": round(alg_bytes(M, N, K, G) / (pms / 1e3) / 1e9, 1),
                                 "tok_tile": route["tile_m"], "grid": route["grid"]})
                    tot_flops += flops
                    tot_ms += pms
                    del ws_list, x, q, s, Wp, y
                    torch.cuda.empty_cache()
        tflops = tot_flops / (tot_ms / 1e3) / 1e12
        prefill = {"workload": "configs[2]: M in {128,512,2048,8192} x (14336x4096, 4096x14336) x G in {64,128}",
                   "value": round(tflops, 1), "unit": "TFLOP/s", "ms_per_pass": round(tot_ms, 4),
                   "timing": "per shape: CUDA graph over distinct weight copies (>= 256 MB), mean per call",
                   "roofline": {"bound": "tensor", "kernel": "w4a16::prefill_kernel", "achieved": round(tflops, 1),
                                "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                                "frac": round(tflops / peaks["bf16_tflops"], 4),
                                "peak_source": f"bf16_tflops burst ({peak_kind}; dense fp16 = bf16 rate)",
                                "frac_of_sustained": round(tflops / peaks["bf16_tflops_sustained"], 4)},
                   "per_shape": rows}

    # ---- baselines (rank 0, N = 1): the reference's CPU path on the host cores, and the
    # reference's own CUDA extension rebuilt for sm_100a on this GPU, same inputs and method
    cpu, gpu_ref = None, None
    if world == 1 and rank == 0 and not args.no_cpu_baseline:
        cunits = [(u["x"].cpu(), u["q"], u["s"].cpu(), DECODE_G) for u in units]
        threads = os.cpu_count() or 1
        secs = cpu_reference_pass(cunits, threads)
        cpu = {"value": round(step_bytes / secs / 1e9, 3), "unit": "GB/s", "cores": threads, "kind": "port",
               "seconds": round(secs, 2),
               "sample": "one pass over the 16 GEMMs of the decode sweep (fp16 dequant + fp32 matmul, torch CPU)"}
    if world == 1 and rank == 0 and not args.no_gpu_reference:
        gpu_ref = gpu_reference_baseline(units, step_bytes, value, prefill, args)

    # ---- Llama-3-70B tensor-parallel projections over the N ranks (N = 1 included)
    tp70b = None if args.no_tp else run_tp70b(world, rank, args, peaks, peak_kind)

    if world > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return 0
    config = bench_config(world)
    config.update(timing="CUDA graph of one step, K replays between CUDA events, max over ranks",
                  weights_resident=True)
    out = {
        "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms_step, 5), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f16",
        "data": "synthetic (seeded: x~N(0,1) fp16, q~U{0..15}, scales~U[0.002,0.02] fp16)",
        "config": config, "default_mode": default_mode, "fp32_scale_mode": fp32_scale_mode,
        "e2e": e2e, "host_us_per_call": host_us, "roofline": roofline, "prefill": prefill, "cpu_baseline": cpu,
        "gpu_reference": gpu_ref, "tp70b": tp70b, "clocks": clocks.summary(),
        "gpu_launches": launches_per_step * args.steps,
    }
    print(json.dumps(out), flush=True)
    return 0


TP70B = (("gate/up", "col", 28672, 8192), ("down", "row", 8192, 28672))
TP70B_DECODE_M = (1, 16)
TP70B_PREFILL_M = 4096


def run_tp70b(world, rank, args, peaks, peak_kind):
    """Llama-3-70B gate/up (28672 x 8192, split along N: each rank's
    columns, then an all-gather of y) and down (8192 x 28672, split along K: each rank's fp32
    partial, then an all-reduce and one cast), G = 128, at M in {1, 16} (GB/s of the full,
    unsharded GEMMs) and M = 4096 (TFLOP/s).  Total work is fixed as N grows (strong
    scaling); times are the max over ranks.  The sharded GEMMs are also timed alone, so the
    collectives' share of each step is reported."""
    import w4a16_opt
    from w4a16_opt import tp
    G = DECODE_G

    def build(Ms, seed):
        ops, nbytes, flops = [], 0, 0
        for M in Ms:
            for name, kind, N, K in TP70B:
                x, q, s, Wp = make_inputs(M, N, K, G, seed, "cuda")
                seed += 1
                del q
                op = {"M": M, "kind": kind}
                if world == 1:
                    op.update(Wp=Wp, x=x, s=s, y=torch.empty(M, N, dtype=torch.float16, device="cuda"))
                elif kind == "col":
                    layer = tp.ColumnParallelW4A16(Wp, s, N, K)
                    op.update(layer=layer, x=x, y_local=torch.empty(M, N // world, dtype=torch.float16, device="cuda"),
                              y=torch.empty(M, N, dtype=torch.float16, device="cuda"))
                else:
                    layer = tp.RowParallelW4A16(Wp, s, N, K)
                    op.update(layer=layer, x_local=layer.x_slice(x),
                              part=torch.empty(M, N, dtype=torch.float32, device="cuda"),
                              y=torch.empty(M, N, dtype=torch.float16, device="cuda"))
                if world > 1:
                    del Wp, s
                ops.append(op)
                nbytes += alg_bytes(M, N, K, G)
                flops += 2 * M * N * K
        torch.cuda.synchronize()
        return ops, nbytes, flops

    def full_step(ops):
        def step():
            for op in ops:
                if world == 1:
                    w4a16_opt.w4a16_gemm_out(op["Wp"], op["x"], op["s"], op["y"], weights_resident=True)
                elif op["kind"] == "col":
                    op["layer"].local(op["x"], out=op["y_local"])
                    op["layer"].gather(op["y_local"], out=op["y"])
                else:
                    op["layer"].partial(op["x_local"], out=op["part"])
                    op["layer"].reduce(op["part"], out=op["y"])
        return step

    def fused_step(ops):
        def step():
            for op in ops:
                if op["kind"] == "col":
                    op["y"] = op["layer"].fused(op["x"])
                else:
                    op["y"] = op["layer"].fused(op["x_local"])
        return step

    def gemm_step(ops):
        def step():
            for op in ops:
                if world == 1:
                    w4a16_opt.w4a16_gemm_out(op["Wp"], op["x"], op["s"], op["y"], weights_resident=True)
                elif op["kind"] == "col":
                    op["layer"].local(op["x"], out=op["y_local"])
                else:
                    op["layer"].partial(op["x_local"], out=op["part"])
        return step

    out = {"workload": "configs[4]: Llama-3-70B gate/up 28672x8192 (column split + all-gather of y) and down "
                       "8192x28672 (row split + fp32 all-reduce + cast), G=128",
           "tp": world, "scaling": "strong",
           "collectives": "none (one GPU)" if world == 1 else "NCCL all_gather_into_tensor / all_reduce (fp32)"}
    # the peer-memory exchange (one buffer per rank, mapped by all; the library's exchange
    # kernel instead of NCCL), sized for the largest step
    ex = None
    if world > 1:
        Ms = TP70B_DECODE_M + (() if args.no_prefill else (TP70B_PREFILL_M,))
        src_bytes = max(max(M * (N // world) * 2, M * N * 4) for M in Ms for _, _, N, _ in TP70B)
        y_bytes = max(M * N * 2 for M in Ms for _, _, N, _ in TP70B)
        ex = tp.PeerExchange(src_bytes, y_bytes)

    def with_fused(ops, steps, warmup, unit_value):
        if ex is None:
            return None
        for op in ops:
            op["layer"].exchange = ex
        fms = graph_time_ms(fused_step(ops), steps, warmup, world) / steps
        return {"value": round(unit_value(fms), 1), "ms_per_step": round(fms, 5),
                "exchange": "peer-memory exchange kernel (w4a16_tp_allgather / w4a16_tp_allreduce) over NVLink"}

    ops, nbytes, _ = build(TP70B_DECODE_M, 7000)
    steps = max(20, min(args.steps, 2000))
    ms = graph_time_ms(full_step(ops), steps, args.warmup, world) / steps
    gms = graph_time_ms(gemm_step(ops), steps, args.warmup, world) / steps
    gbs = nbytes / (ms / 1e3) / 1e9
    out["decode"] = {"M": list(TP70B_DECODE_M), "value": round(gbs, 1), "unit": "GB/s", "ms_per_step": round(ms, 5),
                     "gemm_only_ms": round(gms, 5), "collective_share": round(max(0.0, 1 - gms / ms), 3),
                     "frac_of_hbm_per_gpu": round(gbs / world / peaks["hbm_gbs"], 4),
                     "fused": with_fused(ops, steps, args.warmup, lambda t: nbytes / (t / 1e3) / 1e9)}
    del ops
    torch.cuda.empty_cache()
    if not args.no_prefill:
        ops, _, flops = build((TP70B_PREFILL_M,), 8000)
        psteps = 5
        ms = graph_time_ms(full_step(ops), psteps, 2, world) / psteps
        gms = graph_time_ms(gemm_step(ops), psteps, 2, world) / psteps
        tf = flops / (ms / 1e3) / 1e12
        out["prefill"] = {"M": TP70B_PREFILL_M, "value": round(tf, 1), "unit": "TFLOP/s", "ms_per_step": round(ms, 4),
                          "gemm_only_ms": round(gms, 4), "collective_share": round(max(0.0, 1 - gms / ms), 3),
                          "frac_of_tensor_peak_per_gpu": round(tf / world / peaks["bf16_tflops"], 4),
                          "peak_source": f"bf16_tflops burst ({peak_kind})",
                          "fused": with_fused(ops, psteps, 2, lambda t: flops / (t / 1e3) / 1e12)}
        del ops
        torch.cuda.empty_cache()
    if ex is not None:
        ex.close()
    return out


def gpu_reference_baseline(units, step_bytes, value, prefill, args):
    """The reference's own CUDA extension (src/vectorized: mma.sync decode and prefill kernels),
    compiled for sm_100a into the checker module oracle/_ref, timed on the same decode sweep
    and configs[2] shapes with the same CUDA-graph method: a baseline, never the product."""
    from oracle import build_ref
    ref = build_ref.load()
    if ref is None:
        return {"unavailable": "oracle/_ref/w4a16_ref not built on this machine"}

    def dstep():
        for u in units:
            ref.w4a16_gemm(u["Wp"], u["x"], u["s"], -1)

    steps = max(20, min(args.steps, 2000))
    ms = graph_time_ms(dstep, steps, 3, 1)
    ref_gbs = step_bytes * steps / (ms / 1e3) / 1e9
    out = {"impl": "reference src/vectorized built for sm_100a (oracle/_ref)", "value": round(ref_gbs, 2),
           "unit": "GB/s", "ms_per_step": round(ms / steps, 5), "speedup": round(value / ref_gbs, 3),
           "workload": "same decode sweep step (16 GEMMs, same inputs), CUDA graph replays"}
    if prefill is not None:
        rows, tot_flops, tot_ms = [], 0.0, 0.0
        seed = 5000
        for (N, K) in PREFILL_SHAPES:
            for G in PREFILL_G:
                for M in PREFILL_M:
                    x, q, s, Wp = make_inputs(M, N, K, G, seed, "cuda")
                    seed += 1
                    copies = max(2, -(-(256 << 20) // (Wp.numel() * 4)))
                    ws_list = [(Wp, s)] + [(Wp.clone(), s.clone()) for _ in range(copies - 1)]

                    def pstep(ws_list=ws_list, x=x):
                        for w, sc in ws_list:
                            ref.w4a16_gemm(w, x, sc, -1)

                    pms = graph_time_ms(pstep, 2, 1, 1) / (2 * copies)
                    rows.append({"M": M, "N": N, "K": K, "G": G, "us": round(pms * 1e3, 2),
                                 "tflops": round(2.0 * M * N * K / (pms / 1e3) / 1e12, 1)})
                    tot_flops += 2.0 * M * N * K
                    tot_ms += pms
                    del ws_list, x, q, s, Wp
                    torch.cuda.empty_cache()
        ref_tf = tot_flops / (tot_ms / 1e3) / 1e12
        out["prefill"] = {"value": round(ref_tf, 1), "unit": "TFLOP/s", "speedup": round(prefill["value"] / ref_tf, 3),
                          "per_shape": rows}
    return out


# ---------------------------------------------------------------------------------------------- reference

def run_reference(args):
    """The reference's CPU implementation of the path (its tests/quant.py dequant + torch
    matmul, restated in oracle/cpu_reference.py) on this host's cores; rank 0 only.

    A step is one pass over the 16 GEMMs of the decode sweep, as in the GPU arm.  When the
    requested steps would run past about two minutes, each step covers the same leading
    fraction of every GEMM's output columns instead (a bounded sample of the same work)."""
    world, rank, _ = dist_env()
    if rank != 0:
        return 0
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    from oracle import cpu_reference
    units, seed = [], 1000
    for name, N, K in DECODE_SHAPES:
        for M in DECODE_M:
            x, q, s, _ = make_inputs(M, N, K, DECODE_G, seed, "cpu")
            seed += 1
            units.append((x, q, s, M, N, K))

    def one_pass(frac):
        nbytes = 0
        for x, q, s, M, N, K in units:
            n = N if frac >= 1.0 else max(16, int(N * frac) // 16 * 16)
            cpu_reference.ref_gemm(x, q[:n], s[:, :n], DECODE_G)
            nbytes += alg_bytes(M, n, K, DECODE_G)
        return nbytes

    t0 = time.perf_counter()
    one_pass(1.0)
    t_pass = time.perf_counter() - t0
    frac = min(1.0, 120.0 / max(1e-9, t_pass * (args.steps + args.warmup)))
    for _ in range(max(0, args.warmup - 1)):
        one_pass(frac)
    total, t0 = 0, time.perf_counter()
    for _ in range(args.steps):
        total += one_pass(frac)
    secs = time.perf_counter() - t0
    value = total / secs / 1e9
    sample = ("each step: one pass over the 16 GEMMs of the decode sweep" if frac >= 1.0 else
              f"each step: the leading {frac:.3f} of every GEMM's output columns, for the 16 GEMMs of the sweep") + \
        " (fp16 dequant + fp32 matmul, torch CPU)"
    out = {"impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": "GB/s", "n_gpus": world,
           "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(secs * 1e3 / args.steps, 3),
           "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f16",
           "data": "synthetic (seeded, same inputs as the GPU arm)",
           "config": bench_config(world),
           "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": threads, "kind": "port",
                            "sample": sample},
           "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(out), flush=True)
    return 0


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None)
    ap.add_argument("--warmup", type=int, default=None)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--prefill-steps", type=int, default=40)
    ap.add_argument("--no-prefill", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-gpu-reference", action="store_true")
    ap.add_argument("--no-tp", action="store_true", help="skip the configs[4] tensor-parallel block")
    args = ap.parse_args()
    if args.impl == "reference":
        args.steps = 16 if args.steps is None else args.steps
        args.warmup = 3 if args.warmup is None else args.warmup
        return run_reference(args)
    args.steps = 20000 if args.steps is None else args.steps
    args.warmup = 200 if args.warmup is None else args.warmup
    if args.warmup < 3:
        args.warmup = 3
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if args.gpus != world:
        print(f"bench.py: --gpus {args.gpus} but WORLD_SIZE={world}; launch N>1 with torchrun", file=sys.stderr)
        if world == 1 and args.gpus > 1:
            return 2
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
