"""Per-shape GEMM timings written in the reference benchmark's result schema.

    PYTHONPATH=w4a16-gemm_b200 python -m w4a16_opt.gemm_benchmark [--phase decode] [--json out.json] [--md]

Counterpart of akshay919191/W4A16-GEMM benchmarks/bench_gemm.py for the one backend this
package has.  It takes the same options (bench_gemm.py:189-204, less the Triton and Marlin
comparators, which are not on this path), times each (phase, layer, M) the same way (a
CUDA graph over distinct weight copies, median per operation; bench_gemm.py:36-56,
59-60), and writes the same document: top-level keys of bench_gemm.py:307-331 and rows
with the keys of bench_gemm.py:296-301 under the backend key ``cuda``
(``cuda_us``, ``cuda_min_us``, ``cuda_tflops``).  Its rows therefore drop into the
reference's tables next to its published ones.  Additions, which the reference's readers
ignore: ``cuda_gbs`` (algorithmic HBM bytes per second) and ``route`` (the kernel the
call ran on) in each row, and ``device`` facts at the top level.

Differences, each for B200:
* ``--target-mb`` defaults to 512 MiB rather than 128 MiB.  B200's L2 holds 126 MB, so a
  128 MiB rotation would time part of the weights out of L2.
* Weights come from this package's on-device ``quantize_pack`` of ``randn * 0.02`` rather
  than the Triton quantiser (same distribution and format; the Triton kernel is not
  part of this package).
* No chart: ``plot`` is null (matplotlib is not a dependency).
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import sys
from datetime import datetime

import torch

# Llama-3-8B projection shapes (N, K) of the reference's default sweep (bench_gemm.py:23-28).
LLAMA3_8B = {
    "qkv": (6144, 4096),
    "o": (4096, 4096),
    "gate_up": (28672, 4096),
    "down": (4096, 14336),
}
BACKEND_LABEL = "CUDA W4A16"
BACKEND_KEY = "cuda"
MAX_COPIES = 64
TIMING = ("CUDA graph median per operation; W4A16 backends use distinct packed weight copies")


def parse_args(argv=None) -> argparse.Namespace:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--shape", action="append", help="N,K (repeatable); defaults to Llama 3 8B projection shapes")
    ap.add_argument("--phase", choices=("both", "prefill", "decode"), default="both")
    ap.add_argument("--prefill-M", default="128,512,1024,2048,4096,8192", help="comma-separated prefill M values")
    ap.add_argument("--decode-M", default="1,2,4,8,16,32", help="comma-separated decode M values")
    ap.add_argument("--M", default=None, help="use these M values for every selected phase")
    ap.add_argument("--G", type=int, default=128, help="group size (64 or 128)")
    ap.add_argument("--target-mb", type=float, default=512, help="packed weight + scale working set (MiB)")
    ap.add_argument("--reps", type=int, default=30)
    ap.add_argument("--json", default=None, help="result JSON path (default: print the document)")
    ap.add_argument("--md", action="store_true", help="print a Markdown table")
    ap.add_argument("--fp32-scale", action="store_true",
                    help="decode path, M <= 8: apply scales in fp32 after the products (W4A16_FLAG_FP32_SCALE)")
    return ap.parse_args(argv)


def resolve_shapes(shape_args) -> list:
    """[(name, (N, K))]: ``--shape N,K`` values named "NxK", else the Llama-3-8B table."""
    if not shape_args:
        return list(LLAMA3_8B.items())
    out = []
    for value in shape_args:
        n, k = (int(v) for v in value.split(","))
        out.append((f"{n}x{k}", (n, k)))
    return out


def resolve_phase_m(phase: str, prefill_m: str, decode_m: str, override: str | None) -> dict:
    """{mode: [M, ...]} in selection order, duplicates dropped; every M must be >= 1."""
    phases = []
    if phase in ("both", "prefill"):
        phases.append(("prefill", prefill_m))
    if phase in ("both", "decode"):
        phases.append(("decode", decode_m))
    if override is not None:
        phases = [(mode, override) for mode, _ in phases]
    out = {mode: list(dict.fromkeys(int(v) for v in values.split(","))) for mode, values in phases}
    if any(not ms or any(m < 1 for m in ms) for ms in out.values()):
        raise ValueError("M values must be positive integers")
    return out


def copies_for(bytes_per_copy: int, target_mib: float) -> int:
    """Distinct weight copies that fill the working set (1 .. 64)."""
    return max(1, min(MAX_COPIES, math.ceil(target_mib * 2**20 / bytes_per_copy)))


def tflops(M: int, N: int, K: int, time_us: float) -> float:
    return 2 * M * N * K / (time_us * 1e6)


def algorithmic_bytes(M: int, N: int, K: int, G: int) -> int:
    """Bytes one call must move: packed codes, fp16 scales, fp16 x and fp16 y."""
    return N * K // 2 + 2 * N * (K // G) + 2 * M * K + 2 * M * N


def graph_time_us(calls, reps: int):
    """(median, min) microseconds per call: the calls captured as one CUDA graph
    (``timing.GraphStep``), each of ``reps`` replays timed on its own."""
    from .timing import GraphStep

    def step():
        for call in calls:
            call()

    g = GraphStep(step)
    g.warm(3)
    per_call = [ms * 1e3 / len(calls) for ms in g.each_ms(reps)]
    g.close()
    return statistics.median(per_call), min(per_call)


def make_weights(N: int, K: int, G: int, target_mib: float, device, seed: int = 0):
    """Distinct (Wp, scales) copies of one RTN-quantised ``randn * 0.02`` matrix."""
    from . import quantize_pack
    gen = torch.Generator(device=device).manual_seed(seed)
    w16 = torch.randn((N, K), generator=gen, device=device, dtype=torch.float16) * 0.02
    Wp, scales = quantize_pack(w16, G)
    del w16
    count = copies_for(Wp.numel() * Wp.element_size() + scales.numel() * scales.element_size(), target_mib)
    weights = [(Wp, scales)] + [(Wp.clone(), scales.clone()) for _ in range(count - 1)]
    return weights


def make_row(mode: str, layer: str, N: int, K: int, M: int, G: int, median_us: float, min_us: float,
             route: str) -> dict:
    row = {"mode": mode, "layer": layer, "N": N, "K": K, "M": M, "G": G}
    row[f"{BACKEND_KEY}_us"] = median_us
    row[f"{BACKEND_KEY}_min_us"] = min_us
    row[f"{BACKEND_KEY}_tflops"] = tflops(M, N, K, median_us)
    row[f"{BACKEND_KEY}_gbs"] = algorithmic_bytes(M, N, K, G) / (median_us * 1e3)
    row["route"] = route
    return row


def route_name(M: int, N: int, K: int, G: int) -> str:
    """"decode" or "prefill/<token tile>" for the call as routed with variant -1."""
    from . import query_route
    r = query_route(M, N, K, K // G, -1)
    return r["kernel"] if r["kernel"] == "decode" else f"prefill/{r['tile_m']}"


def run(shapes, phase_m: dict, G: int, target_mib: float, reps: int, device="cuda", timer=graph_time_us,
        route=route_name, log=print, fp32_scale: bool = False) -> list:
    """Rows for every (layer, mode, M), in the reference's loop order (layer outermost).
    ``timer(calls, reps) -> (median_us, min_us)`` and ``route(M, N, K, G) -> str`` are the
    device-side steps.  ``fp32_scale`` selects W4A16_FLAG_FP32_SCALE for every call."""
    from . import w4a16_gemm, w4a16_gemm_out
    rows = []
    for layer, (N, K) in shapes:
        weights = make_weights(N, K, G, target_mib, device)
        for mode, ms in phase_m.items():
            for M in ms:
                x = torch.randn((M, K), device=device, dtype=torch.float16)
                if fp32_scale:
                    y = torch.empty((M, N), device=device, dtype=torch.float16)
                    calls = [lambda w=w, s=s: w4a16_gemm_out(w, x, s, y, fp32_scale=True) for w, s in weights]
                else:
                    calls = [lambda w=w, s=s: w4a16_gemm(w, x, s, variant=-1) for w, s in weights]
                median_us, min_us = timer(calls, reps)
                rows.append(make_row(mode, layer, N, K, M, G, median_us, min_us, route(M, N, K, G)))
                log(f"finished {mode} {layer} M={M}")
        del weights
        if torch.cuda.is_available():
            torch.cuda.empty_cache()
    return rows


def device_facts(device=0) -> dict:
    props = torch.cuda.get_device_properties(device)
    return {"name": props.name, "sms": props.multi_processor_count,
            "l2_bytes": getattr(props, "L2_cache_size", None)}


def document(shapes, phase_m: dict, G: int, target_mib: float, reps: int, rows: list, device: dict) -> dict:
    """The result document, keyed as bench_gemm.py:307-331."""
    return {
        "generated_at": datetime.now().astimezone().isoformat(timespec="seconds"),
        "gpu": device.get("name"),
        "torch": torch.__version__,
        "cuda_runtime": torch.version.cuda,
        "triton": None,
        "parameters": {
            "group_size": G,
            "target_weight_mib": target_mib,
            "repetitions": reps,
            "shapes": [{"name": name, "N": nk[0], "K": nk[1]} for name, nk in shapes],
            "phase_M": phase_m,
            "marlin": False,
            "marlin_version": None,
            "backends": [BACKEND_LABEL] if rows else [],
            "timing": TIMING,
        },
        "python_executable": sys.executable,
        "rows": rows,
        "plot": None,
        "device": device,
    }


def format_table(rows: list, md: bool) -> str:
    """The reference's console table (bench_gemm.py:333-344): phase, layer, M, time per call."""
    headers = ["Phase", "Layer", "M", f"{BACKEND_KEY} us"]
    body = [[r["mode"], r["layer"], str(r["M"]), f"{r[f'{BACKEND_KEY}_us']:.2f}"] for r in rows]
    if md:
        lines = ["| " + " | ".join(headers) + " |", "|" + "---|" * len(headers)]
        lines += ["| " + " | ".join(v) + " |" for v in body]
    else:
        lines = ["  ".join(f"{h:>20}" for h in headers)]
        lines += ["  ".join(f"{v:>20}" for v in values) for values in body]
    return "\n".join(lines)


def main(argv=None) -> dict:
    args = parse_args(argv)
    shapes = resolve_shapes(args.shape)
    phase_m = resolve_phase_m(args.phase, args.prefill_M, args.decode_M, args.M)
    if args.G not in (64, 128):
        raise ValueError("--G must be 64 or 128")
    if not torch.cuda.is_available():
        raise RuntimeError("a CUDA device is required")
    device = device_facts()
    print(f"# {device['name']}  SMs={device['sms']}  torch={torch.__version__} cuda={torch.version.cuda}  "
          f"weight working set={args.target_mb:.0f} MiB")
    rows = run(shapes, phase_m, args.G, args.target_mb, args.reps, fp32_scale=args.fp32_scale)
    doc = document(shapes, phase_m, args.G, args.target_mb, args.reps, rows, device)
    if args.json:
        os.makedirs(os.path.dirname(os.path.abspath(args.json)), exist_ok=True)
        with open(args.json, "w", encoding="utf-8") as f:
            json.dump(doc, f, indent=2)
            f.write("\n")
    print(format_table(rows, args.md))
    if not args.json:
        print(json.dumps(doc))
    return doc


if __name__ == "__main__":
    main()
