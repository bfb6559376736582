"""Same-box speed against the reference's own extension rebuilt for sm_100a.

The reference's CUDA extension (src/vectorized, mma.sync kernels) is compiled for sm_100a
into oracle/_ref as a checker module.  This measurement times it and this package on the
same B200, inputs and method: BASELINE configs[1] (decode sweep) and configs[2]
(prefill).  The method is one CUDA graph over distinct weight copies of at least
512 MiB, over 4x the 126 MB L2, taking the median per call (the reference benchmark's
method, benchmarks/bench_gemm.py:36-60).

It is a measurement, so it runs only on request:
    W4A16_SAME_BOX=1 [W4A16_SAME_BOX_OUT=out.json] python -m pytest tests/test_same_box_speed_gpu.py -m gpu -s
It prints one row per GEMM (and writes them as JSON when asked).  The only checks are
that both implementations agree on each workload and that every timing is positive.
"""
import json
import os

import pytest
import torch

from helpers import assert_close, make_workload

pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(os.environ.get("W4A16_SAME_BOX") != "1", reason="measurement; set W4A16_SAME_BOX=1"),
]

DECODE = [(M, N, K, 128) for N, K in ((4096, 4096), (1024, 4096), (14336, 4096), (4096, 14336))
          for M in (1, 4, 8, 16)]
PREFILL = [(M, N, K, G) for G in (64, 128) for N, K in ((14336, 4096), (4096, 14336))
           for M in (128, 512, 2048, 8192)]
WORKING_SET_MIB = 512


def _time_both(ref, M, N, K, G, reps):
    from w4a16_opt import gemm_benchmark as gb
    from w4a16_opt import w4a16_gemm
    x, q, s, Wp = make_workload(M, N, K, G, seed=M + N + K + G)
    y_ours = w4a16_gemm(Wp, x, s)
    y_ref = ref.w4a16_gemm(Wp, x, s, -1)
    torch.cuda.synchronize()
    assert_close(y_ours, y_ref.float().cpu().numpy())
    count = gb.copies_for(Wp.numel() * 4 + s.numel() * 2, WORKING_SET_MIB)
    weights = [(Wp, s)] + [(Wp.clone(), s.clone()) for _ in range(count - 1)]
    ours_calls = [lambda w=w, sc=sc: w4a16_gemm(w, x, sc) for w, sc in weights]
    ref_calls = [lambda w=w, sc=sc: ref.w4a16_gemm(w, x, sc, -1) for w, sc in weights]
    ours_us, _ = gb.graph_time_us(ours_calls, reps)
    ref_us, _ = gb.graph_time_us(ref_calls, reps)
    return ours_us, ref_us


@pytest.fixture(scope="module")
def ref():
    from oracle import build_ref
    mod = build_ref.load()
    if mod is None:
        pytest.skip("reference checker module oracle/_ref/w4a16_ref not built")
    return mod


def test_same_box_speed(ref, cuda_device):
    from w4a16_opt import gemm_benchmark as gb
    rows = []
    for phase, cases, reps in (("decode", DECODE, 20), ("prefill", PREFILL, 5)):
        for M, N, K, G in cases:
            ours_us, ref_us = _time_both(ref, M, N, K, G, reps)
            assert ours_us > 0 and ref_us > 0
            row = {"phase": phase, "M": M, "N": N, "K": K, "G": G, "ours_us": ours_us, "ref_us": ref_us,
                   "speedup": ref_us / ours_us}
            if phase == "decode":
                b = gb.algorithmic_bytes(M, N, K, G)
                row.update(ours_gbs=b / (ours_us * 1e3), ref_gbs=b / (ref_us * 1e3))
            else:
                row.update(ours_tflops=gb.tflops(M, N, K, ours_us), ref_tflops=gb.tflops(M, N, K, ref_us))
            rows.append(row)
            torch.cuda.empty_cache()
    for phase in ("decode", "prefill"):
        sel = [r for r in rows if r["phase"] == phase]
        ours_t, ref_t = sum(r["ours_us"] for r in sel), sum(r["ref_us"] for r in sel)
        print(f"{phase}: {len(sel)} GEMMs, ours {ours_t:.1f} us, reference {ref_t:.1f} us, "
              f"speed-up {ref_t / ours_t:.2f}x")
        for r in sel:
            unit = ("GB/s", "ours_gbs", "ref_gbs") if phase == "decode" else ("TFLOP/s", "ours_tflops", "ref_tflops")
            print(f"  M={r['M']:5d} N={r['N']:5d} K={r['K']:5d} G={r['G']:3d}  ours {r['ours_us']:9.2f} us "
                  f"({r[unit[1]]:8.1f} {unit[0]})  ref {r['ref_us']:9.2f} us ({r[unit[2]]:8.1f} {unit[0]})  "
                  f"x{r['speedup']:.2f}")
    out = os.environ.get("W4A16_SAME_BOX_OUT")
    if out:
        with open(out, "w", encoding="utf-8") as f:
            json.dump({"gpu": torch.cuda.get_device_name(0), "working_set_mib": WORKING_SET_MIB,
                       "timing": "CUDA graph over distinct weight copies, median per call", "rows": rows}, f,
                      indent=1)
