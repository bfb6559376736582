"""The per-shape benchmark's options and result document against the reference's
benchmarks/bench_gemm.py (options 189-204, rows 296-301, document 307-331, table 333-344).

CPU cases drive ``run`` with a stand-in timer and router, so the document is checked
without a device; the GPU case runs the real CUDA-graph timing on one small shape.
"""
import json
import math

import pytest
import torch

from w4a16_opt import gemm_benchmark as gb

# Keys the reference writes (bench_gemm.py:296-301, 307-331).
REF_ROW_KEYS = {"mode", "layer", "N", "K", "M", "G", "cuda_us", "cuda_min_us", "cuda_tflops"}
REF_TOP_KEYS = {"generated_at", "gpu", "torch", "cuda_runtime", "triton", "parameters",
                "python_executable", "rows", "plot"}
REF_PARAM_KEYS = {"group_size", "target_weight_mib", "repetitions", "shapes", "phase_M", "marlin",
                  "marlin_version", "backends", "timing"}


def test_default_shapes_are_llama3_8b():
    shapes = gb.resolve_shapes(None)
    assert shapes == [("qkv", (6144, 4096)), ("o", (4096, 4096)), ("gate_up", (28672, 4096)),
                      ("down", (4096, 14336))]
    assert gb.resolve_shapes(["1024,4096", "64,512"]) == [("1024x4096", (1024, 4096)), ("64x512", (64, 512))]


def test_phase_m_selection():
    assert gb.resolve_phase_m("both", "128,512,128", "1,2", None) == {"prefill": [128, 512], "decode": [1, 2]}
    assert gb.resolve_phase_m("decode", "128", "4,1,4", None) == {"decode": [4, 1]}
    assert gb.resolve_phase_m("both", "128", "1", "7,9") == {"prefill": [7, 9], "decode": [7, 9]}
    with pytest.raises(ValueError, match="positive"):
        gb.resolve_phase_m("prefill", "0,128", "1", None)


def test_defaults_match_reference_options():
    a = gb.parse_args([])
    assert (a.phase, a.prefill_M, a.decode_M, a.M, a.G, a.reps) == (
        "both", "128,512,1024,2048,4096,8192", "1,2,4,8,16,32", None, 128, 30)
    # larger than the reference's 128 MiB: B200's L2 holds 126 MB
    assert a.target_mb * 2**20 >= 4 * 126e6


def test_copies_and_units():
    assert gb.copies_for(8 * 2**20, 512) == 64
    assert gb.copies_for(64 * 2**20, 512) == 8
    assert gb.copies_for(2**40, 512) == 1
    # 4096 x 4096, M = 1, G = 128: codes 8 MiB + scales 256 KiB + x 8 KiB + y 8 KiB
    assert gb.algorithmic_bytes(1, 4096, 4096, 128) == 8_667_136
    assert math.isclose(gb.tflops(2048, 14336, 4096, 1e6), 2 * 2048 * 14336 * 4096 / 1e12)


def _fake_run(shapes, phase_m, G=64):
    seen = []

    def timer(calls, reps):
        seen.append((len(calls), reps))
        return 10.0 + len(seen), 9.0

    def route(M, N, K, G):
        return "decode" if M <= 16 else "prefill/64"

    rows = gb.run(shapes, phase_m, G, target_mib=1, reps=5, device="cpu", timer=timer, route=route,
                  log=lambda *_: None)
    return rows, seen


def test_rows_match_reference_schema():
    shapes = [("a", (64, 256)), ("b", (32, 128))]
    rows, seen = _fake_run(shapes, {"prefill": [128], "decode": [1, 16]})
    assert [(r["layer"], r["mode"], r["M"]) for r in rows] == [
        ("a", "prefill", 128), ("a", "decode", 1), ("a", "decode", 16),
        ("b", "prefill", 128), ("b", "decode", 1), ("b", "decode", 16)]
    for r in rows:
        assert REF_ROW_KEYS <= set(r) and set(r) - REF_ROW_KEYS == {"cuda_gbs", "route"}
        assert r["cuda_tflops"] == pytest.approx(gb.tflops(r["M"], r["N"], r["K"], r["cuda_us"]))
        assert r["cuda_gbs"] == pytest.approx(gb.algorithmic_bytes(r["M"], r["N"], r["K"], 64) / (r["cuda_us"] * 1e3))
    # one call per distinct weight copy: 1 MiB working set / (64*256/2 + 2*64*4) bytes
    per_copy = 64 * 256 // 2 + 2 * 64 * (256 // 64)
    assert seen[0] == (gb.copies_for(per_copy, 1), 5)


def test_document_matches_reference_schema():
    shapes = [("a", (64, 256))]
    phase_m = {"decode": [1]}
    rows, _ = _fake_run(shapes, phase_m)
    doc = gb.document(shapes, phase_m, 64, 1, 5, rows, {"name": "test", "sms": 148, "l2_bytes": None})
    assert REF_TOP_KEYS <= set(doc) and set(doc) - REF_TOP_KEYS == {"device"}
    assert set(doc["parameters"]) == REF_PARAM_KEYS
    assert doc["parameters"]["backends"] == ["CUDA W4A16"]
    assert doc["parameters"]["shapes"] == [{"name": "a", "N": 64, "K": 256}]
    assert json.loads(json.dumps(doc)) == doc


def test_tables():
    rows, _ = _fake_run([("a", (64, 256))], {"decode": [1, 4]})
    md = gb.format_table(rows, md=True).splitlines()
    assert md[0] == "| Phase | Layer | M | cuda us |" and md[1] == "|---|---|---|---|"
    assert md[2] == "| decode | a | 1 | 11.00 |"
    plain = gb.format_table(rows, md=False).splitlines()
    assert plain[0].split() == ["Phase", "Layer", "M", "cuda", "us"] and len(plain) == 3


def test_rejects_group_size():
    with pytest.raises(ValueError, match="--G"):
        gb.main(["--G", "96"])


@pytest.mark.gpu
def test_gpu_run(cuda_device, tmp_path):
    out = tmp_path / "gemm.json"
    doc = gb.main(["--shape", "1024,4096", "--decode-M", "1,16", "--prefill-M", "128",
                   "--reps", "3", "--target-mb", "64", "--json", str(out)])
    assert json.loads(out.read_text())["rows"] == doc["rows"]
    rows = doc["rows"]
    assert [(r["mode"], r["M"]) for r in rows] == [("prefill", 128), ("decode", 1), ("decode", 16)]
    assert rows[0]["route"].startswith("prefill/") and [r["route"] for r in rows[1:]] == ["decode", "decode"]
    for r in rows:
        assert math.isfinite(r["cuda_us"]) and 0 < r["cuda_min_us"] <= r["cuda_us"]
    assert doc["gpu"] == torch.cuda.get_device_name(0)
