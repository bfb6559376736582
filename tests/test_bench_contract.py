"""bench.py's reference arm on the CPU: one JSON line with the keys the driver reads, on the
same metric and config as the GPU arm, with none of this package's code loaded; under a
multi-rank launch only rank 0 prints."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _run(env_extra):
    env = dict(os.environ, **env_extra)
    return subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference",
                           "--steps", "3", "--warmup", "3"],
                          cwd=ROOT, env=env, capture_output=True, text=True, timeout=600)


def test_reference_arm_line():
    r = _run({"WORLD_SIZE": "1", "RANK": "0", "LOCAL_RANK": "0"})
    assert r.returncode == 0, r.stderr
    lines = [ln for ln in r.stdout.splitlines() if ln.strip()]
    assert len(lines) == 1, r.stdout
    d = json.loads(lines[0])
    with open(os.path.join(ROOT, "BASELINE.json"), encoding="utf-8") as f:
        metric = json.load(f)["metric"]
    assert d["impl"] == "reference" and d["metric"] == metric and d["unit"] == "GB/s"
    assert d["value"] > 0 and d["higher_is_better"] is True
    assert (d["n_gpus"], d["steps"], d["warmup"]) == (1, 3, 3)
    assert d["ms_per_step"] > 0 and d["vs_baseline"] is None and "workload" in d["config"]
    cb = d["cpu_baseline"]
    assert cb["value"] == d["value"] and cb["kind"] in ("port", "reference") and cb["cores"] >= 1 and cb["sample"]
    assert d["e2e"] == {"value": d["value"], "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


# Runs the reference arm in-process and reports whether any module or shared library of this
# package was loaded (the reference arm must time the reference's path alone).
PROBE = r"""
import json, runpy, sys
sys.argv = ["bench.py", "--impl", "reference", "--steps", "2", "--warmup", "3"]
try:
    runpy.run_path(BENCH, run_name="__main__")
except SystemExit:
    pass
mods = sorted(m for m in sys.modules if m.split(".")[0] == "w4a16_opt")
libs = sorted({ln.split()[-1] for ln in open("/proc/self/maps") if "w4a16" in ln and ".so" in ln})
print(json.dumps({"modules": mods, "libs": libs}))
"""


def test_reference_arm_loads_nothing_of_this_package():
    env = dict(os.environ, WORLD_SIZE="1", RANK="0", LOCAL_RANK="0")
    code = PROBE.replace("BENCH", repr(os.path.join(ROOT, "bench.py")))
    r = subprocess.run([sys.executable, "-c", code], cwd=ROOT,
                       env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr
    lines = [json.loads(ln) for ln in r.stdout.splitlines() if ln.startswith("{")]
    line, probe = lines[0], lines[-1]
    assert probe == {"modules": [], "libs": []}, probe
    # the same config dict as the GPU arm, so the driver compares like with like
    sys.path.insert(0, ROOT)
    import bench
    assert line["config"] == bench.bench_config(1)


def test_reference_arm_other_ranks_exit_quietly():
    r = _run({"WORLD_SIZE": "2", "RANK": "1", "LOCAL_RANK": "1"})
    assert r.returncode == 0, r.stderr
    assert r.stdout.strip() == ""
