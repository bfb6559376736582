"""Environment switches of the library, each run in a fresh process.

* W4A16_PDL=0: every kernel runs in plain stream order (no programmatic dependent
  launch).  The kernels and their summation order are the same, so outputs must be
  bit-identical to the default mode's.
* W4A16_DEBUG_PREFILL (the reference's switch) / W4A16_DEBUG_ROUTE: one stderr line per
  prefill dispatch / per call, naming the chosen kernel and tile config.
"""
import os
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
PKG = os.path.join(ROOT, "w4a16-gemm_b200")

# decode with column groups split across CTAs (+ combine kernel), decode with whole groups
# per CTA (one launch), prefill; G = 64 and 128
CASES = [(1, 4096, 4096, 128), (16, 1024, 4096, 64), (4, 256 * 148, 64, 64), (300, 1024, 2048, 64)]

SCRIPT = r"""
import sys, torch
sys.path[:0] = [{here!r}, {pkg!r}, {root!r}]
from helpers import make_workload
from w4a16_opt import w4a16_gemm
outs = []
for (M, N, K, G) in {cases!r}:
    x, q, s, Wp = make_workload(M, N, K, G, seed=M + N + K)
    outs.append(w4a16_gemm(Wp, x, s).cpu())
torch.cuda.synchronize()
torch.save(outs, sys.argv[1])
"""


def _run(path, pdl, extra_env=None):
    env = dict(os.environ)
    for k in ("W4A16_PDL", "W4A16_DEBUG_PREFILL", "W4A16_DEBUG_ROUTE"):
        env.pop(k, None)
    if not pdl:
        env["W4A16_PDL"] = "0"
    env.update(extra_env or {})
    code = SCRIPT.format(here=HERE, pkg=PKG, root=ROOT, cases=CASES)
    r = subprocess.run([sys.executable, "-c", code, str(path)], env=env, capture_output=True, text=True,
                       timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    return torch.load(str(path)), r.stderr


def test_pdl_off_matches_default(cuda_device, tmp_path):
    on, _ = _run(tmp_path / "on.pt", True)
    off, _ = _run(tmp_path / "off.pt", False)
    assert len(on) == len(off) == len(CASES)
    for (M, N, K, G), a, b in zip(CASES, on, off):
        assert a.shape == (M, N) and torch.isfinite(a.float()).all()
        assert torch.equal(a, b), (M, N, K, G)


def test_debug_route_trace(cuda_device, tmp_path):
    _, err = _run(tmp_path / "p.pt", True, {"W4A16_DEBUG_PREFILL": "1"})
    lines = [ln for ln in err.splitlines() if ln.startswith("w4a16 ")]
    assert len(lines) == 1 and lines[0].startswith("w4a16 prefill dispatch G=64 M=300 N=1024 K=2048 cfg=")
    assert " tok=" in lines[0] and " grid=" in lines[0]
    outs, err = _run(tmp_path / "r.pt", True, {"W4A16_DEBUG_ROUTE": "1"})
    lines = [ln for ln in err.splitlines() if ln.startswith("w4a16 ")]
    assert [ln.split()[1] for ln in lines] == ["decode", "decode", "decode", "prefill"]
    assert lines[0].startswith("w4a16 decode G=128 M=1 N=4096 K=4096 ")
    assert lines[2].endswith("launches=1") and lines[0].endswith("launches=2")
