"""Launch modes: with W4A16_PDL=0 every kernel runs in plain stream order (no
programmatic dependent launch).  The kernels and their summation order are the same,
so outputs must be bit-identical to the default mode's."""
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


def _run(path, pdl):
    env = dict(os.environ)
    env.pop("W4A16_PDL", None)
    if not pdl:
        env["W4A16_PDL"] = "0"
    code = SCRIPT.format(here=HERE, pkg=PKG, root=ROOT, cases=CASES)
    r = subprocess.run([sys.executable, "-c", code, str(path)], env=env, capture_output=True, text=True,
                       timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    return torch.load(str(path))


def test_pdl_off_matches_default(cuda_device, tmp_path):
    on = _run(tmp_path / "on.pt", True)
    off = _run(tmp_path / "off.pt", False)
    assert len(on) == len(off) == len(CASES)
    for (M, N, K, G), a, b in zip(CASES, on, off):
        assert a.shape == (M, N) and torch.isfinite(a.float()).all()
        assert torch.equal(a, b), (M, N, K, G)
