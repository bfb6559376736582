"""Shared test helpers: seeded problems and the tolerance checks.

``make_problem`` follows the reference's test generator (tests/test_w4a16.py:33-38:
W ~ N(0, 1) * 0.02 quantised with RTN); ``make_workload`` follows the
BASELINE draw order (x ~ N(0,1) fp16, q ~ U{0..15}, scales ~ U[0.002, 0.02]).
Both draw on the CPU from a seeded torch.Generator, so inputs are identical on
every machine.  The expected outputs always come from the CPU oracle.
"""
from __future__ import annotations

import functools

import numpy as np
import torch

from oracle import w4a16_oracle as oracle

GS = [64, 128]


def make_problem(M, N, K, G, seed=0, w_std=0.02, device="cuda"):
    """Returns x (fp16, device), q (uint8, CPU), scales (fp16, device), Wp (int32, device)."""
    from w4a16_opt import pack_int4, quantize_w4
    gen = torch.Generator().manual_seed(seed)
    W = torch.randn(N, K, generator=gen) * w_std
    x = torch.randn(M, K, generator=gen).half()
    q, scales = quantize_w4(W, G)
    Wp = pack_int4(q)
    return x.to(device), q, scales.to(device), Wp.to(device)


def make_workload(M, N, K, G, seed=0, device="cuda"):
    """BASELINE-config inputs: returns x, q (CPU uint8), scales, Wp (device)."""
    from w4a16_opt import pack_int4
    gen = torch.Generator().manual_seed(seed)
    x = torch.randn(M, K, generator=gen).half()
    q = torch.randint(0, 16, (N, K), generator=gen, dtype=torch.uint8)
    scales = (torch.rand(K // G, N, generator=gen) * 0.018 + 0.002).half()
    Wp = pack_int4(q.to(device) if device != "cpu" else q)
    return x.to(device), q, scales.to(device), Wp


def to_np(t):
    return t.detach().cpu().numpy()


@functools.lru_cache(maxsize=8)
def _deq_cached(key):
    q_bytes, N, K, s_bytes, G = key
    q = np.frombuffer(q_bytes, dtype=np.uint8).reshape(N, K)
    s = np.frombuffer(s_bytes, dtype=np.float16).reshape(K // G, N)
    return oracle.dequantize_w4(q, s, G).astype(np.float32)


def ref_gemm(x, q, scales, G, rows=None):
    """fp32 oracle y = x @ dequant(q, scales)^T (optionally only for the given rows)."""
    qn = to_np(q)
    sn = to_np(scales)
    Wd = _deq_cached((qn.tobytes(), qn.shape[0], qn.shape[1], sn.tobytes(), G))
    xn = to_np(x).astype(np.float32)
    if rows is not None:
        xn = xn[rows]
    return xn @ Wd.T


def assert_close(y, ref, tol=2e-3):
    """Reference criterion (tests/test_w4a16.py:41-44) plus the north-star tolerance:
    max|d| / max|ref| < tol (the reference's 2e-3, relaxed by its own tests to 4e-3 for hard
    scale ranges), and always relative Frobenius error <= 1e-3 and max|d| <= 5e-3 * max|ref|."""
    yf = to_np(y).astype(np.float32) if isinstance(y, torch.Tensor) else np.asarray(y, np.float32)
    ref = np.asarray(ref, np.float32)
    assert np.isfinite(yf).all(), "NaN/Inf in output"
    denom = float(np.abs(ref).max())
    if denom == 0.0:
        assert float(np.abs(yf).max()) == 0.0
        return
    d = np.abs(yf - ref)
    rel = float(d.max()) / denom
    assert rel < tol, f"max-abs error / max|ref| = {rel:.3e} (tol {tol:.0e})"
    fro = float(np.linalg.norm(yf - ref) / max(np.linalg.norm(ref), 1e-30))
    assert fro <= 1e-3, f"relative Frobenius error {fro:.3e}"
    assert float(d.max()) <= 5e-3 * denom, "max|d| > 5e-3 * max|y_ref|"
