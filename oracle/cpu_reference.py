"""The reference's CPU path for the hot path, restated with torch CPU ops --
TEST / BASELINE INFRASTRUCTURE ONLY (timed by bench.py as the CPU baseline and
the ``--impl reference`` arm; never part of the shipped GEMM).

The reference computes its expected outputs with torch on the host:
``dequantize_w4`` (tests/quant.py:77-80) followed by ``ref_gemm``
(tests/quant.py:83-85): fp16 ``(q - 8) * scale`` then an fp32 matmul.  This
module performs the same two steps with the same library so the timing is the
reference's own CPU algorithm on this machine's cores; ``tests/test_oracle.py``
checks it against the numpy oracle, which is pinned to the reference's golden
vectors.
"""
from __future__ import annotations

import torch


def dequantize_w4(q: torch.Tensor, scales: torch.Tensor, group_size: int) -> torch.Tensor:
    """fp16 [N, K] = (q - 8) * scales[k // G, n] (tests/quant.py:77-80)."""
    s = scales.t().repeat_interleave(group_size, dim=1)
    return (q.to(torch.float16) - 8) * s


def ref_gemm(x: torch.Tensor, q: torch.Tensor, scales: torch.Tensor, group_size: int) -> torch.Tensor:
    """fp32 [M, N] = x.float() @ dequantize_w4(...).float().T (tests/quant.py:83-85)."""
    return x.float() @ dequantize_w4(q, scales, group_size).float().t()
