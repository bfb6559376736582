"""CPU oracle for the W4A16 GEMM hot path -- TEST INFRASTRUCTURE ONLY.

This module is the checker, never the product.  Only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline / reference arms may
import it.  The shipped GEMM path is CUDA-only and fails loudly without its
extension.

It is a numpy restatement of the reference's format and numerics, which live in
the reference repository at ``tests/quant.py`` (akshay919191/W4A16-GEMM):

* ``fragment_map``    follows tests/quant.py:10-25
* ``pack_int4``       follows tests/quant.py:34-48
* ``unpack_int4``     follows tests/quant.py:51-59
* ``quantize_w4``     follows tests/quant.py:62-74
* ``dequantize_w4``   follows tests/quant.py:77-80
* ``ref_gemm``        follows tests/quant.py:83-85
* ``kernel_word_decode`` restates the device-side ``dequant8`` bit trick
  (src/vectorized/common.cuh:45-55) lane by lane, as the reference's own
  test_pack_matches_kernel_decode does (tests/test_w4a16.py:60-78).

Parity pin: ``tests/golden/`` holds vectors produced by importing the
reference's own ``tests/quant.py`` (script: ``tests/golden/make_golden.py``);
``tests/test_oracle.py`` checks every function here against them bit for bit.

Weight format (the contract every kernel consumes):
    W[n, k] = (q[n, k] - 8) * scales[k // G, n]      q in 0..15, scales fp16 [K/G, N]
    word index = (((n/16) * (K/64) + k/64) * 32 + lane) * 4 + s,   s = (k % 64) / 16
    nibble i (bits 4i..4i+3) of a lane's word: p = i & 3, h = i >> 2,
    n = 16*nb + g + 8*(p & 1),  k = 64*kc + 16*s + 2*t + 8*(p >> 1) + h,
    g = lane >> 2, t = lane & 3.
"""
from __future__ import annotations

import numpy as np

__all__ = [
    "fragment_map", "pack_int4", "unpack_int4", "quantize_w4", "dequantize_w4",
    "ref_gemm", "ref_gemm_from_packed", "kernel_word_decode", "dequant_from_packed",
]


def fragment_map():
    """(n_idx, k_idx), each int [32, 8]: position inside one 16x16 (n x k) tile of
    nibble i of lane ``lane``'s word (tests/quant.py:10-25)."""
    lane = np.arange(32)[:, None]
    i = np.arange(8)[None, :]
    g, t = lane >> 2, lane & 3
    p, h = i & 3, i >> 2
    n_idx = g + 8 * (p & 1)
    k_idx = 2 * t + 8 * (p >> 1) + h
    return n_idx.astype(np.int64), k_idx.astype(np.int64)


def pack_int4(q: np.ndarray) -> np.ndarray:
    """uint8 codes [N, K] (0..15) -> int32 [N*K/8] in kernel word order
    (tests/quant.py:34-48)."""
    q = np.asarray(q)
    N, K = q.shape
    if N % 16 or K % 64:
        raise ValueError("N must be a multiple of 16 and K of 64")
    if q.size and (q.min() < 0 or q.max() > 15):
        raise ValueError("codes must be in 0..15")
    NB, KC = N // 16, K // 64
    n_idx, k_idx = fragment_map()
    # [NB, 16n, KC, 4s, 16k] -> [NB, KC, 4s, 16n, 16k]
    t = q.astype(np.uint8).reshape(NB, 16, KC, 4, 16).transpose(0, 2, 3, 1, 4)
    v = t[..., n_idx, k_idx].astype(np.uint32)            # [NB, KC, 4, 32 lanes, 8 nibbles]
    shifts = (np.arange(8, dtype=np.uint32) * 4)
    w = np.bitwise_or.reduce(v << shifts, axis=-1)         # disjoint bit fields
    return np.ascontiguousarray(w.transpose(0, 1, 3, 2)).reshape(-1).view(np.int32)


def unpack_int4(Wp: np.ndarray, N: int, K: int) -> np.ndarray:
    """int32 [N*K/8] -> uint8 codes [N, K] (tests/quant.py:51-59)."""
    NB, KC = N // 16, K // 64
    n_idx, k_idx = fragment_map()
    w = np.asarray(Wp).view(np.uint32).reshape(NB, KC, 32, 4).transpose(0, 1, 3, 2)  # [NB,KC,4,32]
    shifts = (np.arange(8, dtype=np.uint32) * 4)
    v = ((w[..., None] >> shifts) & 0xF).astype(np.uint8)  # [NB, KC, 4, 32, 8]
    t = np.zeros((NB, KC, 4, 16, 16), dtype=np.uint8)
    t[..., n_idx, k_idx] = v
    return t.transpose(0, 3, 1, 2, 4).reshape(N, K)


def quantize_w4(W: np.ndarray, group_size: int):
    """Symmetric RTN, absmax/7 per (n, k-group), zero point 8 (tests/quant.py:62-74).

    Returns q uint8 [N, K] and scales fp16 [K/G, N]."""
    W = np.asarray(W, dtype=np.float32)
    N, K = W.shape
    G = group_size
    if K % G:
        raise ValueError("K must be a multiple of the group size")
    Wg = W.reshape(N, K // G, G)
    s = np.maximum(np.abs(Wg).max(-1, keepdims=True) / np.float32(7), np.float32(1e-4))
    s = s.astype(np.float16).astype(np.float32)             # fp16-representable
    q = (np.clip(np.round(Wg / s), -8, 7) + 8).astype(np.uint8).reshape(N, K)
    scales = np.ascontiguousarray(s[..., 0].T).astype(np.float16)
    return q, scales


def dequantize_w4(q: np.ndarray, scales: np.ndarray, group_size: int) -> np.ndarray:
    """fp16 [N, K] = (q - 8) * scale, one fp16 rounding (tests/quant.py:77-80).

    numpy evaluates float16 * float16 in float32 and rounds to nearest-even once;
    the float32 product of two fp16 values is exact, so this equals an IEEE fp16
    multiply bit for bit."""
    s = np.repeat(np.asarray(scales, dtype=np.float16).T, group_size, axis=1)   # [N, K]
    return (np.asarray(q).astype(np.float16) - np.float16(8)) * s


def ref_gemm(x: np.ndarray, q: np.ndarray, scales: np.ndarray, group_size: int) -> np.ndarray:
    """fp32 [M, N] = x.float() @ dequantize_w4(...).float().T (tests/quant.py:83-85)."""
    Wd = dequantize_w4(q, scales, group_size).astype(np.float32)
    return np.asarray(x).astype(np.float32) @ Wd.T


def kernel_word_decode(word: int):
    """Restates the device dequant bit trick for one 32-bit word (common.cuh:45-55).

    Returns 4 pairs (lo, hi) of (q - 8) values, pair p holding nibbles p and p+4,
    computed as fp16(0x6400 | nibble) - 1032 exactly like the kernel."""
    word &= 0xFFFFFFFF
    out = []
    for p in range(4):
        bits = ((word >> (4 * p)) & 0x000F000F) | 0x64006400
        lo = np.array([bits & 0xFFFF], dtype=np.uint16).view(np.float16)[0]
        hi = np.array([bits >> 16], dtype=np.uint16).view(np.float16)[0]
        out.append((float(lo - np.float16(1032)), float(hi - np.float16(1032))))
    return out


def dequant_from_packed(Wp: np.ndarray, scales: np.ndarray, N: int, K: int) -> np.ndarray:
    """fp16 [N, K] dequantized straight from the packed words."""
    G = K // scales.shape[0]
    return dequantize_w4(unpack_int4(Wp, N, K), scales, G)


def ref_gemm_from_packed(x: np.ndarray, Wp: np.ndarray, scales: np.ndarray) -> np.ndarray:
    """fp32 reference for y = x @ W^T given the packed operands the kernel sees."""
    x = np.asarray(x)
    K = x.shape[1]
    N = scales.shape[1]
    G = K // scales.shape[0]
    return ref_gemm(x, unpack_int4(Wp, N, K), scales, G)
