"""Weight-format utilities (load-time, torch; run on CPU or CUDA tensors).

The format is the reference's (akshay919191/W4A16-GEMM tests/quant.py):

    W[n, k] ~= (q[n, k] - 8) * scales[k // G, n],   q in 0..15, scales fp16 [K/G, N]

packed so that each lane's 32-bit word is an mma.m16n8k16 A fragment: word
(((n/16)*(K/64) + k/64)*32 + lane)*4 + (k%64)/16 holds, in nibble i (bits
4i..4i+3), the code at n = 16*nb + g + 8*((i&3)&1), k = 64*kc + 16*s + 2t +
8*((i&3)>>1) + (i>>2), with g = lane // 4, t = lane % 4.

These functions produce operands for the GEMM; they are not on its hot path.  On
CUDA tensors, ``pack_int4``, ``quantize_w4`` and ``quantize_pack`` run the library's
format kernels (w4a16_pack / w4a16_quantize / w4a16_quantize_pack); on CPU tensors
(and non-fp32/fp16 weights) they run the torch restatement below, with the same
results bit for bit.
"""
from __future__ import annotations

import torch

__all__ = ["pack_int4", "unpack_int4", "quantize_w4", "quantize_pack", "dequantize_w4"]


def _ext():
    from . import _C
    return _C


def _lane_tables(device):
    lane = torch.arange(32, device=device).view(32, 1)
    i = torch.arange(8, device=device).view(1, 8)
    g, t = lane // 4, lane % 4
    p, h = i % 4, i // 4
    n_in = g + 8 * (p % 2)                 # [32, 8] row inside the 16x16 tile
    k_in = 2 * t + 8 * (p // 2) + h        # [32, 8] column inside the 16x16 tile
    return n_in, k_in


def pack_int4(q: torch.Tensor) -> torch.Tensor:
    """uint8 codes [N, K] (values 0..15) -> int32 [N*K/8] in kernel word order."""
    if q.dim() != 2:
        raise ValueError("q must be [N, K]")
    N, K = q.shape
    if N % 16 or K % 64:
        raise ValueError("N must be a multiple of 16 and K of 64")
    if q.is_cuda and q.dtype == torch.uint8:
        return _ext().pack(q.contiguous())
    NB, KC = N // 16, K // 64
    n_in, k_in = _lane_tables(q.device)
    # tiles[nb, kc, s, 16 n, 16 k]
    tiles = q.reshape(NB, 16, KC, 4, 16).permute(0, 2, 3, 1, 4)
    nib = tiles[..., n_in, k_in].to(torch.int64)                  # [NB, KC, 4, 32, 8]
    shifts = torch.arange(0, 32, 4, device=q.device, dtype=torch.int64)
    words = (nib << shifts).sum(-1)                               # disjoint fields, < 2**32
    words = words - ((words >> 31) << 32)                         # reinterpret as signed int32
    return words.to(torch.int32).permute(0, 1, 3, 2).contiguous().view(-1)


def unpack_int4(Wp: torch.Tensor, N: int, K: int) -> torch.Tensor:
    """int32 [N*K/8] -> uint8 codes [N, K]."""
    NB, KC = N // 16, K // 64
    n_in, k_in = _lane_tables(Wp.device)
    w = Wp.view(NB, KC, 32, 4).permute(0, 1, 3, 2).to(torch.int64) & 0xFFFFFFFF   # [NB, KC, 4, 32]
    shifts = torch.arange(0, 32, 4, device=Wp.device, dtype=torch.int64)
    nib = ((w.unsqueeze(-1) >> shifts) & 0xF).to(torch.uint8)                   # [NB, KC, 4, 32, 8]
    tiles = torch.empty(NB, KC, 4, 16, 16, dtype=torch.uint8, device=Wp.device)
    tiles[..., n_in, k_in] = nib
    return tiles.permute(0, 3, 1, 2, 4).reshape(N, K)


def quantize_w4(W: torch.Tensor, group_size: int):
    """Symmetric round-to-nearest-even, scale = absmax/7 per (n, k-group) clamped to
    >= 1e-4 and rounded to fp16; returns (q uint8 [N, K], scales fp16 [K/G, N])."""
    N, K = W.shape
    G = group_size
    if K % G:
        raise ValueError("K must be a multiple of the group size")
    if W.is_cuda and W.dtype in (torch.float32, torch.float16) and G in (64, 128) and N % 16 == 0 and K % 64 == 0:
        q, s = _ext().quantize(W.contiguous(), G, False)
        return q, s
    grouped = W.float().reshape(N, K // G, G)
    s = (grouped.abs().amax(-1, keepdim=True) / 7).clamp_min(1e-4).half().float()
    q = (torch.round(grouped / s).clamp(-8, 7) + 8).to(torch.uint8).reshape(N, K)
    return q, s.squeeze(-1).t().contiguous().half()


def quantize_pack(W: torch.Tensor, group_size: int):
    """quantize_w4 then pack_int4 in one pass: returns (Wp int32 [N*K/8], scales fp16 [K/G, N])."""
    if W.is_cuda and W.dtype in (torch.float32, torch.float16):
        Wp, s = _ext().quantize(W.contiguous(), group_size, True)
        return Wp, s
    q, s = quantize_w4(W, group_size)
    return pack_int4(q), s


def dequantize_w4(q: torch.Tensor, scales: torch.Tensor, group_size: int) -> torch.Tensor:
    """fp16 [N, K] = (q - 8) * scale with one fp16 rounding."""
    s = scales.t().repeat_interleave(group_size, dim=1)
    return (q.to(torch.float16) - 8) * s
