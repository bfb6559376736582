"""Tensor-parallel W4A16 projections over torch.distributed (NCCL on B200s).

The packed format shards without repacking along N and with one slice along K:

* Column-parallel (q/k/v/gate/up): rank r owns n16 blocks
  [r*NB/P, (r+1)*NB/P) -- a contiguous slab of the packed words viewed as
  [NB, KC, 32, 4] -- and scales[:, n-slice].  Each rank computes y_r [M, N/P];
  an all-gather over NVLink assembles y [M, N].
* Row-parallel (o/down): rank r owns 64-wide K chunks [r*KC/P, (r+1)*KC/P)
  (``[:, kslice]`` of the same view, copied once at load) and scales[g-slice, :].
  Each rank multiplies its K slice of x into an fp32 partial [M, N]; an fp32
  all-reduce sums the partials and one cast gives fp16 y.

The reference has no distributed code; this layer follows the sharding the
north-star configuration asks for (Llama-3-70B gate/up split along N, down
split along K).  The GEMM itself is always the CUDA kernel; ``gemm_out`` is
injectable only so the host-side sharding logic can be exercised on CPU
process groups in tests.
"""
from __future__ import annotations

from typing import Callable, Optional

import torch
import torch.distributed as dist

GemmOut = Callable[[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor], torch.Tensor]


def _default_gemm_out(Wp, x, scales, y, workspace=None):
    # the shards were made once, at construction, and settled: resident weights
    from . import w4a16_gemm_out
    return w4a16_gemm_out(Wp, x, scales, y, workspace=workspace, weights_resident=True)


def _settle(*tensors: torch.Tensor) -> None:
    """Wait for the copies that made CUDA shards, so that every later GEMM may declare them
    resident (fetched before the previous kernel on the stream has finished)."""
    for t in tensors:
        if t.is_cuda:
            torch.cuda.current_stream(t.device).synchronize()


def shard_columns(Wp: torch.Tensor, scales: torch.Tensor, N: int, K: int, rank: int, world: int):
    """(Wp_r, scales_r) for rank r of a column-parallel split of N."""
    NB, KC = N // 16, K // 64
    if NB % world:
        raise ValueError(f"N/16 = {NB} n16 blocks do not split evenly over {world} ranks")
    nb = NB // world
    Wp_r = Wp.view(NB, KC, 32, 4)[rank * nb:(rank + 1) * nb].contiguous().view(-1)
    s_r = scales[:, rank * nb * 16:(rank + 1) * nb * 16].contiguous()
    _settle(Wp_r, s_r)
    return Wp_r, s_r


def shard_rows(Wp: torch.Tensor, scales: torch.Tensor, N: int, K: int, rank: int, world: int):
    """(Wp_r, scales_r) for rank r of a row-parallel split of K."""
    NB, KC = N // 16, K // 64
    G = K // scales.shape[0]
    if KC % world or (K // world) % G:
        raise ValueError(f"K = {K} does not split into {world} slices of whole 64-chunks and {G}-groups")
    kc = KC // world
    Wp_r = Wp.view(NB, KC, 32, 4)[:, rank * kc:(rank + 1) * kc].contiguous().view(-1)
    gpr = (K // world) // G
    s_r = scales[rank * gpr:(rank + 1) * gpr].contiguous()
    _settle(Wp_r, s_r)
    return Wp_r, s_r


class ColumnParallelW4A16:
    """y = x @ W^T with W split along N over the process group; returns full y [M, N]."""

    def __init__(self, Wp, scales, N, K, group=None, gemm_out: Optional[GemmOut] = None):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.N, self.K = N, K
        self.N_local = N // self.world
        self.Wp, self.scales = shard_columns(Wp, scales, N, K, self.rank, self.world)
        self.gemm_out = gemm_out or _default_gemm_out
        self.workspace: Optional[torch.Tensor] = None   # optional GEMM workspace (scratch)
        self._gather_bufs: dict = {}

    def local(self, x: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        y = out if out is not None else torch.empty(x.shape[0], self.N_local, dtype=torch.float16, device=x.device)
        return self._gemm(x, y)

    def _gemm(self, x, y):
        if self.workspace is not None:
            return self.gemm_out(self.Wp, x, self.scales, y, workspace=self.workspace)
        return self.gemm_out(self.Wp, x, self.scales, y)

    def gather(self, y_local: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """y [M, N] from every rank's y_local [M, N/P]; written into ``out`` when given."""
        M = y_local.shape[0]
        y = out if out is not None else torch.empty(M, self.N, dtype=y_local.dtype, device=y_local.device)
        if M == 1:
            # one token: the ranks' blocks concatenated are already y's row
            dist.all_gather_into_tensor(y.view(-1), y_local.contiguous().view(-1), group=self.group)
            return y
        # ranks' blocks concatenated along dim 0 ([world * M, N/P]: the layout every backend
        # takes) into a staging buffer kept per (M, dtype), then one strided copy into y
        key = (M, y_local.dtype, y_local.device)
        buf = self._gather_bufs.get(key)
        if buf is None:
            buf = torch.empty(self.world * M, self.N_local, dtype=y_local.dtype, device=y_local.device)
            self._gather_bufs[key] = buf
        dist.all_gather_into_tensor(buf, y_local.contiguous(), group=self.group)
        y.view(M, self.world, self.N_local).copy_(buf.view(self.world, M, self.N_local).permute(1, 0, 2))
        return y

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        return self.gather(self.local(x))


class RowParallelW4A16:
    """y = x @ W^T with W split along K; the caller passes this rank's K slice of x."""

    def __init__(self, Wp, scales, N, K, group=None, gemm_out: Optional[GemmOut] = None):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.N, self.K = N, K
        self.K_local = K // self.world
        self.Wp, self.scales = shard_rows(Wp, scales, N, K, self.rank, self.world)
        self.gemm_out = gemm_out or _default_gemm_out
        self.workspace: Optional[torch.Tensor] = None   # optional GEMM workspace (scratch)

    def x_slice(self, x: torch.Tensor) -> torch.Tensor:
        return x[:, self.rank * self.K_local:(self.rank + 1) * self.K_local].contiguous()

    def partial(self, x_local: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        y = out if out is not None else torch.empty(x_local.shape[0], self.N, dtype=torch.float32,
                                                    device=x_local.device)
        if self.workspace is not None:
            return self.gemm_out(self.Wp, x_local, self.scales, y, workspace=self.workspace)
        return self.gemm_out(self.Wp, x_local, self.scales, y)

    def reduce(self, partial: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Sums the ranks' fp32 partials in place, then casts to fp16 (into ``out`` when given)."""
        dist.all_reduce(partial, op=dist.ReduceOp.SUM, group=self.group)
        if out is None:
            return partial.half()
        out.copy_(partial)
        return out

    def __call__(self, x_local: torch.Tensor) -> torch.Tensor:
        return self.reduce(self.partial(x_local))
