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

The exchange step is NCCL (all_gather_into_tensor / all_reduce) by default.  Given a
``PeerExchange`` the layers instead exchange through one buffer per rank that every rank
maps (CUDA IPC): the row-parallel sums are reduced and the column-parallel outputs
gathered by the library's own exchange kernel (w4a16_tp_allreduce / w4a16_tp_allgather),
which loads and stores the peers' buffers directly -- one small launch per exchange, the
partials summed in rank order, the result written into every rank's buffer.

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


class _CudaRegion:
    """A device-memory range presented through __cuda_array_interface__ (for a zero-copy view)."""

    def __init__(self, ptr, shape, typestr):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr, "data": (ptr, False),
                                         "version": 3, "strides": None}


class PeerExchange:
    """One exchange buffer per rank of ``group``, mapped by every rank (CUDA IPC over NVLink).

    Layout of each buffer: the exchange's flags (``TP_CTRL_BYTES``), then a source region of
    ``src_bytes`` (this rank's GEMM output: fp32 partials or fp16 columns), then a result
    region of ``y_bytes`` (fp16 y), then a receive area of 2 * world slots of
    ``min(src_bytes, push_bytes)`` (``push_bytes`` at most ``TP_PUSH_MAX_BYTES``; 0: no
    receive area): exchanges whose per-rank contribution fits a slot (decode sizes) run in one
    round through it, larger ones in two rounds, with the same results.  Layers sharing one exchange must
    be called in the same order on every rank, on one stream each; a result view stays valid
    until the next exchange.  ``close()`` unmaps and frees (collective).
    """

    def __init__(self, src_bytes: int, y_bytes: int, group=None, push_bytes: Optional[int] = None):
        from . import capi
        import ctypes
        self._capi, self._ct = capi, ctypes
        self.lib = capi.load()
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.world > capi.TP_MAX_RANKS:
            raise ValueError(f"at most {capi.TP_MAX_RANKS} ranks")
        self.src_off = capi.TP_CTRL_BYTES
        self.y_off = self.src_off + (int(src_bytes) + 255) // 256 * 256
        self.recv_off = self.y_off + (int(y_bytes) + 255) // 256 * 256
        push = capi.TP_PUSH_MAX_BYTES if push_bytes is None else min(int(push_bytes), capi.TP_PUSH_MAX_BYTES)
        slot = (min(int(src_bytes), push) + 255) // 256 * 256
        self.recv_bytes = 2 * self.world * slot if self.world > 1 and push > 0 else 0
        self.nbytes = self.recv_off + self.recv_bytes
        own = ctypes.c_void_p()
        handle = capi.IpcHandle()
        capi.check(self.lib.w4a16_peer_alloc(self.nbytes, ctypes.byref(own), ctypes.byref(handle)), self.lib)
        handles = [None] * self.world
        dist.all_gather_object(handles, bytes(handle.bytes), group=group)
        self.ptrs = []
        for r, hb in enumerate(handles):
            if r == self.rank:
                self.ptrs.append(own.value)
                continue
            h = capi.IpcHandle()
            ctypes.memmove(h.bytes, hb, len(hb))
            p = ctypes.c_void_p()
            capi.check(self.lib.w4a16_peer_open(ctypes.byref(h), ctypes.byref(p)), self.lib)
            self.ptrs.append(p.value)
        self.tp_group = capi.TpGroup(self.rank, self.world,
                                     (ctypes.c_void_p * capi.TP_MAX_RANKS)(*self.ptrs), self.nbytes,
                                     self.recv_off, self.recv_bytes)
        dist.barrier(group=group)   # every rank has mapped every buffer before the first exchange

    def view(self, offset: int, shape, dtype: torch.dtype) -> torch.Tensor:
        """A tensor over this rank's own buffer at ``offset`` (no copy, no ownership)."""
        typestr = {torch.float16: "<f2", torch.float32: "<f4"}[dtype]
        return torch.as_tensor(_CudaRegion(self.ptrs[self.rank] + offset, shape, typestr), device="cuda")

    def src(self, shape, dtype: torch.dtype) -> torch.Tensor:
        return self.view(self.src_off, shape, dtype)

    def y(self, M: int, N: int) -> torch.Tensor:
        return self.view(self.y_off, (M, N), torch.float16)

    def allreduce(self, M: int, N: int) -> torch.Tensor:
        """Every rank's fp32 partial [M, N] (its source region) summed in rank order into
        every rank's y [M, N] fp16; returns this rank's y."""
        self._capi.check(self.lib.w4a16_tp_allreduce(self._ct.byref(self.tp_group), self.src_off, self.y_off, M, N,
                                                     self._ct.c_void_p(torch.cuda.current_stream().cuda_stream)),
                         self.lib)
        return self.y(M, N)

    def allgather(self, M: int, N: int) -> torch.Tensor:
        """Every rank's fp16 columns [M, N / world] (its source region) into every rank's y
        [M, N], rank r's at columns [r N / world, (r + 1) N / world); returns this rank's y."""
        self._capi.check(self.lib.w4a16_tp_allgather(self._ct.byref(self.tp_group), self.src_off, self.y_off, M, N,
                                                     self._ct.c_void_p(torch.cuda.current_stream().cuda_stream)),
                         self.lib)
        return self.y(M, N)

    def close(self) -> None:
        torch.cuda.synchronize()
        dist.barrier(group=self.group)   # nobody touches a peer's buffer any more
        for r, p in enumerate(self.ptrs):
            if r != self.rank:
                self._capi.check(self.lib.w4a16_peer_close(self._ct.c_void_p(p)), self.lib)
        dist.barrier(group=self.group)   # every peer has unmapped this rank's buffer
        self._capi.check(self.lib.w4a16_peer_free(self._ct.c_void_p(self.ptrs[self.rank])), self.lib)
        self.ptrs = []


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
    """y = x @ W^T with W split along N over the process group; returns full y [M, N].

    With ``exchange`` (a PeerExchange of this group) ``fused(x)`` writes the local columns into
    the exchange buffer and gathers them with the library's exchange kernel."""

    def __init__(self, Wp, scales, N, K, group=None, gemm_out: Optional[GemmOut] = None,
                 exchange: Optional[PeerExchange] = None):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.N, self.K = N, K
        self.N_local = N // self.world
        self.Wp, self.scales = shard_columns(Wp, scales, N, K, self.rank, self.world)
        self.gemm_out = gemm_out or _default_gemm_out
        self.workspace: Optional[torch.Tensor] = None   # optional GEMM workspace (scratch)
        self._gather_bufs: dict = {}
        self.exchange = exchange

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

    def fused(self, x: torch.Tensor) -> torch.Tensor:
        """y [M, N] through the peer exchange: a view of the exchange buffer, valid until
        the exchange's next call."""
        M = x.shape[0]
        self._gemm(x, self.exchange.src((M, self.N_local), torch.float16))
        return self.exchange.allgather(M, self.N)


class RowParallelW4A16:
    """y = x @ W^T with W split along K; the caller passes this rank's K slice of x.

    With ``exchange`` (a PeerExchange of this group) ``fused(x_local)`` writes the fp32
    partial into the exchange buffer and reduces it with the library's exchange kernel."""

    def __init__(self, Wp, scales, N, K, group=None, gemm_out: Optional[GemmOut] = None,
                 exchange: Optional[PeerExchange] = None):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.N, self.K = N, K
        self.K_local = K // self.world
        self.Wp, self.scales = shard_rows(Wp, scales, N, K, self.rank, self.world)
        self.gemm_out = gemm_out or _default_gemm_out
        self.workspace: Optional[torch.Tensor] = None   # optional GEMM workspace (scratch)
        self.exchange = exchange

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

    def fused(self, x_local: torch.Tensor) -> torch.Tensor:
        """y [M, N] fp16 through the peer exchange: a view of the exchange buffer, valid until
        the exchange's next call."""
        M = x_local.shape[0]
        self.partial(x_local, out=self.exchange.src((M, self.N), torch.float32))
        return self.exchange.allreduce(M, self.N)
