"""The tensor-parallel exchange kernels on one GPU, through the C ABI.

* A one-rank group: the reduction is a cast of the rank's fp32 partial to fp16 and the
  gather a copy, over several calls that alternate decode sizes with contributions of
  8-16 MiB, which run on the larger grid (the rank's call count advances the same way
  whatever the grid), in the two-round form (no receive area) and the one-round form (a
  receive area, used by the small calls).
* A bounded wait that runs out: a two-rank group whose second buffer is memory of this GPU
  that no rank ever flags.  The kernel must give up after its wait limit (about 2 s),
  record kDevTimeoutPeer (7) in the device status word and return, leaving the context
  usable.  No second kernel waits on the first: the flag is one that nothing sets.
"""
import ctypes
import time

import pytest
import torch

pytestmark = pytest.mark.gpu


def _alloc(lib, capi, nbytes):
    p, h = ctypes.c_void_p(), capi.IpcHandle()
    capi.check(lib.w4a16_peer_alloc(nbytes, ctypes.byref(p), ctypes.byref(h)), lib)
    return p.value


def _view(ptr, shape, dtype):
    from w4a16_opt.tp import _CudaRegion
    typestr = {torch.float16: "<f2", torch.float32: "<f4"}[dtype]
    return torch.as_tensor(_CudaRegion(ptr, shape, typestr), device="cuda")


@pytest.mark.parametrize("one_round", [False, True])
def test_one_rank_exchange(one_round, cuda_device):
    from w4a16_opt import capi
    lib = capi.load()
    N, Ms = 4096, (16, 1024)
    M = max(Ms)
    src_off, y_off = capi.TP_CTRL_BYTES, capi.TP_CTRL_BYTES + M * N * 4
    recv_off = y_off + M * N * 2
    recv_bytes = 2 * capi.TP_PUSH_MAX_BYTES if one_round else 0
    nbytes = recv_off + recv_bytes
    buf = _alloc(lib, capi, nbytes)
    g = capi.TpGroup(0, 1, (ctypes.c_void_p * capi.TP_MAX_RANKS)(buf), nbytes, recv_off, recv_bytes)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    try:
        for i in range(6):
            M = Ms[i % 2]
            part = torch.randn(M, N, device="cuda") * (i + 1)
            _view(buf + src_off, (M, N), torch.float32).copy_(part)
            capi.check(lib.w4a16_tp_allreduce(ctypes.byref(g), src_off, y_off, M, N, stream), lib)
            torch.cuda.synchronize()
            assert torch.equal(_view(buf + y_off, (M, N), torch.float16), part.half())
            cols = torch.randn(M, N, device="cuda").half()
            _view(buf + src_off, (M, N), torch.float16).copy_(cols)
            capi.check(lib.w4a16_tp_allgather(ctypes.byref(g), src_off, y_off, M, N, stream), lib)
            torch.cuda.synchronize()
            assert torch.equal(_view(buf + y_off, (M, N), torch.float16), cols)
    finally:
        torch.cuda.synchronize()
        capi.check(lib.w4a16_peer_free(ctypes.c_void_p(buf)), lib)


@pytest.mark.parametrize("one_round", [False, True])
def test_peer_that_never_arrives_times_out(one_round, cuda_device):
    from w4a16_opt import capi, device_status
    lib = capi.load()
    M, N = 1, 256
    src_off, y_off = capi.TP_CTRL_BYTES, capi.TP_CTRL_BYTES + M * N * 4
    recv_off = y_off + M * N * 2
    recv_bytes = 2 * 2 * M * N * 4 if one_round else 0
    nbytes = recv_off + recv_bytes
    assert device_status(reset=True) == 0
    bufs = [_alloc(lib, capi, nbytes) for _ in range(2)]
    # rank 0 of two; "rank 1" is a buffer of this GPU that no kernel ever flags
    g = capi.TpGroup(0, 2, (ctypes.c_void_p * capi.TP_MAX_RANKS)(*bufs), nbytes, recv_off, recv_bytes)
    try:
        t0 = time.monotonic()
        capi.check(lib.w4a16_tp_allreduce(ctypes.byref(g), src_off, y_off, M, N,
                                          ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)), lib)
        torch.cuda.synchronize()
        waited = time.monotonic() - t0
        assert 1.0 < waited < 60.0, waited
        assert device_status(reset=True) == 7
        assert device_status() == 0
        # the context is still usable
        x = torch.ones(4, device="cuda")
        assert float((x * 2).sum()) == 8.0
    finally:
        torch.cuda.synchronize()
        for b in bufs:
            capi.check(lib.w4a16_peer_free(ctypes.c_void_p(b)), lib)
