"""w4a16_gemm_noalloc (built-in scratch) against w4a16_gemm (caller workspace), through the C ABI.

w4a16_gemm_noalloc serves callers that may not allocate device memory (a fixed device-memory
budget, a binding with no device allocator): its decode scratch is an array built into the
library.  Collected last (file name) so it also runs after every other GPU test has used the
device.
"""
import ctypes

import pytest
import torch

from helpers import assert_close, make_workload

pytestmark = pytest.mark.gpu


def _call_gemm(lib, Wp, x, s, y, M, N, K, G, ws, ws_bytes, stream):
    return lib.w4a16_gemm(Wp.data_ptr(), x.data_ptr(), s.data_ptr(), y.data_ptr(), M, N, K, K // G, Wp.numel(),
                          -1, 0, ws, ws_bytes, ctypes.c_void_p(stream))


def _call_noalloc(lib, Wp, x, s, y, M, N, K, G, stream):
    return lib.w4a16_gemm_noalloc(Wp.data_ptr(), x.data_ptr(), s.data_ptr(), y.data_ptr(), M, N, K, K // G,
                                  Wp.numel(), -1, 0, ctypes.c_void_p(stream))


# decode shapes whose column groups are split across CTAs (they use the scratch), and one
# prefill shape (no scratch at all)
@pytest.mark.parametrize("M,N,K,uses_scratch", [(1, 4096, 4096, True), (16, 14336, 4096, True),
                                                (5, 1024, 4096, True), (8, 4096, 14336, True),
                                                (64, 4096, 4096, False)])
def test_noalloc_matches_workspace_entry(M, N, K, uses_scratch, cuda_device):
    from w4a16_opt import capi
    lib = capi.load()
    G = 128
    stream = torch.cuda.current_stream().cuda_stream
    nbytes = ctypes.c_uint64(0)
    capi.check(lib.w4a16_workspace_bytes(M, N, K, K // G, -1, ctypes.byref(nbytes)), lib)
    # the decode scratch is 2 partial slots of 16 KB per CTA: 4.6 MiB on 148 SMs, inside the
    # 6 MiB array whatever the shape (the array's size covers GPUs of up to 192 SMs)
    assert (nbytes.value > 0) == uses_scratch and nbytes.value <= 6 << 20
    # the scratch shapes really split column groups (decode kernel + combine kernel), so the
    # built-in array is read back by a second launch on every call
    from w4a16_opt import query_route
    assert query_route(M, N, K, K // G)["launches"] == (2 if uses_scratch else 1)
    ws = torch.empty(max(256, nbytes.value), dtype=torch.uint8, device="cuda")
    for rep in range(2):   # the built-in scratch is reused by consecutive calls
        x, q, s, Wp = make_workload(M, N, K, G, seed=100 * rep + M + N)
        y_ref = torch.empty(M, N, dtype=torch.half, device="cuda")
        capi.check(_call_gemm(lib, Wp, x, s, y_ref, M, N, K, G, ws.data_ptr(), nbytes.value, stream), lib)
        y = torch.full((M, N), float("nan"), dtype=torch.half, device="cuda")
        capi.check(_call_noalloc(lib, Wp, x, s, y, M, N, K, G, stream), lib)
        torch.cuda.synchronize()
        assert_close(y, y_ref.float().cpu().numpy())


def test_noalloc_validates_like_gemm(cuda_device):
    from w4a16_opt import capi
    lib = capi.load()
    x, q, s, Wp = make_workload(2, 256, 1024, 128)
    y = torch.empty(2, 256, dtype=torch.half, device="cuda")
    st = lib.w4a16_gemm_noalloc(Wp.data_ptr(), x.data_ptr(), s.data_ptr(), y.data_ptr(), 2, 256, 1024, 8,
                                Wp.numel(), 9, 0, ctypes.c_void_p(0))
    assert st == 2 and "variant" in capi.last_error(lib)
