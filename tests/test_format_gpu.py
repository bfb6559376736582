"""GPU parity of the load-time format kernels (w4a16_pack, w4a16_quantize,
w4a16_quantize_pack) against the reference's own outputs (golden vectors made by its
tests/quant.py) and the CPU oracle, bit for bit."""
import ctypes
import os

import numpy as np
import pytest
import torch

from oracle import w4a16_oracle as oracle

pytestmark = pytest.mark.gpu

GOLDEN = np.load(os.path.join(os.path.dirname(__file__), "golden", "golden.npz"))


@pytest.fixture(autouse=True)
def _gpu(cuda_device):
    yield


@pytest.mark.parametrize("shape", ["16x64", "32x128", "48x192", "64x512", "80x640", "208x384"])
def test_pack_matches_reference_golden(shape):
    from w4a16_opt import pack_int4
    q = torch.from_numpy(GOLDEN[f"pack_{shape}_q"]).cuda()
    wp = pack_int4(q)
    assert wp.is_cuda and wp.dtype == torch.int32
    assert np.array_equal(wp.cpu().numpy(), GOLDEN[f"pack_{shape}_wp"])


@pytest.mark.parametrize("G", [64, 128])
def test_quantize_matches_reference_golden(G):
    from w4a16_opt import quantize_w4
    W = torch.from_numpy(GOLDEN[f"quant_G{G}_W"]).cuda()
    q, s = quantize_w4(W, G)
    assert q.is_cuda and s.dtype == torch.float16
    assert np.array_equal(q.cpu().numpy(), GOLDEN[f"quant_G{G}_q"])
    assert np.array_equal(s.cpu().numpy().view(np.uint16), GOLDEN[f"quant_G{G}_scales"].view(np.uint16))


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16])
@pytest.mark.parametrize("G", [64, 128])
@pytest.mark.parametrize("N,K", [(16, 128), (48, 256), (208, 384), (4096, 4096), (1024, 14336)])
def test_quantize_and_pack_match_oracle(N, K, G, dtype):
    from w4a16_opt import pack_int4, quantize_pack, quantize_w4
    if K % G:
        pytest.skip("K must be a multiple of G")
    gen = torch.Generator().manual_seed(N + K + G)
    W = (torch.randn(N, K, generator=gen) * 0.02).to(dtype)
    # a few exact ties and tiny groups: round-half-even and the 1e-4 clamp
    W[0, :G] = 0
    W[1, :8] = torch.tensor([7, -7, 3.5, -3.5, 0.5, -0.5, 2.5, 1.5], dtype=dtype)
    q_ref, s_ref = oracle.quantize_w4(W.float().numpy(), G)
    q, s = quantize_w4(W.cuda(), G)
    assert np.array_equal(q.cpu().numpy(), q_ref)
    assert np.array_equal(s.cpu().numpy().view(np.uint16), s_ref.view(np.uint16))
    wp_ref = oracle.pack_int4(q_ref)
    assert np.array_equal(pack_int4(q).cpu().numpy(), wp_ref)
    wp, s2 = quantize_pack(W.cuda(), G)
    assert np.array_equal(wp.cpu().numpy(), wp_ref)
    assert torch.equal(s2, s)


def test_quantize_pack_feeds_the_gemm():
    """quantize_pack on the device gives the same GEMM as the CPU quantise + pack."""
    from helpers import assert_close, ref_gemm
    from w4a16_opt import quantize_pack, w4a16_gemm
    gen = torch.Generator().manual_seed(7)
    W = torch.randn(512, 1024, generator=gen) * 0.02
    x = torch.randn(5, 1024, generator=gen).half()
    Wp, s = quantize_pack(W.cuda(), 128)
    q_ref, _ = oracle.quantize_w4(W.numpy(), 128)
    assert_close(w4a16_gemm(Wp, x.cuda(), s), ref_gemm(x, torch.from_numpy(q_ref), s, 128))


def test_format_entries_reject_bad_input():
    from w4a16_opt import capi
    lib = capi.load()
    q = torch.zeros(16, 64, dtype=torch.uint8, device="cuda")
    wp = torch.empty(128, dtype=torch.int32, device="cuda")
    s = torch.empty(1, 16, dtype=torch.half, device="cuda")
    W = torch.zeros(16, 64, device="cuda")
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    assert lib.w4a16_pack(q.data_ptr(), wp.data_ptr(), 16, 60, stream) == 5                  # K % 64
    assert lib.w4a16_pack(q.data_ptr(), wp.data_ptr(), 8, 64, stream) == 6                   # N % 16
    assert lib.w4a16_pack(q.data_ptr() + 1, wp.data_ptr(), 16, 64, stream) == 9              # alignment
    assert lib.w4a16_quantize(W.data_ptr(), 0, q.data_ptr(), s.data_ptr(), 16, 64, 96, stream) == 10   # G
    assert "group size" in capi.last_error(lib)
    assert lib.w4a16_quantize_pack(W.data_ptr(), 7, wp.data_ptr(), s.data_ptr(), 16, 64, 64, stream) == 12
    assert lib.w4a16_quantize_pack(W.data_ptr(), 0, wp.data_ptr(), s.data_ptr(), 16, 64, 64, stream) == 0
