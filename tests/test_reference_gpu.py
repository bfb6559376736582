"""Parity against the reference's own CUDA implementation, run on the same GPU.

oracle/build_ref.py compiles akshay919191/W4A16-GEMM's extension
(src/vectorized/kernel.cu) for sm_100a into oracle/_ref/ as a checker module
``w4a16_ref``.  These tests feed both implementations identical inputs and
compare: outputs within the north-star tolerance of each other (both use the
bit-identical fp16 dequantisation and fp32 accumulation; only the summation
order differs), one-hot inputs bit-identical, and the same rejection messages
(kernel.cu:219-249).  Skipped when the checker module was not built.
"""
import pytest
import torch

from helpers import assert_close, make_problem, make_workload

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ref():
    from oracle import build_ref
    mod = build_ref.load()
    if mod is None:
        pytest.skip("reference checker module oracle/_ref/w4a16_ref not built")
    return mod


def ours(Wp, x, s, variant=-1):
    from w4a16_opt import w4a16_gemm
    return w4a16_gemm(Wp, x, s, variant)


CASES = [
    # decode sweep shapes (G = 128)
    (1, 4096, 4096, 128), (4, 1024, 4096, 128), (8, 14336, 4096, 128), (16, 4096, 14336, 128),
    # prefill shapes at small M, both group sizes
    (128, 14336, 4096, 64), (512, 4096, 14336, 128),
    # ragged contract edge cases (the reference routes these to its prefill kernel)
    (1, 4112, 4160, 64), (17, 4112, 4160, 64), (37, 4112, 4160, 64), (129, 4112, 4160, 64), (3, 1040, 2048, 128),
    # configs[4] shard shapes: 70B gate/up and down at tp8
    (1, 3584, 8192, 128), (16, 8192, 3584, 128),
]


@pytest.mark.parametrize("M,N,K,G", CASES)
def test_matches_reference_kernel(ref, M, N, K, G, cuda_device):
    x, q, s, Wp = make_workload(M, N, K, G, seed=M * 7 + N + K)
    y_ref = ref.w4a16_gemm(Wp, x, s, -1)
    y = ours(Wp, x, s)
    torch.cuda.synchronize()
    assert y.shape == y_ref.shape and y.dtype == y_ref.dtype
    assert_close(y, y_ref.float().cpu().numpy())


@pytest.mark.parametrize("G", [64, 128])
def test_onehot_identical_to_reference(ref, G, cuda_device):
    """x = e_k: both implementations return dequantised weight columns, bit for bit."""
    N, K = 256, 1024
    _, q, s, Wp = make_problem(1, N, K, G)
    ks = [0, 1, 15, 16, 63, 64, 511, 512, 1023]
    x = torch.zeros(len(ks), K, dtype=torch.half, device="cuda")
    for m, k in enumerate(ks):
        x[m, k] = 1
    for variant in (-1, 0):
        assert torch.equal(ours(Wp, x, s, variant), ref.w4a16_gemm(Wp, x, s, variant))


def test_same_rejections_as_reference(ref, cuda_device):
    """Invalid calls raise RuntimeError with the same key phrase in both implementations."""
    x, q, s, Wp = make_problem(4, 256, 1024, 128)
    bad = [
        ((Wp, x, s, 7), "variant"),
        ((Wp.float(), x, s, -1), "int32"),
        ((Wp, x.float(), s, -1), "fp16"),
        ((Wp, x[:, :1000].contiguous(), s, -1), "multiple of 64"),
        ((Wp, x.t().contiguous().t(), s, -1), "contiguous"),
        ((Wp, x, s[:, :250].contiguous(), -1), "multiple of 16"),
    ]
    for args, phrase in bad:
        with pytest.raises(RuntimeError, match=phrase):
            ref.w4a16_gemm(*args)
        with pytest.raises(RuntimeError, match=phrase):
            ours(*args)
