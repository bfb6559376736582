"""Out-of-bounds writes: every route writes exactly y[M, N] and nothing around it.

Memory safety of the stores is checked directly: y is a window inside a larger buffer
filled with a canary byte pattern.  The guard bands before and after the window must keep
the pattern, and every element inside it must be written: the window must equal a
fresh-output call bit for bit.  Cases: decode with split groups (combine kernel),
with whole groups, with N and K tails; prefill with M and N tails; fp16 and fp32 outputs.
"""
import pytest
import torch

from helpers import make_workload

pytestmark = pytest.mark.gpu

GUARD = 4096          # elements on each side of the window
CANARY = 0xA5         # byte pattern: fp16 0xA5A5 / fp32 0xA5A5A5A5, finite, never a result here

CASES = [
    (1, 4096, 4096, 128),      # decode, groups split across CTAs + combine kernel
    (7, 1040, 2048, 128),      # decode, N tail (4 whole groups + 16 columns)
    (16, 272, 1152, 64),       # decode, N and K tails
    (4, 256 * 148, 64, 64),    # decode, whole groups per CTA, K < 256
    (17, 4112, 4160, 64),      # prefill, M and N tails
    (129, 208, 384, 64),       # prefill, small ragged
    (300, 1024, 2048, 128),    # prefill
]


@pytest.mark.parametrize("out_dtype", [torch.float16, torch.float32])
@pytest.mark.parametrize("M,N,K,G", CASES)
def test_guard_bands_untouched(M, N, K, G, out_dtype, cuda_device):
    from w4a16_opt import w4a16_gemm, w4a16_gemm_out
    x, q, s, Wp = make_workload(M, N, K, G, seed=M + N + K)
    buf = torch.empty(GUARD + M * N + GUARD, dtype=out_dtype, device="cuda")
    buf.view(torch.uint8).fill_(CANARY)
    y = buf[GUARD:GUARD + M * N].view(M, N)
    w4a16_gemm_out(Wp, x, s, y)
    fresh = w4a16_gemm(Wp, x, s)
    torch.cuda.synchronize()
    raw = buf.view(torch.uint8)
    esz = buf.element_size()
    head, tail = raw[:GUARD * esz], raw[(GUARD + M * N) * esz:]
    assert bool((head == CANARY).all()), "write before y"
    assert bool((tail == CANARY).all()), "write after y"
    got = y if out_dtype == torch.float16 else y.half()   # fp16 output = fp32 output rounded once
    assert torch.equal(got, fresh), "y not fully written or differs from a fresh-output call"
