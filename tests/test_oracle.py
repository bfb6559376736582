"""CPU tests: the oracle and the product's format utilities against the golden
vectors produced by the reference's own tests/quant.py (tests/golden/make_golden.py)."""
import hashlib
import os

import numpy as np
import pytest
import torch

from oracle import w4a16_oracle as oracle

GOLDEN = np.load(os.path.join(os.path.dirname(__file__), "golden", "golden.npz"))


def _keys(prefix, suffix):
    return sorted(k[: -len(suffix)] for k in GOLDEN.files if k.startswith(prefix) and k.endswith(suffix))


# ---------------------------------------------------------------- oracle pinned to the reference

def test_fragment_map_is_bijection():
    n_idx, k_idx = oracle.fragment_map()
    cells = {(int(n), int(k)) for n, k in zip(n_idx.ravel(), k_idx.ravel())}
    assert len(cells) == 256 and all(0 <= n < 16 and 0 <= k < 16 for n, k in cells)


@pytest.mark.parametrize("base", _keys("pack_", "_q"))
def test_oracle_pack_matches_reference(base):
    q = GOLDEN[base + "_q"]
    wp = oracle.pack_int4(q)
    assert wp.dtype == np.int32
    assert np.array_equal(wp, GOLDEN[base + "_wp"])
    assert np.array_equal(oracle.unpack_int4(wp, *q.shape), q)


@pytest.mark.parametrize("G", [64, 128])
def test_oracle_quantize_dequant_matches_reference(G):
    q, s = oracle.quantize_w4(GOLDEN[f"quant_G{G}_W"], G)
    assert np.array_equal(q, GOLDEN[f"quant_G{G}_q"])
    assert np.array_equal(s.view(np.uint16), GOLDEN[f"quant_G{G}_scales"].view(np.uint16))
    d = oracle.dequantize_w4(q, s, G)
    assert np.array_equal(d.view(np.uint16), GOLDEN[f"quant_G{G}_deq"].view(np.uint16))


@pytest.mark.parametrize("base", _keys("gemm_", "_y"))
def test_oracle_gemm_matches_reference(base):
    y = oracle.ref_gemm_from_packed(GOLDEN[base + "_x"], GOLDEN[base + "_wp"], GOLDEN[base + "_scales"])
    ref = GOLDEN[base + "_y"]
    # same fp16 operands, fp32 accumulation in a different order
    assert np.abs(y - ref).max() <= 1e-5 * max(1.0, np.abs(ref).max())


def test_kernel_word_decode_matches_pack():
    """Decode packed words the way the device dequant does (bit trick per lane) and
    recover the codes (reference: tests/test_w4a16.py:60-78)."""
    N, K = 32, 128
    q = GOLDEN[f"pack_{N}x{K}_q"]
    Wp = GOLDEN[f"pack_{N}x{K}_wp"].view(np.uint32).reshape(N // 16, K // 64, 32, 4)
    out = np.full((N, K), -1, dtype=np.int64)
    for nb in range(N // 16):
        for kc in range(K // 64):
            for lane in range(32):
                g, t = lane >> 2, lane & 3
                for s in range(4):
                    pairs = oracle.kernel_word_decode(int(Wp[nb, kc, lane, s]))
                    for p, (lo, hi) in enumerate(pairs):
                        row = nb * 16 + g + 8 * (p & 1)
                        col = kc * 64 + s * 16 + 2 * t + 8 * (p >> 1)
                        out[row, col] = int(lo) + 8
                        out[row, col + 1] = int(hi) + 8
    assert np.array_equal(out, q.astype(np.int64))


def test_magic_constants_exact():
    """The device dequant's two fp16 magic forms give q - 8 exactly for all 16 codes."""
    h = lambda b: np.array([b], dtype=np.uint16).view(np.float16)[0]
    for nib in range(16):
        assert float(h(0x6400 | nib) - h(0x6408)) == nib - 8          # mantissa bits 0..3, 2^10
        assert float(h(0x5400 | (nib << 4)) - h(0x5480)) == nib - 8   # mantissa bits 4..7, 2^6


def test_cfg0_workload_checksums():
    """BASELINE configs[0] inputs (seed 0) and their packed words match the reference's."""
    from helpers import make_workload
    x, q, s, wp = make_workload(1, 4096, 4096, 128, seed=0, device="cpu")
    sha = lambda a: hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()
    assert sha(x.numpy()) == str(GOLDEN["cfg0_sha_x"])
    assert sha(s.numpy()) == str(GOLDEN["cfg0_sha_scales"])
    assert sha(wp.numpy()) == str(GOLDEN["cfg0_sha_wp"])
    assert sha(oracle.pack_int4(q.numpy())) == str(GOLDEN["cfg0_sha_wp"])


def test_cfg0_oracle_output():
    from helpers import make_workload
    x, q, s, _ = make_workload(1, 4096, 4096, 128, seed=0, device="cpu")
    y = oracle.ref_gemm(x.numpy(), q.numpy(), s.numpy(), 128)
    ref = GOLDEN["cfg0_y"]
    assert np.abs(y - ref).max() <= 1e-5 * np.abs(ref).max()


# ---------------------------------------------------------------- product format utilities

@pytest.mark.parametrize("base", _keys("pack_", "_q"))
def test_product_pack_matches_reference(base):
    from w4a16_opt import pack_int4, unpack_int4
    q = torch.from_numpy(GOLDEN[base + "_q"])
    wp = pack_int4(q)
    assert wp.dtype == torch.int32
    assert np.array_equal(wp.numpy(), GOLDEN[base + "_wp"])
    assert torch.equal(unpack_int4(wp, *q.shape), q)


@pytest.mark.parametrize("G", [64, 128])
def test_product_quantize_matches_reference(G):
    from w4a16_opt import dequantize_w4, quantize_w4
    q, s = quantize_w4(torch.from_numpy(GOLDEN[f"quant_G{G}_W"]), G)
    assert np.array_equal(q.numpy(), GOLDEN[f"quant_G{G}_q"])
    assert np.array_equal(s.numpy().view(np.uint16), GOLDEN[f"quant_G{G}_scales"].view(np.uint16))
    d = dequantize_w4(q, s, G)
    assert np.array_equal(d.numpy().view(np.uint16), GOLDEN[f"quant_G{G}_deq"].view(np.uint16))


@pytest.mark.parametrize("N,K", [(16, 64), (64, 512), (272, 1152), (1040, 2048)])
def test_product_pack_matches_oracle(N, K):
    from w4a16_opt import pack_int4
    gen = torch.Generator().manual_seed(N + K)
    q = torch.randint(0, 16, (N, K), generator=gen, dtype=torch.uint8)
    assert np.array_equal(pack_int4(q).numpy(), oracle.pack_int4(q.numpy()))


@pytest.mark.parametrize("G", [64, 128])
def test_quantization_sanity(G):
    """Not a kernel test: the RTN quantizer is reasonable (tests/test_w4a16.py:81-88)."""
    W = np.random.default_rng(G).standard_normal((256, 1024)).astype(np.float32) * 0.02
    q, s = oracle.quantize_w4(W, G)
    Wd = oracle.dequantize_w4(q, s, G).astype(np.float32)
    cos = float((W * Wd).sum() / np.linalg.norm(W) / np.linalg.norm(Wd))
    assert cos > 0.98


def test_pack_rejects_bad_shapes():
    from w4a16_opt import pack_int4
    with pytest.raises(ValueError):
        oracle.pack_int4(np.zeros((24, 64), np.uint8))
    with pytest.raises(ValueError):
        pack_int4(torch.zeros(16, 96, dtype=torch.uint8))


# ---------------------------------------------------------------- properties over random shapes and values

from hypothesis import HealthCheck, assume, given, settings  # noqa: E402
from hypothesis import strategies as st  # noqa: E402

_shapes = st.tuples(st.integers(1, 6).map(lambda b: 16 * b), st.integers(1, 4).map(lambda c: 64 * c))
_prop = settings(max_examples=40, deadline=None, suppress_health_check=[HealthCheck.too_slow])


@_prop
@given(shape=_shapes, seed=st.integers(0, 2**31 - 1))
def test_prop_pack_roundtrip_and_product_equals_oracle(shape, seed):
    from w4a16_opt import pack_int4, unpack_int4
    N, K = shape
    q = np.random.default_rng(seed).integers(0, 16, (N, K), dtype=np.uint8)
    wp = oracle.pack_int4(q)
    assert np.array_equal(oracle.unpack_int4(wp, N, K), q)
    assert np.array_equal(pack_int4(torch.from_numpy(q)).numpy(), wp)
    assert torch.equal(unpack_int4(torch.from_numpy(wp.view(np.int32)), N, K), torch.from_numpy(q))


@_prop
@given(shape=_shapes, G=st.sampled_from([64, 128]), seed=st.integers(0, 2**31 - 1),
       scale_exp=st.integers(-12, 3))
def test_prop_quantize_product_equals_oracle(shape, G, seed, scale_exp):
    """The product's quantize_w4 (torch) and the oracle's (numpy) agree bit for bit over
    magnitudes from 2^-12 to 2^3, including the 1e-4 scale floor and exact .5 ties."""
    from w4a16_opt import quantize_w4
    N, K = shape
    assume(K % G == 0)
    rng = np.random.default_rng(seed)
    W = (rng.standard_normal((N, K)) * 2.0 ** scale_exp).astype(np.float32)
    W[0, : min(K, 8)] = np.float32(2.0 ** scale_exp) * np.array([3.5, -3.5, 0.5, -0.5, 7, -7, 0, 2.5],
                                                                 np.float32)[: min(K, 8)]
    q_o, s_o = oracle.quantize_w4(W, G)
    q_p, s_p = quantize_w4(torch.from_numpy(W), G)
    assert np.array_equal(q_p.numpy(), q_o)
    assert np.array_equal(s_p.numpy().view(np.uint16), np.asarray(s_o, np.float16).view(np.uint16))


@_prop
@given(shape=_shapes, seed=st.integers(0, 2**31 - 1))
def test_prop_kernel_word_decode_dequant_equals_reference_dequant(shape, seed):
    """Dequantising through the kernel's word decode (magic-number form) equals the
    reference's (q - 8) * scale in fp16 bit for bit, for random codes and scales."""
    N, K = shape
    G = 64
    rng = np.random.default_rng(seed)
    q = rng.integers(0, 16, (N, K), dtype=np.uint8)
    s = (rng.random((K // G, N)) * 0.05 + 1e-4).astype(np.float16)
    wp = oracle.pack_int4(q)
    ref = oracle.dequantize_w4(q, s, G)
    words = wp.reshape(N // 16, K // 64, 32, 4)
    n_idx, k_idx = oracle.fragment_map()
    for nb in range(N // 16):
        for kc in range(K // 64):
            for lane in range(0, 32, 7):
                for sub in range(4):
                    pairs = oracle.kernel_word_decode(int(words[nb, kc, lane, sub]))
                    for p in range(4):
                        for h in range(2):
                            i = p + 4 * h
                            n = nb * 16 + int(n_idx[lane, i])
                            k = kc * 64 + sub * 16 + int(k_idx[lane, i])
                            got = np.float16(np.float16(pairs[p][h]) * s[k // G, n])
                            assert got.view(np.uint16) == ref[n, k].view(np.uint16)
