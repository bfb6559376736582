"""decode_ns_kernel (csrc/decode_ns.cuh) checked on the CPU: its plan, and its per-lane data flow.

* ``ns_plan_check.cpp`` (g++, no GPU) includes the plan header the kernel is built from
  (csrc/decode_ns_plan.h) and sweeps some 7,700 (M, N, K, G, #SMs) cases: the CTAs' block
  ranges and batches tile the blocks, a step's chunk count suits the 8 consumer warps, the
  shared-memory layout fits and is aligned, and every tensor copy starts inside its tensor.
* The emulation restates, in numpy, what the kernel does per lane: it builds each stage as
  the producer's tensor copies leave it -- per block S chunks of packed words, M activation
  rows per chunk (unpadded, 128-byte swizzle), per block R scale rows; garbage wherever no
  copy writes -- and reads it back through the consumer warps' own addressing: chunk i of a
  step goes to warp i % 8, ldmatrix rows >= M read the zero row, scales and words at the
  kernel's offsets.  The exact dequantisation and m16n8k16 fragment maps are the ones the
  stream-K emulation uses (test_decode_emulation.py).  Each warp's sums are added in warp
  order, as the batch-end reduction does, and the result is compared with the oracle GEMM
  (float64 products: this checks the index mapping).  This plays the role of the
  reference's numpy emulation of its kernel (akshay919191/W4A16-GEMM tests/layout.py).
"""
import json
import os
import shutil
import subprocess

import numpy as np
import pytest

from oracle import w4a16_oracle as oracle
from test_decode_emulation import dequant_word

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(os.path.dirname(HERE), "w4a16-gemm_b200", "csrc")
WARPS = 8

pytestmark = pytest.mark.skipif(shutil.which("g++") is None, reason="needs g++")


@pytest.fixture(scope="module")
def checker(tmp_path_factory):
    exe = tmp_path_factory.mktemp("ns") / "ns_plan_check"
    subprocess.run(["g++", "-O2", "-std=c++17", "-Wall", "-Werror", "-I", CSRC,
                    os.path.join(HERE, "ns_plan_check.cpp"), "-o", str(exe)], check=True)
    return str(exe)


def plan(checker, M, N, K, G, sms):
    out = subprocess.run([checker, str(M), str(N), str(K), str(G), str(sms)], capture_output=True, text=True,
                         check=True).stdout
    return json.loads(out)


def test_ns_plan_sweep(checker):
    r = subprocess.run([checker], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout + r.stderr
    assert r.stdout.startswith("ok ")


def test_ns_preferred_on_the_decode_sweep(checker):
    """On 148 SMs every Llama-3-8B decode projection takes the whole-column kernel."""
    for N, K in [(4096, 4096), (1024, 4096), (14336, 4096), (4096, 14336)]:
        assert plan(checker, 1, N, K, 128, 148)["preferred"] == 1


def build_stage(p, Wp4, x, scales, bk0, bb, t, N, K, G, rng):
    """One stage as the step's tensor copies leave it (garbage where no copy writes)."""
    M = x.shape[0]
    NB, KC = N // 16, K // 64
    S, R = p["S"], p["R"]
    img = rng.integers(0, 256, p["stage_bytes"], dtype=np.uint8)
    for j in range(bb):                         # packed words: box {128, S, 1} at (0, t*S, block)
        for i in range(S):
            kc = t * S + i
            words = Wp4[bk0 + j, kc] if kc < KC else np.zeros((32, 4), np.uint32)
            off = p["w_off"] + j * S * 512 + i * 512
            img[off:off + 512] = words.astype(np.uint32).reshape(-1).view(np.uint8)
    for i in range(S):                          # activations: box {64, M, S}, 128-byte swizzle
        kc = t * S + i
        for r in range(M):
            row = x[r, kc * 64:(kc + 1) * 64] if kc < KC else np.zeros(64, np.float16)
            rb = row.view(np.uint8)
            q = i * M + r
            for u in range(8):
                off = p["x_off"] + q * 128 + ((u ^ (q % 8)) << 4)
                img[off:off + 16] = rb[u * 16:(u + 1) * 16]
    for j in range(bb):                         # scales: box {16, R} at (block*16, t*S*64/G)
        for rr in range(R):
            row = t * S * 64 // G + rr
            vals = scales[row, (bk0 + j) * 16:(bk0 + j + 1) * 16] if row < K // G else np.zeros(16, np.float16)
            off = p["s_off"] + j * R * 32 + rr * 32
            img[off:off + 32] = np.asarray(vals, np.float16).view(np.uint8)
    return img


def ldmatrix_b(img, zero, addrs):
    """ldmatrix .x4 of 32 row addresses (None = the zero row): b[reg][thread][half]."""
    lanes = np.arange(32)
    rows = np.stack([zero if a is None else img[a:a + 16].view(np.float16) for a in addrs])
    b = np.zeros((4, 32, 2))
    for i in range(4):
        mat = rows[8 * i:8 * i + 8]
        b[i] = np.stack([mat[lanes // 4, 2 * (lanes % 4)], mat[lanes // 4, 2 * (lanes % 4) + 1]], 1)
    return b


def emulate(p, Wp, x, scales, N, K, G, seed=0):
    M = x.shape[0]
    MT = 1 if M <= 8 else 2
    NB, KC = N // 16, K // 64
    S, R = p["S"], p["R"]
    Wp4 = Wp.view(np.uint32).reshape(NB, KC, 32, 4)
    rng = np.random.default_rng(seed)
    lanes = np.arange(32)
    g8, t4, xr, xu = lanes >> 2, lanes & 3, lanes & 7, lanes >> 3
    zero = np.zeros(8, np.float16)
    y = np.full((M, N), np.nan)
    ctas = p["ctas"]
    b0 = [c * NB // ctas for c in range(ctas + 1)]
    for c in range(ctas):
        blocks = b0[c + 1] - b0[c]
        nbat = -(-blocks // 8)
        blo = [k * blocks // nbat for k in range(nbat + 1)]
        for k in range(nbat):
            bk0, bb = b0[c] + blo[k], blo[k + 1] - blo[k]
            acc = np.zeros((WARPS, bb, MT, 16, 8))
            for t in range(-(-KC // S)):
                img = build_stage(p, Wp4, x, scales, bk0, bb, t, N, K, G, rng)
                for w in range(WARPS):
                    for i in range(w, S, WARPS):
                        if t * S + i >= KC:
                            break
                        bfr = []
                        for mt in range(MT):
                            row = mt * 8 + xr
                            q = i * M + row
                            base = p["x_off"] + q * 128
                            a0 = [int(base[L] + ((xu[L] ^ (q[L] & 7)) << 4)) if row[L] < M else None for L in lanes]
                            a1 = [int(base[L] + (((xu[L] + 4) ^ (q[L] & 7)) << 4)) if row[L] < M else None for L in lanes]
                            bfr.append(np.concatenate([ldmatrix_b(img, zero, a0), ldmatrix_b(img, zero, a1)]))
                        srow = p["s_off"] + ((i * 64) // G) * 32 + g8 * 2
                        wrow = p["w_off"] + i * 512 + lanes * 16
                        for j in range(bb):
                            s_lo = np.array([img[a:a + 2].view(np.float16)[0] for a in srow + j * R * 32])
                            s_hi = np.array([img[a:a + 2].view(np.float16)[0] for a in srow + j * R * 32 + 16])
                            words = np.stack([img[a:a + 16].view(np.uint32) for a in wrow + j * S * 512])
                            for ks in range(4):
                                a = dequant_word(words[:, ks], s_lo, s_hi)
                                A = np.zeros((16, 16))
                                for pp in range(4):
                                    for h in range(2):
                                        A[g8 + 8 * (pp & 1), 2 * t4 + 8 * (pp >> 1) + h] = a[pp][h].astype(np.float64)
                                for mt in range(MT):
                                    B = np.zeros((16, 8))
                                    for h in range(2):
                                        B[2 * t4 + h, lanes // 4] = bfr[mt][2 * ks, :, h]
                                        B[8 + 2 * t4 + h, lanes // 4] = bfr[mt][2 * ks + 1, :, h]
                                    acc[w, j, mt] += A @ B
            # batch end: warp j writes block j, the 8 warps' sums added in warp order
            for j in range(bb):
                for mt in range(MT):
                    v = np.zeros((16, 8))
                    for w in range(WARPS):
                        v = v + acc[w, j, mt]
                    for tk in range(8):
                        tok = mt * 8 + tk
                        if tok < M:
                            y[tok, (bk0 + j) * 16:(bk0 + j + 1) * 16] = v[:, tk]
    return y


CASES = [
    # M, N, K, G, sms: one and two 8-token tiles, a K tail inside a step, several batches
    # (10 blocks per CTA), a CTA with a single block, G = 64 and 128
    (1, 256, 4160, 64, 2),
    (3, 160, 1024, 64, 1),
    (9, 320, 640, 64, 2),
    (16, 48, 2048, 128, 3),
    (5, 64, 4096, 64, 4),
]


@pytest.mark.parametrize("M,N,K,G,sms", CASES)
def test_ns_emulation_matches_oracle(checker, M, N, K, G, sms):
    p = plan(checker, M, N, K, G, sms)
    assert p["valid"] == 1
    rng = np.random.default_rng(M * 1000 + N + K)
    q = rng.integers(0, 16, (N, K), dtype=np.uint8)
    scales = (rng.random((K // G, N)) * 0.018 + 0.002).astype(np.float16)
    x = rng.standard_normal((M, K)).astype(np.float16)
    Wp = oracle.pack_int4(q)
    y = emulate(p, Wp, x, scales, N, K, G)
    ref = oracle.ref_gemm(x, q, scales, G).astype(np.float64)
    assert np.isfinite(y).all(), "an output was not written, or garbage leaked into it"
    err = np.abs(y - ref).max() / np.abs(ref).max()
    assert err < 1e-5, err


def test_ns_emulation_constants_match_kernel_sources():
    import re
    src = open(os.path.join(CSRC, "decode_ns_plan.h")).read()
    assert re.search(r"constexpr int kNsWarps = (\d+);", src).group(1) == str(WARPS)
    kern = open(os.path.join(CSRC, "decode_ns.cuh")).read()
    for line in [
        "for (int i = warp; i < S; i += kNsWarps) {",
        "const int q = i * M + row;",
        "const uint32_t a0 = row < M ? ra + (uint32_t)((xu ^ (q & 7)) << 4) : zero_row;",
        "const uint32_t a1 = row < M ? ra + (uint32_t)(((xu + 4) ^ (q & 7)) << 4) : zero_row;",
        "const uint32_t srow = sb + p.s_off + (uint32_t)(((i * 64) / G) * 32 + g8 * 2);",
        "const uint32_t wrow = sb + p.w_off + (uint32_t)(i * 512 + lane * 16);",
        "const uint4 w4 = lds128(wrow + (uint32_t)(j * S * 512));",
        "tma_load_3d(stage(s) + p.w_off + (uint32_t)(j * S * 512), &tw, 0, t * S, bk0 + j, full(s));",
        "tma_load_3d(stage(s) + p.x_off, &tx, 0, 0, t * S, full(s));",
    ]:
        assert line in kern, line
