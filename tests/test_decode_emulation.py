"""CPU emulation of decode_kernel's per-lane data flow, checked against the oracle.

This is the counterpart, for this package's decode kernel, of the reference's numpy
emulation of its own decode kernel (akshay919191/W4A16-GEMM tests/layout.py).  For every
CTA of the stream-K partition and every step it does three things:

1. It builds the shared-memory stage that the step's tensor copies produce (csrc/decode.cuh,
   producer warp):
   * packed words as [block][chunk][512 B];
   * activation rows as [chunk][row][128 B] with the 128-byte swizzle;
   * one scale row per chunk.
   Bytes the copies do not write hold garbage (random words, NaN scales): lanes that read
   them must not leak into y.
2. It reads the stage back through the consumer warps' own addressing: `w_lane`,
   `x_lane0/1` with `ldmatrix.x4`, `s_lane`.  The A fragments restate the same bit tricks
   (csrc/dequant.cuh): by default the exact fp16 (q - 8) * s (`dequant_word`); with
   W4A16_FLAG_FP32_SCALE and M <= 8 the unscaled integers q - 8 (`unscaled_word`), whose
   four products per chunk start from zero and are then scaled per output row by the
   chunk's scale (the rows of lanes g8 and g8 + 8).  Either way the chunk's result goes to one of 2 accumulator sets per
   block (alternating by chunk), and the sets are added and stored like the kernel's
   epilogue: straight to y for a whole group, else a partial slot that the combine kernel
   sums in CTA order.
3. It compares the emulated y with the oracle's GEMM.

Hardware facts assumed, from the PTX ISA:
* the 128-byte swizzle: 16-byte unit u of 128-byte row r sits at unit u ^ (r % 8) inside
  each 1024-byte atom;
* ldmatrix .x4: lanes 8i..8i+7 give the row addresses of matrix i, and thread T receives
  row T/4, elements 2(T%4) and 2(T%4)+1 of each matrix;
* the m16n8k16 A/B/C fragment layouts.

Products are accumulated in float64: this checks the index mapping, not the tensor cores'
rounding.  By default the result must equal the oracle (whose weights are the same fp16
values) to 1e-5; in the fp32-scale form it must equal float64 x @ ((q - 8) * s)^T to
1e-12 and lie within the north-star tolerance of the oracle.
"""
import numpy as np
import pytest

from oracle import w4a16_oracle as oracle

# csrc/decode_partition.h and csrc/decode.cuh constants
BLOCKS, BPW, WARPS, STEP, COLS, MIN_UNITS, MAX_CTAS = 16, 2, 8, 4, 256, 4, 1024


def partition(N, K, sms):
    """dc_cut (csrc/decode_partition.h): CTA count and range starts c0(c)."""
    groups, kc = (N // 16 + BLOCKS - 1) // BLOCKS, K // 64
    total = groups * kc
    ctas = min(sms, max(total // MIN_UNITS, 1), MAX_CTAS)
    return groups, kc, total, ctas, (lambda c: c * total // ctas)


def steps(c0, c1, KC):
    """DcSteps: (group, chunk, nk, ends_part) for each step of a CTA's range."""
    pos, g, kc = c0, c0 // KC, c0 % KC
    while pos < c1:
        nk = min(STEP, KC - kc, c1 - pos)
        g_step, kc_step = g, kc
        pos += nk
        kc += nk
        if kc == KC:
            kc, g = 0, g + 1
            ends = True
        else:
            ends = pos == c1
        yield g_step, kc_step, nk, ends


def f16_bits(u16):
    return np.asarray(u16, np.uint16).view(np.float16)


def dequant_word(q, s_lo, s_hi):
    """csrc/dequant.cuh dequant_word for 32 lanes: a[p] = (lo half, hi half) as fp16 arrays."""
    q = q.astype(np.uint32)
    q8 = q >> 8

    def half2(bits, magic_bias, scale):
        lo = f16_bits(bits & 0xFFFF) - np.float16(magic_bias)
        hi = f16_bits(bits >> 16) - np.float16(magic_bias)
        return (lo * scale).astype(np.float16), (hi * scale).astype(np.float16)

    return [half2((q & 0x000F000F) | 0x64006400, 1032, s_lo),
            half2((q & 0x00F000F0) | 0x54005400, 72, s_hi),
            half2((q8 & 0x000F000F) | 0x64006400, 1032, s_lo),
            half2((q8 & 0x00F000F0) | 0x54005400, 72, s_hi)]


def unscaled_word(q):
    """csrc/dequant.cuh unscaled_word for 32 lanes: a[p] = (lo half, hi half) as fp16 arrays
    of q - 8."""
    one = np.ones(32, np.float16)
    return dequant_word(q, one, one)


def build_stage(Wp4, x, scales, g, kc0, nk, N, K, G, MP, rng):
    """The stage's three regions as byte arrays, as the producer's copies leave them."""
    NB, KC = N // 16, K // 64
    box_blocks, box_chunks = min(BLOCKS, NB), min(STEP, KC)
    wimg = rng.integers(0, 256, STEP * BLOCKS * 512, dtype=np.uint8)        # stale ring contents
    for b in range(box_blocks):
        for j in range(box_chunks):
            nb, kc = g * BLOCKS + b, kc0 + j
            words = Wp4[nb, kc] if nb < NB and kc < KC else np.zeros((32, 4), np.uint32)
            off = (b * box_chunks + j) * 512
            wimg[off:off + 512] = words.astype(np.uint32).reshape(-1).view(np.uint8)
    M = x.shape[0]
    xchunk = MP * 128
    ximg = np.zeros(STEP * xchunk, np.uint8)          # chunks >= box_chunks: zeroed at kernel start
    for j in range(box_chunks):
        for r in range(MP):
            row = np.zeros(64, np.float16)
            if r < M and kc0 + j < KC:
                row = x[r, (kc0 + j) * 64:(kc0 + j + 1) * 64]
            rb = row.view(np.uint8)
            for u in range(8):
                off = j * xchunk + r * 128 + ((u ^ (r % 8)) << 4)
                ximg[off:off + 16] = rb[u * 16:(u + 1) * 16]
    simg = np.full(STEP * 512, 0xFF, np.uint8)         # NaN where no copy wrote
    for j in range(nk):
        row = ((kc0 + j) * 64) // G
        vals = np.zeros(16 * box_blocks, np.float16)
        cols = np.arange(g * COLS, g * COLS + 16 * box_blocks)
        ok = cols < N
        vals[ok] = scales[row, cols[ok]]
        simg[j * 512:j * 512 + vals.size * 2] = vals.view(np.uint8)
    return wimg, ximg, simg, box_chunks


def consume(wimg, ximg, simg, box_chunks, nk, MT, acc, fs=False):
    """One step of the 8 consumer warps; acc[w][bb][ch][mt] are 16 x 8 float64 tiles."""
    lanes = np.arange(32)
    g8, t4 = lanes >> 2, lanes & 3
    xr, xu = lanes & 7, lanes >> 3
    w_blk = box_chunks * 512
    xchunk = MT * 8 * 128
    for w in range(WARPS):
        for bb in range(BPW):
            for j in range(STEP):
                # scales: columns g8 and g8 + 8 of block w*BPW + bb; zero for chunks past nk
                sa = j * 512 + (w * BPW + bb) * 32 + g8 * 2
                s_lo = simg.view(np.uint16)[sa // 2].view(np.float16) if j < nk else np.zeros(32, np.float16)
                s_hi = simg.view(np.uint16)[sa // 2 + 8].view(np.float16) if j < nk else np.zeros(32, np.float16)
                wa = w * BPW * w_blk + lanes * 16 + j * 512 + bb * w_blk
                words = np.stack([wimg[a:a + 16].view(np.uint32) for a in wa])       # [32 lanes, 4]
                srow = np.zeros(16)                       # the chunk's scale of each row of the block
                srow[g8] = s_lo.astype(np.float64)
                srow[g8 + 8] = s_hi.astype(np.float64)
                for mt in range(MT):
                    xa = j * xchunk + mt * 1024
                    b = np.zeros((8, 32, 2), np.float64)      # b[reg][thread][half]
                    for x4 in range(2):
                        addr = xa + xr * 128 + (((xu + 4 * x4) ^ xr) << 4)
                        rows = np.stack([ximg[a:a + 16].view(np.float16) for a in addr])   # [32, 8]
                        for i in range(4):
                            mat = rows[8 * i:8 * i + 8]                # matrix i: 8 rows x 8 halves
                            b[4 * x4 + i] = np.stack([mat[lanes // 4, 2 * (lanes % 4)],
                                                      mat[lanes // 4, 2 * (lanes % 4) + 1]], 1)
                    prod = np.zeros((16, 8))
                    for ks in range(4):
                        a = unscaled_word(words[:, ks]) if fs and MT == 1 else dequant_word(words[:, ks], s_lo, s_hi)
                        A = np.zeros((16, 16))
                        for p in range(4):
                            for h in range(2):
                                A[g8 + 8 * (p & 1), 2 * t4 + 8 * (p >> 1) + h] = a[p][h].astype(np.float64)
                        B = np.zeros((16, 8))
                        for h in range(2):
                            B[2 * t4 + h, lanes // 4] = b[2 * ks, :, h]
                            B[8 + 2 * t4 + h, lanes // 4] = b[2 * ks + 1, :, h]
                        prod += A @ B
                    acc[w][bb][j % 2][mt] += srow[:, None] * prod if fs and MT == 1 else prod


def emulate(Wp, x, scales, N, K, G, sms, seed=0, fs=False):
    M = x.shape[0]
    MT = 1 if M <= 8 else 2
    MP = 8 * MT
    NB = N // 16
    groups, KC, total, ctas, c0 = partition(N, K, sms)
    Wp4 = Wp.view(np.uint32).reshape(NB, KC, 32, 4)
    rng = np.random.default_rng(seed)
    y = np.full((M, N), np.nan)
    partials = {}
    for c in range(ctas):
        acc = [[[[np.zeros((16, 8)) for _ in range(MT)] for _ in range(2)] for _ in range(BPW)] for _ in range(WARPS)]
        gkc0 = c0(c) % KC
        for g, kc0, nk, ends in steps(c0(c), c0(c + 1), KC):
            whole = kc0 + nk == KC and gkc0 == 0
            wimg, ximg, simg, box_chunks = build_stage(Wp4, x, scales, g, kc0, nk, N, K, G, MP, rng)
            consume(wimg, ximg, simg, box_chunks, nk, MT, acc, fs)
            for w in range(WARPS):
                if g * BLOCKS + w * BPW >= NB:                 # the kernel skips these warps
                    for bb in range(BPW):
                        for ch in range(2):
                            for mt in range(MT):
                                acc[w][bb][ch][mt][:] = 0.0
            if ends:
                slot = 2 * c + (0 if g == c0(c) // KC else 1)
                for w in range(WARPS):
                    for bb in range(BPW):
                        nb = g * BLOCKS + w * BPW + bb
                        for mt in range(MT):
                            v = acc[w][bb][0][mt] + acc[w][bb][1][mt]          # chains in fixed order
                            acc[w][bb][0][mt] = np.zeros((16, 8))
                            acc[w][bb][1][mt] = np.zeros((16, 8))
                            if nb >= NB:
                                continue
                            for T in range(32):
                                for i in range(4):
                                    n = (T >> 2) + 8 * (i >> 1)
                                    tk = 2 * (T & 3) + (i & 1)
                                    tok = mt * 8 + tk
                                    if tok >= M:
                                        continue
                                    col = g * COLS + (w * BPW + bb) * 16 + n
                                    if whole:
                                        y[tok, col] = v[n, tk]
                                    else:
                                        partials[(slot, tok, col)] = v[n, tk]
                gkc0 = 0
    # combine kernel: split groups summed in CTA order
    for g in range(groups):
        lo, hi = g * KC, (g + 1) * KC
        cs = [c for c in range(ctas) if c0(c) < hi and c0(c + 1) > lo]
        if len(cs) == 1:
            continue
        cf = cs[0]
        slot_f = 2 * cf + (0 if g == c0(cf) // KC else 1)
        for tok in range(M):
            for col in range(g * COLS, min((g + 1) * COLS, N)):
                s = 0.0
                for c in cs:                  # decode_combine_kernel's reads: slot_f, then 2c
                    s += partials.get((slot_f if c == cf else 2 * c, tok, col), np.nan)
                y[tok, col] = s
    return y


CASES = [
    # M, N, K, G, sms: split groups (MT 1 and 2), whole groups, odd block count, K < 256
    (3, 512, 576, 64, 3),
    (9, 512, 576, 64, 3),
    (5, 272, 512, 128, 2),
    (16, 272, 192, 64, 1),
    (1, 1024, 256, 128, 148),
]


@pytest.mark.parametrize("fs", [False, True])
@pytest.mark.parametrize("M,N,K,G,sms", CASES)
def test_decode_emulation_matches_oracle(M, N, K, G, sms, fs):
    rng = np.random.default_rng(M * 1000 + N + K)
    q = rng.integers(0, 16, (N, K), dtype=np.uint8)
    scales = (rng.random((K // G, N)) * 0.018 + 0.002).astype(np.float16)
    x = rng.standard_normal((M, K)).astype(np.float16)
    Wp = oracle.pack_int4(q)
    y = emulate(Wp, x, scales, N, K, G, sms, fs=fs)
    assert np.isfinite(y).all(), "an output was not written, or garbage leaked into it"
    ref = oracle.ref_gemm(x, q, scales, G).astype(np.float64)
    if fs and M <= 8:
        # scaled after the products: the exact counterpart is float64 (q - 8) * s, without
        # the oracle's fp16 rounding of each weight
        w64 = (q.astype(np.float64) - 8.0) * np.repeat(scales.astype(np.float64).T, G, axis=1)
        exact = x.astype(np.float64) @ w64.T
        err = np.abs(y - exact).max() / np.abs(exact).max()
        assert err < 1e-12, err
        assert np.linalg.norm(y - ref) / np.linalg.norm(ref) <= 1e-3
    else:
        err = np.abs(y - ref).max() / np.abs(ref).max()
        assert err < 1e-5, err


def _header_ints(path, names):
    """Integer constants as the kernel sources define them (`constexpr int kX = 16;`)."""
    import os
    import re
    src = open(os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                            "w4a16-gemm_b200", "csrc", path)).read()
    out = {}
    for name in names:
        m = re.search(r"constexpr int %s = (\d+);" % name, src)
        assert m, f"{name} not found as a literal in {path}"
        out[name] = int(m.group(1))
    return out


def test_emulation_constants_match_kernel_sources():
    """The emulation's constants are the kernel's: a change there must be mirrored here."""
    part = _header_ints("decode_partition.h", ["kDcBlocks", "kDcStep", "kDcMaxCTAs", "kDcMinUnits"])
    assert (part["kDcBlocks"], part["kDcStep"], part["kDcMaxCTAs"], part["kDcMinUnits"]) == \
        (BLOCKS, STEP, MAX_CTAS, MIN_UNITS)
    assert _header_ints("decode.cuh", ["kDcBPW"])["kDcBPW"] == BPW
    assert BLOCKS // BPW == WARPS and BLOCKS * 16 == COLS


def test_emulation_index_expressions_match_kernel_source():
    """The addressing the emulation restates is the kernel's, expression for expression."""
    import os
    src = open(os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                            "w4a16-gemm_b200", "csrc", "decode.cuh")).read()
    for line in [
        "const uint32_t w_lane = (uint32_t)warp * BPW * w_blk + lane * 16;",
        "const uint32_t x_lane0 = C::W_BYTES + xr * 128 + ((xu ^ xr) << 4);",
        "const uint32_t x_lane1 = C::W_BYTES + xr * 128 + (((xu + 4) ^ xr) << 4);",
        "const uint32_t s_lane = (uint32_t)(C::W_BYTES + C::X_BYTES + warp * BPW * 32 + g8 * 2);",
        "wv[jj][bb] = lds128(wb + (jb + jj) * 512 + bb * w_blk);",
        "const uint32_t xa = sb + (jb + jj) * C::X_CHUNK + mt * 1024;",
        "unscaled_word(wq, a);",
        "if (ks == 0) mma_16816_zero(cc[jj][bb][mt], a, b[jj][mt][0], b[jj][mt][1]);",
        "else mma_16816(cc[jj][bb][mt], a, b[jj][mt][2 * ks], b[jj][mt][2 * ks + 1]);",
        "float& d = acc[bb][(jb + jj) % CH][mt][i];",
        "d = fmaf(i < 2 ? f_lo[bb][jb + jj] : f_hi[bb][jb + jj], cc[jj][bb][mt][i], d);",
        "dequant_word(wq, h_lo[bb][jb + jj], h_hi[bb][jb + jj], a);",
        "mma_16816(acc[bb][(jb + jj) % CH][mt], a, b[jj][mt][2 * ks], b[jj][mt][2 * ks + 1]);",
        "constexpr bool SCALE_AFTER = FP32_SCALE && MT == 1;",
        "const int colb = (warp * BPW + bb) * 16 + g8;",
        "const int tok = mt * 8 + 2 * t4 + (i & 1);",
        "const int dc = 8 * (i >> 1);",
        "const bool whole = st.kc + nk == KC && gkc0 == 0;",
        "v[i] = c <= cl ? __ldcg(p + (size_t)(c == cf ? slot_f : 2 * c) * kDcSlotFloats) : 0.f;",
    ]:
        assert line in src, line
