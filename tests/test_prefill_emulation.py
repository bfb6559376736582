"""CPU emulation of prefill_kernel's index mapping, checked against the oracle.

The counterpart, for this package's tcgen05 prefill kernel, of the reference's numpy
emulation of its own prefill kernel (akshay919191/W4A16-GEMM tests/layout_prefill.py).
One CTA walks every (token tile, 128-row tile) and every pipeline stage as prefill_kernel
does (csrc/prefill.cuh); a stage holds KCH 64-wide K chunks (KCH = pf_kch(TOK): 6, 6, 3, 2
for 32, 64, 128, 256-token tiles; a last stage may hold fewer):

* Dequant warps 2..9 each take n16 block `nbl = 2 (warp & 3) + (qi & 1)` of every chunk's
  packed words and scales ([block][chunk][512 B] and [chunk][128] in the stage). They
  dequantise with the kernel's bit tricks and store each chunk's 16 registers with
  `tcgen05.st.16x128b.x8` into the A ring: TMEM lane base 16 nbl, columns
  A_COL0 + slot * 32 KCH + 32 chunk.
* The MMA of each chunk's 16-wide k slices reads A from the chunk's TMEM columns + 8 k16.
  It reads B as the chunk's activation rows, through a K-major 128-byte-swizzle descriptor
  advanced by 32 bytes per slice. It accumulates into columns b * TOK of the fp32
  accumulator, overwriting on the first slice of a tile, in K order.
* Epilogue warp (quarter q = warp & 3, part h) reads TMEM lanes 32q..32q+31 and token
  columns h * TOK/4 .. (h + 1) * TOK/4 - 1 (channel n = 128 tn + 32q + lane); lanes 2i and
  2i + 1 trade halves, and the even lane stores token j, the odd lane token j + 1, each as
  one 4-byte pair of channels (n0, n0 + 1), guarded by N and M.

Hardware facts assumed, from the PTX ISA:
* tcgen05.st .16x128b: thread T's register 2j goes to lane T/4, column 4j + T%4, and
  register 2j+1 to lane T/4 + 8;
* a warp may access only TMEM lanes 32 (warp % 4) .. +31; the emulation asserts this for
  every access;
* an A operand in TMEM holds row i in lane i, two fp16 K elements per column;
* the swizzled descriptor reads the activation rows as B[k][token] = x[token][k].

The emulation also checks that every A column an MMA reads was written in that k-step,
that no store touches the accumulator columns, and that every y element is written once.
"""
import numpy as np
import pytest

from oracle import w4a16_oracle as oracle

ROWS, DQ_WARP0, DQ_WARPS, EPI_WARP0, EPI_WARPS = 128, 2, 8, 10, 16


def pf_kch(TOK):
    return 6 if TOK <= 64 else 3 if TOK == 128 else 2


def cfg(TOK):
    accs = 2 if TOK <= 128 else 1
    a_col0 = accs * TOK
    a_cols = 32 * pf_kch(TOK)
    return accs, a_col0, min((512 - a_col0) // a_cols, 8), pf_kch(TOK), a_cols


def dequant16(words, s_lo, s_hi):
    """dequant_word on a lane's 4 words: 16 32-bit registers, each 2 fp16 (lo, hi)."""
    regs = []
    for q in words.astype(np.uint32):
        q8 = q >> 8
        for bits, bias, s in ((q & 0x000F000F) | 0x64006400, 1032, s_lo), \
                             ((q & 0x00F000F0) | 0x54005400, 72, s_hi), \
                             ((q8 & 0x000F000F) | 0x64006400, 1032, s_lo), \
                             ((q8 & 0x00F000F0) | 0x54005400, 72, s_hi):
            lo = np.array([bits & 0xFFFF], np.uint16).view(np.float16)[0] - np.float16(bias)
            hi = np.array([bits >> 16], np.uint16).view(np.float16)[0] - np.float16(bias)
            regs.append((np.float16(lo * s), np.float16(hi * s)))
    return regs


def check_lane(warp, lane):
    assert 32 * (warp % 4) <= lane < 32 * (warp % 4) + 32, f"warp {warp} touched TMEM lane {lane}"


def emulate(Wp, x, scales, N, K, G, TOK):
    M = x.shape[0]
    NB, KC = N // 16, K // 64
    Wp4 = Wp.view(np.uint32).reshape(NB, KC, 32, 4)
    accs, a_col0, na, kch, a_cols = cfg(TOK)
    KT = (KC + kch - 1) // kch
    n_tiles, t_tiles = (N + ROWS - 1) // ROWS, (M + TOK - 1) // TOK
    tmem = np.full((ROWS, 512, 2), np.nan)                  # [lane][column][half]
    y = np.full((M, N), np.nan)
    written = np.zeros((M, N), np.int32)
    it = 0
    for tc, tile in enumerate(range(n_tiles * t_tiles)):
        tt, tn = tile // n_tiles, tile % n_tiles
        b = tc % accs
        for kt in range(KT):
            a = it % na
            it += 1
            nch = min(kch, KC - kt * kch)
            KB = min(kch, KC)
            # the stage's weight box {128 words, KB chunks, 8 blocks} as the tensor copy lays it
            # out: [block][chunk][32 lanes x 4 words], zeros past K and past N
            wimg = np.zeros(8 * KB * 128, np.uint32)
            for nbl in range(8):
                for jj in range(KB):
                    if tn * 8 + nbl < NB and kt * kch + jj < KC:
                        wimg[(nbl * KB + jj) * 128:(nbl * KB + jj + 1) * 128] = Wp4[tn * 8 + nbl, kt * kch + jj].reshape(-1)
            fresh = np.zeros((ROWS, a_cols), bool)
            xts = []
            for j in range(nch):
                kc = kt * kch + j
                # chunk j of the stage: its scale row and x rows; the packed words are read from
                # the stage image at the dequant warps' address (nbl * KB + j) * 512 + lane * 16
                srow = np.zeros(ROWS, np.float16)
                cols = np.arange(tn * ROWS, tn * ROWS + ROWS)
                srow[cols < N] = scales[(kc * 64) // G, cols[cols < N]]
                xt = np.zeros((TOK, 64), np.float64)
                rows = np.arange(tt * TOK, tt * TOK + TOK)
                xt[rows < M] = x[rows[rows < M], kc * 64:(kc + 1) * 64]
                xts.append(xt)
                # dequant warps -> TMEM A slot, chunk j's 32 columns
                for warp in range(DQ_WARP0, DQ_WARP0 + DQ_WARPS):
                    qi = (warp - 2) >> 2
                    nbl = 2 * (warp & 3) + (qi & 1)
                    for L in range(32):
                        g = L >> 2
                        off = ((nbl * KB + j) * 512 + L * 16) // 4
                        regs = dequant16(wimg[off:off + 4], srow[nbl * 16 + g], srow[nbl * 16 + g + 8])
                        for R, (lo, hi) in enumerate(regs):
                            lane = 16 * nbl + L // 4 + 8 * (R % 2)
                            col = a_col0 + a * a_cols + j * 32 + 4 * (R // 2) + (L % 4)
                            check_lane(warp, lane)
                            assert a_col0 <= col < 512, "A store outside the A ring"
                            tmem[lane, col] = (lo, hi)
                            fresh[lane, col - a_col0 - a * a_cols] = True
            assert fresh[:, :32 * nch].all(), "an A column the MMA reads was not written this stage"
            # MMA: per chunk, 4 slices of 16 k, in K order
            for j in range(nch):
                for k16 in range(4):
                    cols_a = a_col0 + a * a_cols + j * 32 + k16 * 8 + np.arange(8)
                    A = tmem[:, cols_a, :].reshape(ROWS, 16)        # lane i = row i, 2 k per column
                    B = xts[j][:, k16 * 16:(k16 + 1) * 16].T        # [16 k, TOK]
                    D = tmem[:, b * TOK:(b + 1) * TOK, 0]
                    tmem[:, b * TOK:(b + 1) * TOK, 0] = A @ B + (D if (kt | j | k16) != 0 else 0.0)
        # epilogue warps: each lane loads its channel's tokens; lanes 2i and 2i + 1 then trade
        # halves, the even lane storing token j and the odd lane token j + 1 of both channels
        cw = TOK // (EPI_WARPS // 4)
        for warp in range(EPI_WARP0, EPI_WARP0 + EPI_WARPS):
            q, h = warp & 3, (warp - EPI_WARP0) >> 2
            vals = np.zeros((32, cw))
            for L in range(32):
                lane = 32 * q + L
                check_lane(warp, lane)
                vals[L] = tmem[lane, b * TOK + h * cw:b * TOK + (h + 1) * cw, 0]
            tok0 = tt * TOK + h * cw
            for L in range(32):
                p = L & 1
                n0 = tn * ROWS + 32 * q + L - p            # the pair's even channel
                for j in range(0, cw, 2):
                    row = tok0 + j + p
                    if n0 < N and row < M:
                        for c in range(2):                  # channels n0, n0 + 1 of one 4-byte store
                            y[row, n0 + c] = vals[L - p + c, j + p]
                            written[row, n0 + c] += 1
    assert (written == 1).all(), "y elements written zero or several times"
    return y


CASES = [
    # M, N, K, G, TOK: ragged M and N, every token tile, both group sizes; stages of
    # 6, 6 + 2, 3 + 1 and 2 + 1 chunks (a last partial stage), one chunk only
    (17, 208, 384, 64, 32),
    (100, 272, 512, 128, 64),
    (129, 128, 256, 64, 128),
    (40, 384, 320, 64, 256),
    (20, 144, 64, 64, 128),
]


@pytest.mark.parametrize("M,N,K,G,TOK", CASES)
def test_prefill_emulation_matches_oracle(M, N, K, G, TOK):
    rng = np.random.default_rng(M * 7 + N + K + TOK)
    q = rng.integers(0, 16, (N, K), dtype=np.uint8)
    scales = (rng.random((K // G, N)) * 0.018 + 0.002).astype(np.float16)
    x = rng.standard_normal((M, K)).astype(np.float16)
    y = emulate(oracle.pack_int4(q), x, scales, N, K, G, TOK)
    ref = oracle.ref_gemm(x, q, scales, G).astype(np.float64)
    assert np.isfinite(y).all()
    err = np.abs(y - ref).max() / np.abs(ref).max()
    assert err < 1e-5, err


def test_emulation_constants_match_kernel_sources():
    """The emulation's warp layout and TMEM plan are the kernel's (csrc/prefill.cuh)."""
    import os
    import re
    src = open(os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                            "w4a16-gemm_b200", "csrc", "prefill.cuh")).read()

    def define(name):
        return int(re.search(r"#define %s (\d+)" % name, src).group(1))

    phases, epi = define("W4A16_PF_DQ_PHASES"), define("W4A16_PF_EPI_WARPS")
    assert (2, 8 * phases, 2 + 8 * phases, epi) == (DQ_WARP0, DQ_WARPS, EPI_WARP0, EPI_WARPS)
    assert int(re.search(r"constexpr int kPfRows = (\d+);", src).group(1)) == ROWS
    assert "ACCS = TOK <= 128 ? 2 : 1" in src and "A_COL0 = ACCS * TOK" in src
    assert "A_COLS = 32 * KCH" in src and "(512 - A_COL0) / A_COLS < 8 ? (512 - A_COL0) / A_COLS : 8" in src
    assert "return tok <= 64 ? W4A16_PF_KCH_SMALL : tok == 128 ? W4A16_PF_KCH_128 : 2;" in src
    assert [define("W4A16_PF_KCH_SMALL"), define("W4A16_PF_KCH_128")] == [pf_kch(32), pf_kch(128)]
    assert "const int nbl = 2 * (warp & 3) + (qi & 1);" in src
    assert "tmem_st_16x128b_x8(tmem + lane_field + (uint32_t)(C::A_COL0 + a * C::A_COLS + j * 32), r[j]);" in src
    assert "w[j] = lds128(sbw + (uint32_t)((nbl * KB + j) * 512 + lane * 16));" in src
    assert "uint32_t* y32 = reinterpret_cast<uint32_t*>(static_cast<__half*>(yv) + (size_t)(tok0 + p) * N + n0);" in src
    assert "const uint32_t out = p ? __byte_perm(got, w, 0x7610) : __byte_perm(w, got, 0x5410);" in src
    assert "if (n0 < N && tok0 + j + p < M) y32[(size_t)j * N / 2] = out;" in src
    assert ("tc_mma_ts(d, at + j * 32 + k16 * 8, pf_sw128_desc(xa + j * C::X_CHUNK + k16 * 32), idesc,\n"
            "                                      (kt | j | k16) != 0);") in src
