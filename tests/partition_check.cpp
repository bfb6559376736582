// Host-only check of the decode kernel's stream-K partition (csrc/decode_partition.h),
// built with g++ by tests/test_partition_cpu.py.  For a sweep of (N, K, #SMs) it walks
// every CTA's range exactly as decode_kernel does (DcSteps, the "whole group" test, the
// partial slot) and checks what decode_kernel and decode_combine_kernel rely on:
//   * the CTA ranges tile the (group, chunk) units, each unit exactly once, in steps of
//     at most kDcStep chunks that never cross a group or range boundary;
//   * first_cta / last_cta (closed forms) equal the brute-force definitions;
//   * a group inside one CTA is written once to y and no partial is written for it;
//   * a split group gets one partial from each of CTAs first..last, in distinct slots
//     below 2 * ctas, at exactly the slots the combine kernel reads;
//   * the split flag and the workspace size agree with the partials written;
//   * the tensor-copy coordinates the producer issues per step (decode_kernel's
//     issue_weights and activation copy) start inside the tensors, and every innermost
//     coordinate is a multiple of 16 bytes (the TMA alignment rule).
// This is the same role as the reference's numpy emulation of its kernel's data flow
// (akshay919191/W4A16-GEMM tests/layout.py), for this kernel's work split.
#include <cstdio>
#include <cstdlib>
#include <vector>

#include "decode_partition.h"

using namespace w4a16;

static int g_fail = 0;
static long g_cases = 0;

#define CHECK(cond, ...)                                                    \
    do {                                                                    \
        if (!(cond)) {                                                      \
            if (g_fail < 20) {                                              \
                std::printf("FAIL N=%d K=%d sms=%d: ", N, K, sms);          \
                std::printf(__VA_ARGS__);                                   \
                std::printf("\n");                                          \
            }                                                               \
            ++g_fail;                                                       \
            return;                                                         \
        }                                                                   \
    } while (0)

// Largest c in [0, ctas) with pred(c0(c)), c0 being non-decreasing and pred monotone.
template <typename Pred>
static int largest_c(const DcPartition& p, Pred pred) {
    int lo = 0, hi = p.ctas - 1;
    while (lo < hi) {
        const int mid = lo + (hi - lo + 1) / 2;
        if (pred(p.c0(mid))) lo = mid;
        else hi = mid - 1;
    }
    return lo;
}

static void check_closed_forms(const DcPartition& p, int g, int N, int K, int sms) {
    const long long lo = (long long)g * p.kc, hi = (long long)(g + 1) * p.kc;
    const int f = largest_c(p, [&](int v) { return v <= lo; });
    const int l = largest_c(p, [&](int v) { return v < hi; });
    CHECK(p.first_cta(g) == f, "first_cta(%d) = %d, expected %d", g, p.first_cta(g), f);
    CHECK(p.last_cta(g) == l, "last_cta(%d) = %d, expected %d", g, p.last_cta(g), l);
}

// The copies one step issues, as decode_kernel's producer does: packed words at
// (0, kc, g * kDcBlocks) of [NB][KC][128] int32, activations at (0, 0, kc) of [KC][M][64]
// fp16, and per chunk j < nk the scale row ((kc + j) * 64) / G at column g * kDcCols of
// [K/G][N] fp16.
static void check_step_copies(int g, int kc, int nk, int N, int K, int sms, int G) {
    const int NB = N / 16, KC = K / 64;
    CHECK(kc >= 0 && kc < KC, "weight/activation chunk coordinate %d of %d", kc, KC);
    CHECK(g * kDcBlocks >= 0 && g * kDcBlocks < NB, "weight block coordinate %d of %d", g * kDcBlocks, NB);
    // the innermost coordinate of the word and activation copies is always 0
    const long long col = (long long)g * kDcCols;
    CHECK(col < N && (col * 2) % 16 == 0, "scale column %lld (N = %d)", col, N);
    for (int j = 0; j < nk; ++j) {
        const int row = ((kc + j) * 64) / G;
        CHECK(row >= 0 && row < K / G, "scale row %d of %d", row, K / G);
    }
}

static void check_shape(int N, int K, int sms) {
    ++g_cases;
    const int fails_before = g_fail;
    const DcPartition p = dc_cut(N, K, sms);
    const long long total = (long long)((N / 16 + kDcBlocks - 1) / kDcBlocks) * (K / 64);
    CHECK(p.valid == (total > 0 && total < (1ll << 31)), "valid flag");
    if (!p.valid) return;
    const int cap = total / kDcMinUnits > 0 ? (int)(total / kDcMinUnits) : 1;
    CHECK(p.ctas >= 1 && p.ctas <= sms && p.ctas <= cap && p.ctas <= kDcMaxCTAs, "ctas = %d", p.ctas);
    CHECK(p.c0(0) == 0 && p.c0(p.ctas) == p.total, "range ends");
    const int min_units = p.total < kDcMinUnits ? p.total : kDcMinUnits;
    for (int c = 0; c < p.ctas; ++c)
        CHECK(p.c0(c + 1) - p.c0(c) >= min_units, "CTA %d has %d units", c, p.c0(c + 1) - p.c0(c));

    if (p.total > 4000000) {   // too large to walk: the closed forms on sampled groups
        const int gs[] = {0, 1, p.groups / 3, p.groups / 2, p.groups - 2, p.groups - 1};
        for (int g : gs)
            if (g >= 0 && g < p.groups) check_closed_forms(p, g, N, K, sms);
        return;
    }
    for (int g = 0; g < p.groups && g_fail == fails_before; ++g) check_closed_forms(p, g, N, K, sms);
    if (g_fail != fails_before) return;

    const int KC = p.kc;
    std::vector<unsigned char> covered(p.total, 0);
    std::vector<int> direct(p.groups, 0);
    std::vector<std::vector<int>> writer_cta(p.groups), writer_slot(p.groups);
    std::vector<int> slot_owner(2 * p.ctas, -1);
    for (int c = 0; c < p.ctas; ++c) {
        DcSteps st;
        st.start(p.c0(c), p.c0(c + 1), KC);
        int gkc0 = st.kc;
        while (st.more()) {
            const int nk = st.nk(KC);
            CHECK(nk >= 1 && nk <= kDcStep && st.kc + nk <= KC && st.pos + nk <= st.end, "step of %d chunks", nk);
            for (int G : {64, 128})
                if (K % G == 0) check_step_copies(st.g, st.kc, nk, N, K, sms, G);
            for (int j = 0; j < nk; ++j) {
                const int u = st.g * KC + st.kc + j;
                CHECK(u == st.pos + j, "unit order");
                CHECK(!covered[u], "unit %d covered twice", u);
                covered[u] = 1;
            }
            const int g = st.g;
            const bool whole = st.kc + nk == KC && gkc0 == 0;
            if (st.advance(nk, KC)) {
                if (whole) {
                    ++direct[g];
                } else {
                    const int s = p.slot(c, g);
                    CHECK(s >= 0 && s < 2 * p.ctas, "slot %d of CTA %d", s, c);
                    CHECK(slot_owner[s] < 0, "slot %d written by CTAs %d and %d", s, slot_owner[s], c);
                    slot_owner[s] = c;
                    writer_cta[g].push_back(c);
                    writer_slot[g].push_back(s);
                }
                gkc0 = 0;
            }
        }
    }
    for (int u = 0; u < p.total; ++u) CHECK(covered[u], "unit %d not covered", u);

    bool any_split = false;
    for (int g = 0; g < p.groups; ++g) {
        const int cf = p.first_cta(g), cl = p.last_cta(g);
        if (cf == cl) {
            CHECK(direct[g] == 1 && writer_cta[g].empty(), "group %d in one CTA: %d direct writes, %d partials",
                  g, direct[g], (int)writer_cta[g].size());
            continue;
        }
        any_split = true;
        CHECK(direct[g] == 0, "split group %d written directly", g);
        CHECK((int)writer_cta[g].size() == cl - cf + 1, "split group %d: %d partials for CTAs %d..%d", g,
              (int)writer_cta[g].size(), cf, cl);
        for (int i = 0; i < (int)writer_cta[g].size(); ++i) {
            const int c = cf + i;
            // decode_combine_kernel reads slot(cf, g) for the first CTA and 2c for the others
            const int read_slot = c == cf ? p.slot(cf, g) : 2 * c;
            CHECK(writer_cta[g][i] == c && writer_slot[g][i] == read_slot,
                  "group %d: partial %d from CTA %d in slot %d, combine reads CTA %d slot %d", g, i,
                  writer_cta[g][i], writer_slot[g][i], c, read_slot);
        }
    }
    CHECK(any_split == p.split, "split flag %d, walk found %d", (int)p.split, (int)any_split);
    const size_t need = any_split ? (size_t)2 * p.ctas * kDcSlotFloats * 4 : 0;
    CHECK(dc_workspace_bytes(p) == need, "workspace bytes");
}

int main() {
    const int sms_small[] = {1, 2, 3, 5, 148};
    for (int N = 16; N <= 2048; N += 16)
        for (int K : {64, 128, 192, 256, 320, 512, 1024})
            for (int sms : sms_small) check_shape(N, K, sms);

    const int Ns[] = {16, 64, 240, 256, 272, 1024, 1040, 3584, 4096, 4112, 6144, 7168, 14336, 28672, 57344};
    const int Ks[] = {64, 448, 512, 2048, 3584, 4096, 4160, 8192, 14336, 28672};
    const int sms_big[] = {1, 7, 64, 132, 148, 160, 296, 1024, 4096};
    for (int N : Ns)
        for (int K : Ks)
            for (int sms : sms_big) check_shape(N, K, sms);

    // sizes near the 32-bit unit limit: closed forms only; past it the partition is invalid
    check_shape(262144, 64 * (1 << 20), 148);         // 2^30 units
    check_shape(16 * 16 * 2047, 64 * (1 << 20), 1024);  // just under 2^31
    check_shape(16 * 16 * 2048, 64 * (1 << 20), 148);   // 2^31: invalid

    if (g_fail) {
        std::printf("%d failures in %ld cases\n", g_fail, g_cases);
        return 1;
    }
    std::printf("ok %ld cases\n", g_cases);
    return 0;
}
