// Host-only check of decode_ns_kernel's plan (csrc/decode_ns_plan.h), built with g++ by
// tests/test_decode_ns_cpu.py.  With no arguments it sweeps (M, N, K, G, #SMs) and checks
// what the kernel relies on:
//   * the CTAs' block ranges tile the n16 blocks exactly once, each CTA owning at least
//     one block and any two CTAs within one block of each other;
//   * a CTA's batches tile its blocks, each of at most bmax <= 8 blocks;
//   * a step covers S chunks, a multiple of the 8 consumer warps, at most 64, and R = S*64/G
//     scale rows; there are at least 3 stages, and everything fits the 227 KB of shared
//     memory with each region on the alignment its accesses need (the activation box on
//     1024 bytes for the 128-byte swizzle, 16-byte vectors elsewhere, 8-byte barriers);
//   * every tensor copy a step issues starts inside its tensor: the packed-word box at
//     (0, t*S, block), the activation box at (0, 0, t*S) and the scale box at
//     (block*16, t*S*64/G), innermost coordinates on 16-byte boundaries (the TMA rule).
// With arguments "M N K G sms" it prints that shape's plan as one JSON line (the CPU
// emulation of the kernel reads its layout from there).
#include <cstdio>
#include <cstdlib>
#include <vector>

#include "decode_ns_plan.h"

using namespace w4a16;

static int g_fail = 0;
static long g_cases = 0;

#define CHECK(cond, ...)                                                          \
    do {                                                                          \
        if (!(cond)) {                                                            \
            if (g_fail < 20) {                                                    \
                std::printf("FAIL M=%d N=%d K=%d G=%d sms=%d: ", M, N, K, G, sms); \
                std::printf(__VA_ARGS__);                                         \
                std::printf("\n");                                                \
            }                                                                     \
            ++g_fail;                                                             \
            return;                                                               \
        }                                                                         \
    } while (0)

static void check_shape(int M, int N, int K, int G, int sms) {
    ++g_cases;
    const NsPlan p = ns_plan(M, N, K, G, sms);
    CHECK(p.valid, "plan not valid");
    const int NB = N / 16, KC = K / 64, mt = M <= 8 ? 1 : 2;
    CHECK(p.nb == NB && p.ctas >= 1 && p.ctas <= sms && p.ctas <= NB, "ctas %d", p.ctas);
    CHECK(p.b0(0) == 0 && p.b0(p.ctas) == NB, "block range ends");
    int lo = NB, hi = 0, bmax = 0;
    for (int c = 0; c < p.ctas; ++c) {
        const int b = p.b0(c + 1) - p.b0(c);
        lo = b < lo ? b : lo;
        hi = b > hi ? b : hi;
        const int nbat = p.batches(b);
        CHECK(p.batch_lo(b, nbat, 0) == 0 && p.batch_lo(b, nbat, nbat) == b, "batches of CTA %d", c);
        for (int k = 0; k < nbat; ++k) {
            const int bb = p.batch_lo(b, nbat, k + 1) - p.batch_lo(b, nbat, k);
            CHECK(bb >= 1 && bb <= p.bmax && bb <= kNsMaxBatch, "batch %d of CTA %d has %d blocks", k, c, bb);
            bmax = bb > bmax ? bb : bmax;
        }
    }
    CHECK(lo >= 1 && hi - lo <= 1, "blocks per CTA from %d to %d", lo, hi);
    CHECK(bmax == p.bmax, "bmax %d, largest batch %d", p.bmax, bmax);
    CHECK(p.S % kNsWarps == 0 && p.S >= kNsWarps && p.S <= 64, "S = %d", p.S);
    CHECK(p.R == p.S * 64 / G && p.R <= 256, "R = %d", p.R);
    CHECK(p.stages >= 3 && p.stages <= kNsMaxStages, "stages %d", p.stages);
    const uint32_t w = (uint32_t)(p.bmax * p.S * 512), x = (uint32_t)(p.S * M * 128), s = (uint32_t)(p.bmax * p.R * 32);
    CHECK(p.w_off == 0 && p.x_off == w && p.s_off == w + x && p.stage_bytes >= w + x + s, "stage layout");
    CHECK(p.x_off % 1024 == 0 && p.stage_bytes % 1024 == 0, "activation box alignment");
    CHECK(p.s_off % 16 == 0, "scale alignment");
    CHECK(p.red_off == (uint32_t)p.stages * p.stage_bytes && p.red_off % 16 == 0, "reduction buffer");
    CHECK(p.zero_off == p.red_off + ns_red_bytes(p.bmax, mt) && p.zero_off % 16 == 0, "zero row");
    CHECK(p.bar_off == p.zero_off + 128 && p.bar_off % 8 == 0, "barriers");
    CHECK(p.smem == 1024 + p.bar_off + 2 * p.stages * 8 && p.smem <= (uint32_t)kNsSmemBudget, "smem %u", p.smem);
    // the copies of every step
    const int nsteps = (KC + p.S - 1) / p.S;
    for (int t = 0; t < nsteps; ++t) {
        CHECK(t * p.S < KC, "step %d starts past K", t);
        const int row = t * p.S * 64 / G;
        CHECK(row >= 0 && row < K / G, "scale row %d of %d", row, K / G);
    }
    for (int c = 0; c < p.ctas; ++c) {
        const int last = p.b0(c + 1) - 1;
        CHECK(last < NB && ((long long)last * 16 * 2) % 16 == 0 && last * 16 < N, "scale column of block %d", last);
    }
}

int main(int argc, char** argv) {
    if (argc == 6) {
        const int M = std::atoi(argv[1]), N = std::atoi(argv[2]), K = std::atoi(argv[3]), G = std::atoi(argv[4]),
                  sms = std::atoi(argv[5]);
        const NsPlan p = ns_plan(M, N, K, G, sms);
        std::printf("{\"valid\": %d, \"ctas\": %d, \"nb\": %d, \"bmax\": %d, \"S\": %d, \"R\": %d, \"stages\": %d, "
                    "\"w_off\": %u, \"x_off\": %u, \"s_off\": %u, \"stage_bytes\": %u, \"red_off\": %u, "
                    "\"zero_off\": %u, \"bar_off\": %u, \"smem\": %u, \"preferred\": %d}\n",
                    (int)p.valid, p.ctas, p.nb, p.bmax, p.S, p.R, p.stages, p.w_off, p.x_off, p.s_off,
                    p.stage_bytes, p.red_off, p.zero_off, p.bar_off, p.smem, (int)ns_preferred(N, K, sms, true));
        return 0;
    }
    for (int M : {1, 2, 3, 7, 8, 9, 15, 16})
        for (int G : {64, 128})
            for (int N : {16, 48, 256, 1024, 1040, 4096, 4112, 14336, 28672, 57344})
                for (int K : {128, 192, 512, 2048, 4096, 4160, 8192, 14336, 28672})
                    for (int sms : {1, 3, 64, 132, 148, 160})
                        if (K % G == 0) check_shape(M, N, K, G, sms);
    if (g_fail) {
        std::printf("%d failures in %ld cases\n", g_fail, g_cases);
        return 1;
    }
    std::printf("ok %ld cases\n", g_cases);
    return 0;
}
