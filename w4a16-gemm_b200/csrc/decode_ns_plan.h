// Work split and shared-memory plan of decode_ns_kernel (decode_ns.cuh): which n16 blocks
// each CTA owns, how it batches them, how many 64-wide K chunks a pipeline step covers,
// and where everything sits in shared memory.  Plain C++ shared by the host planner, the
// kernel and a host-only checker that compiles it without nvcc.
#pragma once
#include <stddef.h>
#include <stdint.h>

#if defined(__CUDACC__)
#define W4A16_NS_HD __host__ __device__
#else
#define W4A16_NS_HD
#endif

namespace w4a16 {

constexpr int kNsWarps = 8;                 // consumer warps: warp w takes chunks w, w+8, ... of a step
constexpr int kNsMaxBatch = 8;              // n16 blocks per batch (accumulators held per block)
constexpr int kNsSmemBudget = 227 * 1024;   // opt-in dynamic shared memory per CTA on sm_100
constexpr int kNsMaxStages = 8;

struct NsPlan {
    int ctas;        // CTAs (<= #SMs, <= n16 blocks)
    int nb;          // n16 blocks (N / 16)
    int bmax;        // largest batch of any CTA (blocks)
    int S;           // 64-wide K chunks per pipeline step (multiple of kNsWarps)
    int R;           // scale rows per step (S * 64 / G)
    int stages;      // pipeline depth
    uint32_t w_off, x_off, s_off, stage_bytes;   // inside a stage: packed words, activations, scales
    uint32_t red_off, zero_off, bar_off;         // after the stages: reduction buffer, zero row, barriers
    uint32_t smem;                               // dynamic shared memory to request (with alignment slack)
    bool valid;

    // First n16 block of CTA c (c in [0, ctas]): an even split, any two CTAs within one block.
    W4A16_NS_HD int b0(int c) const { return (int)(((long long)c * nb) / ctas); }
    // Batches of a CTA that owns `blocks` blocks, and the first block (relative) of batch k.
    W4A16_NS_HD int batches(int blocks) const { return (blocks + kNsMaxBatch - 1) / kNsMaxBatch; }
    W4A16_NS_HD int batch_lo(int blocks, int nbat, int k) const { return (int)(((long long)k * blocks) / nbat); }
};

// Bytes of the cross-warp reduction buffer: a float4 per (warp, block, 8-token tile, lane).
inline uint32_t ns_red_bytes(int bmax, int mt) { return (uint32_t)(kNsWarps * bmax * mt * 32 * 16); }

// The plan of an M x N x K GEMM (M <= 16) on `num_sms` SMs.  The step covers the most K
// chunks (64, 32, 16 or 8) whose stage still leaves at least 4 stages in shared memory (3 if
// even 8 chunks do not), and never more chunks than K has.
inline NsPlan ns_plan(int M, int N, int K, int G, int num_sms) {
    NsPlan p{};
    const int mt = M <= 8 ? 1 : 2;
    p.nb = N / 16;
    p.ctas = p.nb < num_sms ? p.nb : num_sms;
    p.valid = p.ctas >= 1 && M >= 1 && M <= 16 && K >= 64 && (G == 64 || G == 128);
    if (!p.valid) return p;
    // a CTA owns floor or ceil(nb / ctas) blocks; the largest batch of either count
    p.bmax = 0;
    for (int blocks : {p.nb / p.ctas, (p.nb + p.ctas - 1) / p.ctas}) {
        if (blocks < 1) continue;
        const int nbat = p.batches(blocks);
        const int big = (blocks + nbat - 1) / nbat;
        p.bmax = big > p.bmax ? big : p.bmax;
    }
    const int kc = K / 64;
    const uint32_t red = ns_red_bytes(p.bmax, mt);
    const uint32_t fixed = 1024 /* alignment slack */ + red + 128 /* zero row */ + 2 * kNsMaxStages * 8;
    const uint32_t ring = (uint32_t)kNsSmemBudget - fixed;
    auto stage_bytes = [&](int S) {
        const uint32_t w = (uint32_t)(p.bmax * S * 512), x = (uint32_t)(S * M * 128);
        const uint32_t s = (uint32_t)(p.bmax * (S * 64 / G) * 32);
        return (w + x + s + 1023u) / 1024u * 1024u;
    };
    const int kc8 = (kc + kNsWarps - 1) / kNsWarps * kNsWarps;   // K rounded up to whole steps of 8
    p.S = kNsWarps;
    for (int S : {64, 32, 16}) {
        if (S > kc8) continue;
        if (stage_bytes(S) * 4 <= ring) { p.S = S; break; }
    }
    p.R = p.S * 64 / G;
    p.stage_bytes = stage_bytes(p.S);
    int st = (int)(ring / p.stage_bytes);
    p.stages = st > kNsMaxStages ? kNsMaxStages : st;
    p.valid = p.stages >= 3;
    p.w_off = 0;
    p.x_off = (uint32_t)(p.bmax * p.S * 512);
    p.s_off = p.x_off + (uint32_t)(p.S * M * 128);
    p.red_off = (uint32_t)p.stages * p.stage_bytes;
    p.zero_off = p.red_off + red;
    p.bar_off = p.zero_off + 128;
    p.smem = 1024 + p.bar_off + (uint32_t)(2 * p.stages * 8);
    return p;
}

// Busiest-CTA work of the two decode kernels in units of one n16 block x one 64-wide
// chunk (512 bytes of packed words).  The stream-K kernel splits the units evenly but pays
// for combining split groups: a second launch and its release gaps, about as long as
// streaming kNsCombineUnits units on one SM (measured on B200: 2-3 us per GEMM).
constexpr long long kNsCombineUnits = 170;
inline bool ns_preferred(int N, int K, int num_sms, bool streamk_splits) {
    const long long nb = N / 16, kc = K / 64;
    const long long ctas = nb < num_sms ? nb : num_sms;
    if (ctas < 1) return false;
    const long long ns = (nb + ctas - 1) / ctas * kc;
    const long long sk = (nb * kc + num_sms - 1) / num_sms + (streamk_splits ? kNsCombineUnits : 0);
    return ns <= sk;
}

}  // namespace w4a16
