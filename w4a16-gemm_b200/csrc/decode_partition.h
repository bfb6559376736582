// Stream-K partition of the decode kernel: which (256-column group, 64-wide K chunk)
// units each CTA processes, how a CTA walks its units, and where split groups leave
// their partial sums.  Plain C++ shared by the host planner, decode_kernel,
// decode_combine_kernel and a host-only checker that compiles it without nvcc.
#pragma once
#include <stddef.h>

#if defined(__CUDACC__)
#define W4A16_HD __host__ __device__
#else
#define W4A16_HD
#endif

namespace w4a16 {

constexpr int kDcBlocks = 16;                             // n16 blocks per group
constexpr int kDcCols = kDcBlocks * 16;                   // output columns per group
constexpr int kDcStep = 4;                                // 64-wide K chunks per step
constexpr int kDcSlotFloats = 16 * kDcCols;               // one partial: 16 tokens x 256 columns
constexpr int kDcMaxCTAs = 1024;
// Fewest (group, chunk) units a CTA gets: a small GEMM runs on fewer CTAs rather than
// splitting each column group over dozens of them (its copies are all in flight at once
// either way, and the combine reads fewer partials).
constexpr int kDcMinUnits = 4;

W4A16_HD inline int dc_min(int a, int b) { return a < b ? a : b; }

// Static stream-K partition over (group, chunk) pairs, identical on host and device.
struct DcPartition {
    int groups;    // 256-column groups
    int kc;        // 64-wide K chunks per group (K / 64)
    int total;     // groups * kc
    int ctas;      // CTAs (<= total)
    bool valid;    // total fits 32 bits
    bool split;    // some group is split across CTAs (a CTA boundary inside a group)
    W4A16_HD int c0(int c) const { return (int)(((long long)c * total) / ctas); }
    // First / last CTA whose range intersects group g (closed forms of "largest c with
    // c0(c) <= g*kc" and "largest c with c0(c) < (g+1)*kc"; one division each).
    W4A16_HD int first_cta(int g) const {
        const unsigned long long lo = (unsigned long long)g * kc;
        const int c = (int)(((lo + 1) * (unsigned)ctas - 1) / (unsigned)total);
        return c < ctas - 1 ? c : ctas - 1;
    }
    W4A16_HD int last_cta(int g) const {
        const unsigned long long hi = (unsigned long long)(g + 1) * kc;
        const int c = (int)((hi * (unsigned)ctas - 1) / (unsigned)total);
        return c < ctas - 1 ? c : ctas - 1;
    }
    // Workspace slot of CTA c's partial of group g (only for split groups).
    W4A16_HD int slot(int c, int g) const { return 2 * c + (g == c0(c) / kc ? 0 : 1); }
};

inline DcPartition dc_cut(int N, int K, int num_sms) {
    DcPartition p;
    p.groups = (N / 16 + kDcBlocks - 1) / kDcBlocks;
    p.kc = K / 64;
    const long long total = (long long)p.groups * p.kc;
    p.valid = total > 0 && total < (1ll << 31);
    p.total = p.valid ? (int)total : 1;
    const int cap = p.total / kDcMinUnits > 0 ? p.total / kDcMinUnits : 1;
    p.ctas = num_sms < cap ? num_sms : cap;
    if (p.ctas > kDcMaxCTAs) p.ctas = kDcMaxCTAs;
    p.split = false;
    for (int c = 1; c < p.ctas && !p.split; ++c) p.split = p.c0(c) % p.kc != 0;
    return p;
}

// Workspace: 2 fp32 partial slots per CTA (a CTA's range splits at most its first
// and its last group), only when some group is split.  Always fully written before
// it is read; no initial contents are assumed.
inline size_t dc_workspace_bytes(const DcPartition& p) {
    return p.split ? (size_t)2 * p.ctas * kDcSlotFloats * 4 : 0;
}

// Walks a CTA's chunk range [pos, end) in steps of <= kDcStep chunks that never
// cross a group boundary.
struct DcSteps {
    int pos, end, g, kc;
    W4A16_HD void start(int c0, int c1, int KC) { pos = c0; end = c1; g = c0 / KC; kc = c0 - g * KC; }
    W4A16_HD bool more() const { return pos < end; }
    W4A16_HD int nk(int KC) const { return dc_min(kDcStep, dc_min(KC - kc, end - pos)); }
    // Advances past a step of n chunks; true if that step ended this CTA's part of its group.
    W4A16_HD bool advance(int n, int KC) {
        pos += n;
        kc += n;
        if (kc == KC) { kc = 0; ++g; return true; }
        return pos == end;
    }
};

}  // namespace w4a16
