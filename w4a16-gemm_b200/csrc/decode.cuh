// Decode path (1 <= M <= 16): persistent stream-K weight-streaming GEMV.
// Included by the single device-code translation unit (kernels.cu) only.
//
// Replaces the reference's decode kernel (src/vectorized/decode.cuh:18-159 and
// its launcher kernel.cu:19-53), whose grid of N/64 CTAs leaves most of a
// 148-SM B200 idle, with a design built around HBM3e streaming:
//
//   * Work is a stream of *units*: 4 n16 blocks (64 output columns) x 4
//     64-wide K chunks = 8 KB of packed words.  Units are ordered group-major
//     (a group = the 64 columns over all of K) and the stream is cut into
//     equal contiguous ranges, one per SM (stream-K), so every SM moves the
//     same number of bytes whatever N and K are.
//   * One persistent CTA of 16 warps per SM.  Warp group q (4 warps) takes
//     every 4th unit; warp w of the group handles n16 block w%4 of the unit,
//     whose 4 chunks are one contiguous 2 KB run.  Every warp streams its own
//     runs through a private ring of 1-D bulk copies: the copy engine services
//     one warp's requests one after another (measured), so 16 issuing warps
//     per SM are what reaches HBM bandwidth.
//   * A group's activation rows for its unit (M x 512 B) are double-buffered
//     in shared memory by 16-byte cp.async from the group's 128 threads, rows
//     528 B apart so ldmatrix reads them conflict-free; scales come through
//     the read-only cache.
//   * The packed word of each lane is already an m16n8k16 A fragment, so the
//     exact 13-instruction dequant feeds mma.sync directly (weights = A,
//     the <= 16 tokens = the n8 side); 4 independent fp32 accumulator chains.
//   * When a CTA finishes its part of a group it reduces its 4 K-lanes in
//     shared memory (fixed order).  A group covered by one CTA is written
//     directly; a group split across CTAs leaves one fp32 partial per CTA in
//     the caller's workspace, and the last CTA to finish (self-resetting
//     counter) sums the partials in CTA order -- deterministic.
//   * Programmatic dependent launch: each warp's first packed-word copies are
//     issued before griddepcontrol.wait.
#pragma once
#include <cuda.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include <algorithm>

#include "dequant.cuh"
#include "internal.h"
#include "ptx.cuh"

// Timeline hook for offline analysis builds; compiles to nothing by default.
#ifndef W4A16_DC_TRACE
#define W4A16_DC_TRACE(slot)
#endif
#define W4A16_DC_TRACE_LANE0(slot) do { if (lane == 0) { W4A16_DC_TRACE(slot); } } while (0)

namespace w4a16 {

constexpr int kDcConsumers = 16;                          // warps (each streams its own packed words)
constexpr int kDcThreads = kDcConsumers * 32;
constexpr int kDcNG = 4;                                  // n16 blocks per unit
constexpr int kDcWK = 4;                                  // 64-wide K chunks per unit
constexpr int kDcCols = kDcNG * 16;                       // output columns per group
constexpr int kDcWBytes = kDcNG * kDcWK * 512;            // packed words per unit (8 KB)
constexpr int kDcSBytes = 512;                            // <= 4 scale rows x 64 fp16
constexpr int kDcSlotFloats = 16 * kDcCols;               // one partial: 16 tokens x 64 columns
constexpr int kDcMaxCTAs = 1024;

template <int MP>
struct DcCfg {
    static constexpr int R = 3;                                   // per-warp ring depth (units)
    static constexpr int XT = 3;                                  // activation tiles per warp group (2 units ahead)
    static constexpr int WRUN = kDcWK * 512;                      // one warp's packed words of a unit (2 KB)
    static constexpr int RING_BYTES = kDcConsumers * R * WRUN;
    static constexpr int XROW = kDcWK * 128 + 16;                 // one token row of a unit (+16 B: ldmatrix conflict-free)
    static constexpr int X_BYTES = MP * XROW;                     // one activation tile
    static constexpr int XBUF_BYTES = (kDcConsumers / kDcNG) * XT * X_BYTES;  // XT tiles per warp group
    static constexpr int RED_BYTES = kDcConsumers * MP * 16 * 4;  // per-warp partial tiles
    static constexpr int BAR_BYTES = 1024;
    static constexpr int SMEM = 128 + RING_BYTES + XBUF_BYTES + RED_BYTES + BAR_BYTES;
    static_assert(SMEM <= 227 * 1024, "shared memory budget");
};

// Static stream-K partition, identical on host and device.
struct DcPartition {
    int units;     // total units
    int wg;        // units (K windows) per group
    int groups;    // groups (64 columns each)
    int ctas;      // CTAs (<= units)
    bool valid;    // units * ctas fits the 32-bit partition arithmetic
    // units * ctas < 2^31 is guaranteed by the host (dc_partition), so 32-bit math is exact.
    __host__ __device__ int u0(int c) const { return (int)(((unsigned)c * (unsigned)units) / (unsigned)ctas); }
    __host__ __device__ int u1(int c) const { return u0(c + 1); }
    // First / last CTA whose range intersects group g.
    __host__ __device__ int first_cta(int g) const {
        int c = (int)(((unsigned)(g * wg) * (unsigned)ctas) / (unsigned)units);
        while (c > 0 && u1(c - 1) > g * wg) --c;
        while (u1(c) <= g * wg) ++c;
        return c;
    }
    __host__ __device__ int last_cta(int g) const {
        int c = (int)(((unsigned)((g + 1) * wg - 1) * (unsigned)ctas) / (unsigned)units);
        while (c + 1 < ctas && u0(c + 1) < (g + 1) * wg) ++c;
        while (u0(c) >= (g + 1) * wg) --c;
        return c;
    }
    // Workspace slot of CTA c's partial of group g (only for split groups).
    __host__ __device__ int slot(int c, int g) const { return 2 * c + (g == u0(c) / wg ? 0 : 1); }
};

__host__ __device__ inline DcPartition dc_partition(int N, int K, int num_sms) {
    DcPartition p;
    p.groups = (N / 16 + kDcNG - 1) / kDcNG;
    p.wg = (K / 64 + kDcWK - 1) / kDcWK;
    p.units = p.groups * p.wg;
    p.ctas = num_sms < p.units ? num_sms : p.units;
    if (p.ctas > kDcMaxCTAs) p.ctas = kDcMaxCTAs;
    p.valid = (long long)p.units * p.ctas < (1ll << 31);
    return p;
}

// True if some group's units are split across CTAs (every CTA boundary inside a group).
__host__ __device__ inline bool dc_has_split(const DcPartition& p) {
    for (int c = 1; c < p.ctas; ++c)
        if (p.u0(c) % p.wg != 0) return true;
    return false;
}

// Workspace: 2 fp32 partial slots per CTA (a CTA's range splits at most its first
// and its last group).  Always fully written before it is read; no initial contents
// are assumed.
__host__ __device__ inline size_t dc_workspace_bytes(const DcPartition& p) {
    return (size_t)2 * p.ctas * kDcSlotFloats * 4;
}

// Bar 1: the 16 consumer warps only (the producer never joins).
__device__ __forceinline__ void dc_consumer_sync() {
    asm volatile("bar.sync 1, %0;" :: "n"(kDcConsumers * 32) : "memory");
}

// Named barriers: 1 = all consumer warps, 2 + q = warp group q (4 warps).
__device__ __forceinline__ void dc_group_sync(int q) {
    asm volatile("bar.sync %0, %1;" :: "r"(2 + q), "n"(kDcNG * 32) : "memory");
}

__device__ __forceinline__ void cp_async_commit() {
    asm volatile("cp.async.commit_group;" ::: "memory");
}

template <int N_PENDING>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" :: "n"(N_PENDING) : "memory");
}

template <int G, int MP, bool OUT_F32>
__global__ void __launch_bounds__(kDcThreads, 1)
decode_kernel(const uint8_t* __restrict__ wp, const __half* __restrict__ x,
              const __half* __restrict__ scales, void* __restrict__ yv, int M, int N, int K,
              DcPartition part, float* __restrict__ partials)
{
    using C = DcCfg<MP>;
    constexpr int R = C::R;
    constexpr int XT = C::XT;
    constexpr int MT = MP / 8;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t base = (raw + 127u) & ~127u;
    uint8_t* const gbase = smem_raw + (base - raw);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nbi = warp % kDcNG;          // n16 block inside a unit
    const int q = warp / kDcNG;            // warp group: units it with it % 4 == q
    const int g8 = lane >> 2, t4 = lane & 3;

    const uint32_t ring = base + warp * R * C::WRUN;                        // this warp's ring
    const uint32_t xbuf = base + C::RING_BYTES + q * XT * C::X_BYTES;       // this group's XT tiles
    float* const red = reinterpret_cast<float*>(gbase + C::RING_BYTES + C::XBUF_BYTES);
    const uint32_t bar0 = base + C::RING_BYTES + C::XBUF_BYTES + C::RED_BYTES;
    const uint32_t wfull = bar0 + warp * R * 8;                             // this warp's barriers

    const int c = blockIdx.x;
    const int u0 = part.u0(c), u1 = part.u1(c), n = u1 - u0;
    const int KC = K >> 6, NB = N >> 4;

    if (lane == 0)
        for (int r = 0; r < R; ++r) mbar_init(wfull + 8 * r, 1);
    fence_mbar_init();
    // Token rows M..MP-1 of the activation tiles stay zero (only rows < M are copied).
    for (int i = threadIdx.x; i < C::XBUF_BYTES / 16; i += kDcThreads)
        reinterpret_cast<uint4*>(gbase + C::RING_BYTES)[i] = make_uint4(0, 0, 0, 0);
    __syncthreads();

    // ---- this warp's packed-word stream: units u0 + q + 4j, one 2 KB run each
    auto unit_gw = [&](int it, int& g, int& w) { const int u = u0 + it; g = u / part.wg; w = u - g * part.wg; };
    auto issue_w = [&](int j) {            // lane 0 only
        const int it = q + 4 * j;
        if (it >= n) return;
        int g, w;
        unit_gw(it, g, w);
        const int nb = g * kDcNG + nbi;
        const uint32_t bar = wfull + 8 * (j % R);
        if (nb >= NB) { mbar_arrive(bar); return; }            // block beyond N: nothing to load
        const int kcn = min(kDcWK, KC - w * kDcWK);
        const uint32_t bytes = (uint32_t)(kcn * 512);
        mbar_arrive_expect_tx(bar, bytes);
        bulk_g2s(ring + (j % R) * C::WRUN, wp + ((size_t)nb * KC + w * kDcWK) * 512, bytes, bar);
        // its scale rows stream from DRAM too: pull them into L2 now, load them one unit early
        for (int r = (w * kDcWK * 64) / G; r <= ((w * kDcWK + kcn - 1) * 64) / G; ++r)
            prefetch_l2(scales + (size_t)r * N + nb * 16);
    };
    if (lane == 0)
        for (int j = 0; j < R; ++j) issue_w(j);   // packed words never depend on the previous kernel

    if (threadIdx.x == 0) W4A16_DC_TRACE(0);
    pdl_wait();   // x, the workspace and y may still be in use by the previous kernel
    pdl_launch_dependents();

    // ---- this group's activation tiles: rows < M of the unit's 4 chunks, 16-byte cp.async by the
    //      group's 128 threads, row m at m * XROW (conflict-free ldmatrix)
    const int gt = nbi * 32 + lane;       // thread index inside the group
    auto issue_x = [&](int it, int buf) {
        if (it < n) {
            int g, w;
            unit_gw(it, g, w);
            const int kcn = min(kDcWK, KC - w * kDcWK);
            const uint32_t dst = xbuf + buf * C::X_BYTES;
            for (int e = gt; e < M * kDcWK * 8; e += kDcNG * 32) {
                const int m = e / (kDcWK * 8), sgi = e % (kDcWK * 8);
                if (sgi < kcn * 8)
                    cp_async16(dst + m * C::XROW + sgi * 16, x + (size_t)m * K + (size_t)w * kDcWK * 64 + sgi * 8);
                else   // chunk beyond K: zeros, so whatever stale packed words sit there contribute 0
                    *reinterpret_cast<uint4*>(gbase + (dst - base) + m * C::XROW + sgi * 16) = make_uint4(0, 0, 0, 0);
            }
        }
        cp_async_commit();
    };
    issue_x(q, 0);
    issue_x(q + 4, 1);

    const uint32_t w_lane = (uint32_t)(lane * 16);
    const uint32_t x_lane = (uint32_t)((lane & 7) * C::XROW + (lane >> 3) * 16);
    const unsigned short* srow = reinterpret_cast<const unsigned short*>(scales) + g8;
    // Scale values (raw fp16) of this warp's next unit, loaded one unit ahead of use.
    unsigned short sn_lo[kDcWK], sn_hi[kDcWK];
    auto load_scales = [&](int it) {
        if (it >= n) return;
        int g, w;
        unit_gw(it, g, w);
        const int kcn = min(kDcWK, KC - w * kDcWK);
#pragma unroll
        for (int j = 0; j < kDcWK; ++j) {
            const int srw = j < kcn ? ((w * kDcWK + j) * 64) / G : 0;
            const unsigned short* sp = srow + (size_t)srw * N + (g * kDcNG + nbi) * 16;
            sn_lo[j] = __ldg(sp);
            sn_hi[j] = __ldg(sp + 8);
        }
    };
    load_scales(q);

    float acc[kDcWK][MT][4];
#pragma unroll
    for (int j = 0; j < kDcWK; ++j)
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
#pragma unroll
            for (int i = 0; i < 4; ++i) acc[j][mt][i] = 0.f;

    bool ok = true;
    int jw = 0;                                    // this warp's unit counter
    int g = u0 / part.wg, w = u0 - g * part.wg;    // group / window of unit it (all warps track it)
    for (int it = 0; it < n; ++it) {
        if ((it & 3) == q) {
            // (1) the whole group is done with the tile issue_x is about to refill
            if (lane == 0 && nbi == 0 && jw < 16) W4A16_DC_TRACE(40 + q * 16 + jw);
            dc_group_sync(q);
            if (lane == 0 && nbi == 0 && jw < 16) W4A16_DC_TRACE(120 + q * 16 + jw);
            issue_x(it + 8, (jw + 2) % XT);
            // (2) scales: this unit's were loaded one unit early; start the next unit's now
            uint32_t s_lo[kDcWK], s_hi[kDcWK];
#pragma unroll
            for (int j = 0; j < kDcWK; ++j) {
                s_lo[j] = bcast_half(sn_lo[j]);
                s_hi[j] = bcast_half(sn_hi[j]);
            }
            load_scales(it + 4);
            // (3) this unit's activation tile (all 128 threads' copies) and packed words
            cp_async_wait<XT - 1>();
            if (lane == 0 && nbi == 0 && jw < 16) W4A16_DC_TRACE(60 + q * 16 + jw);
            dc_group_sync(q);
            if (lane == 0 && nbi == 0 && jw < 16) W4A16_DC_TRACE(80 + q * 16 + jw);
            if (ok) ok = __all_sync(0xffffffffu, mbar_wait(wfull + 8 * (jw % R), (jw / R) & 1, kDevTimeoutWeights));
            if (lane == 0 && nbi == 0 && jw < 16) W4A16_DC_TRACE(20 + q * 16 + jw);
            if (ok) {
                const uint32_t wb = ring + (jw % R) * C::WRUN + w_lane;
                const uint32_t xb = xbuf + (jw % XT) * C::X_BYTES + x_lane;
                constexpr int JB = MT == 1 ? 4 : 2;
#pragma unroll
                for (int jb = 0; jb < kDcWK; jb += JB) {
                    uint4 wv[JB];
                    uint32_t b[JB][MT][8];
#pragma unroll
                    for (int jj = 0; jj < JB; ++jj) {
                        wv[jj] = lds128(wb + (jb + jj) * 512);
#pragma unroll
                        for (int mt = 0; mt < MT; ++mt) {
                            const uint32_t xa = xb + mt * 8 * C::XROW + (jb + jj) * 128;
                            ldmatrix_x4(*reinterpret_cast<uint32_t(*)[4]>(&b[jj][mt][0]), xa);
                            ldmatrix_x4(*reinterpret_cast<uint32_t(*)[4]>(&b[jj][mt][4]), xa + 64);
                        }
                    }
                    // No per-chunk guard: chunks beyond K have zero activations (issue_x), and the
                    // unconditional body lets the 4 accumulator chains interleave.
#pragma unroll
                    for (int ks = 0; ks < 4; ++ks)
#pragma unroll
                        for (int jj = 0; jj < JB; ++jj) {
                            const uint32_t wq = ks == 0 ? wv[jj].x : ks == 1 ? wv[jj].y : ks == 2 ? wv[jj].z : wv[jj].w;
                            uint32_t a[4];
                            dequant_word(wq, s_lo[jb + jj], s_hi[jb + jj], a);
#pragma unroll
                            for (int mt = 0; mt < MT; ++mt)
                                mma_16816(acc[jb + jj][mt], a, b[jj][mt][2 * ks], b[jj][mt][2 * ks + 1]);
                        }
                }
            }
            // (4) refill this ring slot with this warp's unit R positions ahead
            if (lane == 0 && nbi == 0 && jw < 16) W4A16_DC_TRACE(100 + q * 16 + jw);
            __syncwarp();
            if (lane == 0 && ok) issue_w(jw + R);
            ++jw;
        }

        // ---------------------------------------------------------------- group boundary
        const bool group_end = (it + 1 == n) || (w + 1 == part.wg);
        if (group_end) {
            if (threadIdx.x == 0) W4A16_DC_TRACE(169);
            // (1) every warp folds its 4 chains (fixed order), then the 4 warp groups are
            //     summed per n16 block in fixed order -> this CTA's partial of group g.
#pragma unroll
            for (int mt = 0; mt < MT; ++mt)
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const int tok = mt * 8 + 2 * t4 + (i & 1);
                    float sum = 0.f;
#pragma unroll
                    for (int j = 0; j < kDcWK; ++j) {
                        sum += acc[j][mt][i];
                        acc[j][mt][i] = 0.f;
                    }
                    red[(warp * MP + tok) * 16 + g8 + 8 * (i >> 1)] = sum;
                }
            dc_consumer_sync();
            if (threadIdx.x == 0) W4A16_DC_TRACE(171);
            const int gu0 = g * part.wg;
            const bool whole = (u0 <= gu0) && (u1 >= gu0 + part.wg);
            const int col0 = g * kDcCols;
            constexpr int PER = MP * kDcCols / (kDcConsumers * 32);
            float v[PER];
#pragma unroll
            for (int r = 0; r < PER; ++r) {
                const int e = threadIdx.x + r * kDcConsumers * 32;
                const int tok = e / kDcCols, col = e % kDcCols;
                const int nb = col >> 4, cc = col & 15;
                float sum = 0.f;
#pragma unroll
                for (int qq = 0; qq < kDcConsumers / kDcNG; ++qq) sum += red[((qq * kDcNG + nb) * MP + tok) * 16 + cc];
                v[r] = sum;
            }
            if (whole) {
#pragma unroll
                for (int r = 0; r < PER; ++r) {
                    const int e = threadIdx.x + r * kDcConsumers * 32;
                    const int tok = e / kDcCols, col = col0 + e % kDcCols;
                    if (tok < M && col < N) {
                        if (OUT_F32) static_cast<float*>(yv)[(size_t)tok * N + col] = v[r];
                        else static_cast<__half*>(yv)[(size_t)tok * N + col] = __float2half_rn(v[r]);
                    }
                }
            } else {
                // (2) split group: leave this CTA's partial; decode_fixup_kernel sums them in CTA order.
                float* my = partials + (size_t)part.slot(c, g) * kDcSlotFloats;
#pragma unroll
                for (int r = 0; r < PER; ++r) {
                    const int e = threadIdx.x + r * kDcConsumers * 32;
                    if (e / kDcCols < M) __stcg(my + e, v[r]);
                }
            }
            dc_consumer_sync();   // red reusable
            if (threadIdx.x == 0) W4A16_DC_TRACE(170);
        }
        if (++w == part.wg) { w = 0; ++g; }
    }
    cp_async_wait<0>();
    if (!ok) {
        // Error path: let this warp's copies still in flight land before the CTA may exit.
        for (int j = jw; j < jw + R; ++j)
            if (q + 4 * j < n) mbar_wait(wfull + 8 * (j % R), (j / R) & 1, kDevTimeoutDrain);
    }
}

// Combines the groups that the stream-K partition split across CTAs: one CTA per
// group; groups owned by a single CTA were written by decode_kernel already.
// Launched right behind decode_kernel with programmatic dependent launch, so it
// is resident early and griddepcontrol.wait releases it when decode_kernel's
// writes are complete and visible.  Sums the partials in CTA order.
template <bool OUT_F32>
__global__ void __launch_bounds__(256) decode_fixup_kernel(void* __restrict__ yv, int M, int N, DcPartition part,
                                                           const float* __restrict__ partials) {
    const int g = blockIdx.x;
    const int cf = part.first_cta(g), cl = part.last_cta(g);
    pdl_launch_dependents();
    if (cf == cl) return;
    pdl_wait();
    const int col0 = g * kDcCols;
    for (int e = threadIdx.x; e < M * kDcCols; e += blockDim.x) {
        float sum = 0.f;
        for (int cc = cf; cc <= cl; ++cc) sum += __ldcg(partials + (size_t)part.slot(cc, g) * kDcSlotFloats + e);
        const int tok = e / kDcCols, col = col0 + e % kDcCols;
        if (col < N) {
            if (OUT_F32) static_cast<float*>(yv)[(size_t)tok * N + col] = sum;
            else static_cast<__half*>(yv)[(size_t)tok * N + col] = __float2half_rn(sum);
        }
    }
}

// ------------------------------------------------------------------ host side
DecodePlan plan_decode(int M, int N, int K, int G, const DeviceInfo& dev) {
    (void)G;
    DecodePlan p;
    const DcPartition part = dc_partition(N, K, dev.num_sms);
    p.mt = M <= 8 ? 1 : 2;
    p.ctas = part.ctas;
    p.units = part.units;
    p.stages = DcCfg<8>::R;
    p.smem = p.mt == 1 ? DcCfg<8>::SMEM : DcCfg<16>::SMEM;
    p.workspace = dc_workspace_bytes(part);
    p.valid = part.valid;
    return p;
}

size_t decode_workspace_bytes(int N, int K, const DeviceInfo& dev) {
    return dc_workspace_bytes(dc_partition(N, K, dev.num_sms));
}

template <int G, int MP, bool F32>
static cudaError_t launch_decode_t(const GemmArgs& a, const DecodePlan& p) {
    auto kern = decode_kernel<G, MP, F32>;
    cudaError_t err = ensure_max_dynamic_smem(reinterpret_cast<const void*>(kern));
    if (err != cudaSuccess) return err;
    DeviceInfo dev;
    if ((err = device_info(&dev)) != cudaSuccess) return err;
    const DcPartition part = dc_partition(a.N, a.K, dev.num_sms);
    float* partials = static_cast<float*>(a.workspace);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(part.ctas, 1, 1);
    cfg.blockDim = dim3(kDcThreads, 1, 1);
    cfg.dynamicSmemBytes = DcCfg<MP>::SMEM;
    cfg.stream = a.stream;
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr.val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = a.pdl ? 1 : 0;
    err = cudaLaunchKernelEx(&cfg, kern, static_cast<const uint8_t*>(a.wp), static_cast<const __half*>(a.x),
                             static_cast<const __half*>(a.scales), a.y, a.M, a.N, a.K, part, partials);
    if (err != cudaSuccess || !dc_has_split(part)) return err;
    // combine split groups; always launched programmatically dependent on decode_kernel
    cudaLaunchConfig_t fc = {};
    fc.gridDim = dim3(part.groups, 1, 1);
    fc.blockDim = dim3(256, 1, 1);
    fc.stream = a.stream;
    cudaLaunchAttribute fattr;
    fattr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
    fattr.val.programmaticStreamSerializationAllowed = 1;
    fc.attrs = &fattr;
    fc.numAttrs = 1;
    return cudaLaunchKernelEx(&fc, decode_fixup_kernel<F32>, a.y, a.M, a.N, part, static_cast<const float*>(partials));
}

cudaError_t launch_decode(const GemmArgs& a, const DecodePlan& p) {
    const bool f32 = a.out_f32;
    if (a.G == 64) {
        if (p.mt == 1) return f32 ? launch_decode_t<64, 8, true>(a, p) : launch_decode_t<64, 8, false>(a, p);
        return f32 ? launch_decode_t<64, 16, true>(a, p) : launch_decode_t<64, 16, false>(a, p);
    }
    if (p.mt == 1) return f32 ? launch_decode_t<128, 8, true>(a, p) : launch_decode_t<128, 8, false>(a, p);
    return f32 ? launch_decode_t<128, 16, true>(a, p) : launch_decode_t<128, 16, false>(a, p);
}

}  // namespace w4a16
