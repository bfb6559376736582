// Decode path (1 <= M <= 16): weight-streaming GEMV with cluster split-K.
// Included by the single device-code translation unit (kernels.cu) only.
//
// Replaces the reference's decode kernel (src/vectorized/decode.cuh:18-159 and
// its launcher kernel.cu:19-53) with a design for 148 SMs and HBM3e:
//
//   * grid = (ceil(N/64), S) with clusters of S CTAs along K.  S is chosen from
//     (N, K) alone so every shape puts >= ~3 CTAs on each SM; a cluster's CTAs
//     own disjoint K slices of the same 64 output columns.
//   * each of the 4 warps of a CTA owns one 16-row block of W (one n16 block)
//     and streams that block's K slice -- a contiguous run of 512-byte chunks in
//     the packed layout -- through a private ring of 1-D bulk copies
//     (cp.async.bulk, completion on an mbarrier).  No CTA-wide sync in the loop.
//   * the CTA's activation slice x[:, slice] and its scale rows are bulk-copied
//     once into shared memory; B fragments come from ldmatrix.
//   * the packed word of each lane is already an m16n8k16 A fragment, so the
//     exact 13-instruction dequant feeds mma.sync directly (weights = A, the
//     M <= 16 tokens = the n8 side).  fp32 accumulation.
//   * split-K partials are reduced across the cluster through distributed
//     shared memory, in fixed rank order (deterministic, independent of timing).
//   * programmatic dependent launch: the weight and scale copies are issued
//     before griddepcontrol.wait, so they overlap the previous kernel's tail.
#pragma once
#include <cuda_fp16.h>
#include <stdint.h>

#include <algorithm>

#include "dequant.cuh"
#include "internal.h"
#include "ptx.cuh"

namespace w4a16 {

constexpr int kDecWarps = 4;
constexpr int kDecChunk = 512;                                    // bytes per (n16 block, 64-k chunk)
constexpr int kDecCH = 4;                                         // chunks per ring stage
constexpr int kDecR = 4;                                          // ring stages per warp
constexpr int kDecStageBytes = kDecCH * kDecChunk;                // 2 KB
constexpr int kDecRingBytes = kDecWarps * kDecR * kDecStageBytes; // 32 KB
constexpr int kDecRS = 68;                                        // fp32 row stride of the partial tile

struct DecodeSmem {
    int x_off, s_off, bar_off, total;
};

__host__ __device__ inline DecodeSmem decode_smem_layout(int mp, int kc_per, int ngrp_max) {
    DecodeSmem L;
    const int xs = kc_per * 64 + 8;                        // halves per token row (+16 B pad)
    const int x_bytes = ((mp * xs * 2) + 127) / 128 * 128;
    L.x_off = kDecRingBytes;
    L.s_off = L.x_off + x_bytes;
    L.bar_off = L.s_off + ngrp_max * 128;
    L.total = L.bar_off + (kDecWarps * kDecR + 1) * 8;
    return L;
}

__host__ __device__ inline int decode_ngrp_max(int kc_per, int G) {
    const int gpc = G / 64;
    return (kc_per + gpc - 1) / gpc + 1;
}

template <int G, int MT, bool OUT_F32>
__global__ void __launch_bounds__(kDecWarps * 32, 4)
decode_kernel(const uint8_t* __restrict__ wp, const __half* __restrict__ x,
              const __half* __restrict__ scales, void* __restrict__ yv,
              int M, int N, int K, int kc_per)
{
    constexpr int GPC = G / 64;      // 64-wide chunks per scale group
    constexpr int MP = MT * 8;       // token rows held in shared memory
    constexpr unsigned FULL = 0xffffffffu;
    extern __shared__ __align__(128) uint8_t smem[];

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, t = lane & 3;
    const int KC = K >> 6, NB = N >> 4;
    const int S = gridDim.y;
    const int kc_begin = blockIdx.y * kc_per;
    const int kc_end = min(KC, kc_begin + kc_per);
    const int nkc = max(0, kc_end - kc_begin);
    const int grp_begin = kc_begin / GPC;
    const int ngrp = nkc > 0 ? (kc_end - 1) / GPC - grp_begin + 1 : 0;
    const int nb0 = blockIdx.x * kDecWarps;
    const int nb = nb0 + warp;
    const bool valid = nb < NB;
    const int nvalid_nb = min(kDecWarps, NB - nb0);

    const DecodeSmem L = decode_smem_layout(MP, kc_per, decode_ngrp_max(kc_per, G));
    const int XS = kc_per * 64 + 8;
    const uint32_t sbase = smem_u32(smem);
    const uint32_t ring = sbase + warp * kDecR * kDecStageBytes;
    const uint32_t xs = sbase + L.x_off;
    const uint32_t ss = sbase + L.s_off;
    const uint32_t full0 = sbase + L.bar_off + warp * kDecR * 8;
    const uint32_t xbar = sbase + L.bar_off + kDecWarps * kDecR * 8;

    if (threadIdx.x == 0) mbar_init(xbar, 1);
    if (lane == 0) {
#pragma unroll
        for (int r = 0; r < kDecR; ++r) mbar_init(full0 + 8 * r, 1);
    }
    fence_mbar_init();
    __syncthreads();

    // ---- weight ring prologue: weights are read-only, so issue before the PDL wait
    const int nstages = (nkc + kDecCH - 1) / kDecCH;
    const uint8_t* wsrc = wp + ((size_t)nb * KC + kc_begin) * kDecChunk;
    const uint64_t pol = policy_evict_first();
    auto issue = [&](int st) {
        const int c0 = st * kDecCH;
        const int cnt = min(kDecCH, nkc - c0);
        const uint32_t bar = full0 + (st % kDecR) * 8;
        mbar_arrive_expect_tx(bar, cnt * kDecChunk);
        bulk_g2s_hint(ring + (st % kDecR) * kDecStageBytes, wsrc + (size_t)c0 * kDecChunk,
                      cnt * kDecChunk, bar, pol);
    };
    if (valid && lane == 0) {
        const int pro = min(kDecR, nstages);
        for (int st = 0; st < pro; ++st) issue(st);
    }

    // ---- scale rows (read-only) and the activation slice (after the PDL wait)
    if (warp == 0) {
        const uint32_t srow = nvalid_nb * 32;
        if (lane == 0) mbar_arrive_expect_tx(xbar, ngrp * srow + (uint32_t)(M * nkc * 128));
        __syncwarp();
        for (int i = lane; i < ngrp; i += 32)
            bulk_g2s(ss + i * 128, scales + (size_t)(grp_begin + i) * N + nb0 * 16, srow, xbar);
        pdl_wait();
        if (nkc > 0)
            for (int m = lane; m < M; m += 32)
                bulk_g2s(xs + m * XS * 2, x + (size_t)m * K + (size_t)kc_begin * 64, nkc * 128, xbar);
    } else {
        pdl_wait();
    }
    // Token rows M..MP-1 are padding B columns: zero them so every lane computes on defined data.
    {
        uint4* xz = reinterpret_cast<uint4*>(smem + L.x_off + (size_t)M * XS * 2);
        const int n16 = (MP - M) * XS * 2 / 16;
        for (int i = threadIdx.x; i < n16; i += kDecWarps * 32) xz[i] = make_uint4(0, 0, 0, 0);
    }
    pdl_launch_dependents();
    __syncthreads();

    bool ok = __all_sync(FULL, mbar_wait(xbar, 0, kDevTimeoutActivations));

    float acc[MT][4];
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[mt][i] = 0.f;

    int st = 0;
    if (valid && ok) {
        const uint32_t ldm = xs + (uint32_t)(((lane & 7) * XS + (lane >> 3) * 8) * 2);
        const uint16_t* sh = reinterpret_cast<const uint16_t*>(smem + L.s_off) + warp * 16 + g;
        for (; st < nstages; ++st) {
            const int slot = st % kDecR;
            if (!__all_sync(FULL, mbar_wait(full0 + slot * 8, (st / kDecR) & 1, kDevTimeoutWeights))) {
                ok = false;
                break;
            }
            const uint32_t wbase = ring + slot * kDecStageBytes + lane * 16;
#pragma unroll
            for (int c = 0; c < kDecCH; ++c) {
                const int ci = st * kDecCH + c;
                if (ci < nkc) {
                    const uint4 w = lds128(wbase + c * kDecChunk);
                    const int grp = (kc_begin + ci) / GPC - grp_begin;
                    const uint32_t s_lo = bcast_half(sh[grp * 64]);
                    const uint32_t s_hi = bcast_half(sh[grp * 64 + 8]);
                    uint32_t b[MT][8];
#pragma unroll
                    for (int mt = 0; mt < MT; ++mt) {
                        const uint32_t p = ldm + (uint32_t)((mt * 8 * XS + ci * 64) * 2);
                        uint32_t (&lo)[4] = *reinterpret_cast<uint32_t(*)[4]>(&b[mt][0]);
                        uint32_t (&hi)[4] = *reinterpret_cast<uint32_t(*)[4]>(&b[mt][4]);
                        ldmatrix_x4(lo, p);
                        ldmatrix_x4(hi, p + 64);
                    }
                    const uint32_t wq[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
                    for (int s = 0; s < 4; ++s) {
                        uint32_t a[4];
                        dequant_word(wq[s], s_lo, s_hi, a);
#pragma unroll
                        for (int mt = 0; mt < MT; ++mt) mma_16816(acc[mt], a, b[mt][2 * s], b[mt][2 * s + 1]);
                    }
                }
            }
            __syncwarp();
            if (lane == 0 && st + kDecR < nstages) issue(st + kDecR);
        }
    }
    if (!ok && valid) {
        // Error path: let every copy this warp issued land before the CTA may exit.
        const int issued = min(nstages, st + kDecR);
        for (int s2 = st; s2 < issued; ++s2) mbar_wait(full0 + (s2 % kDecR) * 8, (s2 / kDecR) & 1, kDevTimeoutDrain);
    }

    // ---- epilogue
    __syncthreads();   // ring idle in every warp: reuse it for the partial tile
    if (S == 1) {
        if (valid) {
#pragma unroll
            for (int mt = 0; mt < MT; ++mt)
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const int tok = mt * 8 + 2 * t + (i & 1);
                    const int n = nb * 16 + g + 8 * (i >> 1);
                    if (tok < M) {
                        if (OUT_F32) static_cast<float*>(yv)[(size_t)tok * N + n] = acc[mt][i];
                        else static_cast<__half*>(yv)[(size_t)tok * N + n] = __float2half_rn(acc[mt][i]);
                    }
                }
        }
        return;
    }
    float* red = reinterpret_cast<float*>(smem);
    if (valid) {
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int tok = mt * 8 + 2 * t + (i & 1);
                red[tok * kDecRS + warp * 16 + g + 8 * (i >> 1)] = acc[mt][i];
            }
    }
    cluster_sync();   // partial tiles of every split visible cluster-wide
    {
        const int rank = (int)cluster_ctarank();
        const int E = M * 64;
        const int per = (E + S - 1) / S;
        const int e1 = min(E, (rank + 1) * per);
        for (int e = rank * per + threadIdx.x; e < e1; e += kDecWarps * 32) {
            const int tok = e >> 6, nl = e & 63;
            if (nl < nvalid_nb * 16) {
                const uint32_t la = smem_u32(red + tok * kDecRS + nl);
                float sum = 0.f;
                for (int r = 0; r < S; ++r) sum += ld_shared_cluster_f32(mapa_shared(la, r));
                const size_t o = (size_t)tok * N + nb0 * 16 + nl;
                if (OUT_F32) static_cast<float*>(yv)[o] = sum;
                else static_cast<__half*>(yv)[o] = __float2half_rn(sum);
            }
        }
    }
    cluster_sync();   // keep this CTA's shared memory alive until every peer finished reading it
}

// ------------------------------------------------------------------ host side
DecodePlan plan_decode(int M, int N, int K, int G, const DeviceInfo& dev) {
    DecodePlan p;
    const int NB = N / 16, KC = K / 64;
    p.grid_x = (NB + kDecWarps - 1) / kDecWarps;
    p.mt = M <= 8 ? 1 : 2;
    // K split from (N, K) only, so a row's result never depends on the batch size:
    // aim for >= 3 CTAs per SM while every split keeps >= 2 chunks ...
    const int target = 3 * dev.num_sms;
    int S = 1;
    while (S < 8 && p.grid_x * S < target && KC / (2 * S) >= 2) S *= 2;
    // ... then split further until a 16-token activation slice fits in shared memory.
    auto smem_for = [&](int s, int mp) {
        const int kc_per = (KC + s - 1) / s;
        return (size_t)decode_smem_layout(mp, kc_per, decode_ngrp_max(kc_per, G)).total;
    };
    while (S < 16 && smem_for(S, 16) > (size_t)dev.max_smem_optin) S *= 2;
    p.valid = smem_for(S, 16) <= (size_t)dev.max_smem_optin;
    p.split = S;
    p.kc_per = (KC + S - 1) / S;
    p.smem = smem_for(S, p.mt * 8);
    return p;
}

template <int G, int MT, bool F32>
static cudaError_t launch_decode_t(const GemmArgs& a, const DecodePlan& p) {
    auto kern = decode_kernel<G, MT, F32>;
    cudaError_t err = ensure_max_dynamic_smem(reinterpret_cast<const void*>(kern));
    if (err != cudaSuccess) return err;
    if (p.split > 8 && (err = ensure_nonportable_cluster(reinterpret_cast<const void*>(kern))) != cudaSuccess)
        return err;

    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(p.grid_x, p.split, 1);
    cfg.blockDim = dim3(kDecWarps * 32, 1, 1);
    cfg.dynamicSmemBytes = p.smem;
    cfg.stream = a.stream;
    cudaLaunchAttribute attrs[2];
    int na = 0;
    attrs[na].id = cudaLaunchAttributeClusterDimension;
    attrs[na].val.clusterDim.x = 1;
    attrs[na].val.clusterDim.y = p.split;
    attrs[na].val.clusterDim.z = 1;
    ++na;
    if (a.pdl) {
        attrs[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attrs[na].val.programmaticStreamSerializationAllowed = 1;
        ++na;
    }
    cfg.attrs = attrs;
    cfg.numAttrs = na;
    return cudaLaunchKernelEx(&cfg, kern, static_cast<const uint8_t*>(a.wp), static_cast<const __half*>(a.x),
                              static_cast<const __half*>(a.scales), a.y, a.M, a.N, a.K, p.kc_per);
}

cudaError_t launch_decode(const GemmArgs& a, const DecodePlan& p) {
    const bool f32 = a.out_f32;
    if (a.G == 64) {
        if (p.mt == 1) return f32 ? launch_decode_t<64, 1, true>(a, p) : launch_decode_t<64, 1, false>(a, p);
        return f32 ? launch_decode_t<64, 2, true>(a, p) : launch_decode_t<64, 2, false>(a, p);
    }
    if (p.mt == 1) return f32 ? launch_decode_t<128, 1, true>(a, p) : launch_decode_t<128, 1, false>(a, p);
    return f32 ? launch_decode_t<128, 2, true>(a, p) : launch_decode_t<128, 2, false>(a, p);
}

}  // namespace w4a16
