// Prefill path (any M): persistent, warp-specialised tcgen05 GEMM.
// Included by the single device-code translation unit (kernels.cu) only.
//
// Replaces the reference's mma.sync prefill kernel (src/vectorized/prefill.cuh:27-184)
// and its config machinery (kernel.cu:56-214).  The contraction is
//
//     D[n, tok] (TMEM, fp32) += Wdeq[n, k] (A, TMEM, fp16) * x[tok, k] (B, smem, fp16)
//
// i.e. the weights are the UMMA M side (128 output channels per tile) and the
// tokens the UMMA N side (TOK = 32..256 per tile).  The dequantised weights
// never touch shared memory: each dequant warp turns its lanes' packed words
// into m16n8k16 A fragments with the exact fp16 dequant and writes them into a
// TMEM ring with tcgen05.st.16x128b, whose register-to-(lane, column) map is
// exactly that fragment order.  Shared memory only carries the TMA-loaded x
// tile (128-byte swizzle), the raw packed words and one scale row per stage.
//
// Warp roles (one CTA per SM, all 512 TMEM columns):
//   warp 0      TMA producer: x tile [TOK x 64] (SW128), packed words of 8 n16
//               blocks for one 64-wide K chunk (3-D tensor map), 128 scales
//   warp 1      TMEM allocator + single-thread tcgen05.mma issuer
//   warps 2..   dequant (kPfDqPhases groups of 8): warp w owns n16 block
//               2*(w%4) + ((w-2)/4 & 1) of the tile, i.e. TMEM lanes inside its own
//               lane quarter, for the k-steps of its group ((w-2)/8)
//   last 16     epilogue: four warps per lane quarter, each tcgen05.ld's a quarter of
//               the tile's token columns; fp16 results are held in registers and the
//               accumulator is released before the global stores
//
// K is walked in one sequential order for every tile shape, so all prefill
// configs (TOK = 32/64/128/256) give bit-identical results and a row's output
// does not depend on the other rows of the batch.
#pragma once
#include <cuda.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include <algorithm>
#include <cmath>

#include "dequant.cuh"
#include "internal.h"
#include "ptx.cuh"

namespace w4a16 {

#ifndef W4A16_PF_DQ_PHASES
#define W4A16_PF_DQ_PHASES 1
#endif
// Dequant warp groups: group p (8 warps, one per n16 block of the tile) takes the k-steps
// it with it % kPfDqPhases == p, so consecutive k-steps are dequantised concurrently.
constexpr int kPfDqPhases = W4A16_PF_DQ_PHASES;
constexpr int kPfDqWarps = 8 * kPfDqPhases;
constexpr int kPfEpiWarp0 = 2 + kPfDqWarps;   // first epilogue warp
// Epilogue warps: four per TMEM lane quarter, each draining a quarter of a tile's token
// columns into registers, so the accumulator is free for the next tile's MMAs early.
#ifndef W4A16_PF_EPI_WARPS
#define W4A16_PF_EPI_WARPS 16
#endif
constexpr int kPfEpiWarps = W4A16_PF_EPI_WARPS;
constexpr int kPfThreads = (kPfEpiWarp0 + kPfEpiWarps) * 32;
constexpr int kPfRows = 128;                 // output channels per tile (UMMA M)
constexpr int kPfWBytes = 8 * 512;           // packed words: 8 n16 blocks x one 64-k chunk
constexpr int kPfSBytes = kPfRows * 2;       // one fp16 scale row slice
// 64-wide K chunks per pipeline stage.  A stage's round trip through the rings (tensor copy
// -> dequant -> TMEM store -> MMA -> commit -> slot free) has a fixed latency, so at small M,
// where that chain and not the tensor core sets the pace, more chunks per stage means
// fewer trips per K.  The chunks are still multiplied in K order, one k16 step at a time.
// Per token tile: as many as keep at least 3 stages in shared memory and 2 A slots in TMEM.
#ifndef W4A16_PF_KCH_SMALL
#define W4A16_PF_KCH_SMALL 6
#endif
#ifndef W4A16_PF_KCH_128
#define W4A16_PF_KCH_128 3
#endif
__host__ __device__ constexpr int pf_kch(int tok) {
    return tok <= 64 ? W4A16_PF_KCH_SMALL : tok == 128 ? W4A16_PF_KCH_128 : 2;
}
constexpr int kPfSmemBudget = 227 * 1024;    // opt-in dynamic shared memory per CTA on sm_100

template <int TOK>
struct PfCfg {
    static_assert(TOK == 32 || TOK == 64 || TOK == 128 || TOK == 256, "token tile");
    static constexpr int KCH = pf_kch(TOK);                           // 64-wide K chunks per stage
    static constexpr int X_CHUNK = TOK * 128;                         // TOK rows x 64 fp16 (one chunk)
    static constexpr int X_BYTES = KCH * X_CHUNK;                     // [chunk][TOK rows][128 B]
    static constexpr int W_BYTES = KCH * kPfWBytes;                   // [n16 block][chunk][512 B]
    static constexpr int S_BYTES = KCH * kPfSBytes;                   // [chunk][128 scales]
    static constexpr int STAGE = (X_BYTES + W_BYTES + S_BYTES + 1023) / 1024 * 1024;
    static constexpr int ACCS = TOK <= 128 ? 2 : 1;                   // TMEM accumulator buffers
    static constexpr int A_COL0 = ACCS * TOK;                         // first A-ring column
    static constexpr int A_COLS = 32 * KCH;                           // TMEM columns of one A slot
    static constexpr int A_STAGES = (512 - A_COL0) / A_COLS < 8 ? (512 - A_COL0) / A_COLS : 8;
    static constexpr int BAR_BYTES = 1024;
    static constexpr int ST_FIT = (kPfSmemBudget - 1024 - BAR_BYTES) / STAGE;
    static constexpr int STAGES = ST_FIT < 12 ? ST_FIT : 12;
    static constexpr int SMEM_USED = 1024 /*alignment slack*/ + STAGES * STAGE + BAR_BYTES;
    // Request > half of the SM's shared memory so at most one CTA (which owns all
    // 512 TMEM columns) is ever resident on an SM.
    static constexpr int SMEM = SMEM_USED > 116 * 1024 ? SMEM_USED : 116 * 1024;
    static_assert(A_COL0 + A_STAGES * A_COLS <= 512 && A_STAGES >= 2, "TMEM budget");
    static_assert(STAGES >= 3, "pipeline depth");
};

// UMMA instruction descriptor, kind::f16: fp16 A/B, fp32 D, both K-major, M=128, N=TOK.
template <int TOK>
__host__ __device__ constexpr uint32_t pf_idesc() {
    return (1u << 4)                         // D format f32
         | (0u << 7) | (0u << 10)            // A, B format f16
         | ((uint32_t)(TOK >> 3) << 17)      // N >> 3
         | ((uint32_t)(kPfRows >> 4) << 24); // M >> 4
}

// Shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row groups 1024 B apart.
__device__ __forceinline__ uint64_t pf_sw128_desc(uint32_t saddr) {
    return (uint64_t)((saddr >> 4) & 0x3FFF)
         | ((uint64_t)1 << 16)               // leading byte offset (unused for swizzled K-major)
         | ((uint64_t)(1024 >> 4) << 32)     // stride byte offset
         | ((uint64_t)1 << 46)               // descriptor version (sm_100)
         | ((uint64_t)2 << 61);              // SWIZZLE_128B
}

template <int G, int TOK, bool OUT_F32>
__global__ void __launch_bounds__(kPfThreads, 1)
prefill_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_w,
               const __grid_constant__ CUtensorMap tm_s, void* __restrict__ yv, int M, int N, int K)
{
    using C = PfCfg<TOK>;
    constexpr int ST = C::STAGES, NA = C::A_STAGES, NACC = C::ACCS;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    const uint32_t bar0 = base + ST * C::STAGE;
    auto full = [&](int s) { return bar0 + 8u * s; };
    auto empty = [&](int s) { return bar0 + 8u * (ST + s); };
    auto afull = [&](int a) { return bar0 + 8u * (2 * ST + a); };
    auto aempty = [&](int a) { return bar0 + 8u * (2 * ST + NA + a); };
    auto accfull = [&](int b) { return bar0 + 8u * (2 * ST + 2 * NA + b); };
    auto accempty = [&](int b) { return bar0 + 8u * (2 * ST + 2 * NA + NACC + b); };
    const uint32_t done_bar = bar0 + 8u * (2 * ST + 2 * NA + 2 * NACC);
    const uint32_t tmem_slot = done_bar + 8u;

    if (threadIdx.x == 0) {
        for (int s = 0; s < ST; ++s) {
            mbar_init(full(s), 1);
            mbar_init(empty(s), 8 * 32 + 1);   // every dequant lane + the MMA commit
        }
        for (int a = 0; a < NA; ++a) {
            mbar_init(afull(a), 8 * 32);
            mbar_init(aempty(a), 1);
        }
        for (int b = 0; b < NACC; ++b) {
            mbar_init(accfull(b), 1);
            mbar_init(accempty(b), kPfEpiWarps * 32);
        }
        mbar_init(done_bar, 1);
        fence_mbar_init();
        prefetch_tmap(&tm_x);
        prefetch_tmap(&tm_w);
        prefetch_tmap(&tm_s);
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, 512);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(smem_raw + (tmem_slot - raw));

    pdl_wait();               // x is produced by the previous kernel; y may still be read by it
    pdl_launch_dependents();

    const int n_tiles = (N + kPfRows - 1) / kPfRows;
    const int total = n_tiles * ((M + TOK - 1) / TOK);
    const int KC = K >> 6;                                  // 64-wide K chunks
    const int KB = KC < C::KCH ? KC : C::KCH;               // chunks in a stage's weight box
    const int KT = (KC + C::KCH - 1) / C::KCH;              // stages per tile

    if (warp == 0) {
        // ------------------------------------------------------------ TMA producer
        if (lane == 0) {
            int it = 0;
            bool ok = true;
            for (int tile = blockIdx.x; tile < total && ok; tile += gridDim.x) {
                const int tt = tile / n_tiles, tn = tile % n_tiles;
                for (int kt = 0; kt < KT; ++kt, ++it) {
                    const int s = it % ST;
                    if (!mbar_wait(empty(s), ((it / ST) & 1) ^ 1, kDevTimeoutPipeline)) { ok = false; break; }
                    // the stage's chunks c0 .. c0 + nch - 1: one x tile and one scale row per
                    // chunk, the packed words of all of them in one box (a last partial stage's
                    // box runs past K and reads zeros)
                    const uint32_t sb = base + s * C::STAGE;
                    const int c0 = kt * C::KCH, nch = KC - c0 < C::KCH ? KC - c0 : C::KCH;
                    mbar_arrive_expect_tx(full(s), (uint32_t)(nch * (C::X_CHUNK + kPfSBytes) + KB * kPfWBytes));
                    for (int j = 0; j < nch; ++j)
                        tma_load_2d(sb + j * C::X_CHUNK, &tm_x, (c0 + j) * 64, tt * TOK, full(s));
                    tma_load_3d(sb + C::X_BYTES, &tm_w, 0, c0, tn * 8, full(s));
                    for (int j = 0; j < nch; ++j)
                        tma_load_2d(sb + C::X_BYTES + C::W_BYTES + j * kPfSBytes, &tm_s, tn * kPfRows,
                                    ((c0 + j) * 64) / G, full(s));
                }
            }
            if (!ok) {
                // Error path: the last ST issued stages may still be landing.
                for (int j = max(0, it - ST); j < it; ++j)
                    mbar_wait(full(j % ST), (j / ST) & 1, kDevTimeoutDrain);
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issuer
        if (lane == 0) {
            constexpr uint32_t idesc = pf_idesc<TOK>();
            int it = 0, tc = 0;
            bool ok = true;
            for (int tile = blockIdx.x; tile < total && ok; tile += gridDim.x, ++tc) {
                const int b = tc % NACC;
                if (!mbar_wait(accempty(b), ((tc / NACC) & 1) ^ 1, kDevTimeoutPipeline)) { ok = false; break; }
                tc_fence_after();
                const uint32_t d = tmem + (uint32_t)(b * TOK);
                for (int kt = 0; kt < KT; ++kt, ++it) {
                    const int s = it % ST, a = it % NA;
                    if (!mbar_wait(full(s), (it / ST) & 1, kDevTimeoutPipeline) ||
                        !mbar_wait(afull(a), (it / NA) & 1, kDevTimeoutPipeline)) { ok = false; break; }
                    tc_fence_after();
                    const uint32_t xa = base + s * C::STAGE;
                    const uint32_t at = tmem + (uint32_t)(C::A_COL0 + a * C::A_COLS);
                    const int nch = KC - kt * C::KCH < C::KCH ? KC - kt * C::KCH : C::KCH;
                    for (int j = 0; j < nch; ++j)
#pragma unroll
                        for (int k16 = 0; k16 < 4; ++k16)
                            tc_mma_ts(d, at + j * 32 + k16 * 8, pf_sw128_desc(xa + j * C::X_CHUNK + k16 * 32), idesc,
                                      (kt | j | k16) != 0);
                    tc_commit(empty(s));
                    tc_commit(aempty(a));
                }
                if (ok) tc_commit(accfull(b));
            }
            tc_commit(done_bar);   // every MMA of this CTA retired before TMEM is released
            mbar_wait(done_bar, 0, kDevTimeoutDrain);
        }
    } else if (warp < kPfEpiWarp0) {
        // ------------------------------------------------------------ dequant -> TMEM A ring
        const int qi = (warp - 2) >> 2;                             // index among this quarter's warps
        const int nbl = 2 * (warp & 3) + (qi & 1);                  // n16 block inside the tile
        const int phase = qi >> 1;                                  // k-steps it % kPfDqPhases == phase
        const int g = lane >> 2;
        const uint32_t lane_field = (uint32_t)(16 * nbl) << 16;
        int it = 0;
        bool ok = true;
        for (int tile = blockIdx.x; tile < total && ok; tile += gridDim.x) {
            for (int kt = 0; kt < KT; ++kt, ++it) {
                if (it % kPfDqPhases != phase) continue;
                const int s = it % ST, a = it % NA;
                bool w_ok = mbar_wait(full(s), (it / ST) & 1, kDevTimeoutPipeline);
                w_ok = w_ok && mbar_wait(aempty(a), ((it / NA) & 1) ^ 1, kDevTimeoutPipeline);
                if (!__all_sync(0xffffffffu, w_ok)) { ok = false; break; }
                tc_fence_after();
                // this warp's block of every chunk of the stage: words [block][chunk][512 B],
                // scales [chunk][128]; all read before the stage is released
                const int nch = KC - kt * C::KCH < C::KCH ? KC - kt * C::KCH : C::KCH;
                const uint32_t sbw = base + s * C::STAGE + C::X_BYTES, sbs = sbw + C::W_BYTES;
                uint4 w[C::KCH];
                uint32_t s_lo[C::KCH], s_hi[C::KCH];
#pragma unroll
                for (int j = 0; j < C::KCH; ++j)
                    if (j < nch) {
                        w[j] = lds128(sbw + (uint32_t)((nbl * KB + j) * 512 + lane * 16));
                        const uint16_t* sc = reinterpret_cast<const uint16_t*>(smem_raw + (sbs + j * kPfSBytes - raw));
                        s_lo[j] = bcast_half(sc[nbl * 16 + g]);
                        s_hi[j] = bcast_half(sc[nbl * 16 + g + 8]);
                    }
                mbar_arrive(empty(s));   // this lane is done with the stage's packed words and scales
                uint32_t r[C::KCH][16];   // one register set per chunk: no store's sources are reused
#pragma unroll
                for (int j = 0; j < C::KCH; ++j)
                    if (j < nch) {
                        dequant_word(w[j].x, s_lo[j], s_hi[j], *reinterpret_cast<uint32_t(*)[4]>(&r[j][0]));
                        dequant_word(w[j].y, s_lo[j], s_hi[j], *reinterpret_cast<uint32_t(*)[4]>(&r[j][4]));
                        dequant_word(w[j].z, s_lo[j], s_hi[j], *reinterpret_cast<uint32_t(*)[4]>(&r[j][8]));
                        dequant_word(w[j].w, s_lo[j], s_hi[j], *reinterpret_cast<uint32_t(*)[4]>(&r[j][12]));
                        tmem_st_16x128b_x8(tmem + lane_field + (uint32_t)(C::A_COL0 + a * C::A_COLS + j * 32), r[j]);
                    }
                tc_wait_st();
                tc_fence_before();
                mbar_arrive(afull(a));
            }
        }
    } else {
        // ------------------------------------------------------------ epilogue
        // warp (quarter q, part h) owns output channels 32q..32q+31 of the tile (TMEM lanes)
        // and token columns [h*CW, (h+1)*CW) of the accumulator
        constexpr int CW = TOK / (kPfEpiWarps / 4);
        constexpr int EC = CW < 16 ? CW : 16;                 // columns per tcgen05.ld
        const int q = warp & 3, h = (warp - kPfEpiWarp0) >> 2;
        const uint32_t lane_field = (uint32_t)(32 * q) << 16;
        int tc = 0;
        for (int tile = blockIdx.x; tile < total; tile += gridDim.x, ++tc) {
            const int tt = tile / n_tiles, tn = tile % n_tiles;
            const int b = tc % NACC;
            if (!__all_sync(0xffffffffu, mbar_wait(accfull(b), (tc / NACC) & 1, kDevTimeoutPipeline))) break;
            tc_fence_after();
            const int n = tn * kPfRows + 32 * q + lane;
            const int tok0 = tt * TOK + h * CW;
            const uint32_t tcol = tmem + lane_field + (uint32_t)(b * TOK + h * CW);
            if (OUT_F32) {
#pragma unroll 1
                for (int c0 = 0; c0 < CW && tok0 + c0 < M; c0 += EC) {
                    uint32_t r[EC];
                    tmem_ld_cols<EC>(tcol + (uint32_t)c0, r);
                    tc_wait_ld();
                    if (n < N) {
                        const int jmax = min(EC, M - (tok0 + c0));
                        float* y = static_cast<float*>(yv) + (size_t)(tok0 + c0) * N + n;
#pragma unroll
                        for (int j = 0; j < EC; ++j)
                            if (j < jmax) y[(size_t)j * N] = __uint_as_float(r[j]);
                    }
                }
                tc_fence_before();
                mbar_arrive(accempty(b));
            } else {
                // all of this warp's columns into registers as fp16 pairs, release the
                // accumulator, then store
                uint32_t hv[CW / 2];
#pragma unroll
                for (int c0 = 0; c0 < CW; c0 += EC) {
                    uint32_t r[EC];
                    tmem_ld_cols<EC>(tcol + (uint32_t)c0, r);
                    tc_wait_ld();
#pragma unroll
                    for (int j = 0; j < EC; j += 2) {
                        const __half2 v = __floats2half2_rn(__uint_as_float(r[j]), __uint_as_float(r[j + 1]));
                        hv[(c0 + j) / 2] = *reinterpret_cast<const uint32_t*>(&v);
                    }
                }
                tc_fence_before();
                mbar_arrive(accempty(b));
                // lanes 2i and 2i+1 (channels n0, n0 + 1) trade halves so that the even lane
                // stores tokens j and the odd lane tokens j + 1 as fp16 pairs of both channels
                {
                    const int p = lane & 1;
                    const int n0 = n - p;
                    uint32_t* y32 = reinterpret_cast<uint32_t*>(static_cast<__half*>(yv) + (size_t)(tok0 + p) * N + n0);
#pragma unroll
                    for (int j = 0; j < CW; j += 2) {
                        const uint32_t w = hv[j / 2];
                        const uint32_t give = p ? w : (w >> 16);          // partner's token of the pair
                        const uint32_t got = __shfl_xor_sync(0xffffffffu, give, 1);
                        const uint32_t out = p ? __byte_perm(got, w, 0x7610) : __byte_perm(w, got, 0x5410);
                        if (n0 < N && tok0 + j + p < M) y32[(size_t)j * N / 2] = out;
                    }
                }
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) tmem_dealloc(tmem, 512);
}

// ------------------------------------------------------------------ host side
inline int pf_tok_of_config(int config) {
    switch (config) {
        case 1: return 32;
        case 2: return 64;
        case 3: return 128;
        default: return 256;
    }
}

PrefillPlan plan_prefill(int M, int N, int K, int G, int config, const DeviceInfo& dev) {
    (void)K; (void)G;
    const int n_tiles = (N + kPfRows - 1) / kPfRows;
    if (config < 1 || config > 4) {
        // Fewest waves of tiles over the SMs; among equal wave counts the smallest token tile.
        // Measured on B200 (design notes, prefill section): below one wave a smaller tile
        // spreads the same weights over more SMs and takes more K chunks per stage (6 for 32-
        // and 64-token tiles, 3 for 128), e.g. M = 128 x 4096 x 14336 in 55-59 us with 32-token
        // tiles against 65.8 with 128; once tiles fill the SMs, a 256-token tile dequantises
        // each weight tile once for twice the tokens.
        long long best = -1;
        config = 4;
        for (int c = 1; c <= 4; ++c) {
            const int tok = pf_tok_of_config(c);
            const long long tiles = (long long)n_tiles * ((M + tok - 1) / tok);
            const long long waves = (tiles + dev.num_sms - 1) / dev.num_sms;
            if (best < 0 || waves < best) { best = waves; config = c; }
        }
    }
    PrefillPlan p;
    p.config = config;
    p.tok = pf_tok_of_config(config);
    switch (p.tok) {
        case 32:  p.stages = PfCfg<32>::STAGES;  p.a_stages = PfCfg<32>::A_STAGES;  p.accs = PfCfg<32>::ACCS;  p.smem = PfCfg<32>::SMEM;  break;
        case 64:  p.stages = PfCfg<64>::STAGES;  p.a_stages = PfCfg<64>::A_STAGES;  p.accs = PfCfg<64>::ACCS;  p.smem = PfCfg<64>::SMEM;  break;
        case 128: p.stages = PfCfg<128>::STAGES; p.a_stages = PfCfg<128>::A_STAGES; p.accs = PfCfg<128>::ACCS; p.smem = PfCfg<128>::SMEM; break;
        default:  p.stages = PfCfg<256>::STAGES; p.a_stages = PfCfg<256>::A_STAGES; p.accs = PfCfg<256>::ACCS; p.smem = PfCfg<256>::SMEM; break;
    }
    p.tiles = n_tiles * ((M + p.tok - 1) / p.tok);
    p.grid = std::min(p.tiles, dev.num_sms);
    return p;
}

// Tensor maps for one call.  x: [M, K] fp16, box {64, TOK}, 128-byte swizzle.
// Packed words as [NB][KC][128] int32, box {128, min(pf_kch(TOK), KC), 8} (8 n16 blocks of a stage).
// Scales: [K/G, N] fp16, box {128, 1}.  Out-of-range boxes read as zero.
cudaError_t make_prefill_tensor_maps(const GemmArgs& a, int tok, CUtensorMap* tx, CUtensorMap* tw, CUtensorMap* ts);

template <int G, int TOK, bool F32>
static cudaError_t launch_prefill_t(const GemmArgs& a, const PrefillPlan& p) {
    CUtensorMap tx, tw, ts;
    cudaError_t err = make_prefill_tensor_maps(a, TOK, &tx, &tw, &ts);
    if (err != cudaSuccess) return err;
    auto kern = prefill_kernel<G, TOK, F32>;
    err = ensure_max_dynamic_smem(reinterpret_cast<const void*>(kern));
    if (err != cudaSuccess) return err;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(p.grid, 1, 1);
    cfg.blockDim = dim3(kPfThreads, 1, 1);
    cfg.dynamicSmemBytes = PfCfg<TOK>::SMEM;
    cfg.stream = a.stream;
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr.val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = a.pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kern, tx, tw, ts, a.y, a.M, a.N, a.K);
}

template <int G, bool F32>
static cudaError_t launch_prefill_g(const GemmArgs& a, const PrefillPlan& p) {
    switch (p.tok) {
        case 32:  return launch_prefill_t<G, 32, F32>(a, p);
        case 64:  return launch_prefill_t<G, 64, F32>(a, p);
        case 128: return launch_prefill_t<G, 128, F32>(a, p);
        default:  return launch_prefill_t<G, 256, F32>(a, p);
    }
}

cudaError_t launch_prefill(const GemmArgs& a, const PrefillPlan& p) {
    if (a.G == 64) return a.out_f32 ? launch_prefill_g<64, true>(a, p) : launch_prefill_g<64, false>(a, p);
    return a.out_f32 ? launch_prefill_g<128, true>(a, p) : launch_prefill_g<128, false>(a, p);
}

}  // namespace w4a16
