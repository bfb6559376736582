// Decode path (1 <= M <= 16): persistent stream-K weight-streaming GEMV.
// Included by the single device-code translation unit (kernels.cu) only.
//
// Replaces the reference's decode kernel (src/vectorized/decode.cuh:18-159 and
// its launcher kernel.cu:19-53), whose grid of N/64 CTAs leaves most of a
// 148-SM B200 idle, with a design built around HBM3e streaming:
//
//   * Output columns form groups of 256 (16 n16 blocks).  The work is the
//     sequence of (group, 64-wide K chunk) pairs, group-major, cut into equal
//     contiguous ranges, one per SM (stream-K): every SM moves the same number
//     of packed-word bytes (to one chunk) whatever N and K are.  Small GEMMs use
//     fewer CTAs (at least kDcMinUnits chunks each) so fewer partials are combined.
//   * One CTA per SM: 8 consumer warps + 1 producer warp.  A CTA walks its range
//     in steps of up to kDcStep chunks inside one group.  One producer lane
//     issues each step as tensor copies (TMA) onto the stage's single mbarrier:
//     the packed words of the group's 16 n16 blocks in ONE box -- for each block
//     its kDcStep chunks are one contiguous run in HBM (2 KB), which DRAM serves
//     far better than 512-byte pieces -- the token rows of the step's chunks in
//     one box (128-byte swizzle, rows >= M zero-filled) and the group's scales.
//   * Consumer warp w owns n16 blocks 2w and 2w+1 of the group.  The packed word
//     of each lane is already an m16n8k16 A fragment, so the exact 13-instruction
//     dequant (the reference's fp16 values, bit for bit) feeds mma.sync directly
//     (weights = A, the <= 16 tokens = the n8 side; one activation fragment serves
//     both blocks).  With W4A16_FLAG_FP32_SCALE and M <= 8 the fragment holds the
//     exact integers q - 8 instead (9 instructions) and each chunk's products are
//     scaled in fp32 after the tensor core, one FMA per accumulator element.
//   * A CTA's columns are complete in registers when it leaves a group: a group
//     covered by one CTA is written to y directly; a group split across CTAs
//     leaves one fp32 partial per CTA in the caller's workspace, and
//     decode_combine_kernel (launched behind with programmatic dependent launch)
//     sums them in CTA order -- deterministic, no atomics, no counters.
//   * Programmatic dependent launch: dependents may launch as soon as every CTA has
//     started.  By default nothing is read from global memory before
//     griddepcontrol.wait, so the GEMM is ordered after whatever the previous kernel
//     on the stream wrote, weights included.  A caller that declares its weights
//     resident (W4A16_FLAG_WEIGHTS_RESIDENT: not written by the kernel launched just
//     before) lets the producer issue the first ring stages of packed words and
//     scales before the wait, so they stream while the previous kernel finishes.
#pragma once
#include <cuda.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include <algorithm>
#include <map>
#include <mutex>
#include <tuple>

#include "decode_partition.h"
#include "dequant.cuh"
#include "internal.h"
#include "ptx.cuh"

namespace w4a16 {

constexpr int kDcBPW = 2;                                 // n16 blocks per consumer warp
constexpr int kDcWarps = kDcBlocks / kDcBPW;              // consumer warps; warp w owns blocks 2w, 2w+1
constexpr int kDcThreads = (kDcWarps + 1) * 32;           // + the producer warp
// Ring stages of packed words and scales issued before griddepcontrol.wait when the
// caller declares its weights resident.  More is not better: a deep early burst from the
// next GEMM delays the previous GEMM's combine kernel (measured on the decode sweep:
// 2 stages 2073 GB/s, all 5 stages 1934 GB/s).
constexpr int kDcPreStages = 2;

template <int MP>
struct DcCfg {
    static constexpr int ST = 5;                                  // stages: steps in flight
    static constexpr int W_CHUNK = kDcBlocks * 512;               // packed words of one chunk of a group (8 KB)
    static constexpr int W_BYTES = kDcStep * W_CHUNK;             // [n16 block][chunk][32 lanes x 16 B]
    static constexpr int X_CHUNK = MP * 128;                      // one chunk's token rows (128-byte swizzle)
    static constexpr int X_BYTES = kDcStep * X_CHUNK;             // [chunk][token row][128 B]
    static constexpr int SROW = kDcCols * 2;                      // one chunk's scales of the group (512 B)
    static constexpr int S_BYTES = kDcStep * SROW;
    static constexpr int STAGE_BYTES = W_BYTES + X_BYTES + S_BYTES;
    static constexpr int BAR_BYTES = 2 * ST * 8;
    static constexpr int SMEM = 1024 + ST * STAGE_BYTES + BAR_BYTES;
    static_assert(STAGE_BYTES % 1024 == 0 && X_CHUNK % 1024 == 0, "stage alignment (128-byte swizzle atoms)");
    static_assert(SMEM <= 227 * 1024, "shared memory budget");
};

// The partition of a shape, computed once per (N, K, #SMs): a GEMM call consults it a few
// times on the host, and finding whether a group is split walks every CTA boundary.
inline DcPartition dc_partition(int N, int K, int num_sms) {
    static std::mutex mu;
    static std::map<std::tuple<int, int, int>, DcPartition> cache;
    const auto key = std::make_tuple(N, K, num_sms);
    std::lock_guard<std::mutex> lk(mu);
    const auto it = cache.find(key);
    if (it != cache.end()) return it->second;
    if (cache.size() >= 4096) cache.clear();
    return cache[key] = dc_cut(N, K, num_sms);
}

template <int G, int MP, bool OUT_F32, bool FP32_SCALE>
__global__ void __launch_bounds__(kDcThreads, 1)
decode_kernel(const __grid_constant__ CUtensorMap tw, const __grid_constant__ CUtensorMap tx,
              const __grid_constant__ CUtensorMap ts, void* __restrict__ yv, int M, int N, int box_blocks,
              int box_chunks, DcPartition part, float* __restrict__ partials, int pre_stages)
{
    using C = DcCfg<MP>;
    constexpr int ST = C::ST;
    constexpr int MT = MP / 8;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    const uint32_t bars = base + ST * C::STAGE_BYTES;
    auto stage = [&](int s) { return base + (uint32_t)s * C::STAGE_BYTES; };
    auto full = [&](int s) { return bars + (uint32_t)s * 8; };
    auto empty = [&](int s) { return bars + (uint32_t)(ST + s) * 8; };

    // The next kernel may launch as soon as every CTA of this one has started: it only
    // prepares and streams weights until its own griddepcontrol.wait releases it.
    pdl_launch_dependents();

    const int c = blockIdx.x;
    const int c0 = part.c0(c), c1 = part.c0(c + 1);
    const int KC = part.kc, NB = N >> 4;

    if (threadIdx.x == 0) {
        for (int s = 0; s < ST; ++s) {
            mbar_init(full(s), 1);           // the producer's arrive.expect_tx + all tensor-copy bytes
            mbar_init(empty(s), kDcWarps);   // one arrival per consumer warp
        }
    }
    fence_mbar_init();
    if (box_chunks < kDcStep) {
        // K < 256: a step's token-row box covers fewer than kDcStep chunks and the rest of the
        // stage's rows are never written; zero them once so those chunks (whose scales are
        // zero) multiply finite values.
        uint8_t* const gbase = smem_raw + (base - raw);
        for (int s = 0; s < ST; ++s)
            for (int i = threadIdx.x; i < C::X_BYTES / 16; i += kDcThreads)
                reinterpret_cast<uint4*>(gbase + s * C::STAGE_BYTES + C::W_BYTES)[i] = make_uint4(0, 0, 0, 0);
        fence_proxy_async_smem();   // the zeros land before any tensor copy into the same rows
    }
    __syncthreads();

    if (warp == kDcWarps) {
        // ------------------------------------------------ producer (one lane): all of a step by tensor copies
        // Per step: the packed words of up to 16 n16 blocks x box_chunks chunks in one box into
        // [block][chunk][512 B] (chunks past K and blocks past N zero-filled); the token rows of
        // the step's chunks (box 64 x MP x box_chunks, rows >= M zero-filled, 128-byte swizzle)
        // into [chunk][row][128 B]; per chunk the group's scales (box 256 x 1).  Chunks of a box
        // past the step's nk are loaded but their scales stay zero, so they add nothing.
        if (lane != 0) return;
        const uint32_t w_bytes = (uint32_t)(box_blocks * box_chunks * 512), s_bytes = (uint32_t)(box_blocks * 16 * 2);
        const uint32_t x_bytes = (uint32_t)(box_chunks * C::X_CHUNK);
        auto issue_weights = [&](int s, const DcSteps& w, int nk) {   // packed words + scales
            mbar_expect_tx(full(s), w_bytes + (uint32_t)nk * s_bytes);
            tma_load_3d(stage(s), &tw, 0, w.kc, w.g * kDcBlocks, full(s));
            for (int j = 0; j < nk; ++j)
                tma_load_2d(stage(s) + C::W_BYTES + C::X_BYTES + j * C::SROW, &ts, w.g * kDcCols,
                            ((w.kc + j) * 64) / G, full(s));
        };
        DcSteps st;
        st.start(c0, c1, KC);
        prefetch_tmap(&tw);
        prefetch_tmap(&tx);
        prefetch_tmap(&ts);
        {
            DcSteps w = st;                  // resident weights: the caller vouches they are settled
            for (int t = 0; t < pre_stages && t < ST && w.more(); ++t) {
                const int nk = w.nk(KC);
                issue_weights(t, w, nk);
                w.advance(nk, KC);
            }
        }
        pdl_wait();   // x may still be written by the previous kernel
        int t = 0;
        for (; st.more(); ++t) {
            const int nk = st.nk(KC), s = t % ST;
            if (t >= ST) {
                if (!mbar_wait_sleep(empty(s), ((t / ST) - 1) & 1, kDevTimeoutActivations)) break;
                issue_weights(s, st, nk);
            } else if (t >= pre_stages) {
                issue_weights(s, st, nk);
            }
            mbar_arrive_expect_tx(full(s), x_bytes);
            tma_load_3d(stage(s) + C::W_BYTES, &tx, 0, 0, st.kc, full(s));
            st.advance(nk, KC);
        }
        // Tensor copies still in flight must land before the CTA may exit: normally the last ST
        // phases have completed already; after a consumer timeout they may not have.  (A break
        // happens only at t >= ST, after every step issued ahead of the loop got its arrival.)
        for (int j = t - 1; j >= 0 && j >= t - ST; --j) mbar_wait(full(j % ST), (j / ST) & 1, kDevTimeoutDrain);
        return;
    }

    // ---------------------------------------------------- consumer warp: n16 blocks 2*warp, 2*warp+1 of each group
    // Default: each word is dequantised exactly to the reference's fp16 (q - 8) * s (13
    // instructions) and the products accumulate directly.
    // FP32_SCALE, M <= 8 (MT = 1): per 64-wide chunk and n16 block, a chain of four m16n8k16
    // products of the exact integers q - 8 (fp16; 9 instructions a word) with the
    // activations, started from zero, then one fp32 FMA per accumulator element by the
    // chunk's scale (a chunk never straddles two scale groups: G is a multiple of 64).  Not
    // used for M > 8: with twice the tensor-core work per word it measured slower there (q/o
    // 9.6 against 7.8 us at M = 16).
    // Either way a block's sums alternate between two accumulator sets, added at the end.
    constexpr int BPW = kDcBPW;
    constexpr int CH = 2;
    constexpr bool SCALE_AFTER = FP32_SCALE && MT == 1;
    const int g8 = lane >> 2, t4 = lane & 3;
    pdl_wait();   // the workspace and y may still be in use by the previous kernel

    const uint32_t w_blk = (uint32_t)box_chunks * 512;            // block stride of a stage's packed words
    const uint32_t w_lane = (uint32_t)warp * BPW * w_blk + lane * 16;
    // ldmatrix row addresses in a 128-byte-swizzled chunk of token rows: row r's 16-byte unit u
    // sits at unit u ^ (r % 8); lanes 8i..8i+7 address rows 0..7 of 8x8 matrix i (k units i, i+4)
    const uint32_t xr = (uint32_t)(lane & 7), xu = (uint32_t)(lane >> 3);
    const uint32_t x_lane0 = C::W_BYTES + xr * 128 + ((xu ^ xr) << 4);
    const uint32_t x_lane1 = C::W_BYTES + xr * 128 + (((xu + 4) ^ xr) << 4);
    const uint32_t s_lane = (uint32_t)(C::W_BYTES + C::X_BYTES + warp * BPW * 32 + g8 * 2);

    float acc[BPW][CH][MT][4];
#pragma unroll
    for (int bb = 0; bb < BPW; ++bb)
#pragma unroll
        for (int ch = 0; ch < CH; ++ch)
#pragma unroll
            for (int mt = 0; mt < MT; ++mt)
#pragma unroll
                for (int i = 0; i < 4; ++i) acc[bb][ch][mt][i] = 0.f;

    DcSteps st;
    st.start(c0, c1, KC);
    int gkc0 = st.kc;                 // first chunk of the current group inside this CTA
    for (int t = 0; st.more(); ++t) {
        const int nk = st.nk(KC), s = t % ST;
        const int nb0 = st.g * kDcBlocks + warp * BPW;      // this warp's first n16 block
        if (!__all_sync(0xffffffffu, mbar_wait_sleep(full(s), (t / ST) & 1, kDevTimeoutWeights))) break;
        if (nb0 < NB) {
            const uint32_t sb = stage(s);
            // scales of this step's chunks (rows g8 and g8 + 8 of each block), as fp32 or as
            // broadcast fp16 pairs; chunks beyond nk get scale 0 (their products are finite)
            float f_lo[BPW][kDcStep], f_hi[BPW][kDcStep];
            uint32_t h_lo[BPW][kDcStep], h_hi[BPW][kDcStep];
#pragma unroll
            for (int bb = 0; bb < BPW; ++bb)
#pragma unroll
                for (int j = 0; j < kDcStep; ++j) {
                    const uint32_t sa = sb + s_lane + bb * 32 + j * C::SROW;
                    const uint16_t lo = lds_u16(sa);
                    const uint16_t hi = lds_u16(sa + 16);
                    if (SCALE_AFTER) {
                        f_lo[bb][j] = j < nk ? __half2float(__ushort_as_half(lo)) : 0.f;
                        f_hi[bb][j] = j < nk ? __half2float(__ushort_as_half(hi)) : 0.f;
                    } else {
                        h_lo[bb][j] = j < nk ? bcast_half(lo) : 0u;
                        h_hi[bb][j] = j < nk ? bcast_half(hi) : 0u;
                    }
                }
            const uint32_t wb = sb + w_lane;
            constexpr int JB = MT == 1 ? 4 : 2;                // chunks whose operands are loaded together
#pragma unroll
            for (int jb = 0; jb < kDcStep; jb += JB) {
                uint4 wv[JB][BPW];
                uint32_t b[JB][MT][8];
#pragma unroll
                for (int jj = 0; jj < JB; ++jj) {
#pragma unroll
                    for (int bb = 0; bb < BPW; ++bb) wv[jj][bb] = lds128(wb + (jb + jj) * 512 + bb * w_blk);
#pragma unroll
                    for (int mt = 0; mt < MT; ++mt) {
                        const uint32_t xa = sb + (jb + jj) * C::X_CHUNK + mt * 1024;
                        ldmatrix_x4(*reinterpret_cast<uint32_t(*)[4]>(&b[jj][mt][0]), xa + x_lane0);
                        ldmatrix_x4(*reinterpret_cast<uint32_t(*)[4]>(&b[jj][mt][4]), xa + x_lane1);
                    }
                }
                // No per-chunk guard: the unconditional body lets the chains interleave.  The
                // activation fragments of a chunk serve both blocks.
                if constexpr (SCALE_AFTER) {
                    float cc[JB][BPW][MT][4];
#pragma unroll
                    for (int ks = 0; ks < 4; ++ks)
#pragma unroll
                        for (int jj = 0; jj < JB; ++jj)
#pragma unroll
                            for (int bb = 0; bb < BPW; ++bb) {
                                const uint4 w4 = wv[jj][bb];
                                const uint32_t wq = ks == 0 ? w4.x : ks == 1 ? w4.y : ks == 2 ? w4.z : w4.w;
                                uint32_t a[4];
                                unscaled_word(wq, a);
#pragma unroll
                                for (int mt = 0; mt < MT; ++mt) {
                                    if (ks == 0) mma_16816_zero(cc[jj][bb][mt], a, b[jj][mt][0], b[jj][mt][1]);
                                    else mma_16816(cc[jj][bb][mt], a, b[jj][mt][2 * ks], b[jj][mt][2 * ks + 1]);
                                }
                            }
                    // C fragment: elements 0, 1 are row g8 of the block, 2, 3 row g8 + 8
#pragma unroll
                    for (int jj = 0; jj < JB; ++jj)
#pragma unroll
                        for (int bb = 0; bb < BPW; ++bb)
#pragma unroll
                            for (int mt = 0; mt < MT; ++mt)
#pragma unroll
                                for (int i = 0; i < 4; ++i) {
                                    float& d = acc[bb][(jb + jj) % CH][mt][i];
                                    d = fmaf(i < 2 ? f_lo[bb][jb + jj] : f_hi[bb][jb + jj], cc[jj][bb][mt][i], d);
                                }
                } else {
#pragma unroll
                    for (int ks = 0; ks < 4; ++ks)
#pragma unroll
                        for (int jj = 0; jj < JB; ++jj)
#pragma unroll
                            for (int bb = 0; bb < BPW; ++bb) {
                                const uint4 w4 = wv[jj][bb];
                                const uint32_t wq = ks == 0 ? w4.x : ks == 1 ? w4.y : ks == 2 ? w4.z : w4.w;
                                uint32_t a[4];
                                dequant_word(wq, h_lo[bb][jb + jj], h_hi[bb][jb + jj], a);
#pragma unroll
                                for (int mt = 0; mt < MT; ++mt)
                                    mma_16816(acc[bb][(jb + jj) % CH][mt], a, b[jj][mt][2 * ks], b[jj][mt][2 * ks + 1]);
                            }
                }
            }
        }
        // release the stage to the producer
        __syncwarp();
        if (lane == 0) mbar_arrive(empty(s));
        const int g = st.g;
        const bool whole = st.kc + nk == KC && gkc0 == 0;
        if (st.advance(nk, KC)) {
            // this CTA's part of group g is done: fold the two sets (fixed order) and store
            float* const my = partials + (size_t)part.slot(c, g) * kDcSlotFloats;
#pragma unroll
            for (int bb = 0; bb < BPW; ++bb) {
                const int nb = g * kDcBlocks + warp * BPW + bb;
                const int colb = (warp * BPW + bb) * 16 + g8;           // column inside the group
#pragma unroll
                for (int mt = 0; mt < MT; ++mt)
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        const int tok = mt * 8 + 2 * t4 + (i & 1);
                        float v = 0.f;
#pragma unroll
                        for (int ch = 0; ch < CH; ++ch) {
                            v += acc[bb][ch][mt][i];
                            acc[bb][ch][mt][i] = 0.f;
                        }
                        if (nb < NB && tok < M) {
                            const int dc = 8 * (i >> 1);
                            if (whole) {
                                const size_t o = (size_t)tok * N + g * kDcCols + colb + dc;
                                if (OUT_F32) static_cast<float*>(yv)[o] = v;
                                else static_cast<__half*>(yv)[o] = __float2half_rn(v);
                            } else {
                                __stcg(my + tok * kDcCols + colb + dc, v);
                            }
                        }
                    }
            }
            gkc0 = 0;
        }
    }
}

// Combines the groups that the stream-K partition split across CTAs: one CTA per
// (group, token); groups owned by a single CTA were written by decode_kernel already.
// Launched right behind decode_kernel with programmatic dependent launch, so it is
// resident early and griddepcontrol.wait releases it once decode_kernel's writes are
// complete and visible.  Sums the partials in CTA order (deterministic); the loads of
// 8 partials are issued together so the sum is not one serial chain of L2 trips.
template <bool OUT_F32>
__global__ void __launch_bounds__(kDcCols) decode_combine_kernel(void* __restrict__ yv, int N, DcPartition part,
                                                                 const float* __restrict__ partials) {
    const int g = blockIdx.x, tok = blockIdx.y;
    const int cf = part.first_cta(g), cl = part.last_cta(g);
    pdl_launch_dependents();
    if (cf == cl) return;
    pdl_wait();
    const int col = g * kDcCols + threadIdx.x;
    if (col >= N) return;
    // CTA cf may have started in an earlier group (its second slot); every later CTA
    // of the group starts inside it (its first slot, 2 * cc).
    const float* const p = partials + tok * kDcCols + threadIdx.x;
    const int slot_f = part.slot(cf, g);
    float sum = 0.f;
    for (int cc = cf; cc <= cl; cc += 8) {
        float v[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int c = cc + i;
            v[i] = c <= cl ? __ldcg(p + (size_t)(c == cf ? slot_f : 2 * c) * kDcSlotFloats) : 0.f;
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) sum += v[i];
    }
    if (OUT_F32) static_cast<float*>(yv)[(size_t)tok * N + col] = sum;
    else static_cast<__half*>(yv)[(size_t)tok * N + col] = __float2half_rn(sum);
}

// ------------------------------------------------------------------ host side
DecodePlan plan_decode(int M, int N, int K, int G, const DeviceInfo& dev) {
    (void)G;
    DecodePlan p;
    const DcPartition part = dc_partition(N, K, dev.num_sms);
    p.mt = M <= 8 ? 1 : 2;
    p.ctas = part.ctas;
    p.units = part.total;
    p.stages = DcCfg<8>::ST;
    p.smem = p.mt == 1 ? DcCfg<8>::SMEM : DcCfg<16>::SMEM;
    p.workspace = dc_workspace_bytes(part);
    p.launches = part.split ? 2 : 1;
    p.valid = part.valid;
    return p;
}

size_t decode_workspace_bytes(int N, int K, const DeviceInfo& dev) {
    return dc_workspace_bytes(dc_partition(N, K, dev.num_sms));
}

// Tensor maps of the decode kernel (kernels.cu): packed words viewed as [NB][KC][128] int32,
// box {128, box_chunks, box_blocks}; x viewed as [KC][M][64] fp16, box {64, MP, box_chunks}
// with 128-byte swizzle; scales [K/G, N] fp16, box {16 * box_blocks, 1}.
cudaError_t make_decode_tensor_maps(const GemmArgs& a, int box_blocks, int box_chunks, int mp, CUtensorMap* tw,
                                    CUtensorMap* tx, CUtensorMap* ts);

template <int G, int MP, bool F32, bool FS>
static cudaError_t launch_decode_t(const GemmArgs& a, const DecodePlan& p) {
    (void)p;
    auto kern = decode_kernel<G, MP, F32, FS>;
    cudaError_t err = ensure_max_dynamic_smem(reinterpret_cast<const void*>(kern));
    if (err != cudaSuccess) return err;
    DeviceInfo dev;
    if ((err = device_info(&dev)) != cudaSuccess) return err;
    const DcPartition part = dc_partition(a.N, a.K, dev.num_sms);
    float* partials = static_cast<float*>(a.workspace);
    const int box_blocks = std::min(kDcBlocks, a.N / 16);
    const int box_chunks = std::min(kDcStep, a.K / 64);
    CUtensorMap tw, tx, ts;
    if ((err = make_decode_tensor_maps(a, box_blocks, box_chunks, MP, &tw, &tx, &ts)) != cudaSuccess) return err;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(part.ctas, 1, 1);
    cfg.blockDim = dim3(kDcThreads, 1, 1);   // consumer warps + 1 producer warp
    cfg.dynamicSmemBytes = DcCfg<MP>::SMEM;
    cfg.stream = a.stream;
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr.val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = a.pdl ? 1 : 0;
    const int pre = a.pdl && a.weights_resident ? kDcPreStages : 0;
    err = cudaLaunchKernelEx(&cfg, kern, tw, tx, ts, a.y, a.M, a.N, box_blocks, box_chunks, part, partials, pre);
    if (err != cudaSuccess || !part.split) return err;
    // combine split groups; always launched programmatically dependent on decode_kernel
    cudaLaunchConfig_t fc = {};
    fc.gridDim = dim3(part.groups, a.M, 1);
    fc.blockDim = dim3(kDcCols, 1, 1);
    fc.stream = a.stream;
    cudaLaunchAttribute fattr;
    fattr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
    fattr.val.programmaticStreamSerializationAllowed = 1;
    fc.attrs = &fattr;
    fc.numAttrs = 1;
    return cudaLaunchKernelEx(&fc, decode_combine_kernel<F32>, a.y, a.N, part, static_cast<const float*>(partials));
}

template <int G, int MP, bool F32>
static cudaError_t launch_decode_fs(const GemmArgs& a, const DecodePlan& p) {
    // the fp32-scale form exists for M <= 8 only (MP = 8)
    if (MP == 8 && a.fp32_scale) return launch_decode_t<G, MP, F32, MP == 8>(a, p);
    return launch_decode_t<G, MP, F32, false>(a, p);
}

cudaError_t launch_decode(const GemmArgs& a, const DecodePlan& p) {
    const bool f32 = a.out_f32;
    if (a.G == 64) {
        if (p.mt == 1) return f32 ? launch_decode_fs<64, 8, true>(a, p) : launch_decode_fs<64, 8, false>(a, p);
        return f32 ? launch_decode_fs<64, 16, true>(a, p) : launch_decode_fs<64, 16, false>(a, p);
    }
    if (p.mt == 1) return f32 ? launch_decode_fs<128, 8, true>(a, p) : launch_decode_fs<128, 8, false>(a, p);
    return f32 ? launch_decode_fs<128, 16, true>(a, p) : launch_decode_fs<128, 16, false>(a, p);
}

}  // namespace w4a16
