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
//     of each lane is already an m16n8k16 A fragment, so the exact
//     13-instruction dequant feeds mma.sync directly (weights = A, the <= 16
//     tokens = the n8 side); one activation fragment serves both blocks.
//   * A CTA's columns are complete in registers when it leaves a group: a group
//     covered by one CTA is written to y directly.  A group split across CTAs leaves
//     one fp32 partial per CTA in the caller's workspace (float4 fragments in register
//     order, so every store and load is a coalesced 16-byte access).  At the end of its
//     range each CTA arrives on the group's sense-reversing arrival word; once all of
//     the group's CTAs have arrived, each sums its own slice of the group's outputs over
//     every partial in CTA order and writes it to y -- one launch per GEMM, a result
//     that does not depend on arrival order, no atomics on data.
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
// next GEMM competes with the tail of the previous one for HBM.
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
    static constexpr int BAR_BYTES = 2 * ST * 8 + 16;              // full/empty barriers + 2 go flags
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

// Sums the fragments [f_lo, f_hi) of split group g's partials over its CTAs in CTA order
// and writes them to y.  Fragment f of a partial is float4 ((w*kDcBPW + bb)*MT + mt)*32 + lane
// of consumer warp w: tokens mt*8 + 2*(lane%4) + {0, 1}, columns (w*kDcBPW + bb)*16 + lane/4
// + {0, 8} of the group.  Called by the 256 consumer threads (index t).
template <int MT, bool OUT_F32>
__device__ __forceinline__ void dc_reduce_slice(const DcPartition& part, int g, int f_lo, int f_hi, int t,
                                                const float* __restrict__ partials, void* __restrict__ yv, int M,
                                                int N) {
    constexpr int kBatch = 8;   // partial loads in flight per thread
    const int cf = part.first_cta(g), pieces = part.last_cta(g) - cf + 1;
    for (int f = f_lo + t; f < f_hi; f += kDcWarps * 32) {
        const int lane = f & 31, r = f >> 5, mt = r % MT, wb = r / MT;
        const int tok0 = mt * 8 + 2 * (lane & 3);
        const int col0 = g * kDcCols + wb * 16 + (lane >> 2);
        if (tok0 >= M || col0 >= N) continue;   // padding rows, or blocks past N
        float4 sum = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int i0 = 0; i0 < pieces; i0 += kBatch) {
            float4 v[kBatch];
#pragma unroll
            for (int i = 0; i < kBatch; ++i)
                if (i0 + i < pieces)
                    v[i] = __ldcg(reinterpret_cast<const float4*>(partials + (size_t)part.piece_slot(g, i0 + i) *
                                                                                 kDcSlotFloats) + f);
#pragma unroll
            for (int i = 0; i < kBatch; ++i)
                if (i0 + i < pieces) {
                    sum.x += v[i].x;
                    sum.y += v[i].y;
                    sum.z += v[i].z;
                    sum.w += v[i].w;
                }
        }
        const float out[4] = {sum.x, sum.y, sum.z, sum.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int tok = tok0 + (i & 1), col = col0 + 8 * (i >> 1);
            if (tok < M) {
                const size_t o = (size_t)tok * N + col;
                if (OUT_F32) static_cast<float*>(yv)[o] = out[i];
                else static_cast<__half*>(yv)[o] = __float2half_rn(out[i]);
            }
        }
    }
}

template <int G, int MP, bool OUT_F32>
__global__ void __launch_bounds__(kDcThreads, 1)
decode_kernel(const __grid_constant__ CUtensorMap tw, const __grid_constant__ CUtensorMap tx,
              const __grid_constant__ CUtensorMap ts, void* __restrict__ yv, int M, int N, int box_blocks,
              int box_chunks, DcPartition part, void* __restrict__ workspace, int pre_stages)
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
    constexpr int BPW = kDcBPW;
    constexpr int CH = 2;                                          // accumulator chains per block
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

    // split groups this CTA holds a piece of (at most two: its first and its last group)
    uint32_t* const words = static_cast<uint32_t*>(workspace);
    float* const partials = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + dc_words_bytes(part));
    int pend0 = 0, pend1 = 0, npend = 0;
    bool ok = true;

    DcSteps st;
    st.start(c0, c1, KC);
    int gkc0 = st.kc;                 // first chunk of the current group inside this CTA
    for (int t = 0; st.more(); ++t) {
        const int nk = st.nk(KC), s = t % ST;
        const int nb0 = st.g * kDcBlocks + warp * BPW;      // this warp's first n16 block
        if (!__all_sync(0xffffffffu, mbar_wait_sleep(full(s), (t / ST) & 1, kDevTimeoutWeights))) { ok = false; break; }
        if (nb0 < NB) {
            const uint32_t sb = stage(s);
            // scales of this step's chunks; chunks beyond nk get scale 0 (their activations are finite)
            uint32_t s_lo[BPW][kDcStep], s_hi[BPW][kDcStep];
#pragma unroll
            for (int bb = 0; bb < BPW; ++bb)
#pragma unroll
                for (int j = 0; j < kDcStep; ++j) {
                    const uint32_t sa = sb + s_lane + bb * 32 + j * C::SROW;
                    const uint16_t lo = lds_u16(sa);
                    const uint16_t hi = lds_u16(sa + 16);
                    s_lo[bb][j] = j < nk ? bcast_half(lo) : 0u;
                    s_hi[bb][j] = j < nk ? bcast_half(hi) : 0u;
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
                // No per-chunk guard: the unconditional body lets the accumulator chains interleave.
                // The activation fragments of a chunk serve both blocks.
#pragma unroll
                for (int ks = 0; ks < 4; ++ks)
#pragma unroll
                    for (int jj = 0; jj < JB; ++jj)
#pragma unroll
                        for (int bb = 0; bb < BPW; ++bb) {
                            const uint4 w4 = wv[jj][bb];
                            const uint32_t wq = ks == 0 ? w4.x : ks == 1 ? w4.y : ks == 2 ? w4.z : w4.w;
                            uint32_t a[4];
                            dequant_word(wq, s_lo[bb][jb + jj], s_hi[bb][jb + jj], a);
#pragma unroll
                            for (int mt = 0; mt < MT; ++mt)
                                mma_16816(acc[bb][(jb + jj) % CH][mt], a, b[jj][mt][2 * ks], b[jj][mt][2 * ks + 1]);
                        }
            }
        }
        // release the stage to the producer
        __syncwarp();
        if (lane == 0) mbar_arrive(empty(s));
        const int g = st.g;
        const bool whole = st.kc + nk == KC && gkc0 == 0;
        if (st.advance(nk, KC)) {
            // this CTA's part of group g is done: fold the chains (fixed order) and store
#pragma unroll
            for (int bb = 0; bb < BPW; ++bb) {
                const int nb = g * kDcBlocks + warp * BPW + bb;
                const int colb = (warp * BPW + bb) * 16 + g8;           // column inside the group
#pragma unroll
                for (int mt = 0; mt < MT; ++mt) {
                    float v[4];
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        v[i] = 0.f;
#pragma unroll
                        for (int ch = 0; ch < CH; ++ch) {
                            v[i] += acc[bb][ch][mt][i];
                            acc[bb][ch][mt][i] = 0.f;
                        }
                    }
                    if (whole) {
#pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            const int tok = mt * 8 + 2 * t4 + (i & 1);
                            const int dc = 8 * (i >> 1);
                            if (nb < NB && tok < M) {
                                const size_t o = (size_t)tok * N + g * kDcCols + colb + dc;
                                if (OUT_F32) static_cast<float*>(yv)[o] = v[i];
                                else static_cast<__half*>(yv)[o] = __float2half_rn(v[i]);
                            }
                        }
                    } else {
                        float4* const my = reinterpret_cast<float4*>(partials + (size_t)part.slot(c, g) * kDcSlotFloats);
                        __stcg(my + ((warp * BPW + bb) * MT + mt) * 32 + lane, make_float4(v[0], v[1], v[2], v[3]));
                    }
                }
            }
            if (!whole) {
                if (npend == 0) pend0 = g;
                else pend1 = g;
                ++npend;
            }
            gkc0 = 0;
        }
    }

    // ------------------------------------------------ split groups: arrive, then reduce this CTA's slice
    if (npend == 0) return;
    volatile uint32_t* const s_go = reinterpret_cast<volatile uint32_t*>(smem_raw + (bars - raw) + 2 * ST * 8);
    // Every consumer warp gets here, also after a timed-out wait (the others then time out
    // too); the barrier orders every consumer's partial stores before the arrival and makes
    // the go / no-go decision the same for the whole CTA.
    if (!bar_red_and_named(1, kDcWarps * 32, ok)) return;
    if (threadIdx.x == 0) {
        // Arrival word: bit 31 = phase sense, bits 0..30 = arrivals.  The CTA whose arrival
        // completes the count starts the next phase (count 0, sense flipped) with a release
        // store; the others wait for the flip.  The acq_rel atomic releases this CTA's
        // partial (ordered before it by the barrier) and acquires the earlier arrivals'.
        const uint32_t old0 = atom_add_acq_rel_gpu(words + pend0, 1u);
        const uint32_t old1 = npend > 1 ? atom_add_acq_rel_gpu(words + pend1, 1u) : 0u;
        for (int j = 0; j < npend; ++j) {
            const int g = j ? pend1 : pend0;
            const uint32_t old = j ? old1 : old0;
            const uint32_t pieces = (uint32_t)(part.last_cta(g) - part.first_cta(g) + 1);
            if ((old & 0x7FFFFFFFu) == pieces - 1) {
                st_release_gpu(words + g, (old & 0x80000000u) ^ 0x80000000u);
                s_go[j] = 1;
            } else {
                s_go[j] = wait_sense_flip(words + g, old >> 31, kDevTimeoutSplit) ? 1 : 0;
            }
        }
    }
    bar_sync_named(1, kDcWarps * 32);
    for (int j = 0; j < npend; ++j) {
        if (!s_go[j]) continue;
        const int g = j ? pend1 : pend0;
        const int cf = part.first_cta(g), pieces = part.last_cta(g) - cf + 1;
        constexpr int F = kDcWarps * kDcBPW * MT * 32;                 // fragments per partial
        const int i = c - cf;
        dc_reduce_slice<MT, OUT_F32>(part, g, part.slice_lo(i, pieces, F), part.slice_lo(i + 1, pieces, F),
                                     threadIdx.x, partials, yv, M, N);
    }
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
    p.launches = 1;
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

template <int G, int MP, bool F32>
static cudaError_t launch_decode_t(const GemmArgs& a, const DecodePlan& p) {
    (void)p;
    auto kern = decode_kernel<G, MP, F32>;
    cudaError_t err = ensure_max_dynamic_smem(reinterpret_cast<const void*>(kern));
    if (err != cudaSuccess) return err;
    DeviceInfo dev;
    if ((err = device_info(&dev)) != cudaSuccess) return err;
    const DcPartition part = dc_partition(a.N, a.K, dev.num_sms);
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
    return cudaLaunchKernelEx(&cfg, kern, tw, tx, ts, a.y, a.M, a.N, box_blocks, box_chunks, part, a.workspace, pre);
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
