// Decode path without cross-CTA reduction (1 <= M <= 16): every CTA owns whole output
// columns.  Included by the single device-code translation unit (kernels.cu) only.
//
// On B200 a reduction of partial sums across CTAs costs microseconds per GEMM (a second
// kernel, or flags through L2 that cross the two dies), which is a large share of a
// 2-30 MB decode GEMM.  This kernel avoids it:
//
//   * CTA c owns the n16 blocks [c*NB/ctas, (c+1)*NB/ctas) over ALL of K (ctas <= #SMs):
//     at most one block more than the average, so the busiest CTA streams
//     ceil(NB/ctas)/(NB/ctas) of the mean -- and under programmatic dependent launch the
//     next GEMM's CTAs start on the SMs that finish early.  The host picks this kernel
//     when that imbalance costs less than the stream-K kernel's combine (decode.cuh).
//   * A CTA walks its blocks in batches of up to 8 and each batch's K range in steps of
//     S chunks (64-wide, S a multiple of 8).  Consumer warp w takes chunks w, w+8, ...
//     of every step for all of the batch's blocks: the activation fragments of a chunk
//     are loaded once (ldmatrix) and serve every block, and each block's accumulator is
//     a single chain in increasing K.  At the batch's end the 8 warps' sums meet in
//     shared memory and are added in warp order: a fixed order, the same for every S
//     and every M <= 16, so results are deterministic and a row does not depend on the
//     other rows of the call.
//   * One producer lane issues each step as tensor copies onto the stage's mbarrier:
//     per block its S chunks of packed words (one contiguous S*512-byte run in HBM) and
//     its scale rows, and the step's activation rows (M rows per chunk, unpadded,
//     128-byte swizzle).  ldmatrix rows >= M read a shared-memory row of zeros.
//   * The same exact dequantisation as the stream-K kernel (dequant.cuh) feeds
//     mma.sync m16n8k16 with the weights as A and the tokens as the n8 side.
//   * Programmatic dependent launch as in decode.cuh: nothing is read before
//     griddepcontrol.wait unless the caller declared its weights resident.
#pragma once
#include <cuda.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include <algorithm>

#include "decode_ns_plan.h"
#include "dequant.cuh"
#include "internal.h"
#include "ptx.cuh"

namespace w4a16 {

constexpr int kNsThreads = (kNsWarps + 1) * 32;   // consumer warps + the producer warp

template <int G, int MT, bool OUT_F32>
__global__ void __launch_bounds__(kNsThreads, 1)
decode_ns_kernel(const __grid_constant__ CUtensorMap tw, const __grid_constant__ CUtensorMap tx,
                 const __grid_constant__ CUtensorMap ts, void* __restrict__ yv, int M, int N, int K, NsPlan p,
                 int pre_stages)
{
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int ST = p.stages, S = p.S;
    auto stage = [&](int s) { return base + (uint32_t)s * p.stage_bytes; };
    auto full = [&](int s) { return base + p.bar_off + (uint32_t)s * 8; };
    auto empty = [&](int s) { return base + p.bar_off + (uint32_t)(ST + s) * 8; };

    pdl_launch_dependents();

    const int c = blockIdx.x;
    const int nb0 = p.b0(c), nb1 = p.b0(c + 1);
    const int nbat = p.batches(nb1 - nb0);
    const int KC = K >> 6, nsteps = (KC + S - 1) / S;

    if (threadIdx.x == 0) {
        for (int s = 0; s < ST; ++s) {
            mbar_init(full(s), 1);              // the producer's arrive.expect_tx + the copies' bytes
            mbar_init(empty(s), kNsWarps);      // one arrival per consumer warp
        }
    }
    if (threadIdx.x < 8) reinterpret_cast<uint4*>(smem_raw + (base - raw) + p.zero_off)[threadIdx.x] = make_uint4(0, 0, 0, 0);
    fence_mbar_init();
    __syncthreads();

    if (warp == kNsWarps) {
        // ------------------------------------------------ producer (one lane)
        if (lane != 0) return;
        const uint32_t x_bytes = (uint32_t)(S * M * 128);
        auto issue_weights = [&](int s, int bk0, int bb, int t) {   // packed words + scales of a step
            mbar_expect_tx(full(s), (uint32_t)bb * (uint32_t)(S * 512 + p.R * 32));
            for (int j = 0; j < bb; ++j) {
                tma_load_3d(stage(s) + p.w_off + (uint32_t)(j * S * 512), &tw, 0, t * S, bk0 + j, full(s));
                tma_load_2d(stage(s) + p.s_off + (uint32_t)(j * p.R * 32), &ts, (bk0 + j) * 16, (t * S * 64) / G,
                            full(s));
            }
        };
        prefetch_tmap(&tw);
        prefetch_tmap(&tx);
        prefetch_tmap(&ts);
        const int total = nbat * nsteps;
        // resident weights: the caller vouches they are settled, so the first stages'
        // packed words and scales are fetched before the previous kernel has finished
        for (int it = 0; it < pre_stages && it < ST && it < total; ++it) {
            const int k = it / nsteps, t = it % nsteps;
            const int bk0 = nb0 + p.batch_lo(nb1 - nb0, nbat, k), bk1 = nb0 + p.batch_lo(nb1 - nb0, nbat, k + 1);
            issue_weights(it, bk0, bk1 - bk0, t);
        }
        pdl_wait();   // x may still be written by the previous kernel
        int it = 0;
        for (; it < total; ++it) {
            const int s = it % ST, k = it / nsteps, t = it % nsteps;
            const int bk0 = nb0 + p.batch_lo(nb1 - nb0, nbat, k), bk1 = nb0 + p.batch_lo(nb1 - nb0, nbat, k + 1);
            if (it >= ST) {
                if (!mbar_wait_sleep(empty(s), ((it / ST) - 1) & 1, kDevTimeoutActivations)) break;
                issue_weights(s, bk0, bk1 - bk0, t);
            } else if (it >= pre_stages) {
                issue_weights(s, bk0, bk1 - bk0, t);
            }
            mbar_arrive_expect_tx(full(s), x_bytes);
            tma_load_3d(stage(s) + p.x_off, &tx, 0, 0, t * S, full(s));
        }
        // copies still in flight must land before the CTA may exit (a break happens only at
        // it >= ST, after every stage issued ahead of the loop got its arrival)
        for (int j = it - 1; j >= 0 && j >= it - ST; --j) mbar_wait(full(j % ST), (j / ST) & 1, kDevTimeoutDrain);
        return;
    }

    // ---------------------------------------------------- consumer warp w: chunks w, w+8, ... of every step
    const int g8 = lane >> 2, t4 = lane & 3;
    pdl_wait();   // y may still be in use by the previous kernel
    // ldmatrix rows: lanes 8i..8i+7 address token rows 0..7 of 8x8 matrix i (16-byte units i
    // and i+4 of the 128-byte row); a row >= M reads the zero row.  Row q of the step's
    // activation box (q = chunk*M + token) sits at q*128 with its unit u at u ^ (q % 8).
    const int xr = lane & 7, xu = lane >> 3;
    const uint32_t zero_row = base + p.zero_off + (uint32_t)(xu << 4);

    float acc[kNsMaxBatch][MT][4];
    bool ok = true;
    int it = 0;
    for (int k = 0; k < nbat && ok; ++k) {
        const int bk0 = nb0 + p.batch_lo(nb1 - nb0, nbat, k), bb = nb0 + p.batch_lo(nb1 - nb0, nbat, k + 1) - bk0;
#pragma unroll
        for (int j = 0; j < kNsMaxBatch; ++j)
#pragma unroll
            for (int mt = 0; mt < MT; ++mt)
#pragma unroll
                for (int i = 0; i < 4; ++i) acc[j][mt][i] = 0.f;
        for (int t = 0; t < nsteps; ++t, ++it) {
            const int s = it % ST;
            if (!__all_sync(0xffffffffu, mbar_wait_sleep(full(s), (it / ST) & 1, kDevTimeoutWeights))) {
                ok = false;
                break;
            }
            const uint32_t sb = stage(s);
            for (int i = warp; i < S; i += kNsWarps) {
                if (t * S + i >= KC) break;                         // chunks past K (zero-filled)
                uint32_t b[MT][8];
#pragma unroll
                for (int mt = 0; mt < MT; ++mt) {
                    const int row = mt * 8 + xr;
                    const int q = i * M + row;
                    const uint32_t ra = sb + p.x_off + (uint32_t)q * 128;
                    const uint32_t a0 = row < M ? ra + (uint32_t)((xu ^ (q & 7)) << 4) : zero_row;
                    const uint32_t a1 = row < M ? ra + (uint32_t)(((xu + 4) ^ (q & 7)) << 4) : zero_row;
                    ldmatrix_x4(*reinterpret_cast<uint32_t(*)[4]>(&b[mt][0]), a0);
                    ldmatrix_x4(*reinterpret_cast<uint32_t(*)[4]>(&b[mt][4]), a1);
                }
                const uint32_t srow = sb + p.s_off + (uint32_t)(((i * 64) / G) * 32 + g8 * 2);
                const uint32_t wrow = sb + p.w_off + (uint32_t)(i * 512 + lane * 16);
#pragma unroll
                for (int j = 0; j < kNsMaxBatch; ++j) {
                    if (j < bb) {
                        const uint32_t s_lo = bcast_half(lds_u16(srow + (uint32_t)(j * p.R * 32)));
                        const uint32_t s_hi = bcast_half(lds_u16(srow + (uint32_t)(j * p.R * 32 + 16)));
                        const uint4 w4 = lds128(wrow + (uint32_t)(j * S * 512));
#pragma unroll
                        for (int ks = 0; ks < 4; ++ks) {
                            const uint32_t wq = ks == 0 ? w4.x : ks == 1 ? w4.y : ks == 2 ? w4.z : w4.w;
                            uint32_t a[4];
                            dequant_word(wq, s_lo, s_hi, a);
#pragma unroll
                            for (int mt = 0; mt < MT; ++mt)
                                mma_16816(acc[j][mt], a, b[mt][2 * ks], b[mt][2 * ks + 1]);
                        }
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(empty(s));
        }
        // every consumer warp reaches the batch's end (a timed-out wait makes the others
        // time out too); the decision to write is the same for the whole CTA
        if (!bar_red_and_named(1, kNsWarps * 32, ok)) return;
        // the 8 warps' sums of each block, added in warp order: warp j writes block j
        const uint32_t red = base + p.red_off;
#pragma unroll
        for (int j = 0; j < kNsMaxBatch; ++j)
            if (j < bb)
#pragma unroll
                for (int mt = 0; mt < MT; ++mt)
                    sts128(red + (uint32_t)((((warp * p.bmax + j) * MT + mt) * 32 + lane) * 16),
                           make_float4(acc[j][mt][0], acc[j][mt][1], acc[j][mt][2], acc[j][mt][3]));
        bar_sync_named(1, kNsWarps * 32);
        if (warp < bb) {
            const int nb = bk0 + warp;
#pragma unroll
            for (int mt = 0; mt < MT; ++mt) {
                float v[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
                for (int ww = 0; ww < kNsWarps; ++ww) {
                    const float4 f = lds128f(red + (uint32_t)((((ww * p.bmax + warp) * MT + mt) * 32 + lane) * 16));
                    v[0] += f.x;
                    v[1] += f.y;
                    v[2] += f.z;
                    v[3] += f.w;
                }
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const int tok = mt * 8 + 2 * t4 + (i & 1);
                    if (tok < M) {
                        const size_t o = (size_t)tok * N + nb * 16 + g8 + 8 * (i >> 1);
                        if (OUT_F32) static_cast<float*>(yv)[o] = v[i];
                        else static_cast<__half*>(yv)[o] = __float2half_rn(v[i]);
                    }
                }
            }
        }
        bar_sync_named(1, kNsWarps * 32);   // the reduction buffer is read before the next batch
    }
}

// ------------------------------------------------------------------ host side
cudaError_t make_decode_ns_tensor_maps(const GemmArgs& a, const NsPlan& p, CUtensorMap* tw, CUtensorMap* tx,
                                       CUtensorMap* ts);

template <int G, int MT, bool F32>
static cudaError_t launch_decode_ns_t(const GemmArgs& a, const NsPlan& p) {
    auto kern = decode_ns_kernel<G, MT, F32>;
    cudaError_t err = ensure_max_dynamic_smem(reinterpret_cast<const void*>(kern));
    if (err != cudaSuccess) return err;
    CUtensorMap tw, tx, ts;
    if ((err = make_decode_ns_tensor_maps(a, p, &tw, &tx, &ts)) != cudaSuccess) return err;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(p.ctas, 1, 1);
    cfg.blockDim = dim3(kNsThreads, 1, 1);
    cfg.dynamicSmemBytes = p.smem;
    cfg.stream = a.stream;
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr.val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = a.pdl ? 1 : 0;
    const int pre = a.pdl && a.weights_resident ? kDcPreStages : 0;
    return cudaLaunchKernelEx(&cfg, kern, tw, tx, ts, a.y, a.M, a.N, a.K, p, pre);
}

cudaError_t launch_decode_ns(const GemmArgs& a, const NsPlan& p) {
    const bool f32 = a.out_f32;
    const bool mt1 = a.M <= 8;
    if (a.G == 64) {
        if (mt1) return f32 ? launch_decode_ns_t<64, 1, true>(a, p) : launch_decode_ns_t<64, 1, false>(a, p);
        return f32 ? launch_decode_ns_t<64, 2, true>(a, p) : launch_decode_ns_t<64, 2, false>(a, p);
    }
    if (mt1) return f32 ? launch_decode_ns_t<128, 1, true>(a, p) : launch_decode_ns_t<128, 1, false>(a, p);
    return f32 ? launch_decode_ns_t<128, 2, true>(a, p) : launch_decode_ns_t<128, 2, false>(a, p);
}

}  // namespace w4a16
