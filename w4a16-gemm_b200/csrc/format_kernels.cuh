// Load-time weight preparation on the GPU: quantisation of fp32/fp16 weights to 4-bit
// codes with fp16 group scales, and packing of codes into the kernels' word order.
// Included by the single device-code translation unit (kernels.cu) only.
//
// Semantics are the reference's load-time helpers (tests/quant.py:34-48 pack_int4,
// 62-74 quantize_w4), bit for bit:
//   scale[g, n] = fp16( max(absmax(W[n, gG:(g+1)G]) / 7, 1e-4) )      (fp32 math, one fp16 rounding)
//   q[n, k]     = clamp(round_half_even(W[n, k] / scale), -8, 7) + 8    (fp32 IEEE division)
//   word (((n/16)*(K/64) + k/64)*32 + lane)*4 + (k%64)/16, nibble i at bits 4i..4i+3 holds
//   the code at n = 16*nb + g + 8*((i&3)&1), k = 64*kc + 16*s + 2t + 8*((i&3)>>1) + (i>>2),
//   g = lane/4, t = lane%4.
//
// Both are HBM-bound streaming passes: a CTA stages one tile (16 rows of W or of the
// codes) in shared memory with coalesced 16-byte loads and writes whole 512-byte runs of
// packed words.
#pragma once
#include <cuda_fp16.h>
#include <stdint.h>

#include "internal.h"

namespace w4a16 {

constexpr int kFmtThreads = 128;

// The word of (lane, s) in a 16-row x 64-column tile of codes held in shared memory,
// row stride `ld` bytes (codes in the low 4 bits).
__device__ __forceinline__ uint32_t pack_word_from_tile(const uint8_t* tile, int ld, int lane, int s) {
    const int g = lane >> 2, t = lane & 3;
    uint32_t w = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int p = i & 3, h = i >> 2;
        const int n = g + 8 * (p & 1);
        const int k = 16 * s + 2 * t + 8 * (p >> 1) + h;
        w |= (uint32_t)(tile[n * ld + k] & 0xF) << (4 * i);
    }
    return w;
}

// codes uint8 [N, K] -> packed int32 words.  Grid (K/64, N/16): one 16 x 64 tile, 128 words.
__global__ void __launch_bounds__(kFmtThreads) pack_kernel(const uint8_t* __restrict__ q, uint32_t* __restrict__ wp,
                                                            int N, int K) {
    __shared__ __align__(16) uint8_t tile[16 * 64];
    const int kc = blockIdx.x, nb = blockIdx.y, KC = K >> 6;
    {   // 16 rows x 64 bytes = 64 uint4, one per thread of the first 64
        const int r = threadIdx.x >> 2, c = (threadIdx.x & 3) * 16;
        if (threadIdx.x < 64)
            *reinterpret_cast<uint4*>(tile + r * 64 + c) =
                __ldg(reinterpret_cast<const uint4*>(q + (size_t)(nb * 16 + r) * K + kc * 64 + c));
    }
    __syncthreads();
    const int lane = threadIdx.x >> 2, s = threadIdx.x & 3;
    wp[((size_t)(nb * KC + kc) * 32 + lane) * 4 + s] = pack_word_from_tile(tile, 64, lane, s);
    (void)N;
}

template <typename T>
__device__ __forceinline__ float to_f32(T v);
template <>
__device__ __forceinline__ float to_f32<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_f32<__half>(__half v) { return __half2float(v); }

// W [N, K] (fp32 or fp16) -> scales fp16 [K/G, N] and either codes uint8 [N, K] (PACK =
// false) or packed words (PACK = true).  Grid (K/G, N/16): one tile of 16 rows x G columns.
template <typename T, int G, bool PACK>
__global__ void __launch_bounds__(kFmtThreads) quantize_kernel(const T* __restrict__ W, uint8_t* __restrict__ q,
                                                                uint32_t* __restrict__ wp, __half* __restrict__ scales,
                                                                int N, int K) {
    __shared__ float tile[16][G + 4];
    __shared__ float srow[16];
    __shared__ __align__(16) uint8_t codes[16 * G];
    const int gi = blockIdx.x, nb = blockIdx.y;
    const int k0 = gi * G, n0 = nb * 16;
    constexpr int VEC = 16 / sizeof(T);              // elements per 16-byte load
    constexpr int PER_ROW = G / VEC;
    for (int v = threadIdx.x; v < 16 * PER_ROW; v += kFmtThreads) {
        const int r = v / PER_ROW, c = (v % PER_ROW) * VEC;
        const uint4 raw = __ldg(reinterpret_cast<const uint4*>(W + (size_t)(n0 + r) * K + k0 + c));
        const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
        for (int j = 0; j < VEC; ++j) tile[r][c + j] = to_f32<T>(e[j]);
    }
    __syncthreads();
    // per-row absmax: warp w handles rows 4w..4w+3
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
#pragma unroll
    for (int rr = 0; rr < 4; ++rr) {
        const int r = warp * 4 + rr;
        float m = 0.f;
        for (int c = lane; c < G; c += 32) m = fmaxf(m, fabsf(tile[r][c]));
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        if (lane == 0) {
            const __half sh = __float2half_rn(fmaxf(__fdiv_rn(m, 7.0f), 1e-4f));
            srow[r] = __half2float(sh);
            scales[(size_t)gi * N + n0 + r] = sh;
        }
    }
    __syncthreads();
    for (int e = threadIdx.x; e < 16 * G; e += kFmtThreads) {
        const int r = e / G, c = e % G;
        const float qf = fminf(fmaxf(rintf(__fdiv_rn(tile[r][c], srow[r])), -8.f), 7.f);
        codes[e] = (uint8_t)((int)qf + 8);
    }
    __syncthreads();
    if (PACK) {
        const int KC = K >> 6;
        for (int w = threadIdx.x; w < 2 * G; w += kFmtThreads) {   // 16 x G codes = 2G words
            const int kcl = w >> 7, lane_ = (w >> 2) & 31, s = w & 3;
            wp[((size_t)(nb * KC + gi * (G / 64) + kcl) * 32 + lane_) * 4 + s] =
                pack_word_from_tile(codes + kcl * 64, G, lane_, s);
        }
    } else {
        constexpr int QV = G / 16;                   // uint4 per row of codes
        for (int v = threadIdx.x; v < 16 * QV; v += kFmtThreads) {
            const int r = v / QV, c = (v % QV) * 16;
            *reinterpret_cast<uint4*>(q + (size_t)(n0 + r) * K + k0 + c) = *reinterpret_cast<const uint4*>(codes + r * G + c);
        }
    }
}

// The GEMM's decode kernel is launched with programmatic dependent launch and fetches
// packed words and scales before griddepcontrol.wait, so it may start while the kernel
// launched just before it is still finishing.  An empty kernel, launched without that
// attribute, after every format kernel makes the weights complete before a GEMM that
// follows can start.
__global__ void format_fence_kernel() {}

static cudaError_t fence_after(cudaStream_t stream) {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    format_fence_kernel<<<1, 32, 0, stream>>>();
    return cudaGetLastError();
}

// ------------------------------------------------------------------ host side
cudaError_t launch_pack(const void* q, void* wp, int N, int K, cudaStream_t stream) {
    pack_kernel<<<dim3(K / 64, N / 16), kFmtThreads, 0, stream>>>(static_cast<const uint8_t*>(q),
                                                                    static_cast<uint32_t*>(wp), N, K);
    return fence_after(stream);
}

template <typename T, bool PACK>
static cudaError_t launch_quantize_t(const void* W, void* q, void* wp, void* scales, int N, int K, int G,
                                     cudaStream_t stream) {
    const dim3 grid(K / G, N / 16);
    const T* w = static_cast<const T*>(W);
    if (G == 64)
        quantize_kernel<T, 64, PACK><<<grid, kFmtThreads, 0, stream>>>(w, static_cast<uint8_t*>(q),
            static_cast<uint32_t*>(wp), static_cast<__half*>(scales), N, K);
    else
        quantize_kernel<T, 128, PACK><<<grid, kFmtThreads, 0, stream>>>(w, static_cast<uint8_t*>(q),
            static_cast<uint32_t*>(wp), static_cast<__half*>(scales), N, K);
    return fence_after(stream);
}

cudaError_t launch_quantize(const void* W, bool w_f16, void* q, void* wp, void* scales, int N, int K, int G,
                            cudaStream_t stream) {
    const bool pack = wp != nullptr;
    if (w_f16) return pack ? launch_quantize_t<__half, true>(W, q, wp, scales, N, K, G, stream)
                           : launch_quantize_t<__half, false>(W, q, wp, scales, N, K, G, stream);
    return pack ? launch_quantize_t<float, true>(W, q, wp, scales, N, K, G, stream)
                : launch_quantize_t<float, false>(W, q, wp, scales, N, K, G, stream);
}

}  // namespace w4a16
