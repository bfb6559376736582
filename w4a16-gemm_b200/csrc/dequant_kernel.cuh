// Debug / verification kernel: materialise the dequantised weight matrix.
// Included by the single device-code translation unit (kernels.cu) only.
// out[n, k] = fp16((q[n, k] - 8) * scales[k / G, n]) -- the same per-word
// dequant the GEMM kernels use, so it must equal the reference's
// dequantize_w4 (tests/quant.py:77-80) bit for bit.
#pragma once
#include <cuda_fp16.h>
#include <stdint.h>

#include <algorithm>

#include "dequant.cuh"

namespace w4a16 {

template <int G>
__global__ void __launch_bounds__(256) dequant_kernel(const uint4* __restrict__ wp, const uint16_t* __restrict__ scales,
                                                      uint32_t* __restrict__ out, int N, int K) {
    const int KC = K >> 6;
    const long long total = (long long)(N >> 4) * KC * 32;     // one uint4 (4 words) per thread
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        const int lane = (int)(i & 31);
        const long long chunk = i >> 5;
        const int kc = (int)(chunk % KC);
        const int nb = (int)(chunk / KC);
        const int g = lane >> 2, t = lane & 3;
        const uint4 w = wp[i];
        const int grp = (kc * 64) / G;
        const uint32_t s_lo = bcast_half(scales[(size_t)grp * N + nb * 16 + g]);
        const uint32_t s_hi = bcast_half(scales[(size_t)grp * N + nb * 16 + g + 8]);
        const uint32_t wq[4] = {w.x, w.y, w.z, w.w};
        const size_t row0 = (size_t)(nb * 16 + g) * K, row1 = row0 + (size_t)8 * K;
#pragma unroll
        for (int s = 0; s < 4; ++s) {
            uint32_t a[4];
            dequant_word(wq[s], s_lo, s_hi, a);
            const int k0 = kc * 64 + 16 * s + 2 * t;     // even: half2-aligned
            out[(row0 + k0) >> 1] = a[0];
            out[(row1 + k0) >> 1] = a[1];
            out[(row0 + k0 + 8) >> 1] = a[2];
            out[(row1 + k0 + 8) >> 1] = a[3];
        }
    }
}

cudaError_t launch_dequant(const void* wp, const void* scales, void* out, int N, int K, int G,
                                  cudaStream_t stream) {
    const long long total = (long long)(N >> 4) * (K >> 6) * 32;
    const int blocks = (int)std::min<long long>((total + 255) / 256, 148LL * 16);
    if (G == 64)
        dequant_kernel<64><<<blocks, 256, 0, stream>>>(static_cast<const uint4*>(wp), static_cast<const uint16_t*>(scales),
                                                       static_cast<uint32_t*>(out), N, K);
    else
        dequant_kernel<128><<<blocks, 256, 0, stream>>>(static_cast<const uint4*>(wp), static_cast<const uint16_t*>(scales),
                                                        static_cast<uint32_t*>(out), N, K);
    return cudaGetLastError();
}

}  // namespace w4a16
