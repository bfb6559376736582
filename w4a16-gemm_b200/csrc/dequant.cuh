// Exact int4 -> fp16 dequantisation of one packed 32-bit word.
//
// Semantics (reference: tests/quant.py:77-80, src/vectorized/common.cuh:45-55):
//     w = fp16( (q - 8) * scale )   -- q - 8 is exact in fp16, one rounding in the multiply.
//
// A word holds 8 nibbles.  Pair p (p = 0..3) is nibble p (bits 4p..4p+3) and
// nibble p+4 (bits 4p+16..4p+19); it becomes one half2 = the m16n8k16
// A-fragment register a[p]: row n = g + 8*(p&1), columns k = 2t + 8*(p>>1) + {0,1}.
// Pairs 0 and 2 belong to row g (scale s_lo), pairs 1 and 3 to row g+8 (s_hi).
//
// The (q - 8) values are formed with fp16 "magic number" bit tricks:
//   * a nibble in mantissa bits 0..3 under exponent 2^10:  0x6400|nib = 1024+nib, minus 1032
//   * a nibble in mantissa bits 4..7 under exponent 2^6 :  0x5400|nib<<4 = 64+nib, minus 72
// The second form reads pair 1 (and pair 3 after one 8-bit shift) in place,
// so a word costs 1 shift + 4 LOP3 + 4 HSUB2 + 4 HMUL2 = 13 instructions while
// every value stays bit-identical to the reference dequantisation.
#pragma once
#include <cuda_fp16.h>
#include <stdint.h>

namespace w4a16 {

__device__ __forceinline__ uint32_t and_or(uint32_t a, uint32_t mask, uint32_t bits) {
    uint32_t d;
    // (a & mask) | bits  -- LUT 0xEA = (0xF0 & 0xCC) | 0xAA
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(a), "r"(mask), "r"(bits));
    return d;
}

__device__ __forceinline__ uint32_t hsub2_u32(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}

__device__ __forceinline__ uint32_t hmul2_u32(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}

// s_lo / s_hi: the row-g / row-(g+8) scale broadcast into both halves.
__device__ __forceinline__ void dequant_word(uint32_t q, uint32_t s_lo, uint32_t s_hi, uint32_t (&a)[4]) {
    constexpr uint32_t kLoMask = 0x000F000Fu, kLoMagic = 0x64006400u, kLoBias = 0x64086408u;  // 1024, 1032
    constexpr uint32_t kHiMask = 0x00F000F0u, kHiMagic = 0x54005400u, kHiBias = 0x54805480u;  // 64, 72
    const uint32_t q8 = q >> 8;
    a[0] = hmul2_u32(hsub2_u32(and_or(q,  kLoMask, kLoMagic), kLoBias), s_lo);
    a[1] = hmul2_u32(hsub2_u32(and_or(q,  kHiMask, kHiMagic), kHiBias), s_hi);
    a[2] = hmul2_u32(hsub2_u32(and_or(q8, kLoMask, kLoMagic), kLoBias), s_lo);
    a[3] = hmul2_u32(hsub2_u32(and_or(q8, kHiMask, kHiMagic), kHiBias), s_hi);
}

// The same word as four half2 registers of the exact integers q - 8 (no scale): the decode
// path multiplies by the scale after the tensor-core product, in fp32 (see decode.cuh).
__device__ __forceinline__ void unscaled_word(uint32_t q, uint32_t (&a)[4]) {
    constexpr uint32_t kLoMask = 0x000F000Fu, kLoMagic = 0x64006400u, kLoBias = 0x64086408u;  // 1024, 1032
    constexpr uint32_t kHiMask = 0x00F000F0u, kHiMagic = 0x54005400u, kHiBias = 0x54805480u;  // 64, 72
    const uint32_t q8 = q >> 8;
    a[0] = hsub2_u32(and_or(q,  kLoMask, kLoMagic), kLoBias);
    a[1] = hsub2_u32(and_or(q,  kHiMask, kHiMagic), kHiBias);
    a[2] = hsub2_u32(and_or(q8, kLoMask, kLoMagic), kLoBias);
    a[3] = hsub2_u32(and_or(q8, kHiMask, kHiMagic), kHiBias);
}

// Broadcast an fp16 bit pattern into both halves of a half2.
__device__ __forceinline__ uint32_t bcast_half(uint16_t h) {
    return (uint32_t)h | ((uint32_t)h << 16);
}

}  // namespace w4a16
