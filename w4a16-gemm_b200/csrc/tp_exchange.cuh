// Tensor-parallel exchange over peer memory: the reduction of row-parallel partial sums
// and the gather of column-parallel outputs, done by one small kernel per rank that
// loads and stores the other ranks' exchange buffers directly (mapped with CUDA IPC,
// reached over NVLink).  Included by the single device-code translation unit only.
//
// Buffer layout (every rank's buffer alike): the first W4A16_TP_CTRL_BYTES hold
//   ready[src]            u32, written by rank src into every buffer: "my data for call e is
//                         in place and I am ready to receive call e's results"
//   done[src][cta]        u32, written by CTA cta of rank src into every buffer: "my part of
//                         call e's results is in your buffer"
//   epoch[cta]            u32, this rank's own count of calls, per CTA (every call launches
//                         the same kTpCtas CTAs, of whatever size, so all epochs agree)
// and the caller's data regions follow.  Call e of an exchange (e = epoch + 1, the same on
// every rank: all ranks issue the same exchanges in the same order):
//   A. every CTA writes ready[rank] = e into every buffer, then waits until its own buffer
//      shows ready[src] >= e for every src;
//   B. reduce: the rank owns columns [rank*N/world, (rank+1)*N/world); its CTAs load those
//      columns of every rank's fp32 partial, add them in rank order, and store the fp16 sums
//      into every rank's y.  gather: its CTAs store their own columns into every rank's y;
//   C. every CTA writes done[rank][cta] = e into every buffer (release, after its stores),
//      then waits until its own buffer shows done[src][cta] >= e for every src -- CTA cta of
//      each rank wrote the same share of that rank's columns -- and stores epoch = e.
// Comparing with >= makes a flag that a faster rank already moved to e + 1 still count;
// no flag is ever reset, so CUDA-graph replays keep working.  A rank cannot overwrite a
// peer's y (or read its partial) for call e + 1 before that peer has finished call e: it
// needs the peer's ready flag for e + 1, which the peer writes only once its stream has
// moved past call e.  Every wait is bounded (kWaitLimitNs); a peer that never arrives sets
// the device status to kDevTimeoutPeer and the kernel returns.
#pragma once
#include <cuda_fp16.h>
#include <stdint.h>

#include "../../include/w4a16.h"
#include "internal.h"
#include "ptx.cuh"

namespace w4a16 {

constexpr int kTpMaxRanks = W4A16_TP_MAX_RANKS;
// Every exchange launches the same kTpCtas CTAs, whatever its size, so that each CTA's
// epoch counts every call and the ranks' epochs stay equal.
constexpr int kTpCtas = 64;
constexpr int kTpMaxCtas = kTpCtas;
constexpr int kTpThreads = 256;
constexpr uint32_t kTpReadyOff = 0;
constexpr uint32_t kTpDoneOff = 1024;
constexpr uint32_t kTpEpochOff = kTpDoneOff + kTpMaxRanks * kTpMaxCtas * 4;
static_assert(kTpEpochOff + kTpMaxCtas * 4 <= W4A16_TP_CTRL_BYTES, "exchange flags fit the control region");

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" :: "l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ float4 ld_relaxed_sys_f4(const float4* p) {
    float4 v;
    asm volatile("ld.relaxed.sys.global.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void fence_acq_rel_sys() {
    asm volatile("fence.acq_rel.sys;" ::: "memory");
}

// Bounded wait until *p >= e (as a difference, so the epoch may wrap).
__device__ __forceinline__ bool wait_at_least(const uint32_t* p, uint32_t e) {
    if ((int32_t)(ld_acquire_sys(p) - e) >= 0) return true;
    const uint64_t t0 = globaltimer_ns();
    while (true) {
        __nanosleep(32);
        if ((int32_t)(ld_acquire_sys(p) - e) >= 0) return true;
        if (globaltimer_ns() - t0 > kWaitLimitNs) {
            record_device_error(kDevTimeoutPeer);
            return false;
        }
    }
}

// GATHER = false: row-parallel reduction (src_off: fp32 partial [M, N] in every buffer).
// GATHER = true: column-parallel gather (src_off: fp16 [M, N/world] in every buffer).
// Either way every buffer receives fp16 y [M, N] at y_off.
template <bool GATHER>
__global__ void __launch_bounds__(kTpThreads) tp_exchange_kernel(TpPtrs P, int rank, int world, uint64_t src_off,
                                                                 uint64_t y_off, int M, int N) {
    __shared__ uint32_t s_e;
    __shared__ int s_ok;
    const int cta = blockIdx.x, tid = threadIdx.x;
    char* const own = P.buf[rank];
    uint32_t* const epoch = reinterpret_cast<uint32_t*>(own + kTpEpochOff) + cta;
    if (tid == 0) {
        s_e = *epoch + 1u;
        s_ok = 1;
    }
    __syncthreads();
    const uint32_t e = s_e;

    // A. ready: this rank's data is in place and its y may be written
    if (tid < world) st_release_sys(reinterpret_cast<uint32_t*>(P.buf[tid] + kTpReadyOff) + rank, e);
    if (tid < world && !wait_at_least(reinterpret_cast<const uint32_t*>(own + kTpReadyOff) + tid, e)) s_ok = 0;
    __syncthreads();
    if (!s_ok) return;

    // B. this CTA's share of this rank's columns, 4 at a time
    const int nl = N / world, q = nl / 4;                          // columns per rank, float4 units per row
    const long long units = (long long)M * q;
    const long long u0 = units * cta / gridDim.x, u1 = units * (cta + 1) / gridDim.x;
    for (long long u = u0 + tid; u < u1; u += kTpThreads) {
        const int m = (int)(u / q), c4 = (int)(u % q) * 4;
        uint2 h;
        if (!GATHER) {
            const size_t at = (size_t)m * N + (size_t)rank * nl + c4;   // element index of the 4 columns
            float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
            for (int src = 0; src < world; ++src) {                       // rank order
                const float4 v = ld_relaxed_sys_f4(reinterpret_cast<const float4*>(P.buf[src] + src_off) + at / 4);
                s.x += v.x;
                s.y += v.y;
                s.z += v.z;
                s.w += v.w;
            }
            const __half2 lo = __floats2half2_rn(s.x, s.y), hi = __floats2half2_rn(s.z, s.w);
            h = make_uint2(*reinterpret_cast<const uint32_t*>(&lo), *reinterpret_cast<const uint32_t*>(&hi));
            for (int t = 0; t < world; ++t) *reinterpret_cast<uint2*>(P.buf[t] + y_off + at * 2) = h;
        } else {
            h = *reinterpret_cast<const uint2*>(own + src_off + ((size_t)m * nl + c4) * 2);
            const size_t at = (size_t)m * N + (size_t)rank * nl + c4;
            for (int t = 0; t < world; ++t) *reinterpret_cast<uint2*>(P.buf[t] + y_off + at * 2) = h;
        }
    }
    __syncthreads();

    // C. done: this CTA's stores are in every buffer; wait for CTA cta of every rank
    if (tid < world) {
        fence_acq_rel_sys();   // the CTA's stores (ordered before by the barrier) before the flag
        st_release_sys(reinterpret_cast<uint32_t*>(P.buf[tid] + kTpDoneOff) + rank * kTpMaxCtas + cta, e);
    }
    if (tid < world && !wait_at_least(reinterpret_cast<const uint32_t*>(own + kTpDoneOff) + tid * kTpMaxCtas + cta, e))
        s_ok = 0;
    __syncthreads();
    if (tid == 0 && s_ok) *epoch = e;
}

cudaError_t launch_tp_exchange(bool gather, const TpPtrs& p, int rank, int world, uint64_t src_off, uint64_t y_off,
                               int M, int N, cudaStream_t stream) {
    const int b = kTpCtas;
    if (gather) tp_exchange_kernel<true><<<b, kTpThreads, 0, stream>>>(p, rank, world, src_off, y_off, M, N);
    else tp_exchange_kernel<false><<<b, kTpThreads, 0, stream>>>(p, rank, world, src_off, y_off, M, N);
    return cudaGetLastError();
}

}  // namespace w4a16
