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
//   epoch, count          u32 each: this rank's own count of calls, advanced by the last
//                         CTA of each call to finish (tp_count_out), and how many CTAs of
//                         the current call have finished
// and the caller's data regions follow (source, result and, optionally, a receive area of
// 2 * world slots used by the one-round form, tp_push_kernel, below).  A call launches
// kTpCtasSmall or kTpCtasLarge CTAs, chosen from its size alone, so every rank launches the
// same grid for the same call.  Call e of an exchange (e = epoch + 1, the same on every
// rank: all ranks issue the same exchanges in the same order, and every call of either form
// advances the epoch once), two-round form:
//   A. every CTA writes ready[rank] = e into every buffer (after a system-scope fence), then
//      waits until its own buffer shows ready[src] >= e for every src;
//   B. reduce: the rank owns columns [rank*N/world, (rank+1)*N/world); its CTAs load those
//      columns of every rank's fp32 partial, add them in rank order, and store the fp16 sums
//      into every rank's y.  gather: its CTAs store their own columns into every rank's y;
//   C. every CTA writes done[rank][cta] = e into every buffer (release, after its stores),
//      then waits until its own buffer shows done[src][cta] >= e for every src -- CTA cta of
//      each rank wrote the same share of that rank's columns -- and counts itself out.
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
// CTAs per call.  Decode-size exchanges are bound by the flag rounds, which more CTAs only
// lengthen; prefill-size ones by how much peer traffic each SM issues (B200, 2 GPUs, gather
// of 117 MB per rank: 315 us with 32 CTAs, 201 us with 128), so contributions of at least
// kTpLargeBytes per rank take the larger grid.
constexpr int kTpCtasSmall = 32;
constexpr int kTpCtasLarge = 128;
constexpr uint64_t kTpLargeBytes = 8ull << 20;
constexpr int kTpMaxCtas = kTpCtasLarge;
constexpr int kTpThreads = 512;
constexpr int kTpUnroll = 4;   // 8-column units a thread moves per round: their peer loads are in flight together
constexpr uint32_t kTpReadyOff = 0;
constexpr uint32_t kTpDoneOff = 1024;
constexpr uint32_t kTpEpochOff = kTpDoneOff + kTpMaxRanks * kTpMaxCtas * 4;   // epoch, then the count-out word
static_assert(kTpEpochOff + 8 <= W4A16_TP_CTRL_BYTES, "exchange flags fit the control region");

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

__device__ __forceinline__ uint4 ld_relaxed_sys_u4(const uint4* p) {
    uint4 v;
    asm volatile("ld.relaxed.sys.global.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void st_relaxed_sys(uint32_t* p, uint32_t v) {
    asm volatile("st.relaxed.sys.global.u32 [%0], %1;" :: "l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ void fence_acq_rel_sys() {
    asm volatile("fence.acq_rel.sys;" ::: "memory");
}

// Every CTA of a call counts itself out when it is done, also after a wait that ran out; the
// last one to do so advances the rank's call count (epoch[0]) and clears the count
// (epoch[1]).  A CTA reads the epoch once, at its start, before it counts out, so none can
// see the new value early; the next call reads it after griddepcontrol.wait, when this grid
// has completed.  So every CTA of a call agrees on e whatever the grid sizes of the calls.
// Thread 0 only.
__device__ __forceinline__ void tp_count_out(uint32_t* epoch, uint32_t e) {
    if (atomicAdd(epoch + 1, 1u) + 1u == gridDim.x) {
        epoch[1] = 0u;
        epoch[0] = e;
    }
}

// Bounded wait until *p >= e (as a difference, so the epoch may wrap).
__device__ __forceinline__ bool wait_at_least(const uint32_t* p, uint32_t e) {
    if ((int32_t)(ld_acquire_sys(p) - e) >= 0) return true;
    const uint64_t t0 = globaltimer_ns();
    while (true) {
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
__global__ void __launch_bounds__(kTpThreads) tp_exchange_kernel(const __grid_constant__ TpPtrs P, int rank, int world, uint64_t src_off,
                                                                 uint64_t y_off, int M, int N) {
    __shared__ uint32_t s_e;
    __shared__ int s_ok;
    const int cta = blockIdx.x, tid = threadIdx.x;
    char* const own = P.buf[rank];
    uint32_t* const epoch = reinterpret_cast<uint32_t*>(own + kTpEpochOff);
    // Launched with programmatic dependent launch: the next kernel may start early (it waits
    // for this one), and this one waits here until the GEMM that wrote the source region has
    // completed and its writes are visible.
    pdl_launch_dependents();
    pdl_wait();
    if (tid == 0) {
        s_e = *reinterpret_cast<volatile uint32_t*>(epoch) + 1u;
        s_ok = 1;
    }
    __syncthreads();
    const uint32_t e = s_e;

    // A. ready: this rank's data is in place and its y may be written (one thread; the
    // release orders the source region, written before this kernel, before the flags)
    if (tid == 0) {
        fence_acq_rel_sys();
        for (int t = 0; t < world; ++t) st_relaxed_sys(reinterpret_cast<uint32_t*>(P.buf[t] + kTpReadyOff) + rank, e);
    }
    if (tid < world && !wait_at_least(reinterpret_cast<const uint32_t*>(own + kTpReadyOff) + tid, e)) s_ok = 0;
    __syncthreads();
    if (!s_ok) {
        if (tid == 0) tp_count_out(epoch, e);
        return;
    }

    // B. this CTA's share of this rank's columns, 8 at a time (16-byte peer accesses); a thread
    // moves kTpUnroll units per round, issuing their loads together
    const int nl = N / world, q = nl / 8;                          // columns per rank, 8-column units per row
    const long long units = (long long)M * q;
    const long long u0 = units * cta / gridDim.x, u1 = units * (cta + 1) / gridDim.x;
    for (long long ub = u0 + tid; ub < u1; ub += (long long)kTpThreads * kTpUnroll) {
        size_t at[kTpUnroll];                                      // element index of a unit's 8 columns in y
        bool live[kTpUnroll];
#pragma unroll
        for (int i = 0; i < kTpUnroll; ++i) {
            const long long u = ub + (long long)i * kTpThreads;
            live[i] = u < u1;
            const int m = live[i] ? (int)(u / q) : 0, c8 = live[i] ? (int)(u % q) * 8 : 0;
            at[i] = (size_t)m * N + (size_t)rank * nl + c8;
        }
        uint4 h[kTpUnroll];
        if (!GATHER) {
            float4 a[kTpUnroll], b[kTpUnroll];
#pragma unroll
            for (int i = 0; i < kTpUnroll; ++i) a[i] = b[i] = make_float4(0.f, 0.f, 0.f, 0.f);
            for (int src = 0; src < world; ++src) {                    // rank order
                float4 v[kTpUnroll], w[kTpUnroll];
#pragma unroll
                for (int i = 0; i < kTpUnroll; ++i)
                    if (live[i]) {
                        const float4* p = reinterpret_cast<const float4*>(P.buf[src] + src_off) + at[i] / 4;
                        v[i] = ld_relaxed_sys_f4(p);
                        w[i] = ld_relaxed_sys_f4(p + 1);
                    }
#pragma unroll
                for (int i = 0; i < kTpUnroll; ++i)
                    if (live[i]) {
                        a[i].x += v[i].x; a[i].y += v[i].y; a[i].z += v[i].z; a[i].w += v[i].w;
                        b[i].x += w[i].x; b[i].y += w[i].y; b[i].z += w[i].z; b[i].w += w[i].w;
                    }
            }
#pragma unroll
            for (int i = 0; i < kTpUnroll; ++i) {
                const __half2 h0 = __floats2half2_rn(a[i].x, a[i].y), h1 = __floats2half2_rn(a[i].z, a[i].w);
                const __half2 h2 = __floats2half2_rn(b[i].x, b[i].y), h3 = __floats2half2_rn(b[i].z, b[i].w);
                h[i] = make_uint4(*reinterpret_cast<const uint32_t*>(&h0), *reinterpret_cast<const uint32_t*>(&h1),
                                  *reinterpret_cast<const uint32_t*>(&h2), *reinterpret_cast<const uint32_t*>(&h3));
            }
        } else {
#pragma unroll
            for (int i = 0; i < kTpUnroll; ++i)
                if (live[i]) {
                    const size_t col = at[i] - (size_t)rank * nl;         // m*N + c8
                    const size_t m = col / (size_t)N, c8 = col % (size_t)N;
                    h[i] = *reinterpret_cast<const uint4*>(own + src_off + (m * nl + c8) * 2);
                }
        }
#pragma unroll
        for (int i = 0; i < kTpUnroll; ++i)
            if (live[i])
                for (int t = 0; t < world; ++t) *reinterpret_cast<uint4*>(P.buf[t] + y_off + at[i] * 2) = h[i];
    }
    __syncthreads();

    // C. done: this CTA's stores are in every buffer (one thread: the fence orders the CTA's
    // stores, made visible to it by the barrier, before the flags); then wait for CTA cta of
    // every rank
    if (tid == 0) {
        fence_acq_rel_sys();
        for (int t = 0; t < world; ++t)
            st_relaxed_sys(reinterpret_cast<uint32_t*>(P.buf[t] + kTpDoneOff) + rank * kTpMaxCtas + cta, e);
    }
    if (tid < world && !wait_at_least(reinterpret_cast<const uint32_t*>(own + kTpDoneOff) + tid * kTpMaxCtas + cta, e))
        s_ok = 0;
    __syncthreads();
    if (tid == 0) tp_count_out(epoch, e);
}

// One-round form for small contributions: call e (parity e & 1) of rank r stores its
// contribution (gather: its fp16 columns [M, N/world]; reduce: its whole fp32 partial
// [M, N]) into slot (e & 1, r) of every peer's receive area, raises done[r][cta] = e in every
// peer's buffer after a system-scope fence, waits until every peer's CTA cta has done the
// same, and builds its own y from its source region and the received slots: the gather
// places each rank's columns, the reduction adds the ranks' partials in rank order.  Each
// CTA sends and then reads the same range of 16-byte units of a contribution, so CTA cta's
// flags cover exactly the units it reads.  A slot of parity p is written again two calls
// later, after the writer has seen this rank's CTA cta finish the call in between (a
// one-round call has the kTpCtasSmall CTAs that every call has), which this rank starts only
// after the call that read the slot has completed.  One fence per CTA and call (the
// two-round form needs two; each costs microseconds at system scope).
template <bool GATHER>
__global__ void __launch_bounds__(kTpThreads) tp_push_kernel(const __grid_constant__ TpPtrs P, int rank, int world,
                                                             uint64_t src_off, uint64_t y_off, uint64_t recv_off,
                                                             uint64_t slot_bytes, int M, int N) {
    __shared__ uint32_t s_e;
    __shared__ int s_ok;
    const int cta = blockIdx.x, tid = threadIdx.x;
    char* const own = P.buf[rank];
    uint32_t* const epoch = reinterpret_cast<uint32_t*>(own + kTpEpochOff);
    pdl_launch_dependents();
    pdl_wait();   // the GEMM that wrote the source region has completed
    if (tid == 0) {
        s_e = *reinterpret_cast<volatile uint32_t*>(epoch) + 1u;
        s_ok = 1;
    }
    __syncthreads();
    const uint32_t e = s_e;
    const int nl = N / world;
    const long long units = GATHER ? (long long)M * nl / 8 : (long long)M * N / 4;   // 16-byte units
    const long long u0 = units * cta / gridDim.x, u1 = units * (cta + 1) / gridDim.x;
    const uint64_t slot0 = recv_off + (uint64_t)(e & 1u) * (uint64_t)world * slot_bytes;   // this parity's slots
    const uint4* const src = reinterpret_cast<const uint4*>(own + src_off);

    // A. this CTA's units of the contribution into slot (parity, rank) of every peer
    for (long long u = u0 + tid; u < u1; u += kTpThreads) {
        const uint4 v = src[u];
        for (int t = 0; t < world; ++t)
            if (t != rank) reinterpret_cast<uint4*>(P.buf[t] + slot0 + (uint64_t)rank * slot_bytes)[u] = v;
    }
    __syncthreads();
    // B. one flag per peer, after the CTA's stores; then wait for CTA cta of every peer
    if (tid == 0) {
        fence_acq_rel_sys();
        for (int t = 0; t < world; ++t)
            if (t != rank) st_relaxed_sys(reinterpret_cast<uint32_t*>(P.buf[t] + kTpDoneOff) + rank * kTpMaxCtas + cta, e);
    }
    if (tid < world && tid != rank &&
        !wait_at_least(reinterpret_cast<const uint32_t*>(own + kTpDoneOff) + tid * kTpMaxCtas + cta, e))
        s_ok = 0;
    __syncthreads();
    if (!s_ok) {
        if (tid == 0) tp_count_out(epoch, e);
        return;
    }

    // C. this rank's y from the same units: own source region and the received slots
    for (long long u = u0 + tid; u < u1; u += kTpThreads) {
        if (GATHER) {
            const long long m = u / (nl / 8), c8 = (u % (nl / 8)) * 8;
            for (int sr = 0; sr < world; ++sr) {
                const uint4 v = sr == rank ? src[u]
                                           : ld_relaxed_sys_u4(reinterpret_cast<const uint4*>(own + slot0 +
                                                                                               (uint64_t)sr * slot_bytes) + u);
                *reinterpret_cast<uint4*>(own + y_off + ((size_t)m * N + (size_t)sr * nl + c8) * 2) = v;
            }
        } else {
            float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
            for (int sr = 0; sr < world; ++sr) {   // rank order
                const float4 v = sr == rank ? reinterpret_cast<const float4*>(src)[u]
                                            : ld_relaxed_sys_f4(reinterpret_cast<const float4*>(own + slot0 +
                                                                                                 (uint64_t)sr * slot_bytes) + u);
                a.x += v.x; a.y += v.y; a.z += v.z; a.w += v.w;
            }
            const __half2 h0 = __floats2half2_rn(a.x, a.y), h1 = __floats2half2_rn(a.z, a.w);
            *reinterpret_cast<uint2*>(own + y_off + (size_t)u * 8) =
                make_uint2(*reinterpret_cast<const uint32_t*>(&h0), *reinterpret_cast<const uint32_t*>(&h1));
        }
    }
    __syncthreads();
    if (tid == 0) tp_count_out(epoch, e);
}

cudaError_t launch_tp_exchange(bool gather, bool push, const TpPtrs& p, int rank, int world, uint64_t src_off,
                               uint64_t y_off, uint64_t recv_off, uint64_t slot_bytes, int M, int N,
                               cudaStream_t stream) {
    cudaLaunchConfig_t cfg = {};
    const uint64_t contribution = gather ? (uint64_t)M * (uint64_t)(N / world) * 2u : (uint64_t)M * (uint64_t)N * 4u;
    cfg.gridDim = dim3(!push && contribution >= kTpLargeBytes ? kTpCtasLarge : kTpCtasSmall, 1, 1);
    cfg.blockDim = dim3(kTpThreads, 1, 1);
    cfg.stream = stream;
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr.val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    if (push) {
        if (gather)
            return cudaLaunchKernelEx(&cfg, tp_push_kernel<true>, p, rank, world, src_off, y_off, recv_off, slot_bytes, M, N);
        return cudaLaunchKernelEx(&cfg, tp_push_kernel<false>, p, rank, world, src_off, y_off, recv_off, slot_bytes, M, N);
    }
    if (gather) return cudaLaunchKernelEx(&cfg, tp_exchange_kernel<true>, p, rank, world, src_off, y_off, M, N);
    return cudaLaunchKernelEx(&cfg, tp_exchange_kernel<false>, p, rank, world, src_off, y_off, M, N);
}

}  // namespace w4a16
