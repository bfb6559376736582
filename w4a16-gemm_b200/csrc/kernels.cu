// The single device-code translation unit: decode, prefill, dequant and format kernels,
// the device status word, and the host helpers they need (device properties,
// shared-memory opt-in, TMA tensor maps).
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <cmath>
#include <cstring>
#include <mutex>
#include <set>
#include <utility>

#include "internal.h"
#include "ptx.cuh"
#include "decode.cuh"
#include "prefill.cuh"
#include "dequant_kernel.cuh"
#include "format_kernels.cuh"
#include "tp_exchange.cuh"

namespace w4a16 {

cudaError_t device_info(DeviceInfo* out) {
    static std::mutex mu;
    static DeviceInfo cache[64];
    static bool have[64] = {};
    int dev = 0;
    cudaError_t err = cudaGetDevice(&dev);
    if (err != cudaSuccess) return err;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> lk(mu);
    if (!have[dev]) {
        DeviceInfo d;
        d.device = dev;
        if ((err = cudaDeviceGetAttribute(&d.num_sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess) return err;
        if ((err = cudaDeviceGetAttribute(&d.max_smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev)) != cudaSuccess) return err;
        if ((err = cudaDeviceGetAttribute(&d.cc_major, cudaDevAttrComputeCapabilityMajor, dev)) != cudaSuccess) return err;
        if ((err = cudaDeviceGetAttribute(&d.cc_minor, cudaDevAttrComputeCapabilityMinor, dev)) != cudaSuccess) return err;
        cache[dev] = d;
        have[dev] = true;
    }
    *out = cache[dev];
    return cudaSuccess;
}

cudaError_t ensure_max_dynamic_smem(const void* func) {
    static std::mutex mu;
    static std::set<std::pair<const void*, int>> done;
    DeviceInfo d;
    cudaError_t err = device_info(&d);
    if (err != cudaSuccess) return err;
    std::lock_guard<std::mutex> lk(mu);
    if (done.count({func, d.device})) return cudaSuccess;
    // the opt-in maximum covers static and dynamic shared memory together
    cudaFuncAttributes fa;
    if ((err = cudaFuncGetAttributes(&fa, func)) != cudaSuccess) return err;
    err = cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               d.max_smem_optin - (int)fa.sharedSizeBytes);
    // all of the unified L1/shared array as shared memory (the kernels stage through it)
    if (err == cudaSuccess)
        err = cudaFuncSetAttribute(func, cudaFuncAttributePreferredSharedMemoryCarveout, cudaSharedmemCarveoutMaxShared);
    if (err == cudaSuccess) done.insert({func, d.device});
    return err;
}

cudaError_t read_device_status(int* code, bool reset) {
    cudaError_t err = cudaDeviceSynchronize();
    if (err != cudaSuccess) return err;
    err = cudaMemcpyFromSymbol(code, w4a16_device_status, sizeof(int));
    if (err != cudaSuccess || !reset) return err;
    const int zero = 0;
    return cudaMemcpyToSymbol(w4a16_device_status, &zero, sizeof(int));
}

// One thread waits for phase 0 of an mbarrier that nothing arrives at, with the wait the
// GEMM kernels use (busy polls, or polls that sleep between tries): after the wait limit it
// records `code` in the device status word and returns.
__global__ void wait_limit_kernel(int sleeping, int code) {
    __shared__ __align__(8) uint64_t bar;
    if (threadIdx.x == 0) {
        mbar_init(smem_u32(&bar), 1);
        fence_mbar_init();
        if (sleeping) mbar_wait_sleep(smem_u32(&bar), 0, code);
        else mbar_wait(smem_u32(&bar), 0, code);
    }
}

cudaError_t run_wait_limit_check(bool sleeping, int code) {
    wait_limit_kernel<<<1, 32>>>(sleeping ? 1 : 0, code);
    const cudaError_t err = cudaGetLastError();
    return err != cudaSuccess ? err : cudaDeviceSynchronize();
}

static PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

// Everything a tiled tensor map is encoded from.  A map is a pure function of these
// fields, so a cached map is exactly what a fresh encode would return.
struct TmapKey {
    const void* ptr;
    uint64_t dims[3];
    uint64_t strides[2];   // bytes, dimensions 1.. (dimension 0 is dense)
    uint32_t box[3];
    uint32_t rank, dtype, swizzle, promo;
};

// Encodes a tiled tensor map, through a small per-thread cache keyed by every encode
// argument: a GEMM call's weight and scale maps (and, with reused activation buffers,
// its x map) are then found instead of re-encoded on every call.  Per thread, so the
// host hot path takes no lock.
static cudaError_t encode_tiled(const TmapKey& k, CUtensorMap* out) {
    struct Entry {
        TmapKey key;
        CUtensorMap map;
        bool valid;
    };
    constexpr int kEntries = 64;
    thread_local Entry cache[kEntries];
    uint64_t h = 1469598103934665603ull;   // FNV-1a over the key bytes
    const unsigned char* kb = reinterpret_cast<const unsigned char*>(&k);
    for (size_t i = 0; i < sizeof(TmapKey); ++i) h = (h ^ kb[i]) * 1099511628211ull;
    Entry& e = cache[h % kEntries];
    if (e.valid && std::memcmp(&e.key, &k, sizeof(TmapKey)) == 0) {
        *out = e.map;
        return cudaSuccess;
    }
    auto encode = tensor_map_encoder();
    if (!encode) return cudaErrorNotSupported;
    const cuuint32_t one[3] = {1, 1, 1};
    const cuuint64_t dims[3] = {k.dims[0], k.dims[1], k.dims[2]};
    const cuuint64_t strides[2] = {k.strides[0], k.strides[1]};
    const cuuint32_t box[3] = {k.box[0], k.box[1], k.box[2]};
    if (encode(out, (CUtensorMapDataType)k.dtype, k.rank, const_cast<void*>(k.ptr), dims, strides, box, one,
               CU_TENSOR_MAP_INTERLEAVE_NONE, (CUtensorMapSwizzle)k.swizzle, (CUtensorMapL2promotion)k.promo,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return cudaErrorInvalidValue;
    e.key = k;
    e.map = *out;
    e.valid = true;
    return cudaSuccess;
}

static TmapKey tmap_key(const void* ptr, uint32_t rank, CUtensorMapDataType dtype, CUtensorMapSwizzle swizzle,
                        CUtensorMapL2promotion promo) {
    TmapKey k;
    std::memset(&k, 0, sizeof k);   // padding bytes take part in the cache comparison
    k.ptr = ptr;
    k.rank = rank;
    k.dtype = (uint32_t)dtype;
    k.swizzle = (uint32_t)swizzle;
    k.promo = (uint32_t)promo;
    return k;
}

cudaError_t make_prefill_tensor_maps(const GemmArgs& a, int tok, CUtensorMap* tx, CUtensorMap* tw, CUtensorMap* ts) {
    cudaError_t err;
    {   // x [M, K] fp16, box {64, tok}, 128-byte swizzle (one swizzle atom per row)
        TmapKey k = tmap_key(a.x, 2, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, CU_TENSOR_MAP_SWIZZLE_128B,
                             CU_TENSOR_MAP_L2_PROMOTION_L2_256B);
        k.dims[0] = (uint64_t)a.K; k.dims[1] = (uint64_t)a.M;
        k.strides[0] = (uint64_t)a.K * 2;
        k.box[0] = 64; k.box[1] = (uint32_t)tok;
        if ((err = encode_tiled(k, tx)) != cudaSuccess) return err;
    }
    {   // packed words viewed as [NB][KC][128] int32, box {128, min(pf_kch(tok), KC), 8}: a stage's
        // chunks of 8 n16 blocks, each block's chunks one contiguous run
        TmapKey k = tmap_key(a.wp, 3, CU_TENSOR_MAP_DATA_TYPE_INT32, CU_TENSOR_MAP_SWIZZLE_NONE,
                             CU_TENSOR_MAP_L2_PROMOTION_L2_256B);
        k.dims[0] = 128; k.dims[1] = (uint64_t)(a.K / 64); k.dims[2] = (uint64_t)(a.N / 16);
        k.strides[0] = 512; k.strides[1] = (uint64_t)(a.K / 64) * 512;
        k.box[0] = 128; k.box[1] = (uint32_t)std::min(pf_kch(tok), a.K / 64); k.box[2] = 8;
        if ((err = encode_tiled(k, tw)) != cudaSuccess) return err;
    }
    {   // scales [K/G, N] fp16, box {128, 1}
        TmapKey k = tmap_key(a.scales, 2, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, CU_TENSOR_MAP_SWIZZLE_NONE,
                             CU_TENSOR_MAP_L2_PROMOTION_L2_256B);
        k.dims[0] = (uint64_t)a.N; k.dims[1] = (uint64_t)(a.K / a.G);
        k.strides[0] = (uint64_t)a.N * 2;
        k.box[0] = 128; k.box[1] = 1;
        if ((err = encode_tiled(k, ts)) != cudaSuccess) return err;
    }
    return cudaSuccess;
}

cudaError_t make_decode_tensor_maps(const GemmArgs& a, int box_blocks, int box_chunks, int mp, CUtensorMap* tw,
                                    CUtensorMap* tx, CUtensorMap* ts) {
    cudaError_t err;
    {   // packed words [NB][KC][128] int32, box {128, box_chunks, box_blocks}: per n16 block one
        // contiguous run of box_chunks * 512 bytes
        TmapKey k = tmap_key(a.wp, 3, CU_TENSOR_MAP_DATA_TYPE_INT32, CU_TENSOR_MAP_SWIZZLE_NONE,
                             CU_TENSOR_MAP_L2_PROMOTION_L2_256B);
        k.dims[0] = 128; k.dims[1] = (uint64_t)(a.K / 64); k.dims[2] = (uint64_t)(a.N / 16);
        k.strides[0] = 512; k.strides[1] = (uint64_t)(a.K / 64) * 512;
        k.box[0] = 128; k.box[1] = (uint32_t)box_chunks; k.box[2] = (uint32_t)box_blocks;
        if ((err = encode_tiled(k, tw)) != cudaSuccess) return err;
    }
    {   // x [M, K] fp16 viewed as [K/64][M][64], box {64, mp, box_chunks} (rows >= M and chunks
        // past K read as zeros), 128-byte swizzle
        TmapKey k = tmap_key(a.x, 3, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, CU_TENSOR_MAP_SWIZZLE_128B,
                             CU_TENSOR_MAP_L2_PROMOTION_L2_128B);
        k.dims[0] = 64; k.dims[1] = (uint64_t)a.M; k.dims[2] = (uint64_t)(a.K / 64);
        k.strides[0] = (uint64_t)a.K * 2; k.strides[1] = 128;
        k.box[0] = 64; k.box[1] = (uint32_t)mp; k.box[2] = (uint32_t)box_chunks;
        if ((err = encode_tiled(k, tx)) != cudaSuccess) return err;
    }
    {   // scales [K/G, N] fp16, box {16 * box_blocks, 1}
        TmapKey k = tmap_key(a.scales, 2, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, CU_TENSOR_MAP_SWIZZLE_NONE,
                             CU_TENSOR_MAP_L2_PROMOTION_L2_256B);
        k.dims[0] = (uint64_t)a.N; k.dims[1] = (uint64_t)(a.K / a.G);
        k.strides[0] = (uint64_t)a.N * 2;
        k.box[0] = (uint32_t)(16 * box_blocks); k.box[1] = 1;
        if ((err = encode_tiled(k, ts)) != cudaSuccess) return err;
    }
    return cudaSuccess;
}

// ---------------------------------------------------------------- built-in scratch (w4a16_gemm_noalloc)
// Scratch for callers that are not allowed to allocate device memory themselves:
// e.g. a host integration whose device memory budget is fixed at start-up, or a
// foreign-language binding with no device allocator to hand a workspace from.
// The decode path's split-group partials then live in this array, which the module
// loader reserves on every device alongside the kernels; nothing is allocated per
// call.  The kernels write every byte of it they read, so its contents never need to
// start at zero.  All calls on one device share it.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

cudaError_t noalloc_scratch(void** ptr, size_t* bytes, cudaStream_t stream) {
    int dev = 0;
    cudaError_t err = cudaGetDevice(&dev);
    if (err != cudaSuccess) return err;
    if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
    static std::mutex mu;
    static void* addr[kMaxDevices] = {};
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    if ((err = cudaStreamIsCapturing(stream, &cap)) != cudaSuccess) return err;
    std::lock_guard<std::mutex> lk(mu);
    if (!addr[dev] || cap == cudaStreamCaptureStatusNone) {
        // The array's device address on this device (with it current).  Looked up again on
        // every call made outside stream capture, so a context that was torn down and
        // re-created (cudaDeviceReset) never leaves a stale address behind; under capture
        // the address from the last call outside it is used.
        void* p = nullptr;
        err = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (err != cudaSuccess) return err;
        addr[dev] = p;
    }
    *ptr = addr[dev];
    *bytes = kNoAllocScratchBytes;
    return cudaSuccess;
}

}  // namespace w4a16
