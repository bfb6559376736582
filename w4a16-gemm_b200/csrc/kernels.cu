// The single device-code translation unit: decode, prefill, dequant and format kernels,
// the device status word, and the host helpers they need (device properties,
// shared-memory opt-in, TMA tensor maps).
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <cmath>
#include <mutex>
#include <set>
#include <utility>

#include "internal.h"
#include "ptx.cuh"
#include "decode.cuh"
#include "prefill.cuh"
#include "dequant_kernel.cuh"
#include "format_kernels.cuh"

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
    err = cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, d.max_smem_optin);
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

cudaError_t make_prefill_tensor_maps(const GemmArgs& a, int tok, CUtensorMap* tx, CUtensorMap* tw, CUtensorMap* ts) {
    auto encode = tensor_map_encoder();
    if (!encode) return cudaErrorNotSupported;
    const cuuint32_t one[3] = {1, 1, 1};
    {   // x [M, K] fp16, box {64, tok}, 128-byte swizzle (one swizzle atom per row)
        const cuuint64_t dims[2] = {(cuuint64_t)a.K, (cuuint64_t)a.M};
        const cuuint64_t strides[1] = {(cuuint64_t)a.K * 2};
        const cuuint32_t box[2] = {64, (cuuint32_t)tok};
        if (encode(tx, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(a.x), dims, strides, box, one,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return cudaErrorInvalidValue;
    }
    {   // packed words viewed as [NB][KC][128] int32, box {128, 1, 8}
        const cuuint64_t dims[3] = {128, (cuuint64_t)(a.K / 64), (cuuint64_t)(a.N / 16)};
        const cuuint64_t strides[2] = {512, (cuuint64_t)(a.K / 64) * 512};
        const cuuint32_t box[3] = {128, 1, 8};
        if (encode(tw, CU_TENSOR_MAP_DATA_TYPE_INT32, 3, const_cast<void*>(a.wp), dims, strides, box, one,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return cudaErrorInvalidValue;
    }
    {   // scales [K/G, N] fp16, box {128, 1}
        const cuuint64_t dims[2] = {(cuuint64_t)a.N, (cuuint64_t)(a.K / a.G)};
        const cuuint64_t strides[1] = {(cuuint64_t)a.N * 2};
        const cuuint32_t box[2] = {128, 1};
        if (encode(ts, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(a.scales), dims, strides, box, one,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return cudaErrorInvalidValue;
    }
    return cudaSuccess;
}

cudaError_t make_decode_tensor_maps(const GemmArgs& a, int box_blocks, int box_chunks, int mp, CUtensorMap* tw,
                                    CUtensorMap* tx, CUtensorMap* ts) {
    auto encode = tensor_map_encoder();
    if (!encode) return cudaErrorNotSupported;
    const cuuint32_t one[3] = {1, 1, 1};
    {   // packed words [NB][KC][128] int32, box {128, box_chunks, box_blocks}: per n16 block one
        // contiguous run of box_chunks * 512 bytes
        const cuuint64_t dims[3] = {128, (cuuint64_t)(a.K / 64), (cuuint64_t)(a.N / 16)};
        const cuuint64_t strides[2] = {512, (cuuint64_t)(a.K / 64) * 512};
        const cuuint32_t box[3] = {128, (cuuint32_t)box_chunks, (cuuint32_t)box_blocks};
        if (encode(tw, CU_TENSOR_MAP_DATA_TYPE_INT32, 3, const_cast<void*>(a.wp), dims, strides, box, one,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return cudaErrorInvalidValue;
    }
    {   // x [M, K] fp16 viewed as [K/64][M][64], box {64, mp, box_chunks} (rows >= M and chunks
        // past K read as zeros), 128-byte swizzle
        const cuuint64_t dims[3] = {64, (cuuint64_t)a.M, (cuuint64_t)(a.K / 64)};
        const cuuint64_t strides[2] = {(cuuint64_t)a.K * 2, 128};
        const cuuint32_t box[3] = {64, (cuuint32_t)mp, (cuuint32_t)box_chunks};
        if (encode(tx, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void*>(a.x), dims, strides, box, one,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return cudaErrorInvalidValue;
    }
    {   // scales [K/G, N] fp16, box {16 * box_blocks, 1}
        const cuuint64_t dims[2] = {(cuuint64_t)a.N, (cuuint64_t)(a.K / a.G)};
        const cuuint64_t strides[1] = {(cuuint64_t)a.N * 2};
        const cuuint32_t box[2] = {(cuuint32_t)(16 * box_blocks), 1};
        if (encode(ts, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(a.scales), dims, strides, box, one,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return cudaErrorInvalidValue;
    }
    return cudaSuccess;
}

// ---------------------------------------------------------------- built-in scratch (w4a16_gemm_noalloc)
// Scratch for callers that are not allowed to allocate device memory themselves:
// e.g. a host integration whose device memory budget is fixed at start-up, or a
// foreign-language binding with no device allocator to hand a workspace from.
// The decode path's split-group partials then live in this array, which the
// module loader reserves on every device alongside the kernels; nothing is
// allocated per call.  The kernels write every byte of it they read, so its
// contents never need to start at zero.  All calls on one device share it.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

cudaError_t noalloc_scratch(void** ptr, size_t* bytes) {
    int dev = 0;
    cudaError_t err = cudaGetDevice(&dev);
    if (err != cudaSuccess) return err;
    if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
    static std::mutex mu;
    static void* addr[kMaxDevices] = {};
    std::lock_guard<std::mutex> lk(mu);
    if (!addr[dev]) {
        // one-time set-up for this device (with it current): the array's device address
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
