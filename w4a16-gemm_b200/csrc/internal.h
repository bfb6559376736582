// Host-side interfaces shared by the C-ABI launcher and the kernel translation units.
#pragma once
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "../../include/w4a16.h"

namespace w4a16 {

// One validated GEMM call: y[M, N] = x[M, K] @ W^T, W from packed nibbles + fp16 scales.
struct GemmArgs {
    const void* wp;       // int32 [N*K/8] packed nibbles (fragment order)
    const void* x;        // fp16 [M, K]
    const void* scales;   // fp16 [K/G, N]
    void* y;              // fp16 or fp32 [M, N]
    int M, N, K, G;
    bool out_f32;         // fp32 output (tensor-parallel partials) instead of fp16
    cudaStream_t stream;
    bool pdl;             // launch with programmatic dependent launch enabled
    bool weights_resident;// wp/scales are not written by the kernel launched just before:
                          // the decode producer may fetch them before griddepcontrol.wait
    bool fp32_scale;      // decode, M <= 8: scales applied in fp32 after the MMA (W4A16_FLAG_FP32_SCALE)
    void* workspace;      // decode scratch (split-group partials); no initial contents needed
    size_t workspace_bytes;
};

struct DeviceInfo {
    int device;
    int num_sms;
    int max_smem_optin;
    int cc_major, cc_minor;
};

// Cached properties of the current device (thread-safe).
cudaError_t device_info(DeviceInfo* out);

// Raise a kernel's dynamic shared-memory cap to the device opt-in maximum, once
// per (kernel, device) (thread-safe).
cudaError_t ensure_max_dynamic_smem(const void* func);


// Read (and optionally clear) the device status word that bounded waits set on
// timeout.  Synchronises with the device.
cudaError_t read_device_status(int* code, bool reset);
// Launches one kernel whose bounded mbarrier wait runs out (about kWaitLimitNs) and waits
// for it; the wait records `code` in the device status word.
cudaError_t run_wait_limit_check(bool sleeping, int code);

// Built-in scratch of w4a16_gemm_noalloc: a device array of kNoAllocScratchBytes
// compiled into the library.  Returns its address on the current device (looked up
// on every call outside stream capture; under capture, the last address found).
constexpr size_t kNoAllocScratchBytes = W4A16_NOALLOC_SCRATCH_BYTES;
constexpr int kMaxDevices = 64;
cudaError_t noalloc_scratch(void** ptr, size_t* bytes, cudaStream_t stream);

// ---------------------------------------------------------------- decode (M <= 16)
struct DecodePlan {
    int mt;           // 8-token tiles (1: M <= 8, 2: M <= 16)
    int ctas;         // persistent CTAs (one per SM)
    int units;        // stream-K work units (256 columns x one 64-wide K chunk each)
    int stages;       // TMA ring depth
    size_t smem;      // dynamic shared memory bytes
    size_t workspace; // bytes of workspace the launch needs
    int launches;     // kernels launched: 1, or 2 when a group is split (combine kernel)
    bool valid;
};
DecodePlan plan_decode(int M, int N, int K, int G, const DeviceInfo& dev);
cudaError_t launch_decode(const GemmArgs& a, const DecodePlan& p);
size_t decode_workspace_bytes(int N, int K, const DeviceInfo& dev);

// ---------------------------------------------------------------- prefill (any M)
struct PrefillPlan {
    int config;     // 1..4
    int tok;        // token tile (UMMA N): 32, 64, 128 or 256
    int stages;     // shared-memory pipeline depth
    int a_stages;   // TMEM A-operand ring depth
    int accs;       // TMEM accumulator buffers
    int tiles;      // total output tiles
    int grid;       // persistent CTAs
    size_t smem;
};
// config 1..4 forces a token tile (32 / 64 / 128 / 256); 0 = choose from the shape.
PrefillPlan plan_prefill(int M, int N, int K, int G, int config, const DeviceInfo& dev);
cudaError_t launch_prefill(const GemmArgs& a, const PrefillPlan& p);

// ---------------------------------------------------------------- load-time format kernels
// codes uint8 [N, K] -> packed words (N % 16 == 0, K % 64 == 0, 16-byte aligned pointers).
cudaError_t launch_pack(const void* q, void* wp, int N, int K, cudaStream_t stream);
// W [N, K] fp32 (or fp16 when w_f16) -> scales fp16 [K/G, N] and codes uint8 [N, K] (wp ==
// nullptr) or packed words (q == nullptr).
cudaError_t launch_quantize(const void* W, bool w_f16, void* q, void* wp, void* scales, int N, int K, int G,
                            cudaStream_t stream);

// ---------------------------------------------------------------- tensor-parallel exchange
struct TpPtrs {
    char* buf[W4A16_TP_MAX_RANKS];   // every rank's exchange buffer as mapped in this process
};
constexpr size_t kTpCtrlBytes = W4A16_TP_CTRL_BYTES;
// push: the one-round protocol through receive slots of slot_bytes at recv_off (2 * world
// slots per buffer); otherwise the two-round pull from the peers' source regions.
cudaError_t launch_tp_exchange(bool gather, bool push, const TpPtrs& p, int rank, int world, uint64_t src_off,
                               uint64_t y_off, uint64_t recv_off, uint64_t slot_bytes, int M, int N,
                               cudaStream_t stream);

// ---------------------------------------------------------------- debug dequant
cudaError_t launch_dequant(const void* wp, const void* scales, void* out, int N, int K, int G,
                           cudaStream_t stream);

}  // namespace w4a16
