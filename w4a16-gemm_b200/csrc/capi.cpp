// extern "C" entry points of libw4a16.so (declared in include/w4a16.h).
//
// Validation order and messages follow the reference's host entry
// w4a16_gemm_cuda (src/vectorized/kernel.cu:218-249) so callers see the same
// errors; tensor-level checks (CUDA residency, contiguity, dtypes, ranks) are
// the torch shim's job because plain pointers carry none of that.
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>

#include "../../include/w4a16.h"
#include "internal.h"

namespace {

thread_local std::string g_last_error;

w4a16_status fail(w4a16_status s, const std::string& msg) {
    g_last_error = msg;
    return s;
}

w4a16_status ok() {
    return W4A16_OK;
}

bool pdl_enabled() {
    static const bool on = [] {
        const char* v = std::getenv("W4A16_PDL");
        return !(v && (std::strcmp(v, "0") == 0 || std::strcmp(v, "off") == 0));
    }();
    return on;
}

bool decode_contract(int64_t M, int64_t N, int64_t K) {
    return M >= 1 && M <= 16 && N % 64 == 0 && K % 512 == 0;
}

w4a16_status check_device(w4a16::DeviceInfo* d) {
    cudaError_t err = w4a16::device_info(d);
    if (err != cudaSuccess) return fail(W4A16_ERR_CUDA, std::string("CUDA error: ") + cudaGetErrorString(err));
    if (d->cc_major != 10 || d->cc_minor != 0)
        return fail(W4A16_ERR_DEVICE, "w4a16 kernels are built for sm_100a (B200); current device is sm_" +
                                          std::to_string(d->cc_major) + std::to_string(d->cc_minor));
    return ok();
}

struct Route {
    bool decode;
    w4a16::DecodePlan dp;
    w4a16::PrefillPlan pp;
};

// Routing: the decode kernel serves every M <= 16 call under variant -1 (it
// handles N % 16 and K % 64 tails, unlike the reference's decode kernel, whose
// stricter contract kernel.cu:243 is still enforced for an explicit variant 0);
// everything else goes to the tcgen05 prefill kernel.
Route make_route(int M, int N, int K, int G, int variant, const w4a16::DeviceInfo& d) {
    Route r{};
    r.decode = (variant == 0) || (variant == -1 && M <= 16);
    if (r.decode) {
        r.dp = w4a16::plan_decode(M, N, K, G, d);
        // A K slice too long for shared memory even at 16 splits: the prefill
        // kernel streams K instead (same result within tolerance).
        if (!r.dp.valid) r.decode = false;
    }
    if (!r.decode) r.pp = w4a16::plan_prefill(M, N, K, G, variant > 0 ? variant : 0, d);
    return r;
}

size_t route_workspace(const Route& r) {
    return r.decode ? r.dp.workspace : 0;
}

// Route tracing on stderr, read once per process.  W4A16_DEBUG_PREFILL is the reference's
// switch (src/vectorized/kernel.cu:110-112, 199-201): one line per prefill dispatch with the
// chosen tile config and pipeline depth.  W4A16_DEBUG_ROUTE adds a line per decode call.
int debug_level() {
    static const int level = [] {
        if (std::getenv("W4A16_DEBUG_ROUTE")) return 2;
        if (std::getenv("W4A16_DEBUG_PREFILL")) return 1;
        return 0;
    }();
    return level;
}

void trace_route(const Route& r, int M, int N, int K, int G) {
    const int level = debug_level();
    if (level == 0 || (r.decode && level < 2)) return;
    if (r.decode)
        std::fprintf(stderr, "w4a16 decode G=%d M=%d N=%d K=%d ctas=%d units=%d stages=%d smem=%zu launches=%d\n", G, M,
                     N, K, r.dp.ctas, r.dp.units, r.dp.stages, r.dp.smem, r.dp.launches);
    else
        std::fprintf(stderr, "w4a16 prefill dispatch G=%d M=%d N=%d K=%d cfg=%d tok=%d grid=%d tiles=%d stages=%d smem=%zu\n",
                     G, M, N, K, r.pp.config, r.pp.tok, r.pp.grid, r.pp.tiles, r.pp.stages, r.pp.smem);
}

}  // namespace

extern "C" {

int32_t w4a16_abi_version(void) {
    return W4A16_ABI_VERSION;
}

w4a16_status w4a16_validate(const void* Wp, const void* x, const void* scales, int64_t M, int64_t N, int64_t K,
                            int64_t groups, int64_t wp_words, int32_t variant) {
    if (variant < -1 || variant > 4) return fail(W4A16_ERR_VARIANT, "variant must be -1 (auto), 0 (decode) or 1..4");
    if (M < 1) return fail(W4A16_ERR_M, "M must be at least 1");
    if (M >= (1LL << 31) || K >= (1LL << 31) || N >= (1LL << 31) || N < 0 || K < 0)
        return fail(W4A16_ERR_DIM_RANGE, "dimensions must fit in int32");
    if (K % 64 != 0) return fail(W4A16_ERR_K_MULTIPLE, "K must be a multiple of 64");
    if (N % 16 != 0) return fail(W4A16_ERR_N_MULTIPLE, "N must be a multiple of 16");
    if (groups <= 0 || K % groups != 0) return fail(W4A16_ERR_GROUPS, "K must be divisible by the number of groups");
    if (wp_words != N * K / 8) return fail(W4A16_ERR_WP_SIZE, "Wp must hold N*K/8 words");
    if ((Wp && reinterpret_cast<uintptr_t>(Wp) % 16) || (x && reinterpret_cast<uintptr_t>(x) % 16) ||
        (scales && reinterpret_cast<uintptr_t>(scales) % 16))
        return fail(W4A16_ERR_ALIGNMENT, "Wp, x and scales must be 16-byte aligned");
    const int64_t G = K / groups;
    if (G != 64 && G != 128)
        return fail(W4A16_ERR_GROUP_SIZE, "unsupported group size " + std::to_string(G) + ", supported: 64, 128");
    if (variant == 0 && !decode_contract(M, N, K))
        return fail(W4A16_ERR_DECODE_SHAPE,
                    "decode kernel needs M in [1, 16], N a multiple of 64 and K a multiple of 512 "
                    "(use variant=-1 or 1..4 for other shapes)");
    return ok();
}

w4a16_status w4a16_gemm_ex(const int32_t* Wp, const void* x, const void* scales, void* y, int64_t M, int64_t N,
                           int64_t K, int64_t groups, int64_t wp_words, int32_t variant, int32_t out_dtype,
                           uint32_t flags, void* workspace, uint64_t workspace_bytes, void* stream) {
    w4a16_status s = w4a16_validate(Wp, x, scales, M, N, K, groups, wp_words, variant);
    if (s != W4A16_OK) return s;
    if (!Wp || !x || !scales || !y) return fail(W4A16_ERR_NULL_POINTER, "Wp, x, scales and y must be non-null");
    if (out_dtype != W4A16_OUT_F16 && out_dtype != W4A16_OUT_F32)
        return fail(W4A16_ERR_OUT_DTYPE, "out_dtype must be 0 (fp16) or 1 (fp32)");
    constexpr uint32_t kKnownFlags = W4A16_FLAG_WEIGHTS_RESIDENT | W4A16_FLAG_FP32_SCALE;
    if (flags & ~kKnownFlags) return fail(W4A16_ERR_FLAGS, "unknown flag bits " + std::to_string(flags & ~kKnownFlags));
    w4a16::DeviceInfo d;
    if ((s = check_device(&d)) != W4A16_OK) return s;
    const int G = (int)(K / groups);
    w4a16::GemmArgs a{Wp, x, scales, y, (int)M, (int)N, (int)K, G, out_dtype == W4A16_OUT_F32,
                      static_cast<cudaStream_t>(stream), pdl_enabled(), (flags & W4A16_FLAG_WEIGHTS_RESIDENT) != 0,
                      (flags & W4A16_FLAG_FP32_SCALE) != 0, workspace, (size_t)workspace_bytes};
    const Route r = make_route(a.M, a.N, a.K, G, variant, d);
    const size_t need = route_workspace(r);
    if (need > 0) {
        if (!workspace) return fail(W4A16_ERR_WORKSPACE, "this call needs a workspace of " + std::to_string(need) + " bytes");
        if (workspace_bytes < need)
            return fail(W4A16_ERR_WORKSPACE, "workspace too small: " + std::to_string(workspace_bytes) + " < " +
                                                 std::to_string(need) + " bytes");
        if (reinterpret_cast<uintptr_t>(workspace) % 256) return fail(W4A16_ERR_WORKSPACE, "workspace must be 256-byte aligned");
    }
    trace_route(r, a.M, a.N, a.K, G);
    cudaError_t err = r.decode ? w4a16::launch_decode(a, r.dp) : w4a16::launch_prefill(a, r.pp);
    if (err == cudaSuccess) err = cudaGetLastError();
    if (err != cudaSuccess) return fail(W4A16_ERR_CUDA, std::string("kernel launch failed: ") + cudaGetErrorString(err));
    return ok();
}

w4a16_status w4a16_gemm(const int32_t* Wp, const void* x, const void* scales, void* y, int64_t M, int64_t N,
                        int64_t K, int64_t groups, int64_t wp_words, int32_t variant, int32_t out_dtype,
                        void* workspace, uint64_t workspace_bytes, void* stream) {
    return w4a16_gemm_ex(Wp, x, scales, y, M, N, K, groups, wp_words, variant, out_dtype, 0u, workspace,
                         workspace_bytes, stream);
}

// The GEMM with the library's built-in scratch in place of a caller workspace: the
// same validation, routing and kernels as w4a16_gemm, which it calls.
w4a16_status w4a16_gemm_noalloc(const int32_t* Wp, const void* x, const void* scales, void* y, int64_t M, int64_t N,
                                int64_t K, int64_t groups, int64_t wp_words, int32_t variant, int32_t out_dtype,
                                void* stream) {
    w4a16_status s = w4a16_validate(Wp, x, scales, M, N, K, groups, wp_words, variant);
    if (s != W4A16_OK) return s;
    uint64_t need = 0;
    if ((s = w4a16_workspace_bytes(M, N, K, groups, variant, &need)) != W4A16_OK) return s;
    if (need == 0)
        return w4a16_gemm(Wp, x, scales, y, M, N, K, groups, wp_words, variant, out_dtype, nullptr, 0, stream);
    void* scratch = nullptr;
    size_t cap = 0;
    const cudaError_t err = w4a16::noalloc_scratch(&scratch, &cap, static_cast<cudaStream_t>(stream));
    if (err != cudaSuccess) return fail(W4A16_ERR_CUDA, std::string("CUDA error: ") + cudaGetErrorString(err));
    if (need > cap)
        return fail(W4A16_ERR_WORKSPACE, "this call needs " + std::to_string(need) +
                                             " bytes of scratch; the built-in scratch holds " + std::to_string(cap) +
                                             " (use w4a16_gemm with a caller workspace)");
    return w4a16_gemm(Wp, x, scales, y, M, N, K, groups, wp_words, variant, out_dtype, scratch, cap, stream);
}

w4a16_status w4a16_query_route(int64_t M, int64_t N, int64_t K, int64_t groups, int32_t variant, w4a16_route* out) {
    w4a16_status s = w4a16_validate(nullptr, nullptr, nullptr, M, N, K, groups, N * K / 8, variant);
    if (s != W4A16_OK) return s;
    if (!out) return fail(W4A16_ERR_NULL_POINTER, "out must be non-null");
    w4a16::DeviceInfo d;
    if ((s = check_device(&d)) != W4A16_OK) return s;
    const Route r = make_route((int)M, (int)N, (int)K, (int)(K / groups), variant, d);
    std::memset(out, 0, sizeof(*out));
    out->workspace_bytes = route_workspace(r);
    if (r.decode) {
        out->kernel = 0;
        out->config = 0;
        out->tile_m = r.dp.mt * 8;
        out->tile_n = 256;
        out->split_k = r.dp.units;
        out->grid = r.dp.ctas;
        out->stages = r.dp.stages;
        out->smem_bytes = (int32_t)r.dp.smem;
        out->launches = r.dp.launches;
    } else {
        out->kernel = 1;
        out->config = r.pp.config;
        out->tile_m = r.pp.tok;
        out->tile_n = 128;
        out->split_k = 1;
        out->grid = r.pp.grid;
        out->stages = r.pp.stages;
        out->smem_bytes = (int32_t)r.pp.smem;
        out->launches = 1;
    }
    return ok();
}

w4a16_status w4a16_workspace_bytes(int64_t M, int64_t N, int64_t K, int64_t groups, int32_t variant,
                                   uint64_t* bytes) {
    w4a16_status s = w4a16_validate(nullptr, nullptr, nullptr, M, N, K, groups, N * K / 8, variant);
    if (s != W4A16_OK) return s;
    if (!bytes) return fail(W4A16_ERR_NULL_POINTER, "bytes must be non-null");
    w4a16::DeviceInfo d;
    if ((s = check_device(&d)) != W4A16_OK) return s;
    *bytes = route_workspace(make_route((int)M, (int)N, (int)K, (int)(K / groups), variant, d));
    return ok();
}

w4a16_status w4a16_dequant(const int32_t* Wp, const void* scales, void* out, int64_t N, int64_t K, int64_t groups,
                           void* stream) {
    w4a16_status s = w4a16_validate(Wp, nullptr, scales, 1, N, K, groups, N * K / 8, -1);
    if (s != W4A16_OK) return s;
    if (!Wp || !scales || !out) return fail(W4A16_ERR_NULL_POINTER, "Wp, scales and out must be non-null");
    if (reinterpret_cast<uintptr_t>(out) % 4) return fail(W4A16_ERR_ALIGNMENT, "out must be 4-byte aligned");
    w4a16::DeviceInfo d;
    if ((s = check_device(&d)) != W4A16_OK) return s;
    cudaError_t err = w4a16::launch_dequant(Wp, scales, out, (int)N, (int)K, (int)(K / groups),
                                            static_cast<cudaStream_t>(stream));
    if (err != cudaSuccess) return fail(W4A16_ERR_CUDA, std::string("kernel launch failed: ") + cudaGetErrorString(err));
    return ok();
}

namespace {

// Shape and pointer checks shared by the load-time format entries.
w4a16_status check_format(const void* a, const void* b, const void* c, int64_t N, int64_t K, int64_t G) {
    if (N < 0 || K < 0 || N >= (1LL << 31) || K >= (1LL << 31) || N * K >= (1LL << 40))
        return fail(W4A16_ERR_DIM_RANGE, "dimensions must fit in int32");
    if (K % 64 != 0) return fail(W4A16_ERR_K_MULTIPLE, "K must be a multiple of 64");
    if (N % 16 != 0) return fail(W4A16_ERR_N_MULTIPLE, "N must be a multiple of 16");
    if (G != 0) {
        if (G != 64 && G != 128)
            return fail(W4A16_ERR_GROUP_SIZE, "unsupported group size " + std::to_string(G) + ", supported: 64, 128");
        if (K % G != 0) return fail(W4A16_ERR_GROUPS, "K must be divisible by the group size");
    }
    if (!a || !b || !c) return fail(W4A16_ERR_NULL_POINTER, "pointers must be non-null");
    if (reinterpret_cast<uintptr_t>(a) % 16 || reinterpret_cast<uintptr_t>(b) % 16 || reinterpret_cast<uintptr_t>(c) % 16)
        return fail(W4A16_ERR_ALIGNMENT, "pointers must be 16-byte aligned");
    return ok();
}

}  // namespace

w4a16_status w4a16_pack(const uint8_t* q, int32_t* Wp, int64_t N, int64_t K, void* stream) {
    w4a16_status s = check_format(q, Wp, Wp, N, K, 0);
    if (s != W4A16_OK) return s;
    w4a16::DeviceInfo d;
    if ((s = check_device(&d)) != W4A16_OK) return s;
    if (N == 0 || K == 0) return ok();
    const cudaError_t err = w4a16::launch_pack(q, Wp, (int)N, (int)K, static_cast<cudaStream_t>(stream));
    if (err != cudaSuccess) return fail(W4A16_ERR_CUDA, std::string("kernel launch failed: ") + cudaGetErrorString(err));
    return ok();
}

w4a16_status w4a16_quantize(const void* W, int32_t w_dtype, uint8_t* q, void* scales, int64_t N, int64_t K,
                            int64_t group_size, void* stream) {
    if (w_dtype != W4A16_W_F32 && w_dtype != W4A16_W_F16)
        return fail(W4A16_ERR_OUT_DTYPE, "w_dtype must be 0 (fp32) or 1 (fp16)");
    w4a16_status s = check_format(W, q, scales, N, K, group_size);
    if (s != W4A16_OK) return s;
    w4a16::DeviceInfo d;
    if ((s = check_device(&d)) != W4A16_OK) return s;
    if (N == 0 || K == 0) return ok();
    const cudaError_t err = w4a16::launch_quantize(W, w_dtype == W4A16_W_F16, q, nullptr, scales, (int)N, (int)K,
                                                   (int)group_size, static_cast<cudaStream_t>(stream));
    if (err != cudaSuccess) return fail(W4A16_ERR_CUDA, std::string("kernel launch failed: ") + cudaGetErrorString(err));
    return ok();
}

w4a16_status w4a16_quantize_pack(const void* W, int32_t w_dtype, int32_t* Wp, void* scales, int64_t N, int64_t K,
                                 int64_t group_size, void* stream) {
    if (w_dtype != W4A16_W_F32 && w_dtype != W4A16_W_F16)
        return fail(W4A16_ERR_OUT_DTYPE, "w_dtype must be 0 (fp32) or 1 (fp16)");
    w4a16_status s = check_format(W, Wp, scales, N, K, group_size);
    if (s != W4A16_OK) return s;
    w4a16::DeviceInfo d;
    if ((s = check_device(&d)) != W4A16_OK) return s;
    if (N == 0 || K == 0) return ok();
    const cudaError_t err = w4a16::launch_quantize(W, w_dtype == W4A16_W_F16, nullptr, Wp, scales, (int)N, (int)K,
                                                   (int)group_size, static_cast<cudaStream_t>(stream));
    if (err != cudaSuccess) return fail(W4A16_ERR_CUDA, std::string("kernel launch failed: ") + cudaGetErrorString(err));
    return ok();
}

// ------------------------------------------------------------------ tensor-parallel exchange
w4a16_status w4a16_peer_alloc(uint64_t bytes, void** ptr, w4a16_ipc_handle* handle) {
    static_assert(sizeof(w4a16_ipc_handle) == sizeof(cudaIpcMemHandle_t), "IPC handle size");
    if (!ptr || !handle) return fail(W4A16_ERR_NULL_POINTER, "ptr and handle must be non-null");
    if (bytes < w4a16::kTpCtrlBytes)
        return fail(W4A16_ERR_TP_GROUP, "an exchange buffer holds at least W4A16_TP_CTRL_BYTES of flags");
    void* p = nullptr;
    cudaError_t err = cudaMalloc(&p, (size_t)bytes);
    if (err == cudaSuccess) err = cudaMemset(p, 0, (size_t)bytes);   // flags and epochs start at zero
    cudaIpcMemHandle_t h;
    if (err == cudaSuccess) err = cudaIpcGetMemHandle(&h, p);
    if (err == cudaSuccess) err = cudaDeviceSynchronize();
    if (err != cudaSuccess) {
        if (p) cudaFree(p);
        return fail(W4A16_ERR_CUDA, std::string("CUDA error: ") + cudaGetErrorString(err));
    }
    std::memcpy(handle->bytes, &h, sizeof(h));
    *ptr = p;
    return ok();
}

w4a16_status w4a16_peer_open(const w4a16_ipc_handle* handle, void** ptr) {
    if (!ptr || !handle) return fail(W4A16_ERR_NULL_POINTER, "ptr and handle must be non-null");
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handle->bytes, sizeof(h));
    const cudaError_t err = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
    if (err != cudaSuccess) return fail(W4A16_ERR_CUDA, std::string("CUDA error: ") + cudaGetErrorString(err));
    return ok();
}

w4a16_status w4a16_peer_close(void* ptr) {
    if (!ptr) return fail(W4A16_ERR_NULL_POINTER, "ptr must be non-null");
    const cudaError_t err = cudaIpcCloseMemHandle(ptr);
    if (err != cudaSuccess) return fail(W4A16_ERR_CUDA, std::string("CUDA error: ") + cudaGetErrorString(err));
    return ok();
}

w4a16_status w4a16_peer_free(void* ptr) {
    if (!ptr) return fail(W4A16_ERR_NULL_POINTER, "ptr must be non-null");
    const cudaError_t err = cudaFree(ptr);
    if (err != cudaSuccess) return fail(W4A16_ERR_CUDA, std::string("CUDA error: ") + cudaGetErrorString(err));
    return ok();
}

namespace {

// Checks a group and one exchange's regions: src_bytes at src_off and M*N fp16 at y_off,
// inside every buffer, past the flags, 16-byte aligned.
w4a16_status tp_check(const w4a16_tp_group* g, uint64_t src_off, uint64_t src_bytes, uint64_t y_off, int64_t M,
                      int64_t N, w4a16::TpPtrs* p) {
    if (!g) return fail(W4A16_ERR_NULL_POINTER, "group must be non-null");
    if (g->world < 1 || g->world > W4A16_TP_MAX_RANKS || g->rank < 0 || g->rank >= g->world)
        return fail(W4A16_ERR_TP_GROUP, "group needs 1 <= world <= W4A16_TP_MAX_RANKS and 0 <= rank < world");
    if (M < 1 || N < 1 || M >= (1LL << 31) || N >= (1LL << 31)) return fail(W4A16_ERR_DIM_RANGE, "dimensions must fit in int32");
    if (N % (8 * g->world)) return fail(W4A16_ERR_TP_GROUP, "N must be a multiple of 8 * world");
    const uint64_t y_bytes = (uint64_t)M * (uint64_t)N * 2;
    if (src_off % 16 || y_off % 16) return fail(W4A16_ERR_ALIGNMENT, "exchange offsets must be multiples of 16");
    if (src_off < w4a16::kTpCtrlBytes || y_off < w4a16::kTpCtrlBytes || src_off + src_bytes > g->buf_bytes ||
        y_off + y_bytes > g->buf_bytes)
        return fail(W4A16_ERR_TP_GROUP, "exchange regions must lie past the flags and inside the buffers");
    if ((src_off < y_off + y_bytes) && (y_off < src_off + src_bytes))
        return fail(W4A16_ERR_TP_GROUP, "the source and result regions must not overlap");
    if (g->recv_bytes > 0) {
        if (g->recv_off % 256) return fail(W4A16_ERR_ALIGNMENT, "the receive area must start on a 256-byte boundary");
        if (g->recv_off < w4a16::kTpCtrlBytes || g->recv_off + g->recv_bytes > g->buf_bytes)
            return fail(W4A16_ERR_TP_GROUP, "the receive area must lie past the flags and inside the buffers");
        if ((g->recv_off < y_off + y_bytes && y_off < g->recv_off + g->recv_bytes) ||
            (g->recv_off < src_off + src_bytes && src_off < g->recv_off + g->recv_bytes))
            return fail(W4A16_ERR_TP_GROUP, "the receive area must not overlap the source and result regions");
    }
    for (int r = 0; r < g->world; ++r) {
        if (!g->buf[r]) return fail(W4A16_ERR_NULL_POINTER, "every rank's buffer must be mapped");
        if (reinterpret_cast<uintptr_t>(g->buf[r]) % 256) return fail(W4A16_ERR_ALIGNMENT, "buffers must be 256-byte aligned");
        p->buf[r] = static_cast<char*>(g->buf[r]);
    }
    for (int r = g->world; r < W4A16_TP_MAX_RANKS; ++r) p->buf[r] = nullptr;
    return ok();
}

w4a16_status tp_launch(bool gather, const w4a16_tp_group* g, uint64_t src_off, uint64_t y_off, int64_t M, int64_t N,
                       void* stream) {
    w4a16::TpPtrs p;
    const uint64_t src_bytes = gather ? (uint64_t)M * (uint64_t)(N / (g ? g->world : 1)) * 2 : (uint64_t)M * (uint64_t)N * 4;
    w4a16_status s = tp_check(g, src_off, src_bytes, y_off, M, N, &p);
    if (s != W4A16_OK) return s;
    w4a16::DeviceInfo d;
    if ((s = check_device(&d)) != W4A16_OK) return s;
    // one round through the receive slots when the contribution is small and fits
    const uint64_t slot = (src_bytes + 255) / 256 * 256;
    const bool push = src_bytes <= W4A16_TP_PUSH_MAX_BYTES && g->recv_bytes >= 2ull * (uint64_t)g->world * slot;
    const cudaError_t err = w4a16::launch_tp_exchange(gather, push, p, g->rank, g->world, src_off, y_off, g->recv_off,
                                                      slot, (int)M, (int)N, static_cast<cudaStream_t>(stream));
    if (err != cudaSuccess) return fail(W4A16_ERR_CUDA, std::string("kernel launch failed: ") + cudaGetErrorString(err));
    return ok();
}

}  // namespace

w4a16_status w4a16_tp_allreduce(const w4a16_tp_group* group, uint64_t partial_off, uint64_t y_off, int64_t M,
                                int64_t N, void* stream) {
    return tp_launch(false, group, partial_off, y_off, M, N, stream);
}

w4a16_status w4a16_tp_allgather(const w4a16_tp_group* group, uint64_t src_off, uint64_t y_off, int64_t M, int64_t N,
                                void* stream) {
    return tp_launch(true, group, src_off, y_off, M, N, stream);
}

w4a16_status w4a16_device_status(int32_t* code, int32_t reset) {
    if (!code) return fail(W4A16_ERR_NULL_POINTER, "code must be non-null");
    int c = 0;
    cudaError_t err = w4a16::read_device_status(&c, reset != 0);
    if (err != cudaSuccess) return fail(W4A16_ERR_CUDA, std::string("CUDA error: ") + cudaGetErrorString(err));
    *code = c;
    if (c != 0) return fail(W4A16_ERR_DEVICE_TIMEOUT, "a kernel wait timed out (device status " + std::to_string(c) + ")");
    return ok();
}

w4a16_status w4a16_check_wait_limits(int32_t* codes) {
    if (!codes) return fail(W4A16_ERR_NULL_POINTER, "codes must be non-null");
    w4a16::DeviceInfo d;
    w4a16_status s = check_device(&d);
    if (s != W4A16_OK) return s;
    int c = 0;
    cudaError_t err = w4a16::read_device_status(&c, true);   // start from a clean status word
    const int expect[2] = {4, 1};                             // the pipeline and weight-ring codes
    for (int i = 0; i < 2 && err == cudaSuccess; ++i) {
        err = w4a16::run_wait_limit_check(i == 1, expect[i]);
        if (err == cudaSuccess) err = w4a16::read_device_status(&c, true);
        codes[i] = c;
    }
    if (err != cudaSuccess) return fail(W4A16_ERR_CUDA, std::string("CUDA error: ") + cudaGetErrorString(err));
    return ok();
}

const char* w4a16_status_string(w4a16_status status) {
    switch (status) {
        case W4A16_OK: return "W4A16_OK";
        case W4A16_ERR_NULL_POINTER: return "W4A16_ERR_NULL_POINTER";
        case W4A16_ERR_VARIANT: return "W4A16_ERR_VARIANT";
        case W4A16_ERR_M: return "W4A16_ERR_M";
        case W4A16_ERR_DIM_RANGE: return "W4A16_ERR_DIM_RANGE";
        case W4A16_ERR_K_MULTIPLE: return "W4A16_ERR_K_MULTIPLE";
        case W4A16_ERR_N_MULTIPLE: return "W4A16_ERR_N_MULTIPLE";
        case W4A16_ERR_GROUPS: return "W4A16_ERR_GROUPS";
        case W4A16_ERR_WP_SIZE: return "W4A16_ERR_WP_SIZE";
        case W4A16_ERR_ALIGNMENT: return "W4A16_ERR_ALIGNMENT";
        case W4A16_ERR_GROUP_SIZE: return "W4A16_ERR_GROUP_SIZE";
        case W4A16_ERR_DECODE_SHAPE: return "W4A16_ERR_DECODE_SHAPE";
        case W4A16_ERR_OUT_DTYPE: return "W4A16_ERR_OUT_DTYPE";
        case W4A16_ERR_DEVICE: return "W4A16_ERR_DEVICE";
        case W4A16_ERR_CUDA: return "W4A16_ERR_CUDA";
        case W4A16_ERR_DEVICE_TIMEOUT: return "W4A16_ERR_DEVICE_TIMEOUT";
        case W4A16_ERR_WORKSPACE: return "W4A16_ERR_WORKSPACE";
        case W4A16_ERR_FLAGS: return "W4A16_ERR_FLAGS";
        case W4A16_ERR_TP_GROUP: return "W4A16_ERR_TP_GROUP";
    }
    return "W4A16_ERR_UNKNOWN";
}

const char* w4a16_last_error(void) {
    return g_last_error.c_str();
}

}  // extern "C"
