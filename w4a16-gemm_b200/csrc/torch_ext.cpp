// Thin PyTorch binding over the C ABI (include/w4a16.h), module w4a16_opt._C.
//
// Keeps the reference's Python surface -- w4a16_gemm(Wp, x, scales, variant=-1)
// (src/vectorized/extension.cpp:5-8) -- and its tensor checks, in the same
// order and with the same messages (src/vectorized/kernel.cu:219-223); every
// other check and the launch happen behind the C ABI.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <climits>
#include <map>
#include <vector>
#include <mutex>
#include <utility>

#include "../../include/w4a16.h"

namespace {

void check(w4a16_status s) {
    TORCH_CHECK(s == W4A16_OK, w4a16_last_error());
}

int32_t clamp_variant(int64_t v) {
    return (v < -1 || v > 4) ? INT32_MAX : (int32_t)v;   // out of range -> rejected by w4a16_validate
}

void check_tensors(const torch::Tensor& Wp, const torch::Tensor& x, const torch::Tensor& scales) {
    TORCH_CHECK(Wp.is_cuda() && x.is_cuda() && scales.is_cuda(), "all tensors must be CUDA");
    TORCH_CHECK(Wp.is_contiguous() && x.is_contiguous() && scales.is_contiguous(), "contiguous only");
    TORCH_CHECK(Wp.dtype() == torch::kInt32, "Wp must be int32");
    TORCH_CHECK(x.dtype() == torch::kHalf && scales.dtype() == torch::kHalf, "x, scales must be fp16");
    TORCH_CHECK(x.dim() == 2 && scales.dim() == 2, "x must be [M, K], scales must be [K/G, N]");
    TORCH_CHECK(Wp.device() == x.device() && scales.device() == x.device(), "all tensors must be on one device");
}

// Workspace for the split-K decode path (scratch, no initialisation needed): one buffer
// serves every call on a stream, since calls on one stream never overlap.  Eager calls
// use one buffer per (device, stream).  While a stream is being captured into a CUDA
// graph, the calls of that capture share a buffer taken from the graph's pool; a new
// capture on the stream releases the previous capture's.  Both maps are capped: streams
// come and go in serving engines, and a released buffer's memory is only reused in
// stream order.
torch::Tensor workspace_for(const torch::Tensor& x, uint64_t bytes, cudaStream_t stream) {
    if (bytes == 0) return torch::Tensor();
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    unsigned long long capture_id = 0;
    TORCH_CHECK(cudaStreamGetCaptureInfo(stream, &cap, &capture_id) == cudaSuccess, "cudaStreamGetCaptureInfo failed");
    auto opts = torch::TensorOptions().dtype(torch::kUInt8).device(x.device());
    constexpr size_t kMaxEntries = 64;
    static std::mutex mu;
    static std::map<std::pair<int, cudaStream_t>, torch::Tensor> eager;
    static std::map<std::pair<int, cudaStream_t>, std::pair<unsigned long long, torch::Tensor>> captured;
    const auto key = std::make_pair((int)x.get_device(), stream);
    std::lock_guard<std::mutex> lk(mu);
    if (cap != cudaStreamCaptureStatusNone) {
        auto it = captured.find(key);
        if (it != captured.end() && it->second.first == capture_id && (uint64_t)it->second.second.numel() >= bytes)
            return it->second.second;
        if (it == captured.end() && captured.size() >= kMaxEntries) captured.clear();
        auto ws = torch::empty({(int64_t)bytes}, opts);
        captured[key] = {capture_id, ws};
        return ws;
    }
    auto it = eager.find(key);
    if (it != eager.end() && (uint64_t)it->second.numel() >= bytes) return it->second;
    if (it == eager.end() && eager.size() >= kMaxEntries) eager.clear();
    auto ws = torch::empty({(int64_t)bytes}, opts);
    eager[key] = ws;
    return ws;
}

void run(const torch::Tensor& Wp, const torch::Tensor& x, const torch::Tensor& scales, torch::Tensor& y,
         int32_t variant, const c10::optional<torch::Tensor>& user_ws = c10::nullopt, uint32_t flags = 0) {
    const at::cuda::CUDAGuard guard(x.device());
    cudaStream_t stream = at::cuda::getCurrentCUDAStream().stream();
    uint64_t ws_bytes = 0;
    torch::Tensor ws;
    if (user_ws.has_value() && user_ws->defined()) {
        ws = *user_ws;
        TORCH_CHECK(ws.is_cuda() && ws.device() == x.device() && ws.is_contiguous(),
                    "workspace must be a contiguous CUDA tensor on x's device");
        ws_bytes = (uint64_t)ws.numel() * ws.element_size();
    } else {
        check(w4a16_workspace_bytes(x.size(0), scales.size(1), x.size(1), scales.size(0), variant, &ws_bytes));
        ws = workspace_for(x, ws_bytes, stream);
    }
    check(w4a16_gemm_ex(Wp.data_ptr<int32_t>(), x.data_ptr(), scales.data_ptr(), y.data_ptr(), x.size(0),
                        scales.size(1), x.size(1), scales.size(0), Wp.numel(), variant,
                        y.scalar_type() == torch::kFloat ? W4A16_OUT_F32 : W4A16_OUT_F16, flags,
                        ws.defined() ? ws.data_ptr() : nullptr, ws_bytes, stream));
}

}  // namespace

// y = x @ W^T, fresh fp16 [M, N] output (reference: kernel.cu:218-267).
torch::Tensor w4a16_gemm_py(torch::Tensor Wp, torch::Tensor x, torch::Tensor scales, int64_t variant) {
    check_tensors(Wp, x, scales);
    const int32_t v = clamp_variant(variant);
    check(w4a16_validate(Wp.data_ptr(), x.data_ptr(), scales.data_ptr(), x.size(0), scales.size(1), x.size(1),
                         scales.size(0), Wp.numel(), v));
    auto y = torch::empty({x.size(0), scales.size(1)}, x.options());
    run(Wp, x, scales, y, v);
    return y;
}

// Same GEMM into a caller-provided contiguous y: fp16, or fp32 for row-parallel partial sums.
// `workspace` (optional): a CUDA buffer of >= workspace_bytes(...) bytes (scratch) that the
// caller keeps for calls issued in stream order; otherwise the binding supplies one.
// `weights_resident`: Wp and scales are not written by the kernel launched just before
// (W4A16_FLAG_WEIGHTS_RESIDENT).  `fp32_scale`: W4A16_FLAG_FP32_SCALE.
torch::Tensor w4a16_gemm_out_py(torch::Tensor Wp, torch::Tensor x, torch::Tensor scales, torch::Tensor y,
                                int64_t variant, c10::optional<torch::Tensor> workspace, bool weights_resident,
                                bool fp32_scale) {
    check_tensors(Wp, x, scales);
    TORCH_CHECK(y.is_cuda() && y.device() == x.device(), "y must be a CUDA tensor on x's device");
    TORCH_CHECK(y.is_contiguous(), "contiguous only");
    TORCH_CHECK(y.dtype() == torch::kHalf || y.dtype() == torch::kFloat, "y must be fp16 or fp32");
    TORCH_CHECK(y.dim() == 2 && y.size(0) == x.size(0) && y.size(1) == scales.size(1), "y must be [M, N]");
    const int32_t v = clamp_variant(variant);
    check(w4a16_validate(Wp.data_ptr(), x.data_ptr(), scales.data_ptr(), x.size(0), scales.size(1), x.size(1),
                         scales.size(0), Wp.numel(), v));
    run(Wp, x, scales, y, v, workspace,
        (weights_resident ? (uint32_t)W4A16_FLAG_WEIGHTS_RESIDENT : 0u) | (fp32_scale ? (uint32_t)W4A16_FLAG_FP32_SCALE : 0u));
    return y;
}

int64_t workspace_bytes_py(int64_t M, int64_t N, int64_t K, int64_t groups, int64_t variant) {
    uint64_t b = 0;
    check(w4a16_workspace_bytes(M, N, K, groups, clamp_variant(variant), &b));
    return (int64_t)b;
}

// Dequantised weights fp16 [N, K] (debug / verification).
torch::Tensor w4a16_dequant_py(torch::Tensor Wp, torch::Tensor scales, int64_t K) {
    TORCH_CHECK(Wp.is_cuda() && scales.is_cuda(), "all tensors must be CUDA");
    TORCH_CHECK(Wp.is_contiguous() && scales.is_contiguous(), "contiguous only");
    TORCH_CHECK(Wp.dtype() == torch::kInt32, "Wp must be int32");
    TORCH_CHECK(scales.dtype() == torch::kHalf && scales.dim() == 2, "scales must be fp16 [K/G, N]");
    const at::cuda::CUDAGuard guard(Wp.device());
    const int64_t N = scales.size(1);
    auto out = torch::empty({N, K}, scales.options());
    check(w4a16_validate(Wp.data_ptr(), nullptr, scales.data_ptr(), 1, N, K, scales.size(0), Wp.numel(), -1));
    check(w4a16_dequant(Wp.data_ptr<int32_t>(), scales.data_ptr(), out.data_ptr(), N, K, scales.size(0),
                        at::cuda::getCurrentCUDAStream().stream()));
    return out;
}

// Load-time format kernels (codes -> packed words; weights -> codes/packed + scales).
torch::Tensor pack_py(torch::Tensor q) {
    TORCH_CHECK(q.is_cuda() && q.is_contiguous() && q.dtype() == torch::kUInt8 && q.dim() == 2,
                "q must be a contiguous CUDA uint8 [N, K] tensor");
    const at::cuda::CUDAGuard guard(q.device());
    const int64_t N = q.size(0), K = q.size(1);
    auto wp = torch::empty({N * K / 8}, q.options().dtype(torch::kInt32));
    check(w4a16_pack(q.data_ptr<uint8_t>(), wp.data_ptr<int32_t>(), N, K, at::cuda::getCurrentCUDAStream().stream()));
    return wp;
}

std::vector<torch::Tensor> quantize_py(torch::Tensor W, int64_t group_size, bool pack) {
    TORCH_CHECK(W.is_cuda() && W.is_contiguous() && W.dim() == 2, "W must be a contiguous CUDA [N, K] tensor");
    TORCH_CHECK(W.dtype() == torch::kFloat || W.dtype() == torch::kHalf, "W must be fp32 or fp16");
    const at::cuda::CUDAGuard guard(W.device());
    const int64_t N = W.size(0), K = W.size(1);
    TORCH_CHECK(group_size > 0 && K % group_size == 0, "K must be a multiple of the group size");
    const int32_t wd = W.dtype() == torch::kHalf ? W4A16_W_F16 : W4A16_W_F32;
    auto scales = torch::empty({K / group_size, N}, W.options().dtype(torch::kHalf));
    cudaStream_t st = at::cuda::getCurrentCUDAStream().stream();
    if (pack) {
        auto wp = torch::empty({N * K / 8}, W.options().dtype(torch::kInt32));
        check(w4a16_quantize_pack(W.data_ptr(), wd, wp.data_ptr<int32_t>(), scales.data_ptr(), N, K, group_size, st));
        return {wp, scales};
    }
    auto q = torch::empty({N, K}, W.options().dtype(torch::kUInt8));
    check(w4a16_quantize(W.data_ptr(), wd, q.data_ptr<uint8_t>(), scales.data_ptr(), N, K, group_size, st));
    return {q, scales};
}

pybind11::dict query_route_py(int64_t M, int64_t N, int64_t K, int64_t groups, int64_t variant) {
    w4a16_route r;
    check(w4a16_query_route(M, N, K, groups, clamp_variant(variant), &r));
    pybind11::dict d;
    d["kernel"] = r.kernel == 0 ? "decode" : "prefill";
    d["config"] = r.config;
    d["tile_m"] = r.tile_m;
    d["tile_n"] = r.tile_n;
    d["split_k"] = r.split_k;
    d["grid"] = r.grid;
    d["stages"] = r.stages;
    d["smem_bytes"] = r.smem_bytes;
    d["workspace_bytes"] = r.workspace_bytes;
    d["launches"] = r.launches;
    return d;
}

int64_t device_status_py(bool reset) {
    int32_t code = 0;
    w4a16_status s = w4a16_device_status(&code, reset ? 1 : 0);
    TORCH_CHECK(s == W4A16_OK || s == W4A16_ERR_DEVICE_TIMEOUT, w4a16_last_error());
    return code;
}

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
    m.def("w4a16_gemm", &w4a16_gemm_py,
          "W4A16 GEMM on B200: decode (M <= 16) weight-streaming kernel + tcgen05 prefill for any M",
          pybind11::arg("Wp"), pybind11::arg("x"), pybind11::arg("scales"), pybind11::arg("variant") = -1);
    m.def("w4a16_gemm_out", &w4a16_gemm_out_py, "W4A16 GEMM into a preallocated fp16/fp32 output",
          pybind11::arg("Wp"), pybind11::arg("x"), pybind11::arg("scales"), pybind11::arg("y"),
          pybind11::arg("variant") = -1, pybind11::arg("workspace") = pybind11::none(),
          pybind11::arg("weights_resident") = false, pybind11::arg("fp32_scale") = false);
    m.def("workspace_bytes", &workspace_bytes_py, "workspace bytes a GEMM call needs on the current device",
          pybind11::arg("M"), pybind11::arg("N"), pybind11::arg("K"), pybind11::arg("groups"),
          pybind11::arg("variant") = -1);
    m.def("w4a16_dequant", &w4a16_dequant_py, "dequantised fp16 [N, K] weights", pybind11::arg("Wp"),
          pybind11::arg("scales"), pybind11::arg("K"));
    m.def("query_route", &query_route_py, "kernel / tile / grid the GEMM would launch", pybind11::arg("M"),
          pybind11::arg("N"), pybind11::arg("K"), pybind11::arg("groups"), pybind11::arg("variant") = -1);
    m.def("device_status", &device_status_py, "device status word set by timed-out kernel waits",
          pybind11::arg("reset") = false);
    m.def("pack", &pack_py, "uint8 codes [N, K] -> packed int32 words (GPU)", pybind11::arg("q"));
    m.def("quantize", &quantize_py, "fp32/fp16 W [N, K] -> (codes or packed words, fp16 scales [K/G, N]) (GPU)",
          pybind11::arg("W"), pybind11::arg("group_size"), pybind11::arg("pack") = false);
    m.attr("ABI_VERSION") = w4a16_abi_version();
}
