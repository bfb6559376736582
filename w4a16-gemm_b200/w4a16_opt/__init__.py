"""B200-native W4A16 GEMM with the reference's drop-in surface.

    from w4a16_opt import w4a16_gemm
    y = w4a16_gemm(Wp, x, scales, variant=-1)      # y[M, N] = x @ ((q - 8) * scale)^T

Same module name, function name, argument meaning, weight format and error
messages as akshay919191/W4A16-GEMM (src/vectorized/extension.cpp:5-8,
kernel.cu:218-267).  ``variant``: -1 auto, 0 the decode kernel (M <= 16,
N % 64 == 0, K % 512 == 0), 1..4 force a prefill tile config (token tile
32 / 64 / 128 / 256 on the tcgen05 kernel).

There is exactly one implementation: CUDA kernels for sm_100a behind the C ABI
in ``libw4a16.so`` (include/w4a16.h).  Importing this package without the built
extension raises ImportError -- there is no CPU fallback.
"""
from __future__ import annotations

import os

import torch  # noqa: F401  (loads libc10 / libtorch before the binding)

_HERE = os.path.dirname(os.path.abspath(__file__))

try:
    from . import _C  # type: ignore[attr-defined]
except ImportError as exc:  # pragma: no cover - exercised only when unbuilt
    raise ImportError(
        "w4a16_opt: the CUDA extension is not built (expected w4a16_opt/_C*.so and libw4a16.so); "
        "run `python w4a16-gemm_b200/build.py`"
    ) from exc

from .format import dequantize_w4, pack_int4, quantize_pack, quantize_w4, unpack_int4  # noqa: E402

LIBRARY_PATH = os.path.join(_HERE, "libw4a16.so")
ABI_VERSION = _C.ABI_VERSION
PREFILL_VARIANTS = (1, 2, 3, 4)


def w4a16_gemm(Wp: torch.Tensor, x: torch.Tensor, scales: torch.Tensor, variant: int = -1) -> torch.Tensor:
    """y = x @ W^T with W[n, k] = (q[n, k] - 8) * scales[k // G, n]; fresh fp16 [M, N].

    Wp: int32 [N*K/8] packed codes; x: fp16 [M, K]; scales: fp16 [K/G, N], G in {64, 128}.
    Runs on the current CUDA stream of x's device.  Raises RuntimeError on bad input.
    """
    return _C.w4a16_gemm(Wp, x, scales, variant)


def w4a16_gemm_out(Wp: torch.Tensor, x: torch.Tensor, scales: torch.Tensor, y: torch.Tensor,
                   variant: int = -1, workspace: torch.Tensor | None = None,
                   weights_resident: bool = False, fp32_scale: bool = False) -> torch.Tensor:
    """Same GEMM into a preallocated contiguous ``y`` (fp16, or fp32 for partial sums).

    ``workspace``: optional scratch CUDA buffer (see ``make_workspace``; no initialisation
    needed) reused by calls issued in stream order.  Without it the binding keeps one per
    (device, stream), or one per capture under CUDA-graph capture.

    ``weights_resident``: the caller declares that ``Wp`` and ``scales`` were not written by
    the kernel launched just before this call on the stream (loaded earlier, copied, or made
    by this package's format functions).  The decode kernel then starts streaming them
    before that kernel has finished.  By default the GEMM reads nothing before the previous
    kernel's writes are visible, as plain stream order promises.

    ``fp32_scale``: for M <= 8 on the decode path, multiply by the group scales in fp32
    after the tensor-core products instead of rounding every dequantised weight to fp16
    first (more accurate and about 6 % faster on the decode sweep, but not the reference's
    bit-identical dequantised values; ignored for M > 8 and for prefill).
    """
    return _C.w4a16_gemm_out(Wp, x, scales, y, variant, workspace, weights_resident, fp32_scale)


def workspace_bytes(M: int, N: int, K: int, groups: int, variant: int = -1) -> int:
    """Workspace bytes a call with these dimensions needs on the current device."""
    return _C.workspace_bytes(M, N, K, groups, variant)


def make_workspace(nbytes: int, device=None) -> torch.Tensor:
    """A workspace buffer of at least ``nbytes`` bytes (zero-filled, though no call needs that)."""
    return torch.zeros(max(256, int(nbytes)), dtype=torch.uint8, device=device or "cuda")


def w4a16_dequant(Wp: torch.Tensor, scales: torch.Tensor, K: int) -> torch.Tensor:
    """Dequantised weights fp16 [N, K], bit-identical to the reference dequantisation."""
    return _C.w4a16_dequant(Wp, scales, K)


def query_route(M: int, N: int, K: int, groups: int, variant: int = -1) -> dict:
    """Kernel, tile shape, split and grid the GEMM would launch on the current device."""
    return _C.query_route(M, N, K, groups, variant)


def device_status(reset: bool = False) -> int:
    """Device status word (non-zero if a kernel's bounded wait ran out); synchronises."""
    return _C.device_status(reset)


__all__ = [
    "w4a16_gemm", "w4a16_gemm_out", "w4a16_dequant", "query_route", "device_status",
    "workspace_bytes", "make_workspace",
    "pack_int4", "unpack_int4", "quantize_w4", "quantize_pack", "dequantize_w4",
    "LIBRARY_PATH", "ABI_VERSION", "PREFILL_VARIANTS",
]
