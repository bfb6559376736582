"""ctypes binding of the C ABI (include/w4a16.h) -- the binding a non-torch host adds.

    lib = load()                         # libw4a16.so next to this file
    st = lib.w4a16_gemm(Wp_ptr, x_ptr, s_ptr, y_ptr, M, N, K, groups, wp_words,
                        variant, W4A16_OUT_F16, ws_ptr, ws_bytes, stream_ptr)

Every exported function and its argument types are declared here; the
``EXPORTS`` table is the list include/w4a16.h declares.
"""
from __future__ import annotations

import ctypes
import os

W4A16_OK = 0
W4A16_OUT_F16 = 0
W4A16_OUT_F32 = 1
W4A16_FLAG_WEIGHTS_RESIDENT = 1
W4A16_FLAG_FP32_SCALE = 2

STATUS_NAMES = {
    0: "W4A16_OK", 1: "W4A16_ERR_NULL_POINTER", 2: "W4A16_ERR_VARIANT", 3: "W4A16_ERR_M",
    4: "W4A16_ERR_DIM_RANGE", 5: "W4A16_ERR_K_MULTIPLE", 6: "W4A16_ERR_N_MULTIPLE", 7: "W4A16_ERR_GROUPS",
    8: "W4A16_ERR_WP_SIZE", 9: "W4A16_ERR_ALIGNMENT", 10: "W4A16_ERR_GROUP_SIZE",
    11: "W4A16_ERR_DECODE_SHAPE", 12: "W4A16_ERR_OUT_DTYPE", 13: "W4A16_ERR_DEVICE", 14: "W4A16_ERR_CUDA",
    15: "W4A16_ERR_DEVICE_TIMEOUT", 16: "W4A16_ERR_WORKSPACE", 17: "W4A16_ERR_FLAGS", 18: "W4A16_ERR_TP_GROUP",
}
TP_MAX_RANKS = 8
TP_CTRL_BYTES = 8192
TP_PUSH_MAX_BYTES = 1 << 20


class Route(ctypes.Structure):
    _fields_ = [(name, ctypes.c_int32) for name in
                ("kernel", "config", "tile_m", "tile_n", "split_k", "grid", "stages", "smem_bytes")] + \
               [("workspace_bytes", ctypes.c_uint64), ("launches", ctypes.c_int32), ("reserved", ctypes.c_int32)]


_i64, _i32, _u64, _vp = ctypes.c_int64, ctypes.c_int32, ctypes.c_uint64, ctypes.c_void_p


class IpcHandle(ctypes.Structure):
    _fields_ = [("bytes", ctypes.c_ubyte * 64)]


class TpGroup(ctypes.Structure):
    _fields_ = [("rank", ctypes.c_int32), ("world", ctypes.c_int32), ("buf", ctypes.c_void_p * TP_MAX_RANKS),
                ("buf_bytes", ctypes.c_uint64), ("recv_off", ctypes.c_uint64), ("recv_bytes", ctypes.c_uint64)]

# name -> (restype, argtypes), one entry per declaration in include/w4a16.h
EXPORTS = {
    "w4a16_abi_version": (_i32, []),
    "w4a16_validate": (_i32, [_vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _i32]),
    "w4a16_workspace_bytes": (_i32, [_i64, _i64, _i64, _i64, _i32, ctypes.POINTER(_u64)]),
    "w4a16_gemm": (_i32, [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _i32, _i32, _vp, _u64, _vp]),
    "w4a16_gemm_ex": (_i32, [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _i32, _i32, ctypes.c_uint32, _vp,
                             _u64, _vp]),
    "w4a16_gemm_noalloc": (_i32, [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _i32, _i32, _vp]),
    "w4a16_query_route": (_i32, [_i64, _i64, _i64, _i64, _i32, ctypes.POINTER(Route)]),
    "w4a16_dequant": (_i32, [_vp, _vp, _vp, _i64, _i64, _i64, _vp]),
    "w4a16_pack": (_i32, [_vp, _vp, _i64, _i64, _vp]),
    "w4a16_quantize": (_i32, [_vp, _i32, _vp, _vp, _i64, _i64, _i64, _vp]),
    "w4a16_quantize_pack": (_i32, [_vp, _i32, _vp, _vp, _i64, _i64, _i64, _vp]),
    "w4a16_peer_alloc": (_i32, [_u64, ctypes.POINTER(_vp), ctypes.POINTER(IpcHandle)]),
    "w4a16_peer_open": (_i32, [ctypes.POINTER(IpcHandle), ctypes.POINTER(_vp)]),
    "w4a16_peer_close": (_i32, [_vp]),
    "w4a16_peer_free": (_i32, [_vp]),
    "w4a16_tp_allreduce": (_i32, [ctypes.POINTER(TpGroup), _u64, _u64, _i64, _i64, _vp]),
    "w4a16_tp_allgather": (_i32, [ctypes.POINTER(TpGroup), _u64, _u64, _i64, _i64, _vp]),
    "w4a16_device_status": (_i32, [ctypes.POINTER(_i32), _i32]),
    "w4a16_check_wait_limits": (_i32, [ctypes.POINTER(_i32)]),
    "w4a16_status_string": (ctypes.c_char_p, [_i32]),
    "w4a16_last_error": (ctypes.c_char_p, []),
}

_LIB = None


def library_path() -> str:
    return os.path.join(os.path.dirname(os.path.abspath(__file__)), "libw4a16.so")


def load(path: str | None = None) -> ctypes.CDLL:
    """Load libw4a16.so and declare every exported signature."""
    global _LIB
    if _LIB is not None and path is None:
        return _LIB
    lib = ctypes.CDLL(path or library_path())
    for name, (res, args) in EXPORTS.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    if path is None:
        _LIB = lib
    return lib


def last_error(lib: ctypes.CDLL | None = None) -> str:
    lib = lib or load()
    return lib.w4a16_last_error().decode()


class W4A16Error(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"{STATUS_NAMES.get(status, status)}: {message}")
        self.status = status


def check(status: int, lib: ctypes.CDLL | None = None) -> None:
    if status != W4A16_OK:
        raise W4A16Error(status, last_error(lib))
