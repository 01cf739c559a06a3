"""ctypes binding of libqgemm.so (include/qgemm.h).

The library is loaded from the package's own ``lib/`` directory.  There is no
fallback: if libqgemm.so is missing or cannot be loaded, importing the binding
raises, so a product call can never silently run somewhere else.
"""
from __future__ import annotations

import ctypes
import os

PKG_DIR = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB_PATH = os.path.join(PKG_DIR, "lib", "libqgemm.so")
HEADER_PATH = os.path.join(os.path.dirname(PKG_DIR), "include", "qgemm.h")

# status codes (qgemm.h)
OK = 0
ERR_INVALID_ARG = -1
ERR_BAD_ALIGN = -2
ERR_CUDA = -3
ERR_NCCL = -4
ERR_TIMEOUT = -5
ERR_UNSUPPORTED = -6
ERR_NO_DEVICE = -7
ERR_OOM = -8
ERR_BAD_HANDLE = -9

F32 = 0
BF16 = 1
B_KN = 0
B_NK = 1
ALGO_AUTO = 0
ALGO_TCGEN05 = 1
ALGO_SIMT = 2
PREFILL_FRAG = 1
PREFILL_ONE_TERM = 2

BLOB_VERSION = 1
BLOB_W4_TILED = 1
BLOB_W8_KN = 2
BLOB_W8_NK = 3
BLOB_W4_FRAG = 4


class BlobInfo(ctypes.Structure):
    """qgemm_blob_info (include/qgemm.h)."""
    _fields_ = [("version", ctypes.c_uint32), ("kind", ctypes.c_int32), ("K", ctypes.c_int32),
                ("N", ctypes.c_int32), ("group_size", ctypes.c_int32),
                ("zero_point", ctypes.c_int32), ("weight_bytes", ctypes.c_uint64),
                ("scale_bytes", ctypes.c_uint64)]


_S = ctypes.c_int32
_P = ctypes.c_void_p
_U64 = ctypes.c_uint64
_I = ctypes.c_int
_SZ = ctypes.c_size_t

# name -> (restype, argtypes), in header order.
SIGNATURES = {
    "qgemm_last_error": (ctypes.c_char_p, []),
    "qgemm_status_string": (ctypes.c_char_p, [_S]),
    "qgemm_version": (_I, []),
    "qgemm_device_count": (_S, [ctypes.POINTER(_I)]),
    "qgemm_device_open": (_S, [_I, ctypes.POINTER(_P)]),
    "qgemm_device_close": (_S, [_P]),
    "qgemm_device_info": (_S, [_P, ctypes.POINTER(_I), ctypes.POINTER(_I), ctypes.POINTER(_I),
                               ctypes.POINTER(_SZ), ctypes.POINTER(_I)]),
    "qgemm_device_set_wait_limit": (_S, [_P, _U64]),
    "qgemm_device_get_wait_limit": (_S, [_P, ctypes.POINTER(_U64)]),
    "qgemm_debug_hold_split": (_S, [_P, _I]),
    "qgemm_stream_create": (_S, [_P, ctypes.POINTER(_P)]),
    "qgemm_stream_wrap": (_S, [_P, _P, ctypes.POINTER(_P)]),
    "qgemm_stream_destroy": (_S, [_P]),
    "qgemm_stream_sync": (_S, [_P]),
    "qgemm_buffer_alloc": (_S, [_P, _SZ, ctypes.POINTER(_U64)]),
    "qgemm_buffer_free": (_S, [_P, _U64]),
    "qgemm_memcpy_h2d": (_S, [_P, _U64, _P, _SZ]),
    "qgemm_memcpy_d2h": (_S, [_P, _P, _U64, _SZ]),
    "qgemm_memset": (_S, [_P, _U64, _I, _SZ]),
    "qgemm_host_alloc": (_S, [_SZ, ctypes.POINTER(_P)]),
    "qgemm_host_free": (_S, [_P]),
    "qgemm_w8a32_gemm": (_S, [_P, _U64, _U64, _U64, _U64, _U64, _I, _I, _I]),
    "qgemm_w4a16_gemm": (_S, [_P, _U64, _U64, _U64, _U64, _I, _I, _I]),
    "qgemm_w8a16_gemm": (_S, [_P, _U64, _U64, _U64, _U64, _U64, _I, _I, _I, _I]),
    "qgemm_w8a16_gemm_rowwise": (_S, [_P, _U64, _U64, _U64, _U64, _I, _I, _I]),
    "qgemm_dynamic_quantize": (_S, [_P, _U64, _U64, _U64, _I, _I, _I]),
    "qgemm_weight_only_quantize_per_channel": (_S, [_P, _U64, _U64, _U64, _U64, _I, _I]),
    "qgemm_dequantize": (_S, [_P, _U64, _U64, _U64, _I, _I]),
    "qgemm_w8a8_gemm": (_S, [_P, _U64, _U64, _I, _U64, _U64, _U64, _I, _I, _I, _I, _I, _U64, _I]),
    "qgemm_tensor_core_gemm_int8": (_S, [_P, _U64, _U64, _U64, _U64, _U64, _U64, _I, _I, _I, _I,
                                         _I, _I, _I, _I]),
    "qgemm_int8_gemm_kernel": (_S, [_P, _U64, _U64, _U64, _I, _I, _I, _I, _I, _I, ctypes.c_float,
                                    ctypes.c_float]),
    "qgemm_w8a8_gemm_static_scratch": (_S, [_P, _U64, _U64, _I, _U64, _U64, _U64, _I, _I, _I, _I,
                                             _I, _U64, _I]),
    "qgemm_w4a16_grouped_gemm": (_S, [_P, _U64, _U64, _U64, _I, _I, _U64, _I, _I, _I]),
    "qgemm_w4a16_grouped_gemm_tiled": (_S, [_P, _U64, _U64, _U64, _I, _I, _U64, _I, _I, _I]),
    "qgemm_w4_tiled_bytes": (_S, [_I, _I, ctypes.POINTER(_SZ)]),
    "qgemm_prepack_w4_tiled": (_S, [_P, _U64, _U64, _I, _I]),
    "qgemm_w4a16_grouped_gemm_frag": (_S, [_P, _U64, _U64, _U64, _I, _I, _U64, _I, _I, _I]),
    "qgemm_w4_frag_bytes": (_S, [_I, _I, ctypes.POINTER(_SZ)]),
    "qgemm_prepack_w4_frag": (_S, [_P, _U64, _U64, _I, _I]),
    "qgemm_w4a16_grouped_gemm_prefill_frag": (_S, [_P, _U64, _U64, _U64, _I, _I, _U64, _I, _I,
                                                   _I, _U64, _SZ]),
    "qgemm_w4a16_prefill_workspace_bytes": (_S, [_I, _I, ctypes.POINTER(_SZ)]),
    "qgemm_w4a16_grouped_gemm_prefill": (_S, [_P, _U64, _U64, _U64, _I, _I, _U64, _I, _I, _I,
                                               _U64, _SZ]),
    "qgemm_w4a16_prefill_workspace_bytes_ex": (_S, [_I, _I, _I, ctypes.POINTER(_SZ)]),
    "qgemm_w4a16_grouped_gemm_prefill_ex": (_S, [_P, _U64, _U64, _U64, _I, _I, _U64, _I, _I,
                                                 _I, _U64, _SZ, _I]),
    "qgemm_gemm_bf16_nk": (_S, [_P, _U64, _U64, _U64, _I, _I, _I, _I]),
    "qgemm_quantize_per_token": (_S, [_P, _U64, _I, _U64, _U64, _I, _I]),
    "qgemm_gemm_f32": (_S, [_P, _U64, _U64, _U64, _U64, _I, _I, _I, ctypes.c_float,
                            ctypes.c_float, _I, _I]),
    "qgemm_matmul_f32": (_S, [_P, _U64, _U64, _U64, _I, _I, _I]),
    "qgemm_matmul_add_bias_f32": (_S, [_P, _U64, _U64, _U64, _U64, _I, _I, _I]),
    "qgemm_sgemm": (_S, [_P, _U64, _U64, _U64, _I, _I, _I, ctypes.c_float, ctypes.c_float]),
    "qgemm_gemv_f32": (_S, [_P, _U64, _U64, _U64, _I, _I]),
    "qgemm_prepack_w8_nk": (_S, [_P, _U64, _U64, _I, _I]),
    "qgemm_launch_by_name": (_S, [_P, ctypes.c_char_p, ctypes.POINTER(_U64), _I,
                                  ctypes.POINTER(_I), _I]),
    "qgemm_bridge_launch_kernel": (ctypes.c_int64, [_P, ctypes.c_char_p, _I, _I, _I, _I, _I, _I,
                                                    ctypes.POINTER(_U64), _I,
                                                    ctypes.POINTER(ctypes.c_float),
                                                    ctypes.POINTER(ctypes.c_char_p), _I]),
    "qgemm_blob_save": (_S, [ctypes.c_char_p, ctypes.POINTER(BlobInfo), _P, _P]),
    "qgemm_blob_info_read": (_S, [ctypes.c_char_p, ctypes.POINTER(BlobInfo)]),
    "qgemm_blob_load": (_S, [ctypes.c_char_p, _P, _SZ, _P, _SZ]),
    "qgemm_blob_load_device": (_S, [_P, ctypes.c_char_p, _U64, _SZ, _U64, _SZ]),
    "qgemm_shard_columns": (_S, [_I, _I, _I, _I, ctypes.POINTER(_I), ctypes.POINTER(_I)]),
    "qgemm_comm_unique_id": (_S, [_P]),
    "qgemm_comm_init": (_S, [_P, _P, _I, _I, ctypes.POINTER(_P)]),
    "qgemm_comm_destroy": (_S, [_P]),
    "qgemm_comm_allgather_bf16": (_S, [_P, _P, _U64, _U64, _SZ]),
    "qgemm_unshard_columns_bf16": (_S, [_P, _U64, _U64, _I, _I, _I]),
    "qgemm_w8a8_allgather_work_bytes": (_SZ, [_I, _I, _I]),
    "qgemm_w8a8_gemm_allgather_bf16": (_S, [_P, _P, _P, _U64, _U64, _I, _U64, _U64, _U64, _I, _I,
                                            _I, _I, _U64, _SZ]),
    "qgemm_comm_window_register": (_S, [_P, _P, _U64, _SZ, ctypes.POINTER(_P)]),
    "qgemm_comm_window_release": (_S, [_P]),
    "qgemm_w8a8_gemm_allgather_window_bf16": (_S, [_P, _P, _P, _U64, _U64, _I, _U64, _U64, _I,
                                                   _I, _I, _I]),
    "qgemm_w8a8_gemm_allgather_fused_bf16": (_S, [_P, _P, _U64, _U64, _I, _U64, _U64, _I, _I,
                                                  _I]),
}

_lib = None


class QGemmError(RuntimeError):
    """A libqgemm call returned a non-OK status."""

    def __init__(self, status: int, func: str, message: str):
        self.status = status
        self.func = func
        super().__init__(f"{func}: {status_name(status)} ({status}): {message}")


def lib():
    """Loads libqgemm.so (once).  Raises if the library has not been built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"libqgemm.so not found at {LIB_PATH}; build it with "
                              f"cuda-triton-scala_b200/build.py")
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _lib = L
    return _lib


def status_name(s: int) -> str:
    return lib().qgemm_status_string(s).decode()


def last_error() -> str:
    return lib().qgemm_last_error().decode()


def check(status: int, func: str) -> None:
    if status != OK:
        raise QGemmError(status, func, last_error())


def call(name: str, *args) -> None:
    """Calls an entry point and raises QGemmError on a non-OK status."""
    check(getattr(lib(), name)(*args), name)


def try_call(name: str, *args) -> int:
    """Calls an entry point and returns its status (no exception)."""
    return int(getattr(lib(), name)(*args))


def addr(x) -> int:
    """Device address of a Ptr-like argument: an int address (the reference's
    Ptr.address), an object with ``.address`` or a torch tensor (data_ptr)."""
    if x is None:
        return 0
    if isinstance(x, int):
        return x
    if hasattr(x, "data_ptr"):
        return int(x.data_ptr())
    if hasattr(x, "address"):
        return int(x.address)
    raise TypeError(f"cannot take a device address of {type(x).__name__}")
