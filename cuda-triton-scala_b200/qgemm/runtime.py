"""Device, stream and buffer handles over libqgemm.

These replace the reference's DeviceRuntime / CUDARuntime buffer management
(src/main/scala/cuda/dsl/runtime/DeviceRuntime.scala:13-45,
runtime/CUDARuntime.scala:204-311) and Ptr.alloc/free (core/Ptr.scala:148-149):
buffers are explicit device allocations addressed by a 64-bit ``address``.
"""
from __future__ import annotations

import ctypes

import numpy as np

from . import _lib as L


def device_count() -> int:
    n = ctypes.c_int(0)
    L.call("qgemm_device_count", ctypes.byref(n))
    return n.value


class Device:
    """An opened GPU (qgemm_device_t)."""

    def __init__(self, ordinal: int = 0):
        h = ctypes.c_void_p()
        L.call("qgemm_device_open", ordinal, ctypes.byref(h))
        self.handle = h
        self.ordinal = ordinal
        sm, ma, mi, l2, tc = (ctypes.c_int(), ctypes.c_int(), ctypes.c_int(),
                              ctypes.c_size_t(), ctypes.c_int())
        L.call("qgemm_device_info", h, ctypes.byref(sm), ctypes.byref(ma), ctypes.byref(mi),
               ctypes.byref(l2), ctypes.byref(tc))
        self.sm_count = sm.value
        self.cc = (ma.value, mi.value)
        self.l2_bytes = l2.value
        self.has_tcgen05 = bool(tc.value)

    def close(self):
        if self.handle:
            L.call("qgemm_device_close", self.handle)
            self.handle = None

    @property
    def wait_limit_ns(self) -> int:
        """Limit of every bounded device-side wait of the tensor-core GEMM kernels."""
        v = ctypes.c_uint64()
        L.call("qgemm_device_get_wait_limit", self.handle, ctypes.byref(v))
        return v.value

    @wait_limit_ns.setter
    def wait_limit_ns(self, ns: int):
        L.call("qgemm_device_set_wait_limit", self.handle, int(ns))

    def debug_hold_split(self, enable: bool):
        """Test hook: make the W8A8 GEMM's split waits run out (the timeout path)."""
        L.call("qgemm_debug_hold_split", self.handle, 1 if enable else 0)

    def stream(self) -> "Stream":
        return Stream(self)

    def wrap_stream(self, cuda_stream: int) -> "Stream":
        return Stream(self, cuda_stream=cuda_stream)

    def alloc(self, nbytes: int) -> "Buffer":
        return Buffer(self, nbytes)


class Stream:
    """qgemm_stream_t: an owned CUDA stream, or an adopted one (e.g. torch's)."""

    def __init__(self, dev: Device, cuda_stream: int | None = None):
        h = ctypes.c_void_p()
        if cuda_stream is None:
            L.call("qgemm_stream_create", dev.handle, ctypes.byref(h))
        else:
            L.call("qgemm_stream_wrap", dev.handle, ctypes.c_void_p(cuda_stream), ctypes.byref(h))
        self.handle = h
        self.dev = dev

    def sync(self):
        L.call("qgemm_stream_sync", self.handle)

    def destroy(self):
        if self.handle:
            L.call("qgemm_stream_destroy", self.handle)
            self.handle = None

    # host <-> device
    def h2d(self, dst, host: np.ndarray):
        host = np.ascontiguousarray(host)
        L.call("qgemm_memcpy_h2d", self.handle, L.addr(dst), host.ctypes.data_as(ctypes.c_void_p),
               host.nbytes)

    def d2h(self, host: np.ndarray, src):
        assert host.flags["C_CONTIGUOUS"]
        L.call("qgemm_memcpy_d2h", self.handle, host.ctypes.data_as(ctypes.c_void_p), L.addr(src),
               host.nbytes)

    def h2d_ptr(self, dst: int, host_ptr: int, nbytes: int):
        """Copy from a raw host address (e.g. pinned memory) to a device address."""
        L.call("qgemm_memcpy_h2d", self.handle, int(dst), ctypes.c_void_p(host_ptr), nbytes)

    def d2h_ptr(self, host_ptr: int, src: int, nbytes: int):
        L.call("qgemm_memcpy_d2h", self.handle, ctypes.c_void_p(host_ptr), int(src), nbytes)

    def memset(self, dst, value: int, nbytes: int):
        L.call("qgemm_memset", self.handle, L.addr(dst), value, nbytes)


class Buffer:
    """A device allocation; ``address`` is the reference's Ptr.address."""

    def __init__(self, dev: Device, nbytes: int):
        a = ctypes.c_uint64(0)
        L.call("qgemm_buffer_alloc", dev.handle, nbytes, ctypes.byref(a))
        self.address = a.value
        self.nbytes = nbytes
        self.dev = dev

    def free(self):
        if self.address:
            L.call("qgemm_buffer_free", self.dev.handle, self.address)
            self.address = 0

    def __del__(self):
        try:
            if self.address and self.dev.handle:
                L.try_call("qgemm_buffer_free", self.dev.handle, self.address)
        except Exception:
            pass

    @staticmethod
    def from_numpy(dev: Device, stream: Stream, arr: np.ndarray) -> "Buffer":
        arr = np.ascontiguousarray(arr)
        b = Buffer(dev, max(arr.nbytes, 1))
        stream.h2d(b, arr)
        return b

    def to_numpy(self, stream: Stream, dtype, shape) -> np.ndarray:
        out = np.empty(shape, dtype=dtype)
        stream.d2h(out, self)
        stream.sync()
        return out
