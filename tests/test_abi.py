"""The C-ABI library loads here (no GPU) and exports exactly what
include/qgemm.h declares; host-only entry points behave; no compute calls."""
import ctypes
import re
import subprocess

import pytest


def header_functions():
    import qgemm._lib as L
    src = open(L.HEADER_PATH).read()
    return sorted(set(re.findall(r"QGEMM_API\s+[\w\s\*]+?\b(qgemm_\w+)\s*\(", src)))


def test_library_loads():
    import qgemm
    assert qgemm.lib() is not None
    assert qgemm.lib().qgemm_version() >= 10000


def test_exports_every_header_symbol():
    import qgemm._lib as L
    declared = header_functions()
    assert len(declared) >= 30
    out = subprocess.run(["nm", "-D", "--defined-only", L.LIB_PATH], capture_output=True,
                         text=True, check=True).stdout
    exported = set(re.findall(r"\sT\s(qgemm_\w+)", out))
    missing = [f for f in declared if f not in exported]
    assert not missing, f"declared but not exported: {missing}"
    extra = sorted(exported - set(declared))
    assert not extra, f"exported but not declared: {extra}"
    # and the Python binding knows every one of them
    assert set(L.SIGNATURES) == set(declared)


def test_status_strings():
    import qgemm
    import qgemm._lib as L
    assert qgemm.status_name(L.OK) == "QGEMM_OK"
    assert qgemm.status_name(L.ERR_TIMEOUT) == "QGEMM_ERR_TIMEOUT"
    assert qgemm.status_name(12345) == "QGEMM_ERR_UNKNOWN"


def test_null_handles_return_status():
    import qgemm._lib as L
    lib = L.lib()
    assert lib.qgemm_stream_sync(None) == L.ERR_BAD_HANDLE
    assert "stream" in L.last_error()
    assert lib.qgemm_w8a32_gemm(None, 1, 1, 1, 1, 1, 4, 4, 4) == L.ERR_BAD_HANDLE
    assert lib.qgemm_device_close(None) == L.ERR_BAD_HANDLE
    assert lib.qgemm_comm_destroy(None) == L.ERR_BAD_HANDLE
    assert lib.qgemm_device_open(0, None) == L.ERR_INVALID_ARG


def test_device_count_without_gpu():
    import torch
    import qgemm
    if torch.cuda.is_available():
        pytest.skip("a GPU is visible")
    assert qgemm.device_count() == 0
    import qgemm._lib as L
    h = ctypes.c_void_p()
    assert L.lib().qgemm_device_open(0, ctypes.byref(h)) == L.ERR_NO_DEVICE


@pytest.mark.parametrize("N,world,align", [(28672, 8, 256), (28672, 2, 256), (4096, 4, 128),
                                           (1000, 3, 16), (7, 4, 1), (256, 8, 256)])
def test_shard_columns_partition(N, world, align):
    import qgemm
    bounds = [qgemm.shard_columns(N, world, r, align) for r in range(world)]
    assert bounds[0][0] == 0 and bounds[-1][1] == N
    for (a0, a1), (b0, b1) in zip(bounds, bounds[1:]):
        assert a1 == b0 and a0 <= a1
    for a0, _ in bounds:
        assert a0 % align == 0 or a0 == N
    if N % (world * align) == 0:
        assert len({b - a for a, b in bounds}) == 1


def test_shard_columns_rejects_bad_input():
    import qgemm._lib as L
    a, b = ctypes.c_int(), ctypes.c_int()
    assert L.lib().qgemm_shard_columns(100, 2, 2, 16, ctypes.byref(a), ctypes.byref(b)) == \
        L.ERR_INVALID_ARG
    assert L.lib().qgemm_shard_columns(100, 0, 0, 16, ctypes.byref(a), ctypes.byref(b)) == \
        L.ERR_INVALID_ARG


def test_by_name_rejects_unknown_without_a_stream():
    import qgemm._lib as L
    bufs = (ctypes.c_uint64 * 1)(0)
    ints = (ctypes.c_int * 1)(0)
    assert L.lib().qgemm_launch_by_name(None, b"noSuchKernel", bufs, 1, ints, 1) == \
        L.ERR_INVALID_ARG


def test_bridge_argument_errors_without_gpu():
    """The Java bridge's by-name form (CUDARuntimeJavaBridge.scala:121-165) answers -1, as
    the bridge's -1L, for a bad name, buffer count, scalar key or scalar value, before it
    touches a device; a valid request on a null stream fails on the handle."""
    import ctypes
    import qgemm._lib as L
    lib = L.lib()

    def launch(name, nbufs, vals, keys):
        bufs = (ctypes.c_uint64 * max(1, nbufs))(*([1] * nbufs))
        n = len(vals)
        v = (ctypes.c_float * max(1, n))(*vals)
        k = None if keys is None else (ctypes.c_char_p * max(1, n))(*[x.encode() for x in keys])
        return lib.qgemm_bridge_launch_kernel(None, name.encode(), 1, 1, 1, 1, 1, 1, bufs, nbufs,
                                              v if n else None, k, n)

    assert launch("noSuchKernel", 1, [], None) == -1
    assert "unknown kernel name" in L.last_error()
    assert launch("sgemm", 2, [4, 4, 4, 1, 0], None) == -1
    assert "takes 3 buffers" in L.last_error()
    assert launch("sgemm", 3, [4, 4, 4, 1, 0], ["M", "N", "K", "alpha", "gamma"]) == -1
    assert "no scalar 'gamma'" in L.last_error()
    assert launch("sgemm", 3, [4, 4, 4, 1, 0], ["M", "M", "K", "alpha", "beta"]) == -1
    assert "given twice" in L.last_error()
    assert launch("sgemm", 3, [4.5, 4, 4, 1, 0], None) == -1
    assert "exact Int" in L.last_error()
    assert launch("w8a16Gemm", 5, [4, 4, 4, 3], None) == -1
    assert "Bool" in L.last_error()
    assert launch("int8GemmKernel", 3, [4, 4, 4, 4, 4, 4, 1.0], None) == -1
    assert "missing" in L.last_error()
    # qBits of dynamicQuantize has a default (QuantizedGemmOps.scala:127): only the handle fails
    assert launch("dynamicQuantize", 3, [4, 4], ["K", "N"]) == -1
    assert "stream" in L.last_error()


def test_prefill_workspace_sizes_without_gpu():
    """Host-only sizing: the one-term workspace is half the exact one; unknown flags are
    refused."""
    import qgemm
    import qgemm._lib as L
    ops = qgemm.QuantizedGemmOps
    for K, N in ((4096, 22016), (11008, 4096), (1056, 520)):
        kp = (K + 63) // 64 * 64
        ncols = (N + 255) // 256 * 256
        assert ops.w4PrefillWorkspaceBytes(K, N) == ncols * kp * 4
        assert ops.w4PrefillWorkspaceBytes(K, N, one_term=True) == ncols * kp * 2
    n = ctypes.c_size_t(0)
    assert L.lib().qgemm_w4a16_prefill_workspace_bytes_ex(64, 64, 4, ctypes.byref(n)) == \
        L.ERR_INVALID_ARG
    assert L.lib().qgemm_w4a16_prefill_workspace_bytes_ex(64, 64, L.PREFILL_FRAG,
                                                          ctypes.byref(n)) == L.OK
    assert n.value == 256 * 64 * 4


def test_fused_gather_rejects_a_null_window_without_gpu():
    import qgemm._lib as L
    assert L.lib().qgemm_w8a8_gemm_allgather_fused_bf16(None, None, 16, 16, 0, 16, 16, 64, 64,
                                                         64) == L.ERR_BAD_HANDLE
