"""ctypes front end of the CPU oracle (oracle/qgemm_oracle.c).

TEST INFRASTRUCTURE ONLY.  tests/, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of bench.py import this module as
the checker or as the timed CPU restatement of the reference.  The product
path (libqgemm) never imports it and has no CPU fallback.

Parity status: UNPINNED -- the reference's operators
(src/main/scala/cuda/dsl/operators/linalg/QuantizedGemmOps.scala) have no
golden vectors or tests and cannot run here; the restatement is pinned by
hand-computed known answers and by an independent pure-Python restatement
(tests/golden/make_golden.py).
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")
_lib = None

_P = ctypes.c_void_p
_I = ctypes.c_int


def build(force: bool = False) -> str:
    """Compile liboracle.so with the committed Makefile (gcc, OpenMP)."""
    src = os.path.join(_HERE, "qgemm_oracle.c")
    if force or not os.path.exists(_LIB_PATH) or (
            os.path.getmtime(_LIB_PATH) < os.path.getmtime(src)):
        subprocess.run(["make", "-s", "-C", _HERE, "-B" if force else "liboracle.so"],
                       check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = ctypes.CDLL(_LIB_PATH)
        L.oracle_f32_to_bf16_rne.restype = ctypes.c_uint16
        L.oracle_f32_to_bf16_rne.argtypes = [ctypes.c_float]
        L.oracle_f32_to_bf16_trunc.restype = ctypes.c_uint16
        L.oracle_f32_to_bf16_trunc.argtypes = [ctypes.c_float]
        L.oracle_scala_f2i.restype = ctypes.c_int32
        L.oracle_scala_f2i.argtypes = [ctypes.c_float]
        L.oracle_w8a32_gemm.argtypes = [_P, _P, _P, _P, _P, _I, _I, _I, _P]
        L.oracle_w8a8_gemm_rows.argtypes = [_P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I]
        L.oracle_w4a16_gemm.argtypes = [_P, _P, _P, _P, _I, _I, _I]
        L.oracle_w4a16_grouped.argtypes = [_P, _P, _I, _I, _P, _P, _P, _I, _I, _I, _I, _I, _I]
        L.oracle_w8a16_gemm.argtypes = [_P, _P, _P, _P, _P, _I, _I, _I, _I]
        L.oracle_w8a16_gemm_rowwise.argtypes = [_P, _P, _P, _P, _I, _I, _I]
        L.oracle_dynamic_quantize.argtypes = [_P, _P, _P, _I, _I, _I]
        L.oracle_weight_only_quantize_per_channel.argtypes = [_P, _P, _P, _P, _I, _I]
        L.oracle_dequantize.argtypes = [_P, _P, _P, _I, _I]
        L.oracle_matmul_f32.argtypes = [_P, _P, _P, _P, _I, _I, _I, ctypes.c_float,
                                        ctypes.c_float, _I, _I]
        L.oracle_gemv_f32.argtypes = [_P, _P, _P, _I, _I]
        L.oracle_tensor_core_gemm_int8.argtypes = [_P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _I,
                                                   _I]
        L.oracle_int8_gemm_kernel.argtypes = [_P, _P, _P, _I, _I, _I, _I, _I, _I,
                                              ctypes.c_float, ctypes.c_float, _I]
        L.oracle_max_threads.restype = _I
        _lib = L
    return _lib


def _ptr(a: np.ndarray | None):
    if a is None:
        return None
    assert a.flags["C_CONTIGUOUS"], "oracle inputs must be C-contiguous"
    return a.ctypes.data_as(ctypes.c_void_p)


def _c(a, dtype):
    return np.ascontiguousarray(a, dtype=dtype)


def max_threads() -> int:
    return int(lib().oracle_max_threads())


# ---- scalar helpers ---------------------------------------------------------

def bf16_rne(a) -> np.ndarray:
    """float32 -> bf16 bits, round to nearest even (vectorised restatement of
    oracle_f32_to_bf16_rne; NaNs are quieted)."""
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32).astype(np.uint64)
    nan = ((u & 0x7F800000) == 0x7F800000) & ((u & 0x007FFFFF) != 0)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    r = np.where(nan, ((u >> 16) | 0x40).astype(np.uint16), r)
    return r.astype(np.uint16)


def bf16_to_f32(h) -> np.ndarray:
    return (np.ascontiguousarray(h, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16_scalar(f: float) -> int:
    return int(lib().oracle_f32_to_bf16_rne(f))


def scala_f2i(f: float) -> int:
    return int(lib().oracle_scala_f2i(f))


# ---- operators (QuantizedGemmOps.scala) -------------------------------------

def w8a32_gemm(wInt8, scalesW, x, scalesX):
    """QuantizedGemmOps.w8a32Gemm (:90-115).  Returns (y fp32 [M,N], acc int32 [M,N])."""
    w = _c(wInt8, np.int8); sw = _c(scalesW, np.float32)
    xx = _c(x, np.int8); sx = _c(scalesX, np.float32)
    M, K = xx.shape
    K2, N = w.shape
    assert K == K2 and sw.shape == (N,) and sx.shape == (M,)
    y = np.empty((M, N), np.float32)
    acc = np.empty((M, N), np.int32)
    lib().oracle_w8a32_gemm(_ptr(w), _ptr(sw), _ptr(xx), _ptr(sx), _ptr(y), M, N, K, _ptr(acc))
    return y, acc


def w8a8_gemm_rows(wInt8, scalesW, x, scalesX, m0=0, m1=None, threads=0,
                   want_f32=True, want_bf16=True, want_acc=False):
    """Rows [m0, m1) of the W8A8 GEMM (same arithmetic as w8a32_gemm, OpenMP).
    Returns (y fp32 [m1-m0, N] or None, y bf16 bits [m1-m0, N] or None), and the int32
    sums [m1-m0, N] as a third element when want_acc."""
    w = _c(wInt8, np.int8); sw = _c(scalesW, np.float32)
    xx = _c(x, np.int8); sx = _c(scalesX, np.float32)
    M, K = xx.shape
    N = w.shape[1]
    if m1 is None:
        m1 = M
    # The C routine indexes outputs by absolute row; hand it buffers that start at row 0.
    y = np.empty((M, N), np.float32) if want_f32 else None
    yb = np.empty((M, N), np.uint16) if want_bf16 else None
    acc = np.empty((M, N), np.int32) if want_acc else None
    lib().oracle_w8a8_gemm_rows(_ptr(w), _ptr(sw), _ptr(xx), _ptr(sx), _ptr(y), _ptr(yb),
                                _ptr(acc), M, N, K, m0, m1, threads)
    out = (y[m0:m1] if y is not None else None, yb[m0:m1] if yb is not None else None)
    return out + (acc[m0:m1],) if want_acc else out


def w4a16_gemm(wInt4, scalesW, x, N):
    """QuantizedGemmOps.w4a16Gemm (:218-247).  wInt4: uint8 bytes holding K*N nibbles."""
    w = _c(wInt4, np.uint8); sw = _c(scalesW, np.float32); xx = _c(x, np.float32)
    M, K = xx.shape
    assert w.size * 2 >= K * N
    y = np.empty((M, N), np.float32)
    lib().oracle_w4a16_gemm(_ptr(w), _ptr(sw), _ptr(xx), _ptr(y), M, N, K)
    return y


def w4a16_grouped(wq, scales, zero_point, group_size, x, n0=0, n1=None, threads=0):
    """Group-wise W4A16.  wq uint32 [K, N/8]; scales bf16 bits [ceil(K/G), N];
    x bf16 bits [M,K].  Returns (y fp32 [M, n1-n0], y bf16 bits [M, n1-n0])."""
    w = _c(wq, np.uint32); s = _c(scales, np.uint16); xx = _c(x, np.uint16)
    M, K = xx.shape
    N = s.shape[1]
    assert w.size * 8 >= K * N
    if n1 is None:
        n1 = N
    y = np.zeros((M, N), np.float32)
    yb = np.zeros((M, N), np.uint16)
    lib().oracle_w4a16_grouped(_ptr(w), _ptr(s), int(zero_point), int(group_size), _ptr(xx),
                               _ptr(y), _ptr(yb), M, N, K, n0, n1, threads)
    return y[:, n0:n1], yb[:, n0:n1]


def w8a16_gemm(wInt8, scalesW, x, bias=None):
    """QuantizedGemmOps.w8a16Gemm (:24-55)."""
    w = _c(wInt8, np.int8); sw = _c(scalesW, np.float32); xx = _c(x, np.float32)
    M, K = xx.shape
    N = w.shape[1]
    b = _c(bias, np.float32) if bias is not None else np.zeros(N, np.float32)
    y = np.empty((M, N), np.float32)
    lib().oracle_w8a16_gemm(_ptr(w), _ptr(sw), _ptr(xx), _ptr(b), _ptr(y), M, N, K,
                            1 if bias is not None else 0)
    return y


def w8a16_gemm_rowwise(wInt8, scalesW, x):
    """QuantizedGemmOps.w8a16GemmRowWise (:61-84); scalesW has K entries."""
    w = _c(wInt8, np.int8); sw = _c(scalesW, np.float32); xx = _c(x, np.float32)
    M, K = xx.shape
    N = w.shape[1]
    y = np.empty((M, N), np.float32)
    lib().oracle_w8a16_gemm_rowwise(_ptr(w), _ptr(sw), _ptr(xx), _ptr(y), M, N, K)
    return y


def dynamic_quantize(weight, qBits=8):
    """QuantizedGemmOps.dynamicQuantize (:121-157).  Returns (scales [N], q int8 [K,N])."""
    w = _c(weight, np.float32)
    K, N = w.shape
    s = np.empty(N, np.float32); q = np.empty((K, N), np.int8)
    lib().oracle_dynamic_quantize(_ptr(w), _ptr(s), _ptr(q), K, N, int(qBits))
    return s, q


def weight_only_quantize_per_channel(weight):
    """QuantizedGemmOps.weightOnlyQuantizePerChannel (:163-192).
    Returns (scales [N], q int8 [K,N], zeros int8 [N])."""
    w = _c(weight, np.float32)
    K, N = w.shape
    s = np.empty(N, np.float32); q = np.empty((K, N), np.int8); z = np.empty(N, np.int8)
    lib().oracle_weight_only_quantize_per_channel(_ptr(w), _ptr(s), _ptr(q), _ptr(z), K, N)
    return s, q, z


def dequantize(qWeight, scales):
    """QuantizedGemmOps.dequantize (:198-212)."""
    q = _c(qWeight, np.int8); s = _c(scales, np.float32)
    K, N = q.shape
    w = np.empty((K, N), np.float32)
    lib().oracle_dequantize(_ptr(q), _ptr(s), _ptr(w), K, N)
    return w


# ---- fp32 operators (MatrixOps.scala) ----------------------------------------

def matmul_f32(A, B, bias=None, C=None, alpha=1.0, beta=0.0, mode=0, threads=0):
    """MatrixOps.matmul (:16-28) / matmulAddBias (:31-44) / BLASOps.sgemm (:230-243).
    mode 0: A @ B; 1: A @ B + bias; 2: alpha * (A @ B) + beta * C (C is the input C)."""
    a = _c(A, np.float32); b = _c(B, np.float32)
    M, K = a.shape
    K2, N = b.shape
    assert K == K2
    out = np.array(C, dtype=np.float32, copy=True) if mode == 2 else np.empty((M, N), np.float32)
    assert out.shape == (M, N)
    bb = _c(bias, np.float32) if bias is not None else None
    lib().oracle_matmul_f32(_ptr(a), _ptr(b), _ptr(bb), _ptr(out), M, N, K, float(alpha),
                            float(beta), int(mode), int(threads))
    return out


def gemv_f32(A, x):
    """MatrixOps.gemv (:166-177): y = A x, A [M,N]."""
    a = _c(A, np.float32); xx = _c(x, np.float32)
    M, N = a.shape
    y = np.empty(M, np.float32)
    lib().oracle_gemv_f32(_ptr(a), _ptr(xx), _ptr(y), M, N)
    return y


# ---- the int8 GEMM names of TensorCoreOps / CutlassGemm ----------------------

def tensor_core_gemm_int8(a, b, c=None, *, M, N, K, lda=None, ldb=None, ldc=None, ldd=None):
    """TensorCoreOps.tensorCoreGemmInt8 (TensorCoreOps.scala:294-340), its arithmetic for
    every output: d = a @ b (+ c), int32 wrapping, through leading dimensions.  a int8
    with rows of lda, b int8 with rows of ldb, c int32 with rows of ldc (None: hasC
    false).  Returns d int32 [M, ldd] (columns past N zero)."""
    lda = K if lda is None else lda
    ldb = N if ldb is None else ldb
    ldd = N if ldd is None else ldd
    aa = _c(a, np.int8); bb = _c(b, np.int8)
    assert aa.size >= (M - 1) * lda + K if M and K else True
    assert bb.size >= (K - 1) * ldb + N if K and N else True
    cc = None
    if c is not None:
        ldc = N if ldc is None else ldc
        cc = _c(c, np.int32)
        assert cc.size >= (M - 1) * ldc + N if M and N else True
    d = np.zeros((M, ldd), np.int32)
    lib().oracle_tensor_core_gemm_int8(_ptr(aa), _ptr(bb), _ptr(cc), _ptr(d), M, N, K, lda, ldb,
                                       ldc or 0, ldd, 1 if c is not None else 0)
    return d


def int8_gemm_kernel(A, B, scaleA, scaleB, *, M, N, K, lda=None, ldb=None, ldd=None, threads=0):
    """CutlassGemm.int8GemmKernel (CutlassGemm.scala:987-1041) with one fp32 accumulator per
    output: A, B int32 arrays (rows of lda / ldb); returns D fp32 [M, ldd] (columns past N
    zero)."""
    lda = K if lda is None else lda
    ldb = N if ldb is None else ldb
    ldd = N if ldd is None else ldd
    aa = _c(A, np.int32); bb = _c(B, np.int32)
    D = np.zeros((M, ldd), np.float32)
    lib().oracle_int8_gemm_kernel(_ptr(D), _ptr(aa), _ptr(bb), M, N, K, lda, ldb, ldd,
                                  float(scaleA), float(scaleB), int(threads))
    return D
