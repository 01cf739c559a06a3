"""QuantizedGemmOps -- the reference operator object, backed by libqgemm.

Mirrors ``object QuantizedGemmOps`` of
src/main/scala/cuda/dsl/operators/linalg/QuantizedGemmOps.scala:17-247: the same
method names, the same parameter order and meaning (``Ptr[T]`` arguments are
device addresses -- ints, objects with ``.address`` such as qgemm.Buffer, or
torch CUDA tensors -- followed by the Int sizes).  Each call is one
asynchronous launch on the object's stream.

Error behaviour: the reference swallows native errors and prints them
(runtime/CUDARuntime.scala:216,256,294); here every failure raises
``QGemmError`` carrying the library status and message.
"""
from __future__ import annotations

import ctypes

from . import _lib as L


class QuantizedGemmOps:
    def __init__(self, stream):
        self.stream = stream
        self._h = stream.handle

    # -- QuantizedGemmOps.scala:24-55
    def w8a16Gemm(self, wInt8, scalesW, x, bias, y, M: int, N: int, K: int, hasBias: bool):
        L.call("qgemm_w8a16_gemm", self._h, L.addr(wInt8), L.addr(scalesW), L.addr(x),
               L.addr(bias), L.addr(y), M, N, K, 1 if hasBias else 0)

    # -- QuantizedGemmOps.scala:61-84
    def w8a16GemmRowWise(self, wInt8, scalesW, x, y, M: int, N: int, K: int):
        L.call("qgemm_w8a16_gemm_rowwise", self._h, L.addr(wInt8), L.addr(scalesW), L.addr(x),
               L.addr(y), M, N, K)

    # -- QuantizedGemmOps.scala:90-115
    def w8a32Gemm(self, wInt8, scalesW, x, scalesX, y, M: int, N: int, K: int):
        L.call("qgemm_w8a32_gemm", self._h, L.addr(wInt8), L.addr(scalesW), L.addr(x),
               L.addr(scalesX), L.addr(y), M, N, K)

    # -- QuantizedGemmOps.scala:121-157
    def dynamicQuantize(self, weight, scales, qWeight, K: int, N: int, qBits: int = 8):
        L.call("qgemm_dynamic_quantize", self._h, L.addr(weight), L.addr(scales),
               L.addr(qWeight), K, N, qBits)

    # -- QuantizedGemmOps.scala:163-192
    def weightOnlyQuantizePerChannel(self, weight, scales, qWeight, zeros, K: int, N: int):
        L.call("qgemm_weight_only_quantize_per_channel", self._h, L.addr(weight),
               L.addr(scales), L.addr(qWeight), L.addr(zeros), K, N)

    # -- QuantizedGemmOps.scala:198-212
    def dequantize(self, qWeight, scales, weight, K: int, N: int):
        L.call("qgemm_dequantize", self._h, L.addr(qWeight), L.addr(scales), L.addr(weight), K, N)

    # -- QuantizedGemmOps.scala:218-247
    def w4a16Gemm(self, wInt4, scalesW, x, y, M: int, N: int, K: int):
        L.call("qgemm_w4a16_gemm", self._h, L.addr(wInt4), L.addr(scalesW), L.addr(x),
               L.addr(y), M, N, K)

    # -- B200 entry points behind the same object ------------------------------

    def w8a8Gemm(self, A, B, sA, sB, out, M: int, N: int, K: int, *, b_layout: int = L.B_KN,
                 out_dtype: int = L.BF16, ldc: int | None = None, acc_i32=None,
                 algo: int = L.ALGO_AUTO):
        """W8A8 with per-token sA [M] x per-channel sB [N] dequant (the w8a32Gemm
        arithmetic), bf16 (RNE) or fp32 output, optional int32 accumulators."""
        L.call("qgemm_w8a8_gemm", self._h, L.addr(A), L.addr(B), b_layout, L.addr(sA),
               L.addr(sB), L.addr(out), out_dtype, N if ldc is None else ldc, M, N, K,
               L.addr(acc_i32), algo)

    def w8a8GemmStaticScratch(self, A, B, sA, sB, out, M: int, N: int, K: int, *,
                              b_layout: int = L.B_KN, out_dtype: int = L.BF16,
                              ldc: int | None = None, acc_i32=None, algo: int = L.ALGO_AUTO):
        """w8a8Gemm that never allocates: its split scratch is a static device array."""
        L.call("qgemm_w8a8_gemm_static_scratch", self._h, L.addr(A), L.addr(B), b_layout,
               L.addr(sA), L.addr(sB), L.addr(out), out_dtype, N if ldc is None else ldc, M, N,
               K, L.addr(acc_i32), algo)

    def w4a16GemmGrouped(self, x, wq, scales, y, M: int, N: int, K: int, *,
                         zero_point: int = 8, group_size: int = 128):
        """Group-wise W4A16: x bf16 [M,K], wq uint32 [K,N/8] (reference nibble order),
        scales bf16 [K/group_size, N], y bf16 [M,N]."""
        L.call("qgemm_w4a16_grouped_gemm", self._h, L.addr(x), L.addr(wq), L.addr(scales),
               zero_point, group_size, L.addr(y), M, N, K)

    def w4a16GemmGroupedTiled(self, x, wt, scales, y, M: int, N: int, K: int, *,
                              zero_point: int = 8, group_size: int = 128):
        """Group-wise W4A16 on weights prepacked by prepackW4Tiled (the fast decode path)."""
        L.call("qgemm_w4a16_grouped_gemm_tiled", self._h, L.addr(x), L.addr(wt), L.addr(scales),
               zero_point, group_size, L.addr(y), M, N, K)

    def w4a16GemmGroupedFrag(self, x, wf, scales, y, M: int, N: int, K: int, *,
                             zero_point: int = 8, group_size: int = 128):
        """Group-wise W4A16 on weights prepacked by prepackW4Frag (the fast decode path:
        8-column groups for M <= 4, 16-column pairs in 16-row passes above)."""
        L.call("qgemm_w4a16_grouped_gemm_frag", self._h, L.addr(x), L.addr(wf), L.addr(scales),
               zero_point, group_size, L.addr(y), M, N, K)

    @staticmethod
    def w4PrefillWorkspaceBytes(K: int, N: int, *, one_term: bool = False) -> int:
        """Workspace that holds all of N in one slab: two bf16 terms per weight (exact),
        or one with one_term."""
        n = ctypes.c_size_t(0)
        if one_term:
            L.call("qgemm_w4a16_prefill_workspace_bytes_ex", K, N, L.PREFILL_ONE_TERM,
                   ctypes.byref(n))
        else:
            L.call("qgemm_w4a16_prefill_workspace_bytes", K, N, ctypes.byref(n))
        return n.value

    def w4a16GemmGroupedPrefill(self, x, wt, scales, y, M: int, N: int, K: int, workspace,
                                workspace_bytes: int, *, zero_point: int = 8,
                                group_size: int = 128, one_term: bool = False):
        """Group-wise W4A16 for prefill-sized M on prepackW4Tiled weights: bf16 slabs
        expanded in `workspace`, then the tensor-core bf16 GEMM.  Exact by default: q - zp
        in the slab and the group scales applied in fp32 to each group's partial sums
        (group_size a multiple of 64, 16-byte aligned scales), else hi + lo per weight;
        with one_term, bf16((q - zp) * s) alone (relative weight error <= 2^-9)."""
        if one_term:
            L.call("qgemm_w4a16_grouped_gemm_prefill_ex", self._h, L.addr(x), L.addr(wt),
                   L.addr(scales), zero_point, group_size, L.addr(y), M, N, K,
                   L.addr(workspace), workspace_bytes, L.PREFILL_ONE_TERM)
        else:
            L.call("qgemm_w4a16_grouped_gemm_prefill", self._h, L.addr(x), L.addr(wt),
                   L.addr(scales), zero_point, group_size, L.addr(y), M, N, K,
                   L.addr(workspace), workspace_bytes)

    def w4a16GemmGroupedPrefillFrag(self, x, wf, scales, y, M: int, N: int, K: int, workspace,
                                    workspace_bytes: int, *, zero_point: int = 8,
                                    group_size: int = 128, one_term: bool = False):
        """The prefill GEMM on prepackW4Frag weights (one weight copy for prefill and
        decode); one_term as in w4a16GemmGroupedPrefill."""
        if one_term:
            L.call("qgemm_w4a16_grouped_gemm_prefill_ex", self._h, L.addr(x), L.addr(wf),
                   L.addr(scales), zero_point, group_size, L.addr(y), M, N, K,
                   L.addr(workspace), workspace_bytes, L.PREFILL_FRAG | L.PREFILL_ONE_TERM)
        else:
            L.call("qgemm_w4a16_grouped_gemm_prefill_frag", self._h, L.addr(x), L.addr(wf),
                   L.addr(scales), zero_point, group_size, L.addr(y), M, N, K,
                   L.addr(workspace), workspace_bytes)

    def gemmBf16NK(self, A, B, out, M: int, N: int, K: int, *, ldc: int | None = None):
        """out[M, ldc] bf16 = A[M,K] (bf16) x B[N,K]^T (bf16), fp32 sums."""
        L.call("qgemm_gemm_bf16_nk", self._h, L.addr(A), L.addr(B), L.addr(out),
               N if ldc is None else ldc, M, N, K)

    @staticmethod
    def w4TiledBytes(K: int, N: int) -> int:
        n = ctypes.c_size_t(0)
        L.call("qgemm_w4_tiled_bytes", K, N, ctypes.byref(n))
        return n.value

    def prepackW4Tiled(self, wq, dst, K: int, N: int):
        """uint32 [K, N/8] reference-order int4 weights -> 64-column tiles (one time)."""
        L.call("qgemm_prepack_w4_tiled", self._h, L.addr(wq), L.addr(dst), K, N)

    @staticmethod
    def w4FragBytes(K: int, N: int) -> int:
        n = ctypes.c_size_t(0)
        L.call("qgemm_w4_frag_bytes", K, N, ctypes.byref(n))
        return n.value

    def prepackW4Frag(self, wq, dst, K: int, N: int):
        """uint32 [K, N/8] reference-order int4 weights -> fragment order (one time)."""
        L.call("qgemm_prepack_w4_frag", self._h, L.addr(wq), L.addr(dst), K, N)

    def quantizePerToken(self, x, q, sA, M: int, K: int, *, in_dtype: int = L.BF16):
        """dynamicQuantize along rows: x [M,K] (bf16 or fp32) -> int8 q [M,K], sA [M]."""
        L.call("qgemm_quantize_per_token", self._h, L.addr(x), in_dtype, L.addr(q), L.addr(sA),
               M, K)

    def prepackW8NK(self, src_kn, dst_nk, K: int, N: int):
        L.call("qgemm_prepack_w8_nk", self._h, L.addr(src_kn), L.addr(dst_nk), K, N)

    # -- by-name launch (dsl/TritonKernelRunner.scala:68-73) --------------------

    def launchKernel(self, name: str, buffers, ints):
        bufs = (ctypes.c_uint64 * max(1, len(buffers)))(*[L.addr(b) for b in buffers])
        iv = (ctypes.c_int * max(1, len(ints)))(*[int(i) for i in ints])
        L.call("qgemm_launch_by_name", self._h, name.encode(), bufs, len(buffers), iv, len(ints))


class CUDARuntimeJavaBridge:
    """``CUDARuntimeJavaBridge.launchKernel`` (driver/CUDARuntimeJavaBridge.scala:121-165):
    launch by name with the result buffer first in ``bufferAddrs`` and Float scalars named
    by ``scalarKeys`` (or positional when keys are None).  Returns the result buffer's
    address, or -1 on failure, as the bridge does; ``last_error()`` then says why."""

    def __init__(self, stream):
        self.stream = stream
        self._h = stream.handle

    def launchKernel(self, name: str, gridX: int, gridY: int, gridZ: int, blockX: int,
                     blockY: int, blockZ: int, bufferAddrs, scalarVals=None,
                     scalarKeys=None) -> int:
        bufs = (ctypes.c_uint64 * max(1, len(bufferAddrs)))(*[L.addr(b) for b in bufferAddrs])
        n = 0 if scalarVals is None else len(scalarVals)
        vals = (ctypes.c_float * max(1, n))(*[float(v) for v in (scalarVals or [])])
        keys = None
        if scalarKeys is not None:
            if len(scalarKeys) != n:
                raise ValueError("scalarKeys and scalarVals differ in length")
            keys = (ctypes.c_char_p * max(1, n))(*[k.encode() for k in scalarKeys])
        return int(L.lib().qgemm_bridge_launch_kernel(
            self._h, name.encode(), gridX, gridY, gridZ, blockX, blockY, blockZ, bufs,
            len(bufferAddrs), vals if n else None, keys, n))


class TensorCoreOps:
    """``TensorCoreOps.tensorCoreGemmInt8`` (operators/intrinsic/TensorCoreOps.scala:294-340):
    same parameters; d = a x b (+ c) with int32 sums, on the W8A8 tensor-core kernel."""

    def __init__(self, stream):
        self.stream = stream
        self._h = stream.handle

    def tensorCoreGemmInt8(self, a, b, scalesA, scalesB, c, d, M: int, N: int, K: int,
                           lda: int, ldb: int, ldc: int, ldd: int, hasC: bool):
        L.call("qgemm_tensor_core_gemm_int8", self._h, L.addr(a), L.addr(b), L.addr(scalesA),
               L.addr(scalesB), L.addr(c), L.addr(d), M, N, K, lda, ldb, ldc, ldd,
               1 if hasC else 0)


class CutlassGemm:
    """``CutlassGemm.int8GemmKernel`` (cutlass/CutlassGemm.scala:987-1041): same parameters;
    D = (A x B) * scaleA * scaleB for int8 values held in Int arrays."""

    def __init__(self, stream):
        self.stream = stream
        self._h = stream.handle

    def int8GemmKernel(self, D, A, B, M: int, N: int, K: int, lda: int, ldb: int, ldd: int,
                       scaleA: float, scaleB: float):
        L.call("qgemm_int8_gemm_kernel", self._h, L.addr(D), L.addr(A), L.addr(B), M, N, K,
               lda, ldb, ldd, float(scaleA), float(scaleB))


class MatrixOps:
    """The fp32 entry points of ``object MatrixOps``
    (src/main/scala/cuda/dsl/operators/linalg/MatrixOps.scala): same names, parameter
    order and meaning.  The GEMMs run as three tf32 tensor-core products per fp32
    product with fp32 sums (|C - exact| <= 1e-5 * sum_k |A_ik * B_kj|)."""

    def __init__(self, stream):
        self.stream = stream
        self._h = stream.handle

    # -- MatrixOps.scala:16-28
    def matmul(self, A, B, C, M: int, N: int, K: int):
        L.call("qgemm_matmul_f32", self._h, L.addr(A), L.addr(B), L.addr(C), M, N, K)

    # -- MatrixOps.scala:31-44
    def matmulAddBias(self, A, B, bias, C, M: int, N: int, K: int):
        L.call("qgemm_matmul_add_bias_f32", self._h, L.addr(A), L.addr(B), L.addr(bias),
               L.addr(C), M, N, K)

    def gemmF32(self, A, B, C, M: int, N: int, K: int, *, bias=None, alpha: float = 1.0,
                beta: float = 0.0, mode: int = 0, algo: int = L.ALGO_AUTO):
        """The general form behind matmul / matmulAddBias / sgemm: mode 0, 1, 2 and a
        path choice (ALGO_TCGEN05: tensor cores, ALGO_SIMT: CUDA cores)."""
        L.call("qgemm_gemm_f32", self._h, L.addr(A), L.addr(B), L.addr(bias), L.addr(C), M, N,
               K, float(alpha), float(beta), int(mode), int(algo))

    # -- MatrixOps.scala:166-177
    def gemv(self, A, x, y, M: int, N: int):
        L.call("qgemm_gemv_f32", self._h, L.addr(A), L.addr(x), L.addr(y), M, N)


class BLASOps:
    """``object BLASOps`` (MatrixOps.scala:227+): sgemm on the same tensor-core path."""

    def __init__(self, stream):
        self.stream = stream
        self._h = stream.handle

    # -- MatrixOps.scala:230-243: C = alpha * (A x B) + beta * C (C always read)
    def sgemm(self, A, B, C, M: int, N: int, K: int, alpha: float, beta: float):
        L.call("qgemm_sgemm", self._h, L.addr(A), L.addr(B), L.addr(C), M, N, K,
               float(alpha), float(beta))


def shard_columns(N: int, world: int, rank: int, align: int = 256) -> tuple[int, int]:
    """Column range [n0, n1) of rank ``rank`` for an N-column weight split into
    ``world`` contiguous slices whose boundaries are multiples of ``align``."""
    a, b = ctypes.c_int(), ctypes.c_int()
    L.call("qgemm_shard_columns", N, world, rank, align, ctypes.byref(a), ctypes.byref(b))
    return a.value, b.value
