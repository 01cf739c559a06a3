"""qgemm -- host-side mirror of the reference's quantized-matmul operator API
over libqgemm.so, the B200 (sm_100a) C-ABI library.

    from qgemm import Device, QuantizedGemmOps
    dev = Device(0); st = dev.stream(); ops = QuantizedGemmOps(st)
    ops.w8a32Gemm(wInt8, scalesW, x, scalesX, y, M, N, K)   # reference signature
"""
from ._lib import (ALGO_AUTO, ALGO_SIMT, ALGO_TCGEN05, B_KN, B_NK, BF16, F32, QGemmError,
                   last_error, lib, status_name)
from .comm import NCCLCommunicator, OutputWindow
from .ops import (BLASOps, CUDARuntimeJavaBridge, CutlassGemm, MatrixOps, QuantizedGemmOps,
                  TensorCoreOps, shard_columns)
from .runtime import Buffer, Device, Stream, device_count

__all__ = [
    "ALGO_AUTO", "ALGO_SIMT", "ALGO_TCGEN05", "B_KN", "B_NK", "BF16", "F32", "QGemmError",
    "last_error", "lib", "status_name", "BLASOps", "CUDARuntimeJavaBridge", "CutlassGemm",
    "MatrixOps", "QuantizedGemmOps", "TensorCoreOps", "shard_columns", "Buffer", "Device",
    "Stream", "device_count", "NCCLCommunicator", "OutputWindow",
]
