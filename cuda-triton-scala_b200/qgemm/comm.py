"""The column-sharded W8A8 layer's communicator, over libqgemm's NCCL entry points.

Mirrors nccl/NCCLCommunicator.scala (class NCCLCommunicator :35-77: rank, world
size, getRank / getWorldSize / isNative / barrier) and NCCLOps.ncclAllGather
(:302-320) for this path, with two differences a caller sees:

* the reference calls ncclGetUniqueId on every rank, so its ranks never share an
  id; here rank 0 makes the id (``NCCLCommunicator.unique_id()``) and the caller
  carries the 128 bytes to the other ranks (a torch.distributed broadcast, a
  file, a queue);
* the reference swallows NCCL errors and falls back to a host copy; here every
  failure raises QGemmError and nothing falls back.

Buffers are device addresses (ints) or objects with ``address`` / ``data_ptr()``.
Every rank must make the same calls in the same order.
"""
from __future__ import annotations

import ctypes

from . import _lib as L
from ._lib import B_KN


class NCCLCommunicator:
    """One rank of a communicator on ``dev`` (a qgemm.Device)."""

    @staticmethod
    def unique_id() -> bytes:
        """A fresh 128-byte NCCL unique id (made once, on rank 0)."""
        buf = ctypes.create_string_buffer(128)
        L.call("qgemm_comm_unique_id", buf)
        return bytes(buf.raw)

    def __init__(self, dev, rank: int, world_size: int, uid: bytes):
        if len(uid) != 128:
            raise ValueError("the unique id is 128 bytes")
        self.rank, self.worldSize, self.dev = rank, world_size, dev
        self.handle = ctypes.c_void_p()
        L.call("qgemm_comm_init", dev.handle, ctypes.create_string_buffer(uid, 128), rank,
               world_size, ctypes.byref(self.handle))

    def getRank(self) -> int:
        return self.rank

    def getWorldSize(self) -> int:
        return self.worldSize

    def isNative(self) -> bool:
        return bool(self.handle)

    def allGather(self, stream, send, recv, count: int) -> None:
        """bf16 all-gather of ``count`` elements per rank into recv [world][count]
        on ``stream`` (send may be recv + rank * count: in place)."""
        L.call("qgemm_comm_allgather_bf16", self._h(), stream.handle, L.addr(send),
               L.addr(recv), count)

    def unshardColumns(self, stream, gathered, out, M: int, ncols: int) -> None:
        """[world][M][ncols] bf16 -> [M][world * ncols]."""
        L.call("qgemm_unshard_columns_bf16", stream.handle, L.addr(gathered), L.addr(out),
               self.worldSize, M, ncols)

    @staticmethod
    def gemmAllGatherWorkBytes(world: int, chunk_rows: int, n_local: int) -> int:
        return int(L.lib().qgemm_w8a8_allgather_work_bytes(world, chunk_rows, n_local))

    def w8a8GemmAllGather(self, s, cs, A, B, sA, sB, out, M: int, n_local: int, K: int,
                          chunk_rows: int, work, work_bytes: int, b_layout: int = B_KN) -> None:
        """This rank's W8A8 columns (B [K, n_local], sB [n_local]) for the whole A [M, K],
        gathered to out [M, n_local * world] bf16 on every rank, chunk by chunk of
        ``chunk_rows`` rows: GEMMs on stream s, NCCL gathers and unshards on stream cs."""
        L.call("qgemm_w8a8_gemm_allgather_bf16", self._h(), s.handle, cs.handle, L.addr(A),
               L.addr(B), b_layout, L.addr(sA), L.addr(sB), L.addr(out), M, n_local, K,
               chunk_rows, L.addr(work), work_bytes)

    def registerWindow(self, stream, buf, nbytes: int) -> "OutputWindow":
        """Registers this rank's output buffer (collective; same size on every rank)."""
        return OutputWindow(self, stream, buf, nbytes)

    def destroy(self) -> None:
        if self.handle:
            L.call("qgemm_comm_destroy", self.handle)
            self.handle = ctypes.c_void_p()

    def _h(self):
        if not self.handle:
            raise L.QGemmError(L.ERR_BAD_HANDLE, "NCCLCommunicator", "destroyed communicator")
        return self.handle

    def __repr__(self) -> str:
        return (f"NCCLCommunicator(rank={self.rank}, world={self.worldSize}, "
                f"native={self.isNative()})")


class OutputWindow:
    """An [M, N] bf16 output buffer registered by every rank: the peers' copies of it
    are mapped into this process, and the GEMM's columns reach them by copy-engine
    copies, in the final layout."""

    def __init__(self, comm: NCCLCommunicator, stream, buf, nbytes: int):
        self.comm = comm
        self.handle = ctypes.c_void_p()
        L.call("qgemm_comm_window_register", comm._h(), stream.handle, L.addr(buf), nbytes,
               ctypes.byref(self.handle))

    def w8a8GemmAllGather(self, s, cs, A, B, sA, sB, M: int, n_local: int, K: int,
                          chunk_rows: int, b_layout: int = B_KN) -> None:
        if not self.handle:
            raise L.QGemmError(L.ERR_BAD_HANDLE, "OutputWindow", "released window")
        L.call("qgemm_w8a8_gemm_allgather_window_bf16", self.handle, s.handle, cs.handle,
               L.addr(A), L.addr(B), b_layout, L.addr(sA), L.addr(sB), M, n_local, K,
               chunk_rows)

    def w8a8GemmAllGatherFused(self, s, A, B, sA, sB, M: int, n_local: int, K: int,
                               b_layout: int = B_KN) -> None:
        """The GEMM and the gather as one kernel: its epilogue stores each output chunk
        into every rank's window (TMA stores over NVLink)."""
        if not self.handle:
            raise L.QGemmError(L.ERR_BAD_HANDLE, "OutputWindow", "released window")
        L.call("qgemm_w8a8_gemm_allgather_fused_bf16", self.handle, s.handle, L.addr(A),
               L.addr(B), b_layout, L.addr(sA), L.addr(sB), M, n_local, K)

    def release(self) -> None:
        """Local; call once every rank has finished with the window."""
        if self.handle:
            L.call("qgemm_comm_window_release", self.handle)
            self.handle = ctypes.c_void_p()
