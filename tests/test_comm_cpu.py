"""The host side of qgemm.NCCLCommunicator (nccl/NCCLCommunicator.scala:35-92 and
NCCLOps.ncclAllGather :302-320 for this path), without a GPU: the unique id, the
work-buffer size, and that every use of a missing or destroyed communicator or
window raises instead of falling back as the reference does."""
import pytest

import qgemm
import qgemm._lib as L
from qgemm import NCCLCommunicator, OutputWindow


def test_unique_id_is_128_fresh_bytes():
    a, b = NCCLCommunicator.unique_id(), NCCLCommunicator.unique_id()
    assert len(a) == len(b) == 128 and a != b


def test_work_bytes():
    assert NCCLCommunicator.gemmAllGatherWorkBytes(4, 2048, 7168) == 2 * 4 * 2048 * 7168 * 2
    assert NCCLCommunicator.gemmAllGatherWorkBytes(4, 0, 7168) == 0


def test_bad_unique_id_length():
    with pytest.raises(ValueError):
        NCCLCommunicator(None, 0, 2, b"short")


def test_destroyed_communicator_and_released_window_raise():
    import ctypes
    c = object.__new__(NCCLCommunicator)
    c.rank, c.worldSize, c.dev, c.handle = 0, 2, None, ctypes.c_void_p()
    assert not c.isNative() and c.getRank() == 0 and c.getWorldSize() == 2
    with pytest.raises(qgemm.QGemmError) as e:
        c.allGather(None, 0, 0, 1)
    assert e.value.status == L.ERR_BAD_HANDLE
    with pytest.raises(qgemm.QGemmError):
        c.registerWindow(None, 0, 16)
    c.destroy()  # nothing to destroy: no call, no error
    w = object.__new__(OutputWindow)
    w.comm, w.handle = c, ctypes.c_void_p()
    with pytest.raises(qgemm.QGemmError) as e:
        w.w8a8GemmAllGather(None, None, 0, 0, 0, 0, 16, 16, 16, 16)
    assert e.value.status == L.ERR_BAD_HANDLE
    w.release()


def test_null_handles_are_refused_by_the_library():
    """The C entry points themselves refuse null communicators and windows."""
    lib = L.lib()
    assert lib.qgemm_comm_window_release(None) == L.ERR_BAD_HANDLE
    assert lib.qgemm_w8a8_gemm_allgather_window_bf16(None, None, None, 0, 0, 0, 0, 0, 16, 16,
                                                     16, 16) == L.ERR_BAD_HANDLE
    assert lib.qgemm_w8a8_gemm_allgather_bf16(None, None, None, 0, 0, 0, 0, 0, 0, 16, 16, 16, 16,
                                              0, 0) == L.ERR_BAD_HANDLE
