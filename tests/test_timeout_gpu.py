"""The bounded-wait error path on the GPU, made to run out on purpose without a fault.

The W8A8 GEMM's last-wave split has the final K part of each leftover tile wait,
bounded, for the other parts' count-ins.  With the test hook qgemm_debug_hold_split the
final part waits for one count-in more than ever arrives (a flag nothing sets), under a
20 ms device wait limit: the kernel gives up, records the timeout in the device error
word and ends; qgemm_stream_sync() reports QGEMM_ERR_TIMEOUT and clears the word and the
split counters.  The same stream then runs the same GEMM correctly."""
import numpy as np
import pytest

import qgemm
import qgemm.synthetic as syn
from helpers import Out, dev_array

pytestmark = pytest.mark.gpu


def test_split_wait_runs_out_then_stream_recovers(gpu, oracle):
    dev, st, ops = gpu
    # 240 pair tiles on 74 CTA pairs: 18 leftover tiles cut into 4 K parts each
    M, N, K = 3840, 4096, 1024
    A, B, sA, sB = syn.w8a8_inputs(M, N, K, seed=77)
    dA, dB, dsA, dsB = (dev_array(gpu, a) for a in (A, B, sA, sB))
    y = Out(dev, st, M * N * 2)
    acc = Out(dev, st, M * N * 4)
    st.sync()
    old = dev.wait_limit_ns
    assert old == 2_000_000_000
    dev.wait_limit_ns = 20_000_000
    dev.debug_hold_split(True)
    try:
        ops.w8a8Gemm(dA, dB, dsA, dsB, y, M, N, K, acc_i32=acc, algo=qgemm.ALGO_TCGEN05)
        with pytest.raises(qgemm.QGemmError) as e:
            st.sync()
        assert e.value.status == qgemm._lib.ERR_TIMEOUT
    finally:
        dev.debug_hold_split(False)
        dev.wait_limit_ns = old
    st.sync()  # the error word was cleared: nothing left to report
    # the same stream, the same split shape, a correct result
    ops.w8a8Gemm(dA, dB, dsA, dsB, y, M, N, K, acc_i32=acc, algo=qgemm.ALGO_TCGEN05)
    st.sync()
    got_acc = acc.read(np.int32, (M, N))
    got_y = y.read(np.uint16, (M, N))
    rows = np.unique(np.concatenate([np.random.default_rng(3).choice(M, 16, replace=False),
                                     [0, M - 1]]))
    _, yb, acc_o = oracle.w8a8_gemm_rows(B, sB, A[rows], sA[rows], want_f32=False, want_acc=True)
    np.testing.assert_array_equal(got_acc[rows], acc_o)
    np.testing.assert_array_equal(got_y[rows], yb)
    # the leftover tiles (the last 256-row block) in full against the CUDA-core kernel
    ys = Out(dev, st, M * N * 2)
    accs = Out(dev, st, M * N * 4)
    ops.w8a8Gemm(dA, dB, dsA, dsB, ys, M, N, K, acc_i32=accs, algo=qgemm.ALGO_SIMT)
    st.sync()
    np.testing.assert_array_equal(got_acc, accs.read(np.int32, (M, N)))
    np.testing.assert_array_equal(got_y, ys.read(np.uint16, (M, N)))


def test_wait_limit_range(gpu):
    dev, _, _ = gpu
    with pytest.raises(qgemm.QGemmError):
        dev.wait_limit_ns = 10
    with pytest.raises(qgemm.QGemmError):
        dev.wait_limit_ns = 120 * 10**9
    assert dev.wait_limit_ns == 2_000_000_000
