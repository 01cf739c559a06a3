"""qgemm_w8a8_gemm_static_scratch: the W8A8 GEMM whose last-wave split takes its
scratch from a static device array.  It must give the same bits as qgemm_w8a8_gemm,
twice in a row (its counters are cleared per call), and allocate nothing."""
import numpy as np
import pytest

import qgemm
import qgemm.synthetic as syn
from helpers import Out, dev_array

pytestmark = pytest.mark.gpu


def gemm(gpu, fn, A, B, sA, sB, M, N, K, layout):
    dev, st, _ = gpu
    Bd = dev_array(gpu, B if layout == qgemm.B_KN else np.ascontiguousarray(B.T))
    y = Out(dev, st, M * N * 2)
    acc = Out(dev, st, M * N * 4)
    fn(dev_array(gpu, A), Bd, dev_array(gpu, sA), dev_array(gpu, sB), y, M, N, K,
       b_layout=layout, acc_i32=acc, algo=qgemm.ALGO_TCGEN05)
    st.sync()
    return y.read(np.uint16, (M, N)).copy(), acc.read(np.int32, (M, N)).copy()


@pytest.mark.parametrize("M,N,K,layout", [
    (3840, 1280, 1024, qgemm.B_KN),   # 75 pair tiles: the leftover tile is split in 4
    (3840, 1536, 1024, qgemm.B_NK),   # 90 pair tiles: 16 leftover tiles split in 4
    (4096, 4096, 512, qgemm.B_KN),    # no split (34 leftover tiles as column halves)
    (200, 512, 256, qgemm.B_NK),      # 1-CTA tiles
])
def test_static_scratch_matches_default_twice(gpu, M, N, K, layout):
    _, _, ops = gpu
    A, B, sA, sB = syn.w8a8_inputs(M, N, K, seed=M * 3 + N + K)
    y0, a0 = gemm(gpu, ops.w8a8Gemm, A, B, sA, sB, M, N, K, layout)
    for _ in range(2):
        y, a = gemm(gpu, ops.w8a8GemmStaticScratch, A, B, sA, sB, M, N, K, layout)
        np.testing.assert_array_equal(a, a0)
        np.testing.assert_array_equal(y, y0)


def test_static_scratch_allocates_nothing(gpu):
    """On a fresh stream handle, after a first call (which may load the library's device
    code), two more calls of a splitting shape leave the device's free memory unchanged."""
    dev, st, _ = gpu
    M, N, K = 3840, 1280, 1024
    A, B, sA, sB = syn.w8a8_inputs(M, N, K, seed=5)
    Ad, Bd, sAd, sBd = (dev_array(gpu, a) for a in (A, B, sA, sB))
    y = Out(dev, st, M * N * 2)
    st2 = dev.stream()
    ops2 = qgemm.QuantizedGemmOps(st2)
    try:
        ops2.w8a8GemmStaticScratch(Ad, Bd, sAd, sBd, y, M, N, K, algo=qgemm.ALGO_TCGEN05)
        st2.sync()
        import torch
        free0, _ = torch.cuda.mem_get_info(0)
        for _ in range(2):
            ops2.w8a8GemmStaticScratch(Ad, Bd, sAd, sBd, y, M, N, K, algo=qgemm.ALGO_TCGEN05)
        st2.sync()
        free1, _ = torch.cuda.mem_get_info(0)
        assert free1 == free0
    finally:
        st2.destroy()
