"""W8A8 GEMM on the GPU against the CPU oracle (QuantizedGemmOps.w8a32Gemm,
QuantizedGemmOps.scala:90-115).  Integer accumulators must be bit-exact, and so
must the fp32 and bf16 outputs (the epilogue repeats the reference's two
roundings in order; bf16 is RNE of that fp32 value)."""
import numpy as np
import pytest

import qgemm
import qgemm.synthetic as syn
from helpers import Out, dev_array

pytestmark = pytest.mark.gpu


def run(gpu, A, B, sA, sB, *, layout=qgemm.B_KN, out_dtype=qgemm.BF16, algo=qgemm.ALGO_AUTO,
        ldc=None, acc=True):
    dev, st, ops = gpu
    M, K = A.shape
    N = B.shape[1]
    ldc = N if ldc is None else ldc
    Bd = dev_array(gpu, B if layout == qgemm.B_KN else np.ascontiguousarray(B.T))
    Ad, sAd, sBd = dev_array(gpu, A), dev_array(gpu, sA), dev_array(gpu, sB)
    esize = 2 if out_dtype == qgemm.BF16 else 4
    out = Out(dev, st, M * ldc * esize)
    accb = Out(dev, st, M * N * 4) if acc else None
    ops.w8a8Gemm(Ad, Bd, sAd, sBd, out, M, N, K, b_layout=layout, out_dtype=out_dtype, ldc=ldc,
                 acc_i32=accb, algo=algo)
    st.sync()
    y = out.read(np.uint16 if out_dtype == qgemm.BF16 else np.float32, (M, ldc))[:, :N]
    a = accb.read(np.int32, (M, N)) if acc else None
    return y, a


def check_exact(oracle, A, B, sA, sB, y, acc, out_dtype, rows=None):
    rows = np.arange(A.shape[0]) if rows is None else rows
    yo, acco = oracle.w8a32_gemm(B, sB, A[rows], sA[rows])
    if acc is not None:
        np.testing.assert_array_equal(acc[rows], acco)
    if out_dtype == qgemm.BF16:
        np.testing.assert_array_equal(y[rows], oracle.bf16_rne(yo))
    else:
        np.testing.assert_array_equal(y[rows].view(np.uint32), yo.view(np.uint32))


def test_reference_entry_point_config1(gpu, oracle):
    """w8a32Gemm with the reference signature at 64x512x512, fp32 output."""
    dev, st, ops = gpu
    A, B, sA, sB = syn.w8a8_inputs(64, 512, 512, seed=11)
    d = [dev_array(gpu, a) for a in (B, sB, A, sA)]
    y = Out(dev, st, 64 * 512 * 4)
    ops.w8a32Gemm(d[0], d[1], d[2], d[3], y, 64, 512, 512)
    st.sync()
    yo, _ = oracle.w8a32_gemm(B, sB, A, sA)
    np.testing.assert_array_equal(y.read(np.uint32, (64, 512)), yo.view(np.uint32))


@pytest.mark.parametrize("layout", [qgemm.B_KN, qgemm.B_NK])
@pytest.mark.parametrize("out_dtype", [qgemm.F32, qgemm.BF16])
def test_tcgen05_config1(gpu, oracle, layout, out_dtype):
    A, B, sA, sB = syn.w8a8_inputs(64, 512, 512, seed=12)
    y, acc = run(gpu, A, B, sA, sB, layout=layout, out_dtype=out_dtype, algo=qgemm.ALGO_TCGEN05)
    check_exact(oracle, A, B, sA, sB, y, acc, out_dtype)


@pytest.mark.parametrize("M,N,K", [(1, 256, 128), (130, 272, 144), (257, 512, 16),
                                   (128, 256, 4096), (333, 784, 400), (64, 4096, 256)])
@pytest.mark.parametrize("layout", [qgemm.B_KN, qgemm.B_NK])
def test_tcgen05_ragged_shapes(gpu, oracle, M, N, K, layout):
    A, B, sA, sB = syn.w8a8_inputs(M, N, K, seed=M * 7 + N + K)
    y, acc = run(gpu, A, B, sA, sB, layout=layout, algo=qgemm.ALGO_TCGEN05)
    check_exact(oracle, A, B, sA, sB, y, acc, qgemm.BF16)


@pytest.mark.parametrize("M,N,K", [(256, 256, 128), (512, 768, 4096), (1000, 1040, 272),
                                   (4096, 256, 1024), (257, 4096, 512)])
@pytest.mark.parametrize("layout", [qgemm.B_KN, qgemm.B_NK])
def test_tcgen05_cta_pair_shapes(gpu, oracle, M, N, K, layout):
    """Shapes with at least one full 256 x 256 tile run on CTA pairs (cta_group::2)."""
    A, B, sA, sB = syn.w8a8_inputs(M, N, K, seed=M + 3 * N + 7 * K)
    y, acc = run(gpu, A, B, sA, sB, layout=layout, algo=qgemm.ALGO_TCGEN05)
    check_exact(oracle, A, B, sA, sB, y, acc, qgemm.BF16)


@pytest.mark.parametrize("M,N,K,layout,out_dtype,ldc", [
    (3840, 1280, 1024, qgemm.B_KN, qgemm.BF16, None),   # 75 pair tiles: one tile in 4 K parts
    (3840, 1536, 1024, qgemm.B_NK, qgemm.BF16, None),   # 90 tiles: 16 leftover tiles in 4 parts
    (3840, 1280, 1024, qgemm.B_KN, qgemm.F32, 1281),    # parts summed on the plain-store path
    (4096, 4096, 512, qgemm.B_NK, qgemm.BF16, None),    # 256 tiles: 34 leftover as 68 column halves
    (2048, 6144, 1024, qgemm.B_KN, qgemm.F32, 6150),    # 192 tiles: last round left whole
    (3840, 4224, 512, qgemm.B_KN, qgemm.BF16, None),    # 255 tiles: 33 leftover as halves, the
    (3840, 4224, 640, qgemm.B_NK, qgemm.F32, 4230),     # last tile column's second half past N
])
def test_tcgen05_last_wave_split(gpu, oracle, M, N, K, layout, out_dtype, ldc):
    """The last-wave forms (tail tiles cut along K over idle CTA pairs, int32 partials
    summed by the last part; or done as 256 x 128 column halves) give the same bits as
    the CUDA-core kernel, and the sampled rows equal the oracle; run twice to check
    that the counters reset."""
    A, B, sA, sB = syn.w8a8_inputs(M, N, K, seed=M + N + K + 5)
    y1, a1 = run(gpu, A, B, sA, sB, layout=layout, out_dtype=out_dtype, ldc=ldc,
                 algo=qgemm.ALGO_TCGEN05)
    y2, a2 = run(gpu, A, B, sA, sB, layout=layout, out_dtype=out_dtype, ldc=ldc,
                 algo=qgemm.ALGO_TCGEN05)
    ys, as_ = run(gpu, A, B, sA, sB, layout=layout, out_dtype=out_dtype, ldc=ldc,
                  algo=qgemm.ALGO_SIMT)
    np.testing.assert_array_equal(a1, as_)
    np.testing.assert_array_equal(y1, ys)
    np.testing.assert_array_equal(a2, as_)
    np.testing.assert_array_equal(y2, ys)
    rows = np.unique(np.concatenate([np.random.default_rng(1).choice(M, 12, replace=False),
                                     [0, M - 1]]))
    check_exact(oracle, A, B, sA, sB, y1, a1, out_dtype, rows=rows)


def test_tcgen05_cta_pair_ldc_f32(gpu, oracle):
    A, B, sA, sB = syn.w8a8_inputs(384, 512, 640, seed=17)
    y, acc = run(gpu, A, B, sA, sB, out_dtype=qgemm.F32, ldc=520, algo=qgemm.ALGO_TCGEN05)
    check_exact(oracle, A, B, sA, sB, y, acc, qgemm.F32)


def test_tcgen05_extreme_values(gpu, oracle):
    """-128 * -128 everywhere: the largest int32 sums the operand range allows."""
    M, N, K = 128, 256, 8192
    A = np.full((M, K), -128, np.int8)
    B = np.full((K, N), -128, np.int8)
    B[:, ::2] = 127
    sA = np.ones(M, np.float32)
    sB = np.ones(N, np.float32)
    y, acc = run(gpu, A, B, sA, sB, out_dtype=qgemm.F32, algo=qgemm.ALGO_TCGEN05)
    check_exact(oracle, A, B, sA, sB, y, acc, qgemm.F32)
    assert acc[0, 1] == 128 * 128 * K


def test_ldc_padding_untouched(gpu, oracle):
    A, B, sA, sB = syn.w8a8_inputs(200, 512, 256, seed=13)
    y, acc = run(gpu, A, B, sA, sB, ldc=520, algo=qgemm.ALGO_TCGEN05)
    check_exact(oracle, A, B, sA, sB, y, acc, qgemm.BF16)


@pytest.mark.parametrize("M,N,K,layout", [(5, 100, 20, qgemm.B_KN), (70, 33, 7, qgemm.B_NK),
                                          (3, 24, 0, qgemm.B_KN)])
def test_simt_any_shape(gpu, oracle, M, N, K, layout):
    A, B, sA, sB = syn.w8a8_inputs(M, N, K, seed=14)
    y, acc = run(gpu, A, B, sA, sB, layout=layout, out_dtype=qgemm.F32)  # AUTO -> SIMT
    check_exact(oracle, A, B, sA, sB, y, acc, qgemm.F32)


def test_config2_full_shape(gpu, oracle):
    """4096^3, bf16 out: tcgen05 == SIMT bit for bit over the whole output, and
    a seeded sample of rows (plus the first and last 128-row tiles' corners)
    equals the CPU oracle."""
    M = N = K = 4096
    A, B, sA, sB = syn.w8a8_inputs(M, N, K, seed=2, sa=(0.001, 0.01), sb=(0.0005, 0.005))
    y_tc, acc_tc = run(gpu, A, B, sA, sB, algo=qgemm.ALGO_TCGEN05)
    y_st, acc_st = run(gpu, A, B, sA, sB, algo=qgemm.ALGO_SIMT)
    np.testing.assert_array_equal(acc_tc, acc_st)
    np.testing.assert_array_equal(y_tc, y_st)
    rng = np.random.default_rng(99)
    rows = np.unique(np.concatenate([rng.choice(M, 48, replace=False), [0, 1, 127, 128, M - 1]]))
    check_exact(oracle, A, B, sA, sB, y_tc, acc_tc, qgemm.BF16, rows=rows)


def test_repeat_calls_identical(gpu):
    A, B, sA, sB = syn.w8a8_inputs(512, 1024, 1024, seed=15)
    y1, a1 = run(gpu, A, B, sA, sB, algo=qgemm.ALGO_TCGEN05)
    y2, a2 = run(gpu, A, B, sA, sB, algo=qgemm.ALGO_TCGEN05)
    np.testing.assert_array_equal(a1, a2)
    np.testing.assert_array_equal(y1, y2)


def test_error_statuses(gpu):
    dev, st, ops = gpu
    A, B, sA, sB = syn.w8a8_inputs(16, 32, 20, seed=16)
    d = [dev_array(gpu, a) for a in (A, B, sA, sB)]
    out = Out(dev, st, 16 * 32 * 4)
    with pytest.raises(qgemm.QGemmError) as e:  # K % 16 != 0 on the tensor-core path
        ops.w8a8Gemm(d[0], d[1], d[2], d[3], out, 16, 32, 20, algo=qgemm.ALGO_TCGEN05)
    assert e.value.status == qgemm._lib.ERR_UNSUPPORTED
    with pytest.raises(qgemm.QGemmError) as e:
        ops.w8a8Gemm(d[0], d[1], d[2], d[3], out.address + 1, 16, 32, 20, out_dtype=qgemm.F32)
    assert e.value.status == qgemm._lib.ERR_BAD_ALIGN
    with pytest.raises(qgemm.QGemmError) as e:
        ops.w8a8Gemm(d[0], d[1], d[2], d[3], out, -1, 32, 20)
    assert e.value.status == qgemm._lib.ERR_INVALID_ARG
    with pytest.raises(qgemm.QGemmError) as e:
        ops.w8a8Gemm(0, d[1], d[2], d[3], out, 16, 32, 20)
    assert e.value.status == qgemm._lib.ERR_INVALID_ARG
    with pytest.raises(qgemm.QGemmError) as e:
        ops.w8a8Gemm(d[0], d[1], d[2], d[3], out, 16, 32, 20, ldc=8)
    assert e.value.status == qgemm._lib.ERR_INVALID_ARG
    st.sync()  # the stream is still healthy
