"""The fp32 entry points of the facade on the GPU (MatrixOps.scala:16-44 matmul /
matmulAddBias, :166-177 gemv, :230-243 BLASOps.sgemm) against the CPU oracle and a
float64 product.

Tolerance (fp32 gate): the forward error of every element, measured against the
exact (float64) value and divided by sum_k |A_ik B_kj| (plus |bias_j|, |beta C_ij|),
is at most 1e-5 -- helpers.gemm_bound_ratio.  The oracle (the reference's sequential
fp32 loop) is held to the same bound, so the two agree to within fp32 summation error;
bitwise equality is not expected (three tf32 tensor-core products per fp32 product,
and a different summation order) except on the exact-order path that infinite inputs
take.
"""
import numpy as np
import pytest

import qgemm
import qgemm._lib as L
import qgemm.synthetic as syn
from helpers import Out, dev_array, gemm_bound_ratio, gemv_bound_ratio, rel_err

pytestmark = pytest.mark.gpu

TOL = 1e-5


@pytest.fixture(scope="module")
def mops(gpu):
    dev, st, _ = gpu
    return qgemm.MatrixOps(st), qgemm.BLASOps(st)


def rand(shape, rng, scale=1.0):
    return (rng.standard_normal(shape) * scale).astype(np.float32)


ALGOS = {"auto": L.ALGO_AUTO, "tc": L.ALGO_TCGEN05, "simt": L.ALGO_SIMT}


def run_matmul(gpu, mops, A, B, *, bias=None, C=None, alpha=1.0, beta=0.0, algo=None):
    """Through the reference-named entry points, or through qgemm_gemm_f32 with a path
    choice when `algo` is given."""
    dev, st, _ = gpu
    M, K = A.shape
    N = B.shape[1]
    out = Out(dev, st, M * N * 4)
    if C is not None:
        st.h2d(out.address, np.ascontiguousarray(C, np.float32))
    m, b = mops
    dA = dev_array(gpu, A if K else np.zeros(1, np.float32))
    dB = dev_array(gpu, B if K else np.zeros(1, np.float32))
    if algo is not None:
        mode = 2 if C is not None else (1 if bias is not None else 0)
        m.gemmF32(dA, dB, out, M, N, K, bias=None if bias is None else dev_array(gpu, bias),
                  alpha=alpha, beta=beta, mode=mode, algo=ALGOS[algo])
    elif C is not None:
        b.sgemm(dA, dB, out, M, N, K, alpha, beta)
    elif bias is not None:
        m.matmulAddBias(dA, dB, dev_array(gpu, bias), out, M, N, K)
    else:
        m.matmul(dA, dB, out, M, N, K)
    st.sync()
    return out.read(np.float32, (M, N))


def same_bits(y, ref):
    """Bit-identical, except that a NaN matches any NaN: CUDA makes 0x7fffffff where
    x86 makes 0xffc00000 for inf - inf and inf * 0."""
    nan = np.isnan(ref)
    np.testing.assert_array_equal(np.isnan(y), nan)
    np.testing.assert_array_equal(y[~nan].view(np.uint32), ref[~nan].view(np.uint32))


def finite_ratio(y, ref, A, B):
    """gemm_bound_ratio over the elements where the oracle is finite."""
    fin = np.isfinite(ref)
    exact = A.astype(np.float64) @ B.astype(np.float64)
    scale = np.abs(A.astype(np.float64)) @ np.abs(B.astype(np.float64))
    return float(np.max(np.abs(y[fin] - exact[fin]) / scale[fin]))


SHAPES = [(1, 1, 1), (3, 5, 7), (64, 64, 64), (127, 255, 33), (256, 256, 256),
          (300, 520, 1000), (513, 1030, 96), (1, 4096, 512), (130, 8, 4100)]


@pytest.mark.parametrize("M,N,K", SHAPES)
def test_matmul(gpu, mops, oracle, M, N, K):
    rng = np.random.default_rng(M * 7 + N * 3 + K)
    A, B = rand((M, K), rng), rand((K, N), rng)
    y = run_matmul(gpu, mops, A, B)
    assert np.isfinite(y).all()
    assert gemm_bound_ratio(y, A, B) <= TOL
    assert gemm_bound_ratio(oracle.matmul_f32(A, B), A, B) <= TOL


@pytest.mark.parametrize("algo", ["tc", "simt"])
@pytest.mark.parametrize("M,N,K", [(1, 1, 1), (3, 5, 7), (64, 300, 129), (65, 66, 67),
                                   (256, 256, 256), (512, 512, 512), (1024, 768, 640),
                                   (16, 4096, 1024), (2000, 8, 300), (40, 1030, 4100)])
def test_matmul_each_path(gpu, mops, M, N, K, algo):
    # Both paths on every shape class: tiny, ragged, one tile cut into many K parts
    # (256^3, 512^3), several tiles split, skinny in M or N, long K.
    rng = np.random.default_rng(M * 5 + N * 11 + K + len(algo))
    A, B = rand((M, K), rng), rand((K, N), rng)
    y = run_matmul(gpu, mops, A, B, algo=algo)
    assert gemm_bound_ratio(y, A, B) <= TOL
    y2 = run_matmul(gpu, mops, A, B, algo=algo)
    np.testing.assert_array_equal(y.view(np.uint32), y2.view(np.uint32))  # deterministic


@pytest.mark.parametrize("algo", ["tc", "simt"])
def test_sgemm_each_path(gpu, mops, algo):
    rng = np.random.default_rng(606)
    M, N, K = 48, 520, 333
    A, B, C, bias = rand((M, K), rng), rand((K, N), rng), rand((M, N), rng), rand(N, rng)
    y = run_matmul(gpu, mops, A, B, C=C, alpha=-0.75, beta=1.5, algo=algo)
    assert gemm_bound_ratio(y, A, B, C=C, alpha=-0.75, beta=1.5) <= TOL
    y = run_matmul(gpu, mops, A, B, bias=bias, algo=algo)
    assert gemm_bound_ratio(y, A, B, bias=bias) <= TOL


def test_matmul_small_integers_exact(gpu, mops, oracle):
    # Products and sums of small integers are exact in every order: bit-identical.
    rng = np.random.default_rng(77)
    M, N, K = 300, 264, 200
    A = rng.integers(-8, 9, (M, K)).astype(np.float32)
    B = rng.integers(-8, 9, (K, N)).astype(np.float32)
    y = run_matmul(gpu, mops, A, B)
    same_bits(y, oracle.matmul_f32(A, B))


def test_matmul_last_wave_split(gpu, mops):
    # 9 x 9 pair tiles on 74 pairs: the leftover 7 tiles are cut along K into four
    # parts whose fp32 partial sums are added in part order.
    M = N = 2304
    K = 256
    rng = np.random.default_rng(2304)
    A, B = rand((M, K), rng), rand((K, N), rng)
    y = run_matmul(gpu, mops, A, B)
    assert gemm_bound_ratio(y, A, B) <= TOL
    y2 = run_matmul(gpu, mops, A, B)
    np.testing.assert_array_equal(y.view(np.uint32), y2.view(np.uint32))  # deterministic


def test_matmul_add_bias(gpu, mops, oracle):
    rng = np.random.default_rng(11)
    M, N, K = 300, 260, 200
    A, B, bias = rand((M, K), rng), rand((K, N), rng), rand(N, rng, 10.0)
    y = run_matmul(gpu, mops, A, B, bias=bias)
    assert gemm_bound_ratio(y, A, B, bias=bias) <= TOL
    assert gemm_bound_ratio(oracle.matmul_f32(A, B, bias=bias, mode=1), A, B, bias=bias) <= TOL


@pytest.mark.parametrize("alpha,beta", [(1.0, 0.0), (0.5, 2.0), (-3.0, -1.0)])
def test_sgemm(gpu, mops, oracle, alpha, beta):
    rng = np.random.default_rng(int(alpha * 10 + beta + 40))
    M, N, K = 270, 300, 129
    A, B, C = rand((M, K), rng), rand((K, N), rng), rand((M, N), rng)
    y = run_matmul(gpu, mops, A, B, C=C, alpha=alpha, beta=beta)
    assert gemm_bound_ratio(y, A, B, C=C, alpha=alpha, beta=beta) <= TOL
    ref = oracle.matmul_f32(A, B, C=C, alpha=alpha, beta=beta, mode=2)
    assert gemm_bound_ratio(ref, A, B, C=C, alpha=alpha, beta=beta) <= TOL


def test_sgemm_reads_c_whatever_beta(gpu, mops, oracle):
    # alpha * sum + beta * C as the reference writes it: beta = 0 keeps C's NaN, and
    # 0 * inf is NaN too.
    rng = np.random.default_rng(5)
    M, N, K = 40, 36, 20
    A, B = rand((M, K), rng), rand((K, N), rng)
    C = np.zeros((M, N), np.float32)
    C[3, 4] = np.nan
    C[7, 9] = np.inf
    y = run_matmul(gpu, mops, A, B, C=C, alpha=1.0, beta=0.0)
    ref = oracle.matmul_f32(A, B, C=C, alpha=1.0, beta=0.0, mode=2)
    assert np.array_equal(np.isnan(y), np.isnan(ref))
    assert np.isnan(y[3, 4]) and np.isnan(y[7, 9])
    assert finite_ratio(y, ref, A, B) <= TOL


def test_empty_k(gpu, mops):
    M, N = 5, 9
    A = np.zeros((M, 0), np.float32)
    B = np.zeros((0, N), np.float32)
    np.testing.assert_array_equal(run_matmul(gpu, mops, A, B), np.zeros((M, N), np.float32))
    bias = np.arange(N, dtype=np.float32)
    np.testing.assert_array_equal(run_matmul(gpu, mops, A, B, bias=bias),
                                  np.broadcast_to(bias, (M, N)))
    C = np.full((M, N), 2.0, np.float32)
    np.testing.assert_array_equal(run_matmul(gpu, mops, A, B, C=C, alpha=3.0, beta=0.5),
                                  np.ones((M, N), np.float32))


def test_nan_propagates(gpu, mops, oracle):
    rng = np.random.default_rng(9)
    M, N, K = 40, 24, 48
    A, B = rand((M, K), rng), rand((K, N), rng)
    A[4, 1] = np.nan
    B[7, 3] = np.nan
    y = run_matmul(gpu, mops, A, B)
    ref = oracle.matmul_f32(A, B)
    assert np.array_equal(np.isnan(y), np.isnan(ref))
    assert finite_ratio(y, ref, A, B) <= TOL


@pytest.mark.parametrize("algo", [None, "simt"])
@pytest.mark.parametrize("mode", ["matmul", "bias", "sgemm"])
def test_infinite_inputs_take_the_exact_order_path(gpu, mops, oracle, mode, algo):
    # An infinite input routes the whole product to the CUDA-core kernel that runs the
    # reference's loop (k ascending, separate roundings): bit-identical to the oracle,
    # including +-inf where three tf32 products would give inf - inf or inf * 0.
    rng = np.random.default_rng(10)
    M, N, K = 300, 260, 70
    A, B = rand((M, K), rng), rand((K, N), rng)
    B[5, :] = np.round(B[5, :])  # exact in tf32: lo parts of zero
    A[2, 5] = np.inf
    A[9, 5] = -np.inf
    B[11, 7] = np.inf
    bias, C = rand(N, rng), rand((M, N), rng)
    if mode == "matmul":
        y, ref = run_matmul(gpu, mops, A, B, algo=algo), oracle.matmul_f32(A, B)
    elif mode == "bias":
        y = run_matmul(gpu, mops, A, B, bias=bias, algo=algo)
        ref = oracle.matmul_f32(A, B, bias=bias, mode=1)
    else:
        y = run_matmul(gpu, mops, A, B, C=C, alpha=0.5, beta=-2.0, algo=algo)
        ref = oracle.matmul_f32(A, B, C=C, alpha=0.5, beta=-2.0, mode=2)
    same_bits(y, ref)
    assert np.isinf(y[2]).sum() > N // 2
    # the next call without infinities is back on the tensor cores and within the bound
    A2, B2 = rand((M, K), rng), rand((K, N), rng)
    assert gemm_bound_ratio(run_matmul(gpu, mops, A2, B2, algo=algo), A2, B2) <= TOL


def test_matmul_large_sampled(gpu, mops):
    # 4096^3: the full product through the GPU, float64 rows sampled on the CPU.
    M = N = K = 4096
    rng = np.random.default_rng(4096)
    A, B = rand((M, K), rng), rand((K, N), rng)
    y = run_matmul(gpu, mops, A, B)
    rows = rng.choice(M, 48, replace=False)
    assert gemm_bound_ratio(y[rows], A[rows], B) <= TOL


@pytest.mark.parametrize("M,N", [(1, 1), (1, 4096), (7, 1001), (4096, 4096), (100000, 64),
                                 (3, 100003), (513, 36), (1, 65536), (2, 200000), (100, 5000),
                                 (600, 3000)])
def test_gemv(gpu, mops, oracle, M, N):
    dev, st, _ = gpu
    rng = np.random.default_rng(M + N)
    A, x = rand((M, N), rng), rand(N, rng)
    y = Out(dev, st, M * 4)
    mops[0].gemv(dev_array(gpu, A), dev_array(gpu, x), y, M, N)
    st.sync()
    got = y.read(np.float32, (M,))
    assert gemv_bound_ratio(got, A, x) <= TOL
    if M * N <= 1 << 22:
        assert gemv_bound_ratio(oracle.gemv_f32(A, x), A, x) <= TOL


def test_gemv_empty_rows(gpu, mops):
    dev, st, _ = gpu
    M = 6
    y = Out(dev, st, M * 4)
    st.memset(y.address, 0xFF, M * 4)
    mops[0].gemv(16, 16, y, M, 0)  # N = 0: every sum is 0
    st.sync()
    np.testing.assert_array_equal(y.read(np.float32, (M,)), np.zeros(M, np.float32))


def test_by_name(gpu, mops):
    dev, st, ops = gpu
    rng = np.random.default_rng(21)
    M, N, K = 33, 40, 50
    A, B, bias = rand((M, K), rng), rand((K, N), rng), rand(N, rng)
    dA, dB, db = dev_array(gpu, A), dev_array(gpu, B), dev_array(gpu, bias)
    out = Out(dev, st, M * N * 4)
    ops.launchKernel("matmul", [dA, dB, out], [M, N, K])
    st.sync()
    assert gemm_bound_ratio(out.read(np.float32, (M, N)), A, B) <= TOL
    ops.launchKernel("matmulAddBias", [dA, dB, db, out], [M, N, K])
    st.sync()
    assert gemm_bound_ratio(out.read(np.float32, (M, N)), A, B, bias=bias) <= TOL
    x = rand(K, rng)
    y = Out(dev, st, M * 4)
    ops.launchKernel("gemv", [dA, dev_array(gpu, x), y], [M, K])
    st.sync()
    assert gemv_bound_ratio(y.read(np.float32, (M,)), A, x) <= TOL


def test_bad_arguments(gpu, mops):
    m, b = mops
    with pytest.raises(qgemm.QGemmError) as e:
        m.matmul(0, 16, 16, 4, 4, 4)
    assert e.value.status == L.ERR_INVALID_ARG
    with pytest.raises(qgemm.QGemmError) as e:
        m.matmul(16, 16, 16, -1, 4, 4)
    assert e.value.status == L.ERR_INVALID_ARG
    with pytest.raises(qgemm.QGemmError) as e:
        b.sgemm(16, 18, 16, 4, 4, 4, 1.0, 0.0)
    assert e.value.status == L.ERR_BAD_ALIGN
    with pytest.raises(qgemm.QGemmError) as e:
        m.gemv(16, 0, 16, 4, 4)
    assert e.value.status == L.ERR_INVALID_ARG
    with pytest.raises(qgemm.QGemmError) as e:
        m.gemmF32(16, 16, 16, 4, 4, 4, mode=3)
    assert e.value.status == L.ERR_INVALID_ARG
    with pytest.raises(qgemm.QGemmError) as e:
        m.gemmF32(16, 16, 16, 4, 4, 4, algo=7)
    assert e.value.status == L.ERR_INVALID_ARG
    m.matmul(0, 0, 0, 0, 4, 4)  # M = 0: nothing to do
    m.gemv(0, 0, 0, 0, 4)


def test_bf16_gemm_last_wave_split(gpu):
    # 15 x 5 pair tiles on 74 pairs: the last tile is cut along K into four parts whose
    # fp32 partial sums are added as floats.
    dev, st, ops = gpu
    M, N, K = 3840, 1280, 512
    rng = np.random.default_rng(3840)
    A = syn.bf16_bits(rand((M, K), rng))
    B = syn.bf16_bits(rand((N, K), rng))
    out = Out(dev, st, M * N * 2)
    ops.gemmBf16NK(dev_array(gpu, A), dev_array(gpu, B), out, M, N, K)
    st.sync()
    y = syn.bf16_to_float(out.read(np.uint16, (M, N)))
    ref = syn.bf16_to_float(A).astype(np.float64) @ syn.bf16_to_float(B).astype(np.float64).T
    assert rel_err(y, ref) <= 1e-2
