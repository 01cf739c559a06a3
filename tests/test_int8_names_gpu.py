"""The int8 GEMM names of the reference's other operator objects, against the oracle:
TensorCoreOps.tensorCoreGemmInt8 (operators/intrinsic/TensorCoreOps.scala:294-340) and
CutlassGemm.int8GemmKernel (cutlass/CutlassGemm.scala:987-1041), called directly, by
name (TritonKernelRunner.launchKernel) and through the Java bridge's by-name form
(CUDARuntimeJavaBridge.launchKernel, driver/CUDARuntimeJavaBridge.scala:121-165).
int32 outputs must be bit-exact; the fp32 output of int8GemmKernel is bit-exact while
no partial sum leaves +-2^24, and beyond that it is the exact sum rounded once, from
which the reference's fp32 loop departs by its own rounding (at most K * 2^-24 of
sum |a*b|)."""
import numpy as np
import pytest

import qgemm
from helpers import Out, dev_array

pytestmark = pytest.mark.gpu


def rand_i8(rng, shape):
    return rng.integers(-128, 128, shape).astype(np.int8)


def tc_case(gpu, oracle, M, N, K, lda, ldb, ldc, ldd, hasC, seed, via="direct"):
    dev, st, _ = gpu
    rng = np.random.default_rng(seed)
    a = rand_i8(rng, (M, lda))
    b = rand_i8(rng, (K, ldb))
    c = rng.integers(-2**31, 2**31, (M, ldc), dtype=np.int64).astype(np.int32) if hasC else None
    da, db = dev_array(gpu, a), dev_array(gpu, b)
    dc = dev_array(gpu, c) if hasC else None
    d = Out(dev, st, M * ldd * 4)
    st.memset(d.address, 0x5A, M * ldd * 4)
    if via == "direct":
        qgemm.TensorCoreOps(st).tensorCoreGemmInt8(da, db, 0, 0, dc, d, M, N, K, lda, ldb, ldc,
                                                   ldd, hasC)
    elif via == "name":
        qgemm.QuantizedGemmOps(st).launchKernel(
            "tensorCoreGemmInt8", [da, db, 0, 0, dc or 0, d.address],
            [M, N, K, lda, ldb, ldc, ldd, int(hasC)])
    else:
        r = qgemm.CUDARuntimeJavaBridge(st).launchKernel(
            "tensorCoreGemmInt8", 1, 1, 1, 256, 1, 1, [d.address, da, db, 0, 0, dc or 0],
            [M, N, K, lda, ldb, ldc, ldd, float(hasC)],
            ["M", "N", "K", "lda", "ldb", "ldc", "ldd", "hasC"])
        assert r == d.address, qgemm.last_error()
    st.sync()
    got = d.read(np.int32, (M, ldd))
    ref = oracle.tensor_core_gemm_int8(a, b, c, M=M, N=N, K=K, lda=lda, ldb=ldb, ldc=ldc,
                                       ldd=ldd)
    np.testing.assert_array_equal(got[:, :N], ref[:, :N])
    # columns between N and ldd are not written
    assert (got[:, N:].view(np.uint32) == 0x5A5A5A5A).all()


@pytest.mark.parametrize("M,N,K,lda,ldb,ldc,ldd,hasC", [
    (300, 520, 200, 208, 528, 530, 536, True),     # tensor cores, 1-CTA tiles, scalar c
    (256, 256, 128, 128, 256, 256, 256, True),     # tensor cores, one pair tile, vector c
    (1024, 2048, 4096, 4096, 2048, 0, 2048, False),  # pair tiles, no c
    (3840, 1280, 1024, 1024, 1280, 1280, 1280, True),  # last-wave split: parts summed
    (70, 33, 7, 9, 40, 33, 35, True),               # lda % 16 != 0: CUDA cores
    (5, 48, 0, 16, 48, 48, 48, True),               # K = 0: d = c
])
def test_tensor_core_gemm_int8(gpu, oracle, M, N, K, lda, ldb, ldc, ldd, hasC):
    tc_case(gpu, oracle, M, N, K, lda, ldb, ldc, ldd, hasC, seed=M + N + K)


@pytest.mark.parametrize("via", ["name", "bridge"])
def test_tensor_core_gemm_int8_by_name(gpu, oracle, via):
    tc_case(gpu, oracle, 512, 768, 512, 528, 784, 770, 772, True, seed=3, via=via)


def test_tensor_core_gemm_int8_wraps(gpu, oracle):
    """-128 * -128 over K = 8192 plus c near 2^31 wraps modulo 2^32 like Scala Int."""
    dev, st, _ = gpu
    M, N, K = 256, 256, 8192
    a = np.full((M, K), -128, np.int8)
    b = np.full((K, N), -128, np.int8)
    c = np.full((M, N), 2**31 - 7, np.int32)
    d = Out(dev, st, M * N * 4)
    qgemm.TensorCoreOps(st).tensorCoreGemmInt8(dev_array(gpu, a), dev_array(gpu, b), 0, 0,
                                               dev_array(gpu, c), d, M, N, K, K, N, N, N, True)
    st.sync()
    ref = oracle.tensor_core_gemm_int8(a, b, c, M=M, N=N, K=K)
    got = d.read(np.int32, (M, N))
    np.testing.assert_array_equal(got, ref)
    assert int(got[0, 0]) == ((128 * 128 * K + 2**31 - 7 + 2**31) % 2**32) - 2**31


def i8k_case(gpu, oracle, M, N, K, lda, ldb, ldd, A, B, sa, sb, via="direct"):
    dev, st, _ = gpu
    dA, dB = dev_array(gpu, A), dev_array(gpu, B)
    D = Out(dev, st, M * ldd * 4)
    if via == "direct":
        qgemm.CutlassGemm(st).int8GemmKernel(D, dA, dB, M, N, K, lda, ldb, ldd, sa, sb)
    elif via == "bridge_keys":
        r = qgemm.CUDARuntimeJavaBridge(st).launchKernel(
            "int8GemmKernel", (N + 63) // 64, (M + 63) // 64, 1, 256, 1, 1, [D.address, dA, dB],
            [sb, sa, M, N, K, lda, ldb, ldd],
            ["scaleB", "scaleA", "M", "N", "K", "lda", "ldb", "ldd"])
        assert r == D.address, qgemm.last_error()
    else:  # positional scalars, declaration order
        r = qgemm.CUDARuntimeJavaBridge(st).launchKernel(
            "int8GemmKernel", 1, 1, 1, 256, 1, 1, [D.address, dA, dB],
            [M, N, K, lda, ldb, ldd, sa, sb], None)
        assert r == D.address, qgemm.last_error()
    st.sync()
    got = D.read(np.float32, (M, ldd))[:, :N]
    ref = oracle.int8_gemm_kernel(A, B, sa, sb, M=M, N=N, K=K, lda=lda, ldb=ldb, ldd=ldd)[:, :N]
    return got, ref


@pytest.mark.parametrize("M,N,K,lda,ldb,ldd", [
    (64, 512, 512, 512, 512, 512),        # the reference test's shape family
    (300, 520, 1000, 1003, 530, 521),     # padded leading dimensions, K % 16 != 0
    (2048, 1024, 1024, 1024, 1024, 1024),  # pair tiles
])
@pytest.mark.parametrize("via", ["direct", "bridge_keys", "bridge_positional"])
def test_int8_gemm_kernel_in_range(gpu, oracle, M, N, K, lda, ldb, ldd, via):
    """int8 values, K <= 1040: every partial sum stays within 2^24, so the tensor-core
    integer sum rounded once is the reference's fp32 loop bit for bit."""
    rng = np.random.default_rng(M * N + K)
    A = rng.integers(-128, 128, (M, lda)).astype(np.int32)
    B = rng.integers(-128, 128, (K, ldb)).astype(np.int32)
    got, ref = i8k_case(gpu, oracle, M, N, K, lda, ldb, ldd, A, B, 0.0123, 3.5, via=via)
    np.testing.assert_array_equal(got.view(np.uint32), ref.view(np.uint32))


def test_int8_gemm_kernel_large_k(gpu, oracle):
    """K = 4096 all 127: partial sums pass 2^24, where the reference's fp32 loop rounds in
    k order (4.6e-5 low here).  The result is the exact sum rounded once, and the oracle
    stays inside the loop's own error bound of it, K * 2^-24 of sum |a*b|."""
    M, N, K = 256, 512, 4096
    A = np.full((M, K), 127, np.int32)
    B = np.full((K, N), 127, np.int32)
    got, ref = i8k_case(gpu, oracle, M, N, K, K, N, N, A, B, 0.5, 0.25)
    exact = np.float32(127 * 127 * K) * np.float32(0.5) * np.float32(0.25)
    assert (got == exact).all()
    bound = K * 2.0**-24 * (127 * 127 * K * 0.125)
    assert np.abs(got.astype(np.float64) - ref).max() <= bound
    # random int8 data at the same K stays far from 2^24: bit-exact again
    rng = np.random.default_rng(41)
    A = rng.integers(-128, 128, (M, K)).astype(np.int32)
    B = rng.integers(-128, 128, (K, N)).astype(np.int32)
    got, ref = i8k_case(gpu, oracle, M, N, K, K, N, N, A, B, 0.01, 0.02)
    np.testing.assert_array_equal(got.view(np.uint32), ref.view(np.uint32))


def test_int8_gemm_kernel_out_of_range_runs_reference_loop(gpu, oracle):
    """A value outside [-128, 127] sends the whole call through the reference's fp32 loop
    on CUDA cores: bit-identical to the oracle for any Int values."""
    rng = np.random.default_rng(8)
    M, N, K = 200, 300, 700
    A = rng.integers(-1000, 1000, (M, K)).astype(np.int32)
    B = rng.integers(-128, 128, (K, N)).astype(np.int32)
    B[5, 7] = 40000
    got, ref = i8k_case(gpu, oracle, M, N, K, K, N, N, A, B, 1.25, -0.75)
    np.testing.assert_array_equal(got.view(np.uint32), ref.view(np.uint32))


def test_bridge_result_and_errors(gpu, oracle):
    """The bridge returns the result buffer's address, or -1 (like the reference's -1L) with
    the reason in last_error(); a failed launch leaves the stream usable."""
    dev, st, _ = gpu
    br = qgemm.CUDARuntimeJavaBridge(st)
    rng = np.random.default_rng(4)
    M, N, K = 64, 128, 96
    A = rng.standard_normal((M, K)).astype(np.float32)
    B = rng.standard_normal((K, N)).astype(np.float32)
    C0 = rng.standard_normal((M, N)).astype(np.float32)
    dA, dB, dC = dev_array(gpu, A), dev_array(gpu, B), dev_array(gpu, C0)
    # sgemm's Float alpha / beta, reachable by name only here
    r = br.launchKernel("sgemm", 1, 1, 1, 16, 16, 1, [dC, dA, dB], [M, N, K, 1.5, -0.5],
                        ["M", "N", "K", "alpha", "beta"])
    assert r == dC.address, qgemm.last_error()
    st.sync()
    got = dC.to_numpy(st, np.float32, (M, N)).astype(np.float64)
    ref = oracle.matmul_f32(A, B, C=C0, alpha=1.5, beta=-0.5, mode=2).astype(np.float64)
    scale = 1.5 * (np.abs(A.astype(np.float64)) @ np.abs(B.astype(np.float64))) + 0.5 * np.abs(C0)
    assert (np.abs(got - ref) / scale).max() <= 2e-5
    # errors: unknown name, wrong buffer count, non-integral Int, Bool not 0/1, missing scalar
    assert br.launchKernel("noSuchKernel", 1, 1, 1, 1, 1, 1, [dC], [], []) == -1
    assert "unknown kernel" in qgemm.last_error()
    assert br.launchKernel("sgemm", 1, 1, 1, 1, 1, 1, [dC, dA], [M, N, K, 1, 0], None) == -1
    assert br.launchKernel("sgemm", 1, 1, 1, 1, 1, 1, [dC, dA, dB], [M + 0.5, N, K, 1, 0],
                           None) == -1
    assert "exact Int" in qgemm.last_error()
    assert br.launchKernel("w8a16Gemm", 1, 1, 1, 1, 1, 1, [dC, dA, dB, dC, dC],
                           [M, N, K, 2], ["M", "N", "K", "hasBias"]) == -1
    assert br.launchKernel("sgemm", 1, 1, 1, 1, 1, 1, [dC, dA, dB], [M, N, K], ["M", "N", "K"]) == -1
    assert "missing" in qgemm.last_error()
    st.sync()
