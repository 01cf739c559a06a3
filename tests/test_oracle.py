"""CPU oracle: known answers, golden vectors, and internal consistency.

The oracle restates QuantizedGemmOps.scala (bytedeco/cuda-triton-scala,
src/main/scala/cuda/dsl/operators/linalg/QuantizedGemmOps.scala); these tests
pin it to hand-computed cases and to the independent pure-Python restatement in
tests/golden/make_golden.py.
"""
import os

import numpy as np
import pytest

GOLD = os.path.join(os.path.dirname(__file__), "golden", "golden.npz")


@pytest.fixture(scope="module")
def gold():
    return np.load(GOLD)


# ---- hand-computed known answers ---------------------------------------------

def test_w8a32_known_answer(oracle):
    # acc = x @ w by hand; power-of-two scales make every fp32 product exact.
    x = np.array([[1, 2, 3, 4], [-1, 0, 1, -128]], np.int8)
    w = np.array([[1, 0, -1], [2, 1, 0], [0, 3, 1], [127, -1, 2]], np.int8)
    sw = np.array([0.5, 0.25, 2.0], np.float32)
    sx = np.array([1.0, 0.5], np.float32)
    y, acc = oracle.w8a32_gemm(w, sw, x, sx)
    assert acc.tolist() == [[513, 7, 10], [-16257, 131, -254]]
    assert y.tolist() == [[256.5, 1.75, 20.0], [-4064.25, 16.375, -254.0]]


def test_w8a32_k1_and_extremes(oracle):
    x = np.array([[-128], [127]], np.int8)
    w = np.array([[-128, 127]], np.int8)
    y, acc = oracle.w8a32_gemm(w, np.ones(2, np.float32), x, np.ones(2, np.float32))
    assert acc.tolist() == [[16384, -16256], [-16256, 16129]]


def test_w4a16_known_answer(oracle):
    # N = 3 (odd): element k*N+n lives in byte (k*N+n)//2, low nibble first.
    q = [[9, 8, 15], [0, 7, 10]]          # w - 8 = [[1,0,7],[-8,-1,2]]
    flat = [v for row in q for v in row]
    wb = np.array([flat[0] | flat[1] << 4, flat[2] | flat[3] << 4, flat[4] | flat[5] << 4],
                  np.uint8)
    assert wb.tolist() == [0x89, 0x0F, 0xA7]
    y = oracle.w4a16_gemm(wb, np.array([1.0, 2.0, 0.5], np.float32),
                          np.array([[1.0, 2.0]], np.float32), N=3)
    assert y.tolist() == [[-15.0, -4.0, 5.5]]


def test_scala_float_to_int(oracle):
    assert oracle.scala_f2i(31.75) == 31
    assert oracle.scala_f2i(-31.75) == -31
    assert oracle.scala_f2i(float("nan")) == 0
    assert oracle.scala_f2i(float("inf")) == 2147483647
    assert oracle.scala_f2i(-3e10) == -2147483648


def test_bf16_encoders(oracle):
    L = oracle.lib()
    assert L.oracle_f32_to_bf16_rne(1.0) == 0x3F80
    # 1 + 2^-8 is a tie between 0x3F80 and 0x3F81: RNE keeps the even one
    assert L.oracle_f32_to_bf16_rne(1.00390625) == 0x3F80
    assert L.oracle_f32_to_bf16_rne(1.01171875) == 0x3F82
    # the reference encoder truncates (core/Types.scala:515-519)
    assert L.oracle_f32_to_bf16_trunc(1.01171875) == 0x3F81
    v = np.array([1.0, 1.00390625, 1.01171875, -2.5, 3.0e38], np.float32)
    assert oracle.bf16_rne(v).tolist() == [oracle.f32_to_bf16_scalar(float(a)) for a in v]


# ---- golden vectors (independent pure-Python restatement) --------------------

@pytest.mark.parametrize("name", ["w8a32_rand", "w8a32_ext"])
def test_golden_w8a32(oracle, gold, name):
    y, acc = oracle.w8a32_gemm(gold[f"{name}_w"], gold[f"{name}_sw"], gold[f"{name}_x"],
                               gold[f"{name}_sx"])
    np.testing.assert_array_equal(acc, gold[f"{name}_acc"])
    np.testing.assert_array_equal(y.view(np.uint32), gold[f"{name}_y"].view(np.uint32))


def test_golden_w4a16(oracle, gold):
    y = oracle.w4a16_gemm(gold["w4a16_w"], gold["w4a16_sw"], gold["w4a16_x"],
                          N=int(gold["w4a16_N"]))
    np.testing.assert_array_equal(y.view(np.uint32), gold["w4a16_y"].view(np.uint32))


def test_golden_w8a16(oracle, gold):
    w, x, b = gold["w8a16_w"], gold["w8a16_x"], gold["w8a16_b"]
    for bias, key in ((b, "w8a16_y_bias"), (None, "w8a16_y_nobias")):
        y = oracle.w8a16_gemm(w, gold["w8a16_swc"], x, bias)
        np.testing.assert_array_equal(y.view(np.uint32), gold[key].view(np.uint32))
    y = oracle.w8a16_gemm_rowwise(w, gold["w8a16_swr"], x)
    np.testing.assert_array_equal(y.view(np.uint32), gold["w8a16_y_rowwise"].view(np.uint32))


@pytest.mark.parametrize("qbits", [8, 4])
def test_golden_quantize(oracle, gold, qbits):
    s, q = oracle.dynamic_quantize(gold["quant_w"], qBits=qbits)
    np.testing.assert_array_equal(q, gold[f"quant{qbits}_q"])
    np.testing.assert_array_equal(s.view(np.uint32), gold[f"quant{qbits}_scales"].view(np.uint32))
    if qbits == 8:
        s2, q2, z = oracle.weight_only_quantize_per_channel(gold["quant_w"])
        np.testing.assert_array_equal(q2, q)
        np.testing.assert_array_equal(s2.view(np.uint32), s.view(np.uint32))
        assert (z == 0).all()


def test_quantize_edge_semantics(oracle, gold):
    _, q = oracle.dynamic_quantize(gold["quant_w"], qBits=8)
    # column 1 holds a NaN: NaN never wins `v > maxAbs` and NaN.toInt == 0
    assert q[0, 1] == 0
    # column 2 has max |w| < 1e-6: the applied scale is 1.0, so values truncate to 0
    assert (q[:, 2] == 0).all()
    # column 0: 0.25 * 127 = 31.75 truncates to 31
    assert q[0, 0] == 31


def test_golden_dequantize(oracle, gold):
    w = oracle.dequantize(gold["dq_q"], gold["dq_s"])
    np.testing.assert_array_equal(w.view(np.uint32), gold["dq_w"].view(np.uint32))


@pytest.mark.parametrize("zp", [8, 3])
def test_golden_grouped(oracle, gold, zp):
    y, yb = oracle.w4a16_grouped(gold["grp_wq"], gold["grp_sc"], zp, int(gold["grp_G"]),
                                 gold["grp_x"], threads=1)
    np.testing.assert_array_equal(y.view(np.uint32), gold[f"grp{zp}_y"].view(np.uint32))
    np.testing.assert_array_equal(yb, gold[f"grp{zp}_yb"])


# ---- internal consistency ----------------------------------------------------

def test_w8a32_matches_int64_gemm(oracle):
    rng = np.random.default_rng(1)
    M, N, K = 17, 33, 70
    x = rng.integers(-128, 128, (M, K), dtype=np.int8)
    w = rng.integers(-128, 128, (K, N), dtype=np.int8)
    _, acc = oracle.w8a32_gemm(w, np.ones(N, np.float32), x, np.ones(M, np.float32))
    np.testing.assert_array_equal(acc, x.astype(np.int64) @ w.astype(np.int64))


def test_rows_variant_is_bit_identical(oracle):
    import qgemm.synthetic as syn
    A, B, sA, sB = syn.w8a8_inputs(64, 512, 512, seed=3)
    y, _ = oracle.w8a32_gemm(B, sB, A, sA)
    y2, yb = oracle.w8a8_gemm_rows(B, sB, A, sA, threads=4)
    np.testing.assert_array_equal(y.view(np.uint32), y2.view(np.uint32))
    np.testing.assert_array_equal(yb, oracle.bf16_rne(y))
    _, ys = oracle.w8a8_gemm_rows(B, sB, A, sA, m0=10, m1=20, threads=2, want_f32=False)
    np.testing.assert_array_equal(ys, oracle.bf16_rne(y[10:20]))
    _, _, acc_rows = oracle.w8a8_gemm_rows(B, sB, A, sA, m0=5, m1=9, want_acc=True)
    np.testing.assert_array_equal(acc_rows, A[5:9].astype(np.int64) @ B.astype(np.int64))


# ---- the int8 GEMM names (TensorCoreOps.tensorCoreGemmInt8, CutlassGemm.int8GemmKernel) ----

def test_tensor_core_gemm_int8_known_answer(oracle):
    """d = a @ b + c through leading dimensions; padding columns are never read."""
    a = np.array([[1, 2, 9], [3, 4, 9]], np.int8)          # lda 3, K 2
    b = np.array([[5, 6, 0, 0], [7, 8, 0, 0]], np.int8)    # ldb 4, N 2
    c = np.array([[100, 200, 7], [300, 400, 7]], np.int32)  # ldc 3
    d = oracle.tensor_core_gemm_int8(a, b, c, M=2, N=2, K=2, lda=3, ldb=4, ldc=3, ldd=3)
    assert d.tolist() == [[119, 222, 0], [343, 450, 0]]
    d = oracle.tensor_core_gemm_int8(a, b, None, M=2, N=2, K=2, lda=3, ldb=4)
    assert d.tolist() == [[19, 22], [43, 50]]


def test_tensor_core_gemm_int8_wraps_like_scala_int(oracle):
    a = np.full((1, 4), -128, np.int8)
    b = np.full((4, 1), -128, np.int8)
    c = np.array([[2**31 - 65536]], np.int32)
    d = oracle.tensor_core_gemm_int8(a, b, c, M=1, N=1, K=4)
    assert int(d[0, 0]) == ((4 * 16384 + 2**31 - 65536 + 2**31) % 2**32) - 2**31


def test_int8_gemm_kernel_known_answer(oracle):
    """(acc * scaleA) * scaleB with one fp32 accumulator per output."""
    A = np.array([[1, 2], [3, 4]], np.int32)
    B = np.array([[5, 6], [7, 8]], np.int32)
    D = oracle.int8_gemm_kernel(A, B, 0.5, 2.0, M=2, N=2, K=2)
    assert D.tolist() == [[19.0, 22.0], [43.0, 50.0]]


def test_int8_gemm_kernel_rounds_in_k_order(oracle):
    """Past 2^24 the fp32 accumulator rounds: 2^24 + 1 + 1 stays 2^24 in k order, so the
    result differs from the exact integer sum (2^24 + 2) -- the reference's own loop."""
    A = np.array([[1, 1, 1]], np.int32)
    B = np.array([[2**24], [1], [1]], np.int32)
    D = oracle.int8_gemm_kernel(A, B, 1.0, 1.0, M=1, N=1, K=3)
    assert float(D[0, 0]) == float(2**24)
    B2 = np.array([[1], [1], [2**24]], np.int32)
    D2 = oracle.int8_gemm_kernel(A, B2, 1.0, 1.0, M=1, N=1, K=3)
    assert float(D2[0, 0]) == float(2**24 + 2)


def test_int8_gemm_kernel_matches_exact_sums_in_range(oracle):
    """int8-range values with K <= 1024 keep every partial sum below 2^24: the fp32 loop is
    then the exact integer sum rounded once."""
    rng = np.random.default_rng(21)
    M, N, K = 9, 33, 1024
    A = rng.integers(-128, 128, (M, K)).astype(np.int32)
    B = rng.integers(-128, 128, (K, N)).astype(np.int32)
    D = oracle.int8_gemm_kernel(A, B, 0.03, 1.7, M=M, N=N, K=K, threads=2)
    exact = (A.astype(np.int64) @ B.astype(np.int64)).astype(np.float32)
    np.testing.assert_array_equal(D, (exact * np.float32(0.03)) * np.float32(1.7))


def test_grouped_reduces_to_reference(oracle):
    """With G = K, zp = 8 and bf16-representable x / scales the grouped form is
    exactly w4a16Gemm (same per-element order)."""
    import qgemm.synthetic as syn
    M, N, K = 3, 24, 40
    x, wq, _ = syn.w4a16_inputs(M, N, K, group=8, seed=5)
    rng = np.random.default_rng(6)
    sc = syn.bf16_bits(rng.uniform(0.005, 0.02, size=(1, N)).astype(np.float32))
    y_g, _ = oracle.w4a16_grouped(wq, sc, 8, K, x, threads=1)
    wb = wq.view(np.uint8).reshape(-1)  # little-endian words = reference byte order
    y_r = oracle.w4a16_gemm(wb, syn.bf16_to_float(sc[0]), syn.bf16_to_float(x), N=N)
    np.testing.assert_array_equal(y_g.view(np.uint32), y_r.view(np.uint32))


def test_pack_int4_roundtrip():
    import qgemm.synthetic as syn
    rng = np.random.default_rng(7)
    q = rng.integers(0, 16, (9, 40), dtype=np.uint8)
    w = syn.pack_int4(q)
    np.testing.assert_array_equal(syn.unpack_int4(w, 40), q)
    # nibble order: element k*N+n at nibble (k*N+n)%8 of little-endian word (k*N+n)//8
    flat = q.reshape(-1)
    b = w.view(np.uint8).reshape(-1)
    assert all(((b[i // 2] >> (4 * (i % 2))) & 0xF) == flat[i] for i in range(flat.size))


def test_grouped_threads_deterministic(oracle):
    import qgemm.synthetic as syn
    x, wq, sc = syn.w4a16_inputs(2, 512, 256, group=128, seed=9)
    a, ab = oracle.w4a16_grouped(wq, sc, 8, 128, x, threads=1)
    b, bb = oracle.w4a16_grouped(wq, sc, 8, 128, x, threads=4)
    np.testing.assert_array_equal(a.view(np.uint32), b.view(np.uint32))
    np.testing.assert_array_equal(ab, bb)


# ---- fp32 operators of the same facade (MatrixOps.scala) ----------------------

def test_matmul_known_answer(oracle):
    A = np.array([[1, 2, 3, 4], [5, 6, 7, 8]], np.float32)
    B = np.array([[1, 0, 2], [0, 1, 0], [1, 1, 1], [2, 0, 1]], np.float32)
    np.testing.assert_array_equal(oracle.matmul_f32(A, B), [[12, 5, 9], [28, 13, 25]])
    bias = np.array([0.5, -1, 2], np.float32)
    np.testing.assert_array_equal(oracle.matmul_f32(A, B, bias=bias, mode=1),
                                  [[12.5, 4, 11], [28.5, 12, 27]])
    C = np.ones((2, 3), np.float32)
    np.testing.assert_array_equal(oracle.matmul_f32(A, B, C=C, alpha=2.0, beta=-3.0, mode=2),
                                  [[21, 7, 15], [53, 23, 47]])
    np.testing.assert_array_equal(oracle.gemv_f32(A, np.array([1, 0, -1, 2], np.float32)),
                                  [6, 14])


def test_matmul_sequential_fp32_order(oracle):
    # k ascending with each sum rounded to binary32: (1e8 + 1) rounds back to 1e8, so
    # the loop gives 0 where the exact value is 1.
    A = np.ones((1, 3), np.float32)
    B = np.array([[1e8], [1.0], [-1e8]], np.float32)
    assert oracle.matmul_f32(A, B)[0, 0] == 0.0
    assert oracle.gemv_f32(B.T.copy(), np.ones(3, np.float32))[0] == 0.0


def test_sgemm_reads_c_whatever_beta(oracle):
    # BLASOps.sgemm computes alpha*sum + beta*C literally: beta = 0 keeps C's NaN.
    A = np.ones((2, 2), np.float32)
    C = np.array([[np.nan, 1], [np.inf, 2]], np.float32)
    y = oracle.matmul_f32(A, A, C=C, alpha=1.0, beta=0.0, mode=2)
    assert np.isnan(y[0, 0]) and np.isnan(y[1, 0])
    assert y[0, 1] == 2 and y[1, 1] == 2


@pytest.mark.parametrize("M,N,K", [(1, 1, 1), (7, 13, 33), (64, 48, 1000)])
def test_matmul_within_fp32_bound(oracle, M, N, K):
    from helpers import gemm_bound_ratio, gemv_bound_ratio
    rng = np.random.default_rng(M * 100 + K)
    A = rng.standard_normal((M, K)).astype(np.float32)
    B = rng.standard_normal((K, N)).astype(np.float32)
    y = oracle.matmul_f32(A, B)
    assert gemm_bound_ratio(y, A, B) <= K * 2.0 ** -24
    x = rng.standard_normal(K).astype(np.float32)
    assert gemv_bound_ratio(oracle.gemv_f32(A, x), A, x) <= K * 2.0 ** -24


def test_matmul_threads_identical(oracle):
    rng = np.random.default_rng(3)
    A = rng.standard_normal((33, 70)).astype(np.float32)
    B = rng.standard_normal((70, 45)).astype(np.float32)
    y1 = oracle.matmul_f32(A, B, threads=1)
    y4 = oracle.matmul_f32(A, B, threads=4)
    np.testing.assert_array_equal(y1.view(np.uint32), y4.view(np.uint32))
