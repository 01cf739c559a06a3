"""The remaining reference operators on the GPU, bit-exact against the oracle
(QuantizedGemmOps.scala:24-84 w8a16Gemm / RowWise, :121-192 quantizers,
:198-212 dequantize), the by-name launch path, the weight prepack and the
column unshard used after the multi-GPU all-gather."""
import os

import numpy as np
import pytest

import qgemm
import qgemm.synthetic as syn
from helpers import Out, dev_array

pytestmark = pytest.mark.gpu

GOLD = np.load(os.path.join(os.path.dirname(__file__), "golden", "golden.npz"))


def f32_bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


@pytest.mark.parametrize("has_bias", [True, False])
def test_w8a16(gpu, oracle, has_bias):
    dev, st, ops = gpu
    rng = np.random.default_rng(51)
    M, N, K = 37, 300, 129
    w = rng.integers(-127, 128, (K, N), dtype=np.int8)
    sw = rng.uniform(0.001, 0.01, N).astype(np.float32)
    x = rng.standard_normal((M, K), dtype=np.float32)
    b = rng.standard_normal(N).astype(np.float32)
    y = Out(dev, st, M * N * 4)
    ops.w8a16Gemm(dev_array(gpu, w), dev_array(gpu, sw), dev_array(gpu, x), dev_array(gpu, b), y,
                  M, N, K, has_bias)
    st.sync()
    ref = oracle.w8a16_gemm(w, sw, x, b if has_bias else None)
    np.testing.assert_array_equal(y.read(np.uint32, (M, N)), f32_bits(ref))


@pytest.mark.parametrize("M,N,K,has_bias,rowwise", [
    (1, 14336, 4096, True, False),   # the decode-GEMV shape, int8 weights
    (9, 512, 1000, False, False),    # three 4-row passes, a 232-row last stage
    (4, 4112, 256, True, False),     # a partial last 128-column block
    (3, 1024, 520, False, True),     # row-wise scales
    (2, 48, 4, True, False),         # a single short stage
])
def test_w8a16_weight_stream_path(gpu, oracle, M, N, K, has_bias, rowwise):
    """N % 16 == 0 and K % 4 == 0 take the TMA weight-stream kernel: still the
    reference's sequential fp32 order, bit for bit."""
    dev, st, ops = gpu
    rng = np.random.default_rng(M * N + K)
    w = rng.integers(-127, 128, (K, N), dtype=np.int8)
    sw = rng.uniform(0.001, 0.01, K if rowwise else N).astype(np.float32)
    x = rng.standard_normal((M, K), dtype=np.float32)
    b = rng.standard_normal(N).astype(np.float32)
    y = Out(dev, st, M * N * 4)
    if rowwise:
        ops.w8a16GemmRowWise(dev_array(gpu, w), dev_array(gpu, sw), dev_array(gpu, x), y, M, N, K)
        ref = oracle.w8a16_gemm_rowwise(w, sw, x)
    else:
        ops.w8a16Gemm(dev_array(gpu, w), dev_array(gpu, sw), dev_array(gpu, x), dev_array(gpu, b),
                      y, M, N, K, has_bias)
        ref = oracle.w8a16_gemm(w, sw, x, b if has_bias else None)
    st.sync()
    np.testing.assert_array_equal(y.read(np.uint32, (M, N)), f32_bits(ref))


def test_w8a16_rowwise_golden(gpu):
    dev, st, ops = gpu
    w, x = GOLD["w8a16_w"], GOLD["w8a16_x"]
    K, N = w.shape
    M = x.shape[0]
    y = Out(dev, st, M * N * 4)
    ops.w8a16GemmRowWise(dev_array(gpu, w), dev_array(gpu, GOLD["w8a16_swr"]), dev_array(gpu, x),
                         y, M, N, K)
    st.sync()
    np.testing.assert_array_equal(y.read(np.uint32, (M, N)), f32_bits(GOLD["w8a16_y_rowwise"]))


@pytest.mark.parametrize("qbits", [8, 4])
def test_dynamic_quantize_golden(gpu, qbits):
    dev, st, ops = gpu
    wt = GOLD["quant_w"]
    K, N = wt.shape
    s = Out(dev, st, N * 4)
    q = Out(dev, st, K * N)
    ops.dynamicQuantize(dev_array(gpu, wt), s, q, K, N, qbits)
    st.sync()
    np.testing.assert_array_equal(q.read(np.int8, (K, N)), GOLD[f"quant{qbits}_q"])
    np.testing.assert_array_equal(s.read(np.uint32, (N,)), f32_bits(GOLD[f"quant{qbits}_scales"]))


def test_quantizers_random(gpu, oracle):
    dev, st, ops = gpu
    rng = np.random.default_rng(52)
    K, N = 513, 333
    wt = (rng.standard_normal((K, N)) * rng.uniform(0.01, 3, N)).astype(np.float32)
    s, q, z = Out(dev, st, N * 4), Out(dev, st, K * N), Out(dev, st, N)
    ops.weightOnlyQuantizePerChannel(dev_array(gpu, wt), s, q, z, K, N)
    st.sync()
    so, qo, zo = oracle.weight_only_quantize_per_channel(wt)
    np.testing.assert_array_equal(q.read(np.int8, (K, N)), qo)
    np.testing.assert_array_equal(s.read(np.uint32, (N,)), f32_bits(so))
    np.testing.assert_array_equal(z.read(np.int8, (N,)), zo)
    # dequantize the result back (QuantizedGemmOps.scala:198-212)
    w2 = Out(dev, st, K * N * 4)
    ops.dequantize(dev_array(gpu, qo), dev_array(gpu, so), w2, K, N)
    st.sync()
    np.testing.assert_array_equal(w2.read(np.uint32, (K, N)), f32_bits(oracle.dequantize(qo, so)))


def test_by_name_matches_direct(gpu, oracle):
    dev, st, ops = gpu
    A, B, sA, sB = syn.w8a8_inputs(64, 512, 512, seed=53)
    d = {k: dev_array(gpu, v) for k, v in dict(A=A, B=B, sA=sA, sB=sB).items()}
    y = Out(dev, st, 64 * 512 * 4)
    ops.launchKernel("w8a32Gemm", [d["B"], d["sB"], d["A"], d["sA"], y], [64, 512, 512])
    st.sync()
    yo, _ = oracle.w8a32_gemm(B, sB, A, sA)
    np.testing.assert_array_equal(y.read(np.uint32, (64, 512)), f32_bits(yo))
    with pytest.raises(qgemm.QGemmError):
        ops.launchKernel("w8a32Gemm", [d["B"]], [64, 512, 512])
    with pytest.raises(qgemm.QGemmError):
        ops.launchKernel("tritonNoSuchKernel", [], [])


def test_prepack_roundtrip_and_gemm(gpu, oracle):
    dev, st, ops = gpu
    M, N, K = 96, 768, 640
    A, B, sA, sB = syn.w8a8_inputs(M, N, K, seed=54)
    nk = Out(dev, st, N * K)
    ops.prepackW8NK(dev_array(gpu, B), nk, K, N)
    st.sync()
    np.testing.assert_array_equal(nk.read(np.int8, (N, K)), B.T)
    y = Out(dev, st, M * N * 2)
    ops.w8a8Gemm(dev_array(gpu, A), nk, dev_array(gpu, sA), dev_array(gpu, sB), y, M, N, K,
                 b_layout=qgemm.B_NK)
    st.sync()
    yo, _ = oracle.w8a32_gemm(B, sB, A, sA)
    np.testing.assert_array_equal(y.read(np.uint16, (M, N)), oracle.bf16_rne(yo))


@pytest.mark.parametrize("world,M,ncols", [(4, 33, 24), (2, 16, 13), (8, 5, 256)])
def test_unshard_columns(gpu, world, M, ncols):
    import qgemm._lib as L
    dev, st, _ = gpu
    rng = np.random.default_rng(55)
    g = rng.integers(0, 65535, (world, M, ncols), dtype=np.uint16)
    out = Out(dev, st, M * world * ncols * 2)
    L.call("qgemm_unshard_columns_bf16", st.handle, dev_array(gpu, g).address, out.address, world,
           M, ncols)
    st.sync()
    np.testing.assert_array_equal(out.read(np.uint16, (M, world * ncols)),
                                  np.concatenate(list(g), axis=1))


@pytest.mark.parametrize("M,K,dt", [(7, 300, "f32"), (64, 4096, "bf16"), (3, 13, "f32"),
                                    (129, 1024, "bf16"),
                                    # a warp per row: 4 and 8 vectors per lane
                                    (9, 512, "bf16"), (17, 1000, "f32"), (33, 2040, "bf16"),
                                    (33, 2048, "f32"),
                                    # rows held in registers: 3 and 4 vectors per thread
                                    (5, 6000, "bf16"), (4, 4096, "f32"), (3, 8192, "bf16"),
                                    # rows too long for registers, or K not a multiple of 8
                                    (2, 8200, "bf16"), (3, 4100, "f32"), (6, 1028, "bf16")])
def test_quantize_per_token_matches_reference_rows(gpu, oracle, M, K, dt):
    """Per-token quantisation == the reference dynamicQuantize applied to x^T, bit for bit
    (scales and int8 values), for fp32 and bf16 activations."""
    import qgemm
    dev, st, ops = gpu
    rng = np.random.default_rng(M * K)
    xf = (rng.standard_normal((M, K)) * rng.uniform(0.1, 10, (M, 1))).astype(np.float32)
    xf[0, :] = 0.0                      # an all-zero row: scale 0, mul 1
    if K > 5:
        xf[1, 3] = np.nan               # NaN is ignored by the max and quantises to 0
        xf[2 % M, 5] = 1e30             # saturation
    if dt == "bf16":
        xb = syn.bf16_bits(xf)
        x_dev, x_ref, in_dtype = dev_array(gpu, xb), syn.bf16_to_float(xb), qgemm.BF16
    else:
        x_dev, x_ref, in_dtype = dev_array(gpu, xf), xf, qgemm.F32
    q = Out(dev, st, M * K)
    s = Out(dev, st, M * 4)
    ops.quantizePerToken(x_dev, q, s, M, K, in_dtype=in_dtype)
    st.sync()
    ref_s, ref_q = oracle.dynamic_quantize(np.ascontiguousarray(x_ref.T), 8)
    np.testing.assert_array_equal(q.read(np.int8, (M, K)), ref_q.T)
    np.testing.assert_array_equal(s.read(np.uint32, (M,)), ref_s.view(np.uint32))


def test_quantize_then_w8a8_pipeline(gpu, oracle):
    """bf16 activations -> per-token int8 + sA -> W8A8 GEMM, against the oracle."""
    import qgemm
    dev, st, ops = gpu
    M, N, K = 256, 512, 768
    rng = np.random.default_rng(9)
    xb = syn.bf16_bits(rng.standard_normal((M, K)).astype(np.float32))
    _, B, _, sB = syn.w8a8_inputs(M, N, K, seed=10)
    q = Out(dev, st, M * K)
    sA = Out(dev, st, M * 4)
    ops.quantizePerToken(dev_array(gpu, xb), q, sA, M, K, in_dtype=qgemm.BF16)
    y = Out(dev, st, M * N * 2)
    ops.w8a8Gemm(q, dev_array(gpu, B), sA, dev_array(gpu, sB), y, M, N, K,
                 algo=qgemm.ALGO_TCGEN05)
    st.sync()
    ref_s, ref_q = oracle.dynamic_quantize(np.ascontiguousarray(syn.bf16_to_float(xb).T), 8)
    yo, _ = oracle.w8a32_gemm(B, sB, np.ascontiguousarray(ref_q.T), ref_s)
    np.testing.assert_array_equal(y.read(np.uint16, (M, N)), oracle.bf16_rne(yo))
