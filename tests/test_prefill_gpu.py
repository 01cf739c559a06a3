"""W4A16 prefill path and the bf16 tensor-core GEMM behind it, on the GPU.

* bf16 GEMM: against a float64 numpy product of the same bf16 operands (exact
  products; only the fp32 summation order and the final bf16 rounding differ), max
  elementwise relative error <= 1e-2 (helpers.rel_err);
* prefill W4A16 (QuantizedGemmOps.scala:229-245 generalised to groups), exact
  expansion: q - zp in the slab and the group scales applied in fp32 to each group's
  tensor-core partial sums (group sizes that are multiples of 64, 16-byte aligned
  scales), else the two-term hi + lo slab; against the CPU oracle, <= 1e-2; results do
  not depend on the slab width the workspace allows;
* the one-term expansion (bf16((q - zp) * s), relative weight error <= 2^-9) is gated on
  the forward error of a floating-point GEMM instead, max |y - exact| / sum_k |x w| <=
  2^-8 + K 2^-24 (helpers.gemm_bound_ratio): its weight roundings are relative to each
  product, not to each output, so the elementwise gate above does not hold for outputs
  far below the output scale (it reaches ~0.5 at K = 1024), and that gate is printed.
"""
import numpy as np
import pytest

import qgemm
import qgemm.synthetic as syn
from helpers import Out, dev_array, gemm_bound_ratio, rel_err, rel_errs

pytestmark = pytest.mark.gpu

TOL_BF16 = 1e-2


def bf16_rand(shape, rng, scale=1.0):
    return syn.bf16_bits((rng.standard_normal(shape) * scale).astype(np.float32))


def gemm_bf16(gpu, A, B, M, N, K, ldc=None):
    dev, st, ops = gpu
    ldc = N if ldc is None else ldc
    out = Out(dev, st, M * ldc * 2)
    ops.gemmBf16NK(dev_array(gpu, A), dev_array(gpu, B), out, M, N, K, ldc=ldc)
    st.sync()
    return out.read(np.uint16, (M, ldc))[:, :N]


@pytest.mark.parametrize("M,N,K", [(256, 256, 64), (300, 520, 136), (100, 304, 512),
                                   (512, 1024, 4096), (1, 256, 8)])
def test_bf16_gemm(gpu, M, N, K):
    rng = np.random.default_rng(M + N + K)
    A = bf16_rand((M, K), rng)
    B = bf16_rand((N, K), rng)
    y = gemm_bf16(gpu, A, B, M, N, K)
    ref = syn.bf16_to_float(A).astype(np.float64) @ syn.bf16_to_float(B).astype(np.float64).T
    assert rel_err(syn.bf16_to_float(y), ref) <= TOL_BF16


def test_bf16_gemm_ldc(gpu):
    M, N, K, ldc = 384, 264, 96, 272
    rng = np.random.default_rng(5)
    A, B = bf16_rand((M, K), rng), bf16_rand((N, K), rng)
    y = gemm_bf16(gpu, A, B, M, N, K, ldc=ldc)
    ref = syn.bf16_to_float(A).astype(np.float64) @ syn.bf16_to_float(B).astype(np.float64).T
    assert rel_err(syn.bf16_to_float(y), ref) <= TOL_BF16


def prefill(gpu, x, wq, sc, M, N, K, G, zp=8, ws_bytes=None, one_term=False):
    dev, st, ops = gpu
    wt = Out(dev, st, ops.w4TiledBytes(K, N))
    ops.prepackW4Tiled(dev_array(gpu, wq), wt, K, N)
    full = ops.w4PrefillWorkspaceBytes(K, N, one_term=one_term)
    ws_bytes = full if ws_bytes is None else ws_bytes
    ws = Out(dev, st, max(ws_bytes, 16))
    y = Out(dev, st, M * N * 2)
    ops.w4a16GemmGroupedPrefill(dev_array(gpu, x), wt, dev_array(gpu, sc), y, M, N, K, ws,
                                ws_bytes, zero_point=zp, group_size=G, one_term=one_term)
    st.sync()
    return y.read(np.uint16, (M, N))


@pytest.mark.parametrize("M,N,K,G,zp", [
    (300, 512, 1024, 128, 8),
    (256, 768, 2048, 64, 3),
    (513, 1000, 512, 32, 8),     # N not a multiple of 64
    (64, 4096, 4096, 128, 8),    # small M: 1-CTA tiles
    (1, 264, 512, 16, 0),
    (260, 4096, 11008, 128, 8),  # Llama-2-7B down projection (K not a multiple of 256)
    (300, 520, 1024, 128, 5),    # group-scaled: the last tile's columns past N
    (520, 2304, 1536, 192, 8),   # group-scaled: three k-blocks a group
])
def test_prefill_vs_oracle(gpu, oracle, M, N, K, G, zp):
    x, wq, sc = syn.w4a16_inputs(M, N, K, group=G, seed=M + N + K + G)
    y = prefill(gpu, x, wq, sc, M, N, K, G, zp)
    ref, _ = oracle.w4a16_grouped(wq, sc, zp, G, x)
    assert rel_err(syn.bf16_to_float(y), ref) <= TOL_BF16


def test_prefill_large_sampled_rows(gpu, oracle):
    """M=2048, N=4096, K=4096: a seeded sample of rows against the oracle."""
    M, N, K, G = 2048, 4096, 4096, 128
    x, wq, sc = syn.w4a16_inputs(M, N, K, group=G, seed=71)
    y = prefill(gpu, x, wq, sc, M, N, K, G)
    rows = np.unique(np.concatenate([np.random.default_rng(3).choice(M, 24, replace=False),
                                     [0, 255, 256, M - 1]]))
    ref, _ = oracle.w4a16_grouped(wq, sc, 8, G, x[rows])
    assert rel_err(syn.bf16_to_float(y[rows]), ref) <= TOL_BF16


def test_prefill_unaligned_scales_take_the_two_term_form(gpu, oracle):
    """Scales that are not 16-byte aligned go through the hi + lo slab instead of the
    group-scaled multiply: both within the tolerance of the oracle, different bits."""
    M, N, K, G = 300, 512, 1024, 128
    x, wq, sc = syn.w4a16_inputs(M, N, K, group=G, seed=77)
    dev, st, ops = gpu
    y_gs = prefill(gpu, x, wq, sc, M, N, K, G)
    wt = Out(dev, st, ops.w4TiledBytes(K, N))
    ops.prepackW4Tiled(dev_array(gpu, wq), wt, K, N)
    # the same scales one element into a buffer: 2-byte aligned only
    sc_pad = np.concatenate([np.zeros(1, sc.dtype), sc.reshape(-1)])
    sc_dev = dev_array(gpu, sc_pad)
    y = Out(dev, st, M * N * 2)
    kp = (K + 63) // 64 * 64
    ws = Out(dev, st, N * kp * 4)
    ops.w4a16GemmGroupedPrefill(dev_array(gpu, x), wt, sc_dev.address + 2, y, M, N, K, ws,
                                N * kp * 4, group_size=G)
    st.sync()
    y_two = y.read(np.uint16, (M, N))
    ref, _ = oracle.w4a16_grouped(wq, sc, 8, G, x)
    assert rel_err(syn.bf16_to_float(y_gs), ref) <= TOL_BF16
    assert rel_err(syn.bf16_to_float(y_two), ref) <= TOL_BF16
    assert not np.array_equal(y_gs, y_two)


def test_prefill_slab_width_does_not_change_results(gpu):
    M, N, K, G = 320, 1000, 768, 64
    x, wq, sc = syn.w4a16_inputs(M, N, K, group=G, seed=72)
    full = prefill(gpu, x, wq, sc, M, N, K, G)
    kp = (K + 63) // 64 * 64
    one_slab_of_256 = prefill(gpu, x, wq, sc, M, N, K, G, ws_bytes=256 * kp * 4)
    np.testing.assert_array_equal(full, one_slab_of_256)


def test_prefill_and_decode_paths_agree(gpu):
    """The prefill expansion and the decode kernel compute the same function."""
    M, N, K, G = 16, 2048, 2048, 128
    x, wq, sc = syn.w4a16_inputs(M, N, K, group=G, seed=73)
    dev, st, ops = gpu
    a = syn.bf16_to_float(prefill(gpu, x, wq, sc, M, N, K, G)).astype(np.float64)
    wt = Out(dev, st, ops.w4TiledBytes(K, N))
    ops.prepackW4Tiled(dev_array(gpu, wq), wt, K, N)
    y = Out(dev, st, M * N * 2)
    ops.w4a16GemmGroupedTiled(dev_array(gpu, x), wt, dev_array(gpu, sc), y, M, N, K, group_size=G)
    st.sync()
    b = syn.bf16_to_float(y.read(np.uint16, (M, N))).astype(np.float64)
    assert rel_err(a, b) <= TOL_BF16


def prefill_frag(gpu, x, wq, sc, M, N, K, G, zp=8, ws_bytes=None, one_term=False):
    """The same prefill GEMM on fragment-ordered weights (qgemm_prepack_w4_frag)."""
    dev, st, ops = gpu
    wf = Out(dev, st, ops.w4FragBytes(K, N))
    ops.prepackW4Frag(dev_array(gpu, wq), wf, K, N)
    full = ops.w4PrefillWorkspaceBytes(K, N, one_term=one_term)
    ws_bytes = full if ws_bytes is None else ws_bytes
    ws = Out(dev, st, max(ws_bytes, 16))
    y = Out(dev, st, M * N * 2)
    ops.w4a16GemmGroupedPrefillFrag(dev_array(gpu, x), wf, dev_array(gpu, sc), y, M, N, K, ws,
                                    ws_bytes, zero_point=zp, group_size=G, one_term=one_term)
    st.sync()
    return y.read(np.uint16, (M, N))


@pytest.mark.parametrize("M,N,K,G,zp", [
    (300, 512, 1024, 128, 8),
    (256, 768, 2048, 64, 3),
    (300, 520, 1056, 32, 8),     # N % 64 == 8 and K % 128 == 32: partial last CTA and block
    (64, 4096, 4096, 256, 15),
])
def test_prefill_frag_vs_oracle_and_tiled(gpu, oracle, M, N, K, G, zp):
    """Against the oracle, and bit for bit against the tiled-weight prefill: both
    expand to the same bf16 slab and run the same GEMM."""
    x, wq, sc = syn.w4a16_inputs(M, N, K, group=G, seed=M + N + K + G + 1)
    y = prefill_frag(gpu, x, wq, sc, M, N, K, G, zp)
    ref, _ = oracle.w4a16_grouped(wq, sc, zp, G, x)
    assert rel_err(syn.bf16_to_float(y), ref) <= TOL_BF16
    np.testing.assert_array_equal(y, prefill(gpu, x, wq, sc, M, N, K, G, zp))


def test_prefill_frag_slab_width_and_refusals(gpu):
    M, N, K, G = 200, 1000, 768, 64
    x, wq, sc = syn.w4a16_inputs(M, N, K, group=G, seed=74)
    kp = (K + 63) // 64 * 64
    np.testing.assert_array_equal(prefill_frag(gpu, x, wq, sc, M, N, K, G),
                                  prefill_frag(gpu, x, wq, sc, M, N, K, G, ws_bytes=256 * kp * 4))
    x, wq, sc = syn.w4a16_inputs(8, 64, 96, group=48, seed=75)
    with pytest.raises(qgemm.QGemmError) as e:
        prefill_frag(gpu, x, wq, sc, 8, 64, 96, 48)
    assert e.value.status == qgemm._lib.ERR_UNSUPPORTED
    gpu[1].sync()


@pytest.mark.parametrize("M,N,K,G,zp", [
    (300, 512, 1024, 128, 8),
    (256, 768, 2048, 64, 3),
    (300, 520, 1056, 32, 8),     # K not a multiple of 64: the slab pitch is padded
    (260, 4096, 11008, 128, 8),  # Llama-2-7B down projection
])
def test_prefill_one_term_vs_oracle(gpu, oracle, M, N, K, G, zp):
    """One bf16 term per weight: forward error within 2^-8 + K 2^-24 of sum |x w| (the
    weight rounding, the fp32 sums and the bf16 output), frag and tiled weights bit for
    bit equal, and not the same bits as the exact expansion."""
    x, wq, sc = syn.w4a16_inputs(M, N, K, group=G, seed=M + N + K + G + 2)
    y = prefill_frag(gpu, x, wq, sc, M, N, K, G, zp, one_term=True)
    ref, _ = oracle.w4a16_grouped(wq, sc, zp, G, x)
    floored, plain = rel_errs(syn.bf16_to_float(y), ref)
    w = (syn.unpack_int4(wq, N).astype(np.float64) - zp) * \
        np.repeat(syn.bf16_to_float(sc).astype(np.float64), G, axis=0)
    ratio = gemm_bound_ratio(syn.bf16_to_float(y), syn.bf16_to_float(x), w)
    print(f"one term M={M} N={N} K={K}: forward {ratio:.3e}; vs oracle floored "
          f"{floored:.3e}, plain {plain:.3e}")
    assert ratio <= 2.0 ** -8 + K * 2.0 ** -24, ratio
    np.testing.assert_array_equal(y, prefill(gpu, x, wq, sc, M, N, K, G, zp, one_term=True))
    exact = prefill_frag(gpu, x, wq, sc, M, N, K, G, zp)
    assert not np.array_equal(y, exact)


def test_prefill_one_term_slab_width(gpu):
    M, N, K, G = 320, 1000, 768, 64
    x, wq, sc = syn.w4a16_inputs(M, N, K, group=G, seed=76)
    kp = (K + 63) // 64 * 64
    full = prefill_frag(gpu, x, wq, sc, M, N, K, G, one_term=True)
    np.testing.assert_array_equal(
        full, prefill_frag(gpu, x, wq, sc, M, N, K, G, ws_bytes=256 * kp * 2, one_term=True))
    dev, st, ops = gpu
    assert ops.w4PrefillWorkspaceBytes(K, N, one_term=True) * 2 == ops.w4PrefillWorkspaceBytes(K, N)


def test_prefill_errors(gpu):
    dev, st, ops = gpu
    M, N, K, G = 256, 256, 512, 128
    x, wq, sc = syn.w4a16_inputs(M, N, K, group=G, seed=74)
    wt = Out(dev, st, ops.w4TiledBytes(K, N))
    y = Out(dev, st, M * N * 2)
    ws = Out(dev, st, 1024)
    with pytest.raises(qgemm.QGemmError) as e:  # workspace below one 256-column slab
        ops.w4a16GemmGroupedPrefill(dev_array(gpu, x), wt, dev_array(gpu, sc), y, M, N, K, ws,
                                    1024, group_size=G)
    assert e.value.status == qgemm._lib.ERR_INVALID_ARG
    with pytest.raises(qgemm.QGemmError) as e:  # K % 8 != 0
        ops.w4a16GemmGroupedPrefill(dev_array(gpu, x), wt, dev_array(gpu, sc), y, M, N, 20, ws,
                                    1024, group_size=4)
    assert e.value.status == qgemm._lib.ERR_UNSUPPORTED
    with pytest.raises(qgemm.QGemmError) as e:
        ops.gemmBf16NK(8, 8, 8, 16, 16, 12)  # K % 8 != 0
    assert e.value.status == qgemm._lib.ERR_UNSUPPORTED
    st.sync()
