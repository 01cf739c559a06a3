"""W4A16 on the GPU against the CPU oracle.

* reference entry point (QuantizedGemmOps.w4a16Gemm, QuantizedGemmOps.scala:218-247):
  bit-exact, same per-element fp32 order;
* group-wise decode path (bf16 x, per-group bf16 scales, zero point):
  - tensor-core fast path: max elementwise relative error <= 1e-2 on bf16
    outputs (helpers.rel_err: |y-r| / max(|r|, 1e-2*rms(r)));
  - any-shape CUDA-core path: bit-exact (same order as the oracle).
"""
import numpy as np
import pytest

import qgemm.synthetic as syn
from helpers import Out, dev_array, rel_err

pytestmark = pytest.mark.gpu

TOL_BF16 = 1e-2


def grouped(gpu, x, wq, sc, M, N, K, G, zp=8):
    dev, st, ops = gpu
    y = Out(dev, st, M * N * 2)
    ops.w4a16GemmGrouped(dev_array(gpu, x), dev_array(gpu, wq), dev_array(gpu, sc), y, M, N, K,
                         zero_point=zp, group_size=G)
    st.sync()
    return y.read(np.uint16, (M, N))


def tiled(gpu, x, wq, sc, M, N, K, G, zp=8):
    """Prepack once, then the tiled fast path."""
    dev, st, ops = gpu
    wt = Out(dev, st, ops.w4TiledBytes(K, N))
    ops.prepackW4Tiled(dev_array(gpu, wq), wt, K, N)
    y = Out(dev, st, M * N * 2)
    ops.w4a16GemmGroupedTiled(dev_array(gpu, x), wt, dev_array(gpu, sc), y, M, N, K,
                              zero_point=zp, group_size=G)
    st.sync()
    return y.read(np.uint16, (M, N))


def tiled_layout_numpy(wq, K, N):
    """The documented tiled layout: tiled[t][k][j] = byte 32*t + j of row k (64-column tiles)."""
    rows = wq.view(np.uint8).reshape(K, N // 2)
    nt = (N + 63) // 64
    pad = np.zeros((K, nt * 32), np.uint8)
    pad[:, : N // 2] = rows
    return pad.reshape(K, nt, 32).transpose(1, 0, 2).copy()


@pytest.mark.parametrize("K,N", [(64, 512), (48, 8 * 41), (16, 14336), (128, 264)])
def test_prepack_w4_tiled_layout(gpu, K, N):
    dev, st, ops = gpu
    _, wq, _ = syn.w4a16_inputs(1, N, K, group=16, seed=K + N)
    nbytes = ops.w4TiledBytes(K, N)
    assert nbytes == ((N + 63) // 64) * K * 32
    wt = Out(dev, st, nbytes)
    ops.prepackW4Tiled(dev_array(gpu, wq), wt, K, N)
    st.sync()
    got = wt.read(np.uint8, ((N + 63) // 64, K, 32))
    np.testing.assert_array_equal(got, tiled_layout_numpy(wq, K, N))


def frag(gpu, x, wq, sc, M, N, K, G, zp=8):
    """Prepack once into fragment order, then the frag decode path."""
    dev, st, ops = gpu
    wf = Out(dev, st, ops.w4FragBytes(K, N))
    ops.prepackW4Frag(dev_array(gpu, wq), wf, K, N)
    y = Out(dev, st, M * N * 2)
    ops.w4a16GemmGroupedFrag(dev_array(gpu, x), wf, dev_array(gpu, sc), y, M, N, K,
                             zero_point=zp, group_size=G)
    st.sync()
    return y.read(np.uint16, (M, N))


def frag_layout_numpy(wq, K, N):
    """The documented fragment order: unit (c, kb) = columns 8c..8c+7 x rows
    128kb..128kb+127; lane 4g+t, word s holds column 8c+g at rows 128kb + 32s + 8t +
    {0, 4, 2, 6, 1, 5, 3, 7}, nibble i at bits 4i.."""
    nkb = (K + 127) // 128
    q = (wq[:, :, None] >> (4 * np.arange(8, dtype=np.uint32))) & 0xF   # [K, N/8, 8]
    q = q.reshape(K, N).astype(np.uint32)
    qp = np.zeros((nkb * 128, N), np.uint32)
    qp[:K] = q
    g, t = np.arange(32) // 4, np.arange(32) % 4
    offs = np.array([0, 4, 2, 6, 1, 5, 3, 7])
    out = np.zeros((N // 8, nkb, 32, 4), np.uint32)
    for kb in range(nkb):
        for s in range(4):
            rows = kb * 128 + 32 * s + 8 * t[:, None] + offs[None, :]    # [32 lanes, 8 nibbles]
            for c in range(N // 8):
                vals = qp[rows, 8 * c + g[:, None]]                        # [32, 8]
                out[c, kb, :, s] = (vals << (4 * np.arange(8, dtype=np.uint32))).sum(axis=1)
    return out


@pytest.mark.parametrize("K,N", [(128, 64), (160, 24), (4096, 16)])
def test_prepack_w4_frag_layout(gpu, K, N):
    dev, st, ops = gpu
    _, wq, _ = syn.w4a16_inputs(1, N, K, group=32, seed=K + N)
    nbytes = ops.w4FragBytes(K, N)
    assert nbytes == (N // 8) * ((K + 127) // 128) * 512
    wf = Out(dev, st, nbytes)
    ops.prepackW4Frag(dev_array(gpu, wq), wf, K, N)
    st.sync()
    got = wf.read(np.uint32, (N // 8, (K + 127) // 128, 32, 4))
    np.testing.assert_array_equal(got, frag_layout_numpy(wq, K, N))


@pytest.mark.parametrize("M,N,K,G,zp", [
    (1, 14336, 4096, 128, 8),    # decode shape
    (4, 14336, 4096, 128, 0),
    (16, 14336, 4096, 128, 8),   # column pairs, one 16-row pass
    (3, 1000, 512, 64, 8),       # fewer column groups than SMs on some CTAs, G = 64
    (1, 4104, 4128, 32, 8),      # K not a multiple of 128, G = 32
    (2, 4096, 8192, 256, 15),    # eight blocks per warp, G = 256
    (1, 22016, 4096, 128, 8),    # 19 column groups on some CTAs
    (5, 8, 32, 32, 8),           # one column group, one partial block, two passes
    # more than 4 rows, N % 16 == 0: 16-column pairs, 16-row passes
    (8, 4096, 4096, 64, 8),      # one 8-row tile
    (12, 4112, 1024, 32, 3),     # 12 of 16 rows, group 32, 257 pairs
    (16, 1024, 4128, 32, 8),     # K not a multiple of 128
    (33, 2048, 2048, 128, 8),    # passes of 16, 16 and 1 rows
    (2, 131072, 512, 128, 8),    # wide N: the columns go out in several chunks
    (16, 65536, 1024, 64, 8),    # wide N on column pairs: several chunks
    # 17 to 32 rows a pass, or K past 8192: the K-split cluster kernel
    (32, 12288, 4096, 128, 8),   # Llama-2-7B qkv, one 32-row pass
    (32, 4096, 11008, 128, 8),   # Llama-2-7B down projection, K > 8192
    (1, 4096, 11008, 128, 8),    # one row, K > 8192 (8-row tile)
    (24, 22016, 4096, 128, 8),   # 24 of 32 rows, 1376 pairs
    (17, 1008, 2048, 64, 3),     # 17 rows, G = 64, 63 pairs
    (32, 4112, 4128, 32, 8),     # G = 32, K not a multiple of 128, 257 pairs
    (40, 2048, 16384, 256, 15),  # K = 16384 (the limit), G = 256, passes of 32 and 8
    (9, 48, 9984, 128, 8),       # three pairs, K > 8192
    (64, 512, 1024, 128, 0),     # two full 32-row passes
    (16, 1024, 6144, 128, 8),    # 16 rows, K past the 16-row kernel's 4096
    (32, 131072, 512, 128, 8),   # wide N: the pairs go out in several launches
])
def test_grouped_frag_path(gpu, oracle, M, N, K, G, zp):
    x, wq, sc = syn.w4a16_inputs(M, N, K, group=G, seed=M * 5 + N + K + G)
    y = frag(gpu, x, wq, sc, M, N, K, G, zp)
    ref, _ = oracle.w4a16_grouped(wq, sc, zp, G, x)
    err = rel_err(syn.bf16_to_float(y), ref)
    assert err <= TOL_BF16, err


@pytest.mark.parametrize("M,N", [(4, 2048), (16, 2048), (32, 2048)])
def test_frag_activation_magnitudes(gpu, oracle, M, N):
    """Rows of very different magnitude (bf16 values from 1e-30 to 1e30, and an all-zero
    row): the frag kernels' fp16 arithmetic scales activations by powers of two, so the
    results stay within the tolerance at every magnitude."""
    K, G = 2048, 128
    x, wq, sc = syn.w4a16_inputs(M, N, K, group=G, seed=83)
    xf = syn.bf16_to_float(x).astype(np.float32)
    mags = np.array([1.0, 1e30, 1e-30, 0.0, 3e4, 1e-5, 7e12, 2.0] * 4, np.float32)[:M]
    xf = xf * mags[:, None]
    xf[M - 1, : K // 2] *= 1e6  # one row whose first half is much larger than its second
    xb = syn.bf16_bits(xf)
    y = frag(gpu, xb, wq, sc, M, N, K, G)
    ref, _ = oracle.w4a16_grouped(wq, sc, 8, G, xb)
    got = syn.bf16_to_float(y).astype(np.float64)
    for m in range(M):  # per row: the floor of rel_err scales with the row
        assert rel_err(got[m], ref[m]) <= TOL_BF16, (m, mags[m])


def test_frag_cluster_deterministic(gpu):
    """The cluster kernel adds the K slices' partial sums in rank order: repeat runs are
    bit-identical."""
    M, N, K, G = 32, 4096, 11008, 128
    x, wq, sc = syn.w4a16_inputs(M, N, K, group=G, seed=66)
    a = frag(gpu, x, wq, sc, M, N, K, G)
    b = frag(gpu, x, wq, sc, M, N, K, G)
    np.testing.assert_array_equal(a, b)


def test_frag_deterministic_and_matches_tiled(gpu):
    M, N, K, G = 4, 14336, 4096, 128
    x, wq, sc = syn.w4a16_inputs(M, N, K, group=G, seed=64)
    a = frag(gpu, x, wq, sc, M, N, K, G)
    b = frag(gpu, x, wq, sc, M, N, K, G)
    np.testing.assert_array_equal(a, b)
    c = syn.bf16_to_float(tiled(gpu, x, wq, sc, M, N, K, G)).astype(np.float64)
    assert rel_err(syn.bf16_to_float(a).astype(np.float64), c) <= TOL_BF16


@pytest.mark.parametrize("K,G,N", [(480, 48, 64), (8320, 128, 72), (16512, 128, 64)])
def test_frag_rejects_unsupported_shapes(gpu, K, G, N):
    """Group 48 (not 32, 64 or a multiple of 128), K > 8192 with N not a multiple of 16,
    and K > 16384 are refused."""
    import qgemm
    dev, st, ops = gpu
    x, wq, sc = syn.w4a16_inputs(1, N, K, group=G, seed=65)
    wf = Out(dev, st, ops.w4FragBytes(K, N))
    ops.prepackW4Frag(dev_array(gpu, wq), wf, K, N)
    y = Out(dev, st, N * 2)
    with pytest.raises(qgemm.QGemmError) as e:
        ops.w4a16GemmGroupedFrag(dev_array(gpu, x), wf, dev_array(gpu, sc), y, 1, N, K,
                                 group_size=G)
    assert e.value.status == qgemm._lib.ERR_UNSUPPORTED
    st.sync()


def test_reference_entry_point(gpu, oracle):
    dev, st, ops = gpu
    M, N, K = 64, 512, 512
    rng = np.random.default_rng(21)
    wb = rng.integers(0, 256, size=K * N // 2, dtype=np.uint8)
    sw = rng.uniform(0.005, 0.02, N).astype(np.float32)
    x = rng.standard_normal((M, K), dtype=np.float32)
    y = Out(dev, st, M * N * 4)
    ops.w4a16Gemm(dev_array(gpu, wb), dev_array(gpu, sw), dev_array(gpu, x), y, M, N, K)
    st.sync()
    ref = oracle.w4a16_gemm(wb, sw, x, N)
    np.testing.assert_array_equal(y.read(np.uint32, (M, N)), ref.view(np.uint32))


def test_reference_entry_point_odd_n(gpu, oracle):
    import os
    g = np.load(os.path.join(os.path.dirname(__file__), "golden", "golden.npz"))
    dev, st, ops = gpu
    x = g["w4a16_x"]
    M, K = x.shape
    N = int(g["w4a16_N"])
    y = Out(dev, st, M * N * 4)
    ops.w4a16Gemm(dev_array(gpu, g["w4a16_w"]), dev_array(gpu, g["w4a16_sw"]), dev_array(gpu, x),
                  y, M, N, K)
    st.sync()
    np.testing.assert_array_equal(y.read(np.uint32, (M, N)), g["w4a16_y"].view(np.uint32))


@pytest.mark.parametrize("M", [1, 4, 16])
def test_grouped_config3(gpu, oracle, M):
    N, K, G = 14336, 4096, 128
    x, wq, sc = syn.w4a16_inputs(M, N, K, group=G, seed=30 + M)
    y = grouped(gpu, x, wq, sc, M, N, K, G)
    ref, _ = oracle.w4a16_grouped(wq, sc, 8, G, x)
    err = rel_err(syn.bf16_to_float(y), ref)
    assert err <= TOL_BF16, err


@pytest.mark.parametrize("M,N,K,G,zp", [(3, 400, 512, 64, 8), (20, 256, 1024, 128, 3),
                                        (8, 128, 256, 128, 8), (2, 2048, 4096, 32, 0),
                                        (9, 1040, 2048, 128, 15)])
def test_grouped_fast_path_shapes(gpu, oracle, M, N, K, G, zp):
    x, wq, sc = syn.w4a16_inputs(M, N, K, group=G, seed=M + N + K)
    y = grouped(gpu, x, wq, sc, M, N, K, G, zp)
    ref, _ = oracle.w4a16_grouped(wq, sc, zp, G, x)
    err = rel_err(syn.bf16_to_float(y), ref)
    assert err <= TOL_BF16, err


@pytest.mark.parametrize("M,N,K,G,zp", [
    (1, 32, 512, 16, 8),         # one partial tile, group 16 (32 scale rows per stage)
    (5, 8192 + 32, 512, 16, 8),  # partial last tile
    (16, 4096, 1024, 64, 4),     # few tiles: K split over a 2-CTA cluster
    (2, 2048, 2048, 32, 8),      # 32 tiles: K split over a 4-CTA cluster
    (7, 3072, 2048, 256, 8),     # group larger than a warp's rows
    (2, 1024, 2048, 512, 8),     # group as large as a stage
    (33, 512, 1024, 128, 8),     # three M passes (16 + 16 + 1)
    (1, 14336, 4096, 128, 0),    # decode shape, other zero point
    (4, 14336, 4096, 128, 8),
    (16, 14336, 4096, 128, 8),
    (3, 1000, 512, 64, 8),       # N not a multiple of 64
    (1, 4096, 11008, 128, 8),    # Llama-2-7B down projection: K not a multiple of 512
    (32, 4096, 11008, 128, 8),   # two 16-row passes
    (2, 264, 1040, 16, 8),       # 16-row last stage, group 16
    (1, 11008, 4096, 128, 8),
])
def test_grouped_tiled_path(gpu, oracle, M, N, K, G, zp):
    x, wq, sc = syn.w4a16_inputs(M, N, K, group=G, seed=M * 3 + N + K + G)
    y = tiled(gpu, x, wq, sc, M, N, K, G, zp)
    ref, _ = oracle.w4a16_grouped(wq, sc, zp, G, x)
    err = rel_err(syn.bf16_to_float(y), ref)
    assert err <= TOL_BF16, err


def test_grouped_tiled_repeat_counters_reset(gpu):
    """Split-K arrival counters return to zero: repeated calls, alternating
    shapes, give identical results."""
    a = syn.w4a16_inputs(4, 14336, 4096, group=128, seed=60)
    b = syn.w4a16_inputs(16, 6144, 2048, group=64, seed=61)
    ya = [tiled(gpu, *a, 4, 14336, 4096, 128) for _ in range(2)]
    yb = tiled(gpu, *b, 16, 6144, 2048, 64)
    ya.append(tiled(gpu, *a, 4, 14336, 4096, 128))
    yb2 = tiled(gpu, *b, 16, 6144, 2048, 64)
    np.testing.assert_array_equal(ya[0], ya[1])
    np.testing.assert_array_equal(ya[0], ya[2])
    np.testing.assert_array_equal(yb, yb2)


@pytest.mark.parametrize("M,N,K,G", [(2, 24, 40, 8), (3, 8, 16, 16), (1, 40, 30, 10)])
def test_grouped_simt_path_exact(gpu, oracle, M, N, K, G):
    x, wq, _ = syn.w4a16_inputs(M, N, K, group=K, seed=7)
    rng = np.random.default_rng(8)
    sc = syn.bf16_bits(rng.uniform(0.005, 0.02, (K // G, N)).astype(np.float32))
    y = grouped(gpu, x, wq, sc, M, N, K, G)
    _, refb = oracle.w4a16_grouped(wq, sc, 8, G, x)
    np.testing.assert_array_equal(y, refb)


def test_grouped_deterministic(gpu):
    M, N, K, G = 4, 14336, 4096, 128
    x, wq, sc = syn.w4a16_inputs(M, N, K, group=G, seed=40)
    a = grouped(gpu, x, wq, sc, M, N, K, G)
    b = grouped(gpu, x, wq, sc, M, N, K, G)
    np.testing.assert_array_equal(a, b)


@pytest.mark.parametrize("K,G", [(480, 48), (768, 192)])
def test_tiled_rejects_unsupported_shapes(gpu, K, G):
    """Groups that do not tile 512-row stages (48, 192) are refused, not miscomputed."""
    import qgemm
    dev, st, ops = gpu
    x, wq, sc = syn.w4a16_inputs(1, 256, K, group=G, seed=63)
    wt = Out(dev, st, ops.w4TiledBytes(K, 256))
    ops.prepackW4Tiled(dev_array(gpu, wq), wt, K, 256)
    y = Out(dev, st, 256 * 2)
    with pytest.raises(qgemm.QGemmError) as e:
        ops.w4a16GemmGroupedTiled(dev_array(gpu, x), wt, dev_array(gpu, sc), y, 1, 256, K,
                                  group_size=G)
    assert e.value.status == qgemm._lib.ERR_UNSUPPORTED
    st.sync()


def test_tiled_and_canonical_agree(gpu):
    M, N, K, G = 8, 4096, 2048, 128
    x, wq, sc = syn.w4a16_inputs(M, N, K, group=G, seed=62)
    a = syn.bf16_to_float(tiled(gpu, x, wq, sc, M, N, K, G)).astype(np.float64)
    b = syn.bf16_to_float(grouped(gpu, x, wq, sc, M, N, K, G)).astype(np.float64)
    assert rel_err(a, b) <= TOL_BF16


def test_grouped_rejects_bad_args(gpu):
    import qgemm
    dev, st, ops = gpu
    with pytest.raises(qgemm.QGemmError) as e:
        ops.w4a16GemmGrouped(8, 8, 8, 8, 1, 12, 64, group_size=64)  # N % 8 != 0
    assert e.value.status == qgemm._lib.ERR_INVALID_ARG
    with pytest.raises(qgemm.QGemmError) as e:
        ops.w4a16GemmGrouped(8, 8, 8, 8, 1, 16, 100, group_size=64)  # K % G != 0
    assert e.value.status == qgemm._lib.ERR_INVALID_ARG
    with pytest.raises(qgemm.QGemmError) as e:
        ops.w4a16GemmGrouped(8, 8, 8, 8, 1, 16, 64, group_size=64, zero_point=16)
    assert e.value.status == qgemm._lib.ERR_INVALID_ARG
    st.sync()


def test_frag_blob_round_trip_through_the_device(gpu, tmp_path):
    """Fragment-ordered weights saved as a blob and loaded straight into device memory
    decode to the same bits as the freshly prepacked ones."""
    from qgemm import blob
    dev, st, ops = gpu
    M, N, K, G = 2, 1024, 2048, 128
    x, wq, sc = syn.w4a16_inputs(M, N, K, group=G, seed=82)
    nbytes = ops.w4FragBytes(K, N)
    wf = Out(dev, st, nbytes)
    ops.prepackW4Frag(dev_array(gpu, wq), wf, K, N)
    st.sync()
    p = str(tmp_path / "layer_frag.qgb")
    blob.save(p, "w4_frag", K, N, wf.read(np.uint8, (nbytes,)), sc, group_size=G, zero_point=8)
    wf2 = Out(dev, st, nbytes)
    sc2 = Out(dev, st, sc.nbytes)
    blob.load_to_device(st, p, wf2, nbytes, sc2, sc.nbytes)
    ys = []
    for w_, s_ in ((wf, dev_array(gpu, sc)), (wf2, sc2)):
        y = Out(dev, st, M * N * 2)
        ops.w4a16GemmGroupedFrag(dev_array(gpu, x), w_, s_, y, M, N, K, group_size=G)
        st.sync()
        ys.append(y.read(np.uint16, (M, N)).copy())
    np.testing.assert_array_equal(ys[0], ys[1])


def test_blob_round_trip_through_the_device(gpu, tmp_path):
    """Prepacked weights saved as a blob and loaded straight into device memory run
    the tiled GEMM to the same bits as the freshly prepacked ones."""
    from qgemm import blob
    dev, st, ops = gpu
    M, N, K, G = 4, 1024, 2048, 128
    x, wq, sc = syn.w4a16_inputs(M, N, K, group=G, seed=81)
    nbytes = ops.w4TiledBytes(K, N)
    wt = Out(dev, st, nbytes)
    ops.prepackW4Tiled(dev_array(gpu, wq), wt, K, N)
    st.sync()
    p = str(tmp_path / "layer.qgb")
    blob.save(p, "w4_tiled", K, N, wt.read(np.uint8, (nbytes,)), sc, group_size=G, zero_point=8)
    wt2 = Out(dev, st, nbytes)
    sc2 = Out(dev, st, sc.nbytes)
    blob.load_to_device(st, p, wt2, nbytes, sc2, sc.nbytes)
    ys = []
    for w_, s_ in ((wt, dev_array(gpu, sc)), (wt2, sc2)):
        y = Out(dev, st, M * N * 2)
        ops.w4a16GemmGroupedTiled(dev_array(gpu, x), w_, s_, y, M, N, K, group_size=G)
        st.sync()
        ys.append(y.read(np.uint16, (M, N)).copy())
    np.testing.assert_array_equal(ys[0], ys[1])
