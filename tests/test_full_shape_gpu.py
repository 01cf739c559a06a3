"""Parity at the full sizes of the multi-GPU and prefill workloads, on one GPU.

* W8A8 at M=16384, N=28672, K=8192 (the column-sharded GEMM's whole problem,
  QuantizedGemmOps.scala:102-113): the tensor-core kernel equals the CUDA-core kernel
  over every one of the 470 M outputs (int32 accumulators and bf16), and the CPU oracle
  over 256 seeded full rows and the four corner 256 x 256 tiles, bit for bit.
* W4A16 prefill at M=16384 on the Llama-2-7B gate+up (K=4096, N=22016, fragment-ordered
  weights) and down (K=11008, N=4096, tiled weights) projections: against the oracle
  (QuantizedGemmOps.scala:229-245 with groups of 128) on 256 seeded rows plus the first
  and last rows, floored max relative error <= 1e-2 (the plain one is printed beside it);
  with the one-term expansion, the forward error max |y - exact| / sum_k |x w| <= 2^-8 +
  K 2^-24 on the same rows (the elementwise figures are printed).
"""
import numpy as np
import pytest

import qgemm
import qgemm.synthetic as syn
from helpers import gemm_bound_ratio, rel_errs

pytestmark = pytest.mark.gpu

TOL_BF16 = 1e-2


def test_w8a8_sharded_problem_full_shape(gpu, oracle):
    import torch
    dev, st, ops = gpu
    M, N, K = 16384, 28672, 8192
    rng = np.random.default_rng(5)
    A = rng.integers(-127, 128, size=(M, K), dtype=np.int8)
    B = rng.integers(-127, 128, size=(K, N), dtype=np.int8)
    sA = rng.uniform(0.001, 0.01, size=M).astype(np.float32)
    sB = rng.uniform(0.001, 0.01, size=N).astype(np.float32)
    dA, dB, dsA, dsB = (torch.from_numpy(x).cuda() for x in (A, B, sA, sB))
    y_tc = torch.empty((M, N), dtype=torch.bfloat16, device="cuda")
    acc_tc = torch.empty((M, N), dtype=torch.int32, device="cuda")
    y_st = torch.empty_like(y_tc)
    acc_st = torch.empty_like(acc_tc)
    torch.cuda.synchronize()
    ops.w8a8Gemm(dA, dB, dsA, dsB, y_tc, M, N, K, acc_i32=acc_tc, algo=qgemm.ALGO_TCGEN05)
    ops.w8a8Gemm(dA, dB, dsA, dsB, y_st, M, N, K, acc_i32=acc_st, algo=qgemm.ALGO_SIMT)
    st.sync()
    assert torch.equal(acc_tc, acc_st), "tensor-core and CUDA-core int32 sums differ"
    assert torch.equal(y_tc.view(torch.int16), y_st.view(torch.int16)), "bf16 outputs differ"
    # the CPU oracle: 256 seeded full rows ...
    rows = np.sort(rng.choice(M, 256, replace=False))
    _, yb, acc = oracle.w8a8_gemm_rows(B, sB, A[rows], sA[rows], want_f32=False, want_acc=True)
    ridx = torch.from_numpy(rows).cuda()
    np.testing.assert_array_equal(acc_tc[ridx].cpu().numpy(), acc)
    np.testing.assert_array_equal(y_tc[ridx].view(torch.int16).cpu().numpy().view(np.uint16), yb)
    # ... and the four corner 256 x 256 tiles
    for r0 in (0, M - 256):
        for c0 in (0, N - 256):
            Bc = np.ascontiguousarray(B[:, c0:c0 + 256])
            _, yb, acc = oracle.w8a8_gemm_rows(Bc, sB[c0:c0 + 256], A[r0:r0 + 256],
                                               sA[r0:r0 + 256], want_f32=False, want_acc=True)
            np.testing.assert_array_equal(acc_tc[r0:r0 + 256, c0:c0 + 256].cpu().numpy(), acc)
            got = y_tc[r0:r0 + 256, c0:c0 + 256].contiguous().view(torch.int16).cpu().numpy()
            np.testing.assert_array_equal(got.view(np.uint16), yb)


def llama_inputs(M, N, K, seed):
    rng = np.random.default_rng(seed)
    x = syn.bf16_bits(rng.standard_normal(size=(M, K), dtype=np.float32))
    q = rng.integers(0, 16, size=(K, N), dtype=np.uint8)
    wq = syn.pack_int4(q)
    sc = syn.bf16_bits(rng.uniform(0.005, 0.02, size=(K // 128, N)).astype(np.float32))
    return x, wq, sc, rng


@pytest.mark.parametrize("N,K,layout,one_term", [(22016, 4096, "frag", False),
                                                  (4096, 11008, "tiled", False),
                                                  (22016, 4096, "frag", True),
                                                  (4096, 11008, "frag", True)])
def test_w4a16_prefill_llama_full_shape(gpu, oracle, N, K, layout, one_term):
    import torch
    dev, st, ops = gpu
    M, G = 16384, 128
    x, wq, sc, rng = llama_inputs(M, N, K, seed=N + K)
    dx, dwq, dsc = (torch.from_numpy(a.view(np.int16) if a.dtype == np.uint16 else
                                     a.view(np.int32)).cuda() for a in (x, wq, sc))
    if layout == "frag":
        wt = torch.empty(ops.w4FragBytes(K, N), dtype=torch.uint8, device="cuda")
        torch.cuda.synchronize()
        ops.prepackW4Frag(dwq, wt, K, N)
        f = ops.w4a16GemmGroupedPrefillFrag
    else:
        wt = torch.empty(ops.w4TiledBytes(K, N), dtype=torch.uint8, device="cuda")
        torch.cuda.synchronize()
        ops.prepackW4Tiled(dwq, wt, K, N)
        f = ops.w4a16GemmGroupedPrefill
    ws_bytes = ops.w4PrefillWorkspaceBytes(K, N, one_term=one_term)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device="cuda")
    y = torch.empty((M, N), dtype=torch.int16, device="cuda")
    f(dx, wt, dsc, y, M, N, K, ws, ws_bytes, zero_point=8, group_size=G, one_term=one_term)
    st.sync()
    rows = np.unique(np.concatenate([rng.choice(M, 256, replace=False), [0, M - 1]]))
    ref, _ = oracle.w4a16_grouped(wq, sc, 8, G, np.ascontiguousarray(x[rows]))
    got = y[torch.from_numpy(rows).cuda()].cpu().numpy().view(np.uint16)
    floored, plain = rel_errs(syn.bf16_to_float(got), ref)
    print(f"prefill M={M} N={N} K={K} one_term={one_term}: floored max rel err "
          f"{floored:.3e}, plain {plain:.3e}")
    if not one_term:
        assert floored <= TOL_BF16, (floored, plain)
        return
    w = (syn.unpack_int4(wq, N).astype(np.float64) - 8) * \
        np.repeat(syn.bf16_to_float(sc).astype(np.float64), G, axis=0)
    ratio = gemm_bound_ratio(syn.bf16_to_float(got), syn.bf16_to_float(x[rows]), w)
    print(f"  one term forward error {ratio:.3e}")
    assert ratio <= 2.0 ** -8 + K * 2.0 ** -24, ratio
