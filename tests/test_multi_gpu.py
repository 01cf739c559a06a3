"""Column-sharded W8A8 with its output all-gather on two GPUs, one process per GPU.

qgemm_w8a8_gemm_allgather_bf16 runs each rank's GEMM slice chunk by chunk of M and
all-gathers every chunk over NCCL while the next chunk's GEMM runs (NCCLOps.scala:302-320
is the reference's all-gather); qgemm_w8a8_gemm_allgather_window_bf16 instead copies each
chunk into the peers' registered output windows; qgemm_w8a8_gemm_allgather_fused_bf16
stores each output chunk into every rank's window from the GEMM's own epilogue (TMA
stores over NVLink).  Every rank must end with the whole [M, N] output, bit for bit the
unsharded product from the oracle.  Skipped with fewer than two GPUs.
"""
import os
import sys

import numpy as np
import pytest
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CASES = [  # M, N, K, chunk_rows
    (300, 512, 256, 64),     # five chunks, the last one 44 rows
    (256, 1024, 512, 1000),  # one chunk
    (130, 528, 96, 16),      # many chunks; 264 columns per rank
]


def _rank_main(rank, world, q_id, q_out):
    sys.path[:0] = [ROOT, os.path.join(ROOT, "cuda-triton-scala_b200")]
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    import ctypes
    import qgemm
    import qgemm._lib as L
    import qgemm.synthetic as syn
    dev = qgemm.Device(rank)
    s, cs = dev.stream(), dev.stream()
    uid = ctypes.create_string_buffer(128)
    if rank == 0:
        L.call("qgemm_comm_unique_id", uid)
        for _ in range(world - 1):
            q_id.put(bytes(uid.raw))
    else:
        uid = ctypes.create_string_buffer(q_id.get(timeout=60), 128)
    comm = ctypes.c_void_p()
    L.call("qgemm_comm_init", dev.handle, uid, rank, world, ctypes.byref(comm))
    results, errors = [], []
    try:
        for M, N, K, R in CASES:
            A, B, sA, sB = syn.w8a8_inputs(M, N, K, seed=M + N + K)
            n0, n1 = qgemm.shard_columns(N, world, rank, 8)
            bufs = [qgemm.Buffer.from_numpy(dev, s, a) for a in
                    (A, np.ascontiguousarray(B[:, n0:n1]), sA, np.ascontiguousarray(sB[n0:n1]))]
            out = qgemm.Buffer(dev, M * N * 2)
            wb = L.lib().qgemm_w8a8_allgather_work_bytes(world, min(R, M), n1 - n0)
            work = qgemm.Buffer(dev, wb)
            args = [b.address for b in bufs]
            L.call("qgemm_w8a8_gemm_allgather_bf16", comm, s.handle, cs.handle, args[0], args[1],
                   qgemm.B_KN, args[2], args[3], out.address, M, n1 - n0, K, R, work.address, wb)
            s.sync()
            y = out.to_numpy(s, np.uint16, (M, N))
            # the registered-window form, twice into the same window
            win_buf = qgemm.Buffer(dev, M * N * 2)
            s.memset(win_buf.address, 0, M * N * 2)
            win = ctypes.c_void_p()
            L.call("qgemm_comm_window_register", comm, s.handle, win_buf.address, M * N * 2,
                   ctypes.byref(win))
            ys = []
            for _ in range(2):
                L.call("qgemm_w8a8_gemm_allgather_window_bf16", win, s.handle, cs.handle,
                       args[0], args[1], qgemm.B_KN, args[2], args[3], M, n1 - n0, K, R)
                ys.append(win_buf.to_numpy(s, np.uint16, (M, N)))
            s.sync()
            cs.sync()
            # the fused form, twice, each time into a window filled with 0xFFFF first; a
            # shard of N % 16 == 8 columns has no tcgen05 GEMM on [K,N] weights, and
            # every rank refuses it before any collective
            if (n1 - n0) % 16 == 0:
                for _ in range(2):
                    s.memset(win_buf.address, 0xFF, M * N * 2)
                    L.call("qgemm_w8a8_gemm_allgather_fused_bf16", win, s.handle, args[0],
                           args[1], qgemm.B_KN, args[2], args[3], M, n1 - n0, K)
                    ys.append(win_buf.to_numpy(s, np.uint16, (M, N)))
            else:
                assert L.try_call("qgemm_w8a8_gemm_allgather_fused_bf16", win, s.handle,
                                  args[0], args[1], qgemm.B_KN, args[2], args[3], M, n1 - n0,
                                  K) == L.ERR_UNSUPPORTED
            s.sync()
            L.call("qgemm_comm_window_release", win)
            results.append((y, *ys))
        # refusals, made identically on every rank before any collective
        M, N, K, R = CASES[0]
        st1 = L.try_call("qgemm_w8a8_gemm_allgather_bf16", comm, s.handle, s.handle, 16, 16,
                         qgemm.B_KN, 16, 16, 16, M, N // world, K, R, 256, 1 << 20)
        st2 = L.try_call("qgemm_w8a8_gemm_allgather_bf16", comm, s.handle, cs.handle, 16, 16,
                         qgemm.B_KN, 16, 16, 16, M, N // world, K, R, 256, 64)
        # K % 16 != 0: no tcgen05 GEMM, so the fused form refuses before any collective
        win_buf = qgemm.Buffer(dev, M * N * 2)
        win = ctypes.c_void_p()
        L.call("qgemm_comm_window_register", comm, s.handle, win_buf.address, M * N * 2,
               ctypes.byref(win))
        st3 = L.try_call("qgemm_w8a8_gemm_allgather_fused_bf16", win, s.handle, 16, 16,
                         qgemm.B_KN, 16, 16, M, N // world, 8)
        L.call("qgemm_comm_window_release", win)
        errors = [st1, st2, st3]
        q_out.put((rank, results, errors))
    except Exception as e:  # report instead of leaving the parent waiting
        q_out.put((rank, None, repr(e)))
    finally:
        s.sync()
        cs.sync()
        L.call("qgemm_comm_destroy", comm)


@pytest.mark.gpu
def test_pipelined_gemm_allgather_matches_full(oracle):
    import qgemm
    import qgemm._lib as L
    import qgemm.synthetic as syn
    if qgemm.device_count() < 2:
        pytest.skip("needs two GPUs")
    world = 2
    ctx = mp.get_context("spawn")
    q_id, q_out = ctx.Queue(), ctx.Queue()
    procs = [ctx.Process(target=_rank_main, args=(r, world, q_id, q_out)) for r in range(world)]
    for p in procs:
        p.start()
    try:
        res = sorted(q_out.get(timeout=240) for _ in range(world))
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    for rank, results, errors in res:
        assert results is not None, f"rank {rank}: {errors}"
        for (M, N, K, _), ys in zip(CASES, results):
            A, B, sA, sB = syn.w8a8_inputs(M, N, K, seed=M + N + K)
            yo, _ = oracle.w8a32_gemm(B, sB, A, sA)
            for y in ys:  # gather buffers, the window (twice), the fused form (twice)
                np.testing.assert_array_equal(y, oracle.bf16_rne(yo))
        assert errors == [L.ERR_INVALID_ARG, L.ERR_INVALID_ARG, L.ERR_UNSUPPORTED]
    for p in procs:
        assert p.exitcode == 0


def test_allgather_work_bytes():
    import qgemm._lib as L
    assert L.lib().qgemm_w8a8_allgather_work_bytes(2, 64, 256) == 2 * 2 * 64 * 256 * 2
    assert L.lib().qgemm_w8a8_allgather_work_bytes(0, 64, 256) == 0


def _rank_main_facade(rank, world, q_id, q_out):
    """One case through qgemm.NCCLCommunicator / OutputWindow instead of raw calls."""
    sys.path[:0] = [ROOT, os.path.join(ROOT, "cuda-triton-scala_b200")]
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    import qgemm
    import qgemm.synthetic as syn
    from qgemm import NCCLCommunicator
    dev = qgemm.Device(rank)
    s, cs = dev.stream(), dev.stream()
    if rank == 0:
        uid = NCCLCommunicator.unique_id()
        for _ in range(world - 1):
            q_id.put(uid)
    else:
        uid = q_id.get(timeout=60)
    comm = NCCLCommunicator(dev, rank, world, uid)
    try:
        M, N, K, R = CASES[0]
        A, B, sA, sB = syn.w8a8_inputs(M, N, K, seed=M + N + K)
        n0, n1 = qgemm.shard_columns(N, world, rank, 8)
        bufs = [qgemm.Buffer.from_numpy(dev, s, a) for a in
                (A, np.ascontiguousarray(B[:, n0:n1]), sA, np.ascontiguousarray(sB[n0:n1]))]
        out = qgemm.Buffer(dev, M * N * 2)
        wb = NCCLCommunicator.gemmAllGatherWorkBytes(world, R, n1 - n0)
        work = qgemm.Buffer(dev, wb)
        comm.w8a8GemmAllGather(s, cs, *bufs, out, M, n1 - n0, K, R, work, wb)
        y = out.to_numpy(s, np.uint16, (M, N))
        win_buf = qgemm.Buffer(dev, M * N * 2)
        win = comm.registerWindow(s, win_buf, M * N * 2)
        win.w8a8GemmAllGather(s, cs, *bufs, M, n1 - n0, K, R)
        yw = win_buf.to_numpy(s, np.uint16, (M, N))
        cs.sync()
        s.memset(win_buf.address, 0xFF, M * N * 2)
        win.w8a8GemmAllGatherFused(s, *bufs, M, n1 - n0, K)
        yf = win_buf.to_numpy(s, np.uint16, (M, N))
        win.release()
        q_out.put((rank, [(y, yw, yf)], []))
    except Exception as e:
        q_out.put((rank, None, repr(e)))
    finally:
        s.sync()
        cs.sync()
        comm.destroy()


@pytest.mark.gpu
def test_communicator_facade_matches_full(oracle):
    import qgemm
    import qgemm.synthetic as syn
    if qgemm.device_count() < 2:
        pytest.skip("needs two GPUs")
    world = 2
    ctx = mp.get_context("spawn")
    q_id, q_out = ctx.Queue(), ctx.Queue()
    procs = [ctx.Process(target=_rank_main_facade, args=(r, world, q_id, q_out))
             for r in range(world)]
    for p in procs:
        p.start()
    try:
        res = sorted(q_out.get(timeout=240) for _ in range(world))
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    M, N, K, _ = CASES[0]
    A, B, sA, sB = syn.w8a8_inputs(M, N, K, seed=M + N + K)
    yo, _ = oracle.w8a32_gemm(B, sB, A, sA)
    for rank, results, err in res:
        assert results is not None, f"rank {rank}: {err}"
        for y in results[0]:
            np.testing.assert_array_equal(y, oracle.bf16_rne(yo))
    for p in procs:
        assert p.exitcode == 0
