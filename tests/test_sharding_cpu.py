"""Column-sharded W8A8 across ranks, host logic on CPU with the gloo backend.

Each rank takes its weight columns from qgemm_shard_columns, computes its slice
with the CPU oracle (the GPU kernel is bit-identical to it), the slices are
all-gathered into [world, M, n_local] exactly as qgemm_comm_allgather_bf16
lays them out, and rearranged the way qgemm_unshard_columns_bf16 does.  The
result must equal the unsharded GEMM bit for bit.  A second case checks that a
rank which dies before the collective makes its peers fail with an error
instead of hanging.
"""
import os
import socket
import sys

import numpy as np
import pytest
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _unshard(gathered: np.ndarray) -> np.ndarray:
    """[world][M][ncols] -> [M][world*ncols] (the unshard kernel's mapping)."""
    world, M, ncols = gathered.shape
    out = np.empty((M, world * ncols), gathered.dtype)
    for r in range(world):
        out[:, r * ncols:(r + 1) * ncols] = gathered[r]
    return out


def _worker(rank, world, port, M, N, K, q):
    sys.path[:0] = [ROOT, os.path.join(ROOT, "cuda-triton-scala_b200")]
    import torch
    import torch.distributed as dist
    import qgemm
    import qgemm.synthetic as syn
    from oracle import oracle
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        A, B, sA, sB = syn.w8a8_inputs(M, N, K, seed=5)   # same seed: A replicated
        n0, n1 = qgemm.shard_columns(N, world, rank, 16)
        _, yb = oracle.w8a8_gemm_rows(np.ascontiguousarray(B[:, n0:n1]), sB[n0:n1], A, sA,
                                      threads=1, want_f32=False)
        # gloo has no 16-bit integer type: carry the bf16 bit patterns as int32
        part = torch.from_numpy(yb.astype(np.int32))
        slabs = [torch.empty_like(part) for _ in range(world)]
        dist.all_gather(slabs, part)   # rank r's slab lands at index r, as in the NCCL gather
        gathered = torch.stack(slabs).numpy().astype(np.uint16)
        q.put((rank, n0, n1, gathered))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2])
def test_sharded_gemm_gather_matches_full(world, oracle):
    import qgemm.synthetic as syn
    M, N, K = 48, 256, 96
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, M, N, K, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=90) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    res.sort()
    bounds = [(n0, n1) for _, n0, n1, _ in res]
    assert bounds[0][0] == 0 and bounds[-1][1] == N
    full = _unshard(res[0][3])
    A, B, sA, sB = syn.w8a8_inputs(M, N, K, seed=5)
    yo, _ = oracle.w8a32_gemm(B, sB, A, sA)
    np.testing.assert_array_equal(full, oracle.bf16_rne(yo))
    # every rank received the same gathered buffer
    for r in res[1:]:
        np.testing.assert_array_equal(r[3], res[0][3])


def _dying_worker(rank, world, port, q):
    import datetime
    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=5))
    if rank == 1:
        os._exit(3)  # leaves between steps, with nothing in flight
    try:
        t = torch.zeros(4)
        dist.all_reduce(t)
        q.put((rank, "no error"))
    except Exception as e:  # the peer is gone: the collective must fail, not hang
        q.put((rank, type(e).__name__))


def test_dead_rank_surfaces_as_error():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_dying_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    rank, what = q.get(timeout=120)
    assert rank == 0 and what != "no error"
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()


def _failing_step_worker(rank, world, port, q):
    """Two steps of the sharded layer's host loop (a collective per step).  Rank 1's
    second step fails on the host before its collective (a stand-in for a failed launch)
    and the rank stays alive without joining; rank 0 must get an error from its
    collective within the process group's timeout, not wait for good."""
    import datetime
    import time
    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=4))
    t = torch.ones(8)
    dist.all_reduce(t)  # step 1 completes on both ranks
    if rank == 1:
        try:
            raise RuntimeError("launch failed")  # step 2 fails on the host
        except RuntimeError as e:
            q.put((rank, f"own error: {e}"))
        time.sleep(12)  # alive, never joins the collective
        os._exit(0)
    t0 = time.time()
    try:
        dist.all_reduce(t)
        q.put((rank, "no error", time.time() - t0))
    except Exception as e:
        q.put((rank, type(e).__name__, time.time() - t0))


def test_rank_failing_between_steps_surfaces_as_error():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_failing_step_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = {}
    for _ in range(2):
        item = q.get(timeout=120)
        got[item[0]] = item[1:]
    assert got[1][0].startswith("own error")
    what, waited = got[0]
    assert what != "no error" and waited < 60
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
