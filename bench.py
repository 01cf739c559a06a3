#!/usr/bin/env python
"""bench.py -- W8A8 GEMM TOPS and W4A16 GEMV HBM GB/s on B200, % of roofline.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Headline (`value`): the column-sharded W8A8 GEMM M=16384, N=28672, K=8192 (strong
scaling): rank r of N holds N/world weight columns and their per-channel scales, the
activations A and per-token scales are the same on every rank, each rank's bf16 output
block stays on its GPU.  One GPU runs the whole GEMM.  One step = one GEMM launch per
rank through libqgemm; value = 2*M*N*K per step over the slowest rank's time.

Also on the same line:
  roofline      the same kernel at 4096^3 on one GPU (the prefill-shaped GEMM) against
                the dense int8 tensor peak (2 x the measured burst bf16 rate)
  e2e           the headline through the C-ABI with host buffers: H2D of the step's
                activations + scales, the GEMM, D2H of this rank's bf16 output block
  parity        sampled rows of the headline output (and at N > 1, of every gathered
                form) against the CPU oracle, outside the timed regions
  allgather     (N > 1) the whole output on every rank: NCCL all-gather + unshard, and
                the GEMM + gather in one call (NCCL pipelined, copy-engine window)
  w8a8_4096     the 4096^3 GEMM itself: TOPS, cuBLASLt context, quantise + GEMM
  w4a16_decode  (N = 1) the W4A16 group-128 GEMV at M = 1, 4, 16, GB/s vs HBM
  cpu_baseline  (N = 1, rank 0) the CPU restatement on bounded samples (OpenMP and one
                thread): the headline GEMM on a row slice, the W4A16 decode GEMV
  clocks        NVML SM clock and throttle reasons sampled during the timed region
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "cuda-triton-scala_b200")
for _p in (ROOT, PKG):
    if _p not in sys.path:
        sys.path.insert(0, _p)

METRIC = "W8A8 GEMM TOPS & W4A16 GEMV HBM GB/s at 1/2/4/8 B200, % of roofline"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
# DRAM bytes (read + write) per launch from one `ncu --set full` capture of the same
# kernel on the same workload: the W8A8 pair kernel at 4096^3, the M = 1 decode on the
# fragment order, and the fp32 matmul's tf32 GEMM at 4096^3.
NCU_TRAFFIC_W8A8_4096 = 33675008 + 2621952
NCU_TRAFFIC_W4A16_M1 = 30306304 + 0
NCU_TRAFFIC_F32_GEMM_4096 = 985069568 + 61620736

# The column-sharded GEMM of the headline: M x N x K, weight columns cut in units of 256.
LARGE_M, LARGE_N, LARGE_K = 16384, 28672, 8192
SHARD_ALIGN = 256
SEED_A, SEED_B = 4321, 9000


def headline_config(world: int) -> dict:
    """The `config` of the headline, the same in both arms."""
    return {"workload": "w8a8_gemm M=16384 N=28672 K=8192, weight columns sharded over the "
                        "GPUs (N/world per rank, resident), activations replicated, "
                        "per-token x per-channel fp32 scales, bf16 output resident per rank, "
                        "B in the reference [K,N] layout",
            "M": LARGE_M, "N": LARGE_N, "K": LARGE_K, "parallelism": f"col{world}",
            "l2": "inputs larger than L2: A 134 MB + B shard >= 29 MB per rank > 126 MB"}


def parse_args():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=50)
    p.add_argument("--warmup", type=int, default=10)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline")
    p.add_argument("--no-llama", action="store_true", help="skip the Llama-shaped W4A16 stack")
    p.add_argument("--only", choices=["all", "w8a8", "large", "w4a16", "llama", "f32", "side",
                                      "prefill"],
                   default="all",
                   help="run one workload alone (for profiling); prints its own JSON line")
    p.add_argument("--as-world", type=int, default=1,
                   help="with --only large: run rank 0's shard of a W-GPU job on this GPU")
    p.add_argument("--profile", action="store_true",
                   help="with --only w8a8|w4a16|prefill: warmup + steps plain launches and "
                        "nothing else (no clock warm-up, no graphs), for ncu captures")
    p.add_argument("--rows", type=int, default=4096,
                   help="with --only prefill: activation rows of the prefill GEMM")
    return p.parse_args()


def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return d, "measured"
    except Exception:
        return dict(FALLBACK_PEAKS), "fallback"


# ---- clocks -----------------------------------------------------------------

class ClockSampler:
    """Samples SM clock and throttle reasons through NVML in a thread."""

    REASONS = {
        "hw_slowdown": "nvmlClocksEventReasonHwSlowdown",
        "hw_thermal_slowdown": "nvmlClocksEventReasonHwThermalSlowdown",
        "sw_thermal_slowdown": "nvmlClocksEventReasonSwThermalSlowdown",
        "sw_power_cap": "nvmlClocksEventReasonSwPowerCap",
        "hw_power_brake": "nvmlClocksEventReasonHwPowerBrakeSlowdown",
    }

    def __init__(self, torch_dev: int, period_s: float = 0.01):
        self.samples, self.reasons = [], set()
        self.max_mhz = None
        self.ok = False
        self.period = period_s
        self._stop = threading.Event()
        try:
            import pynvml as nv
            nv.nvmlInit()
            self.nv = nv
            import torch
            p = torch.cuda.get_device_properties(torch_dev)
            # torch reports the PCI location as integers; NVML wants "DDDDDDDD:BB:DD.F".
            bus = "%08X:%02X:%02X.0" % (int(p.pci_domain_id), int(p.pci_bus_id),
                                        int(p.pci_device_id))
            h = nv.nvmlDeviceGetHandleByPciBusId(bus.encode())
            self.h = h
            self.max_mhz = nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM)
            self.ok = True
        except Exception:
            self.ok = False

    def _run(self):
        nv = self.nv
        while not self._stop.is_set():
            try:
                mhz = nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM)
                util = nv.nvmlDeviceGetUtilizationRates(self.h).gpu
                r = nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                self.samples.append((mhz, util))
                for name, const in self.REASONS.items():
                    if r & getattr(nv, const, 0):
                        self.reasons.add(name)
            except Exception:
                pass
            time.sleep(self.period)

    def __enter__(self):
        if self.ok:
            self.t = threading.Thread(target=self._run, daemon=True)
            self.t.start()
        return self

    def __exit__(self, *a):
        if self.ok:
            self._stop.set()
            self.t.join()

    def summary(self):
        if not self.ok or not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons),
                    "samples": 0, "source": "nvml unavailable"}
        loaded = [m for m, u in self.samples if u > 0] or [m for m, _ in self.samples]
        return {"sm_mhz": statistics.median(loaded), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples),
                "samples_under_load": len(loaded), "source": "nvml"}


# ---- distributed plumbing ------------------------------------------------------

def dist_setup(n_gpus: int):
    import torch
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != n_gpus:
        raise SystemExit(f"--gpus {n_gpus} but WORLD_SIZE={world}: launch N>1 with torchrun")
    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=torch.device("cuda", local),
                                timeout=datetime.timedelta(seconds=300))
    return rank, world, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ---- workloads -------------------------------------------------------------------

def rand_i8(shape, gen):
    import torch
    return torch.randint(-127, 128, shape, dtype=torch.int8, device="cuda", generator=gen)


def rand_u(shape, lo, hi, gen):
    import torch
    return torch.rand(shape, dtype=torch.float32, device="cuda", generator=gen) * (hi - lo) + lo


def timed(fn, steps, world):
    """Barrier + sync, CUDA events around `steps` calls of fn on the current
    stream, sync + barrier; returns (max-over-ranks seconds, local seconds)."""
    import torch
    barrier(world)
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for i in range(steps):
        fn(i)
    e.record()
    torch.cuda.synchronize()
    barrier(world)
    local = s.elapsed_time(e) / 1e3
    return max_over_ranks(local, world), local


def w8a8_4096(ops, steps, warmup, clocks):
    """The 4096^3 GEMM (prefill shape, one GPU): 8 rotating input sets (256 MB > L2),
    `warmup` launches and about 20 ms more of them to raise the clocks, then `steps`
    launches timed with CUDA events on the launching stream (a burst, well short of
    the power cap's time constant)."""
    import torch
    import qgemm
    M = N = K = 4096
    R = 8
    gen = torch.Generator(device="cuda")
    gen.manual_seed(1234)
    A = [rand_i8((M, K), gen) for _ in range(R)]
    B = [rand_i8((K, N), gen) for _ in range(R)]
    sA = [rand_u((M,), 0.001, 0.01, gen) for _ in range(R)]
    sB = [rand_u((N,), 0.0005, 0.005, gen) for _ in range(R)]
    out = torch.empty((M, N), dtype=torch.bfloat16, device="cuda")

    def step(i):
        j = i % R
        ops.w8a8Gemm(A[j], B[j], sA[j], sB[j], out, M, N, K, b_layout=qgemm.B_KN,
                     out_dtype=qgemm.BF16, algo=qgemm.ALGO_TCGEN05)

    for i in range(warmup + 320):
        step(i)
    torch.cuda.synchronize()
    with clocks:
        t, _ = timed(step, steps, 1)
    per = t / steps
    ops_per = 2.0 * M * N * K
    return dict(TOPS=ops_per / per / 1e12, per_launch_s=per, ops_per_launch=ops_per,
                A=A, B=B, sA=sA, sB=sB, M=M, N=N, K=K)


def weight_unit(u: int, K: int):
    """Columns [256u, 256u + 256) of the headline's global weights B [K, N] and of sB:
    every unit has its own seed, so a rank can make any shard, and the global problem is
    the same whatever the number of ranks."""
    import torch
    g = torch.Generator(device="cuda")
    g.manual_seed(SEED_B + u)
    return rand_i8((K, SHARD_ALIGN), g), rand_u((SHARD_ALIGN,), 0.001, 0.01, g)


def weight_columns(n0: int, n1: int, K: int):
    """B[:, n0:n1] (contiguous [K, n1 - n0]) and sB[n0:n1] of the headline's weights."""
    import torch
    assert n0 % SHARD_ALIGN == 0 and n1 % SHARD_ALIGN == 0
    parts = [weight_unit(u, K) for u in range(n0 // SHARD_ALIGN, n1 // SHARD_ALIGN)]
    return (torch.cat([b for b, _ in parts], dim=1).contiguous(),
            torch.cat([s for _, s in parts]).contiguous())


def large_operands(rank, world):
    """This rank's operands of the headline GEMM: A [M, K] and sA [M] (the same on every
    rank), its weight columns B [K, NL] and sB [NL], and an output block [M, NL]."""
    import torch
    import qgemm
    M, N, K = LARGE_M, LARGE_N, LARGE_K
    n0, n1 = qgemm.shard_columns(N, world, rank, SHARD_ALIGN)
    g = torch.Generator(device="cuda")
    g.manual_seed(SEED_A)
    A = rand_i8((M, K), g)
    sA = rand_u((M,), 0.001, 0.01, g)
    B, sB = weight_columns(n0, n1, K)
    out = torch.empty((M, n1 - n0), dtype=torch.bfloat16, device="cuda")
    return dict(A=A, sA=sA, B=B, sB=sB, out=out, n0=n0, n1=n1, NL=n1 - n0, M=M, N=N, K=K)


def headline_large(ops, lo, world, steps, warmup, clocks):
    """`warmup` untimed steps, then `steps` timed ones: one GEMM launch per rank each,
    barrier + synchronize on both sides, CUDA events, the max over ranks."""
    import torch
    import qgemm
    A, B, sA, sB, out = lo["A"], lo["B"], lo["sA"], lo["sB"], lo["out"]
    M, NL, K = lo["M"], lo["NL"], lo["K"]

    def step(i):
        ops.w8a8Gemm(A, B, sA, sB, out, M, NL, K, b_layout=qgemm.B_KN, out_dtype=qgemm.BF16,
                     algo=qgemm.ALGO_TCGEN05)

    for i in range(warmup):
        step(i)
    torch.cuda.synchronize()
    with clocks:
        t_max, t_local = timed(step, steps, world)
    total_ops = 2.0 * M * lo["N"] * K
    return dict(value=total_ops * steps / t_max / 1e12, t_max=t_max, t_local=t_local,
                ops_per_rank_launch=2.0 * M * NL * K)


def e2e_large(ops, st, lo, world, steps):
    """The headline GEMM through the C-ABI with host buffers.  Every step copies that
    step's activations A and per-token scales sA from pinned host memory, runs the GEMM
    on the resident weight columns and copies this rank's bf16 output block back to
    pinned host memory.  Copies in, GEMMs and copies out run on three streams with
    double-buffered device buffers, so step i's GEMM overlaps step i+1's upload and step
    i-1's download (PCIe is full duplex)."""
    import torch
    import qgemm
    M, NL, K = lo["M"], lo["NL"], lo["K"]
    NB = 2
    hA = [lo["A"].cpu().pin_memory() for _ in range(NB)]
    hsA = [lo["sA"].cpu().pin_memory() for _ in range(NB)]
    hout = [torch.empty((M, NL), dtype=torch.bfloat16).pin_memory() for _ in range(NB)]
    dA = [torch.empty_like(lo["A"]) for _ in range(NB)]
    dsA = [torch.empty_like(lo["sA"]) for _ in range(NB)]
    dout = [torch.empty((M, NL), dtype=torch.bfloat16, device="cuda") for _ in range(NB)]
    B, sB = lo["B"], lo["sB"]
    s_in, s_mm, s_out = torch.cuda.Stream(), torch.cuda.Stream(), torch.cuda.Stream()
    q_in, q_mm, q_out = (st.dev.wrap_stream(x.cuda_stream) for x in (s_in, s_mm, s_out))
    mm_ops = type(ops)(q_mm)
    ev = lambda: torch.cuda.Event()  # noqa: E731
    uploaded = [ev() for _ in range(NB)]
    computed = [ev() for _ in range(NB)]
    downloaded = [ev() for _ in range(NB)]
    consumed = [ev() for _ in range(NB)]   # the GEMM finished reading dA/dsA[j]
    used = [False] * NB

    def step(i):
        j = i % NB
        if used[j]:
            s_in.wait_event(consumed[j])
            s_mm.wait_event(downloaded[j])
        q_in.h2d_ptr(dA[j].data_ptr(), hA[j].data_ptr(), hA[j].numel())
        q_in.h2d_ptr(dsA[j].data_ptr(), hsA[j].data_ptr(), hsA[j].numel() * 4)
        uploaded[j].record(s_in)
        s_mm.wait_event(uploaded[j])
        mm_ops.w8a8Gemm(dA[j], B, dsA[j], sB, dout[j], M, NL, K, b_layout=qgemm.B_KN,
                        out_dtype=qgemm.BF16, algo=qgemm.ALGO_TCGEN05)
        computed[j].record(s_mm)
        consumed[j].record(s_mm)
        s_out.wait_event(computed[j])
        q_out.d2h_ptr(hout[j].data_ptr(), dout[j].data_ptr(), M * NL * 2)
        downloaded[j].record(s_out)
        used[j] = True

    def run(n):
        cur = torch.cuda.current_stream()
        for x in (s_in, s_mm, s_out):
            x.wait_stream(cur)
        for i in range(n):
            step(i)
        for x in (s_in, s_mm, s_out):
            cur.wait_stream(x)

    run(3)
    torch.cuda.synchronize()
    t_max, _ = timed(lambda i: run(steps) if i == 0 else None, 1, world)
    ok = bool(torch.equal(hout[(steps - 1) % NB].cuda(), lo["out"]))
    for q in (q_in, q_mm, q_out):
        q.destroy()
    value = 2.0 * M * lo["N"] * K * steps / t_max / 1e12
    return {"value": value, "unit": "TOPS", "h2d_bytes_per_step": M * K + M * 4,
            "d2h_bytes_per_step": M * NL * 2, "steps": steps,
            "ms_per_step": t_max / steps * 1e3,
            "output_equals_device_run": ok,
            "pipelining": "H2D / GEMM / D2H on three streams, double-buffered",
            "resident": "weight columns B [K, N/world] int8 and sB (loaded once, as model "
                        "weights)", "bytes_per_rank": "h2d and d2h are per rank"}


def oracle_rows_check(lo, out, rows, n0, n1, B_host=None, sB_host=None):
    """Rows `rows` of out[:, n0:n1] (bf16, on the device) against the CPU oracle's rows of
    the same GEMM (QuantizedGemmOps.scala:102-113, RNE to bf16): True when bit-equal.
    Runs outside every timed region, as the checker."""
    import numpy as np
    import torch
    from oracle import oracle
    ridx = torch.as_tensor(rows, device="cuda")
    A_rows = lo["A"][ridx].cpu().numpy()
    sA_rows = lo["sA"][ridx].cpu().numpy()
    if B_host is None:
        B_host, sB_host = (x.cpu().numpy() for x in weight_columns(n0, n1, lo["K"]))
    _, yb = oracle.w8a8_gemm_rows(B_host, sB_host, A_rows, sA_rows, want_f32=False,
                                  threads=host_cores())
    got = out[ridx].contiguous().view(torch.int16).cpu().numpy().view(np.uint16)
    return bool(np.array_equal(got, yb))


def check_rows(M: int):
    import numpy as np
    rng = np.random.default_rng(7)
    return np.unique(np.concatenate([[0, 1, M - 1], rng.choice(M, 13, replace=False)]))


def host_cores() -> int:
    """Host threads this process may run on (whatever OMP_NUM_THREADS says)."""
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def cpu_model() -> str:
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def all_ranks_true(flag: bool, world: int) -> bool:
    if world == 1:
        return flag
    import torch
    import torch.distributed as dist
    t = torch.tensor([1 if flag else 0], dtype=torch.int32, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MIN)
    return bool(t.item())


def library_int8_context(hb, steps):
    """cuBLASLt int8 GEMM (torch._int_mm: int32 output, no scales, no bf16
    epilogue) on the same rotating inputs right after the timed region: context
    for the headline, never part of it."""
    import torch
    try:
        A, B = hb["A"], hb["B"]
        R = len(A)
        for i in range(3):
            torch._int_mm(A[i % R], B[i % R])
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for i in range(steps):
            torch._int_mm(A[i % R], B[i % R])
        e.record()
        torch.cuda.synchronize()
        t = s.elapsed_time(e) / 1e3 / steps
        return {"cublaslt_int_mm_TOPS": 2.0 * hb["M"] * hb["N"] * hb["K"] / t / 1e12,
                "note": "int32 out, no dequant epilogue; same inputs, same box"}
    except Exception as ex:  # context only
        return {"cublaslt_int_mm_TOPS": None, "note": f"unavailable: {ex}"}


def w4a16_profile(ops, steps, warmup):
    """The decode GEMV as warmup + steps plain launches each (no graph), for ncu: M = 1
    on the 64-column-tile kernel, then M = 1, 16 and 32 on the fragment order (M = 32 on
    the K-split cluster kernel)."""
    import torch
    N, K, G, R = 14336, 4096, 128, 8
    gen = torch.Generator(device="cuda")
    gen.manual_seed(77)
    wq = []
    for _ in range(R):
        w0 = torch.randint(-2**31, 2**31 - 1, (K, N // 8), dtype=torch.int32, device="cuda",
                           generator=gen)
        wq.append(torch.empty(ops.w4TiledBytes(K, N), dtype=torch.uint8, device="cuda"))
        ops.prepackW4Tiled(w0, wq[-1], K, N)
    sc = [(torch.rand((K // G, N), device="cuda", generator=gen) * 0.015 + 0.005).to(torch.bfloat16)
          for _ in range(R)]
    x = torch.randn((1, K), device="cuda", generator=gen).to(torch.bfloat16)
    y = torch.empty((1, N), dtype=torch.bfloat16, device="cuda")
    for i in range(warmup + steps):
        ops.w4a16GemmGroupedTiled(x, wq[i % R], sc[i % R], y, 1, N, K, zero_point=8, group_size=G)
    torch.cuda.synchronize()
    wf = []
    for i in range(R):
        w0 = torch.randint(-2**31, 2**31 - 1, (K, N // 8), dtype=torch.int32, device="cuda",
                           generator=gen)
        wf.append(torch.empty(ops.w4FragBytes(K, N), dtype=torch.uint8, device="cuda"))
        ops.prepackW4Frag(w0, wf[-1], K, N)
    for i in range(warmup + steps):
        ops.w4a16GemmGroupedFrag(x, wf[i % R], sc[i % R], y, 1, N, K, zero_point=8, group_size=G)
    x16 = torch.randn((16, K), device="cuda", generator=gen).to(torch.bfloat16)
    y16 = torch.empty((16, N), dtype=torch.bfloat16, device="cuda")
    for i in range(warmup + steps):
        ops.w4a16GemmGroupedFrag(x16, wf[i % R], sc[i % R], y16, 16, N, K, zero_point=8,
                                 group_size=G)
    x32 = torch.randn((32, K), device="cuda", generator=gen).to(torch.bfloat16)
    y32 = torch.empty((32, N), dtype=torch.bfloat16, device="cuda")
    for i in range(warmup + steps):
        ops.w4a16GemmGroupedFrag(x32, wf[i % R], sc[i % R], y32, 32, N, K, zero_point=8,
                                 group_size=G)
    torch.cuda.synchronize()
    return {"launches": warmup + steps, "M": [1, 16, 32], "N": N, "K": K}


def w4a16_decode(ops, peaks):
    """Config: x bf16 [M,4096] ~N(0,1), int4 [4096,14336] group 128, zp 8, bf16 out.
    Each M is timed on both prepacked layouts (64-column tiles; fragment order) and
    reported as the faster one, with both times."""
    import torch
    import qgemm.synthetic as syn
    N, K, G = 14336, 4096, 128
    R = 8  # 8 x 30 MB of weights rotating > L2
    res = {}
    gen = torch.Generator(device="cuda")
    gen.manual_seed(77)
    wq0 = [torch.randint(-2**31, 2**31 - 1, (K, N // 8), dtype=torch.int32, device="cuda",
                         generator=gen) for _ in range(R)]
    # one-time prepack of the static weights into 64-column tiles (not timed)
    wq = [torch.empty(ops.w4TiledBytes(K, N), dtype=torch.uint8, device="cuda") for _ in range(R)]
    wf = [torch.empty(ops.w4FragBytes(K, N), dtype=torch.uint8, device="cuda") for _ in range(R)]
    for a, b, c in zip(wq0, wq, wf):
        ops.prepackW4Tiled(a, b, K, N)
        ops.prepackW4Frag(a, c, K, N)
    torch.cuda.synchronize()
    del wq0
    sc = [(torch.rand((K // G, N), device="cuda", generator=gen) * 0.015 + 0.005).to(torch.bfloat16)
          for _ in range(R)]
    def per_launch(M, x, y, path):
        launches = 64
        # one stream handle for warm-up and capture: its scratch is made by the
        # first (uncaptured) call
        cap = torch.cuda.Stream()
        q = ops.stream.dev.wrap_stream(cap.cuda_stream)
        o = type(ops)(q)

        def body():
            for i in range(launches):
                if path == "frag":
                    o.w4a16GemmGroupedFrag(x, wf[i % R], sc[i % R], y, M, N, K, zero_point=8,
                                           group_size=G)
                else:
                    o.w4a16GemmGroupedTiled(x, wq[i % R], sc[i % R], y, M, N, K, zero_point=8,
                                            group_size=G)

        cap.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(cap):
            body()  # warm-up outside capture (also sets kernel attributes)
        torch.cuda.current_stream().wait_stream(cap)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=cap):
            body()
        for _ in range(3):
            g.replay()
        torch.cuda.synchronize()
        reps = 20
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            g.replay()
        e1.record()
        torch.cuda.synchronize()
        per = e0.elapsed_time(e1) / 1e3 / (reps * launches)
        del g
        q.destroy()
        return per

    for M in (1, 4, 16):
        x = torch.randn((M, K), device="cuda", generator=gen).to(torch.bfloat16)
        y = torch.empty((M, N), dtype=torch.bfloat16, device="cuda")
        times = {"tiled": per_launch(M, x, y, "tiled"), "frag": per_launch(M, x, y, "frag")}
        path = min(times, key=times.get)
        per = times[path]
        bytes_alg = K * N // 2 + (K // G) * N * 2 + M * K * 2 + M * N * 2
        gbs = bytes_alg / per / 1e9
        res[f"M{M}"] = {"us_per_launch": per * 1e6, "GB_s": gbs, "bytes_per_launch": bytes_alg,
                        "frac_of_hbm": gbs / peaks["hbm_gbs"],
                        "tflops": 2.0 * M * N * K / per / 1e12, "path": path,
                        "us_by_layout": {k: v * 1e6 for k, v in times.items()}}
    _ = syn
    return res


def w8a8_pipeline(ops, hb, steps, peaks):
    """bf16 activations -> per-token int8 quantisation (qgemm_quantize_per_token) -> the
    headline W8A8 GEMM, on device: the quantiser alone (GB/s of x read + q written) and
    the two kernels back to back (TOPS of the GEMM's 2*M*N*K)."""
    import torch
    import qgemm
    M, N, K = hb["M"], hb["N"], hb["K"]
    R = 4  # 4 x 32 MB of bf16 activations rotating
    gen = torch.Generator(device="cuda")
    gen.manual_seed(99)
    xs = [torch.randn((M, K), device="cuda", generator=gen).to(torch.bfloat16) for _ in range(R)]
    q = torch.empty((M, K), dtype=torch.int8, device="cuda")
    sA = torch.empty((M,), dtype=torch.float32, device="cuda")
    out = torch.empty((M, N), dtype=torch.bfloat16, device="cuda")
    B, sB = hb["B"][0], hb["sB"][0]

    def quant(i):
        ops.quantizePerToken(xs[i % R], q, sA, M, K, in_dtype=qgemm.BF16)

    def both(i):
        quant(i)
        ops.w8a8Gemm(q, B, sA, sB, out, M, N, K, b_layout=qgemm.B_KN, out_dtype=qgemm.BF16,
                     algo=qgemm.ALGO_TCGEN05)

    res = {}
    for name, fn in (("quantize", quant), ("quantize_plus_gemm", both)):
        for i in range(3):
            fn(i)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for i in range(steps):
            fn(i)
        e1.record()
        torch.cuda.synchronize()
        res[name] = e0.elapsed_time(e1) / 1e3 / steps
    qb = M * K * 2 + M * K + M * 4
    return {"quantize_us": res["quantize"] * 1e6, "quantize_GB_s": qb / res["quantize"] / 1e9,
            "quantize_frac_of_hbm": qb / res["quantize"] / 1e9 / peaks["hbm_gbs"],
            "quantize_plus_gemm_us": res["quantize_plus_gemm"] * 1e6,
            "quantize_plus_gemm_TOPS": 2.0 * M * N * K / res["quantize_plus_gemm"] / 1e12}


def f32_facade(st, peaks, steps=10):
    """The fp32 entry points (MatrixOps.matmul / gemv) on device-resident inputs:
    matmul 4096^3 on the tensor cores (3 tf32 products per fp32 product), a skinny
    16 x 4096 x 4096 matmul on the CUDA-core path, gemv 16384 x 16384.  Two rotating input
    sets of 128 MB (matmul) and one 1 GB matrix (gemv) keep every launch above L2."""
    import torch
    import qgemm
    m = qgemm.MatrixOps(st)
    gen = torch.Generator(device="cuda")
    gen.manual_seed(4242)

    def run(fn, n):
        for i in range(3):
            fn(i)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for i in range(n):
            fn(i)
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / 1e3 / n

    res = {}
    M = N = K = 4096
    A = [torch.randn((M, K), device="cuda", generator=gen) for _ in range(2)]
    B = [torch.randn((K, N), device="cuda", generator=gen) for _ in range(2)]
    C = torch.empty((M, N), device="cuda")
    t = run(lambda i: m.matmul(A[i % 2], B[i % 2], C, M, N, K), steps)
    fl = 2.0 * M * N * K
    tf32_peak = 0.5 * peaks["bf16_tflops"]
    res["matmul_4096"] = {"us": t * 1e6, "TFLOP_s": fl / t / 1e12,
                          "gemm_kernel_traffic_bytes": NCU_TRAFFIC_F32_GEMM_4096,
                          "tensor_TFLOP_s": 3 * fl / t / 1e12,
                          "tensor_frac_of_tf32_peak": 3 * fl / t / 1e12 / tf32_peak,
                          "tf32_peak_basis": "0.5 x measured bf16_tflops (dense tf32 runs at "
                                             "half the bf16 rate on B200)",
                          "includes": "two operand split passes (A, B -> hi/lo) + GEMM"}
    rows = torch.randperm(M, device="cuda", generator=gen)[:32]
    ref = A[1][rows].double() @ B[1].double()
    res["matmul_4096"]["max_err_over_sum_abs"] = float(
        ((C[rows].double() - ref).abs() / (A[1][rows].abs().double() @ B[1].abs().double())).max())
    torch.backends.cuda.matmul.allow_tf32 = False
    tt = run(lambda i: torch.matmul(A[i % 2], B[i % 2], out=C), 5)
    res["matmul_4096"]["torch_fp32_TFLOP_s_context"] = fl / tt / 1e12
    Ms = 16
    As = torch.randn((Ms, K), device="cuda", generator=gen)
    Cs = torch.empty((Ms, N), device="cuda")
    t = run(lambda i: m.matmul(As, B[i % 2], Cs, Ms, N, K), steps)
    res["matmul_16x4096x4096"] = {"us": t * 1e6, "TFLOP_s": 2.0 * Ms * N * K / t / 1e12,
                                  "B_read_GB_s": 4.0 * K * N / t / 1e9}
    del A, B, C, As, Cs
    torch.cuda.empty_cache()
    Mv = Nv = 16384
    Av = torch.randn((Mv, Nv), device="cuda", generator=gen)
    x = torch.randn((Nv,), device="cuda", generator=gen)
    y = torch.empty((Mv,), device="cuda")
    t = run(lambda i: m.gemv(Av, x, y, Mv, Nv), steps)
    gbs = 4.0 * (Mv * Nv + Nv + Mv) / t / 1e9
    res["gemv_16384"] = {"us": t * 1e6, "GB_s": gbs, "frac_of_hbm": gbs / peaks["hbm_gbs"]}
    del Av
    torch.cuda.empty_cache()
    return res


def side_kernels(st, ops, steps, warmup):
    """The facade's smaller kernels on their own, each `warmup` + `steps` launches:
    fp32 gemv A [16384, 16384], per-token quantisation of x [4096, 4096] bf16, the
    CUDA-core fp32 GEMM at 64 x 4096 x 4096 (small cases, each one launch that an ncu
    capture can hold), and w8a16Gemm at 1 x 14336 x 4096."""
    import torch
    import qgemm
    m = qgemm.MatrixOps(st)
    gen = torch.Generator(device="cuda")
    gen.manual_seed(2)

    def run(fn):
        for _ in range(warmup):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) * 1e3 / steps

    res = {}
    A = torch.randn((16384, 16384), device="cuda", generator=gen)
    x = torch.randn((16384,), device="cuda", generator=gen)
    y = torch.empty((16384,), device="cuda")
    res["gemv_16384_us"] = run(lambda: m.gemv(A, x, y, 16384, 16384))
    del A
    xb = torch.randn((4096, 4096), device="cuda", generator=gen).to(torch.bfloat16)
    q = torch.empty((4096, 4096), dtype=torch.int8, device="cuda")
    sA = torch.empty((4096,), device="cuda")
    res["quantize_4096_bf16_us"] = run(
        lambda: ops.quantizePerToken(xb, q, sA, 4096, 4096, in_dtype=qgemm.BF16))
    Af = torch.randn((64, 4096), device="cuda", generator=gen)
    Bf = torch.randn((4096, 4096), device="cuda", generator=gen)
    Cf = torch.empty((64, 4096), device="cuda")
    res["rows_gemm_64x4096x4096_us"] = run(
        lambda: m.gemmF32(Af, Bf, Cf, 64, 4096, 4096, algo=qgemm.ALGO_SIMT))
    # QuantizedGemmOps.w8a16Gemm (exact reference order) at the decode shape, M = 1
    w8 = torch.randint(-127, 128, (4096, 14336), dtype=torch.int8, device="cuda", generator=gen)
    s8 = torch.rand((14336,), device="cuda", generator=gen) * 0.01
    b8 = torch.randn((14336,), device="cuda", generator=gen)
    x8 = torch.randn((1, 4096), device="cuda", generator=gen)
    y8 = torch.empty((1, 14336), device="cuda")
    t = run(lambda: ops.w8a16Gemm(w8, s8, x8, b8, y8, 1, 14336, 4096, True))
    res["w8a16_1x14336x4096_us"] = t
    res["w8a16_1x14336x4096_GB_s"] = (4096 * 14336 + 4096 * 4 + 14336 * 12) / t / 1e3
    return res


LLAMA_LINEARS = (("qkv", 4096, 12288), ("o", 4096, 4096), ("gate_up", 4096, 22016),
                 ("down", 11008, 4096))


def llama_stack(ops, peaks, layers=32, prefill_steps=3, decode_steps=50):
    """Quantized linear stack of a Llama-2-7B-shaped decoder: `layers` x {qkv
    4096->12288, o 4096->4096, gate+up 4096->22016, down 11008->4096}, random-init
    int4 group-128 weights (zero point 8, bf16 scales ~U[0.005, 0.02]), bf16
    activations ~N(0,1).  Prefill: batch x seq = 32 x 512 = 16384 rows through the
    prefill path, with the exact expansion (q - zp in the slab, the group scales applied
    in fp32 to each group's partial sums) and with the one-term one;
    decode: 32 rows through the decode kernel (one CUDA graph per step).  One step =
    every linear of every layer once.  Each weight is stored once, in the fragment order
    (qgemm_prepack_w4_frag); prefill and decode read that copy."""
    import torch
    G = 128
    gen = torch.Generator(device="cuda")
    gen.manual_seed(2024)
    W = []  # (name, K, N, prepacked weights, scales, layout)
    for _ in range(layers):
        for name, K, N in LLAMA_LINEARS:
            q = torch.randint(-2**31, 2**31 - 1, (K, N // 8), dtype=torch.int32, device="cuda",
                              generator=gen)
            lay = "frag"
            if lay == "frag":
                wt = torch.empty(ops.w4FragBytes(K, N), dtype=torch.uint8, device="cuda")
                ops.prepackW4Frag(q, wt, K, N)
            else:
                wt = torch.empty(ops.w4TiledBytes(K, N), dtype=torch.uint8, device="cuda")
                ops.prepackW4Tiled(q, wt, K, N)
            sc = (torch.rand((K // G, N), device="cuda", generator=gen) * 0.015 + 0.005).to(
                torch.bfloat16)
            W.append((name, K, N, wt, sc, lay))
            del q
    torch.cuda.synchronize()
    weights_bytes = sum(K * N // 2 + (K // G) * N * 2 for _, K, N, _, _, _ in W)
    flops_per_row = sum(2.0 * K * N for _, K, N, _, _, _ in W)
    res = {"layers": layers, "group_size": G, "weight_bytes": weights_bytes}

    # ---- prefill ----
    M = 16384
    xs = {K: torch.randn((M, K), device="cuda", generator=gen).to(torch.bfloat16)
          for K in (4096, 11008)}
    ys = {N: torch.empty((M, N), dtype=torch.bfloat16, device="cuda")
          for N in (12288, 4096, 22016)}
    ws_bytes = max(ops.w4PrefillWorkspaceBytes(K, N) for _, K, N in LLAMA_LINEARS)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device="cuda")

    def prefill_step(one_term):
        for _, K, N, wt, sc, lay in W:
            f = ops.w4a16GemmGroupedPrefillFrag if lay == "frag" else ops.w4a16GemmGroupedPrefill
            f(xs[K], wt, sc, ys[N], M, N, K, ws, ws_bytes, zero_point=8, group_size=G,
              one_term=one_term)

    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    flops = flops_per_row * M
    sustained = peaks.get("bf16_tflops_sustained", peaks["bf16_tflops"])
    for key, one_term in (("prefill", False), ("prefill_one_term", True)):
        prefill_step(one_term)
        torch.cuda.synchronize()
        e0.record()
        for _ in range(prefill_steps):
            prefill_step(one_term)
        e1.record()
        torch.cuda.synchronize()
        t = e0.elapsed_time(e1) / 1e3 / prefill_steps
        res[key] = {"M": M, "ms_per_step": t * 1e3, "TFLOPs": flops / t / 1e12,
                    "algorithmic_flop_per_step": flops,
                    "frac_of_bf16_sustained_peak": flops / t / 1e12 / sustained,
                    "tensor_work_factor": 1,
                    "note": ("one term: each int4 weight is expanded to bf16((q - zp) * s), "
                             "relative weight error <= 2^-9; forward error <= 2^-8 of "
                             "sum |x w| (tested), not within the elementwise 1e-2 gate for "
                             "outputs far below the output scale"
                             if one_term else
                             "exact: q - zp (exact in bf16) in the slab, the group-128 "
                             "scales applied in fp32 to each group's tensor-core partial "
                             "sums by the epilogue warps (one pass over K)")}
    del xs, ys, ws
    torch.cuda.empty_cache()

    # ---- decode (one graph per step) ----
    M = 32
    xd = {K: torch.randn((M, K), device="cuda", generator=gen).to(torch.bfloat16)
          for K in (4096, 11008)}
    yd = {N: torch.empty((M, N), dtype=torch.bfloat16, device="cuda")
          for N in (12288, 4096, 22016)}
    cap = torch.cuda.Stream()
    q = ops.stream.dev.wrap_stream(cap.cuda_stream)
    o = type(ops)(q)

    def decode_step():
        for _, K, N, wt, sc, lay in W:
            f = o.w4a16GemmGroupedFrag if lay == "frag" else o.w4a16GemmGroupedTiled
            f(xd[K], wt, sc, yd[N], M, N, K, zero_point=8, group_size=G)

    cap.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(cap):
        decode_step()
    torch.cuda.current_stream().wait_stream(cap)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=cap):
        decode_step()
    for _ in range(2):
        g.replay()
    torch.cuda.synchronize()
    # the legacy-MMA-bound decode follows the SM clock: record it beside the time
    with ClockSampler(torch.cuda.current_device(), period_s=0.002) as clk:
        e0.record()
        for _ in range(decode_steps):
            g.replay()
        e1.record()
        torch.cuda.synchronize()
    t = e0.elapsed_time(e1) / 1e3 / decode_steps
    bytes_step = weights_bytes + sum(M * K * 2 + M * N * 2 for _, K, N, _, _, _ in W)
    res["decode"] = {"M": M, "ms_per_step": t * 1e3, "GB_s": bytes_step / t / 1e9,
                     "frac_of_hbm": bytes_step / t / 1e9 / peaks["hbm_gbs"],
                     "bytes_per_step": bytes_step, "clocks": clk.summary()}
    del g
    q.destroy()
    return res


def prefill_one(ops, M, steps, warmup, profile, peaks):
    """One exact W4A16 prefill call of the Llama-2-7B gate+up projection (K=4096,
    N=22016, group 128, fragment-ordered weights) at M rows: the slab expansion and the
    group-scaled multiply.  With `profile`, warmup + steps plain calls and nothing else
    (the form an ncu capture uses)."""
    import torch
    K, N, G = 4096, 22016, 128
    gen = torch.Generator(device="cuda")
    gen.manual_seed(7)
    q = torch.randint(-2**31, 2**31 - 1, (K, N // 8), dtype=torch.int32, device="cuda",
                      generator=gen)
    wt = torch.empty(ops.w4FragBytes(K, N), dtype=torch.uint8, device="cuda")
    ops.prepackW4Frag(q, wt, K, N)
    sc = (torch.rand((K // G, N), device="cuda", generator=gen) * 0.015 + 0.005).to(torch.bfloat16)
    x = torch.randn((M, K), device="cuda", generator=gen).to(torch.bfloat16)
    y = torch.empty((M, N), dtype=torch.bfloat16, device="cuda")
    ws_bytes = ops.w4PrefillWorkspaceBytes(K, N)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device="cuda")

    def call():
        ops.w4a16GemmGroupedPrefillFrag(x, wt, sc, y, M, N, K, ws, ws_bytes, zero_point=8,
                                        group_size=G)
    if profile:
        for _ in range(warmup + steps):
            call()
        torch.cuda.synchronize()
        return {"launches": warmup + steps, "shape": [M, N, K]}
    for _ in range(warmup):
        call()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        call()
    e1.record()
    torch.cuda.synchronize()
    t = e0.elapsed_time(e1) / 1e3 / steps
    flops = 2.0 * M * N * K
    return {"shape": [M, N, K], "ms_per_call": t * 1e3, "TFLOPs": flops / t / 1e12,
            "frac_of_bf16_burst_peak": flops / t / 1e12 / peaks["bf16_tflops"]}


def gather_output(st, lo, rank, world, reps=5):
    """The whole headline output on every rank, timed apart from the headline: the NCCL
    all-gather of the bf16 output blocks and the [world][M][NL] -> [M][N] unshard kernel
    (each alone), then the whole layer (GEMM + gather) three ways: one after the other
    on one stream; qgemm_w8a8_gemm_allgather_bf16, which gathers chunk i of M rows on a
    second stream while the GEMM of chunk i+1 runs; and its window form, where copy-engine
    copies write each chunk into the peers' outputs.  Every form's output equals the
    serial one, and rank 0 checks sampled full rows of it against the CPU oracle.  The
    fused form is one GEMM whose epilogue stores each output chunk into every rank's
    registered output (TMA stores over NVLink)."""
    import ctypes
    import numpy as np
    import torch
    import torch.distributed as dist
    import qgemm._lib as L
    from oracle import oracle
    from qgemm import B_KN, BF16
    from qgemm import QuantizedGemmOps as qgemm_ops
    A, B, sA, sB, out = lo["A"], lo["B"], lo["sA"], lo["sB"], lo["out"]
    M, NL, K, N = lo["M"], lo["NL"], lo["K"], lo["N"]
    rows = check_rows(M)
    expect = None
    if rank == 0:
        Bf, sBf = (x.cpu().numpy() for x in weight_columns(0, N, K))
        ridx = torch.as_tensor(rows, device="cuda")
        _, expect = oracle.w8a8_gemm_rows(Bf, sBf, A[ridx].cpu().numpy(),
                                          sA[ridx].cpu().numpy(), want_f32=False,
                                          threads=host_cores())
        del Bf, sBf
    uid = ctypes.create_string_buffer(128)
    if rank == 0:
        L.call("qgemm_comm_unique_id", uid)
    obj = [bytes(uid.raw) if rank == 0 else None]
    dist.broadcast_object_list(obj, src=0)
    uid = ctypes.create_string_buffer(obj[0], 128)
    comm = ctypes.c_void_p()
    L.call("qgemm_comm_init", st.dev.handle, uid, rank, world, ctypes.byref(comm))
    ops = qgemm_ops(st)
    res = {}

    def oracle_ok(full):
        if rank != 0:
            return None
        got = full[torch.as_tensor(rows, device="cuda")].contiguous().view(torch.int16)
        return bool(np.array_equal(got.cpu().numpy().view(np.uint16), expect))

    try:
        gathered = torch.empty((world, M, NL), dtype=torch.bfloat16, device="cuda")
        full = torch.empty((M, N), dtype=torch.bfloat16, device="cuda")

        def gather(i):
            L.call("qgemm_comm_allgather_bf16", comm, st.handle, out.data_ptr(),
                   gathered.data_ptr(), M * NL)

        def unshard(i):
            L.call("qgemm_unshard_columns_bf16", st.handle, gathered.data_ptr(), full.data_ptr(),
                   world, M, NL)

        for i in range(2):
            gather(i)
            unshard(i)
        tg, _ = timed(gather, reps, world)
        tu, _ = timed(unshard, reps, world)
        recv = (world - 1) * M * NL * 2
        res.update({"gather_ms": tg / reps * 1e3, "recv_GB_s_per_rank": recv / (tg / reps) / 1e9,
                    "unshard_ms": tu / reps * 1e3, "bytes_total": world * M * NL * 2})

        def serial(i):
            ops.w8a8Gemm(A, B, sA, sB, out, M, NL, K, b_layout=B_KN, out_dtype=BF16)
            gather(i)
            unshard(i)

        for i in range(2):
            serial(i)
        ts, _ = timed(serial, reps, world)
        layers = {"serial": ts / reps * 1e3}
        ref = full.clone()
        checks = {"serial": oracle_ok(full)}
        equal = {}
        side = torch.cuda.Stream()
        q_side = st.dev.wrap_stream(side.cuda_stream)
        for R in (4096, 2048, 1024):
            wb = L.lib().qgemm_w8a8_allgather_work_bytes(world, R, NL)
            work = torch.empty(wb, dtype=torch.uint8, device="cuda")

            def piped(i):
                L.call("qgemm_w8a8_gemm_allgather_bf16", comm, st.handle, q_side.handle,
                       A.data_ptr(), B.data_ptr(), B_KN, sA.data_ptr(), sB.data_ptr(),
                       full.data_ptr(), M, NL, K, R, work.data_ptr(), wb)

            full.zero_()
            for i in range(2):
                piped(i)
            tp, _ = timed(piped, reps, world)
            tag = f"nccl_pipelined_rows{R}"
            layers[tag] = tp / reps * 1e3
            equal[tag] = bool(torch.equal(full, ref))
            checks[tag] = oracle_ok(full)
            del work
        # the window form: the copy engines write each finished chunk into the peers'
        # registered output buffers, in the final layout
        win = ctypes.c_void_p()
        try:  # a refusal here is the same on every rank (registration agrees before it returns)
            L.call("qgemm_comm_window_register", comm, st.handle, full.data_ptr(),
                   full.numel() * 2, ctypes.byref(win))
        except L.QGemmError as e:
            res["window_error"] = str(e)
            win = None
        if win is not None:
            try:
                # the peer copies on one stream (the default), then on one stream per peer
                for R, ncp in ((4096, None), (2048, None), (1024, None), (4096, world - 1)):
                    def windowed(i):
                        L.call("qgemm_w8a8_gemm_allgather_window_bf16", win, st.handle,
                               q_side.handle, A.data_ptr(), B.data_ptr(), B_KN, sA.data_ptr(),
                               sB.data_ptr(), M, NL, K, R)

                    if ncp:
                        os.environ["QGEMM_COPY_STREAMS"] = str(ncp)
                    full.zero_()
                    for i in range(2):
                        windowed(i)
                    tw, _ = timed(windowed, reps, world)
                    os.environ.pop("QGEMM_COPY_STREAMS", None)
                    tag = f"window_rows{R}" + (f"_copy_streams{ncp}" if ncp else "")
                    layers[tag] = tw / reps * 1e3
                    equal[tag] = bool(torch.equal(full, ref))
                    checks[tag] = oracle_ok(full)

                # the fused form: the GEMM's epilogue stores into every rank's window
                def fused(i):
                    L.call("qgemm_w8a8_gemm_allgather_fused_bf16", win, st.handle,
                           A.data_ptr(), B.data_ptr(), B_KN, sA.data_ptr(), sB.data_ptr(),
                           M, NL, K)

                try:  # a refusal comes before any collective, the same on every rank
                    full.zero_()
                    for i in range(2):
                        fused(i)
                    tf, _ = timed(fused, reps, world)
                    layers["fused"] = tf / reps * 1e3
                    equal["fused"] = bool(torch.equal(full, ref))
                    checks["fused"] = oracle_ok(full)
                    res["fused_egress_GB_s_per_rank"] = \
                        (world - 1) * M * NL * 2 / (tf / reps) / 1e9
                except L.QGemmError as e:
                    res["fused_error"] = str(e)
            finally:
                torch.cuda.synchronize()
                barrier(world)
                L.call("qgemm_comm_window_release", win)
        q_side.destroy()
        best = min(layers, key=layers.get)
        res.update({"layer_ms": layers, "best_layer_form": best,
                    "best_layer_ms": layers[best],
                    "best_layer_TOPS": 2.0 * M * N * K / (layers[best] / 1e3) / 1e12,
                    "equal_to_serial": equal,
                    "oracle_rows_equal_rank0": checks, "oracle_rows": len(rows),
                    "layer": "GEMM + all-gather: the whole [M, N] bf16 output on every rank"})
        return res
    finally:
        torch.cuda.synchronize()
        L.call("qgemm_comm_destroy", comm)


def cpu_legs(threads: int, w8a8_target_s: float = 5.0, single_target_s: float = 2.0,
             w4_target_s: float = 1.5):
    """The CPU restatement (oracle/, OpenMP) timed on bounded samples of the workloads:
    the headline GEMM on a row slice with `threads` threads and with one (extrapolated to
    the whole GEMM: the per-row work is the same for every row), and the W4A16 decode GEMV
    at M = 1 (the grouped form of QuantizedGemmOps.scala:229-245) both ways."""
    import numpy as np
    from oracle import oracle
    M, N, K = LARGE_M, LARGE_N, LARGE_K
    rng = np.random.default_rng(2)
    B = rng.integers(-127, 128, size=(K, N), dtype=np.int8)
    sB = rng.uniform(0.001, 0.01, size=N).astype(np.float32)
    x = rng.integers(-127, 128, size=(4 * threads + 64, K), dtype=np.int8)
    sx = rng.uniform(0.001, 0.01, size=x.shape[0]).astype(np.float32)

    def rows_rate(th, target):
        # a slice of whole rounds of `th` rows, repeated to fill about `target` seconds
        rows = max(th, x.shape[0] // th * th)
        t0 = time.perf_counter()
        oracle.w8a8_gemm_rows(B, sB, x[:rows], sx[:rows], want_f32=False, threads=th)
        dt = time.perf_counter() - t0
        reps = max(1, int(target / max(dt, 1e-9)))
        t0 = time.perf_counter()
        for _ in range(reps):
            oracle.w8a8_gemm_rows(B, sB, x[:rows], sx[:rows], want_f32=False, threads=th)
        dt = time.perf_counter() - t0
        return 2.0 * rows * N * K * reps / dt / 1e12, rows, reps, dt

    v_mt, r_mt, n_mt, dt_mt = rows_rate(threads, w8a8_target_s)
    v_1, r_1, n_1, dt_1 = rows_rate(1, single_target_s)
    # W4A16 decode GEMV, M = 1, K = 4096, N = 14336, group 128
    Nw, Kw, G = 14336, 4096, 128
    import qgemm.synthetic as syn
    xw, wq, sc = syn.w4a16_inputs(1, Nw, Kw, group=G, seed=3)
    bytes_alg = Kw * Nw // 2 + (Kw // G) * Nw * 2 + Kw * 2 + Nw * 2

    def w4_rate(th):
        oracle.w4a16_grouped(wq, sc, 8, G, xw, threads=th)
        t0 = time.perf_counter()
        n = 0
        while time.perf_counter() - t0 < w4_target_s or n < 1:
            oracle.w4a16_grouped(wq, sc, 8, G, xw, threads=th)
            n += 1
        dt = time.perf_counter() - t0
        return bytes_alg * n / dt / 1e9, n

    g_mt, c_mt = w4_rate(threads)
    g_1, c_1 = w4_rate(1)
    return {
        "value": v_mt, "unit": "TOPS", "cores": threads, "kind": "port",
        "sample": f"{n_mt} x rows 0..{r_mt - 1} of the M=16384 N=28672 K=8192 W8A8 GEMM "
                  f"(bf16 out), {threads} OpenMP threads, extrapolated to the whole GEMM "
                  f"at the same per-row rate ({dt_mt:.1f} s timed)",
        "extrapolated_ms_per_gemm": 2.0 * M * N * K / (v_mt * 1e12) * 1e3,
        "single_thread": {"value": v_1, "unit": "TOPS", "sample": f"{n_1} x {r_1} rows, "
                          f"{dt_1:.1f} s timed", "extrapolated_s_per_gemm":
                          2.0 * M * N * K / (v_1 * 1e12)},
        "w4a16_decode_M1": {"openmp_GB_s": g_mt, "openmp_calls": c_mt,
                            "single_thread_GB_s": g_1, "single_thread_calls": c_1,
                            "bytes_per_call": bytes_alg,
                            "what": "grouped W4A16 GEMV x bf16 [1, 4096], int4 [4096, 14336], "
                                    "group 128, zero point 8"},
        "cpu_model": cpu_model(), "nproc": os.cpu_count(),
    }


def reference_arm(args):
    """The reference's CPU path for the headline: the C restatement of
    QuantizedGemmOps.w8a32Gemm (oracle/, the reference's JVM path being absent) on a row
    slice of the same GEMM per step, all host threads, extrapolated to the whole GEMM.
    Under torchrun only rank 0 runs it."""
    import numpy as np
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    from oracle import oracle
    W, Ksteps = max(args.warmup, 0), max(args.steps, 1)
    threads = host_cores()
    M, N, K = LARGE_M, LARGE_N, LARGE_K
    rng = np.random.default_rng(2)
    B = rng.integers(-127, 128, size=(K, N), dtype=np.int8)
    sB = rng.uniform(0.001, 0.01, size=N).astype(np.float32)
    x = rng.integers(-127, 128, size=(32 * threads, K), dtype=np.int8)
    sx = rng.uniform(0.001, 0.01, size=x.shape[0]).astype(np.float32)
    # size one step at <= 2 s of CPU work, so the whole run stays within a few minutes
    t0 = time.perf_counter()
    oracle.w8a8_gemm_rows(B, sB, x[:threads], sx[:threads], want_f32=False, threads=threads)
    per_round = time.perf_counter() - t0
    budget = min(2.0, 100.0 / (W + Ksteps))
    rounds = max(1, min(32, int(budget / max(per_round, 1e-9))))
    rows = rounds * threads
    for _ in range(W):
        oracle.w8a8_gemm_rows(B, sB, x[:rows], sx[:rows], want_f32=False, threads=threads)
    t0 = time.perf_counter()
    for _ in range(Ksteps):
        oracle.w8a8_gemm_rows(B, sB, x[:rows], sx[:rows], want_f32=False, threads=threads)
    dt = time.perf_counter() - t0
    value = 2.0 * rows * N * K * Ksteps / dt / 1e12
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "TOPS",
        "n_gpus": args.gpus, "steps": Ksteps, "warmup": W, "ms_per_step": dt / Ksteps * 1e3,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "int8",
        "data": "synthetic", "config": headline_config(args.gpus),
        "cpu_baseline": {"value": value, "unit": "TOPS", "cores": threads, "kind": "port",
                         "sample": f"rows 0..{rows - 1} of the M=16384 N=28672 K=8192 GEMM per "
                                   f"step, {threads} OpenMP threads, extrapolated to the whole "
                                   f"GEMM at the same per-row rate",
                         "cpu_model": cpu_model()},
        "e2e": {"value": value, "unit": "TOPS", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "the reference's own path is Scala on the JVM, which is absent here and computes "
                "only element (0,0) per call; its C restatement (oracle/) is timed instead",
    }
    print(json.dumps(line), flush=True)
    return 0


def log(msg: str):
    print(f"[bench] {msg}", file=sys.stderr, flush=True)


def main():
    import faulthandler
    faulthandler.enable()
    args = parse_args()
    if args.impl == "reference":
        return reference_arm(args)
    import torch
    import qgemm
    rank, world, local = dist_setup(args.gpus)
    peaks, peak_src = load_peaks()
    dev = qgemm.Device(local)
    st = dev.wrap_stream(torch.cuda.current_stream().cuda_stream)
    ops = qgemm.QuantizedGemmOps(st)
    K, W = max(1, args.steps), max(3, args.warmup)

    def finish():
        st.destroy()
        dev.close()
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()

    if args.only == "w4a16":
        log("w4a16 decode (only)")
        r = w4a16_profile(ops, K, W) if args.profile else w4a16_decode(ops, peaks)
        if rank == 0:
            print(json.dumps({"only": "w4a16", "w4a16_decode": r}), flush=True)
        finish()
        return 0
    if args.only == "side":
        log("side kernels (only)")
        r = side_kernels(st, ops, K, W)
        if rank == 0:
            print(json.dumps({"only": "side", "side_kernels": r}), flush=True)
        finish()
        return 0
    if args.only == "f32":
        log("fp32 facade (only)")
        r = f32_facade(st, peaks, K)
        if rank == 0:
            print(json.dumps({"only": "f32", "fp32_facade": r}), flush=True)
        finish()
        return 0
    if args.only == "llama":
        log("llama stack (only)")
        r = llama_stack(ops, peaks)
        if rank == 0:
            print(json.dumps({"only": "llama", "llama2_7b_w4a16_stack": r}), flush=True)
        finish()
        return 0
    if args.only == "prefill":
        log("w4a16 exact prefill, gate+up projection (only)")
        r = prefill_one(ops, args.rows, K, W, args.profile, peaks)
        if rank == 0:
            print(json.dumps({"only": "prefill", **r}), flush=True)
        finish()
        return 0
    if args.only == "large":
        W_as = max(1, args.as_world)
        log(f"column-sharded headline GEMM, rank 0 of {W_as} (only)")
        lo = large_operands(0, W_as)
        if args.profile:
            for i in range(W + K):
                ops.w8a8Gemm(lo["A"], lo["B"], lo["sA"], lo["sB"], lo["out"], lo["M"], lo["NL"],
                             lo["K"], b_layout=qgemm.B_KN, out_dtype=qgemm.BF16,
                             algo=qgemm.ALGO_TCGEN05)
            torch.cuda.synchronize()
            r = {"launches": W + K, "shape": [lo["M"], lo["NL"], lo["K"]]}
        else:
            hl = headline_large(ops, lo, 1, K, W, ClockSampler(local))
            r = {"shape": [lo["M"], lo["NL"], lo["K"]],
                 "TOPS_this_gpu": hl["ops_per_rank_launch"] * K / hl["t_local"] / 1e12,
                 "ms_per_launch": hl["t_local"] / K * 1e3}
        if rank == 0:
            print(json.dumps({"only": "large", **r}), flush=True)
        finish()
        return 0
    if args.only == "w8a8":
        log("w8a8 4096^3 (only)")
        if args.profile:
            import qgemm as _q
            M = N = Kd = 4096
            g = torch.Generator(device="cuda")
            g.manual_seed(1234)
            A = rand_i8((M, Kd), g)
            B = rand_i8((Kd, N), g)
            sA = rand_u((M,), 0.001, 0.01, g)
            sB = rand_u((N,), 0.0005, 0.005, g)
            out = torch.empty((M, N), dtype=torch.bfloat16, device="cuda")
            for _ in range(W + K):
                ops.w8a8Gemm(A, B, sA, sB, out, M, N, Kd, b_layout=_q.B_KN, out_dtype=_q.BF16,
                             algo=_q.ALGO_TCGEN05)
            torch.cuda.synchronize()
            r = {"launches": W + K}
        else:
            hb = w8a8_4096(ops, K, W, ClockSampler(local))
            r = {"TOPS": hb["TOPS"], "us_per_launch": hb["per_launch_s"] * 1e6}
        if rank == 0:
            print(json.dumps({"only": "w8a8", **r}), flush=True)
        finish()
        return 0

    clocks_roof = ClockSampler(local)
    clocks = ClockSampler(local)
    int8_burst = 2.0 * peaks["bf16_tflops"]
    int8_sustained = 2.0 * peaks.get("bf16_tflops_sustained", peaks["bf16_tflops"])

    # ---- the roofline kernel: the same GEMM kernel at 4096^3, a burst on every rank ----
    log("w8a8 4096^3 (roofline)")
    hb = w8a8_4096(ops, K, W, clocks_roof)
    achieved = hb["TOPS"]
    roofline = {"bound": "tensor", "kernel": "w8a8_tcgen05_pair_kernel",
                "shape": "M=N=K=4096 (the prefill-shaped W8A8 GEMM, one GPU), bf16 out, B [K,N]",
                "achieved": achieved, "peak": int8_burst, "unit": "TOPS",
                "frac": achieved / int8_burst, "traffic": NCU_TRAFFIC_W8A8_4096,
                "algorithmic_ops_per_launch": hb["ops_per_launch"],
                "algorithmic_bytes_per_launch": 2 * 4096 * 4096 + 2 * 4096 * 4096 + 8 * 4096,
                "us_per_launch": hb["per_launch_s"] * 1e6, "launches_timed": K,
                "peak_basis": f"2 x bf16_tflops ({peak_src}: cuBLAS bf16, burst): dense int8 "
                              f"runs at twice the bf16 rate on B200; the {K} timed launches "
                              f"are a burst of {K * hb['per_launch_s'] * 1e3:.2f} ms",
                "clocks": clocks_roof.summary()}
    w8a8_4096_extra = {"TOPS": achieved}
    if rank == 0 and world == 1:
        w8a8_4096_extra["library_context"] = library_int8_context(hb, K)
        w8a8_4096_extra["w8a8_pipeline_bf16_in"] = w8a8_pipeline(ops, hb, max(10, min(K, 50)),
                                                                 peaks)
    for k in ("A", "B", "sA", "sB"):
        hb.pop(k)
    torch.cuda.empty_cache()

    # ---- the headline: the column-sharded GEMM, strong scaling ----
    log("w8a8 column-sharded headline")
    lo = large_operands(rank, world)
    hl = headline_large(ops, lo, world, K, W, clocks)
    rows = check_rows(LARGE_M)
    parity_ok = all_ranks_true(oracle_rows_check(lo, lo["out"], rows, lo["n0"], lo["n1"],
                                                 lo["B"].cpu().numpy(), lo["sB"].cpu().numpy()),
                               world)
    per_rank_tops = hl["ops_per_rank_launch"] * K / hl["t_local"] / 1e12
    roofline_headline = {"kernel": "w8a8_tcgen05_pair_kernel",
                         "shape": f"M={LARGE_M} N={lo['NL']} K={LARGE_K} per rank",
                         "achieved_per_rank": per_rank_tops, "unit": "TOPS",
                         "peak_sustained": int8_sustained,
                         "frac_of_sustained": per_rank_tops / int8_sustained,
                         "frac_of_burst": per_rank_tops / int8_burst,
                         "basis": "rank 0's own launches; a step of this size runs long enough "
                                  "to meet the power cap, so it is set against 2 x the sustained "
                                  "bf16 rate too"}
    log("e2e")
    e2e = e2e_large(ops, st, lo, world, max(3, min(K, 10)))
    extra = {"w8a8_4096": w8a8_4096_extra, "roofline_headline": roofline_headline,
             "parity": {"oracle_rows_equal_all_ranks": parity_ok, "rows_per_rank": len(rows),
                        "what": "bf16 outputs of sampled rows (first, second, last and 13 "
                                "seeded) of every rank's block, bit for bit against the CPU "
                                "oracle, after the timed region"}}
    if world > 1:
        log("all-gather forms")
        extra["allgather"] = gather_output(st, lo, rank, world)
    del lo
    torch.cuda.empty_cache()
    if world == 1 and rank == 0:
        log("w4a16 decode")
        extra["w4a16_decode"] = w4a16_decode(ops, peaks)
        extra["w4a16_decode"]["peak_GB_s"] = peaks["hbm_gbs"]
        extra["w4a16_decode"]["peak_basis"] = f"hbm_gbs ({peak_src})"
        extra["w4a16_decode"]["traffic_M1"] = NCU_TRAFFIC_W4A16_M1
        torch.cuda.empty_cache()
        log("fp32 facade")
        extra["fp32_facade"] = f32_facade(st, peaks)
        if not args.no_llama:
            log("llama stack")
            extra["llama2_7b_w4a16_stack"] = llama_stack(ops, peaks)
            torch.cuda.empty_cache()
    cpu = None
    if world == 1 and rank == 0 and not args.no_cpu:
        log("cpu baseline")
        cpu = cpu_legs(host_cores())
    if rank == 0:
        line = {
            "metric": METRIC, "value": hl["value"], "unit": "TOPS", "n_gpus": world, "steps": K,
            "warmup": W, "ms_per_step": hl["t_max"] / K * 1e3, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "int8", "data": "synthetic",
            "config": headline_config(world),
            "roofline": roofline, "e2e": e2e, "gpu_launches": K, "clocks": clocks.summary(),
            "cpu_baseline": cpu,
        }
        line.update(extra)
        print(json.dumps(line), flush=True)
    finish()
    return 0


if __name__ == "__main__":
    sys.exit(main())
