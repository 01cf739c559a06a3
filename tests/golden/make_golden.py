"""Generates tests/golden/golden.npz: small golden input/output vectors for the
quantized-matmul operators, from a pure-Python restatement that shares no code
with the C oracle.

The reference (src/main/scala/cuda/dsl/operators/linalg/QuantizedGemmOps.scala)
cannot run here -- there is no JVM, and its operator bodies compute only element
(0,0) because the thread builtins are constant stubs -- so these vectors pin the
C oracle to a second, independent reading of the same Scala statements:
Int arithmetic wraps at 32 bits, Float arithmetic is IEEE binary32 with
round-to-nearest-even (numpy float32 scalars), Float.toInt truncates toward zero
with NaN -> 0 and saturation.

    python tests/golden/make_golden.py      # rewrites golden.npz
"""
from __future__ import annotations

import math
import os
import struct

import numpy as np

f32 = np.float32
HERE = os.path.dirname(os.path.abspath(__file__))


def wrap32(v: int) -> int:
    v &= 0xFFFFFFFF
    return v - (1 << 32) if v >= (1 << 31) else v


def to_int(f) -> int:  # Scala Float.toInt
    f = float(f)
    if math.isnan(f):
        return 0
    if f >= 2147483647.0:
        return 2147483647
    if f <= -2147483648.0:
        return -2147483648
    return int(f)  # truncation toward zero


def bf16_rne(f) -> int:
    u = struct.unpack("<I", struct.pack("<f", float(f32(f))))[0]
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) & 0xFFFF


def bf16_f(h: int):
    return f32(struct.unpack("<f", struct.pack("<I", (int(h) & 0xFFFF) << 16))[0])


def w8a32(w, sw, x, sx, M, N, K):  # QuantizedGemmOps.scala:102-113
    y = np.zeros((M, N), np.float32)
    acc = np.zeros((M, N), np.int32)
    for row in range(M):
        for col in range(N):
            s = 0
            for k in range(K):
                s = wrap32(s + int(w[k * N + col]) * int(x[row * K + k]))
            acc[row, col] = s
            y[row, col] = f32(f32(s) * f32(sw[col])) * f32(sx[row])
    return y, acc


def w4a16(wb, sw, x, M, N, K):  # QuantizedGemmOps.scala:229-245
    y = np.zeros((M, N), np.float32)
    for row in range(M):
        for col in range(N):
            s = f32(0)
            for k in range(K):
                idx = k * N + col
                packed = int(np.int8(wb[idx // 2]))  # Byte.toInt sign-extends
                if idx % 2 == 0:
                    wv = f32(packed & 0x0F) - f32(8)
                else:
                    wv = f32((packed >> 4) & 0x0F) - f32(8)
                s = f32(s + f32(f32(wv * f32(sw[col])) * f32(x[row * K + k])))
            y[row, col] = s
    return y


def w8a16(w, sw, x, bias, M, N, K, has_bias, rowwise):  # :37-53 and :72-82
    y = np.zeros((M, N), np.float32)
    for row in range(M):
        for col in range(N):
            s = f32(0)
            for k in range(K):
                sc = f32(sw[k] if rowwise else sw[col])
                s = f32(s + f32(f32(f32(int(w[k * N + col])) * sc) * f32(x[row * K + k])))
            if has_bias:
                s = f32(s + f32(bias[col]))
            y[row, col] = s
    return y


def quantize(wt, K, N, qbits, with_zeros):  # :131-155 and :173-190
    scales = np.zeros(N, np.float32)
    q = np.zeros((K, N), np.int8)
    for col in range(N):
        mx = f32(0)
        for k in range(K):
            v = f32(abs(f32(wt[k * N + col])))
            if v > mx:
                mx = v
        qmax = f32(127.0) if qbits == 8 else f32(7.0)
        scale = f32(qmax / mx) if mx > f32(1e-6) else f32(1.0)
        scales[col] = f32(mx / qmax)
        lo, hi = (-128, 127) if qbits == 8 else (-8, 7)
        for k in range(K):
            qv = to_int(f32(f32(wt[k * N + col]) * scale))
            q[k, col] = max(lo, min(hi, qv))
    return scales, q


def dequant(q, sc, K, N):  # :207-211
    out = np.zeros(K * N, np.float32)
    for i in range(K * N):
        out[i] = f32(f32(int(q.reshape(-1)[i])) * f32(sc[i % N]))
    return out.reshape(K, N)


def grouped(wq, scales, zp, G, x, M, N, K):
    y = np.zeros((M, N), np.float32)
    yb = np.zeros((M, N), np.uint16)
    for row in range(M):
        for col in range(N):
            s = f32(0)
            for k in range(K):
                idx = k * N + col
                q = (int(wq[idx // 8]) >> (4 * (idx % 8))) & 0xF
                wv = f32(q) - f32(zp)
                s = f32(s + f32(f32(wv * bf16_f(scales[(k // G) * N + col])) * bf16_f(x[row * K + k])))
            y[row, col] = s
            yb[row, col] = bf16_rne(s)
    return y, yb


def main():
    rng = np.random.default_rng(20261201)
    out = {}
    # W8A8 / w8a32Gemm: random, and the int8 extremes (-128 * -128 accumulates)
    for name, (M, N, K, lo) in {"w8a32_rand": (3, 5, 7, -127), "w8a32_ext": (2, 4, 9, -128)}.items():
        w = rng.integers(lo, 128, size=K * N).astype(np.int8)
        x = rng.integers(lo, 128, size=M * K).astype(np.int8)
        if name == "w8a32_ext":
            w[:] = -128
            x[: K] = -128
            x[K:] = 127
        sw = rng.uniform(0.001, 0.01, size=N).astype(np.float32)
        sx = rng.uniform(0.001, 0.01, size=M).astype(np.float32)
        y, acc = w8a32(w, sw, x, sx, M, N, K)
        out.update({f"{name}_w": w.reshape(K, N), f"{name}_sw": sw, f"{name}_x": x.reshape(M, K),
                    f"{name}_sx": sx, f"{name}_y": y, f"{name}_acc": acc})
    # w4a16Gemm with odd N so that nibble pairs straddle rows
    M, N, K = 2, 5, 6
    wb = rng.integers(0, 256, size=(K * N + 1) // 2).astype(np.uint8)
    sw = rng.uniform(0.005, 0.02, size=N).astype(np.float32)
    x = rng.standard_normal(size=M * K).astype(np.float32)
    out.update({"w4a16_w": wb, "w4a16_sw": sw, "w4a16_x": x.reshape(M, K),
                "w4a16_y": w4a16(wb, sw, x, M, N, K), "w4a16_N": np.int32(N)})
    # w8a16Gemm (bias on/off) and RowWise
    M, N, K = 2, 3, 5
    w = rng.integers(-127, 128, size=K * N).astype(np.int8)
    swc = rng.uniform(0.001, 0.01, size=N).astype(np.float32)
    swr = rng.uniform(0.001, 0.01, size=K).astype(np.float32)
    x = rng.standard_normal(size=M * K).astype(np.float32)
    b = rng.standard_normal(size=N).astype(np.float32)
    out.update({"w8a16_w": w.reshape(K, N), "w8a16_swc": swc, "w8a16_swr": swr,
                "w8a16_x": x.reshape(M, K), "w8a16_b": b,
                "w8a16_y_bias": w8a16(w, swc, x, b, M, N, K, True, False),
                "w8a16_y_nobias": w8a16(w, swc, x, b, M, N, K, False, False),
                "w8a16_y_rowwise": w8a16(w, swr, x, b, M, N, K, False, True)})
    # quantizers: NaN, Inf, a tiny column (scale 1), exact and truncated products
    K, N = 4, 5
    wt = np.array([[0.25, np.nan, 1e-7, np.inf, -3.0],
                   [-1.0, 2.0, -5e-8, 1.0, 1.5],
                   [0.5, -0.7, 2e-7, -2.0, -0.01],
                   [0.999, 0.3, 0.0, 0.5, 2.9]], np.float32)
    for qb in (8, 4):
        s, q = quantize(wt.reshape(-1), K, N, qb, False)
        out.update({f"quant{qb}_scales": s, f"quant{qb}_q": q})
    out["quant_w"] = wt
    sdq = rng.uniform(0.001, 0.1, size=N).astype(np.float32)
    qdq = rng.integers(-128, 128, size=(K, N)).astype(np.int8)
    out.update({"dq_q": qdq, "dq_s": sdq, "dq_w": dequant(qdq, sdq, K, N)})
    # grouped W4A16, two zero points
    M, N, K, G = 2, 16, 32, 16
    wq = rng.integers(0, 2**32, size=K * N // 8, dtype=np.uint64).astype(np.uint32)
    sc = np.array([bf16_rne(v) for v in rng.uniform(0.005, 0.02, size=(K // G) * N)], np.uint16)
    xb = np.array([bf16_rne(v) for v in rng.standard_normal(size=M * K)], np.uint16)
    for zp in (8, 3):
        y, yb = grouped(wq, sc, zp, G, xb, M, N, K)
        out.update({f"grp{zp}_y": y, f"grp{zp}_yb": yb})
    out.update({"grp_wq": wq.reshape(K, N // 8), "grp_sc": sc.reshape(K // G, N),
                "grp_x": xb.reshape(M, K), "grp_G": np.int32(G)})
    np.savez_compressed(os.path.join(HERE, "golden.npz"), **out)
    print("wrote", os.path.join(HERE, "golden.npz"), len(out), "arrays")


if __name__ == "__main__":
    main()
