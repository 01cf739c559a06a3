"""Seeded synthetic inputs with the shapes and value distributions of the
benchmark workloads (numpy PCG64; the seed is recorded with every result).

  int8 operands        U{-127..127}
  fp32 scales          U[lo, hi]   (per token / per channel)
  int4 weights         U{0..15}, zero point 8, packed 8 per uint32 in the
                       reference nibble order (element k*N+n at nibble
                       (k*N+n) % 8 of word (k*N+n) // 8, low nibble first)
  bf16 scales          U[0.005, 0.02], round to nearest even
  bf16 activations     N(0, 1), round to nearest even
"""
from __future__ import annotations

import numpy as np


def bf16_bits(a: np.ndarray) -> np.ndarray:
    """float32 -> bf16 bit patterns, round to nearest even (finite inputs)."""
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32).astype(np.uint64)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def bf16_to_float(h: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(h, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def w8a8_inputs(M: int, N: int, K: int, seed: int = 0, sa=(0.001, 0.01), sb=(0.001, 0.01)):
    """A int8 [M,K], B int8 [K,N] (reference layout), sA f32 [M], sB f32 [N]."""
    rng = np.random.default_rng(seed)
    A = rng.integers(-127, 128, size=(M, K), dtype=np.int8)
    B = rng.integers(-127, 128, size=(K, N), dtype=np.int8)
    sA = rng.uniform(sa[0], sa[1], size=M).astype(np.float32)
    sB = rng.uniform(sb[0], sb[1], size=N).astype(np.float32)
    return A, B, sA, sB


def pack_int4(q: np.ndarray) -> np.ndarray:
    """q uint8 [K,N] in 0..15 -> uint32 [K, N/8] (nibble j of word (k,c) = q[k, 8c+j])."""
    K, N = q.shape
    assert N % 8 == 0
    q = q.astype(np.uint32).reshape(K, N // 8, 8)
    w = np.zeros((K, N // 8), np.uint32)
    for j in range(8):
        w |= q[:, :, j] << np.uint32(4 * j)
    return w


def unpack_int4(w: np.ndarray, N: int) -> np.ndarray:
    K = w.shape[0]
    out = np.empty((K, N // 8, 8), np.uint8)
    for j in range(8):
        out[:, :, j] = (w >> np.uint32(4 * j)) & 0xF
    return out.reshape(K, N)


def w4a16_inputs(M: int, N: int, K: int, group: int = 128, seed: int = 0):
    """x bf16 bits [M,K], wq uint32 [K,N/8], scales bf16 bits [K/group, N]."""
    rng = np.random.default_rng(seed)
    x = bf16_bits(rng.standard_normal(size=(M, K), dtype=np.float32))
    q = rng.integers(0, 16, size=(K, N), dtype=np.uint8)
    wq = pack_int4(q)
    scales = bf16_bits(rng.uniform(0.005, 0.02, size=(K // group, N)).astype(np.float32))
    return x, wq, scales
