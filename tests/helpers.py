"""Shared helpers for the GPU parity tests (device buffers via libqgemm)."""
from __future__ import annotations

import numpy as np

import qgemm
from qgemm import Buffer

GUARD = 256  # canary bytes on each side of every output buffer
CANARY = 0xA5


class Out:
    """A device output buffer with canary bands around it."""

    def __init__(self, dev, st, nbytes: int):
        self.buf = Buffer(dev, nbytes + 2 * GUARD)
        st.memset(self.buf.address, CANARY, nbytes + 2 * GUARD)
        self.address = self.buf.address + GUARD
        self.nbytes = nbytes
        self.st = st

    def read(self, dtype, shape):
        raw = self.buf.to_numpy(self.st, np.uint8, (self.nbytes + 2 * GUARD,))
        assert (raw[:GUARD] == CANARY).all(), "write before the output buffer"
        assert (raw[GUARD + self.nbytes:] == CANARY).all(), "write past the output buffer"
        return raw[GUARD:GUARD + self.nbytes].view(dtype).reshape(shape)


def dev_array(gpu, arr: np.ndarray) -> Buffer:
    dev, st, _ = gpu
    return Buffer.from_numpy(dev, st, np.ascontiguousarray(arr))


def rel_err(y: np.ndarray, ref: np.ndarray) -> float:
    """max_i |y_i - r_i| / max(|r_i|, 1e-2 * rms(r)): elementwise relative error
    with a floor so that outputs near zero are judged against the output scale."""
    y = y.astype(np.float64)
    ref = ref.astype(np.float64)
    floor = 1e-2 * float(np.sqrt(np.mean(ref * ref))) + 1e-30
    return float(np.max(np.abs(y - ref) / np.maximum(np.abs(ref), floor)))


def rel_errs(y: np.ndarray, ref: np.ndarray) -> tuple[float, float]:
    """(floored, plain): rel_err above, and the plain elementwise max_i |y_i - r_i| / |r_i|
    over the outputs with r_i != 0 (reported beside the gate: an output near zero makes
    the plain figure large under any change of summation order)."""
    y = y.astype(np.float64)
    ref = ref.astype(np.float64)
    nz = ref != 0
    plain = float(np.max(np.abs(y[nz] - ref[nz]) / np.abs(ref[nz]))) if nz.any() else 0.0
    return rel_err(y, ref), plain


def gemm_bound_ratio(y, A, B, *, bias=None, C=None, alpha=1.0, beta=0.0) -> float:
    """max_ij |y_ij - exact_ij| / (|alpha| sum_k |A_ik B_kj| + |bias_j| + |beta C_ij|),
    the exact value taken in float64: the forward-error measure of a floating-point
    GEMM.  A sequential fp32 loop over K stays below K * 2^-24 of it; the fp32 gate is
    1e-5.  Elements whose denominator is 0 must be exact."""
    A64 = np.asarray(A, np.float64)
    B64 = np.asarray(B, np.float64)
    exact = alpha * (A64 @ B64)
    scale = abs(alpha) * (np.abs(A64) @ np.abs(B64))
    if bias is not None:
        exact = exact + np.asarray(bias, np.float64)[None, :]
        scale = scale + np.abs(np.asarray(bias, np.float64))[None, :]
    if C is not None and beta != 0.0:
        C64 = np.asarray(C, np.float64)
        exact = exact + beta * C64
        scale = scale + abs(beta) * np.abs(C64)
    err = np.abs(np.asarray(y, np.float64) - exact)
    if (err[scale == 0] != 0).any():
        return float("inf")
    nz = scale > 0
    return float(np.max(err[nz] / scale[nz])) if nz.any() else 0.0


def gemv_bound_ratio(y, A, x) -> float:
    """gemm_bound_ratio for y = A x."""
    return gemm_bound_ratio(np.asarray(y)[:, None], A, np.asarray(x)[:, None])
