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
