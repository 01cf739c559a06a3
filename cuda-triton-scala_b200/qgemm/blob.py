"""Versioned weight blobs (qgemm_blob_* in include/qgemm.h): quantised weights in a
kernel layout plus their scales, checked by magic, version, shape and CRC-32."""
from __future__ import annotations

import ctypes

import numpy as np

from . import _lib as L

KINDS = {"w4_tiled": L.BLOB_W4_TILED, "w8_kn": L.BLOB_W8_KN, "w8_nk": L.BLOB_W8_NK,
         "w4_frag": L.BLOB_W4_FRAG}


def _info(kind: str, K: int, N: int, group_size: int = 0, zero_point: int = 0) -> L.BlobInfo:
    return L.BlobInfo(0, KINDS[kind], K, N, group_size, zero_point, 0, 0)


def _section_bytes(kind: str, K: int, N: int, group_size: int,
                   zero_point: int) -> tuple[int, int]:
    """Weight and scale bytes that `kind` and the shape imply (the library reads exactly
    these from the arrays it is given); (-1, -1) for a shape the library refuses before
    reading anything."""
    n = ctypes.c_size_t(0)
    if K <= 0 or N <= 0:
        return -1, -1
    if kind in ("w4_tiled", "w4_frag"):
        if group_size <= 0 or N % 8 or K % group_size or not 0 <= zero_point <= 15:
            return -1, -1
        L.call("qgemm_w4_tiled_bytes" if kind == "w4_tiled" else "qgemm_w4_frag_bytes", K, N,
               ctypes.byref(n))
        return n.value, (K // group_size) * N * 2
    if group_size != 0 or zero_point != 0:
        return -1, -1
    return K * N, N * 4


def save(path: str, kind: str, K: int, N: int, weights: np.ndarray, scales: np.ndarray, *,
         group_size: int = 0, zero_point: int = 0) -> None:
    """Writes host arrays (their bytes, in the layout `kind` names) to `path`.  Arrays
    whose sizes differ from what the kind and shape imply raise ValueError."""
    w = np.ascontiguousarray(weights)
    s = np.ascontiguousarray(scales)
    if kind not in KINDS:
        raise ValueError(f"unknown blob kind {kind!r}")
    wb, sb = _section_bytes(kind, K, N, group_size, zero_point)
    if wb >= 0 and (w.nbytes != wb or s.nbytes != sb):
        raise ValueError(f"{kind} K={K} N={N}: weights must be {wb} bytes and scales {sb} "
                         f"bytes, got {w.nbytes} and {s.nbytes}")
    info = _info(kind, K, N, group_size, zero_point)
    L.call("qgemm_blob_save", path.encode(), ctypes.byref(info), w.ctypes.data, s.ctypes.data)


def info(path: str) -> dict:
    i = L.BlobInfo()
    L.call("qgemm_blob_info_read", path.encode(), ctypes.byref(i))
    kind = {v: k for k, v in KINDS.items()}[i.kind]
    return {"version": i.version, "kind": kind, "K": i.K, "N": i.N, "group_size": i.group_size,
            "zero_point": i.zero_point, "weight_bytes": i.weight_bytes,
            "scale_bytes": i.scale_bytes}


def load(path: str) -> tuple[dict, np.ndarray, np.ndarray]:
    """(info, weight bytes, scale bytes) as uint8 host arrays, after verification."""
    meta = info(path)
    w = np.empty(meta["weight_bytes"], np.uint8)
    s = np.empty(meta["scale_bytes"], np.uint8)
    L.call("qgemm_blob_load", path.encode(), w.ctypes.data, w.nbytes, s.ctypes.data, s.nbytes)
    return meta, w, s


def load_to_device(stream, path: str, weights, weight_bytes: int, scales, scale_bytes: int):
    """Verifies the file and copies both sections into device buffers."""
    L.call("qgemm_blob_load_device", stream.handle, path.encode(), L.addr(weights), weight_bytes,
           L.addr(scales), scale_bytes)
