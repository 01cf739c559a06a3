"""Weight blobs on the host: round trips, and every kind of damage is refused with a
status instead of being loaded (no GPU needed)."""
import os

import numpy as np
import pytest

import qgemm
import qgemm._lib as L
from qgemm import blob


def w4_arrays(K, N, G, seed=0):
    rng = np.random.default_rng(seed)
    nbytes = ((N + 63) // 64) * K * 32
    return (rng.integers(0, 256, nbytes, dtype=np.uint8),
            rng.integers(0, 2**16, (K // G, N), dtype=np.uint16))


def test_round_trip_w4(tmp_path):
    K, N, G = 512, 264, 128
    w, s = w4_arrays(K, N, G)
    p = str(tmp_path / "w.qgb")
    blob.save(p, "w4_tiled", K, N, w, s, group_size=G, zero_point=8)
    meta, w2, s2 = blob.load(p)
    assert meta == {"version": 1, "kind": "w4_tiled", "K": K, "N": N, "group_size": G,
                    "zero_point": 8, "weight_bytes": w.nbytes, "scale_bytes": s.nbytes}
    np.testing.assert_array_equal(w2, w)
    np.testing.assert_array_equal(s2.view(np.uint16).reshape(K // G, N), s)
    assert os.path.getsize(p) == 64 + w.nbytes + s.nbytes


def test_round_trip_w4_frag(tmp_path):
    """The fragment-order kind: weight bytes N/8 * ceil(K/128) * 512 (K = 160: two
    128-row blocks, the second partly past K)."""
    K, N, G = 160, 24, 32
    rng = np.random.default_rng(3)
    w = rng.integers(0, 256, (N // 8) * 2 * 512, dtype=np.uint8)
    s = rng.integers(0, 2**16, (K // G, N), dtype=np.uint16)
    p = str(tmp_path / "f.qgb")
    blob.save(p, "w4_frag", K, N, w, s, group_size=G, zero_point=8)
    meta, w2, s2 = blob.load(p)
    assert meta["kind"] == "w4_frag" and meta["weight_bytes"] == w.nbytes
    np.testing.assert_array_equal(w2, w)
    np.testing.assert_array_equal(s2.view(np.uint16).reshape(K // G, N), s)
    with pytest.raises(ValueError):  # a weight section of the wrong size
        blob.save(p, "w4_frag", K, N, w[:1024], s, group_size=G, zero_point=8)


@pytest.mark.parametrize("kind", ["w8_kn", "w8_nk"])
def test_round_trip_w8(tmp_path, kind):
    K, N = 300, 128
    rng = np.random.default_rng(1)
    w = rng.integers(-128, 128, (K, N) if kind == "w8_kn" else (N, K), dtype=np.int8)
    s = rng.uniform(0.001, 0.01, N).astype(np.float32)
    p = str(tmp_path / "w.qgb")
    blob.save(p, kind, K, N, w, s)
    meta, w2, s2 = blob.load(p)
    assert meta["kind"] == kind
    np.testing.assert_array_equal(w2.view(np.int8).reshape(w.shape), w)
    np.testing.assert_array_equal(s2.view(np.float32), s)


def damaged(tmp_path, offset, value=None, truncate=None):
    K, N, G = 128, 64, 64
    w, s = w4_arrays(K, N, G, seed=2)
    p = str(tmp_path / "d.qgb")
    blob.save(p, "w4_tiled", K, N, w, s, group_size=G, zero_point=8)
    data = bytearray(open(p, "rb").read())
    if truncate is not None:
        data = data[:truncate]
    else:
        data[offset] = (data[offset] ^ 0xFF) if value is None else value
    open(p, "wb").write(bytes(data))
    return p


@pytest.mark.parametrize("offset,what", [(64 + 5, "weight section checksum"),
                                         (64 + 128 * 32 + 3, "scale section checksum"),
                                         (17, "header checksum"), (0, "not a qgemm weight blob")])
def test_damage_is_refused(tmp_path, offset, what):
    p = damaged(tmp_path, offset)
    with pytest.raises(qgemm.QGemmError) as e:
        blob.load(p)
    assert e.value.status == L.ERR_INVALID_ARG
    assert what in str(e.value)


def test_truncated_file_is_refused(tmp_path):
    p = damaged(tmp_path, 0, truncate=64 + 100)
    with pytest.raises(qgemm.QGemmError) as e:
        blob.load(p)
    assert "truncated" in str(e.value)


def test_other_version_is_unsupported(tmp_path):
    K, N, G = 128, 64, 64
    w, s = w4_arrays(K, N, G)
    p = str(tmp_path / "v.qgb")
    blob.save(p, "w4_tiled", K, N, w, s, group_size=G, zero_point=8)
    data = bytearray(open(p, "rb").read())
    data[8] = 2                                   # version 2
    import zlib
    data[56:60] = zlib.crc32(bytes(data[:56])).to_bytes(4, "little")  # a consistent header
    open(p, "wb").write(bytes(data))
    with pytest.raises(qgemm.QGemmError) as e:
        blob.info(p)
    assert e.value.status == L.ERR_UNSUPPORTED


def test_crc_matches_zlib(tmp_path):
    """The section checksums are standard CRC-32 (what zlib computes)."""
    import zlib
    K, N, G = 128, 64, 64
    w, s = w4_arrays(K, N, G, seed=4)
    p = str(tmp_path / "c.qgb")
    blob.save(p, "w4_tiled", K, N, w, s, group_size=G, zero_point=3)
    h = open(p, "rb").read(64)
    assert int.from_bytes(h[48:52], "little") == zlib.crc32(w.tobytes())
    assert int.from_bytes(h[52:56], "little") == zlib.crc32(s.tobytes())


@pytest.mark.parametrize("kind,K,N,G,zp", [("w4_tiled", 100, 64, 64, 8), ("w4_tiled", 128, 60, 64, 8),
                                          ("w4_tiled", 128, 64, 64, 16), ("w8_kn", 64, 64, 32, 0)])
def test_bad_shapes_are_refused_on_save(tmp_path, kind, K, N, G, zp):
    with pytest.raises(qgemm.QGemmError) as e:
        blob.save(str(tmp_path / "b.qgb"), kind, K, N, np.zeros(1 << 16, np.uint8),
                  np.zeros(1 << 16, np.uint8), group_size=G, zero_point=zp)
    assert e.value.status == L.ERR_INVALID_ARG
