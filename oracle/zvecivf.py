"""ZVECIVF version 1 files for the tests: the layout of IVFIndex.Save
(encodeIVFIndex, internal/core/ivf.go:866-904) restated, with the CRC-32C
(Castagnoli) checksums of hashutil.CRC32C (internal/ailego/hash/crc32c.go:22).

Test infrastructure: files written here are read by the library under test
(xvec_gpu_ivf_file_info, xvec_gpu_ivf_open).  Header layout, little endian:
magic "ZVECIVF\\0", version 1, header size 112, reserved, file length, payload
length, count, dimension, effective nlist, metric, converged, reserved, options
NList, NIterations, Workers, Seed, Tolerance, training cost, training
iterations, payload CRC, reserved, header CRC; then nlist float32 centroids and
count records {uint64 key, float32 vector, uint32 list}."""
import struct

import numpy as np

HEADER = 112
_POLY = 0x82F63B78  # reflected Castagnoli polynomial


def _table():
    t = []
    for b in range(256):
        c = b
        for _ in range(8):
            c = (c >> 1) ^ _POLY if c & 1 else c >> 1
        t.append(c)
    return t


_TABLE = _table()


def crc32c(data) -> int:
    """CRC-32C: initial value and final xor 0xFFFFFFFF, reflected."""
    c = 0xFFFFFFFF
    t = _TABLE
    for b in bytes(data):
        c = (c >> 8) ^ t[(c ^ b) & 0xFF]
    return c ^ 0xFFFFFFFF


def encode_ivf(metric, centroids, keys, vectors, lists, nlist_option, iterations, workers=0,
               seed=0, tolerance=1e-4, cost=0.0, train_iterations=0, converged=False) -> bytes:
    """The file IVFIndex.Save writes for an index with these centroids, rows
    (in position order) and the list of each row."""
    centroids = np.ascontiguousarray(centroids, np.float32)
    vectors = np.ascontiguousarray(vectors, np.float32)
    keys = np.ascontiguousarray(keys, np.uint64)
    lists = np.ascontiguousarray(lists, np.uint32)
    count = keys.size
    dim = vectors.shape[1] if vectors.ndim == 2 and vectors.shape[1] else centroids.shape[-1]
    nlist = centroids.shape[0] if count else 0
    rec = np.zeros(count, dtype=[("key", "<u8"), ("vec", "<f4", (dim,)), ("list", "<u4")])
    rec["key"], rec["vec"], rec["list"] = keys, vectors.reshape(count, dim), lists
    payload = (centroids[:nlist].astype("<f4").tobytes() if nlist else b"") + rec.tobytes()
    h = bytearray(HEADER)
    h[0:8] = b"ZVECIVF\x00"
    struct.pack_into("<HH", h, 8, 1, HEADER)
    struct.pack_into("<QQQ", h, 16, HEADER + len(payload), len(payload), count)
    struct.pack_into("<II", h, 40, dim, nlist)
    h[48] = metric
    h[49] = 1 if (converged and count) else 0
    struct.pack_into("<IIqQd", h, 52, nlist_option, iterations, workers, seed, tolerance)
    if count:
        struct.pack_into("<dI", h, 84, cost, train_iterations)
    struct.pack_into("<I", h, 96, crc32c(payload))
    struct.pack_into("<I", h, 108, crc32c(h[:108]))
    return bytes(h) + payload


def rechecksum(buf: bytearray) -> None:
    """Recomputes both checksums after a mutation (rechecksumIVF in the
    reference's tests)."""
    struct.pack_into("<I", buf, 96, crc32c(buf[HEADER:]))
    struct.pack_into("<I", buf, 108, crc32c(buf[:108]))


def csr_of(lists, nlist):
    """list_offsets [nlist + 1] and positions in list order (position order
    within a list), as IVFIndex keeps them."""
    lists = np.asarray(lists, np.int64)
    offsets = np.zeros(nlist + 1, np.int64)
    np.add.at(offsets, lists + 1, 1)
    return np.cumsum(offsets), np.argsort(lists, kind="stable").astype(np.int64)
