"""The ZVECIVF reader on the host (xvec_gpu_ivf_file_info) against files in
the layout of IVFIndex.Save (ivf.go:866-904), with the reference's own
persistence tests ported: TestIVFPersistenceDetectsTruncationAndCorruption
and TestIVFPersistenceRejectsSemanticCorruption (ivf_test.go:842-955),
TestIVFPersistenceEmpty (:762-782).  No device work."""
import math
import struct

import numpy as np
import pytest

from oracle.oracle import COSINE, L2
from oracle.zvecivf import HEADER, crc32c, encode_ivf, rechecksum


@pytest.fixture(scope="module")
def xb():
    import xvec_b200
    return xvec_b200


def persisted(oracle, metric=L2, nlist=2):
    """persistedIVFIndex (ivf_test.go:1046-1073): five 3-d vectors, NList 2,
    NIterations 7, Tolerance 1e-8, Workers 2, Seed 0x123456789abcdef0; the
    centroids from the oracle's TrainKMeans, each row in its nearest list."""
    keys = np.array([41, 7, 99, 5, 123], np.uint64)
    vecs = np.array([[1, 0, 0], [0, 1, 0], [0, 0, 1], [1, 1, 0], [0.5, 0.25, 0.75]], np.float32)
    st, cents, labels = oracle.kmeans_train(metric, vecs, nlist, 7, 1e-8, 0x123456789abcdef0)
    assert st == 0
    return encode_ivf(metric, cents, keys, vecs, labels, nlist, 7, 2, 0x123456789abcdef0, 1e-8,
                      cost=0.5, train_iterations=3, converged=True)


def info_status(xb, tmp_path, data, name="f.ivf"):
    p = tmp_path / name
    p.write_bytes(bytes(data))
    try:
        return 0, xb.ivf_file_info(str(p))
    except xb.XvecGPUError as e:
        return e.status, None


def test_crc32c_check_value():
    # The CRC-32C (Castagnoli) check value of "123456789".
    assert crc32c(b"123456789") == 0xE3069283
    assert crc32c(b"") == 0


def test_round_trip_header(oracle, xb, tmp_path):
    valid = persisted(oracle)
    st, info = info_status(xb, tmp_path, valid)
    assert st == 0
    assert info["count"] == 5 and info["dimension"] == 3 and info["nlist"] == 2
    assert info["metric"] == L2 and info["converged"] == 1
    assert info["options_nlist"] == 2 and info["options_iterations"] == 7
    assert info["options_workers"] == 2 and info["options_seed"] == 0x123456789abcdef0
    assert info["options_tolerance"] == 1e-8 and info["training_cost"] == 0.5
    assert info["training_iterations"] == 3


def test_truncation_and_corruption(oracle, xb, tmp_path):
    valid = persisted(oracle)
    for cut in (0, 1, HEADER - 1, HEADER, len(valid) - 1):
        assert info_status(xb, tmp_path, valid[:cut])[0] == xb.INVALID_ARGUMENT, cut
    assert info_status(xb, tmp_path, valid + b"\x00")[0] == xb.INVALID_ARGUMENT
    bad = bytearray(valid)
    bad[0] ^= 1
    assert info_status(xb, tmp_path, bad)[0] == xb.INVALID_ARGUMENT
    bad = bytearray(valid)
    struct.pack_into("<H", bad, 8, 2)
    assert info_status(xb, tmp_path, bad)[0] == xb.UNSUPPORTED
    bad = bytearray(valid)
    bad[55] ^= 1
    assert info_status(xb, tmp_path, bad)[0] == xb.CHECKSUM_MISMATCH
    bad = bytearray(valid)
    bad[-1] ^= 1
    assert info_status(xb, tmp_path, bad)[0] == xb.CHECKSUM_MISMATCH


def test_semantic_corruption(oracle, xb, tmp_path):
    valid = persisted(oracle)
    dim = struct.unpack_from("<I", valid, 40)[0]
    nlist = struct.unpack_from("<I", valid, 44)[0]
    first = HEADER + nlist * dim * 4
    rec = 12 + dim * 4

    def dup(b):
        b[first + rec:first + rec + 8] = b[first:first + 8]

    def list_range(b):
        struct.pack_into("<I", b, first + 8 + dim * 4, nlist)

    def nan_centroid(b):
        struct.pack_into("<f", b, HEADER, math.nan)

    def inf_vector(b):
        struct.pack_into("<f", b, first + 8, math.inf)

    for mutate in (dup, list_range, nan_centroid, inf_vector):
        b = bytearray(valid)
        mutate(b)
        rechecksum(b)
        assert info_status(xb, tmp_path, b)[0] == xb.INVALID_ARGUMENT, mutate.__name__
    b = bytearray(valid)
    struct.pack_into("<I", b, 52, 0)                # options NList 0
    struct.pack_into("<I", b, 108, crc32c(b[:108]))
    assert info_status(xb, tmp_path, b)[0] == xb.INVALID_ARGUMENT
    b = bytearray(valid)
    struct.pack_into("<Q", b, 16, len(b) + 1)       # file length
    struct.pack_into("<I", b, 108, crc32c(b[:108]))
    assert info_status(xb, tmp_path, b)[0] == xb.INVALID_ARGUMENT
    b = bytearray(valid)
    struct.pack_into("<I", b, 92, 8)                # training iterations above NIterations
    struct.pack_into("<I", b, 108, crc32c(b[:108]))
    assert info_status(xb, tmp_path, b)[0] == xb.INVALID_ARGUMENT
    b = bytearray(valid)
    b[12] = 1                                       # reserved field
    struct.pack_into("<I", b, 108, crc32c(b[:108]))
    assert info_status(xb, tmp_path, b)[0] == xb.INVALID_ARGUMENT


def test_empty_and_list_counts(oracle, xb, tmp_path):
    empty = encode_ivf(COSINE, np.zeros((0, 4), np.float32), np.zeros(0, np.uint64),
                       np.zeros((0, 4), np.float32), np.zeros(0, np.uint32), 8, 10)
    st, info = info_status(xb, tmp_path, empty)
    assert st == 0 and info["count"] == 0 and info["nlist"] == 0 and info["dimension"] == 4
    b = bytearray(empty)
    struct.pack_into("<d", b, 84, 1.0)              # training cost on an empty index
    struct.pack_into("<I", b, 108, crc32c(b[:108]))
    assert info_status(xb, tmp_path, b)[0] == xb.INVALID_ARGUMENT
    # More lists than rows.
    rng = np.random.default_rng(1)
    v = rng.standard_normal((3, 4)).astype(np.float32)
    many = encode_ivf(L2, rng.standard_normal((4, 4)), np.arange(3), v, [0, 1, 2], 4, 10)
    assert info_status(xb, tmp_path, many)[0] == xb.INVALID_ARGUMENT
    with pytest.raises(xb.XvecGPUError):
        xb.ivf_file_info(str(tmp_path / "missing.ivf"))
