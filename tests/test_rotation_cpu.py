"""The rotation reformer's sign state (collectionReformer,
collection.go:1981-2000) needs no GPU: the library's SHA-256 derivation must
equal the oracle's (hashlib over the same seed text and counters), and the
sizes and dimensions the reference rejects are rejected."""
import numpy as np
import pytest

from oracle.oracle import collection_rotation_signs


@pytest.mark.parametrize("schema,field,dim,itype,quant", [
    ("docs", "embedding", 768, 1, 2), ("s", "v", 1, 0, 0), ("schema-with-a-long-name" * 4,
                                                            "f", 65535, 7, 3),
    ("été", "champ", 100, 2, 1), ("", "", 9, 0, 0)])
def test_signs_equal_the_oracle(schema, field, dim, itype, quant):
    import xvec_b200 as xb
    got = xb.rotation_signs(schema, field, dim, itype, quant)
    want = collection_rotation_signs(schema, field, dim, itype, quant)
    assert got.dtype == np.uint8 and got.size == 4 * ((dim + 7) // 8)
    assert np.array_equal(got, want)


def test_signs_argument_checks():
    import ctypes
    import xvec_b200 as xb
    lib = xb.library()
    out = np.zeros(64, np.uint8)
    for dim in (0, -1, 65536):
        assert lib.xvec_gpu_rotation_signs(b"s", b"f", dim, 0, 0, out.ctypes.data, 64) == \
            xb.INVALID_ARGUMENT
    assert lib.xvec_gpu_rotation_signs(b"s", b"f", 100, 0, 0, out.ctypes.data, 64) == \
        xb.INVALID_ARGUMENT  # 100 needs 52 bytes
    assert lib.xvec_gpu_rotation_signs(None, b"f", 8, 0, 0, out.ctypes.data, 4) == \
        xb.INVALID_ARGUMENT
    signs = np.zeros(4, np.uint8)
    assert lib.xvec_gpu_rotate(0, signs.ctypes.data, 4, 9, None, 1, None, 0) == \
        xb.INVALID_ARGUMENT  # 9 needs 8 bytes of signs
    assert ctypes  # (imported for the library's argtypes)
