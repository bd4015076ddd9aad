"""The rotation reformer on the GPU (RotationReformer.Transform / Revert,
internal/core/rotation.go:248-280, over FHTRotator.Rotate / Unrotate,
rotation.go:123-185): bit-identical to the oracle's restatement for powers
of two, even and odd dimensions (the Kac walk's middle element), the
reference's own fixture (rotation_test.go:32-50), the round trip and norm
of rotation_test.go:52-75, non-finite vectors, the device form's per-vector
flags, and a dimension too large for shared memory."""
import json
import os

import numpy as np
import pytest

from oracle.oracle import collection_rotation_signs

pytestmark = pytest.mark.gpu

FIX = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "reference_fixtures.json")))


@pytest.fixture(scope="module")
def xb():
    import xvec_b200
    assert xvec_b200.device_count() >= 1
    return xvec_b200


@pytest.mark.parametrize("dim", [1, 2, 3, 4, 7, 9, 11, 64, 100, 127, 768, 1000, 4096, 5000])
def test_rotate_and_revert_equal_the_oracle(oracle, xb, dim):
    rng = np.random.default_rng(dim)
    signs = collection_rotation_signs("docs", "embedding", dim, 1, 2)
    vecs = rng.standard_normal((37, dim)).astype(np.float32)
    r = xb.RotationReformer(dim, signs)
    got = r.transform(vecs)
    back = r.revert(got)
    for i in range(vecs.shape[0]):
        st, want = oracle.fht_rotate(signs, vecs[i])
        assert st == 0
        assert np.array_equal(got[i].view(np.uint32), want.view(np.uint32)), i
        st, wback = oracle.fht_unrotate(signs, want)
        assert st == 0
        assert np.array_equal(back[i].view(np.uint32), wback.view(np.uint32)), i
    # rotation_test.go:52-75: the round trip and the norm within 2e-4.
    assert np.allclose(back, vecs, atol=2e-4 * max(1.0, float(np.abs(vecs).max())))
    n0 = (vecs.astype(np.float64) ** 2).sum(axis=1)
    n1 = (got.astype(np.float64) ** 2).sum(axis=1)
    assert np.all(np.abs(n0 - n1) <= 2e-4 * np.maximum(1.0, n0))


def test_reference_fixture(xb):
    f = FIX["fht_rotator"]
    r = xb.RotationReformer(len(f["input"]), np.array(f["signs"], np.uint8))
    out = r.transform(np.array(f["input"], np.float32))
    assert np.allclose(out, f["rotated"], atol=1e-6)


def test_non_finite_vectors_fail(xb):
    dim = 33
    signs = collection_rotation_signs("s", "f", dim, 0, 0)
    r = xb.RotationReformer(dim, signs)
    v = np.ones((5, dim), np.float32)
    v[3, 7] = np.inf
    with pytest.raises(xb.XvecGPUError) as e:
        r.transform(v)
    assert e.value.status == xb.NON_FINITE and "vector 3" in str(e.value)
    big = np.full((2, dim), 3e38, np.float32)  # finite input, overflowing result
    with pytest.raises(xb.XvecGPUError):
        r.transform(big)


def test_device_form_flags_each_vector(oracle, xb):
    import torch
    dim, n = 300, 64
    signs = collection_rotation_signs("s", "f", dim, 3, 1)
    rng = np.random.default_rng(5)
    v = rng.standard_normal((n, dim)).astype(np.float32)
    v[10, 0] = np.nan
    d_in = torch.from_numpy(v).cuda()
    d_out = torch.empty_like(d_in)
    failed = torch.full((n,), -1, dtype=torch.int32, device="cuda")
    r = xb.RotationReformer(dim, signs)
    r.transform_device(d_in.data_ptr(), n, d_out.data_ptr(), failed.data_ptr(),
                       stream=torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    f = failed.cpu().numpy()
    assert f[10] == 1 and f.sum() == 1
    out = d_out.cpu().numpy()
    for i in (0, 63):
        _, want = oracle.fht_rotate(signs, v[i])
        assert np.array_equal(out[i].view(np.uint32), want.view(np.uint32))


def test_dimension_beyond_shared_memory(oracle, xb):
    dim = 60001  # rotated in the block's row of global memory
    signs = collection_rotation_signs("s", "f", dim, 0, 0)
    v = np.random.default_rng(6).standard_normal((3, dim)).astype(np.float32)
    r = xb.RotationReformer(dim, signs)
    got = r.transform(v)
    back = r.revert(got)
    for i in range(3):
        _, want = oracle.fht_rotate(signs, v[i])
        assert np.array_equal(got[i].view(np.uint32), want.view(np.uint32))
        _, wback = oracle.fht_unrotate(signs, want)
        assert np.array_equal(back[i].view(np.uint32), wback.view(np.uint32))
