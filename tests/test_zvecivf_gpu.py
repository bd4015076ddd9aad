"""IVF indexes with their lists given: a ZVECIVF file opened onto the device
(xvec_gpu_ivf_open, OpenIVFIndex ivf.go:815-830) and rows added with lists
(xvec_gpu_ivf_add_with_lists) search exactly like the oracle's IVF over those
same lists, which here are not the rows' nearest centroids (as after streaming
adds, ivf.go:653-709).  Keys identical, float32 scores bit-identical."""
import numpy as np
import pytest

from oracle.oracle import COSINE, IP, L2
from oracle.zvecivf import csr_of, encode_ivf

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def xb():
    import xvec_b200
    assert xvec_b200.device_count() >= 1
    return xvec_b200


def data(seed, n=3000, d=48, nlist=16):
    rng = np.random.default_rng(seed)
    centers = rng.standard_normal((20, d)).astype(np.float32)
    rows = (centers[rng.integers(0, 20, n)] + 0.3 * rng.standard_normal((n, d))).astype(np.float32)
    keys = rng.permutation(1 << 20)[:n].astype(np.uint64)
    cents = rows[rng.choice(n, nlist, replace=False)].copy()
    lists = rng.integers(0, nlist, n).astype(np.int32)
    queries = (centers[rng.integers(0, 20, 37)] + 0.3 * rng.standard_normal((37, d))).astype(
        np.float32)
    return rows, keys, cents, lists, queries


def compare(res, ok, os_, oc, ost):
    for q in range(ok.shape[0]):
        if ost[q] != 0:
            assert res.counts[q] < 0, q
            continue
        c = int(oc[q])
        assert int(res.counts[q]) == c, (q, res.counts[q], c)
        assert np.array_equal(res.keys[q, :c], ok[q, :c]), q
        assert np.array_equal(res.scores[q, :c].view(np.uint32), os_[q, :c].view(np.uint32)), q


@pytest.mark.parametrize("metric", [L2, IP, COSINE])
def test_open_file_keeps_its_lists(oracle, xb, tmp_path, metric):
    rows, keys, cents, lists, queries = data(900 + metric)
    path = tmp_path / "index.ivf"
    path.write_bytes(encode_ivf(metric, cents, keys, rows, lists, 16, 10, cost=1.5,
                                train_iterations=4))
    idx = xb.IVFIndex.open(str(path))
    assert len(idx) == rows.shape[0]
    offsets, positions = csr_of(lists, 16)
    for k, nprobe in ((10, 4), (25, 16)):
        res = idx.search_with_options(queries, xb.SearchOptions(top_k=k, nprobe=nprobe),
                                      raise_on_error=False)
        _, ok, os_, oc, ost = oracle.ivf_flat_search(metric, rows, keys, cents, offsets, positions,
                                                     queries, k, nprobe)
        compare(res, ok, os_, oc, ost)
    idx.close()


def test_sq8_ivf_add_with_lists(oracle, xb):
    rows, keys, cents, lists, queries = data(77)
    idx = xb.ScalarQuantizedIVFIndex(rows.shape[1], L2)
    idx.set_model(cents)
    idx.add_with_lists(keys[:1000], rows[:1000], lists[:1000])
    idx.add_with_lists(keys[1000:], rows[1000:], lists[1000:])
    with pytest.raises(xb.XvecGPUError):
        idx.add_with_lists(np.array([1 << 40], np.uint64), rows[:1], np.array([16], np.int32))
    offsets, positions = csr_of(lists, 16)
    codes, params = oracle.quantize_int8_batch(rows)
    for scale in (0.0, 3.0):
        res = idx.search_with_options(queries, xb.SearchOptions(top_k=10, nprobe=5,
                                                                 refine_scale=scale),
                                      raise_on_error=False)
        _, ok, os_, oc, ost = oracle.ivf_sq8_search(L2, codes, params, rows, keys, cents, offsets,
                                                    positions, queries, 10, 5, refine_scale=scale)
        compare(res, ok, os_, oc, ost)
    idx.close()
