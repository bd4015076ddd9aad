"""INT8 scalar-quantized Flat search (+ refinement): the CUDA path against the
oracle's SQ-Flat restatement.  Keys identical, float32 scores bit-identical."""
import numpy as np
import pytest

from oracle.oracle import COSINE, IP, L2, MIPSL2

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def xb():
    import xvec_b200
    assert xvec_b200.device_count() >= 1
    return xvec_b200


def scaled_gaussian(rng, n, d):
    s = rng.uniform(0.5, 2.0, d).astype(np.float32)
    return (rng.standard_normal((n, d)).astype(np.float32) * s)


def run(oracle, xb, metric, rows, keys, queries, k, refine=0.0, radius=0.0, bitmap=None):
    idx = xb.ScalarQuantizedFlatIndex(rows.shape[1], metric)
    idx.add(keys, rows)
    res = idx.search_with_options(queries, xb.SearchOptions(top_k=k, refine_scale=refine,
                                                             radius=radius, filter=bitmap),
                                  raise_on_error=False)
    codes, params = oracle.quantize_int8_batch(rows)
    st, ok, os_, oc, ost = oracle.sq8_search(metric, codes, params, rows, keys, queries, k,
                                             radius, refine, bitmap)
    for q in range(queries.shape[0]):
        if ost[q] != 0:
            assert res.counts[q] == -ost[q], (q, res.counts[q], ost[q])
            continue
        c = int(oc[q])
        assert int(res.counts[q]) == c, (metric, q, res.counts[q], c)
        assert np.array_equal(res.keys[q, :c], ok[q, :c]), (metric, q, res.keys[q, :c], ok[q, :c])
        assert np.array_equal(res.scores[q, :c].view(np.uint32), os_[q, :c].view(np.uint32)), \
            (metric, q, res.scores[q, :c], os_[q, :c])
    idx.close()


@pytest.mark.parametrize("metric", [IP, L2, COSINE, MIPSL2])
@pytest.mark.parametrize("d", [4, 17, 128])
def test_sq8_parity(oracle, xb, metric, d):
    rng = np.random.default_rng(500 + d + metric)
    rows = scaled_gaussian(rng, 2500, d)
    keys = rng.permutation(50000)[:2500].astype(np.uint64)
    queries = scaled_gaussian(rng, 37, d)
    run(oracle, xb, metric, rows, keys, queries, 10)
    run(oracle, xb, metric, rows, keys, queries, 10, refine=4.0)


def test_sq8_1024_ip_refine(oracle, xb):
    """The SQ configuration's shape: d = 1024, IP, k = 10, ScaleFactor 4."""
    rng = np.random.default_rng(7)
    rows = scaled_gaussian(rng, 3000, 1024)
    keys = np.arange(3000, dtype=np.uint64) * 7
    queries = scaled_gaussian(rng, 64, 1024)
    run(oracle, xb, IP, rows, keys, queries, 10, refine=4.0)
    run(oracle, xb, IP, rows, keys, queries, 10)


def test_sq8_filter_radius_edge_vectors(oracle, xb):
    rng = np.random.default_rng(8)
    rows = scaled_gaussian(rng, 800, 32)
    rows[3] = 0.0            # zero vector
    rows[5] = 3.5            # constant vector
    rows[7] = rows[9]        # duplicate row
    keys = np.arange(800, dtype=np.uint64)[::-1].copy()
    queries = scaled_gaussian(rng, 20, 32)
    queries[0] = 0.0
    bitmap = np.zeros(25, np.uint32)
    for p in range(0, 800, 2):
        bitmap[p >> 5] |= np.uint32(1 << (p & 31))
    for metric in (IP, L2):
        run(oracle, xb, metric, rows, keys, queries, 15, bitmap=bitmap)
        run(oracle, xb, metric, rows, keys, queries, 15, refine=2.5, bitmap=bitmap)
    run(oracle, xb, L2, rows, keys, queries, 40, radius=50.0)
    run(oracle, xb, L2, rows, keys, queries, 10, radius=50.0, refine=3.0)
    run(oracle, xb, IP, rows, keys, queries, 40, radius=2.0)


@pytest.mark.parametrize("metric", [IP, L2])
def test_sq8_tensor_core_seeded(oracle, xb, metric):
    """70,000 rows: the INT8 tensor-core scan in seeding launches plus the rest."""
    rng = np.random.default_rng(70 + metric)
    rows = scaled_gaussian(rng, 70_000, 128)
    rows[4300:4400] = rows[100:200]          # duplicates across the first launches
    keys = rng.permutation(1 << 22)[:70_000].astype(np.uint64)
    queries = scaled_gaussian(rng, 200, 128)
    before = xb.stats()["tensor_scans"]
    run(oracle, xb, metric, rows, keys, queries, 10)
    assert xb.stats()["tensor_scans"] > before, "tensor-core path not taken"
    run(oracle, xb, metric, rows, keys, queries, 10, refine=4.0)
