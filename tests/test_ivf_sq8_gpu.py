"""IVF with INT8 scalar-quantized scoring (core.ScalarQuantizedIVFIndex,
ivf_quantized.go:135-192) against the oracle's restatement: the IVF probe
with the original metric, the SQ8 score of every probed position, the refine
stage when a refine scale is given.  Identical keys and bit-identical float32
scores."""
import numpy as np
import pytest

from oracle.oracle import COSINE, IP, L2, MIPSL2

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def xb():
    import xvec_b200
    assert xvec_b200.device_count() >= 1
    return xvec_b200


def mixture(rng, n, d, clusters=20, sigma=0.3):
    c = rng.standard_normal((clusters, d)).astype(np.float32)
    return (c[rng.integers(0, clusters, n)] + sigma * rng.standard_normal((n, d))).astype(np.float32)


def run(oracle, xb, metric, rows, keys, queries, centroids, k, nprobe, radius=0.0, scale=0.0,
        bitmap=None, expect_exact=None):
    d = rows.shape[1]
    idx = xb.ScalarQuantizedIVFIndex(d, metric)
    idx.set_model(centroids)
    idx.add(keys, rows)
    st0 = xb.stats()
    res = idx.search_with_options(queries, xb.SearchOptions(top_k=k, nprobe=nprobe, radius=radius,
                                                             refine_scale=scale, filter=bitmap),
                                  raise_on_error=False)
    st1 = xb.stats()
    st, labels, _ = oracle.kmeans_assign(metric, rows, centroids)
    assert st == 0
    nlist = centroids.shape[0]
    offsets = np.zeros(nlist + 1, np.int64)
    np.add.at(offsets, labels + 1, 1)
    offsets = np.cumsum(offsets)
    positions = np.argsort(labels, kind="stable").astype(np.int64)
    codes, params = oracle.quantize_int8_batch(rows)
    _, ok, os_, oc, ost = oracle.ivf_sq8_search(metric, codes, params, rows, keys, centroids,
                                                offsets, positions, queries, k, nprobe, radius,
                                                scale, bitmap)
    for q in range(queries.shape[0]):
        if ost[q] != 0:
            assert res.counts[q] == -int(ost[q]), (q, res.counts[q], ost[q])
            continue
        c = int(oc[q])
        assert int(res.counts[q]) == c, (metric, q, res.counts[q], c)
        assert np.array_equal(res.keys[q, :c], ok[q, :c]), (metric, q)
        assert np.array_equal(res.scores[q, :c].view(np.uint32), os_[q, :c].view(np.uint32)), \
            (metric, q, res.scores[q, :c], os_[q, :c])
    if expect_exact is not None:
        exact = st1["exact_queries"] - st0["exact_queries"]
        assert (exact > 0) == expect_exact, exact
    idx.close()


@pytest.mark.parametrize("metric", [L2, IP, COSINE, MIPSL2])
@pytest.mark.parametrize("d", [32, 100, 128])
def test_ivf_sq8_parity(oracle, xb, metric, d):
    rng = np.random.default_rng(700 + d + metric)
    rows = mixture(rng, 6000, d)
    keys = rng.permutation(1 << 20)[:6000].astype(np.uint64)
    queries = mixture(rng, 41, d)
    centroids = rows[rng.choice(6000, 32, replace=False)].copy()
    ranked = metric in (L2, IP)
    run(oracle, xb, metric, rows, keys, queries, centroids, 10, 4,
        expect_exact=False if ranked else None)
    run(oracle, xb, metric, rows, keys, queries, centroids, 64, 40)  # more probes than lists


@pytest.mark.parametrize("metric", [L2, IP, COSINE])
def test_ivf_sq8_refine(oracle, xb, metric):
    rng = np.random.default_rng(31 + metric)
    rows = mixture(rng, 5000, 64)
    keys = rng.permutation(1 << 20)[:5000].astype(np.uint64)
    queries = mixture(rng, 29, 64)
    centroids = rows[rng.choice(5000, 20, replace=False)].copy()
    run(oracle, xb, metric, rows, keys, queries, centroids, 10, 5, scale=4.0)
    run(oracle, xb, metric, rows, keys, queries, centroids, 10, 5, scale=1.0)
    radius = 30.0 if metric == L2 else (2.0 if metric == IP else 0.5)
    run(oracle, xb, metric, rows, keys, queries, centroids, 10, 5, radius=radius, scale=2.5)


def test_ivf_sq8_filter_radius_and_invalid_queries(oracle, xb):
    rng = np.random.default_rng(19)
    rows = mixture(rng, 5000, 48)
    keys = np.arange(5000, dtype=np.uint64) * 5 + 1
    queries = mixture(rng, 23, 48)
    queries[4, 7] = np.nan                         # rejected by the query validation
    queries[9] = 0.0                               # a zero query
    centroids = rows[:24].copy()
    bitmap = np.zeros((5000 + 31) // 32, np.uint32)
    for p in range(5000):
        if p % 3:
            bitmap[p >> 5] |= np.uint32(1 << (p & 31))
    for metric in (L2, IP, COSINE):
        run(oracle, xb, metric, rows, keys, queries, centroids, 20, 6, bitmap=bitmap)
    run(oracle, xb, L2, rows, keys, queries, centroids, 50, 8, radius=8.0)
    run(oracle, xb, IP, rows, keys, queries, centroids, 50, 8, radius=5.0)


def test_ivf_sq8_ties_and_zero_rows(oracle, xb):
    rng = np.random.default_rng(29)
    rows = mixture(rng, 6000, 40)
    rows[10:20] = 0.0
    rows[2000:4800] = rows[33]                     # 2800 equal codes: more than the warps' lists
    keys = rng.permutation(1 << 20)[:6000].astype(np.uint64)
    queries = mixture(rng, 9, 40)
    queries[1] = rows[33]
    centroids = rows[rng.choice(6000, 12, replace=False)].copy()
    run(oracle, xb, L2, rows, keys, queries, centroids, 30, 12, expect_exact=True)
    run(oracle, xb, IP, rows, keys, queries, centroids, 30, 12)
    run(oracle, xb, COSINE, rows, keys, queries, centroids, 30, 12)
    run(oracle, xb, L2, rows, keys, queries, centroids, 10, 12, scale=3.0)


def test_ivf_sq8_requires_model_and_nprobe(xb):
    idx = xb.ScalarQuantizedIVFIndex(16, L2)
    with pytest.raises(xb.XvecGPUError):
        idx.add(np.arange(4, dtype=np.uint64), np.ones((4, 16), np.float32))
    idx.set_model(np.eye(4, 16, dtype=np.float32))
    idx.add(np.arange(4, dtype=np.uint64), np.eye(4, 16, dtype=np.float32))
    with pytest.raises(xb.XvecGPUError):
        idx.search_with_options(np.ones((1, 16), np.float32), xb.SearchOptions(top_k=2, nprobe=0))
    res = idx.search_with_options(np.eye(2, 16, dtype=np.float32),
                                  xb.SearchOptions(top_k=2, nprobe=1))
    assert res.keys[0, 0] == 0 and res.keys[1, 0] == 1
    idx.close()


@pytest.mark.parametrize("metric,d", [(L2, 4), (L2, 64), (IP, 32), (COSINE, 24)])
def test_ivf_sq8_full_probe_matches_sq8_flat(xb, metric, d):
    """TestScalarQuantizedIVFFullProbeMatchesQuantizedFlat
    (quantized_index_test.go:173-201), with INT8 codes: probing every list
    with a key filter gives exactly the SQ8 Flat index's result."""
    rng = np.random.default_rng(173 + d)
    n = 320
    rows = rng.standard_normal((n, d)).astype(np.float32)
    keys = np.arange(1, n + 1, dtype=np.uint64) * 3
    centroids = rows[rng.choice(n, 16, replace=False)].copy()
    ivf = xb.ScalarQuantizedIVFIndex(d, metric)
    ivf.set_model(centroids)
    ivf.add(keys, rows)
    flat = xb.ScalarQuantizedFlatIndex(d, metric)
    flat.add(keys, rows)
    bitmap = xb.bitmap_from_predicate(n, keys, lambda k: k % 5 != 0)
    queries = np.concatenate([rows[217:218], rng.standard_normal((7, d)).astype(np.float32)])
    got = ivf.search_with_options(queries, xb.SearchOptions(top_k=31, nprobe=16, filter=bitmap))
    want = flat.search_with_options(queries, xb.SearchOptions(top_k=31, filter=bitmap))
    assert np.array_equal(got.counts, want.counts)
    for q in range(queries.shape[0]):
        c = int(want.counts[q])
        assert np.array_equal(got.keys[q, :c], want.keys[q, :c]), q
        assert np.array_equal(got.scores[q, :c].view(np.uint32), want.scores[q, :c].view(np.uint32))
    ivf.close()
    flat.close()
