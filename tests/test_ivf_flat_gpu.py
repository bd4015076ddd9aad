"""IVF with exact scoring of the probed lists (core.IVFIndex, ivf.go:427-597)
against the oracle's restatement: identical keys and bit-identical float32
scores, cosine with the cached magnitudes (probe and scan)."""
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


def run(oracle, xb, metric, rows, keys, queries, centroids, k, nprobe, radius=0.0, bitmap=None,
        expect_exact=None):
    d = rows.shape[1]
    idx = xb.IVFIndex(d, metric)
    idx.set_model(centroids)
    idx.add(keys, rows)
    st0 = xb.stats()
    res = idx.search_with_options(queries, xb.SearchOptions(top_k=k, nprobe=nprobe, radius=radius,
                                                             filter=bitmap),
                                  raise_on_error=False)
    st1 = xb.stats()
    st, labels, _ = oracle.kmeans_assign(metric, rows, centroids)
    assert st == 0
    nlist = centroids.shape[0]
    offsets = np.zeros(nlist + 1, np.int64)
    np.add.at(offsets, labels + 1, 1)
    offsets = np.cumsum(offsets)
    positions = np.argsort(labels, kind="stable").astype(np.int64)
    _, ok, os_, oc, ost = oracle.ivf_flat_search(metric, rows, keys, centroids, offsets, positions,
                                                 queries, k, nprobe, radius, bitmap)
    for q in range(queries.shape[0]):
        if ost[q] != 0:
            assert res.counts[q] < 0, q
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
def test_ivf_flat_parity(oracle, xb, metric, d):
    rng = np.random.default_rng(500 + d + metric)
    rows = mixture(rng, 6000, d)
    keys = rng.permutation(1 << 20)[:6000].astype(np.uint64)
    queries = mixture(rng, 41, d)
    centroids = rows[rng.choice(6000, 32, replace=False)].copy()
    run(oracle, xb, metric, rows, keys, queries, centroids, 10, 4, expect_exact=False)
    run(oracle, xb, metric, rows, keys, queries, centroids, 64, 40)  # more probes than lists


def test_ivf_flat_filter_radius(oracle, xb):
    rng = np.random.default_rng(17)
    rows = mixture(rng, 5000, 64)
    keys = np.arange(5000, dtype=np.uint64) * 7 + 3
    queries = mixture(rng, 23, 64)
    centroids = rows[:24].copy()
    bitmap = np.zeros((5000 + 31) // 32, np.uint32)
    for p in range(5000):
        if p % 5:
            bitmap[p >> 5] |= np.uint32(1 << (p & 31))
    for metric in (L2, IP, COSINE):
        run(oracle, xb, metric, rows, keys, queries, centroids, 20, 6, bitmap=bitmap)
    run(oracle, xb, L2, rows, keys, queries, centroids, 50, 8, radius=8.0)
    run(oracle, xb, IP, rows, keys, queries, centroids, 50, 8, radius=5.0)


def test_ivf_flat_cosine_zero_vectors_and_ties(oracle, xb):
    rng = np.random.default_rng(23)
    rows = mixture(rng, 6000, 48)
    rows[10:20] = 0.0                              # zero rows: distance 1 (or 0 for a zero query)
    rows[2000:4800] = rows[33]                     # 2800 equal rows: more than the warps' lists
    keys = rng.permutation(1 << 20)[:6000].astype(np.uint64)
    queries = mixture(rng, 9, 48)
    queries[0] = 0.0
    queries[1] = rows[33]
    centroids = rows[rng.choice(6000, 12, replace=False)].copy()
    centroids[3] = 0.0                             # a zero centroid (magnitude 0)
    run(oracle, xb, COSINE, rows, keys, queries, centroids, 30, 12)
    run(oracle, xb, L2, rows, keys, queries, centroids, 30, 12, expect_exact=True)
