"""IVF-PQ list scan and k-means assignment: CUDA path against the oracle.

The scan ranks codes by a float32 look-up sum and rescores its candidates
with the reference's float64 sums, so keys and float32 scores must be
identical."""
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
    return c[rng.integers(0, clusters, n)] + sigma * rng.standard_normal((n, d)).astype(np.float32)


def build_oracle_lists(oracle, metric, rows, centroids):
    st, labels, _ = oracle.kmeans_assign(metric, rows, centroids)
    assert st == 0
    nlist = centroids.shape[0]
    offsets = np.zeros(nlist + 1, np.int64)
    np.add.at(offsets, labels + 1, 1)
    offsets = np.cumsum(offsets)
    positions = np.argsort(labels, kind="stable").astype(np.int64)
    return offsets, positions


def run(oracle, xb, metric, rows, keys, queries, centroids, pivots, chunks, k, nprobe,
        radius=0.0, bitmap=None):
    d = rows.shape[1]
    idx = xb.IVFPQIndex(d, metric)
    idx.set_model(centroids, pivots, chunks)
    idx.add(keys, rows)
    res = idx.search_with_options(queries, xb.SearchOptions(top_k=k, nprobe=nprobe, radius=radius,
                                                             filter=bitmap))
    offsets = oracle.pq_chunk_offsets(d, chunks)
    codes = np.stack([oracle.pq_encode(metric, pivots, offsets, r)[1] for r in rows])
    lo, lp = build_oracle_lists(oracle, metric, rows, centroids)
    st, ok, os_, oc, _ = oracle.ivfpq_search(metric, centroids, pivots, offsets, codes, keys, lo,
                                             lp, queries, k, nprobe, radius, bitmap)
    assert st == 0
    assert np.array_equal(res.counts, oc)
    for q in range(queries.shape[0]):
        c = int(oc[q])
        assert np.array_equal(res.keys[q, :c], ok[q, :c]), q
        assert np.array_equal(res.scores[q, :c].view(np.uint32), os_[q, :c].view(np.uint32)), q
    idx.close()


@pytest.mark.parametrize("metric", [L2, IP])
@pytest.mark.parametrize("d,chunks", [(32, 8), (128, 32), (20, 6)])
def test_ivfpq_parity(oracle, xb, metric, d, chunks):
    rng = np.random.default_rng(900 + d + metric)
    rows = mixture(rng, 4000, d)
    keys = rng.permutation(1 << 20)[:4000].astype(np.uint64)
    queries = mixture(rng, 33, d)
    centroids = rows[rng.choice(4000, 24, replace=False)].copy()
    pivots = rows[rng.choice(4000, 256, replace=False)].copy()
    run(oracle, xb, metric, rows, keys, queries, centroids, pivots, chunks, 10, 5)
    run(oracle, xb, metric, rows, keys, queries, centroids, pivots, chunks, 50, 24)


def test_ivfpq_filter_radius_and_more_probes_than_lists(oracle, xb):
    rng = np.random.default_rng(31)
    rows = mixture(rng, 3000, 64)
    keys = np.arange(3000, dtype=np.uint64)
    queries = mixture(rng, 17, 64)
    centroids = rows[:10].copy()
    pivots = rows[100:356].copy()
    bitmap = np.zeros((3000 + 31) // 32, np.uint32)
    for p in range(3000):
        if p % 3:
            bitmap[p >> 5] |= np.uint32(1 << (p & 31))
    run(oracle, xb, L2, rows, keys, queries, centroids, pivots, 16, 20, 4, bitmap=bitmap)
    run(oracle, xb, L2, rows, keys, queries, centroids, pivots, 16, 20, 99, radius=9.0)


@pytest.mark.parametrize("metric", [L2, IP])
@pytest.mark.parametrize("chunks", [64, 128])
def test_ivfpq_wide_chunks(oracle, xb, metric, chunks):
    """64 chunks: the fast scan with two chunk groups per lane; 128 chunks:
    the exact scan alone."""
    rng = np.random.default_rng(70 + chunks + metric)
    rows = mixture(rng, 3000, 128)
    keys = rng.permutation(1 << 20)[:3000].astype(np.uint64)
    queries = mixture(rng, 21, 128)
    centroids = rows[rng.choice(3000, 12, replace=False)].copy()
    pivots = rows[rng.choice(3000, 256, replace=False)].copy()
    xb.reset_stats()
    run(oracle, xb, metric, rows, keys, queries, centroids, pivots, chunks, 10, 4)
    exact = xb.stats()["exact_queries"]
    assert exact == (0 if chunks == 64 else 21), exact


def test_ivfpq_fast_scan_falls_back_on_ties(oracle, xb):
    """700 copies of one row: more equal fast ranks than a warp's list
    keeps, so the fast pass cannot prove its candidates complete and those
    queries take the exact scan; results stay the reference's."""
    rng = np.random.default_rng(5)
    rows = mixture(rng, 4000, 32)
    rows[1000:1700] = rows[17]
    keys = rng.permutation(1 << 20)[:4000].astype(np.uint64)
    queries = np.concatenate([rows[17:18] + 0.01, mixture(rng, 9, 32)]).astype(np.float32)
    centroids = rows[rng.choice(4000, 8, replace=False)].copy()
    pivots = rows[rng.choice(4000, 256, replace=False)].copy()
    xb.reset_stats()
    run(oracle, xb, L2, rows, keys, queries, centroids, pivots, 8, 10, 8)
    assert xb.stats()["exact_queries"] >= 1


@pytest.mark.parametrize("metric", [L2, IP, COSINE, MIPSL2])
def test_kmeans_assign_parity(oracle, xb, metric):
    rng = np.random.default_rng(40 + metric)
    vectors = mixture(rng, 5000, 48)
    centroids = vectors[rng.choice(5000, 37, replace=False)].copy()
    centroids[5] = centroids[6]  # identical centroids: the lower index wins
    labels, scores = xb.kmeans_assign(metric, vectors, centroids)
    st, ol, os_ = oracle.kmeans_assign(metric, vectors, centroids)
    assert st == 0
    assert np.array_equal(labels, ol)
    assert np.array_equal(scores.view(np.uint32), os_.view(np.uint32))
