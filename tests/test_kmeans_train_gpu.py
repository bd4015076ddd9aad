"""k-means training on the GPU (xvec_gpu_kmeans_train) against the oracle's
TrainKMeans restatement with the IVF builder's options (reservoir seeding,
float64 input-order Lloyd sums, empty clusters reseeded with the
worst-assigned vectors, float64 objective): bit-identical centroids and
identical labels."""
import numpy as np
import pytest

from oracle.oracle import COSINE, IP, L2, MIPSL2

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def xb():
    import xvec_b200
    assert xvec_b200.device_count() >= 1
    return xvec_b200


def mixture(rng, n, d, clusters=15, sigma=0.4):
    c = rng.standard_normal((clusters, d)).astype(np.float32)
    return (c[rng.integers(0, clusters, n)] + sigma * rng.standard_normal((n, d))).astype(np.float32)


@pytest.mark.parametrize("metric", [L2, IP, COSINE, MIPSL2])
@pytest.mark.parametrize("n,d,clusters", [(5000, 32, 24), (3000, 128, 64)])
def test_train_matches_oracle(oracle, xb, metric, n, d, clusters):
    rng = np.random.default_rng(n + d + metric)
    x = mixture(rng, n, d)
    cents, labels, iters, conv, cost = xb.kmeans_train(metric, x, clusters, iterations=10, seed=7)
    st, ocents, olabels = oracle.kmeans_train(metric, x, clusters, iterations=10, seed=7)
    assert st == 0
    assert cents.shape == ocents.shape
    assert np.array_equal(cents.view(np.uint32), ocents.view(np.uint32))
    assert np.array_equal(labels, olabels)
    assert 1 <= iters <= 10


def test_train_reseeds_empty_clusters(oracle, xb):
    """Identical vectors make identical initial centroids: all but the first
    of each group stay empty and are reseeded with the worst-assigned rows."""
    rng = np.random.default_rng(3)
    x = mixture(rng, 2000, 16)
    x[:1200] = x[0]                      # most of the reservoir draws are one point
    cents, labels, iters, conv, cost = xb.kmeans_train(L2, x, 30, iterations=6, seed=11)
    st, ocents, olabels = oracle.kmeans_train(L2, x, 30, iterations=6, seed=11)
    assert st == 0
    assert np.array_equal(cents.view(np.uint32), ocents.view(np.uint32))
    assert np.array_equal(labels, olabels)


def test_train_more_clusters_than_vectors_and_errors(oracle, xb):
    rng = np.random.default_rng(5)
    x = mixture(rng, 40, 8)
    cents, labels, _, _, _ = xb.kmeans_train(L2, x, 64, iterations=3)
    st, ocents, olabels = oracle.kmeans_train(L2, x, 64, iterations=3)
    assert cents.shape[0] == 40 and np.array_equal(cents.view(np.uint32), ocents.view(np.uint32))
    assert np.array_equal(labels, olabels)
    bad = x.copy()
    bad[3, 2] = np.nan
    with pytest.raises(xb.XvecGPUError):
        xb.kmeans_train(L2, bad, 4)
    with pytest.raises(xb.XvecGPUError):
        xb.kmeans_train(L2, x, 0)
    with pytest.raises(xb.XvecGPUError):
        xb.kmeans_train(L2, x, 4, iterations=0)
