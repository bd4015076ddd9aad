"""Product-quantizer training on the GPU (xvec_gpu_pq_train) against the
oracle's TrainPQ restatement (pq.go:107-179: KMC2 seeding with the
pqUniformSampleIndices walk, TrainKMeans from those centroids, padding from
centroid 0): bit-identical pivots and identical chunk offsets."""
import numpy as np
import pytest

from oracle.oracle import COSINE, IP, L2

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def xb():
    import xvec_b200
    assert xvec_b200.device_count() >= 1
    return xvec_b200


def mixture(rng, n, d, clusters=24, sigma=0.5):
    c = rng.standard_normal((clusters, d)).astype(np.float32)
    return (c[rng.integers(0, clusters, n)] + sigma * rng.standard_normal((n, d))).astype(np.float32)


def check(oracle, xb, metric, x, chunks, samples=200_000, iterations=12, seed=0):
    offsets, pivots = xb.pq_train(metric, x, chunks, samples, iterations, seed)
    resolved = chunks or x.shape[1] // 2
    assert np.array_equal(offsets, oracle.pq_chunk_offsets(x.shape[1], resolved))
    st, opivots = oracle.pq_train(metric, x, resolved, samples, iterations, seed)
    assert st == 0
    assert np.array_equal(pivots.view(np.uint32), opivots.view(np.uint32))
    return offsets, pivots


@pytest.mark.parametrize("metric", [L2, IP])
@pytest.mark.parametrize("n,d,chunks", [(5000, 32, 8),     # width 4: scalar sums
                                        (3000, 40, 4),     # width 10: one 8-lane block
                                        (2500, 70, 3),     # widths 24, 23, 23: 16-lane blocks
                                        (6000, 24, 0)])    # chunks 0 -> d / 2
def test_pq_train_matches_oracle(oracle, xb, metric, n, d, chunks):
    rng = np.random.default_rng(n + d + chunks + metric)
    check(oracle, xb, metric, mixture(rng, n, d), chunks, iterations=6, seed=17 + metric)


def test_pq_train_sample_prefix_and_padding(oracle, xb):
    rng = np.random.default_rng(5)
    x = mixture(rng, 12_000, 16)
    # MaxTrainSamples below n: the first rows alone train (three sampling steps).
    check(oracle, xb, L2, x, 4, samples=9_000, iterations=4, seed=3)
    # Fewer rows than centroids: 100 trained rows, the rest repeat centroid 0.
    _, pivots = check(oracle, xb, L2, x[:100], 4, iterations=3, seed=9)
    assert np.array_equal(pivots[100:], np.broadcast_to(pivots[0], pivots[100:].shape))
    # Fewer rows than the chain length.
    check(oracle, xb, IP, x[:20], 8, iterations=2, seed=1)
    check(oracle, xb, L2, x[:1], 2, iterations=2, seed=1)


def test_pq_train_full_sample(oracle, xb):
    """The default 200,000-row sample (49 sampling steps per walk) and 12
    iterations."""
    rng = np.random.default_rng(200)
    x = mixture(rng, 230_000, 32, clusters=64)
    check(oracle, xb, L2, x, 8, seed=42)


def test_pq_train_duplicates(oracle, xb):
    """Zero scores in the chain (duplicate rows) take candidates without a
    draw."""
    rng = np.random.default_rng(8)
    base = mixture(rng, 40, 12)
    x = base[rng.integers(0, 40, 3000)]
    check(oracle, xb, L2, x, 3, iterations=5, seed=77)
    check(oracle, xb, IP, x, 3, iterations=5, seed=78)


def test_pq_train_errors(xb):
    x = np.ones((50, 8), np.float32)
    for kwargs in ({"metric": COSINE}, {"chunks": 9}, {"chunks": -1},
                   {"max_train_samples": 0}, {"max_iterations": 0}):
        args = {"metric": L2, "chunks": 2, "max_train_samples": 100, "max_iterations": 2}
        args.update(kwargs)
        with pytest.raises(xb.XvecGPUError) as e:
            xb.pq_train(args["metric"], x, args["chunks"], args["max_train_samples"],
                        args["max_iterations"])
        assert e.value.status == xb.INVALID_ARGUMENT
    bad = x.copy()
    bad[49, 3] = np.inf          # past the training sample: still validated
    with pytest.raises(xb.XvecGPUError) as e:
        xb.pq_train(L2, bad, 2, 10, 2)
    assert e.value.status == xb.NON_FINITE
    with pytest.raises(xb.XvecGPUError):
        xb.pq_train(L2, np.zeros((0, 8), np.float32), 2)


def test_trained_pivots_drive_ivfpq(oracle, xb):
    """Pivots from the GPU trainer set an IVF-PQ model whose search equals
    the oracle's IVF-PQ over those pivots."""
    from test_ivfpq_gpu import run
    rng = np.random.default_rng(31)
    d = 32
    x = mixture(rng, 6000, d)
    _, pivots = check(oracle, xb, L2, x, 8, iterations=4, seed=5)
    cents = x[rng.choice(6000, 16, replace=False)].copy()
    keys = rng.permutation(1 << 20)[:6000].astype(np.uint64)
    run(oracle, xb, L2, x, keys, mixture(rng, 9, d), cents, pivots, 8, 10, 4)
