"""Sample seeding of the tensor-core Flat scan's shared thresholds.

Before the scan's first launch, each query's shared threshold is lowered to
a bound taken from the FP32 fast ranks of rows evenly spaced over the base
(flat_kernels.cu: sample_rank_kernel, sample_seed_select_kernel): the kp-th
best sample rank plus the sample's and the scan's error bounds.  The bound
must never fall below the query's kp-th best scan key over the rows the
search may return, or rows of its top-k would be dropped.  These cases aim
at that: filters that leave out every sampled row, keep only the sampled
rows, or keep too few of them to seed; every metric on FP32 and FP16 rows;
zero rows under cosine; a base of one repeated row.  Every base has more
than 2^16 rows, so the scan runs a seeding launch and the sample seeding
runs before it.  Keys identical and scores bit-identical to the oracle
(topk.go:105-166, the filter before scoring at topk.go:134-136)."""
import numpy as np
import pytest

from oracle.oracle import COSINE, IP, L2, MIPSL2

pytestmark = pytest.mark.gpu

N, D = 200_000, 64


@pytest.fixture(scope="module")
def xb():
    import xvec_b200
    assert xvec_b200.device_count() >= 1
    return xvec_b200


def data(seed, nq, normalise=False):
    rng = np.random.default_rng(seed)
    centers = rng.standard_normal((100, D)).astype(np.float32)
    rows = centers[rng.integers(0, 100, N)] + 0.3 * rng.standard_normal((N, D), dtype=np.float32)
    queries = centers[rng.integers(0, 100, nq)] + 0.3 * rng.standard_normal((nq, D), dtype=np.float32)
    if normalise:
        rows /= np.linalg.norm(rows, axis=1, keepdims=True)
        queries /= np.linalg.norm(queries, axis=1, keepdims=True)
    keys = (rng.permutation(N).astype(np.uint64) * np.uint64(0x9E3779B1)) & np.uint64((1 << 40) - 1)
    return rows, keys, queries


def bitmap_of(mask):
    words = np.zeros((len(mask) + 31) // 32, np.uint32)
    pos = np.nonzero(mask)[0]
    np.bitwise_or.at(words, pos >> 5, (np.uint32(1) << (pos & 31).astype(np.uint32)))
    return words


def sampled_positions(n):
    """Every position the seeding may sample (sample sizes 1,024 and 2,048)."""
    out = set()
    for s in (1024, 2048):
        out.update((np.arange(s, dtype=np.int64) * n // s).tolist())
    return np.array(sorted(out))


def run(xb, oracle, metric, rows, keys, queries, k, storage=None, bitmap=None):
    fp16 = storage is not None and storage == xb.STORAGE_FP16
    idx = xb.DenseFlatIndex(D, metric, storage or xb.STORAGE_FP32)
    if fp16:
        rows = rows.astype(np.float16)
        queries = queries.astype(np.float16)
        idx.add(keys, rows.view(np.uint16))
        qin = queries.view(np.uint16)
    else:
        idx.add(keys, rows)
        qin = queries
    xb.reset_stats()
    res = idx.search_with_options(qin, xb.SearchOptions(top_k=k, filter=bitmap))
    st = xb.stats()
    idx.close()
    assert st["tensor_scans"] == 1
    ost, ok, os_, oc, _ = oracle.flat_search(metric, rows.astype(np.float32), keys,
                                              queries.astype(np.float32), k, bitmap=bitmap)
    assert ost == 0
    for q in range(len(queries)):
        c = int(oc[q])
        assert int(res.counts[q]) == c, q
        assert np.array_equal(res.keys[q, :c], ok[q, :c]), q
        assert np.array_equal(res.scores[q, :c].view(np.uint32), os_[q, :c].view(np.uint32)), q
    return res, st


@pytest.mark.parametrize("metric", [L2, IP, COSINE, MIPSL2])
@pytest.mark.parametrize("fp16", [False, True])
def test_seed_metrics(oracle, xb, metric, fp16):
    rows, keys, queries = data(100 + metric, 300, normalise=metric == COSINE)
    run(xb, oracle, metric, rows, keys, queries, 10,
        xb.STORAGE_FP16 if fp16 else xb.STORAGE_FP32)


@pytest.mark.parametrize("nq", [96, 300])
def test_seed_filter_leaves_out_every_sampled_row(oracle, xb, nq):
    rows, keys, queries = data(7, nq)
    mask = np.ones(N, bool)
    mask[sampled_positions(N)] = False
    run(xb, oracle, L2, rows, keys, queries, 10, bitmap=bitmap_of(mask))


def test_seed_filter_keeps_only_sampled_rows(oracle, xb):
    # The sampled rows' own ranks then bound the kp-th best of all eligible
    # rows exactly (up to the error bounds).
    rows, keys, queries = data(8, 300)
    mask = np.zeros(N, bool)
    mask[(np.arange(1024, dtype=np.int64) * N // 1024)] = True
    run(xb, oracle, L2, rows, keys, queries, 10, bitmap=bitmap_of(mask))


@pytest.mark.parametrize("keep", [0.01, 0.2])
def test_seed_sparse_filter(oracle, xb, keep):
    # 1 %: about 10 sampled rows pass, fewer than kp, so no query is seeded;
    # 20 %: about 200 pass and every query is seeded from them.
    rows, keys, queries = data(9, 300)
    rng = np.random.default_rng(90)
    run(xb, oracle, IP, rows, keys, queries, 10, bitmap=bitmap_of(rng.random(N) < keep))


def test_seed_zero_rows_cosine(oracle, xb):
    rows, keys, queries = data(10, 300, normalise=True)
    rows[np.random.default_rng(11).random(N) < 0.1] = 0.0
    run(xb, oracle, COSINE, rows, keys, queries, 10)


def test_seed_repeated_row(oracle, xb):
    # Every rank ties: the seeded bound sits at the one rank plus the error
    # bounds, and every row stays a candidate until the coverage check.
    rows, keys, queries = data(12, 200)
    rows[:] = rows[0]
    run(xb, oracle, L2, rows, keys, queries, 10)
