"""Streaming Flat scan for one to four queries: parity with the oracle.

The reference answers one query at a time (Collection.Query,
collection.go:3830; topKPrevalidatedCandidatesWithOptions,
internal/core/topk.go:105-166).  For such batches the library streams the
rows once (a sample pass over every 64th row for the starting thresholds,
then every row) and rescores the candidates in the reference order, so keys
are identical and scores bit-identical to the oracle's.  Cases: both
storages and all four metrics, dimensions that are not multiples of the
load width, a filter, a radius, duplicate rows, a query whose best rows tie
beyond a candidate list (the exact scan takes it), and rows ordered so that
one block of the scan sees most of the query's neighbours (its lists fill
and compact)."""
import numpy as np
import pytest

from oracle.oracle import COSINE, IP, L2, MIPSL2

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def xb():
    import xvec_b200
    assert xvec_b200.device_count() >= 1
    return xvec_b200


def mixture(rng, n, d, clusters=50, sigma=0.3, normalise=True):
    centers = rng.standard_normal((clusters, d)).astype(np.float32)
    x = centers[rng.integers(0, clusters, n)] + sigma * rng.standard_normal((n, d)).astype(np.float32)
    if normalise:
        x /= np.linalg.norm(x, axis=1, keepdims=True)
    return x


def check(oracle, xb, metric, rows, queries, keys, k, fp16, bitmap=None, radius=0.0,
          expect_exact=False):
    d = rows.shape[1]
    if fp16:
        rows = rows.astype(np.float16).astype(np.float32)
        queries = queries.astype(np.float16).astype(np.float32)
        idx = xb.DenseFlatIndex(d, metric, xb.STORAGE_FP16)
        idx.add(keys, rows.astype(np.float16).view(np.uint16))
        q_in = queries.astype(np.float16).view(np.uint16)
    else:
        idx = xb.DenseFlatIndex(d, metric)
        idx.add(keys, rows)
        q_in = queries
    st0 = xb.stats()
    res = idx.search_with_options(q_in, xb.SearchOptions(top_k=k, filter=bitmap, radius=radius))
    st1 = xb.stats()
    assert st1["stream_scans"] == st0["stream_scans"] + 1, "streaming path not taken"
    assert st1["tensor_scans"] == st0["tensor_scans"]
    if expect_exact:
        assert st1["exact_queries"] > st0["exact_queries"]
    st, ok, os_, oc, _ = oracle.flat_search(metric, rows, keys, queries, k, radius, bitmap)
    assert st == 0
    assert np.array_equal(res.counts, oc)
    for q in range(queries.shape[0]):
        c = int(oc[q])
        assert np.array_equal(res.keys[q, :c], ok[q, :c]), q
        assert np.array_equal(res.scores[q, :c].view(np.uint32), os_[q, :c].view(np.uint32)), q
    idx.close()
    return st1["exact_queries"] - st0["exact_queries"]


@pytest.mark.parametrize("metric", [COSINE, IP, L2, MIPSL2])
@pytest.mark.parametrize("fp16", [True, False])
@pytest.mark.parametrize("nq", [1, 3, 4])
def test_stream_metrics(oracle, xb, metric, fp16, nq):
    rng = np.random.default_rng(500 + 10 * metric + nq + (100 if fp16 else 0))
    n, d = 60_000, 128
    rows = mixture(rng, n, d, normalise=metric == COSINE)
    queries = mixture(rng, nq, d, normalise=metric == COSINE)
    keys = rng.permutation(1 << 22)[:n].astype(np.uint64)
    exact = check(oracle, xb, metric, rows, queries, keys, 100, fp16)
    assert exact == 0


@pytest.mark.parametrize("fp16,d", [(True, 8), (True, 104), (True, 768), (False, 4),
                                    (False, 100), (False, 960)])
def test_stream_dims(oracle, xb, fp16, d):
    rng = np.random.default_rng(d + (7 if fp16 else 0))
    n = 20_000
    rows = mixture(rng, n, d)
    queries = mixture(rng, 2, d)
    keys = np.arange(n, dtype=np.uint64)[::-1].copy()
    check(oracle, xb, COSINE, rows, queries, keys, 10, fp16)


def test_stream_filter_radius_duplicates(oracle, xb):
    rng = np.random.default_rng(11)
    base = mixture(rng, 8000, 96)
    rows = np.concatenate([base, base, base])
    n = rows.shape[0]
    keys = rng.permutation(1 << 20)[:n].astype(np.uint64)
    queries = mixture(rng, 4, 96)
    queries[1] = rows[100]
    bitmap = np.zeros((n + 31) // 32, np.uint32)
    for p in range(n):
        if (p * 7) % 5 != 0:
            bitmap[p >> 5] |= np.uint32(1 << (p & 31))
    check(oracle, xb, COSINE, rows, queries, keys, 50, True, bitmap=bitmap)
    check(oracle, xb, COSINE, rows, queries, keys, 50, True, radius=0.05)
    check(oracle, xb, L2, rows, queries, keys, 64, False)


def test_stream_ties_take_the_exact_scan(oracle, xb):
    """600 copies of one row at consecutive positions: the query equal to it
    has 100 best rows that tie, more than one block's list holds."""
    rng = np.random.default_rng(12)
    n, d = 50_000, 64
    rows = mixture(rng, n, d, normalise=False)
    rows[20000:20600] = rows[20000]
    keys = rng.permutation(1 << 22)[:n].astype(np.uint64)
    queries = mixture(rng, 3, d, normalise=False)
    queries[2] = rows[20000]
    check(oracle, xb, L2, rows, queries, keys, 100, False, expect_exact=True)


def test_stream_neighbours_in_one_block(oracle, xb):
    """Rows sorted by distance to the query at the front of the base: the
    first block of the scan sees thousands of rows below the sample's bound,
    so its warps' lists fill and compact many times."""
    rng = np.random.default_rng(13)
    n, d = 1_000_000, 128
    rows = mixture(rng, n, d, clusters=20, normalise=False)
    q = rows[rng.integers(0, n)].copy() + 0.01
    order = np.argsort(((rows - q) ** 2).sum(axis=1), kind="stable")
    rows = np.ascontiguousarray(rows[order])
    keys = rng.permutation(1 << 24)[:n].astype(np.uint64)
    queries = np.stack([q, rows[n // 2] + 0.01]).astype(np.float32)
    check(oracle, xb, L2, rows, queries, keys, 100, False)
    check(oracle, xb, IP, rows, queries, keys, 10, True)


def test_stream_large_property(xb):
    """2,000,000 x 768 FP16 rows, one query equal to a stored row: its best
    result is that row at distance 0 and the list is sorted; no exact scan."""
    import torch
    n, d, k = 2_000_000, 768, 100
    g = torch.Generator(device="cuda").manual_seed(8)
    rows = torch.randn(n, d, device="cuda", generator=g)
    rows = (rows / rows.norm(dim=1, keepdim=True)).half()
    keys = torch.arange(n, device="cuda", dtype=torch.int64) * 5 + 1
    idx = xb.DenseFlatIndex(d, COSINE, xb.STORAGE_FP16)
    idx.add_device(keys.data_ptr(), rows.data_ptr(), n)
    pick = 1_234_567
    q = rows[pick:pick + 1].contiguous()
    ok = torch.empty(k, dtype=torch.int64, device="cuda")
    os_ = torch.empty(k, dtype=torch.float32, device="cuda")
    oc = torch.empty(1, dtype=torch.int32, device="cuda")
    xb.reset_stats()
    idx.search_device(q.data_ptr(), 1, xb.SearchOptions(top_k=k), ok.data_ptr(), os_.data_ptr(),
                      oc.data_ptr())
    torch.cuda.synchronize()
    st = xb.stats()
    assert st["stream_scans"] == 1 and st["exact_queries"] == 0
    assert int(oc.item()) == k
    assert int(ok[0].item()) == pick * 5 + 1
    assert float(os_[0].item()) <= 1e-6
    assert bool((os_[1:] >= os_[:-1]).all())
    idx.close()
