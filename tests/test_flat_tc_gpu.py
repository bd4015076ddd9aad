"""Tensor-core (tcgen05) scan for FP16 Flat search: parity with the oracle.

The FP16 path ranks candidates with tcgen05.mma and rescores them in the
reference order, so scores must be bit-identical and key lists identical."""
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


def run(oracle, xb, metric, rows, queries, keys, k, bitmap=None, radius=0.0):
    r16 = rows.astype(np.float16)
    q16 = queries.astype(np.float16)
    idx = xb.DenseFlatIndex(rows.shape[1], metric, xb.STORAGE_FP16)
    idx.add(keys, r16.view(np.uint16))
    before = xb.stats()["tensor_scans"]
    res = idx.search_with_options(q16.view(np.uint16),
                                  xb.SearchOptions(top_k=k, filter=bitmap, radius=radius))
    assert xb.stats()["tensor_scans"] == before + 1, "tensor-core path not taken"
    st, ok, os_, oc, _ = oracle.flat_search(metric, r16.astype(np.float32), keys,
                                            q16.astype(np.float32), k, radius, bitmap)
    assert st == 0
    assert np.array_equal(res.counts, oc)
    for q in range(queries.shape[0]):
        c = int(oc[q])
        assert np.array_equal(res.keys[q, :c], ok[q, :c]), q
        assert np.array_equal(res.scores[q, :c].view(np.uint32), os_[q, :c].view(np.uint32)), q
    idx.close()


@pytest.mark.parametrize("metric", [COSINE, IP, L2, MIPSL2])
def test_tc_768_many_query_blocks(oracle, xb, metric):
    rng = np.random.default_rng(300 + metric)
    rows = mixture(rng, 9000, 768, normalise=metric == COSINE)
    queries = mixture(rng, 300, 768, normalise=metric == COSINE)
    keys = rng.permutation(100000)[:9000].astype(np.uint64)
    run(oracle, xb, metric, rows, queries, keys, 100)


@pytest.mark.parametrize("d", [64, 72, 128, 200, 960])
def test_tc_dims_and_ragged_rows(oracle, xb, d):
    rng = np.random.default_rng(d)
    rows = mixture(rng, 4097, d)
    queries = mixture(rng, 131, d)
    keys = np.arange(4097, dtype=np.uint64)[::-1].copy()
    run(oracle, xb, COSINE, rows, queries, keys, 10)


@pytest.mark.parametrize("metric", [COSINE, L2])
def test_tc_seeded_threshold(oracle, xb, metric):
    """Bases of 64k rows and more are scanned in two launches: a prefix whose
    lists seed every query's shared threshold, then the rest.  A filter whose
    words straddle the split and duplicate rows on both sides of it."""
    rng = np.random.default_rng(70 + metric)
    n = 70_000
    rows = mixture(rng, n, 128, normalise=metric == COSINE)
    rows[4300:4400] = rows[100:200]           # duplicates across the prefix boundary
    keys = rng.permutation(1 << 22)[:n].astype(np.uint64)
    queries = mixture(rng, 260, 128, normalise=metric == COSINE)
    queries[:5] = rows[[3, 4200, 4400, 50000, 69999]]
    run(oracle, xb, metric, rows, queries, keys, 100)
    bitmap = np.zeros((n + 31) // 32, np.uint32)
    for p in range(n):
        if (p * 13) % 7 != 0:
            bitmap[p >> 5] |= np.uint32(1 << (p & 31))
    run(oracle, xb, metric, rows, queries, keys, 20, bitmap=bitmap)


def test_tc_filter_radius_duplicates(oracle, xb):
    rng = np.random.default_rng(9)
    base = mixture(rng, 1500, 128)
    rows = np.concatenate([base, base, base])
    keys = rng.permutation(1 << 20)[:4500].astype(np.uint64)
    queries = mixture(rng, 70, 128)
    bitmap = np.zeros((4500 + 31) // 32, np.uint32)
    for p in range(4500):
        if (p * 7) % 5 != 0:
            bitmap[p >> 5] |= np.uint32(1 << (p & 31))
    run(oracle, xb, COSINE, rows, queries, keys, 50, bitmap=bitmap)
    run(oracle, xb, COSINE, rows, queries, keys, 50, radius=0.05)
    run(oracle, xb, L2, rows, queries, keys, 64)


def test_tc_large_scale_property(xb):
    """Size-independent checks at a larger size: the top-1 of a query that is
    itself a stored row is that row (cosine distance 0), lists are sorted by
    (score, key), and every batch finishes without exact fallbacks."""
    import torch
    n, d, nq, k = 400_000, 768, 2048, 100
    g = torch.Generator(device="cuda").manual_seed(5)
    rows = torch.randn(n, d, device="cuda", generator=g)
    rows = (rows / rows.norm(dim=1, keepdim=True)).half()
    keys = torch.arange(n, device="cuda", dtype=torch.int64) * 3
    idx = xb.DenseFlatIndex(d, COSINE, xb.STORAGE_FP16)
    idx.add_device(keys.data_ptr(), rows.data_ptr(), n)
    pick = torch.randint(0, n, (nq,), device="cuda", generator=g)
    q = rows[pick].contiguous()
    ok = torch.empty(nq * k, dtype=torch.int64, device="cuda")
    os_ = torch.empty(nq * k, dtype=torch.float32, device="cuda")
    oc = torch.empty(nq, dtype=torch.int32, device="cuda")
    xb.reset_stats()
    idx.search_device(q.data_ptr(), nq, xb.SearchOptions(top_k=k), ok.data_ptr(), os_.data_ptr(),
                      oc.data_ptr())
    torch.cuda.synchronize()
    assert xb.stats()["exact_queries"] == 0
    assert (oc == k).all()
    ok, os_ = ok.view(nq, k), os_.view(nq, k)
    assert torch.equal(ok[:, 0], pick * 3)
    assert (os_[:, 0] <= 1e-6).all()
    assert (os_[:, 1:] >= os_[:, :-1]).all()
