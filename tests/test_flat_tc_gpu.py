"""Tensor-core (tcgen05) scan for Flat search: parity with the oracle.

FP16 storage and FP32 storage (bfloat16 high/low parts, three MMAs per
k-step) rank candidates with tcgen05.mma and rescore them in the reference
order, so scores must be bit-identical and key lists identical."""
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


@pytest.mark.parametrize("d", [64, 72, 128, 200, 512, 520, 960])
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


def run32(oracle, xb, metric, rows, queries, keys, k, bitmap=None, radius=0.0, exact_ok=False):
    """FP32 storage: the tensor-core scan on bfloat16 high/low parts."""
    idx = xb.DenseFlatIndex(rows.shape[1], metric, xb.STORAGE_FP32)
    idx.add(keys, rows)
    st0 = xb.stats()
    res = idx.search_with_options(queries, xb.SearchOptions(top_k=k, filter=bitmap, radius=radius))
    st1 = xb.stats()
    assert st1["tensor_scans"] == st0["tensor_scans"] + 1, "tensor-core path not taken"
    if not exact_ok:
        assert st1["exact_queries"] == st0["exact_queries"], "fast pass did not settle"
    st, ok, os_, oc, _ = oracle.flat_search(metric, rows, keys, queries, k, radius, bitmap)
    assert st == 0
    assert np.array_equal(res.counts, oc)
    for q in range(queries.shape[0]):
        c = int(oc[q])
        assert np.array_equal(res.keys[q, :c], ok[q, :c]), q
        assert np.array_equal(res.scores[q, :c].view(np.uint32), os_[q, :c].view(np.uint32)), q
    idx.close()


@pytest.mark.parametrize("metric", [L2, IP, COSINE, MIPSL2])
def test_tc_fp32_split(oracle, xb, metric):
    """FP32 rows: 70,000 x 128 (a seeding launch plus the rest, CTA pairs),
    k = 1 (nearest-centroid assignment) and k = 64 (an IVF probe), and a
    filter."""
    rng = np.random.default_rng(300 + metric)
    n = 70_000
    rows = mixture(rng, n, 128, normalise=False)
    rows[5000:5050] = rows[10:60]            # duplicates across the prefix boundary
    keys = rng.permutation(1 << 22)[:n].astype(np.uint64)
    queries = mixture(rng, 300, 128, normalise=False)
    queries[:3] = rows[[10, 5000, 69999]]
    run32(oracle, xb, metric, rows, queries, keys, 1)
    run32(oracle, xb, metric, rows, queries, keys, 64)
    bitmap = np.zeros((n + 31) // 32, np.uint32)
    for p in range(n):
        if (p * 11) % 5 != 0:
            bitmap[p >> 5] |= np.uint32(1 << (p & 31))
    run32(oracle, xb, metric, rows, queries[:100], keys, 10, bitmap=bitmap)


@pytest.mark.parametrize("scale", [1e-18, 1e15])
def test_tc_fp32_split_magnitudes(oracle, xb, scale):
    """bfloat16 keeps float32's exponent range: tiny and huge rows need no
    scaling; the bound is relative to the norms."""
    rng = np.random.default_rng(int(-np.log10(scale)) + 40)
    rows = (mixture(rng, 5000, 64, normalise=False) * scale).astype(np.float32)
    keys = np.arange(5000, dtype=np.uint64)
    queries = (mixture(rng, 150, 64, normalise=False) * scale).astype(np.float32)
    for metric in (L2, IP, COSINE):
        run32(oracle, xb, metric, rows, queries, keys, 10, exact_ok=True)
