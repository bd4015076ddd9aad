"""HNSW-RaBitQ graph search on the GPU (HNSWRaBitQIndex.searchPrepared,
hnsw_rabitq.go:589-737, with refinePrepared :780-801) over an uploaded
graph, against the oracle's restatement of the same walk: the descent
through the upper levels on coarse estimates, the base-layer search with its
frontier, accepted set, lower-bound pruning and (estimate, key) order.  Keys
identical and scores bit-identical, one-bit and multi-bit models, with and
without refinement, a filter and a radius, lists that repeat a neighbour,
Linear (the scan), and a graph made stale by an add."""
import numpy as np
import pytest

from oracle.oracle import COSINE, IP, L2, hnsw_test_graph

pytestmark = pytest.mark.gpu

SCALES = {1: 0.0, 4: 24.0, 7: 190.0}


@pytest.fixture(scope="module")
def xb():
    import xvec_b200
    assert xvec_b200.device_count() >= 1
    return xvec_b200


def build(oracle, xb, metric, total_bits, n=3000, d=100, seed=5, degree=10):
    rng = np.random.default_rng(seed)
    centers = rng.standard_normal((12, d)).astype(np.float32)
    rows = (centers[rng.integers(0, 12, n)] + 0.3 * rng.standard_normal((n, d))).astype(np.float32)
    keys = rng.permutation(1 << 22)[:n].astype(np.uint64)
    cents = rows[rng.choice(n, 6, replace=False)].copy()
    padded = oracle.rabitq_padded_dimension(d)
    signs = rng.integers(0, 256, 4 * padded // 8, dtype=np.uint8)
    idx = xb.RaBitQIndex(d, metric)
    idx.set_model(cents, signs, total_bits, SCALES[total_bits])
    idx.add(keys, rows)
    codes, extra, factors = oracle.rabitq_encode_batch(metric, cents, signs, rows, total_bits,
                                                       SCALES[total_bits])
    graph = hnsw_test_graph(rows, degree=degree, seed=seed)
    idx.set_graph(*graph)
    queries = (centers[rng.integers(0, 12, 37)] + 0.3 * rng.standard_normal((37, d))).astype(np.float32)
    return dict(idx=idx, rows=rows, keys=keys, cents=cents, signs=signs, codes=codes, extra=extra,
                factors=factors, graph=graph, queries=queries, tb=total_bits, metric=metric)


def compare(oracle, xb, c, k, ef, refine=True, radius=0.0, bitmap=None, linear=False):
    res = c["idx"].search_with_options(
        c["queries"], xb.SearchOptions(top_k=k, ef=ef, refine=refine, radius=radius,
                                       filter=bitmap, linear=linear), raise_on_error=False)
    if linear:
        st, ok, os_, oc, ost = oracle.rabitq_search(
            c["metric"], c["cents"], c["signs"], c["codes"], c["factors"], c["rows"], c["keys"],
            c["queries"], k, ef, radius, bitmap, refine=refine, total_bits=c["tb"],
            extra=c["extra"])
    else:
        st, ok, os_, oc, ost = oracle.hnsw_rabitq_search(
            c["metric"], c["cents"], c["signs"], c["codes"], c["factors"], c["rows"], c["keys"],
            c["graph"], c["queries"], k, ef, radius, bitmap, refine=refine, total_bits=c["tb"],
            extra=c["extra"])
    for q in range(c["queries"].shape[0]):
        if ost[q] != 0:
            assert res.counts[q] == -ost[q], (q, res.counts[q], ost[q])
            continue
        n = int(oc[q])
        assert int(res.counts[q]) == n, (q, res.counts[q], n)
        assert np.array_equal(res.keys[q, :n], ok[q, :n]), q
        assert np.array_equal(res.scores[q, :n].view(np.uint32), os_[q, :n].view(np.uint32)), q
    return res


@pytest.mark.parametrize("metric", [L2, IP, COSINE])
@pytest.mark.parametrize("total_bits", [1, 4, 7])
def test_walk_equals_the_oracle(oracle, xb, metric, total_bits):
    c = build(oracle, xb, metric, total_bits, seed=10 + metric + total_bits)
    assert c["graph"][0] >= 1
    xb.reset_stats()
    compare(oracle, xb, c, 10, 60, refine=True)
    compare(oracle, xb, c, 10, 60, refine=False)
    compare(oracle, xb, c, 25, 12, refine=False)   # capacity = top_k > ef
    compare(oracle, xb, c, 5, 300, refine=True)
    c["idx"].close()


def test_walk_filter_radius_linear(oracle, xb):
    c = build(oracle, xb, L2, 1, seed=31)
    n = c["rows"].shape[0]
    bitmap = np.zeros((n + 31) // 32, np.uint32)
    for p in range(n):
        if p % 3:
            bitmap[p >> 5] |= np.uint32(1 << (p & 31))
    compare(oracle, xb, c, 10, 50, refine=True, bitmap=bitmap)
    compare(oracle, xb, c, 10, 50, refine=False, bitmap=bitmap)
    compare(oracle, xb, c, 40, 64, refine=False, radius=40.0)
    compare(oracle, xb, c, 10, 50, refine=True, linear=True)
    c["idx"].close()


def test_walk_frontier_outgrows_the_first_buffer(oracle, xb):
    # A filter that passes one row in a hundred keeps the accepted set from
    # filling, so the frontier holds most visited nodes: more than the first
    # launch's buffer of 1024 entries, fewer than the second's.
    c = build(oracle, xb, L2, 1, seed=41)
    n = c["rows"].shape[0]
    bitmap = np.zeros((n + 31) // 32, np.uint32)
    for p in range(0, n, 100):
        bitmap[p >> 5] |= np.uint32(1 << (p & 31))
    compare(oracle, xb, c, 10, 50, refine=True, bitmap=bitmap)
    compare(oracle, xb, c, 10, 50, refine=False, bitmap=bitmap)
    c["idx"].close()


def test_walk_with_repeated_neighbours(oracle, xb):
    """Lists that name a neighbour twice: the reference takes it at its first
    place (the second finds it visited)."""
    c = build(oracle, xb, IP, 1, seed=41)
    max_level, entry, offsets, nbrs = c["graph"]
    n = c["rows"].shape[0]
    off0 = offsets[: n + 1]
    lists = [nbrs[off0[p]:off0[p + 1]] for p in range(n)]
    lists = [np.concatenate([l, l[:3]]) if p % 2 == 0 else l for p, l in enumerate(lists)]
    new0 = np.zeros(n + 1, np.int64)
    new0[1:] = np.cumsum([l.size for l in lists])
    upper = nbrs[off0[n]:]
    shift = new0[n] - off0[n]
    offsets = np.concatenate([new0, offsets[n + 1:] + shift])
    nbrs = np.concatenate(lists + [upper]).astype(np.int32)
    c["graph"] = (max_level, entry, offsets, nbrs)
    c["idx"].set_graph(*c["graph"])
    compare(oracle, xb, c, 10, 40, refine=True)
    compare(oracle, xb, c, 10, 40, refine=False)
    c["idx"].close()


def test_stale_graph_and_validation(oracle, xb):
    c = build(oracle, xb, L2, 1, seed=51)
    idx = c["idx"]
    rows = c["rows"][:5] + 1.0
    idx.add(np.arange(5, dtype=np.uint64) + (1 << 40), rows)
    with pytest.raises(xb.XvecGPUError):
        idx.search_with_options(c["queries"], xb.SearchOptions(top_k=5, ef=20))
    res = idx.search_with_options(c["queries"], xb.SearchOptions(top_k=5, ef=20, linear=True))
    assert (res.counts == 5).all()
    max_level, entry, offsets, nbrs = c["graph"]
    bad = nbrs.copy()
    bad[0] = 1 << 30
    with pytest.raises(xb.XvecGPUError):
        idx.set_graph(max_level, entry, offsets, bad)
    idx.set_graph(-1, 0, None, None)
    res = idx.search_with_options(c["queries"], xb.SearchOptions(top_k=5, ef=20))
    assert (res.counts == 5).all()
    idx.close()
