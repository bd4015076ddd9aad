"""The oracle's HNSW-RaBitQ graph search (hnsw_rabitq.go:589-801), pinned by
the properties the reference's search has on any graph: with EF at least the
node count over a connected level 0 the base layer visits and accepts every
node, so the search equals the linear scan (scanRaBitQCodes + refinePrepared,
the path the oracle pins to the reference's fixtures); with a small EF the
result is a subset of the linear scan's estimates, sorted by (estimate, key);
an entry point on a higher level walks down through the coarse estimates."""
import numpy as np
import pytest

from oracle.oracle import IP, L2, hnsw_test_graph


def case(oracle, metric, n=1500, d=64, total_bits=1, scale=0.0, seed=3):
    rng = np.random.default_rng(seed)
    centers = rng.standard_normal((8, d)).astype(np.float32)
    rows = (centers[rng.integers(0, 8, n)] + 0.3 * rng.standard_normal((n, d))).astype(np.float32)
    keys = rng.permutation(1 << 20)[:n].astype(np.uint64)
    cents = rows[rng.choice(n, 4, replace=False)].copy()
    padded = oracle.rabitq_padded_dimension(d)
    signs = rng.integers(0, 256, 4 * padded // 8, dtype=np.uint8)
    codes, extra, factors = oracle.rabitq_encode_batch(metric, cents, signs, rows, total_bits,
                                                       scale)
    queries = (centers[rng.integers(0, 8, 9)] + 0.3 * rng.standard_normal((9, d))).astype(np.float32)
    return rows, keys, cents, signs, codes, extra, factors, queries


@pytest.mark.parametrize("metric,total_bits,scale", [(L2, 1, 0.0), (IP, 1, 0.0), (L2, 4, 24.0)])
@pytest.mark.parametrize("refine", [True, False])
def test_full_ef_equals_the_linear_scan(oracle, metric, total_bits, scale, refine):
    rows, keys, cents, signs, codes, extra, factors, queries = case(oracle, metric,
                                                                    total_bits=total_bits,
                                                                    scale=scale)
    n = rows.shape[0]
    graph = hnsw_test_graph(rows, degree=10, seed=1)
    g = oracle.hnsw_rabitq_search(metric, cents, signs, codes, factors, rows, keys, graph,
                                  queries, 10, 2048, refine=refine, total_bits=total_bits,
                                  extra=extra)
    lin = oracle.rabitq_search(metric, cents, signs, codes, factors, rows, keys, queries, 10,
                               n if refine else 10, refine=refine, total_bits=total_bits,
                               extra=extra)
    assert g[0] == 0 and lin[0] == 0
    assert np.array_equal(g[3], lin[3])
    for q in range(queries.shape[0]):
        c = int(g[3][q])
        assert np.array_equal(g[1][q, :c], lin[1][q, :c])
        assert np.array_equal(g[2][q, :c].view(np.uint32), lin[2][q, :c].view(np.uint32))


def test_small_ef_is_a_sorted_subset(oracle):
    rows, keys, cents, signs, codes, extra, factors, queries = case(oracle, L2)
    graph = hnsw_test_graph(rows, degree=6, seed=2)
    assert graph[0] >= 1  # the walk descends through upper levels
    st, ok, os_, oc, ost = oracle.hnsw_rabitq_search(L2, cents, signs, codes, factors, rows, keys,
                                                     graph, queries, 20, 24, refine=False)
    lin = oracle.rabitq_search(L2, cents, signs, codes, factors, rows, keys, queries,
                               rows.shape[0], rows.shape[0], refine=False)
    assert st == 0
    for q in range(queries.shape[0]):
        c = int(oc[q])
        assert c == 20
        est = dict(zip(lin[1][q].tolist(), lin[2][q].tolist()))
        for key, score in zip(ok[q, :c].tolist(), os_[q, :c].tolist()):
            assert est[key] == score
        pairs = list(zip(os_[q, :c].tolist(), ok[q, :c].tolist()))
        assert pairs == sorted(pairs)
