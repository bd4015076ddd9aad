"""The oracle's DiskANN graph search (DiskANNIndex.searchDiskANNGraph,
diskann.go:559-683) against the properties the reference's own tests pin
(diskann_test.go:36-109, 247-278): with a list as large as the index the
traversal reaches every node and returns exactly the linear scan's results;
a filter and a radius hold on what it returns; with a list of 64 over 320
nodes it finds at least 80% of the exact top 10; the read batch follows the
node layout."""
import math

import numpy as np
import pytest

from oracle.oracle import COSINE, IP, L2, MIPSL2, OK, Oracle, diskann_test_graph

METRICS = [L2, IP, COSINE, MIPSL2]


def candidates(count, dimension):
    """diskANNIndexCandidates (diskann_test.go:342-353)."""
    rows = np.zeros((count, dimension), np.float32)
    for p in range(count):
        for c in range(dimension):
            angle = float((p + 3) * (c + 5)) * 0.071
            rows[p, c] = np.float32(math.sin(angle) + 0.45 * math.cos(angle * 0.37)
                                    + float(p % 9) * 0.025)
    keys = np.asarray([1000 + p * 7 for p in range(count)], np.uint64)
    return rows, keys


def build(oracle, metric, rows, chunks, degree, seed=0):
    """The DiskANN build's traversal encoding (diskann.go:224-249): TrainPQ
    on the prepared rows under the traversal metric, their codes and, for
    MIPSL2, the code norms; and a proximity graph."""
    tm = oracle.diskann_traversal_metric(metric)
    prepared = oracle.diskann_prepare(metric, rows)
    st, pivots = oracle.pq_train(tm, prepared, chunks, seed=seed)
    assert st == OK
    offsets = oracle.pq_chunk_offsets(rows.shape[1], chunks)
    codes, norms = oracle.diskann_encode(metric, pivots, offsets, rows)
    graph = diskann_test_graph(rows, degree=degree, seed=seed)
    return pivots, offsets, codes, norms, graph


@pytest.fixture(scope="module")
def small():
    return candidates(72, 8)


@pytest.mark.parametrize("metric", METRICS)
def test_full_list_equals_linear(oracle, small, metric):
    rows, keys = small
    pivots, offsets, codes, norms, graph = build(oracle, metric, rows, 4, 8)
    query = rows[17:18].copy()
    beam = oracle.diskann_read_batch(8, 8)
    st, wk, ws, wc, _ = oracle.flat_search(metric, rows, keys, query, 12)
    assert st == OK
    st, gk, gs, gc, gst = oracle.diskann_search(metric, pivots, offsets, codes, norms, rows, keys,
                                                graph, beam, query, 12, list_size=72)
    assert st == OK and gst[0] == OK
    assert gc[0] == wc[0] == 12
    assert np.array_equal(gk, wk)
    assert np.array_equal(gs.view(np.uint32), ws.view(np.uint32))
    assert int(gk[0, 0]) == int(keys[17])


@pytest.mark.parametrize("metric", METRICS)
def test_filter_and_radius_hold(oracle, small, metric):
    rows, keys = small
    pivots, offsets, codes, norms, graph = build(oracle, metric, rows, 4, 8)
    query = rows[17:18].copy()
    beam = oracle.diskann_read_batch(8, 8)
    st, wk, ws, wc, _ = oracle.flat_search(metric, rows, keys, query, 12)
    bitmap = np.zeros(3, np.uint32)
    for p in range(72):
        if int(keys[p]) % 2 == 0:
            bitmap[p >> 5] |= np.uint32(1 << (p & 31))
    st, fk, fs, fc, _ = oracle.diskann_search(metric, pivots, offsets, codes, norms, rows, keys,
                                              graph, beam, query, 12, list_size=72, bitmap=bitmap)
    assert st == OK and fc[0] > 0
    assert all(int(x) % 2 == 0 for x in fk[0, :fc[0]])
    radius = float(ws[0, min(5, wc[0] - 1)])
    if metric == IP and radius <= 0:
        radius = 0.0001
    st, rk, rs, rc, _ = oracle.diskann_search(metric, pivots, offsets, codes, norms, rows, keys,
                                              graph, beam, query, 12, list_size=72,
                                              radius=radius)
    assert st == OK
    for s in rs[0, :rc[0]]:
        assert (s >= radius) if metric == IP else (s <= radius)


def test_approximate_recall(oracle):
    rows, keys = candidates(320, 16)
    pivots, offsets, codes, norms, graph = build(oracle, L2, rows, 8, 12)
    beam = oracle.diskann_read_batch(16, 12)
    qids = [(i * 37 + 11) % 320 for i in range(8)]
    queries = rows[qids].copy()
    st, wk, _, _, _ = oracle.flat_search(L2, rows, keys, queries, 10)
    st, gk, _, gc, _ = oracle.diskann_search(L2, pivots, offsets, codes, norms, rows, keys, graph,
                                             beam, queries, 10, list_size=64)
    assert st == OK
    hits = sum(len(set(gk[q, :gc[q]].tolist()) & set(wk[q].tolist())) for q in range(8))
    assert hits / 80 >= 0.80


def test_invalid_options_and_empty(oracle, small):
    rows, keys = small
    pivots, offsets, codes, norms, graph = build(oracle, L2, rows, 4, 8)
    query = rows[:1].copy()
    st, *_ = oracle.diskann_search(L2, pivots, offsets, codes, norms, rows, keys, graph, 128,
                                   query, 5, list_size=0)
    assert st != OK
    st, *_ = oracle.diskann_search(L2, pivots, offsets, codes, norms, rows, keys, graph, 128,
                                   query, 0, list_size=10)
    assert st != OK
    bad = query.copy()
    bad[0, 3] = np.nan
    st, _, _, c, qst = oracle.diskann_search(L2, pivots, offsets, codes, norms, rows, keys, graph,
                                             128, bad, 5, list_size=10)
    assert qst[0] != OK and c[0] == 0


def test_read_batch_follows_the_layout():
    assert Oracle.diskann_read_batch(8, 8) == 128
    assert Oracle.diskann_read_batch(128, 64) == 128
    assert Oracle.diskann_read_batch(960, 64) == 64  # 4104-byte records: 2 sectors
    assert Oracle.diskann_read_batch(128, 2048) == 42  # 8712 bytes: 3 sectors


def test_batch_encoders_equal_the_row_encoders(oracle):
    rng = np.random.default_rng(4)
    rows = rng.standard_normal((300, 70)).astype(np.float32)
    offsets = oracle.pq_chunk_offsets(70, 9)
    pivots = rng.standard_normal((256, 70)).astype(np.float32)
    codes = oracle.pq_encode_rows(L2, pivots, offsets, rows)
    for i in range(0, 300, 37):
        st, c = oracle.pq_encode(L2, pivots, offsets, rows[i])
        assert st == OK and np.array_equal(c, codes[i])
    cents = rows[:5].copy()
    signs = rng.integers(0, 256, 4 * oracle.rabitq_padded_dimension(70) // 8, dtype=np.uint8)
    for bits, scale in [(1, 0.0), (4, 24.0)]:
        a = oracle.rabitq_encode_rows(L2, cents, signs, rows, bits, scale)
        b = oracle.rabitq_encode_batch(L2, cents, signs, rows, bits, scale)
        assert np.array_equal(a[0], b[0]) and np.array_equal(a[1], b[1])
        assert a[2].tobytes() == b[2].tobytes()
