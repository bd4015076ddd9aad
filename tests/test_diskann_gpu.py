"""DiskANN graph search on the GPU (DiskANNIndex.searchDiskANNGraph,
diskann.go:559-683) against the oracle's restatement of the reference's
sequential traversal: identical keys and bit-identical scores for every
metric, list sizes from below top-k to the whole index, read batches of 128,
64 and 42 nodes (the node layout's MaxDegree), rounds whose neighbour slots
need several merge steps, a visited set beyond the kernel's reset record, a
filter and a radius; Linear (the exact scan); the traversal's errors and the
options it rejects."""
import numpy as np
import pytest

from oracle.oracle import COSINE, IP, L2, MIPSL2, OK, diskann_test_graph

pytestmark = pytest.mark.gpu

METRICS = [L2, IP, COSINE, MIPSL2]


@pytest.fixture(scope="module")
def xb():
    import xvec_b200
    assert xvec_b200.device_count() >= 1
    return xvec_b200


def data(n, d, seed, clusters=12):
    rng = np.random.default_rng(seed)
    centers = rng.standard_normal((clusters, d)).astype(np.float32)
    rows = (centers[rng.integers(0, clusters, n)]
            + 0.3 * rng.standard_normal((n, d))).astype(np.float32)
    keys = rng.permutation(1 << 22)[:n].astype(np.uint64)
    queries = (centers[rng.integers(0, clusters, 24)]
               + 0.3 * rng.standard_normal((24, d))).astype(np.float32)
    return rows, keys, queries


def build(oracle, xb, metric, rows, keys, chunks, degree, max_degree=None, seed=0):
    """Both sides from the same traversal model: TrainPQ on the prepared rows
    under the traversal metric (the oracle's), the codes encoded by each side
    (the GPU at insertion, the oracle here), the same graph."""
    d = rows.shape[1]
    tm = oracle.diskann_traversal_metric(metric)
    prepared = oracle.diskann_prepare(metric, rows)
    st, pivots = oracle.pq_train(tm, prepared, chunks, seed=seed)
    assert st == OK
    offsets = oracle.pq_chunk_offsets(d, chunks)
    codes, norms = oracle.diskann_encode(metric, pivots, offsets, rows)
    graph = diskann_test_graph(rows, degree=degree, seed=seed)
    max_degree = max_degree or int(np.diff(graph[1]).max())
    idx = xb.DiskANNIndex(d, metric)
    idx.set_model(pivots, chunks)
    idx.add(keys, rows)
    idx.set_graph(graph[0], max_degree, graph[1], graph[2])
    ref = dict(pivots=pivots, offsets=offsets, codes=codes, norms=norms, graph=graph,
               beam=oracle.diskann_read_batch(d, max_degree))
    return idx, ref


def compare(oracle, xb, idx, ref, metric, rows, keys, queries, k, list_size, radius=0.0,
            bitmap=None):
    st, ok_, os_, oc, ost = oracle.diskann_search(
        metric, ref["pivots"], ref["offsets"], ref["codes"], ref["norms"], rows, keys,
        ref["graph"], ref["beam"], queries, k, list_size, radius=radius, bitmap=bitmap)
    res = idx.search_with_options(queries, xb.SearchOptions(top_k=k, ef=list_size, radius=radius,
                                                            filter=bitmap),
                                  raise_on_error=False)
    for q in range(queries.shape[0]):
        if ost[q] != OK:
            assert res.counts[q] == -ost[q], (q, ost[q], res.counts[q])
            continue
        c = int(oc[q])
        assert res.counts[q] == c, (q, c, res.counts[q])
        assert np.array_equal(res.keys[q, :c], ok_[q, :c]), q
        assert np.array_equal(res.scores[q, :c].view(np.uint32), os_[q, :c].view(np.uint32)), q
    return oc


@pytest.mark.parametrize("metric", METRICS)
@pytest.mark.parametrize("d,chunks", [(8, 4), (17, 5), (128, 32)])
def test_diskann_parity(oracle, xb, metric, d, chunks):
    rows, keys, queries = data(3000, d, seed=d + metric)
    idx, ref = build(oracle, xb, metric, rows, keys, chunks, degree=16)
    for k, list_size in [(10, 8), (10, 64), (1, 300), (100, 100), (32, 2048)]:
        counts = compare(oracle, xb, idx, ref, metric, rows, keys, queries, k, list_size)
        assert (counts > 0).all()


@pytest.mark.parametrize("max_degree", [16, 1000, 2048])
def test_diskann_read_batches(oracle, xb, max_degree):
    # MaxDegree 16 / 1000 / 2048 at d = 128: 1, 2 and 3 sectors per node,
    # read batches of 128, 64 and 42 nodes.
    rows, keys, queries = data(4000, 128, seed=3)
    idx, ref = build(oracle, xb, L2, rows, keys, 16, degree=16, max_degree=max_degree)
    assert ref["beam"] == {16: 128, 1000: 64, 2048: 42}[max_degree]
    compare(oracle, xb, idx, ref, L2, rows, keys, queries, 10, 300)


def test_diskann_merge_steps_and_visit_overflow(oracle, xb):
    # Degree 40 with 128-node rounds needs three merge steps of 2048 slots;
    # a 2048-node list visits more nodes than the reset record holds.
    rows, keys, queries = data(30000, 32, seed=11, clusters=40)
    idx, ref = build(oracle, xb, IP, rows, keys, 8, degree=40)
    compare(oracle, xb, idx, ref, IP, rows, keys, queries[:8], 50, 2048)
    compare(oracle, xb, idx, ref, IP, rows, keys, queries, 10, 200)


@pytest.mark.parametrize("metric", METRICS)
def test_diskann_filter_radius(oracle, xb, metric):
    rows, keys, queries = data(2500, 24, seed=7)
    idx, ref = build(oracle, xb, metric, rows, keys, 6, degree=12)
    n = rows.shape[0]
    bitmap = np.zeros((n + 31) // 32, np.uint32)
    for p in range(n):
        if int(keys[p]) % 3 != 0:
            bitmap[p >> 5] |= np.uint32(1 << (p & 31))
    compare(oracle, xb, idx, ref, metric, rows, keys, queries, 20, 100, bitmap=bitmap)
    st, _, os_, oc, _ = oracle.diskann_search(metric, ref["pivots"], ref["offsets"], ref["codes"],
                                              ref["norms"], rows, keys, ref["graph"], ref["beam"],
                                              queries[:1], 20, 100)
    radius = float(os_[0, 7])
    if metric == IP and radius <= 0:
        radius = 0.0001
    compare(oracle, xb, idx, ref, metric, rows, keys, queries, 20, 100, radius=radius)


def test_diskann_small_index_and_list_beyond_it(oracle, xb):
    rows, keys, queries = data(40, 16, seed=2)
    idx, ref = build(oracle, xb, COSINE, rows, keys, 4, degree=8)
    compare(oracle, xb, idx, ref, COSINE, rows, keys, queries, 100, 300)
    compare(oracle, xb, idx, ref, COSINE, rows, keys, queries, 5, 1)


def test_diskann_linear_is_the_exact_scan(oracle, xb):
    rows, keys, queries = data(3000, 64, seed=4)
    idx, ref = build(oracle, xb, L2, rows, keys, 16, degree=16)
    res = idx.search_with_options(queries, xb.SearchOptions(top_k=10, linear=True))
    st, ok_, os_, oc, _ = oracle.flat_search(L2, rows, keys, queries, 10)
    assert st == OK
    assert np.array_equal(res.keys, ok_)
    assert np.array_equal(res.scores.view(np.uint32), os_.view(np.uint32))


def test_diskann_errors_and_options(oracle, xb):
    rows, keys, queries = data(600, 16, seed=9)
    idx, ref = build(oracle, xb, L2, rows, keys, 4, degree=8)
    # ErrInvalidDiskANNListSize; capacity beyond the kernel's 2048.
    with pytest.raises(xb.XvecGPUError) as e:
        idx.search_with_options(queries, xb.SearchOptions(top_k=5, ef=-1))
    assert e.value.status == xb.INVALID_ARGUMENT
    with pytest.raises(xb.XvecGPUError) as e:
        idx.search_with_options(queries, xb.SearchOptions(top_k=2049, ef=10))
    # ef 0: DefaultDiskANNQueryList (300).
    a = idx.search_with_options(queries, xb.SearchOptions(top_k=10, ef=0))
    b = idx.search_with_options(queries, xb.SearchOptions(top_k=10, ef=300))
    assert np.array_equal(a.keys, b.keys)
    # A non-finite query fails alone (metric.Compute(query, query)).
    bad = queries.copy()
    bad[3, 2] = np.inf
    res = idx.search_with_options(bad, xb.SearchOptions(top_k=10, ef=50), raise_on_error=False)
    assert res.counts[3] == -xb.NON_FINITE and (np.delete(res.counts, 3) == 10).all()
    # Rows added after the graph make it stale.
    idx.add(np.asarray([1 << 40], np.uint64), rows[:1] + 1.0)
    with pytest.raises(xb.XvecGPUError):
        idx.search_with_options(queries, xb.SearchOptions(top_k=5, ef=20))
    # Graphs the library rejects: a neighbour outside the index, a list
    # longer than MaxDegree.
    offsets = np.arange(0, 602, dtype=np.int64)
    offsets[-1] = 601
    nbrs = np.zeros(601, np.int32)
    nbrs[5] = 601
    with pytest.raises(xb.XvecGPUError):
        idx.set_graph(0, 2, offsets, nbrs)
    nbrs[5] = 0
    with pytest.raises(xb.XvecGPUError):
        idx.set_graph(0, 0, offsets, nbrs)
    idx.close()


def test_diskann_needs_a_model(xb):
    idx = xb.DiskANNIndex(8, L2)
    with pytest.raises(xb.XvecGPUError):
        idx.add(np.arange(4, dtype=np.uint64), np.ones((4, 8), np.float32))
    idx.close()


def test_diskann_empty_index(oracle, xb):
    rng = np.random.default_rng(1)
    idx = xb.DiskANNIndex(8, L2)
    idx.set_model(rng.standard_normal((256, 8)).astype(np.float32), 4)
    res = idx.search_with_options(rng.standard_normal((3, 8)).astype(np.float32),
                                  xb.SearchOptions(top_k=5, ef=10))
    assert (res.counts == 0).all()
    idx.close()
