"""INT4 and FP16 scalar-quantized Flat search on the GPU against the oracle.

INT4 (XVEC_INDEX_SQ4_FLAT): the oracle's SQ-Flat search over INT4 codes
(quantized_index.go:296-335 with QuantizationInt4); the library keeps the
codes one per byte and scans them with the INT8 kind's kernels.  FP16: QuantizedDistance
decodes both binary16 vectors and applies metric.Compute (quantization.go:
187-191), so the oracle is its Flat search over the decoded rows and queries.
Keys identical, float32 scores bit-identical."""
import numpy as np
import pytest

from oracle.oracle import COSINE, IP, L2, MIPSL2

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def xb():
    import xvec_b200
    assert xvec_b200.device_count() >= 1
    return xvec_b200


def scaled_gaussian(rng, n, d):
    s = rng.uniform(0.5, 2.0, d).astype(np.float32)
    return rng.standard_normal((n, d)).astype(np.float32) * s


def compare(res, ok, os_, oc, ost, tag):
    for q in range(ok.shape[0]):
        if ost[q] != 0:
            assert res.counts[q] == -ost[q], (tag, q, res.counts[q], ost[q])
            continue
        c = int(oc[q])
        assert int(res.counts[q]) == c, (tag, q, res.counts[q], c)
        assert np.array_equal(res.keys[q, :c], ok[q, :c]), (tag, q)
        assert np.array_equal(res.scores[q, :c].view(np.uint32), os_[q, :c].view(np.uint32)), \
            (tag, q, res.scores[q, :c], os_[q, :c])


def run_int4(oracle, xb, metric, rows, keys, queries, k, refine=0.0, radius=0.0, bitmap=None):
    idx = xb.Int4QuantizedFlatIndex(rows.shape[1], metric)
    idx.add(keys, rows)
    res = idx.search_with_options(queries, xb.SearchOptions(top_k=k, refine_scale=refine,
                                                             radius=radius, filter=bitmap),
                                  raise_on_error=False)
    packed, params = oracle.quantize_int4_batch(rows)
    st, ok, os_, oc, ost = oracle.sq4_search(metric, packed, params, rows, keys, queries, k,
                                             radius, refine, bitmap)
    compare(res, ok, os_, oc, ost, (metric, refine, radius))
    idx.close()


@pytest.mark.parametrize("metric", [IP, L2, COSINE, MIPSL2])
@pytest.mark.parametrize("d", [4, 18, 128])
def test_int4_parity(oracle, xb, metric, d):
    rng = np.random.default_rng(700 + d + metric)
    rows = scaled_gaussian(rng, 2500, d)
    keys = rng.permutation(50000)[:2500].astype(np.uint64)
    queries = scaled_gaussian(rng, 37, d)
    st0 = xb.stats()
    run_int4(oracle, xb, metric, rows, keys, queries, 10)
    run_int4(oracle, xb, metric, rows, keys, queries, 10, refine=4.0)
    if d == 128 and metric in (L2, IP):     # the tcgen05 kind::i8 scan of the INT8 kind
        assert xb.stats()["tensor_scans"] > st0["tensor_scans"]


def test_int4_filter_radius_ties(oracle, xb):
    rng = np.random.default_rng(41)
    d = 64
    rows = scaled_gaussian(rng, 4000, d)
    rows[200:230] = rows[7]                      # equal codes: ties by key
    rows[300] = 2.5                              # a constant row (inverse scale 0)
    keys = np.arange(4000, dtype=np.uint64) * 5 + 3
    queries = scaled_gaussian(rng, 25, d)
    queries[4] = rows[7]
    queries[5, 3] = np.inf                       # rejected by validateQuery
    bitmap = np.zeros(4000 // 32, np.uint32)
    for p in range(4000):
        if p % 5:
            bitmap[p >> 5] |= np.uint32(1 << (p & 31))
    for metric in (L2, IP):
        run_int4(oracle, xb, metric, rows, keys, queries, 40, bitmap=bitmap)
        radius = 60.0 if metric == L2 else 2.0
        run_int4(oracle, xb, metric, rows, keys, queries, 50, radius=radius)
        run_int4(oracle, xb, metric, rows, keys, queries, 10, refine=3.0, bitmap=bitmap)


def test_int4_odd_dimension(xb):
    idx = xb.Int4QuantizedFlatIndex(5, L2)
    with pytest.raises(xb.XvecGPUError) as e:
        idx.add(np.arange(3, dtype=np.uint64), np.ones((3, 5), np.float32))
    assert e.value.status == xb.INVALID_ARGUMENT
    assert len(idx) == 0
    res = idx.search_with_options(np.ones((2, 5), np.float32), xb.SearchOptions(top_k=3),
                                  raise_on_error=False)
    assert list(res.counts) == [-xb.INVALID_ARGUMENT] * 2
    idx.close()


@pytest.mark.parametrize("metric", [L2, IP, COSINE, MIPSL2])
@pytest.mark.parametrize("d", [18, 64])
def test_int4_ivf_is_int4_over_the_probed_lists(oracle, xb, metric, d):
    """ScalarQuantizedIVFIndex with QuantizationInt4 (ivf_quantized.go:135-192)
    is the INT4 SQ search restricted to the probed lists' positions: per
    query, the oracle's INT4 search with a filter holding exactly those
    positions (the same composition the oracle pins for INT8).  d = 64 runs
    the list-major interleaved code copy (d a multiple of 16); d = 18 the
    scan of the codes by position."""
    from oracle.zvecivf import csr_of
    rng = np.random.default_rng(60 + metric + 10 * d)
    n, nlist = 3000, 16
    rows = scaled_gaussian(rng, n, d)
    keys = rng.permutation(1 << 20)[:n].astype(np.uint64)
    cents = rows[rng.choice(n, nlist, replace=False)].copy()
    lists = rng.integers(0, nlist, n).astype(np.int32)
    queries = scaled_gaussian(rng, 21, d)
    idx = xb.Int4QuantizedIVFIndex(d, metric)
    idx.set_model(cents)
    idx.add_with_lists(keys, rows, lists)
    offsets, positions = csr_of(lists, nlist)
    packed, params = oracle.quantize_int4_batch(rows)
    for nprobe, scale in ((4, 0.0), (4, 3.0), (nlist, 0.0)):
        res = idx.search_with_options(queries, xb.SearchOptions(top_k=10, nprobe=nprobe,
                                                                 refine_scale=scale),
                                      raise_on_error=False)
        for q in range(queries.shape[0]):
            probed = oracle.ivf_probe(metric, cents, queries[q], nprobe)
            bitmap = np.zeros((n + 31) // 32, np.uint32)
            for li in probed:
                for p in positions[offsets[li]:offsets[li + 1]]:
                    bitmap[p >> 5] |= np.uint32(1 << int(p & 31))
            st, ok, os_, oc, ost = oracle.sq4_search(metric, packed, params, rows, keys,
                                                     queries[q:q + 1], 10, 0.0, scale, bitmap)
            one = type(res)(res.keys[q:q + 1], res.scores[q:q + 1], res.counts[q:q + 1])
            compare(one, ok, os_, oc, ost, (metric, nprobe, scale, q))
    idx.close()


@pytest.mark.parametrize("metric", [L2, IP, COSINE, MIPSL2])
def test_fp16_quantized_parity(oracle, xb, metric):
    rng = np.random.default_rng(90 + metric)
    d = 96
    rows = scaled_gaussian(rng, 3000, d) * 7
    keys = rng.permutation(1 << 20)[:3000].astype(np.uint64)
    queries = scaled_gaussian(rng, 33, d) * 7
    queries[2, 0] = 70000.0                      # ErrQuantizationOverflow for this query
    queries[3, 1] = np.nan                       # rejected by validateQuery
    idx = xb.FP16QuantizedFlatIndex(d, metric)
    idx.add(keys, rows)
    res = idx.search_with_options(queries, xb.SearchOptions(top_k=10), raise_on_error=False)
    assert res.counts[2] == -xb.OVERFLOW and res.counts[3] == -xb.NON_FINITE
    dec_rows = rows.astype(np.float16).astype(np.float32)
    good = np.array([q for q in range(33) if q not in (2, 3)])
    dec_q = queries[good].astype(np.float16).astype(np.float32)
    st, ok, os_, oc, ost = oracle.flat_search(metric, dec_rows, keys, dec_q, 10)
    sub = type(res)(res.keys[good], res.scores[good], res.counts[good])
    compare(sub, ok, os_, oc, ost, metric)
    with pytest.raises(xb.XvecGPUError) as e:
        idx.add(np.array([1 << 40], np.uint64), np.full((1, d), 1e6, np.float32))
    assert e.value.status == xb.OVERFLOW
    assert len(idx) == 3000
    idx.close()
