"""One-bit RaBitQ linear search (+ exact refinement): the CUDA path against the
oracle's restatement (hnsw_rabitq.go scan + refine over RaBitQModel codes).

Without refinement the reported scores are the estimates themselves, so a
bit-identical score list also pins the codes, the float64 factors, the
rotation and the query terms.  Keys identical, float32 scores bit-identical."""
import numpy as np
import pytest

from oracle.oracle import COSINE, IP, L2

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def xb():
    import xvec_b200
    assert xvec_b200.device_count() >= 1
    return xvec_b200


def mixture(rng, n, d, centers):
    lab = rng.integers(0, centers.shape[0], n)
    return (centers[lab] + 0.3 * rng.standard_normal((n, d))).astype(np.float32)


def model(rng, d, nc, centers):
    padded = (d + 63) // 64 * 64
    cents = mixture(rng, nc, d, centers)
    signs = rng.integers(0, 256, 4 * padded // 8, dtype=np.uint8)
    return cents, signs


class Case:
    def __init__(self, oracle, xb, metric, rows, keys, cents, signs):
        self.oracle, self.metric = oracle, metric
        self.rows, self.keys, self.cents, self.signs = rows, keys, cents, signs
        self.idx = xb.RaBitQIndex(rows.shape[1], metric)
        self.idx.set_model(cents, signs)
        if rows.shape[0]:
            self.idx.add(keys, rows)
        if rows.shape[0]:
            self.codes, self.factors = oracle.rabitq_encode1_batch(metric, cents, signs, rows)
        else:
            padded = (rows.shape[1] + 63) // 64 * 64
            self.codes = np.zeros((0, padded // 8), np.uint8)
            self.factors = np.zeros(0, self.oracle_factors_dtype())

    @staticmethod
    def oracle_factors_dtype():
        from oracle.oracle import RABITQ_FACTORS_DTYPE
        return RABITQ_FACTORS_DTYPE

    def check(self, xb, queries, k, ef, refine=True, radius=0.0, bitmap=None):
        res = self.idx.search_with_options(
            queries, xb.SearchOptions(top_k=k, ef=ef, refine=refine, radius=radius,
                                      filter=bitmap),
            raise_on_error=False)
        st, ok, os_, oc, ost = self.oracle.rabitq_search(
            self.metric, self.cents, self.signs, self.codes, self.factors, self.rows, self.keys,
            queries, k, ef, radius, bitmap, refine=refine)
        for q in range(queries.shape[0]):
            if ost[q] != 0:
                assert res.counts[q] == -ost[q], (q, res.counts[q], ost[q])
                continue
            c = int(oc[q])
            assert int(res.counts[q]) == c, (self.metric, refine, q, res.counts[q], c)
            assert np.array_equal(res.keys[q, :c], ok[q, :c]), \
                (self.metric, refine, q, res.keys[q, :c], ok[q, :c])
            assert np.array_equal(res.scores[q, :c].view(np.uint32), os_[q, :c].view(np.uint32)), \
                (self.metric, refine, q, res.scores[q, :c], os_[q, :c])
        return res

    def close(self):
        self.idx.close()


@pytest.mark.parametrize("metric", [L2, IP, COSINE])
@pytest.mark.parametrize("d", [64, 100, 256])
def test_rabitq_parity(oracle, xb, metric, d):
    rng = np.random.default_rng(900 + d + metric)
    centers = rng.standard_normal((20, d)).astype(np.float32)
    rows = mixture(rng, 3000, d, centers)
    keys = rng.permutation(100000)[:3000].astype(np.uint64)
    cents, signs = model(rng, d, 8, centers)
    queries = mixture(rng, 37, d, centers)
    case = Case(oracle, xb, metric, rows, keys, cents, signs)
    case.check(xb, queries, 10, 50, refine=False)
    case.check(xb, queries, 10, 50, refine=True)
    case.check(xb, queries, 5, 1, refine=True)     # ef < k: k estimates refined
    case.close()


def test_rabitq_960_shape(oracle, xb):
    """The RaBitQ configuration's shape: d = 960, 16 clusters, k = 10, 10x over-fetch."""
    rng = np.random.default_rng(960)
    d = 960
    centers = rng.standard_normal((50, d)).astype(np.float32)
    rows = mixture(rng, 4000, d, centers)
    keys = np.arange(4000, dtype=np.uint64) * 3 + 11
    cents, signs = model(rng, d, 16, centers)
    queries = mixture(rng, 64, d, centers)
    for metric in (L2, IP):
        case = Case(oracle, xb, metric, rows, keys, cents, signs)
        case.check(xb, queries, 10, 100, refine=True)
        case.check(xb, queries, 10, 100, refine=False)
        case.close()


def test_rabitq_large_candidate_counts(oracle, xb):
    """Candidate counts past the fast accumulators take the exact scan."""
    rng = np.random.default_rng(31)
    d = 128
    centers = rng.standard_normal((10, d)).astype(np.float32)
    rows = mixture(rng, 2500, d, centers)
    keys = rng.permutation(2500).astype(np.uint64)
    cents, signs = model(rng, d, 4, centers)
    queries = mixture(rng, 9, d, centers)
    case = Case(oracle, xb, L2, rows, keys, cents, signs)
    case.check(xb, queries, 10, 2048, refine=True)   # every row refined
    case.check(xb, queries, 10, 700, refine=True)
    case.check(xb, queries, 500, 300, refine=False)
    case.close()


def test_rabitq_filter_radius_edges(oracle, xb):
    rng = np.random.default_rng(77)
    d = 96
    centers = rng.standard_normal((10, d)).astype(np.float32)
    rows = mixture(rng, 900, d, centers)
    rows[3] = 0.0             # zero vector
    rows[8] = rows[12]        # duplicate rows
    rows[20] = 2.5            # constant vector
    keys = np.arange(900, dtype=np.uint64)[::-1].copy()
    cents, signs = model(rng, d, 6, centers)
    queries = mixture(rng, 21, d, centers)
    queries[0] = 0.0
    queries[1] = rows[5]
    queries[2, 7] = np.inf    # PrepareQuery rejects it
    bitmap = np.zeros((900 + 31) // 32, np.uint32)
    for p in range(0, 900, 3):
        bitmap[p >> 5] |= np.uint32(1 << (p & 31))
    for metric in (L2, IP, COSINE):
        case = Case(oracle, xb, metric, rows, keys, cents, signs)
        case.check(xb, queries, 15, 60, refine=True, bitmap=bitmap)
        case.check(xb, queries, 15, 60, refine=False, bitmap=bitmap)
        # Radius: on the public score of the estimate, or on the exact score
        # (a radius must be positive; L2 estimates can fall below zero).
        est = case.check(xb, queries, 40, 60, refine=False)
        mid = float(np.median(np.abs(est.scores[3:, 20])))
        case.check(xb, queries, 40, 60, refine=False, radius=mid)
        ref = case.check(xb, queries, 40, 80, refine=True)
        mid = float(np.median(np.abs(ref.scores[3:, 20])))
        case.check(xb, queries, 40, 80, refine=True, radius=mid)
        case.close()


def test_rabitq_small_and_empty(oracle, xb):
    rng = np.random.default_rng(5)
    d = 64
    centers = rng.standard_normal((3, d)).astype(np.float32)
    cents, signs = model(rng, d, 3, centers)
    queries = mixture(rng, 4, d, centers)
    queries[3, 0] = np.nan
    for n in (0, 1, 7):
        rows = mixture(rng, n, d, centers)
        keys = np.arange(n, dtype=np.uint64)
        case = Case(oracle, xb, L2, rows, keys, cents, signs)
        case.check(xb, queries, 10, 300, refine=True)
        case.check(xb, queries, 10, 300, refine=False)
        case.close()


def test_rabitq_invalid_options(xb):
    rng = np.random.default_rng(1)
    d = 64
    idx = xb.RaBitQIndex(d, L2)
    centers = rng.standard_normal((2, d)).astype(np.float32)
    with pytest.raises(xb.XvecGPUError):          # rows before the model
        idx.add(np.arange(3, dtype=np.uint64), centers[[0, 1, 0]])
    cents, signs = model(rng, d, 2, centers)
    idx.set_model(cents, signs)
    idx.add(np.arange(3, dtype=np.uint64), centers[[0, 1, 0]])
    for ef in (0, 2049):                          # ErrInvalidHNSWEF
        with pytest.raises(xb.XvecGPUError):
            idx.search_with_options(centers, xb.SearchOptions(top_k=1, ef=ef))
    with pytest.raises(xb.XvecGPUError):          # dimension outside [64, 4095]
        xb.RaBitQIndex(63, L2)
    idx.close()


@pytest.mark.parametrize("metric", [L2, IP])
def test_rabitq_tensor_core_seeded(oracle, xb, metric):
    """70,000 rows and 200 queries: the INT8 tensor-core scan on CTA pairs in
    seeding launches plus the rest, refined and not; query magnitudes from
    1e-8 to 1e6 (each query has its own integer scale)."""
    rng = np.random.default_rng(770 + metric)
    d = 128
    centers = rng.standard_normal((40, d)).astype(np.float32)
    rows = mixture(rng, 70_000, d, centers)
    rows[4300:4400] = rows[100:200]          # duplicates across the first launches
    keys = rng.permutation(1 << 22)[:70_000].astype(np.uint64)
    cents, signs = model(rng, d, 16, centers)
    queries = mixture(rng, 200, d, centers)
    case = Case(oracle, xb, metric, rows, keys, cents, signs)
    before = xb.stats()["tensor_scans"]
    case.check(xb, queries, 10, 100, refine=True)
    assert xb.stats()["tensor_scans"] > before, "tensor-core path not taken"
    case.check(xb, queries, 10, 100, refine=False)
    scales = np.repeat(np.array([1e-8, 1e-3, 1.0, 1e3, 1e6], np.float32), 40)
    before = xb.stats()["tensor_scans"]
    case.check(xb, queries * scales[:, None], 10, 100, refine=False)
    assert xb.stats()["tensor_scans"] > before
    case.close()


@pytest.mark.parametrize("nq", [1, 3, 8])
def test_rabitq_small_batches(oracle, xb, nq):
    """Batches of at most 8 queries scan the sign bits through a per-query
    byte table (no tensor-core scan): 70,000 rows, refined and not, a filter,
    and 600 copies of one row (more equal ranks than a part's list keeps)."""
    rng = np.random.default_rng(880 + nq)
    d = 256
    centers = rng.standard_normal((40, d)).astype(np.float32)
    rows = mixture(rng, 70_000, d, centers)
    rows[20_000:20_600] = rows[5]
    keys = rng.permutation(1 << 22)[:70_000].astype(np.uint64)
    cents, signs = model(rng, d, 16, centers)
    queries = mixture(rng, nq, d, centers)
    queries[0] = rows[5] + 0.01
    case = Case(oracle, xb, L2, rows, keys, cents, signs)
    st0 = xb.stats()
    case.check(xb, queries, 10, 100, refine=True)
    st1 = xb.stats()
    assert st1["tensor_scans"] == st0["tensor_scans"], "small batches skip the tensor cores"
    case.check(xb, queries, 10, 100, refine=False)
    bitmap = np.zeros((70_000 + 31) // 32, np.uint32)
    for p in range(70_000):
        if p % 3:
            bitmap[p >> 5] |= np.uint32(1 << (p & 31))
    case.check(xb, queries, 5, 40, refine=True, bitmap=bitmap)
    case.close()
