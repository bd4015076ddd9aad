"""Multi-bit RaBitQ linear search (RaBitQModelState.TotalBits > 1): the CUDA
path against the oracle's restatement of quantizeRaBitQVector with extra bits
(rabitq_quantize.go:99-200), Estimate on the full codes (rabitq.go:434-446)
and the scan + refine of hnsw_rabitq.go:539-642, 780-801.

Without refinement the reported scores are the estimates themselves, so a
bit-identical score list also pins the extra codes and the full factors.
Keys identical, float32 scores bit-identical."""
import numpy as np
import pytest

from oracle.oracle import COSINE, IP, L2

pytestmark = pytest.mark.gpu

# An ExtraScale per TotalBits that spreads the extra codes over their range
# for the rotated unit residuals of these dimensions.
SCALES = {2: 3.0, 4: 24.0, 7: 190.0, 8: 380.0, 9: 760.0}


@pytest.fixture(scope="module")
def xb():
    import xvec_b200
    assert xvec_b200.device_count() >= 1
    return xvec_b200


def mixture(rng, n, d, centers, sigma=0.3):
    lab = rng.integers(0, centers.shape[0], n)
    return (centers[lab] + sigma * rng.standard_normal((n, d))).astype(np.float32)


class MultiCase:
    def __init__(self, oracle, xb, metric, rows, keys, cents, signs, total_bits, scale):
        self.oracle, self.metric, self.tb = oracle, metric, total_bits
        self.rows, self.keys, self.cents, self.signs = rows, keys, cents, signs
        self.idx = xb.RaBitQIndex(rows.shape[1], metric)
        self.idx.set_model(cents, signs, total_bits, scale)
        self.idx.add(keys, rows)
        self.codes, self.extra, self.factors = oracle.rabitq_encode_batch(
            metric, cents, signs, rows, total_bits, scale)

    def check(self, xb, queries, k, ef, refine=True, radius=0.0, bitmap=None):
        res = self.idx.search_with_options(
            queries, xb.SearchOptions(top_k=k, ef=ef, refine=refine, radius=radius,
                                      filter=bitmap),
            raise_on_error=False)
        st, ok, os_, oc, ost = self.oracle.rabitq_search(
            self.metric, self.cents, self.signs, self.codes, self.factors, self.rows, self.keys,
            queries, k, ef, radius, bitmap, refine=refine, total_bits=self.tb, extra=self.extra)
        for q in range(queries.shape[0]):
            if ost[q] != 0:
                assert res.counts[q] == -ost[q], (q, res.counts[q], ost[q])
                continue
            c = int(oc[q])
            assert int(res.counts[q]) == c, (self.tb, self.metric, refine, q, res.counts[q], c)
            assert np.array_equal(res.keys[q, :c], ok[q, :c]), (self.tb, self.metric, refine, q)
            assert np.array_equal(res.scores[q, :c].view(np.uint32), os_[q, :c].view(np.uint32)), \
                (self.tb, self.metric, refine, q, res.scores[q, :c], os_[q, :c])
        return res

    def close(self):
        self.idx.close()


@pytest.mark.parametrize("total_bits", [2, 4, 7, 8, 9])
@pytest.mark.parametrize("metric", [L2, IP, COSINE])
def test_multibit_parity(oracle, xb, metric, total_bits):
    rng = np.random.default_rng(300 + 10 * total_bits + metric)
    d = 100
    centers = rng.standard_normal((12, d)).astype(np.float32)
    rows = mixture(rng, 3000, d, centers)
    keys = rng.permutation(1 << 20)[:3000].astype(np.uint64)
    cents = mixture(rng, 6, d, centers)
    signs = rng.integers(0, 256, 4 * 128 // 8, dtype=np.uint8)
    queries = mixture(rng, 41, d, centers)
    case = MultiCase(oracle, xb, metric, rows, keys, cents, signs, total_bits,
                     SCALES[total_bits])
    case.check(xb, queries, 10, 30, refine=True)
    case.check(xb, queries, 10, 30, refine=False)
    case.check(xb, queries[:3], 5, 12, refine=False)  # one query block
    case.close()


def test_multibit_960_tensor_core(oracle, xb):
    """d = 960 with 150 queries (CTA pairs) and 70,000 rows (the seeded
    launches over row prefixes), TotalBits 7: the INT8 tensor-core scan of
    the code plane against the 16-bit integer query."""
    import xvec_b200
    rng = np.random.default_rng(960)
    d, n = 960, 70_000
    centers = rng.standard_normal((40, d)).astype(np.float32)
    rows = mixture(rng, n, d, centers)
    keys = rng.permutation(1 << 22)[:n].astype(np.uint64)
    cents = mixture(rng, 16, d, centers)
    signs = rng.integers(0, 256, 4 * 960 // 8, dtype=np.uint8)
    queries = mixture(rng, 150, d, centers)
    queries[3] = rows[77]
    case = MultiCase(oracle, xb, L2, rows, keys, cents, signs, 7, 620.0)
    st0 = xvec_b200.stats()
    case.check(xb, queries, 10, 100, refine=True)
    st1 = xvec_b200.stats()
    assert st1["tensor_scans"] > st0["tensor_scans"]
    # The INT8 form's bound (exact integer dots, 16-bit query) is tight
    # enough that no query needs the exact scan.
    assert st1["exact_queries"] == st0["exact_queries"]
    case.check(xb, queries, 10, 50, refine=False)
    case.close()


def test_multibit_filter_radius(oracle, xb):
    rng = np.random.default_rng(71)
    d = 128
    centers = rng.standard_normal((10, d)).astype(np.float32)
    rows = mixture(rng, 4000, d, centers)
    rows[100:110] = rows[5]                      # equal codes: ties by key
    keys = np.arange(4000, dtype=np.uint64) * 3 + 1
    cents = mixture(rng, 5, d, centers)
    signs = rng.integers(0, 256, 4 * 128 // 8, dtype=np.uint8)
    queries = mixture(rng, 30, d, centers)
    queries[2, 4] = np.nan                       # rejected by PrepareQuery
    bitmap = np.zeros(4000 // 32, np.uint32)
    for p in range(4000):
        if p % 7:
            bitmap[p >> 5] |= np.uint32(1 << (p & 31))
    for metric in (L2, IP):
        case = MultiCase(oracle, xb, metric, rows, keys, cents, signs, 5, 48.0)
        case.check(xb, queries, 20, 40, refine=True, bitmap=bitmap)
        case.check(xb, queries, 20, 40, refine=False, bitmap=bitmap)
        radius = 60.0 if metric == L2 else 0.5
        case.check(xb, queries, 50, 80, refine=False, radius=radius)
        case.close()


def test_multibit_model_validation(xb):
    d = 64
    cents = np.zeros((2, d), np.float32)
    cents[1, 0] = 1.0
    signs = np.zeros(4 * 64 // 8, np.uint8)
    for tb, scale in ((0, 1.0), (10, 1.0), (1, 2.0), (4, 0.0), (4, -1.0), (4, float("inf"))):
        idx = xb.RaBitQIndex(d, L2)
        with pytest.raises(xb.XvecGPUError):
            idx.set_model(cents, signs, tb, scale)
        idx.close()


def test_multibit_two_shards_refined(oracle, xb):
    """The two halves of a refined search (candidates, then the refine of the
    merged candidates each shard holds) over multi-bit shards equal one
    refined search over all rows."""
    import torch
    rng = np.random.default_rng(412)
    d, n = 128, 5000
    centers = rng.standard_normal((20, d)).astype(np.float32)
    rows = mixture(rng, n, d, centers)
    keys = rng.permutation(1 << 20)[:n].astype(np.uint64)
    cents = mixture(rng, 8, d, centers)
    signs = rng.integers(0, 256, 4 * 128 // 8, dtype=np.uint8)
    queries = mixture(rng, 29, d, centers)
    opts = xb.SearchOptions(top_k=10, ef=25, refine=True)
    dev = torch.device("cuda", 0)
    q = torch.from_numpy(queries).to(dev)
    nq, k = queries.shape[0], opts.top_k
    shards = []
    for b, e in ((0, 2100), (2100, n)):
        idx = xb.RaBitQIndex(d, L2)
        idx.set_model(cents, signs, 6, 90.0)
        idx.add(keys[b:e], rows[b:e])
        shards.append(idx)
    c = shards[0].candidate_count(opts)
    cands = []
    for idx in shards:
        ck = torch.zeros((nq, c), dtype=torch.int64, device=dev)
        cr = torch.zeros((nq, c), dtype=torch.float32, device=dev)
        cc = torch.zeros((nq,), dtype=torch.int32, device=dev)
        idx.candidates_device(q.data_ptr(), nq, opts, ck.data_ptr(), cr.data_ptr(), cc.data_ptr())
        torch.cuda.synchronize()
        cands.append((ck.cpu().numpy().view(np.uint64), cr.cpu().numpy(), cc.cpu().numpy()))

    def merge(metric, kk, parts):
        mk = np.zeros((nq, kk), np.uint64)
        ms = np.zeros((nq, kk), np.float32)
        mc = np.zeros(nq, np.int32)
        for qi in range(nq):
            allk = np.concatenate([p[0][qi, :p[2][qi]] for p in parts])
            alls = np.concatenate([p[1][qi, :p[2][qi]] for p in parts])
            rk, rs = oracle.merge_results(metric, kk, allk, alls)
            mk[qi, :rk.size], ms[qi, :rk.size], mc[qi] = rk, rs, rk.size
        return mk, ms, mc

    mk, _, mc = merge(L2, c, cands)
    d_mk = torch.from_numpy(mk.view(np.int64)).to(dev)
    d_mc = torch.from_numpy(mc).to(dev)
    refined = []
    for idx in shards:
        ok = torch.zeros((nq, k), dtype=torch.int64, device=dev)
        os_ = torch.zeros((nq, k), dtype=torch.float32, device=dev)
        oc = torch.zeros((nq,), dtype=torch.int32, device=dev)
        idx.refine_device(q.data_ptr(), nq, d_mk.data_ptr(), c, d_mc.data_ptr(), k, 0.0,
                          ok.data_ptr(), os_.data_ptr(), oc.data_ptr())
        torch.cuda.synchronize()
        refined.append((ok.cpu().numpy().view(np.uint64), os_.cpu().numpy(), oc.cpu().numpy()))
    gk, gs, gc = merge(L2, k, refined)
    codes, extra, factors = oracle.rabitq_encode_batch(L2, cents, signs, rows, 6, 90.0)
    _, ok, os_, oc, ost = oracle.rabitq_search(L2, cents, signs, codes, factors, rows, keys,
                                               queries, k, 25, refine=True, total_bits=6,
                                               extra=extra)
    for qi in range(nq):
        cnt = int(oc[qi])
        assert gc[qi] == cnt
        assert np.array_equal(gk[qi, :cnt], ok[qi, :cnt]), qi
        assert np.array_equal(gs[qi, :cnt].view(np.uint32), os_[qi, :cnt].view(np.uint32)), qi
    for idx in shards:
        idx.close()
