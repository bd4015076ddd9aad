"""The two halves of a refined search through the C ABI
(xvec_gpu_index_candidates_device, xvec_gpu_index_refine_device), driven the
way a sharded search drives them: two shard indexes in one process, their
candidates merged by rank, each shard refining the merged candidates it
holds, the refined lists merged.  The result must equal one refined search
over all rows (the oracle's, and the library's own single-index search)."""
import numpy as np
import pytest

from oracle.oracle import IP, L2

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def xb():
    import xvec_b200
    assert xvec_b200.device_count() >= 1
    return xvec_b200


def _merge(oracle, metric, kk, parts):
    """MergeSearchResults of [(keys, scores, counts)] per query."""
    nq = parts[0][2].shape[0]
    keys = np.zeros((nq, kk), np.uint64)
    scores = np.zeros((nq, kk), np.float32)
    counts = np.zeros(nq, np.int32)
    for q in range(nq):
        cs = [p[2][q] for p in parts]
        if min(cs) < 0:
            counts[q] = min(cs)
            continue
        mk = np.concatenate([p[0][q, :p[2][q]] for p in parts])
        ms = np.concatenate([p[1][q, :p[2][q]] for p in parts])
        rk, rs = oracle.merge_results(metric, kk, mk, ms)
        keys[q, :rk.size], scores[q, :rk.size], counts[q] = rk, rs, rk.size
    return keys, scores, counts


def _two_shard_refined(xb, oracle, shards, metric, queries, opts):
    import torch
    dev = torch.device("cuda", 0)
    q = torch.from_numpy(queries).to(dev)
    nq, k = queries.shape[0], opts.top_k
    c = shards[0].candidate_count(opts)
    assert c > 0
    cands = []
    for idx in shards:
        keys = torch.zeros((nq, c), dtype=torch.int64, device=dev)
        ranks = torch.zeros((nq, c), dtype=torch.float32, device=dev)
        counts = torch.zeros((nq,), dtype=torch.int32, device=dev)
        idx.candidates_device(q.data_ptr(), nq, opts, keys.data_ptr(), ranks.data_ptr(),
                              counts.data_ptr())
        torch.cuda.synchronize()
        cands.append((keys.cpu().numpy().view(np.uint64), ranks.cpu().numpy(),
                      counts.cpu().numpy()))
    ck, _, cc = _merge(oracle, L2, c, cands)   # ranks: lower is better
    d_ck = torch.from_numpy(ck.view(np.int64)).to(dev)
    d_cc = torch.from_numpy(cc).to(dev)
    refined = []
    for idx in shards:
        keys = torch.zeros((nq, k), dtype=torch.int64, device=dev)
        scores = torch.zeros((nq, k), dtype=torch.float32, device=dev)
        counts = torch.zeros((nq,), dtype=torch.int32, device=dev)
        idx.refine_device(q.data_ptr(), nq, d_ck.data_ptr(), c, d_cc.data_ptr(), k, opts.radius,
                          keys.data_ptr(), scores.data_ptr(), counts.data_ptr())
        torch.cuda.synchronize()
        refined.append((keys.cpu().numpy().view(np.uint64), scores.cpu().numpy(),
                        counts.cpu().numpy()))
    return _merge(oracle, metric, k, refined)


def _compare(got, ok, os_, oc, ost):
    keys, scores, counts = got
    for q in range(ok.shape[0]):
        if ost[q] != 0:
            assert counts[q] == -int(ost[q]), q
            continue
        c = int(oc[q])
        assert counts[q] == c, (q, counts[q], c)
        assert np.array_equal(keys[q, :c], ok[q, :c]), q
        assert np.array_equal(scores[q, :c].view(np.uint32), os_[q, :c].view(np.uint32)), q


@pytest.mark.parametrize("metric,scale,radius", [(IP, 4.0, 0.0), (L2, 1.0, 0.0), (L2, 2.0, 30.0)])
def test_sq8_two_shards(oracle, xb, metric, scale, radius):
    rng = np.random.default_rng(60 + metric)
    n, d = 6000, 64
    s = rng.uniform(0.5, 2.0, d).astype(np.float32)
    rows = (rng.standard_normal((n, d)) * s).astype(np.float32)
    rows[4000] = rows[12]                      # a tie across the shards
    keys = rng.permutation(1 << 20)[:n].astype(np.uint64)
    queries = (rng.standard_normal((37, d)) * s).astype(np.float32)
    queries[5, 2] = np.inf                     # rejected on every shard
    opts = xb.SearchOptions(top_k=10, refine_scale=scale, radius=radius)
    shards = []
    for b, e in ((0, 2500), (2500, n)):
        idx = xb.ScalarQuantizedFlatIndex(d, metric)
        idx.add(keys[b:e], rows[b:e])
        shards.append(idx)
    got = _two_shard_refined(xb, oracle, shards, metric, queries, opts)
    codes, params = oracle.quantize_int8_batch(rows)
    _, ok, os_, oc, ost = oracle.sq8_search(metric, codes, params, rows, keys, queries, 10, radius,
                                            scale)
    _compare(got, ok, os_, oc, ost)
    whole = xb.ScalarQuantizedFlatIndex(d, metric)
    whole.add(keys, rows)
    res = whole.search_with_options(queries, opts, raise_on_error=False)
    _compare((res.keys, res.scores, res.counts), ok, os_, oc, ost)
    for idx in shards + [whole]:
        idx.close()


@pytest.mark.parametrize("metric", [L2, IP])
def test_rabitq_two_shards(oracle, xb, metric):
    rng = np.random.default_rng(80 + metric)
    n, d = 5000, 128
    centers = rng.standard_normal((30, d)).astype(np.float32)
    rows = (centers[rng.integers(0, 30, n)] + 0.3 * rng.standard_normal((n, d))).astype(np.float32)
    keys = rng.permutation(1 << 20)[:n].astype(np.uint64)
    queries = (centers[rng.integers(0, 30, 29)] + 0.3 * rng.standard_normal((29, d))).astype(
        np.float32)
    cents = (centers[:8] + 0.1).astype(np.float32)
    padded = (d + 63) // 64 * 64
    signs = rng.integers(0, 256, 4 * padded // 8, dtype=np.uint8)
    opts = xb.SearchOptions(top_k=10, ef=20, refine=True)
    shards = []
    for b, e in ((0, 1800), (1800, n)):
        idx = xb.RaBitQIndex(d, metric)
        idx.set_model(cents, signs)
        idx.add(keys[b:e], rows[b:e])
        shards.append(idx)
    got = _two_shard_refined(xb, oracle, shards, metric, queries, opts)
    codes, factors = oracle.rabitq_encode1_batch(metric, cents, signs, rows)
    _, ok, os_, oc, ost = oracle.rabitq_search(metric, cents, signs, codes, factors, rows, keys,
                                               queries, 10, 20, refine=True)
    _compare(got, ok, os_, oc, ost)
    for idx in shards:
        idx.close()


def test_refine_skips_keys_it_does_not_hold(xb):
    import torch
    rows = np.eye(70, 64, dtype=np.float32)
    keys = np.arange(100, 170, dtype=np.uint64)
    idx = xb.DenseFlatIndex(64, L2)
    idx.add(keys, rows)
    dev = torch.device("cuda", 0)
    q = torch.from_numpy(rows[:2].copy()).to(dev)
    cand = torch.tensor([[100, 5, 101, 999], [7, 8, 9, 169]], dtype=torch.int64, device=dev)
    cc = torch.tensor([4, 4], dtype=torch.int32, device=dev)
    ok = torch.zeros((2, 3), dtype=torch.int64, device=dev)
    os_ = torch.zeros((2, 3), dtype=torch.float32, device=dev)
    oc = torch.zeros((2,), dtype=torch.int32, device=dev)
    idx.refine_device(q.data_ptr(), 2, cand.data_ptr(), 4, cc.data_ptr(), 3, 0.0, ok.data_ptr(),
                      os_.data_ptr(), oc.data_ptr())
    torch.cuda.synchronize()
    assert oc.tolist() == [2, 1]
    assert ok[0, :2].tolist() == [100, 101] and ok[1, 0].item() == 169
    # Key 169 is row 69, a zero row (np.eye(70, 64)): distance 1 from e1.
    assert os_[0, :2].tolist() == [0.0, 2.0] and os_[1, 0].item() == 1.0
    idx.close()
