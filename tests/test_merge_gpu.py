"""The cross-shard merge kernel (xvec_gpu_merge_results_device) against the
oracle's MergeSearchResults (query.go:154-191): ties by ascending key,
IP higher-is-better, short and empty lists, and a query failed on the shards
(negative count) staying failed."""
import numpy as np
import pytest

from oracle.oracle import COSINE, IP, L2

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("metric", [L2, IP, COSINE])
def test_merge_results_device_matches_oracle(oracle, metric):
    import torch

    import xvec_b200 as xb
    rng = np.random.default_rng(40 + metric)
    parts, nq, k = 3, 25, 15
    keys = np.zeros((parts, nq, k), np.uint64)
    scores = np.zeros((parts, nq, k), np.float32)
    counts = rng.integers(0, k + 1, (parts, nq)).astype(np.int32)
    counts[:, 0] = 0                       # nothing anywhere
    counts[:, 1] = k                       # full lists everywhere
    for q in range(nq):
        pool = rng.permutation(1 << 20)[:parts * k].astype(np.uint64)
        for p in range(parts):
            c = counts[p, q]
            # Each shard's list is sorted best-first, as a search returns it.
            s = np.round(rng.standard_normal(c), 1).astype(np.float32)  # many ties
            kk = pool[p * k:p * k + c]
            order = np.lexsort((kk, -s if metric == IP else s))
            keys[p, q, :c], scores[p, q, :c] = kk[order], s[order]
    counts[:, 5] = -7                      # the query failed (non-finite)
    dev = torch.device("cuda", 0)
    d_keys = torch.from_numpy(keys.view(np.int64)).to(dev)
    d_scores = torch.from_numpy(scores).to(dev)
    d_counts = torch.from_numpy(counts).to(dev)
    ok = torch.zeros((nq, k), dtype=torch.int64, device=dev)
    os_ = torch.zeros((nq, k), dtype=torch.float32, device=dev)
    oc = torch.zeros((nq,), dtype=torch.int32, device=dev)
    xb.merge_results_device(0, metric, k, nq, parts, d_keys.data_ptr(), d_scores.data_ptr(),
                            d_counts.data_ptr(), ok.data_ptr(), os_.data_ptr(), oc.data_ptr())
    torch.cuda.synchronize()
    ok, os_, oc = ok.cpu().numpy().view(np.uint64), os_.cpu().numpy(), oc.cpu().numpy()
    for q in range(nq):
        if q == 5:
            assert oc[q] == -7
            continue
        mk = np.concatenate([keys[p, q, :counts[p, q]] for p in range(parts)])
        ms = np.concatenate([scores[p, q, :counts[p, q]] for p in range(parts)])
        rk, rs = oracle.merge_results(metric, k, mk, ms)
        assert oc[q] == len(rk), q
        assert np.array_equal(ok[q, :oc[q]], rk), q
        assert np.array_equal(os_[q, :oc[q]].view(np.uint32), rs.view(np.uint32)), q


def test_sharded_search_single_rank(oracle):
    """ShardedSearch on one rank is the plain device search."""
    import torch

    import xvec_b200 as xb
    from xvec_b200.sharded import ShardedSearch
    rng = np.random.default_rng(3)
    rows = rng.standard_normal((2000, 64)).astype(np.float32)
    keys = np.arange(2000, dtype=np.uint64) * 5
    queries = rng.standard_normal((11, 64)).astype(np.float32)
    idx = xb.DenseFlatIndex(64, L2)
    idx.add(keys, rows)
    k_, s_, c_ = ShardedSearch(idx).search_device(torch.from_numpy(queries).cuda(),
                                                   xb.SearchOptions(top_k=9))
    _, ok, os_, oc, _ = oracle.flat_search(L2, rows, keys, queries, 9)
    assert np.array_equal(c_.cpu().numpy(), oc)
    assert np.array_equal(k_.cpu().numpy().view(np.uint64), ok)
    assert np.array_equal(s_.cpu().numpy().view(np.uint32), os_.view(np.uint32))
    idx.close()
