"""Flat search at a base of more than a million rows and a batch of 1,024
queries: parity with the oracle where the scan takes its full launch
sequence.

At n >= 2^20 rows the tensor-core scan runs two seeding launches (the
first 1/256 and then 1/16 of the rows, each followed by the per-query
threshold reduction) before the main launch over the rest, and the per-part
candidate lists of the seeding launches saturate.  One query equals a row
planted at 600 consecutive positions under different keys: its 100 best keys
tie on the score and fall into one row part, more than its candidate lists
hold, so the coverage check sends it to the exact (reference-order) scan.  Every query of the batch runs through the
GPU; the oracle (a scalar restatement) checks a sample of 64 of them plus
the planted one, since all 1,024 would take it minutes.  Keys identical,
scores bit-identical (topk.go:105-166, query.go:154-191)."""
import numpy as np
import pytest

from oracle.oracle import COSINE, IP, L2

pytestmark = pytest.mark.gpu

N, D, NQ, K = 1_200_000, 64, 1024, 100


@pytest.fixture(scope="module")
def xb():
    import xvec_b200
    assert xvec_b200.device_count() >= 1
    return xvec_b200


def mixture(rng, n, d, clusters=200, sigma=0.3, normalise=True):
    centers = rng.standard_normal((clusters, d)).astype(np.float32)
    x = centers[rng.integers(0, clusters, n)]
    x += sigma * rng.standard_normal((n, d), dtype=np.float32)
    if normalise:
        x /= np.linalg.norm(x, axis=1, keepdims=True)
    return x


def base(seed, normalise):
    rng = np.random.default_rng(seed)
    rows = mixture(rng, N, D, normalise=normalise)
    # 600 consecutive positions (at least 300 inside one row part of the main
    # launch), so that a candidate list receives more tied keys than it holds.
    planted = np.arange(700_000, 700_600)
    # Unnormalised bases plant a row of three times the norm, so that under
    # inner product too its copies are the query's best results.
    rows[planted] = rows[planted[0]] * (1.0 if normalise else 3.0)
    # Distinct keys in shuffled order (an odd multiplier is a bijection mod 2^40).
    keys = (rng.permutation(N).astype(np.uint64) * np.uint64(0x9E3779B1)) & np.uint64((1 << 40) - 1)
    queries = mixture(rng, NQ, D, normalise=normalise)
    queries[517] = rows[planted[0]]
    return rows, keys, queries


def check(oracle, xb, res, metric, rows, keys, queries):
    sample = np.unique(np.concatenate([np.linspace(0, NQ - 1, 64).astype(np.int64), [517]]))
    st, ok, os_, oc, _ = oracle.flat_search(metric, rows, keys, queries[sample], K)
    assert st == 0
    for i, q in enumerate(sample):
        c = int(oc[i])
        assert int(res.counts[q]) == c, q
        assert np.array_equal(res.keys[q, :c], ok[i, :c]), q
        assert np.array_equal(res.scores[q, :c].view(np.uint32), os_[i, :c].view(np.uint32)), q
    # The planted query's 100 results are 100 of the 600 identical rows.
    assert len(np.unique(res.scores[517, :K])) == 1


def test_large_fp16_cosine_launch_sequence(oracle, xb):
    rows, keys, queries = base(11, True)
    r16, q16 = rows.astype(np.float16), queries.astype(np.float16)
    idx = xb.DenseFlatIndex(D, COSINE, xb.STORAGE_FP16)
    idx.add(keys, r16.view(np.uint16))
    xb.reset_stats()
    res = idx.search_with_options(q16.view(np.uint16), xb.SearchOptions(top_k=K))
    st = xb.stats()
    idx.close()
    assert st["tensor_scans"] == 1
    assert st["exact_queries"] >= 1, "the planted query did not take the exact scan"
    # prep, 2 x (seeding scan + threshold), main scan, merge, exact scan and
    # its merge, status: at least 9 launches of this library.
    assert st["kernel_launches"] >= 9
    check(oracle, xb, res, COSINE, r16.astype(np.float32), keys, q16.astype(np.float32))


@pytest.mark.parametrize("metric", [L2, IP])
def test_large_fp32_split_launch_sequence(oracle, xb, metric):
    rows, keys, queries = base(20 + metric, False)
    idx = xb.DenseFlatIndex(D, metric, xb.STORAGE_FP32)
    idx.add(keys, rows)
    xb.reset_stats()
    res = idx.search_with_options(queries, xb.SearchOptions(top_k=K))
    st = xb.stats()
    idx.close()
    assert st["tensor_scans"] == 1
    assert st["exact_queries"] >= 1
    check(oracle, xb, res, metric, rows, keys, queries)
