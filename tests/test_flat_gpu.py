"""Flat search parity: the CUDA path (through the C ABI) against the oracle.

Scores must be bit-identical (the library rescores candidates in the
reference's float32 accumulation order) and the key lists identical."""
import json
import os

import numpy as np
import pytest

from oracle.oracle import COSINE, IP, L2, MIPSL2, NON_FINITE as O_NON_FINITE

pytestmark = pytest.mark.gpu

FIX = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "reference_fixtures.json")))
METRICS = (L2, IP, COSINE, MIPSL2)


@pytest.fixture(scope="module")
def xb():
    import xvec_b200
    assert xvec_b200.device_count() >= 1, "no sm_100 device"
    return xvec_b200


def _check_against_oracle(oracle, xb, metric, rows, keys, queries, k, radius=0.0, bitmap=None,
                          storage=None):
    storage = storage or xb.STORAGE_FP32
    idx = xb.DenseFlatIndex(rows.shape[1], metric, storage)
    if storage == xb.STORAGE_FP16:
        idx.add(keys, rows.astype(np.float16).view(np.uint16))
        rows32 = rows.astype(np.float16).astype(np.float32)
        q_in = queries.astype(np.float16).view(np.uint16)
        q32 = queries.astype(np.float16).astype(np.float32)
    else:
        idx.add(keys, rows)
        rows32, q_in, q32 = rows, queries, queries
    res = idx.search_with_options(q_in, xb.SearchOptions(top_k=k, radius=radius, filter=bitmap),
                                  raise_on_error=False)
    st, ok, os_, oc, ost = oracle.flat_search(metric, rows32, keys, q32, k, radius, bitmap)
    for q in range(queries.shape[0]):
        if ost[q] != 0:
            assert res.counts[q] < 0, q
            continue
        c = int(oc[q])
        assert int(res.counts[q]) == c, (metric, q, res.counts[q], c)
        assert np.array_equal(res.keys[q, :c], ok[q, :c]), (metric, q)
        assert np.array_equal(res.scores[q, :c].view(np.uint32), os_[q, :c].view(np.uint32)), \
            (metric, q, res.scores[q, :c], os_[q, :c])
    idx.close()


def test_reference_fixture(xb):
    f = FIX["flat_metrics"]
    keys = np.array([c[0] for c in f["candidates"]], np.uint64)
    rows = np.array([c[1] for c in f["candidates"]], np.float32)
    for metric, want in f["want"].items():
        idx = xb.DenseFlatIndex(2, int(metric))
        idx.add(keys, rows)
        res = idx.search(np.array([f["query"]], np.float32), f["k"])
        assert res.query(0) == [tuple(w) for w in want], metric


@pytest.mark.parametrize("d", [1, 3, 7, 8, 12, 16, 17, 31, 128, 129, 768])
@pytest.mark.parametrize("metric", METRICS)
def test_random_parity(oracle, xb, metric, d):
    rng = np.random.default_rng(1000 + d * 7 + metric)
    n = 3000 if d < 700 else 1200
    rows = rng.standard_normal((n, d)).astype(np.float32)
    keys = rng.permutation(10 * n)[:n].astype(np.uint64)
    queries = rng.standard_normal((19, d)).astype(np.float32)
    for k in (1, 10, 100):
        _check_against_oracle(oracle, xb, metric, rows, keys, queries, k)


@pytest.mark.parametrize("metric", METRICS)
def test_fp16_storage_parity(oracle, xb, metric):
    rng = np.random.default_rng(77 + metric)
    centers = rng.standard_normal((20, 64)).astype(np.float32)
    rows = centers[rng.integers(0, 20, 2500)] + 0.3 * rng.standard_normal((2500, 64)).astype(np.float32)
    rows /= np.linalg.norm(rows, axis=1, keepdims=True)
    queries = centers[rng.integers(0, 20, 23)] + 0.3 * rng.standard_normal((23, 64)).astype(np.float32)
    keys = np.arange(2500, dtype=np.uint64)
    _check_against_oracle(oracle, xb, metric, rows, keys, queries, 100, storage=xb.STORAGE_FP16)


def test_duplicate_rows_tie_break_by_key(oracle, xb):
    rng = np.random.default_rng(5)
    base = rng.standard_normal((50, 24)).astype(np.float32)
    rows = np.concatenate([base] * 8)  # every score appears 8 times
    keys = rng.permutation(100000)[:400].astype(np.uint64)
    queries = base[:5].copy()
    for metric in METRICS:
        _check_against_oracle(oracle, xb, metric, rows, keys, queries, 37)


def test_filter_radius_and_small_n(oracle, xb):
    rng = np.random.default_rng(11)
    rows = rng.standard_normal((700, 40)).astype(np.float32)
    keys = np.arange(700, dtype=np.uint64) * 3 + 1
    queries = rng.standard_normal((9, 40)).astype(np.float32)
    bitmap = np.zeros((700 + 31) // 32, np.uint32)
    for p in range(0, 700, 3):
        bitmap[p >> 5] |= np.uint32(1 << (p & 31))
    for metric in METRICS:
        _check_against_oracle(oracle, xb, metric, rows, keys, queries, 25, bitmap=bitmap)
    _check_against_oracle(oracle, xb, L2, rows, keys, queries, 50, radius=60.0)
    _check_against_oracle(oracle, xb, IP, rows, keys, queries, 50, radius=5.0)
    # k larger than the index.
    _check_against_oracle(oracle, xb, L2, rows[:13], keys[:13], queries, 40)


def test_large_k_exact_path(oracle, xb):
    rng = np.random.default_rng(12)
    rows = rng.standard_normal((4000, 33)).astype(np.float32)
    keys = np.arange(4000, dtype=np.uint64)
    queries = rng.standard_normal((4, 33)).astype(np.float32)
    _check_against_oracle(oracle, xb, COSINE, rows, keys, queries, 700)


def test_zero_vectors(oracle, xb):
    rows = np.array([[0, 0, 0], [1, 0, 0], [0, 2, 0], [0, 0, 0]], np.float32)
    keys = np.array([4, 3, 2, 1], np.uint64)
    queries = np.array([[0, 0, 0], [1, 1, 0]], np.float32)
    for metric in METRICS:
        _check_against_oracle(oracle, xb, metric, rows, keys, queries, 4)


def test_errors(oracle, xb):
    idx = xb.DenseFlatIndex(4, IP)
    idx.add(np.array([1, 2], np.uint64), np.ones((2, 4), np.float32))
    with pytest.raises(xb.XvecGPUError) as e:
        idx.add(np.array([2], np.uint64), np.ones((1, 4), np.float32))
    assert e.value.status == xb.DUPLICATE_KEY
    assert len(idx) == 2
    with pytest.raises(xb.XvecGPUError) as e:
        idx.add(np.array([9], np.uint64), np.array([[1, np.nan, 0, 0]], np.float32))
    assert e.value.status == xb.NON_FINITE
    assert len(idx) == 2
    with pytest.raises(xb.XvecGPUError) as e:
        idx.search_with_options(np.ones((1, 4), np.float32), xb.SearchOptions(top_k=0))
    assert e.value.status == xb.INVALID_ARGUMENT
    with pytest.raises(xb.XvecGPUError) as e:
        idx.search_with_options(np.ones((1, 4), np.float32), xb.SearchOptions(top_k=1, radius=-1))
    assert e.value.status == xb.INVALID_ARGUMENT
    # One non-finite query fails alone; the others are answered.
    q = np.ones((3, 4), np.float32)
    q[1, 2] = np.inf
    res = idx.search_with_options(q, xb.SearchOptions(top_k=2), raise_on_error=False)
    assert res.counts[1] == -xb.NON_FINITE and res.counts[0] == 2 and res.counts[2] == 2
    # Empty index.
    empty = xb.DenseFlatIndex(4, L2)
    res = empty.search(np.ones((2, 4), np.float32), 5)
    assert list(res.counts) == [0, 0]


def test_incremental_adds(oracle, xb):
    rng = np.random.default_rng(21)
    rows = rng.standard_normal((1500, 20)).astype(np.float32)
    keys = rng.permutation(5000)[:1500].astype(np.uint64)
    idx = xb.DenseFlatIndex(20, L2)
    for lo in range(0, 1500, 250):
        idx.add(keys[lo:lo + 250], rows[lo:lo + 250])
    queries = rng.standard_normal((7, 20)).astype(np.float32)
    res = idx.search(queries, 15)
    st, ok, os_, oc, _ = oracle.flat_search(L2, rows, keys, queries, 15)
    assert np.array_equal(res.keys, ok) and np.array_equal(res.scores, os_)
