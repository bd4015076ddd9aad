"""Failure paths of the GPU search, made without a GPU fault.

* Cancellation: the caller's flag (the reference checks ctx.Err() between
  candidates, internal/core/topk.go:130) set before the call ends the
  search with XVEC_GPU_CANCELLED; cleared, the next search is correct.
* A device wait that runs out: the tensor-core scan's wait bound
  (xvec_gpu_set_wait_limit_ns) set to 1 ns makes its first mbarrier wait
  expire; the kernel stops issuing work, drains the copies it issued, frees
  its tensor memory and the search returns XVEC_GPU_TIMEOUT.  The context
  stays usable: with the default bound restored the same search equals the
  oracle.  Both launch shapes (single CTAs for <= 128 queries, CTA pairs
  above) and the INT8 scan are covered."""
import numpy as np
import pytest

from oracle.oracle import COSINE, IP

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def xb():
    import xvec_b200
    assert xvec_b200.device_count() >= 1
    return xvec_b200


def data(seed, n=20000, d=128, nq=64):
    rng = np.random.default_rng(seed)
    c = rng.standard_normal((30, d)).astype(np.float32)
    rows = c[rng.integers(0, 30, n)] + 0.3 * rng.standard_normal((n, d)).astype(np.float32)
    rows /= np.linalg.norm(rows, axis=1, keepdims=True)
    q = c[rng.integers(0, 30, nq)] + 0.3 * rng.standard_normal((nq, d)).astype(np.float32)
    q /= np.linalg.norm(q, axis=1, keepdims=True)
    return rows.astype(np.float16), rng.permutation(1 << 22)[:n].astype(np.uint64), q.astype(
        np.float16)


def check(oracle, res, rows, keys, queries, k):
    _, ok, os_, oc, _ = oracle.flat_search(COSINE, rows.astype(np.float32), keys,
                                           queries.astype(np.float32), k)
    assert np.array_equal(res.counts, oc)
    assert np.array_equal(res.keys, ok)
    assert np.array_equal(res.scores.view(np.uint32), os_.view(np.uint32))


def test_cancel_flag(oracle, xb):
    rows, keys, queries = data(1)
    idx = xb.DenseFlatIndex(128, COSINE, xb.STORAGE_FP16)
    idx.add(keys, rows.view(np.uint16))
    flag = np.ones(1, np.int32)
    with pytest.raises(xb.XvecGPUError) as e:
        idx.search_with_options(queries.view(np.uint16), xb.SearchOptions(top_k=10),
                                cancel_flag=flag)
    assert e.value.status == xb.CANCELLED
    flag[0] = 0
    res = idx.search_with_options(queries.view(np.uint16), xb.SearchOptions(top_k=10),
                                  cancel_flag=flag)
    check(oracle, res, rows, keys, queries, 10)
    idx.close()


@pytest.mark.parametrize("nq", [64, 300])
def test_expired_device_wait(oracle, xb, nq):
    rows, keys, queries = data(2, nq=nq)
    idx = xb.DenseFlatIndex(128, COSINE, xb.STORAGE_FP16)
    idx.add(keys, rows.view(np.uint16))
    before = xb.set_wait_limit_ns(1)
    try:
        assert before == 2_000_000_000
        with pytest.raises(xb.XvecGPUError) as e:
            idx.search_with_options(queries.view(np.uint16), xb.SearchOptions(top_k=20))
        assert e.value.status == 4  # XVEC_GPU_TIMEOUT
        assert "wait expired" in xb.last_error()
    finally:
        assert xb.set_wait_limit_ns(0) == 1
    res = idx.search_with_options(queries.view(np.uint16), xb.SearchOptions(top_k=20))
    check(oracle, res, rows, keys, queries, 20)
    idx.close()


def test_expired_device_wait_int8_scan(oracle, xb):
    rng = np.random.default_rng(3)
    n, d = 30000, 256
    rows = rng.standard_normal((n, d)).astype(np.float32)
    keys = np.arange(n, dtype=np.uint64)
    queries = rng.standard_normal((200, d)).astype(np.float32)
    idx = xb.ScalarQuantizedFlatIndex(d, IP)
    idx.add(keys, rows)
    xb.set_wait_limit_ns(1)
    try:
        with pytest.raises(xb.XvecGPUError) as e:
            idx.search_with_options(queries, xb.SearchOptions(top_k=10))
        assert e.value.status == 4
    finally:
        xb.set_wait_limit_ns(0)
    res = idx.search_with_options(queries, xb.SearchOptions(top_k=10))
    codes, params = oracle.quantize_int8_batch(rows)
    _, ok, os_, oc, _ = oracle.sq8_search(IP, codes, params, rows, keys, queries, 10)
    assert np.array_equal(res.keys, ok)
    assert np.array_equal(res.scores.view(np.uint32), os_.view(np.uint32))
    idx.close()
