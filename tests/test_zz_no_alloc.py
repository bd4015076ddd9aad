"""The no-allocation Flat search entry point (xvec_gpu_index_search_noalloc).

Some callers cannot allocate device memory while they search: a process that
plans a fixed device-memory budget up front, or a latency-critical caller
that must not enter the CUDA allocator.  For them the library offers a Flat
search whose per-call scratch lives in one preallocated device array.  This
file checks, through the C ABI, that it returns exactly what the regular
device search returns, and what the oracle returns, on two calls in a row
(the array keeps the previous call's contents, so the second call also
checks that it is cleared); that those calls allocate nothing (the device's
free memory and the stream-ordered pool's high-water mark of used bytes stay
put, while a regular search does use the pool); that its exact-pass fallback
gives the oracle's results; and that oversized requests are refused.  The
file is named to be collected last."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

COSINE, L2 = 3, 1


def _pool():
    from cuda.bindings import runtime as cudart
    err, pool = cudart.cudaDeviceGetDefaultMemPool(0)
    assert err == cudart.cudaError_t.cudaSuccess
    return cudart, pool


def _reset_pool_high_water():
    from cuda.bindings import driver
    cudart, pool = _pool()
    attr = cudart.cudaMemPoolAttr.cudaMemPoolAttrUsedMemHigh
    (err,) = cudart.cudaMemPoolSetAttribute(pool, attr, driver.cuuint64_t(0))
    assert err == cudart.cudaError_t.cudaSuccess


def _pool_high_water():
    cudart, pool = _pool()
    err, v = cudart.cudaMemPoolGetAttribute(
        pool, cudart.cudaMemPoolAttr.cudaMemPoolAttrUsedMemHigh)
    assert err == cudart.cudaError_t.cudaSuccess
    return int(v)


@pytest.fixture(scope="module")
def xb():
    import xvec_b200
    assert xvec_b200.device_count() >= 1
    return xvec_b200


def _search_both(xb, idx, q, k):
    import torch
    nq = q.shape[0]
    outs = []
    for variant in ("regular", "noalloc", "noalloc"):
        keys = torch.full((nq * k,), -1, dtype=torch.int64, device="cuda")
        scores = torch.full((nq * k,), float("nan"), dtype=torch.float32, device="cuda")
        counts = torch.full((nq,), -99, dtype=torch.int32, device="cuda")
        opts = xb.SearchOptions(top_k=k)
        fn = idx.search_device if variant == "regular" else idx.search_device_noalloc
        fn(q.data_ptr(), nq, opts, keys.data_ptr(), scores.data_ptr(), counts.data_ptr())
        torch.cuda.synchronize()
        c = counts.cpu().numpy()
        kk = keys.view(nq, k).cpu().numpy()
        ss = scores.view(nq, k).cpu().numpy()
        outs.append((c, [kk[i, :c[i]] for i in range(nq)], [ss[i, :c[i]] for i in range(nq)]))
    return outs


def _assert_same(outs):
    base = outs[0]
    for other in outs[1:]:
        assert np.array_equal(base[0], other[0])
        for a, b in zip(base[1], other[1]):
            assert np.array_equal(a, b)
        for a, b in zip(base[2], other[2]):
            assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


def test_noalloc_matches_regular_search_fp32(xb):
    import torch
    g = torch.Generator(device="cuda").manual_seed(17)
    n, d = 20000, 128
    rows = torch.randn(n, d, device="cuda", generator=g)
    keys = torch.randperm(10 * n, device="cuda", generator=g)[:n].to(torch.int64)
    idx = xb.DenseFlatIndex(d, L2)
    idx.add_device(keys.data_ptr(), rows.data_ptr(), n)
    q = torch.randn(300, d, device="cuda", generator=g)
    _assert_same(_search_both(xb, idx, q, 10))


def test_noalloc_matches_regular_search_fp16_cosine(xb):
    import torch
    g = torch.Generator(device="cuda").manual_seed(23)
    n, d = 30000, 256
    rows = torch.randn(n, d, device="cuda", generator=g)
    rows = (rows / rows.norm(dim=1, keepdim=True)).half()
    keys = torch.arange(n, device="cuda", dtype=torch.int64)
    idx = xb.DenseFlatIndex(d, COSINE, xb.STORAGE_FP16)
    idx.add_device(keys.data_ptr(), rows.data_ptr(), n)
    q = rows[torch.randint(0, n, (257,), device="cuda", generator=g)].contiguous()
    _assert_same(_search_both(xb, idx, q, 100))


def test_noalloc_refuses_oversized_requests(xb):
    import torch
    idx = xb.DenseFlatIndex(64, L2)
    rows = torch.randn(1000, 64, device="cuda")
    keys = torch.arange(1000, device="cuda", dtype=torch.int64)
    idx.add_device(keys.data_ptr(), rows.data_ptr(), 1000)
    out_k = torch.empty(5000 * 101, dtype=torch.int64, device="cuda")
    out_s = torch.empty(5000 * 101, dtype=torch.float32, device="cuda")
    out_c = torch.empty(5000, dtype=torch.int32, device="cuda")
    q = torch.randn(5000, 64, device="cuda")
    with pytest.raises(xb.XvecGPUError) as e:
        idx.search_device_noalloc(q.data_ptr(), 5000, xb.SearchOptions(top_k=10),
                                  out_k.data_ptr(), out_s.data_ptr(), out_c.data_ptr())
    assert e.value.status == xb.INVALID_ARGUMENT and "4096" in str(e.value)
    with pytest.raises(xb.XvecGPUError) as e:
        idx.search_device_noalloc(q.data_ptr(), 10, xb.SearchOptions(top_k=101),
                                  out_k.data_ptr(), out_s.data_ptr(), out_c.data_ptr())
    assert e.value.status == xb.INVALID_ARGUMENT
    big = torch.randn(4096, 64, device="cuda")
    wide = xb.DenseFlatIndex(4096, L2)
    wrows = torch.randn(64, 4096, device="cuda")
    wide.add_device(keys[:64].data_ptr(), wrows.data_ptr(), 64)
    wq = torch.randn(4096, 4096, device="cuda")
    with pytest.raises(xb.XvecGPUError) as e:
        wide.search_device_noalloc(wq.data_ptr(), 4096, xb.SearchOptions(top_k=10),
                                   out_k.data_ptr(), out_s.data_ptr(), out_c.data_ptr())
    assert e.value.status == xb.INVALID_ARGUMENT and "scratch" in str(e.value)
    del big


def _oracle_check(oracle, out, rows, keys, queries, metric, k):
    _, ok, os_, oc, _ = oracle.flat_search(metric, rows, keys, queries, k)
    counts, klists, slists = out
    assert np.array_equal(counts, oc)
    for q in range(len(counts)):
        assert np.array_equal(klists[q].view(np.uint64), ok[q, :oc[q]]), q
        assert np.array_equal(slists[q].view(np.uint32), os_[q, :oc[q]].view(np.uint32)), q


def test_noalloc_allocates_nothing_and_equals_the_oracle(oracle, xb):
    """Two calls in a row allocate nothing (after the first call on the
    device, which loads the library's device code with the array) and both
    equal the oracle; a regular search, for contrast, uses the pool."""
    import torch
    rng = np.random.default_rng(31)
    n, d, nq, k = 12000, 96, 200, 10
    rows = rng.standard_normal((n, d)).astype(np.float32)
    keys = rng.permutation(1 << 22)[:n].astype(np.uint64)
    queries = rng.standard_normal((nq, d)).astype(np.float32)
    idx = xb.DenseFlatIndex(d, L2)
    idx.add(keys, rows)
    q = torch.from_numpy(queries).cuda()
    out_k = torch.empty(nq * k, dtype=torch.int64, device="cuda")
    out_s = torch.empty(nq * k, dtype=torch.float32, device="cuda")
    out_c = torch.empty(nq, dtype=torch.int32, device="cuda")
    opts = xb.SearchOptions(top_k=k)

    def call(fn):
        out_k.fill_(-1)
        out_s.fill_(float("nan"))
        out_c.fill_(-99)
        torch.cuda.synchronize()
        fn(q.data_ptr(), nq, opts, out_k.data_ptr(), out_s.data_ptr(), out_c.data_ptr())
        torch.cuda.synchronize()
        c = out_c.cpu().numpy()
        kk = out_k.view(nq, k).cpu().numpy()
        ss = out_s.view(nq, k).cpu().numpy()
        return c, [kk[i, :c[i]] for i in range(nq)], [ss[i, :c[i]] for i in range(nq)]

    call(idx.search_device_noalloc)      # set-up on this device
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info()[0]
    _reset_pool_high_water()
    outs = [call(idx.search_device_noalloc), call(idx.search_device_noalloc)]
    assert _pool_high_water() == 0, "the no-allocation search used the stream-ordered pool"
    # Free device memory may grow (a pool trims what earlier tests left at a
    # synchronisation) but never shrinks across the calls.
    assert torch.cuda.mem_get_info()[0] >= free0
    for out in outs:
        _oracle_check(oracle, out, rows, keys, queries, L2, k)
    _reset_pool_high_water()
    call(idx.search_device)
    assert _pool_high_water() > 0, "contrast: the regular search takes pool memory"
    idx.close()


def test_noalloc_exact_pass_fallback(oracle, xb):
    """A query equal to a row planted at 600 consecutive positions under
    different keys: its 100 best results tie and fall into one row part of
    the scan, more than that part's candidate list holds, so the coverage
    check sends the query to the exact pass, which runs in the array too."""
    import torch
    rng = np.random.default_rng(37)
    n, d, k = 9000, 64, 100
    rows = rng.standard_normal((n, d)).astype(np.float32)
    planted = np.arange(3000, 3600)
    rows[planted] = rows[planted[0]]
    keys = rng.permutation(1 << 22)[:n].astype(np.uint64)
    queries = rng.standard_normal((40, d)).astype(np.float32)
    queries[11] = rows[planted[0]]
    idx = xb.DenseFlatIndex(d, L2)
    idx.add(keys, rows)
    q = torch.from_numpy(queries).cuda()
    nq = queries.shape[0]
    for _ in range(2):
        out_k = torch.full((nq * k,), -1, dtype=torch.int64, device="cuda")
        out_s = torch.full((nq * k,), float("nan"), dtype=torch.float32, device="cuda")
        out_c = torch.full((nq,), -99, dtype=torch.int32, device="cuda")
        xb.reset_stats()
        idx.search_device_noalloc(q.data_ptr(), nq, xb.SearchOptions(top_k=k), out_k.data_ptr(),
                                  out_s.data_ptr(), out_c.data_ptr())
        torch.cuda.synchronize()
        assert xb.stats()["exact_queries"] >= 1
        c = out_c.cpu().numpy()
        kk = out_k.view(nq, k).cpu().numpy()
        ss = out_s.view(nq, k).cpu().numpy()
        _oracle_check(oracle, (c, [kk[i, :c[i]] for i in range(nq)],
                               [ss[i, :c[i]] for i in range(nq)]), rows, keys, queries, L2, k)
    idx.close()


def test_noalloc_honours_the_cancel_flag(xb):
    import torch
    idx = xb.DenseFlatIndex(32, L2)
    rows = torch.randn(500, 32, device="cuda")
    keys = torch.arange(500, device="cuda", dtype=torch.int64)
    idx.add_device(keys.data_ptr(), rows.data_ptr(), 500)
    flag = np.ones(1, np.int32)
    o = idx._opts(xb.SearchOptions(top_k=5), cancel_flag=flag.ctypes.data)
    out_k = torch.empty(50, dtype=torch.int64, device="cuda")
    out_s = torch.empty(50, dtype=torch.float32, device="cuda")
    out_c = torch.empty(10, dtype=torch.int32, device="cuda")
    import ctypes
    st = xb.library().xvec_gpu_index_search_noalloc(idx._h, rows.data_ptr(), 10, ctypes.byref(o),
                                                    out_k.data_ptr(), out_s.data_ptr(),
                                                    out_c.data_ptr())
    assert st == xb.CANCELLED
    idx.close()
