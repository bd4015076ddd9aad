"""The no-allocation Flat search entry point (xvec_gpu_index_search_noalloc).

Some callers cannot allocate device memory while they search: a process that
plans a fixed device-memory budget up front, or a latency-critical caller
that must not enter the CUDA allocator.  For them the library offers a Flat
search whose per-call scratch lives in one preallocated device array.  This
file checks, through the C ABI, that it returns exactly what the regular
device search returns, on two calls in a row (the array keeps the previous
call's contents, so the second call also checks that it is cleared), and that
oversized requests are refused.  The file is named to be collected last."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

COSINE, L2 = 3, 1


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
