"""The multi-GPU search through the C ABI (xvec_gpu_comm_*,
xvec_gpu_sharded_search_device, xvec_gpu_sharded_search): the library's own
NCCL communicator, one all-gather of a packed buffer per exchange, the
MergeSearchResults order (query.go:154-191) on every rank.

On one GPU a communicator of one rank runs the whole path (shard search,
pack, all-gather, merge): it must equal the oracle and the plain search for
Flat (FP16 cosine, FP32 L2), and the refined kinds (SQ8 Flat, RaBitQ and
SQ-IVF, two exchanges).  A rank whose own search fails as a whole still
takes part and the failure reaches every query.  With two or more GPUs, a
shard per GPU in one process (xvec_gpu_comm_init_all) and in one process per
GPU must equal the oracle over all rows.  A rank that never joins ends the
initialisation with XVEC_GPU_TIMEOUT (the failure made on the host); an
aborted communicator fails later calls."""
import multiprocessing as mp
import os
import subprocess
import sys
import tempfile

import numpy as np
import pytest

from oracle.oracle import COSINE, IP, L2

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def xb():
    import xvec_b200
    assert xvec_b200.device_count() >= 1
    return xvec_b200


def mixture(rng, n, d, clusters=40, normalise=False):
    centers = rng.standard_normal((clusters, d)).astype(np.float32)
    x = (centers[rng.integers(0, clusters, n)]
         + 0.3 * rng.standard_normal((n, d))).astype(np.float32)
    if normalise:
        x /= np.linalg.norm(x, axis=1, keepdims=True)
    return x


def device_search(xb, comm, idx, queries, opts):
    import torch
    dev = torch.device("cuda", idx.device)
    if queries.dtype == np.uint16:
        queries = queries.view(np.int16)
    q = torch.from_numpy(np.ascontiguousarray(queries)).to(dev)
    nq, k = queries.shape[0], opts.top_k
    keys = torch.zeros((nq, k), dtype=torch.int64, device=dev)
    scores = torch.zeros((nq, k), dtype=torch.float32, device=dev)
    counts = torch.zeros((nq,), dtype=torch.int32, device=dev)
    status = 0
    try:
        xb.sharded_search_device(comm, idx, q.data_ptr(), nq, opts, keys.data_ptr(),
                                 scores.data_ptr(), counts.data_ptr(),
                                 stream=torch.cuda.current_stream(dev).cuda_stream)
    except xb.XvecGPUError as e:
        status = e.status
    torch.cuda.synchronize(dev)
    return (keys.cpu().numpy().view(np.uint64), scores.cpu().numpy(), counts.cpu().numpy(),
            status)


def same(got, ref):
    gk, gs, gc = got[:3]
    rk, rs, rc = ref[:3]
    assert np.array_equal(gc, rc)
    for q in range(gc.shape[0]):
        c = int(gc[q])
        if c <= 0:
            continue
        assert np.array_equal(gk[q, :c], rk[q, :c]), q
        assert np.array_equal(gs[q, :c].view(np.uint32), rs[q, :c].view(np.uint32)), q


def oracle_counts(oc, ost):
    return np.where(ost != 0, -ost, oc).astype(np.int32)


def test_one_rank_flat_fp16_cosine(oracle, xb):
    rng = np.random.default_rng(5)
    rows = mixture(rng, 20000, 128, normalise=True).astype(np.float16)
    keys = rng.permutation(1 << 24)[:20000].astype(np.uint64)
    queries = mixture(rng, 300, 128, normalise=True).astype(np.float16)
    queries[7, 3] = np.nan                          # fails on its own
    idx = xb.DenseFlatIndex(128, COSINE, xb.STORAGE_FP16)
    idx.add(keys, rows.view(np.uint16))
    comm = xb.Comm.init_rank(0, xb.Comm.unique_id(), 1, 0)
    assert (comm.size, comm.rank) == (1, 0)
    opts = xb.SearchOptions(top_k=50)
    got = device_search(xb, comm, idx, queries.view(np.uint16), opts)
    assert got[3] == xb.NON_FINITE and got[2][7] == -xb.NON_FINITE
    _, ok, os_, oc, ost = oracle.flat_search(COSINE, rows.astype(np.float32), keys,
                                             queries.astype(np.float32), 50)
    same(got, (ok, os_, oracle_counts(oc, ost)))
    plain = idx.search_with_options(queries.view(np.uint16), opts, raise_on_error=False)
    same(got, (plain.keys, plain.scores, plain.counts))
    comm.close()
    idx.close()


def test_one_rank_init_all_host_api(oracle, xb):
    rng = np.random.default_rng(6)
    rows = mixture(rng, 9000, 96)
    keys = rng.permutation(1 << 24)[:9000].astype(np.uint64)
    queries = mixture(rng, 150, 96)
    idx = xb.DenseFlatIndex(96, L2)
    idx.add(keys, rows)
    comms = xb.Comm.init_all([0])
    res = xb.sharded_search(comms, [idx], queries, xb.SearchOptions(top_k=10))
    _, ok, os_, oc, ost = oracle.flat_search(L2, rows, keys, queries, 10)
    same((res.keys, res.scores, res.counts), (ok, os_, oracle_counts(oc, ost)))
    for c in comms:
        c.close()
    idx.close()


def test_one_rank_refined_sq8(oracle, xb):
    rng = np.random.default_rng(7)
    n, d = 8000, 128
    s = rng.uniform(0.5, 2.0, d).astype(np.float32)
    rows = (rng.standard_normal((n, d)) * s).astype(np.float32)
    keys = rng.permutation(1 << 20)[:n].astype(np.uint64)
    queries = (rng.standard_normal((64, d)) * s).astype(np.float32)
    idx = xb.ScalarQuantizedFlatIndex(d, IP)
    idx.add(keys, rows)
    comm = xb.Comm.init_rank(0, xb.Comm.unique_id(), 1, 0)
    opts = xb.SearchOptions(top_k=10, refine_scale=4.0)
    got = device_search(xb, comm, idx, queries, opts)
    codes, params = oracle.quantize_int8_batch(rows)
    _, ok, os_, oc, ost = oracle.sq8_search(IP, codes, params, rows, keys, queries, 10, 0.0, 4.0)
    same(got, (ok, os_, oracle_counts(oc, ost)))
    comm.close()
    idx.close()


def test_one_rank_refined_rabitq_and_ivf_sq8(oracle, xb):
    rng = np.random.default_rng(8)
    n, d = 6000, 128
    rows = mixture(rng, n, d)
    keys = rng.permutation(1 << 20)[:n].astype(np.uint64)
    queries = mixture(rng, 40, d)
    comm = xb.Comm.init_rank(0, xb.Comm.unique_id(), 1, 0)
    # RaBitQ, two exchanges (estimates, then the exact refine).
    cents = rows[:8] + 0.1
    signs = rng.integers(0, 256, 4 * d // 8, dtype=np.uint8)
    rq = xb.RaBitQIndex(d, L2)
    rq.set_model(cents, signs)
    rq.add(keys, rows)
    opts = xb.SearchOptions(top_k=10, ef=40, refine=True)
    got = device_search(xb, comm, rq, queries, opts)
    codes, factors = oracle.rabitq_encode1_batch(L2, cents, signs, rows)
    _, ok, os_, oc, ost = oracle.rabitq_search(L2, cents, signs, codes, factors, rows, keys,
                                               queries, 10, 40, refine=True)
    same(got, (ok, os_, oracle_counts(oc, ost)))
    # SQ-IVF with a refine scale: its candidates go through the exchange too.
    ivf = xb.ScalarQuantizedIVFIndex(d, L2)
    ivf.set_model(rows[::500].copy())
    ivf.add(keys, rows)
    opts = xb.SearchOptions(top_k=10, nprobe=4, refine_scale=3.0)
    assert ivf.candidate_count(opts) == 30
    got = device_search(xb, comm, ivf, queries, opts)
    plain = ivf.search_with_options(queries, opts)
    same(got, (plain.keys, plain.scores, plain.counts))
    comm.close()
    rq.close()
    ivf.close()


def test_rank_failure_reaches_every_query(xb):
    """An IVF index without a model fails its search as a whole; the rank
    still takes part in the exchange and every query reports the status."""
    ivf = xb.IVFIndex(32, L2)
    comm = xb.Comm.init_rank(0, xb.Comm.unique_id(), 1, 0)
    got = device_search(xb, comm, ivf, np.ones((5, 32), np.float32),
                        xb.SearchOptions(top_k=3, nprobe=2))
    assert got[3] == xb.INVALID_ARGUMENT
    assert (got[2] == -xb.INVALID_ARGUMENT).all()
    # The communicator is still healthy.
    rows = np.eye(40, 32, dtype=np.float32)
    flat = xb.DenseFlatIndex(32, L2)
    flat.add(np.arange(40, dtype=np.uint64), rows)
    got = device_search(xb, comm, flat, rows[:4].copy(), xb.SearchOptions(top_k=1))
    assert got[3] == 0 and got[0][:, 0].tolist() == [0, 1, 2, 3]
    comm.close()
    flat.close()
    ivf.close()


def test_aborted_communicator_fails_later_calls(xb):
    rows = np.eye(40, 32, dtype=np.float32)
    flat = xb.DenseFlatIndex(32, L2)
    flat.add(np.arange(40, dtype=np.uint64), rows)
    comm = xb.Comm.init_rank(0, xb.Comm.unique_id(), 1, 0)
    comm.abort()
    got = device_search(xb, comm, flat, rows[:2].copy(), xb.SearchOptions(top_k=1))
    assert got[3] == 6  # XVEC_GPU_NCCL_ERROR
    assert "aborted" in xb.last_error()
    comm.close()
    flat.close()


NEVER_JOINS = r"""
import sys, time
sys.path.insert(0, sys.argv[1])
import xvec_b200 as xb
uid = xb.Comm.unique_id()
t0 = time.time()
try:
    xb.Comm.init_rank(0, uid, 2, 0, timeout_ms=2000)
    print("status 0")
except xb.XvecGPUError as e:
    print("status", e.status, "after", round(time.time() - t0, 1))
"""


def test_rank_that_never_joins_times_out():
    """Rank 1 of 2 never joins: rank 0's initialisation gives up after its
    2 s bound with XVEC_GPU_TIMEOUT (no GPU work is in flight: the wait is
    NCCL's host-side bootstrap)."""
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    out = subprocess.run([sys.executable, "-c", NEVER_JOINS, ROOT], capture_output=True,
                         text=True, timeout=180, env=env)
    assert "status 4" in out.stdout, out.stdout + out.stderr
    secs = float(out.stdout.split("after")[1])
    assert secs < 30


def shard_data(seed, n, d, metric):
    rng = np.random.default_rng(seed)
    rows = mixture(rng, n, d, normalise=metric == COSINE)
    keys = rng.permutation(1 << 24)[:n].astype(np.uint64)
    queries = mixture(rng, 200, d, normalise=metric == COSINE)
    return rows, keys, queries


@pytest.mark.parametrize("case", ["fp16_cosine", "fp32_l2", "fp16_ip_small_shard",
                                  "fp32_l2_planted"])
def test_two_gpus_one_process(oracle, xb, case):
    """Flat over two shards: each shard rescores only the candidates inside
    the band that every shard's k best fast ranks give (one exchange before
    the merge).  Cases: the tensor-core scans (FP16 cosine, FP32 split L2);
    a shard with fewer rows than k (its ranks padded with +inf); a query
    whose 100 best rows tie on one shard (600 copies of one row in one row
    part: that shard's coverage check sends it to the exact scan)."""
    if xb.device_count() < 2:
        pytest.skip("needs two GPUs")
    n, d, k = 30000, 128, 100
    metric = {"fp16_cosine": COSINE, "fp32_l2": L2, "fp16_ip_small_shard": IP,
              "fp32_l2_planted": L2}[case]
    fp16 = case.startswith("fp16")
    rows, keys, queries = shard_data(21, n, d, metric)
    split = 50 if case == "fp16_ip_small_shard" else 13000
    if case == "fp32_l2_planted":
        rows[20000:20600] = rows[20000]
        queries[5] = rows[20000]
    if fp16:
        rows = rows.astype(np.float16).astype(np.float32)
        queries = queries.astype(np.float16).astype(np.float32)
    shards = []
    for dev, (b, e) in enumerate(((0, split), (split, n))):
        if fp16:
            idx = xb.DenseFlatIndex(d, metric, xb.STORAGE_FP16, device=dev)
            idx.add(keys[b:e], rows[b:e].astype(np.float16).view(np.uint16))
        else:
            idx = xb.DenseFlatIndex(d, metric, device=dev)
            idx.add(keys[b:e], rows[b:e])
        shards.append(idx)
    comms = xb.Comm.init_all([0, 1])
    q_in = queries.astype(np.float16).view(np.uint16) if fp16 else queries
    res = xb.sharded_search(comms, shards, q_in, xb.SearchOptions(top_k=k))
    _, ok, os_, oc, ost = oracle.flat_search(metric, rows, keys, queries, k)
    same((res.keys, res.scores, res.counts), (ok, os_, oracle_counts(oc, ost)))
    if case == "fp32_l2_planted":
        assert len(np.unique(res.scores[5, :k])) == 1
    for c in comms:
        c.close()
    for s in shards:
        s.close()


def _rank_main(rank, world, uid, out_dir, n, d):
    import torch

    import xvec_b200 as xb
    rows, keys, queries = shard_data(22, n, d, L2)
    b, e = rank * n // world, (rank + 1) * n // world
    s = rows.std(axis=0) + 0.5
    idx = xb.ScalarQuantizedFlatIndex(d, L2, device=rank)
    idx.add(keys[b:e], rows[b:e] * s)
    torch.cuda.set_device(rank)
    comm = xb.Comm.init_rank(rank, uid, world, rank, timeout_ms=60000)
    got = device_search(xb, comm, idx, queries * s, xb.SearchOptions(top_k=10, refine_scale=4.0))
    np.savez(os.path.join(out_dir, f"rank{rank}.npz"), keys=got[0], scores=got[1],
             counts=got[2], status=got[3])
    comm.close()
    idx.close()


def test_two_gpus_two_processes_refined(oracle, xb):
    """One process per GPU, the id sent by the parent; a refined SQ8 search
    (two exchanges); every rank holds the merged results."""
    if xb.device_count() < 2:
        pytest.skip("needs two GPUs")
    n, d, world = 20000, 128, 2
    uid = xb.Comm.unique_id()
    ctx = mp.get_context("spawn")
    with tempfile.TemporaryDirectory() as tmp:
        procs = [ctx.Process(target=_rank_main, args=(r, world, uid, tmp, n, d))
                 for r in range(world)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(300)
            assert p.exitcode == 0
        outs = [np.load(os.path.join(tmp, f"rank{r}.npz")) for r in range(world)]
    rows, keys, queries = shard_data(22, n, d, L2)
    s = rows.std(axis=0) + 0.5
    codes, params = oracle.quantize_int8_batch(rows * s)
    _, ok, os_, oc, ost = oracle.sq8_search(L2, codes, params, rows * s, keys, queries * s, 10,
                                            0.0, 4.0)
    for o in outs:
        assert int(o["status"]) == 0
        same((o["keys"], o["scores"], o["counts"]), (ok, os_, oracle_counts(oc, ost)))
