"""Multi-rank search host logic on the CPU (world size 2, gloo).

Each rank takes its shard of the rows (shard_range), searches it (here the
oracle stands in for the per-GPU search, so the test runs without a GPU),
the per-shard lists are exchanged with the same all-gather the GPU path uses
(exchange), and every rank merges them with MergeSearchResults
(query.go:154-191).  The merged lists must equal a search over all rows, on
every rank."""
import multiprocessing as mp
import os
import socket

import numpy as np
import pytest

from oracle.oracle import COSINE, IP, L2


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _data(n, nq, d, seed):
    rng = np.random.default_rng(seed)
    rows = rng.standard_normal((n, d)).astype(np.float32)
    rows[n // 2 + 3] = rows[7]  # a tie across the two shards
    keys = rng.permutation(10 * n)[:n].astype(np.uint64)
    queries = rng.standard_normal((nq, d)).astype(np.float32)
    queries[2, 0] = np.nan      # a query every shard rejects
    return rows, keys, queries


def _worker(rank, world, port, metric, n, nq, d, k, out):
    import datetime

    import torch
    import torch.distributed as dist

    from oracle.oracle import Oracle
    from xvec_b200.sharded import exchange, shard_range

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        rows, keys, queries = _data(n, nq, d, seed=metric)
        b, e = shard_range(n, rank, world, align=64)
        ora = Oracle()
        _, ok, os_, oc, ost = ora.flat_search(metric, rows[b:e], keys[b:e], queries, k, threads=2)
        counts = np.where(ost != 0, -ost, oc).astype(np.int32)
        all_k, all_s, all_c = exchange(torch.from_numpy(ok.view(np.int64).copy()),
                                       torch.from_numpy(os_.copy()), torch.from_numpy(counts))
        all_k = all_k.numpy().view(np.uint64)
        all_s, all_c = all_s.numpy(), all_c.numpy()
        merged = []
        for q in range(nq):
            cs = all_c[:, q]
            if (cs < 0).any():
                merged.append(("error", int(cs[cs < 0][0])))
                continue
            mk = np.concatenate([all_k[p, q, :cs[p]] for p in range(world)])
            ms = np.concatenate([all_s[p, q, :cs[p]] for p in range(world)])
            rk, rs = ora.merge_results(metric, k, mk, ms)
            merged.append((rk.tolist(), rs.view(np.uint32).tolist()))
        out.put((rank, (b, e), merged))
    finally:
        dist.destroy_process_group()


def test_shard_range_partitions_rows():
    from xvec_b200.sharded import shard_range
    for n in (0, 1, 63, 64, 1000, 250_001):
        for world in (1, 2, 3, 8):
            spans = [shard_range(n, r, world, align=64) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            for (b0, e0), (b1, _) in zip(spans, spans[1:]):
                assert e0 == b1
            for b, e in spans:  # trailing shards past the data are empty
                assert b == e == n or (b % 64 == 0 and ((e - b) % 64 == 0 or e == n))


@pytest.mark.parametrize("metric", [L2, IP, COSINE])
def test_two_rank_exchange_and_merge_equal_full_search(oracle, metric):
    n, nq, d, k, world = 3000, 9, 24, 17, 2
    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, metric, n, nq, d, k, out))
             for r in range(world)]
    for p in procs:
        p.start()
    import queue
    import time
    results, deadline = [], time.time() + 300
    while len(results) < world:
        try:
            results.append(out.get(timeout=2))
        except queue.Empty:
            assert time.time() < deadline, "ranks did not finish"
            assert all(p.is_alive() or p.exitcode == 0 for p in procs), "a rank failed"
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    rows, keys, queries = _data(n, nq, d, seed=metric)
    _, ok, os_, oc, ost = oracle.flat_search(metric, rows, keys, queries, k)
    spans = sorted(r[1] for r in results)
    assert spans[0][0] == 0 and spans[-1][1] == n and spans[0][1] == spans[1][0]
    for _, _, merged in results:
        for q in range(nq):
            if ost[q] != 0:
                assert merged[q] == ("error", -int(ost[q]))
                continue
            c = int(oc[q])
            mk, ms = merged[q]
            assert mk == ok[q, :c].tolist()
            assert ms == os_[q, :c].view(np.uint32).tolist()
