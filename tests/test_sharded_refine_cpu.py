"""Refined searches over shards on the CPU (world size 2, gloo).

RefinedSearch (refiner.go:133-166) refines the RefinementCandidateCount best
approximate results of the whole index.  Over shards, sharded.refined_search
gathers every shard's candidates with their ranks, merges them (ties by
key), has every shard refine the merged candidates it holds, and merges
those results (query.go:154-191).  The oracle stands in for the per-shard
stages (its SQ8 approximate search and its exact Flat search over the
candidate rows), so the test runs without a GPU; the merged result must
equal one refined SQ8 search over all rows, on every rank.  A shard-local
refine (each shard refining its own best candidates) would differ."""
import multiprocessing as mp
import os
import socket

import numpy as np
import pytest

from oracle.oracle import IP, L2

K = 10


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _data(seed, n=3000, nq=12, d=32):
    rng = np.random.default_rng(seed)
    scale = rng.uniform(0.5, 2.0, d).astype(np.float32)
    rows = (rng.standard_normal((n, d)) * scale).astype(np.float32)
    rows[n // 2 + 5] = rows[9]              # a tie across the two shards
    keys = rng.permutation(20 * n)[:n].astype(np.uint64)
    queries = (rng.standard_normal((nq, d)) * scale).astype(np.float32)
    queries[3, 1] = np.nan                  # a query every shard rejects
    return rows, keys, queries


def _merge(ora, metric, kk, all_keys, all_scores, all_counts):
    import torch
    world, nq = all_counts.shape
    keys = np.zeros((nq, kk), np.uint64)
    scores = np.zeros((nq, kk), np.float32)
    counts = np.zeros(nq, np.int32)
    ak = all_keys.numpy().view(np.uint64)
    asc, ac = all_scores.numpy(), all_counts.numpy()
    for q in range(nq):
        cs = ac[:, q]
        if (cs < 0).any():
            counts[q] = cs[cs < 0][0]
            continue
        mk = np.concatenate([ak[p, q, :cs[p]] for p in range(world)])
        ms = np.concatenate([asc[p, q, :cs[p]] for p in range(world)])
        rk, rs = ora.merge_results(metric, kk, mk, ms)
        keys[q, :rk.size], scores[q, :rk.size], counts[q] = rk, rs, rk.size
    return torch.from_numpy(keys.view(np.int64)), torch.from_numpy(scores), torch.from_numpy(counts)


def _worker(rank, world, port, metric, radius, scale, out):
    import datetime

    import torch
    import torch.distributed as dist

    from oracle.oracle import Oracle
    from xvec_b200.sharded import refined_search, shard_range

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        ora = Oracle()
        rows, keys, queries = _data(seed=metric)
        codes, params = ora.quantize_int8_batch(rows)
        b, e = shard_range(rows.shape[0], rank, world, align=64)
        mine = {int(kk): i for i, kk in enumerate(keys[b:e])}
        nq = queries.shape[0]
        C = int(np.floor(K * scale))

        def candidates():
            _, ok, os_, oc, ost = ora.sq8_search(metric, codes[b:e], params[b:e], rows[b:e],
                                                 keys[b:e], queries, C, threads=2)
            ranks = -os_ if metric == IP else os_
            counts = np.where(ost != 0, -ost, oc).astype(np.int32)
            return (torch.from_numpy(ok.view(np.int64).copy()),
                    torch.from_numpy(np.ascontiguousarray(ranks, np.float32)),
                    torch.from_numpy(counts))

        def refine(cand_keys, cand_counts):
            ck, cc = cand_keys.numpy().view(np.uint64), cand_counts.numpy()
            keys_o = np.zeros((nq, K), np.uint64)
            scores_o = np.zeros((nq, K), np.float32)
            counts_o = np.zeros(nq, np.int32)
            for q in range(nq):
                if cc[q] < 0:
                    counts_o[q] = cc[q]
                    continue
                held = [int(x) for x in ck[q, :cc[q]] if int(x) in mine]
                if not held:
                    continue
                idx = np.array([mine[x] for x in held])
                _, rk, rs, rc, rst = ora.flat_search(metric, rows[b:e][idx],
                                                     np.array(held, np.uint64), queries[q:q + 1],
                                                     K, radius, threads=1)
                counts_o[q] = -rst[0] if rst[0] else rc[0]
                keys_o[q, :rc[0]], scores_o[q, :rc[0]] = rk[0, :rc[0]], rs[0, :rc[0]]
            return (torch.from_numpy(keys_o.view(np.int64)), torch.from_numpy(scores_o),
                    torch.from_numpy(counts_o))

        def merge(m, kk, ak, asc, ac):
            return _merge(ora, m, kk, ak, asc, ac)

        fk, fs, fc = refined_search(candidates, refine, merge, metric, K, C)
        out.put((rank, fk.numpy().view(np.uint64).tolist(), fs.numpy().view(np.uint32).tolist(),
                 fc.numpy().tolist()))
    finally:
        dist.destroy_process_group()


def _shard_local(oracle, metric, rows, keys, codes, params, queries, scale, world):
    """Each shard refining its own best candidates, then one merge: what the
    two-exchange order avoids."""
    from xvec_b200.sharded import shard_range
    parts = []
    for r in range(world):
        b, e = shard_range(rows.shape[0], r, world, align=64)
        parts.append(oracle.sq8_search(metric, codes[b:e], params[b:e], rows[b:e], keys[b:e],
                                       queries, K, 0.0, scale))
    out = []
    for q in range(queries.shape[0]):
        mk = np.concatenate([p[1][q, :max(p[3][q], 0)] for p in parts])
        ms = np.concatenate([p[2][q, :max(p[3][q], 0)] for p in parts])
        out.append(oracle.merge_results(metric, K, mk, ms)[0].tolist())
    return out


@pytest.mark.parametrize("metric,radius,scale",
                         [(IP, 0.0, 4.0), (L2, 0.0, 4.0), (L2, 40.0, 4.0), (IP, 0.0, 1.0),
                          (L2, 0.0, 1.0)])
def test_two_rank_refined_search_equals_one_index(oracle, metric, radius, scale):
    world = 2
    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, metric, radius, scale, out))
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
    rows, keys, queries = _data(seed=metric)
    codes, params = oracle.quantize_int8_batch(rows)
    _, ok, os_, oc, ost = oracle.sq8_search(metric, codes, params, rows, keys, queries, K, radius,
                                            scale)
    if scale == 1.0:
        # With as many candidates as results, refining shard-locally changes
        # the answer for some queries of this data.
        local = _shard_local(oracle, metric, rows, keys, codes, params, queries, scale, world)
        assert any(local[q] != ok[q, :oc[q]].tolist()
                   for q in range(queries.shape[0]) if ost[q] == 0)
    for _, fk, fs, fc in results:
        for q in range(queries.shape[0]):
            if ost[q] != 0:
                assert fc[q] == -int(ost[q]), q
                continue
            c = int(oc[q])
            assert fc[q] == c, (q, fc[q], c)
            assert fk[q][:c] == ok[q, :c].tolist(), q
            assert fs[q][:c] == os_[q, :c].view(np.uint32).tolist(), q
