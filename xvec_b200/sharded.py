"""Sharded search over the GPUs of one node (one process per GPU).

The reference fans a query out over segments and merges the per-segment
top-k with MergeSearchResults (collection.go:4043-4066, query.go:154-191).
Here each rank holds one shard of the rows (its own index on its own GPU,
keys globally unique), searches it, the per-shard lists are exchanged and
every rank merges them on its GPU with the same ordering rule.

With a library communicator (``library_comm``: the id made by rank 0 and
sent over torch.distributed) the whole sharded search is one call of the C
ABI, ``xvec_gpu_sharded_search_device``: the library's own NCCL all-gather of
one packed buffer, bounded waits.  Without one, the exchange below runs over
torch.distributed (any backend; gloo on the CPU) and the merge is the
library's kernel.

Refined searches (SQ8 with a refine scale, RaBitQ with Refine) take two
exchanges, so that the refined candidates are the reference's: the
RefinementCandidateCount (or max(TopK, EF)) best approximate results of the
whole index (refiner.go:133-166, hnsw_rabitq.go:584, 780-801), not of each
shard.  Every rank computes its shard's candidates with their ranks, the
lists are exchanged and merged by rank (ties by key), every rank refines the
merged candidates it holds, and those results are exchanged and merged under
the index metric.
"""
from __future__ import annotations

import numpy as np
import torch
import torch.distributed as dist

from . import (METRIC_L2, Comm, SearchOptions, SearchResults, _Index, merge_results_device,
               sharded_search_device)


def shard_range(n_total: int, rank: int, world: int, align: int = 1):
    """Contiguous row range [begin, end) of `rank`'s shard: the rows are split
    into `world` nearly equal parts, each a multiple of `align` rows except
    the last."""
    units = (n_total + align - 1) // align
    per = (units + world - 1) // world
    begin = min(n_total, rank * per * align)
    end = min(n_total, (rank + 1) * per * align)
    return begin, end


def library_comm(device: int, group=None, timeout_ms: int = 60000) -> Comm:
    """The library's NCCL communicator over the ranks of a torch.distributed
    job: rank 0 makes the id, broadcast_object_list sends it, every rank
    joins on `device`."""
    rank = dist.get_rank(group)
    world = dist.get_world_size(group)
    obj = [Comm.unique_id() if rank == 0 else None]
    dist.broadcast_object_list(obj, src=0, group=group)
    return Comm.init_rank(device, obj[0], world, rank, timeout_ms)


def exchange(keys: torch.Tensor, scores: torch.Tensor, counts: torch.Tensor, group=None):
    """All-gather of every rank's per-shard results: [nq, k] keys / scores and
    [nq] counts in, [world, nq, k] / [world, nq] out, on the tensors' device
    (NCCL on GPUs; gloo on the CPU)."""
    world = dist.get_world_size(group)
    nq, k = keys.shape
    # Outputs concatenated along dim 0 (the layout every backend accepts).
    all_keys = torch.empty((world * nq, k), dtype=keys.dtype, device=keys.device)
    all_scores = torch.empty((world * nq, k), dtype=scores.dtype, device=scores.device)
    all_counts = torch.empty((world * nq,), dtype=counts.dtype, device=counts.device)
    dist.all_gather_into_tensor(all_keys, keys.contiguous(), group=group)
    dist.all_gather_into_tensor(all_scores, scores.contiguous(), group=group)
    dist.all_gather_into_tensor(all_counts, counts.contiguous(), group=group)
    return (all_keys.view(world, nq, k), all_scores.view(world, nq, k),
            all_counts.view(world, nq))


def refined_search(candidates_fn, refine_fn, merge_fn, metric: int, k: int, c: int, group=None):
    """The two-exchange refined search over the ranks of `group`.

    candidates_fn() -> (keys [nq, c] int64, ranks [nq, c] float32, counts [nq] int32):
        this rank's candidates (failed queries: negative counts);
    refine_fn(cand_keys [nq, c], cand_counts [nq]) -> (keys [nq, k], scores, counts):
        the exact top-k among the candidates this rank holds;
    merge_fn(metric, k, keys [world, nq, kk], scores, counts) -> ([nq, kk], [nq, kk], [nq]):
        MergeSearchResults of the gathered lists.
    Returns the merged final (keys, scores, counts), identical on every rank."""
    keys, ranks, counts = candidates_fn()
    all_keys, all_ranks, all_counts = exchange(keys, ranks, counts, group)
    cand_keys, _, cand_counts = merge_fn(METRIC_L2, c, all_keys, all_ranks, all_counts)
    rkeys, rscores, rcounts = refine_fn(cand_keys, cand_counts)
    all_keys, all_scores, all_counts = exchange(rkeys, rscores, rcounts, group)
    return merge_fn(metric, k, all_keys, all_scores, all_counts)


class ShardedSearch:
    def __init__(self, index: _Index, group=None, comm: Comm | None = None):
        self.index = index
        self.group = group
        self.comm = comm
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.device = torch.device("cuda", index.device)

    def search_device(self, queries: torch.Tensor, options: SearchOptions):
        """queries: device tensor [nq, d] (float32, or int16/uint16 bits for FP16 storage).
        Returns merged (keys int64 [nq,k], scores float32 [nq,k], counts int32 [nq])."""
        nq, k = queries.shape[0], options.top_k
        stream = torch.cuda.current_stream(self.device).cuda_stream
        if self.comm is not None:
            keys = torch.empty((nq, k), dtype=torch.int64, device=self.device)
            scores = torch.empty((nq, k), dtype=torch.float32, device=self.device)
            counts = torch.empty((nq,), dtype=torch.int32, device=self.device)
            sharded_search_device(self.comm, self.index, queries.data_ptr(), nq, options,
                                  keys.data_ptr(), scores.data_ptr(), counts.data_ptr(),
                                  stream=stream)
            return keys, scores, counts
        c = self.index.candidate_count(options) if self.world > 1 else 0
        if c > 0:
            return self._refined(queries, options, c, stream)
        keys = torch.empty((nq, k), dtype=torch.int64, device=self.device)
        scores = torch.empty((nq, k), dtype=torch.float32, device=self.device)
        counts = torch.empty((nq,), dtype=torch.int32, device=self.device)
        self.index.search_device(queries.data_ptr(), nq, options, keys.data_ptr(),
                                 scores.data_ptr(), counts.data_ptr(), stream=stream)
        if self.world == 1:
            return keys, scores, counts
        all_keys, all_scores, all_counts = exchange(keys, scores, counts, self.group)
        out_keys = torch.empty_like(keys)
        out_scores = torch.empty_like(scores)
        out_counts = torch.empty_like(counts)
        merge_results_device(self.index.device, self.index.metric, k, nq, self.world,
                             all_keys.data_ptr(), all_scores.data_ptr(), all_counts.data_ptr(),
                             out_keys.data_ptr(), out_scores.data_ptr(), out_counts.data_ptr(),
                             stream=stream)
        return out_keys, out_scores, out_counts

    def _merge(self, metric, kk, all_keys, all_scores, all_counts):
        world, nq = all_counts.shape
        stream = torch.cuda.current_stream(self.device).cuda_stream
        out_keys = torch.empty((nq, kk), dtype=torch.int64, device=self.device)
        out_scores = torch.empty((nq, kk), dtype=torch.float32, device=self.device)
        out_counts = torch.empty((nq,), dtype=torch.int32, device=self.device)
        merge_results_device(self.index.device, metric, kk, nq, world,
                             all_keys.data_ptr(), all_scores.data_ptr(), all_counts.data_ptr(),
                             out_keys.data_ptr(), out_scores.data_ptr(), out_counts.data_ptr(),
                             stream=stream)
        return out_keys, out_scores, out_counts

    def _refined(self, queries: torch.Tensor, options: SearchOptions, c: int, stream: int):
        nq, k = queries.shape[0], options.top_k
        dev = self.device

        def candidates():
            keys = torch.empty((nq, c), dtype=torch.int64, device=dev)
            ranks = torch.empty((nq, c), dtype=torch.float32, device=dev)
            counts = torch.empty((nq,), dtype=torch.int32, device=dev)
            self.index.candidates_device(queries.data_ptr(), nq, options, keys.data_ptr(),
                                         ranks.data_ptr(), counts.data_ptr(), stream=stream)
            return keys, ranks, counts

        def refine(cand_keys, cand_counts):
            keys = torch.empty((nq, k), dtype=torch.int64, device=dev)
            scores = torch.empty((nq, k), dtype=torch.float32, device=dev)
            counts = torch.empty((nq,), dtype=torch.int32, device=dev)
            self.index.refine_device(queries.data_ptr(), nq, cand_keys.data_ptr(), c,
                                     cand_counts.data_ptr(), k, options.radius, keys.data_ptr(),
                                     scores.data_ptr(), counts.data_ptr(), stream=stream)
            return keys, scores, counts

        return refined_search(candidates, refine, self._merge, self.index.metric, k, c,
                              self.group)

    def search(self, queries_host: torch.Tensor, options: SearchOptions) -> SearchResults:
        """End-to-end form: host (pinned) queries in, host results out on every rank."""
        q = queries_host.to(self.device, non_blocking=True)
        keys, scores, counts = self.search_device(q, options)
        return SearchResults(keys.cpu().numpy().view(np.uint64), scores.cpu().numpy(),
                             counts.cpu().numpy())
