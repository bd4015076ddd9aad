#!/usr/bin/env python
"""bench.py — batched Flat cosine search over FP16 storage on B200.

Workload (the Flat half of the metric "queries/sec (Flat & IVF-PQ, batch 10k,
k=10)" as quoted on the Flat-cosine configuration): 10,000,000 base vectors x
dim 768 stored as binary16, drawn from a mixture of 1,000 Gaussian clusters
(centres N(0,1), sigma 0.3) then L2-normalised; 10,000 queries from the same
mixture; top-k = 100; cosine distance.  One step = one batched search of all
queries.  With --gpus N the base is split into N contiguous shards (one per
GPU, one process per GPU); each shard is searched, the per-shard top-k lists
are all-gathered over NCCL and merged on every GPU (strong scaling: the total
work is fixed).

JSON line fields follow the bench contract: value (device-resident queries),
e2e (host queries through the C-ABI, H2D/D2H inside the timed region),
roofline of the dominant kernel (the candidate scan), cpu_baseline (the CPU
oracle on a bounded sample), clocks sampled during the timed region.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

N_BASE, DIM, N_QUERIES, TOP_K, CLUSTERS, SIGMA = 10_000_000, 768, 10_000, 100, 1000, 0.3
CHUNK = 250_000  # generation unit: shards are whole chunks for N in {1, 2, 4, 8}
METRIC = "queries/sec (Flat & IVF-PQ, batch 10k, k=10) at 1/2/4/8 B200; % of roofline"
WORKLOAD = "Flat cosine search, FP16 storage, 10,000,000 x 768 (1,000-cluster mixture, L2-normalised), 10,000 queries, top-k=100"


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=5)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--n", type=int, default=N_BASE)
    p.add_argument("--nq", type=int, default=N_QUERIES)
    p.add_argument("--cpu-sample-rows", type=int, default=1_000_000)
    p.add_argument("--cpu-sample-queries", type=int, default=480)
    p.add_argument("--ref-queries", type=int, default=0,
                   help="--impl reference: queries per step (default: one per host thread)")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-parity", action="store_true",
                   help="skip the check of sampled queries against the oracle over the full base")
    p.add_argument("--batch-sweep", default="",
                   help="comma-separated batch sizes (e.g. 1,8,64): after the main timing, "
                        "the median device latency of one search of each size is added to "
                        "the JSON line as batch_sweep (the default Flat workload, rabitq_l2_refine, ivfpq_l2, "
                        "sq8_ip_refine)")
    p.add_argument("--workload",
                   choices=["flat_cosine_fp16", "ivfpq_l2", "sq8_ip_refine", "rabitq_l2_refine",
                            "diskann_l2",
                            "flat_l2_fp32", "ivf_flat_l2", "ivf_sq8_l2_refine",
                            "rabitq7_l2_refine", "sq4_l2_refine", "pq_train_l2",
                            "rabitq_hnsw_l2_refine"],
                   default="flat_cosine_fp16",
                   help="flat_cosine_fp16: the Flat configuration above (default); ivfpq_l2: "
                        "IVF-PQ L2, 1e8 x 128, nlist 16384, 32 x 256 PQ, nprobe 64, k=10; "
                        "sq8_ip_refine: INT8 SQ Flat IP, 2e7 x 1024, k=10, ScaleFactor 4; "
                        "rabitq_l2_refine: one-bit RaBitQ L2, 1e7 x 960, k=10, EF 100; "
                        "flat_l2_fp32: Flat L2 over FP32 storage, 1e6 x 128 N(0,1), 1,000 "
                        "queries, k=10; ivf_flat_l2: IVF with exact scoring, 1e7 x 128, "
                        "nlist 4096, nprobe 32, k=10; ivf_sq8_l2_refine: the same IVF with "
                        "INT8 list scoring and ScaleFactor 4; rabitq7_l2_refine: the RaBitQ "
                        "data with TotalBits 7; sq4_l2_refine: INT4 SQ Flat L2, 4e6 x 128, "
                        "10,000 queries, k=10, ScaleFactor 4; pq_train_l2: TrainPQ (32 chunks, "
                        "200,000-row sample, 12 iterations) on 1e6 x 128, one training per step; "
                        "rabitq_hnsw_l2_refine: the HNSW-RaBitQ graph walk, 1e6 x 960, degree-32 "
                        "proximity graph built on the GPU, EF 100, k=10, beside the linear scan")
    return p.parse_args()


def peaks():
    """(bf16 TFLOP/s, HBM GB/s, source).  The bf16 figure is the sustained
    one: the timed region runs the scan back to back for about a second under
    the power cap, which is the regime the sustained GEMM measurement covers."""
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            m = json.load(f)
        bf16 = float(m.get("bf16_tflops_sustained") or m["bf16_tflops"])
        return bf16, float(m["hbm_gbs"]), "measured"
    except Exception:
        return 1400.0, 6650.0, "fallback"


def int8_peak(dev, seconds=3.0):
    """Dense INT8 tensor throughput measured here, the denominator of the
    INT8 scans' roofline: torch._int_mm (cuBLASLt, int8 x int8 -> int32)
    on 8192^3, 2 * 8192^3 ops per call, best of 10 (burst) and back to back
    for `seconds` (sustained), CUDA events; TOP/s."""
    import torch
    m = 8192
    g = torch.Generator(device=dev).manual_seed(5)
    a = torch.randint(-127, 128, (m, m), dtype=torch.int8, device=dev, generator=g)
    b = torch.randint(-127, 128, (m, m), dtype=torch.int8, device=dev, generator=g)
    for bt in (b, b.t().contiguous().t()):
        try:
            torch._int_mm(a, bt)
            break
        except RuntimeError:
            continue
    else:
        return None
    ops = 2.0 * m ** 3
    burst = []
    for _ in range(10):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        torch._int_mm(a, bt)
        e1.record()
        e1.synchronize()
        burst.append(e0.elapsed_time(e1))
    calls, t_ms = 0, 0.0
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    t_end = time.time() + seconds
    while time.time() < t_end:
        for _ in range(8):
            torch._int_mm(a, bt)
        calls += 8
        torch.cuda.current_stream().synchronize()
    e1.record()
    e1.synchronize()
    t_ms = e0.elapsed_time(e1)
    return {"burst_tops": ops / (min(burst) / 1e3) / 1e12,
            "sustained_tops": ops * calls / (t_ms / 1e3) / 1e12,
            "how": "torch._int_mm int8 8192^3 (2 x 8192^3 ops): best of 10, and back to back "
                   f"for {seconds:.0f} s; measured in this run on this GPU"}


def int8_roofline(achieved, dev, kernel, note, ops):
    """The INT8 scan's roofline object: against the sustained INT8 GEMM
    figure measured in this run (the scan runs back to back in the timed
    region), the nominal dense figure alongside."""
    meas = int8_peak(dev)
    peak = meas["sustained_tops"] if meas else 4500.0
    return {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TOP/s",
            "frac": (achieved / peak) if achieved else None, "traffic": None,
            "peak_source": ("measured sustained dense INT8 GEMM (" + meas["how"] + ")"
                            if meas else "nominal dense INT8 tensor (measurement failed)"),
            "int8_gemm": meas, "nominal_tops": 4500.0,
            "frac_of_nominal": (achieved / 4500.0) if achieved else None,
            "kernel": kernel, "kernel_ms": None, "algorithmic_int_ops_per_launch": ops,
            "note": note}


# ---------------------------------------------------------------------------
# Synthetic data (seeded, generated on the device where it is used).
# ---------------------------------------------------------------------------
def mixture_centers(torch, device, seed=1234):
    g = torch.Generator(device=device).manual_seed(seed)
    return torch.randn(CLUSTERS, DIM, generator=g, device=device)


def mixture_chunk(torch, centers, chunk_index, rows, device, seed=99):
    g = torch.Generator(device=device).manual_seed(seed * 1_000_003 + chunk_index)
    idx = torch.randint(0, CLUSTERS, (rows,), generator=g, device=device)
    x = centers[idx] + SIGMA * torch.randn(rows, DIM, generator=g, device=device)
    x = x / x.norm(dim=1, keepdim=True)
    return x.to(torch.float16)


def make_queries(torch, centers, nq, device):
    return mixture_chunk(torch, centers, 10**6, nq, device, seed=7)


def host_chunks(torch, centers, n, device):
    """The whole base again, chunk by chunk, as the float32 decoding of the
    stored binary16 rows (what the reference scores for a VectorFP16 field),
    with their keys: (rows [m, 768] float32, keys [m] uint64) on the host."""
    import numpy as np
    for c in range((n + CHUNK - 1) // CHUNK):
        m = min(CHUNK, n - c * CHUNK)
        rows = mixture_chunk(torch, centers, c, m, device).float().cpu().numpy()
        yield rows, np.arange(c * CHUNK, c * CHUNK + m, dtype=np.uint64)


# ---------------------------------------------------------------------------
# Clock sampling during the timed region.
# ---------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
            # The first sample is taken as the timed region starts (at most 3 s
            # of waiting), so a region shorter than the 200 ms period still
            # has one.
            t0 = time.time()
            while not self.lines and time.time() - t0 < 3.0:
                time.sleep(0.005)
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc:
            # One more sample at the end of a short region (at most 0.3 s).
            n0, t0 = len(self.lines), time.time()
            while len(self.lines) == n0 and time.time() - t0 < 0.3:
                time.sleep(0.005)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for name, val in zip(names, parts[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        sm.sort()
        med = sm[len(sm) // 2] if sm else None
        return {"sm_mhz": med, "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------------------
# The oracle over the full base: parity of sampled queries, the CPU baseline
# and the reference arm.
# ---------------------------------------------------------------------------
PARITY_QUERIES = 32


def oracle_with_kernels():
    """The oracle, with the reference's own float kernels (floats_avx512.c,
    compiled in place into oracle/_ref) when they are built and the host has
    AVX-512; returns (oracle, kind)."""
    from oracle.oracle import Oracle, ReferenceFloats
    ora = Oracle()
    if ReferenceFloats.available():
        ora.use_reference_kernels(ReferenceFloats())
        return ora, "reference"
    return ora, "port"


def sample_query_ids(nq, count=PARITY_QUERIES):
    import numpy as np
    return np.unique(np.linspace(0, nq - 1, min(count, nq)).astype(np.int64))


def oracle_flat_over_chunks(ora, metric, chunks, queries, k, threads):
    """Flat top-k of `queries` over every row of `chunks` (an iterable of
    (rows float32 [m, d], keys uint64 [m])) by the oracle: the top-k of each
    chunk (topKPrevalidatedCandidatesWithOptions), then per query the
    oracle's MergeSearchResults of those lists.  Exact: an entry of the top-k
    over all rows is in the top-k of its own chunk under the same (score,
    key) order.  Returns keys [nq, k], scores [nq, k], counts [nq] and the
    seconds spent in the oracle (searches and merges)."""
    import numpy as np
    nq = queries.shape[0]
    lk = [[] for _ in range(nq)]
    ls = [[] for _ in range(nq)]
    secs = 0.0
    for rows, keys in chunks:
        t0 = time.perf_counter()
        st, ok, os_, oc, ost = ora.flat_search(metric, rows, keys, queries, k, threads=threads)
        secs += time.perf_counter() - t0
        if st != 0 or (ost != 0).any():
            raise RuntimeError(f"oracle search status {st} / {ost[ost != 0][:4]}")
        for q in range(nq):
            lk[q].append(ok[q, :oc[q]])
            ls[q].append(os_[q, :oc[q]])
    out_k = np.zeros((nq, k), np.uint64)
    out_s = np.zeros((nq, k), np.float32)
    out_c = np.zeros(nq, np.int32)
    t0 = time.perf_counter()
    for q in range(nq):
        mk, ms = ora.merge_results(metric, k, np.concatenate(lk[q]), np.concatenate(ls[q]))
        out_c[q] = len(mk)
        out_k[q, :len(mk)] = mk
        out_s[q, :len(ms)] = ms
    secs += time.perf_counter() - t0
    return out_k, out_s, out_c, secs


def parity_record(gpu, ref, qids, base_rows, kind, oracle_s, what, how="evenly spaced over the batch"):
    """Compares the GPU's results of the sampled queries with the oracle's:
    identical counts and keys, bit-identical float32 scores."""
    import numpy as np
    gk, gs, gc = gpu
    rk, rs, rc = ref
    bad = []
    for i, q in enumerate(qids):
        c = int(rc[i])
        same = (int(gc[q]) == c and np.array_equal(gk[q, :c].view(np.uint64), rk[i, :c])
                and np.array_equal(gs[q, :c].view(np.uint32), rs[i, :c].view(np.uint32)))
        if not same:
            bad.append(int(q))
    return {"queries": int(len(qids)), "query_ids": f"{len(qids)} ids {how}",
            "base_rows": int(base_rows), "against": what, "oracle_kernels": kind,
            "keys_identical": not bad, "scores_bitwise": not bad, "mismatched_queries": bad[:8],
            "oracle_s": oracle_s}


def merged_refine(ora, metric, cand, k, lists, queries):
    """The refined search over chunked candidates (RefinedSearch,
    refiner.go:133-166): per query, the `cand` best of every chunk's
    approximate candidates (MergeSearchResults of the per-chunk lists, which
    hold each chunk's `cand` best under the same (score, key) order), the exact
    metric.Compute of their originals, and the top k (MergeSearchResults).
    lists[q] = [(keys, approximate scores, originals [m, d])]."""
    import numpy as np
    nq = len(lists)
    out_k = np.zeros((nq, k), np.uint64)
    out_s = np.zeros((nq, k), np.float32)
    out_c = np.zeros(nq, np.int32)
    for q in range(nq):
        keys = np.concatenate([x[0] for x in lists[q]])
        scores = np.concatenate([x[1] for x in lists[q]])
        rows = np.concatenate([x[2] for x in lists[q]])
        ck, _ = ora.merge_results(metric, cand, keys, scores)
        where = {int(kk): i for i, kk in enumerate(keys)}
        exact = np.zeros(len(ck), np.float32)
        for i, kk in enumerate(ck):
            st, exact[i] = ora.metric_compute(metric, queries[q], rows[where[int(kk)]])
            if st != 0:
                raise RuntimeError(f"oracle exact score status {st}")
        mk, ms = ora.merge_results(metric, k, ck, exact)
        out_c[q] = len(mk)
        out_k[q, :len(mk)] = mk
        out_s[q, :len(ms)] = ms
    return out_k, out_s, out_c


def gpu_results_host(search, queries, opts):
    """One more search of the whole batch; its results on the host."""
    import numpy as np
    import torch
    keys, scores, counts = search.search_device(queries, opts)
    torch.cuda.synchronize()
    return (keys.cpu().numpy().view(np.uint64), scores.cpu().numpy(), counts.cpu().numpy())


def run_reference(args):
    """--impl reference: the reference's CPU path for the default workload on
    the host cores.  Each step is a bounded sample of the workload: a few of
    the batch's queries, each scored against every one of the n rows with the
    reference's own floats_avx512.c kernels (when built; the oracle's
    restatement otherwise) and the ported heap/top-k and merge rules, on all
    host threads.  The rows are the float32 decodings of the binary16 base,
    generated once (on the GPU when there is one, which only makes the
    synthetic data) and held in host memory; when the host cannot hold them
    they are regenerated chunk by chunk every step, outside the timed part.
    value = sampled queries / measured step time; nothing is scaled."""
    import numpy as np
    import torch
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from oracle.oracle import COSINE
    dev = torch.device("cuda", 0) if torch.cuda.is_available() else torch.device("cpu")
    n, k = args.n, TOP_K
    centers = mixture_centers(torch, dev)
    queries = make_queries(torch, centers, args.nq, dev)
    threads = os.cpu_count() or 1
    per = max(1, min(args.nq, args.ref_queries or threads))
    ora, kind = oracle_with_kernels()
    need = n * DIM * 4
    try:
        import psutil
        avail = psutil.virtual_memory().available
    except Exception:
        avail = 0
    held = need < 0.6 * avail
    cache = list(host_chunks(torch, centers, n, dev)) if held else None
    step_s = []
    for i in range(args.warmup + args.steps):
        ids = (np.arange(per) + i * per) % args.nq
        q = queries[torch.as_tensor(ids, device=dev)].float().cpu().numpy()
        chunks = cache if held else host_chunks(torch, centers, n, dev)
        _, _, _, secs = oracle_flat_over_chunks(ora, COSINE, chunks, q, k, threads)
        if i >= args.warmup:
            step_s.append(secs)
    ms = 1000.0 * sum(step_s) / len(step_s)
    value = per / (ms / 1000.0)
    sample = (f"{per} of the {args.nq} queries per step, each over all {n} rows (float32 "
              f"decodings of the binary16 base, "
              + ("held in host memory" if held else "regenerated per step outside the timing")
              + f"); {args.steps} timed steps after {args.warmup} warm-up; {threads} threads; "
              "distance kernels: "
              + ("the reference's floats_avx512.c compiled in place" if kind == "reference"
                 else "the oracle's restatement")
              + "; per-chunk top-k merged by MergeSearchResults")
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "queries/sec",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms, "queries_per_step": per, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": WORKLOAD, "global_batch": args.nq, "top_k": k,
                   "base_vectors": n, "dim": DIM, "metric": "cosine", "storage": "fp16",
                   "parallelism": "host threads (one query per task, as core.BatchTopK)"},
        "cpu_baseline": {"value": value, "unit": "queries/sec", "cores": threads, "kind": kind,
                         "sample": sample},
        "e2e": {"value": value, "unit": "queries/sec", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# IVF-PQ L2: 100,000,000 x 128 float32 from a 10,000-cluster mixture (centres
# N(0,1), sigma 0.3); nlist 16,384; PQ 32 chunks x 256 codewords; nprobe 64;
# 10,000 queries; top-k 10.  The 16,384 coarse centroids are trained on the
# GPU with the IVF builder's k-means (xvec_gpu_kmeans_train: reservoir seeding,
# 10 Lloyd iterations) on every row, as the builder trains; the PQ codebook is
# TrainPQ's on the GPU (xvec_gpu_pq_train).
# ---------------------------------------------------------------------------
PQ_N, PQ_DIM, PQ_CLUSTERS, PQ_NLIST, PQ_CHUNKS, PQ_NPROBE, PQ_K = (
    100_000_000, 128, 10_000, 16_384, 32, 64, 10)
PQ_CHUNK_ROWS = 1_000_000
PQ_TRAIN_ITERS, PQ_TRAIN_SEED = 10, 16_384
# TrainPQ (pq.go:107-179) for the codebook: 32 chunks, a 200,000-row sample
# drawn by TrainPQ from the first 4,000,000 rows, 12 Lloyd iterations.
PQ_CODEBOOK_ROWS, PQ_CODEBOOK_SAMPLE, PQ_CODEBOOK_ITERS = 4_000_000, 200_000, 12
PQ_WORKLOAD = ("IVF-PQ L2 search, 100,000,000 x 128 float32 (10,000-cluster mixture), "
               "nlist 16,384, PQ 32 x 256 (8-bit codes), nprobe 64, 10,000 queries, top-k=10")


def pq_mixture(torch, centers, tag, rows, device):
    g = torch.Generator(device=device).manual_seed(7_000_003 * 31 + tag)
    idx = torch.randint(0, centers.shape[0], (rows,), generator=g, device=device)
    return centers[idx] + SIGMA * torch.randn(rows, centers.shape[1], generator=g, device=device)


def run_ivfpq(args):
    import numpy as np
    import torch
    import torch.distributed as dist

    import xvec_b200 as xb
    from xvec_b200.sharded import ShardedSearch, shard_range

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=600), device_id=dev)
    n = args.n if args.n != N_BASE else PQ_N
    nq = args.nq
    g = torch.Generator(device=dev).manual_seed(4321)
    centers = torch.randn(PQ_CLUSTERS, PQ_DIM, generator=g, device=dev)
    # Coarse centroids: GPU k-means on every row, as IVFBuilder.Build trains
    # (ivf.go:144-212); every rank trains the same model.
    train_n = n
    train = torch.empty(train_n, PQ_DIM, device=dev)
    for c in range((train_n + PQ_CHUNK_ROWS - 1) // PQ_CHUNK_ROWS):
        m = min(PQ_CHUNK_ROWS, train_n - c * PQ_CHUNK_ROWS)
        train[c * PQ_CHUNK_ROWS:c * PQ_CHUNK_ROWS + m] = pq_mixture(torch, centers, c, m, dev)
    cents = torch.empty(PQ_NLIST, PQ_DIM, device=dev)
    train_labels = torch.empty(train_n, dtype=torch.int32, device=dev)
    torch.cuda.synchronize()
    t_train = time.perf_counter()
    kc, train_iters, _, _ = xb.kmeans_train_device(
        local, xb.METRIC_L2, train.data_ptr(), train_n, PQ_DIM, PQ_NLIST, cents.data_ptr(),
        train_labels.data_ptr(), iterations=PQ_TRAIN_ITERS, seed=PQ_TRAIN_SEED,
        stream=torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    t_train = time.perf_counter() - t_train
    cents = cents[:kc].contiguous()
    # The PQ codebook: TrainPQ on the GPU (KMC2 seeding per chunk, Lloyd).
    t_pq = time.perf_counter()
    book_rows = train[:min(train_n, PQ_CODEBOOK_ROWS)].cpu().numpy()
    del train, train_labels
    _, pivots = xb.pq_train(xb.METRIC_L2, book_rows, chunks=PQ_CHUNKS,
                            max_train_samples=PQ_CODEBOOK_SAMPLE,
                            max_iterations=PQ_CODEBOOK_ITERS, seed=PQ_TRAIN_SEED, device=local)
    t_pq = time.perf_counter() - t_pq
    del book_rows
    index = xb.IVFPQIndex(PQ_DIM, xb.METRIC_L2, device=local)
    index.set_model(cents.cpu().numpy(), pivots, PQ_CHUNKS)
    b, e = shard_range(n, rank, world, align=PQ_CHUNK_ROWS)
    index.reserve(e - b)
    sizes = torch.zeros(PQ_NLIST, dtype=torch.int64, device=dev)
    labels = torch.empty(PQ_CHUNK_ROWS, dtype=torch.int32, device=dev)
    stream = torch.cuda.current_stream().cuda_stream
    check = rank == 0 and world == 1 and not args.no_parity
    host_labels = np.empty(e - b, np.int32) if check else None
    for c0 in range(b, e, PQ_CHUNK_ROWS):
        m = min(PQ_CHUNK_ROWS, e - c0)
        rows = pq_mixture(torch, centers, c0 // PQ_CHUNK_ROWS, m, dev).contiguous()
        keys = torch.arange(c0, c0 + m, dtype=torch.int64, device=dev)
        index.add_device(keys.data_ptr(), rows.data_ptr(), m, stream)
        xb.kmeans_assign_device(local, xb.METRIC_L2, rows.data_ptr(), m, cents.data_ptr(),
                                cents.shape[0], PQ_DIM, labels.data_ptr(), 0, stream)
        sizes += torch.bincount(labels[:m].long(), minlength=PQ_NLIST)
        if check:
            host_labels[c0 - b:c0 - b + m] = labels[:m].cpu().numpy()
        del rows, keys
    queries = pq_mixture(torch, centers, 10**6 + 3, nq, dev).contiguous()
    torch.cuda.synchronize()
    # Algorithmic bytes of the list scan on this shard: every probed list's
    # codes (32 B per row), the same probe the search makes.
    probe = xb.DenseFlatIndex(PQ_DIM, xb.METRIC_L2, device=local)
    probe.add(np.arange(cents.shape[0], dtype=np.uint64), cents.cpu().numpy())
    pr = probe.search(queries.cpu().numpy(), PQ_NPROBE)
    h_sizes = sizes.cpu().numpy()
    scanned = int(h_sizes[pr.keys.astype(np.int64)].sum())
    probe.close()
    opts = xb.SearchOptions(top_k=PQ_K, nprobe=PQ_NPROBE)
    search = sharded(index, world, local)
    ms, scan_ms, e2e_ms, st, clocks = time_search(search, queries, opts, args, dev, world, local)
    # Parity of sampled queries (one GPU): the oracle's IVF-PQ search over the
    # lists its own probe picks, with every row of those lists regenerated and
    # PQ-encoded by the oracle (the rows' lists are the GPU assignment's).
    parity = None
    if check:
        gpu_res = gpu_results_host(search, queries, opts)
        parity = ivfpq_parity(torch, centers, cents.cpu().numpy(), np.asarray(pivots), host_labels,
                              queries, gpu_res, n, dev)
        del host_labels

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_ivfpq_qps(cents.cpu().numpy(), np.asarray(pivots), h_sizes,
                            queries[:args.cpu_sample_queries].cpu().numpy())
    if rank == 0:
        _, hbm_peak, peak_kind = peaks()
        nbytes = scanned * PQ_CHUNKS
        achieved = nbytes / (scan_ms / 1000.0) / 1e9 if scan_ms > 0 else None
        line = {
            "metric": METRIC, "value": nq / (ms / 1000.0), "unit": "queries/sec",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "u8 codes, f32 tables, f64 sums", "data": "synthetic",
            "config": {"workload": PQ_WORKLOAD, "global_batch": nq, "top_k": PQ_K,
                       "base_vectors": n, "dim": PQ_DIM, "metric": "l2", "nlist": PQ_NLIST,
                       "pq_chunks": PQ_CHUNKS, "nprobe": PQ_NPROBE,
                       "model": f"coarse centroids: GPU k-means (xvec_gpu_kmeans_train, "
                                f"reservoir seed {PQ_TRAIN_SEED}, {train_iters} Lloyd "
                                f"iterations) on all {train_n} rows in {t_train:.1f} s; "
                                f"PQ codebook: TrainPQ on the GPU (xvec_gpu_pq_train: "
                                f"{PQ_CHUNKS} chunks, a {PQ_CODEBOOK_SAMPLE}-row sample of the "
                                f"first {min(train_n, PQ_CODEBOOK_ROWS)} rows, "
                                f"{PQ_CODEBOOK_ITERS} iterations) in {t_pq:.1f} s",
                       "parallelism": f"rows sharded over {world} GPU(s), NCCL all-gather + merge",
                       "l2": "inputs larger than L2 (3.2 GB codes, 51 GB originals)"},
            "e2e": {"value": nq / (e2e_ms / 1000.0), "unit": "queries/sec",
                    "h2d_bytes_per_step": nq * PQ_DIM * 4,
                    "d2h_bytes_per_step": nq * PQ_K * 12 + nq * 4},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm_peak, "unit": "GB/s",
                         "frac": (achieved / hbm_peak) if achieved else None, "traffic": None,
                         "peak_source": f"{peak_kind} HBM copy bandwidth",
                         "kernel": "IVF-PQ list scan", "kernel_ms": scan_ms,
                         "algorithmic_bytes_per_launch": nbytes,
                         "scanned_codes_per_launch": scanned},
            "cpu_baseline": cpu,
            "clocks": clocks,
            "gpu_launches": int(st["kernel_launches"]),
            "parity": parity,
        }
        print(json.dumps(line), flush=True)
    finish_ranks(world)


_COMMS = []


def sharded(index, world, local):
    """The search every rank runs: the plain search at N = 1; above, the
    library's sharded search over its own NCCL communicator (the id made by
    rank 0 and sent over torch.distributed), one C-ABI call per step."""
    from xvec_b200.sharded import ShardedSearch, library_comm
    comm = library_comm(local) if world > 1 else None
    if comm is not None:
        _COMMS.append(comm)
    return ShardedSearch(index, comm=comm)


def close_comms():
    """Frees the library's communicators (every rank, same order) before the
    process group goes."""
    while _COMMS:
        _COMMS.pop().close()


def time_search(search, queries, opts, args, dev, world, local):
    """W warm-up searches, then K timed ones between barriers (CUDA events on
    the stream, max over ranks, clocks sampled meanwhile), then K end-to-end
    searches from pinned host queries.  Returns (ms, scan_ms, e2e_ms, stats,
    clocks); scan_ms is the library's device time of the candidate scan."""
    import torch
    import torch.distributed as dist

    import xvec_b200 as xb

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    for _ in range(args.warmup):
        search.search_device(queries, opts)
    barrier()
    xb.enable_timing(True)
    xb.reset_stats()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        barrier()
        start.record()
        for _ in range(args.steps):
            search.search_device(queries, opts)
        stop.record()
        barrier()
    xb.enable_timing(False)
    st = xb.stats()
    ms = start.elapsed_time(stop) / args.steps
    t = torch.tensor([ms], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    scan_ms = st["scan_ms"] / max(1, args.steps)
    q_host = queries.cpu().pin_memory()
    search.search(q_host, opts)
    barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        search.search(q_host, opts)
    barrier()
    e2e_ms = (time.perf_counter() - t0) * 1000.0 / args.steps
    if world > 1:
        t = torch.tensor([e2e_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())
    return ms, scan_ms, e2e_ms, st, clocks.summary()


def batch_sweep(search, queries, opts, sizes, reps=15):
    """Median device latency (CUDA events) of one search of each batch size,
    queries resident on the device; which scan served it (tensor cores or
    not) from the library's counters."""
    import torch

    import xvec_b200 as xb
    out = []
    for b in sizes:
        q = queries[:b].contiguous()
        for _ in range(3):
            search.search_device(q, opts)
        torch.cuda.synchronize()
        xb.reset_stats()
        times = []
        for _ in range(reps):
            a, z = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            search.search_device(q, opts)
            z.record()
            torch.cuda.synchronize()
            times.append(a.elapsed_time(z))
        times.sort()
        st = xb.stats()
        # One more pass with the library's device timers (scan vs whole search).
        xb.enable_timing(True)
        xb.reset_stats()
        for _ in range(reps):
            search.search_device(q, opts)
        torch.cuda.synchronize()
        xb.enable_timing(False)
        tst = xb.stats()
        med = times[len(times) // 2]
        out.append({"nq": b, "ms": med, "queries_per_sec": b / (med / 1000.0),
                    "tensor_scans_per_search": st["tensor_scans"] / reps,
                    "stream_scans_per_search": st["stream_scans"] / reps,
                    "scan_ms": tst["scan_ms"] / reps, "search_device_ms": tst["search_ms"] / reps,
                    "exact_queries": st["exact_queries"]})
    return out


def init_ranks(args):
    import torch
    import torch.distributed as dist
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=600), device_id=dev)
    return world, rank, local, dev


def finish_ranks(world):
    import torch.distributed as dist
    if world > 1:
        dist.barrier()
        close_comms()
        dist.destroy_process_group()


def common_line(nq, ms, e2e_ms, args, world, dtype, config, roofline, cpu, clocks, st, k, d,
                q_bytes):
    return {
        "metric": METRIC, "value": nq / (ms / 1000.0), "unit": "queries/sec", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": dtype,
        "data": "synthetic", "config": config,
        "e2e": {"value": nq / (e2e_ms / 1000.0), "unit": "queries/sec",
                "h2d_bytes_per_step": nq * d * q_bytes, "d2h_bytes_per_step": nq * k * 12 + nq * 4},
        "roofline": roofline, "cpu_baseline": cpu, "clocks": clocks,
        "gpu_launches": int(st["kernel_launches"]),
    }


# ---------------------------------------------------------------------------
# IVF with exact scoring of the probed lists (IVFIndex.SearchIVF): 10,000,000
# x 128 float32 from the 10,000-cluster mixture, nlist 4,096 centroids trained
# with the GPU k-means on the first 1,000,000 rows, nprobe 32, 10,000
# queries, top-k 10.
# ---------------------------------------------------------------------------
IVF_N, IVF_NLIST, IVF_NPROBE, IVF_K, IVF_TRAIN = 10_000_000, 4096, 32, 10, 1_000_000
IVF_WORKLOAD = ("IVF exact L2 search, 10,000,000 x 128 float32 (10,000-cluster mixture), nlist "
                "4,096 (GPU k-means on the first 1,000,000 rows), nprobe 32, 10,000 queries, "
                "top-k=10")
# The same index with INT8 scalar-quantized list scoring
# (ScalarQuantizedIVFIndex.SearchIVF) and the FP32 refine of the 40 best codes.
IVF_SQ_SCALE = 4.0
IVF_SQ_WORKLOAD = ("IVF INT8 scalar-quantized L2 search with FP32 refinement, 10,000,000 x 128 "
                   "(10,000-cluster mixture), nlist 4,096 (GPU k-means on the first 1,000,000 "
                   "rows), nprobe 32, 10,000 queries, top-k=10, ScaleFactor 4")


def run_ivf_flat(args, sq8=False):
    import numpy as np
    import torch

    import xvec_b200 as xb
    from xvec_b200.sharded import ShardedSearch, shard_range
    world, rank, local, dev = init_ranks(args)
    n = args.n if args.n != N_BASE else IVF_N
    nq = args.nq
    g = torch.Generator(device=dev).manual_seed(4321)
    centers = torch.randn(PQ_CLUSTERS, PQ_DIM, generator=g, device=dev)
    train_n = min(n, IVF_TRAIN)
    train = pq_mixture(torch, centers, 0, train_n, dev).contiguous()
    cents = torch.empty(IVF_NLIST, PQ_DIM, device=dev)
    labels = torch.empty(train_n, dtype=torch.int32, device=dev)
    stream = torch.cuda.current_stream().cuda_stream
    kc, iters, _, _ = xb.kmeans_train_device(local, xb.METRIC_L2, train.data_ptr(), train_n,
                                             PQ_DIM, IVF_NLIST, cents.data_ptr(),
                                             labels.data_ptr(), iterations=10, seed=4096,
                                             stream=stream)
    cents = cents[:kc].contiguous()
    del train, labels
    cls = xb.ScalarQuantizedIVFIndex if sq8 else xb.IVFIndex
    index = cls(PQ_DIM, xb.METRIC_L2, device=local)
    index.set_model(cents.cpu().numpy())
    b, e = shard_range(n, rank, world, align=PQ_CHUNK_ROWS)
    index.reserve(e - b)
    sizes = torch.zeros(kc, dtype=torch.int64, device=dev)
    lab = torch.empty(PQ_CHUNK_ROWS, dtype=torch.int32, device=dev)
    host_rows = ([] if (rank == 0 and world == 1 and not (args.no_cpu_baseline and args.no_parity))
                 else None)
    host_labels = []
    for c0 in range(b, e, PQ_CHUNK_ROWS):
        m = min(PQ_CHUNK_ROWS, e - c0)
        rows = pq_mixture(torch, centers, c0 // PQ_CHUNK_ROWS, m, dev).contiguous()
        keys = torch.arange(c0, c0 + m, dtype=torch.int64, device=dev)
        index.add_device(keys.data_ptr(), rows.data_ptr(), m, stream)
        xb.kmeans_assign_device(local, xb.METRIC_L2, rows.data_ptr(), m, cents.data_ptr(), kc,
                                PQ_DIM, lab.data_ptr(), 0, stream)
        sizes += torch.bincount(lab[:m].long(), minlength=kc)
        if host_rows is not None:
            host_rows.append(rows.cpu().numpy())
            host_labels.append(lab[:m].cpu().numpy())
        del rows, keys
    queries = pq_mixture(torch, centers, 10**6 + 3, nq, dev).contiguous()
    torch.cuda.synchronize()
    probe = xb.DenseFlatIndex(PQ_DIM, xb.METRIC_L2, device=local)
    probe.add(np.arange(kc, dtype=np.uint64), cents.cpu().numpy())
    pr = probe.search(queries.cpu().numpy(), IVF_NPROBE)
    h_sizes = sizes.cpu().numpy()
    scanned = int(h_sizes[pr.keys.astype(np.int64)].sum())
    probe.close()
    opts = xb.SearchOptions(top_k=IVF_K, nprobe=IVF_NPROBE,
                            refine_scale=IVF_SQ_SCALE if sq8 else 0.0)
    search = sharded(index, world, local)
    ms, scan_ms, e2e_ms, st, clocks = time_search(search, queries, opts, args, dev, world, local)
    gpu_res = gpu_results_host(search, queries, opts) if host_rows is not None else None
    cpu, parity = None, None
    if host_rows is not None:
        from oracle.oracle import L2 as OL2, Oracle
        allrows = np.concatenate(host_rows)
        labels_h = np.concatenate(host_labels)  # the GPU's nearest-centroid labels
        offsets = np.zeros(kc + 1, np.int64)
        np.add.at(offsets, labels_h + 1, 1)
        offsets = np.cumsum(offsets)
        positions = np.argsort(labels_h, kind="stable").astype(np.int64)
        # About 10-20 s of CPU work on the box's host cores.
        qs = queries[:max(8, args.cpu_sample_queries * 4)].cpu().numpy()
        threads = os.cpu_count() or 1
        ora = Oracle()
        all_keys = np.arange(n, dtype=np.uint64)
        if sq8:
            codes, params = ora.quantize_int8_batch(allrows)
            t0 = time.perf_counter()
            ost, rk, rs, rc, _ = ora.ivf_sq8_search(OL2, codes, params, allrows, all_keys,
                                                    cents.cpu().numpy(), offsets, positions, qs,
                                                    IVF_K, IVF_NPROBE, refine_scale=IVF_SQ_SCALE,
                                                    threads=threads)
        else:
            t0 = time.perf_counter()
            ost, rk, rs, rc, _ = ora.ivf_flat_search(OL2, allrows, all_keys, cents.cpu().numpy(),
                                                     offsets, positions, qs, IVF_K, IVF_NPROBE,
                                                     threads=threads)
        dt = time.perf_counter() - t0
        if not args.no_cpu_baseline:
            cpu = {"value": qs.shape[0] / dt, "unit": "queries/sec", "cores": threads,
                   "kind": "port",
                   "sample": f"{qs.shape[0]} queries over the full index, {dt:.1f} s on "
                             f"{threads} threads (lists from the GPU assignment"
                             + (", codes from the oracle's quantizer" if sq8 else "")
                             + ", not timed)"}
        if not args.no_parity and ost == 0:
            # The same oracle run is the parity check of those queries.
            parity = parity_record(gpu_res, (rk, rs, rc), np.arange(qs.shape[0]), n, "port", dt,
                                   ("oracle SQ-IVF search + refine" if sq8 else
                                    "oracle IVF exact search")
                                   + " over the full index (lists from the GPU assignment)",
                                   how="first of the batch")
    if rank == 0:
        _, hbm_peak, peak_kind = peaks()
        # Per scanned row: the float32 row, or the INT8 codes and the row's
        # 16-byte scoring terms.
        row_bytes = PQ_DIM + 16 if sq8 else PQ_DIM * 4
        nbytes = scanned * row_bytes
        achieved = nbytes / (scan_ms / 1000.0) / 1e9 if scan_ms > 0 else None
        roof = {"bound": "hbm", "achieved": achieved, "peak": hbm_peak, "unit": "GB/s",
                "frac": (achieved / hbm_peak) if achieved else None, "traffic": None,
                "peak_source": f"{peak_kind} HBM copy bandwidth",
                "kernel": "IVF INT8 list scan" if sq8 else "IVF exact list scan",
                "kernel_ms": scan_ms, "algorithmic_bytes_per_launch": nbytes,
                "scanned_rows_per_launch": scanned}
        config = {"workload": IVF_SQ_WORKLOAD if sq8 else IVF_WORKLOAD, "global_batch": nq,
                  "top_k": IVF_K, "base_vectors": n, "dim": PQ_DIM, "metric": "l2", "nlist": kc,
                  "nprobe": IVF_NPROBE, "kmeans_iterations": iters,
                  "parallelism": f"rows sharded over {world} GPU(s), NCCL all-gather + merge",
                  "l2": ("inputs larger than L2 (1.3 GB codes, 5.1 GB rows)" if sq8
                         else "inputs larger than L2 (5.1 GB rows)")}
        if sq8:
            config["refine_scale"] = IVF_SQ_SCALE
        dtype = "i8 codes, f32/f64 scores" if sq8 else "f32"
        line = common_line(nq, ms, e2e_ms, args, world, dtype, config, roof, cpu, clocks, st,
                           IVF_K, PQ_DIM, 4)
        line["parity"] = parity
        print(json.dumps(line), flush=True)
    finish_ranks(world)


# ---------------------------------------------------------------------------
# Flat L2 over FP32 storage: 1,000,000 x 128 i.i.d. N(0,1), 1,000 queries from
# the same distribution, top-k 10 (the configuration the reference runs on
# its CPU path).
# ---------------------------------------------------------------------------
F32_N, F32_DIM, F32_NQ, F32_K = 1_000_000, 128, 1000, 10
F32_WORKLOAD = ("Flat exact L2 search, FP32 storage, 1,000,000 x 128 i.i.d. N(0,1), 1,000 "
                "queries, top-k=10")


def run_flat_fp32(args):
    import numpy as np
    import torch

    import xvec_b200 as xb
    from xvec_b200.sharded import ShardedSearch, shard_range
    world, rank, local, dev = init_ranks(args)
    n = args.n if args.n != N_BASE else F32_N
    nq = args.nq if args.nq != N_QUERIES else F32_NQ
    index = xb.DenseFlatIndex(F32_DIM, xb.METRIC_L2, xb.STORAGE_FP32, device=local)
    b, e = shard_range(n, rank, world, align=1024)
    index.reserve(e - b)
    g = torch.Generator(device=dev).manual_seed(101)
    rows = torch.randn(n, F32_DIM, generator=g, device=dev)[b:e].contiguous()
    keys = torch.arange(b, e, dtype=torch.int64, device=dev)
    stream = torch.cuda.current_stream().cuda_stream
    index.add_device(keys.data_ptr(), rows.data_ptr(), e - b, stream)
    queries = torch.randn(nq, F32_DIM, generator=torch.Generator(device=dev).manual_seed(202),
                          device=dev)
    torch.cuda.synchronize()
    opts = xb.SearchOptions(top_k=F32_K)
    search = sharded(index, world, local)
    ms, scan_ms, e2e_ms, st, clocks = time_search(search, queries, opts, args, dev, world, local)
    # Parity of sampled queries over all n rows (rank 0 regenerates them).
    gpu_res = gpu_results_host(search, queries, opts)
    parity = None
    if rank == 0 and not args.no_parity:
        from oracle.oracle import L2
        allrows = torch.randn(n, F32_DIM, generator=torch.Generator(device=dev).manual_seed(101),
                              device=dev).cpu().numpy()
        qids = sample_query_ids(nq)
        ora, kind = oracle_with_kernels()
        rk, rs, rc, secs = oracle_flat_over_chunks(
            ora, L2, [(allrows, np.arange(n, dtype=np.uint64))],
            queries[torch.as_tensor(qids, device=dev)].cpu().numpy(), F32_K, os.cpu_count() or 1)
        parity = parity_record(gpu_res, (rk, rs, rc), qids, n, kind, secs,
                               "oracle Flat L2 over all rows")
        del allrows
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_flat_l2_qps(rows.cpu().numpy(), queries[:max(8, args.cpu_sample_queries // 2)]
                              .cpu().numpy())
    if rank == 0:
        bf16_peak, _, peak_kind = peaks()
        flops = 2.0 * nq * (e - b) * F32_DIM
        achieved = flops / (scan_ms / 1000.0) / 1e12 if scan_ms > 0 else None
        roof = {"bound": "tensor", "achieved": achieved, "peak": bf16_peak, "unit": "TFLOP/s",
                "frac": (achieved / bf16_peak) if achieved else None, "traffic": None,
                "peak_source": f"{peak_kind} sustained bf16 dense GEMM; the scan runs three "
                               "bf16 MMAs per element pair (hi*hi, hi*lo, lo*hi), so the "
                               "tensor work is 3x the algorithmic flops",
                "kernel": "Flat FP32 candidate scan (bf16 split)", "kernel_ms": scan_ms,
                "algorithmic_flops_per_launch": flops, "mma_flops_per_launch": 3.0 * flops}
        config = {"workload": F32_WORKLOAD, "global_batch": nq, "top_k": F32_K,
                  "base_vectors": n, "dim": F32_DIM, "metric": "l2", "storage": "fp32",
                  "parallelism": f"rows sharded over {world} GPU(s), NCCL all-gather + merge",
                  "l2": "inputs larger than L2 (512 MB rows + 512 MB bf16 parts)"}
        line = common_line(nq, ms, e2e_ms, args, world, "f32 rows, bf16x3 tensor ranks", config,
                           roof, cpu, clocks, st, F32_K, F32_DIM, 4)
        line["parity"] = parity
        print(json.dumps(line), flush=True)
    finish_ranks(world)


def cpu_flat_l2_qps(rows, queries):
    import numpy as np

    from oracle.oracle import L2, Oracle, ReferenceFloats
    ora = Oracle()
    kind = "port"
    if ReferenceFloats.available():
        ora.use_reference_kernels(ReferenceFloats())
        kind = "reference"
    keys = np.arange(rows.shape[0], dtype=np.uint64)
    threads = os.cpu_count() or 1
    t0 = time.perf_counter()
    st, _, _, _, _ = ora.flat_search(L2, rows, keys, queries, F32_K, threads=threads)
    dt = time.perf_counter() - t0
    if st != 0:
        raise RuntimeError(f"oracle status {st}")
    return {"value": queries.shape[0] / dt, "unit": "queries/sec", "cores": threads, "kind": kind,
            "sample": f"{queries.shape[0]} queries over all {rows.shape[0]} rows, {dt:.1f} s on "
                      f"{threads} threads"}


# ---------------------------------------------------------------------------
# INT8 scalar-quantized Flat, inner product, FP32 refinement: 20,000,000 x
# 1024, N(0,1) scaled per dimension by U(0.5, 2) (seeded), per-vector INT8
# codes; 10,000 queries; top-k 10 with ScaleFactor 4 (40 codes refined).
# ---------------------------------------------------------------------------
SQ_N, SQ_DIM, SQ_K, SQ_SCALE, SQ_CHUNK_ROWS = 20_000_000, 1024, 10, 4.0, 500_000
SQ_PARITY_QUERIES = 16
SQ_WORKLOAD = ("INT8 scalar-quantized Flat IP search with FP32 refinement, 20,000,000 x 1024 "
               "(N(0,1) x per-dimension U(0.5,2)), 10,000 queries, top-k=10, ScaleFactor 4")


def sq_rows(torch, scale, tag, rows, device):
    g = torch.Generator(device=device).manual_seed(9_000_011 + tag)
    return torch.randn(rows, scale.shape[0], generator=g, device=device) * scale


def run_sq8(args):
    import numpy as np
    import torch

    import xvec_b200 as xb
    from xvec_b200.sharded import ShardedSearch, shard_range
    world, rank, local, dev = init_ranks(args)
    n = args.n if args.n != N_BASE else SQ_N
    nq = args.nq
    g = torch.Generator(device=dev).manual_seed(77)
    scale = torch.rand(SQ_DIM, generator=g, device=dev) * 1.5 + 0.5
    index = xb.ScalarQuantizedFlatIndex(SQ_DIM, xb.METRIC_IP, device=local)
    b, e = shard_range(n, rank, world, align=SQ_CHUNK_ROWS)
    index.reserve(e - b)
    stream = torch.cuda.current_stream().cuda_stream
    for c0 in range(b, e, SQ_CHUNK_ROWS):
        m = min(SQ_CHUNK_ROWS, e - c0)
        rows = sq_rows(torch, scale, c0 // SQ_CHUNK_ROWS, m, dev).contiguous()
        keys = torch.arange(c0, c0 + m, dtype=torch.int64, device=dev)
        index.add_device(keys.data_ptr(), rows.data_ptr(), m, stream)
        del rows, keys
    queries = sq_rows(torch, scale, 10**6, nq, dev).contiguous()
    torch.cuda.synchronize()
    opts = xb.SearchOptions(top_k=SQ_K, refine_scale=SQ_SCALE)
    search = sharded(index, world, local)
    ms, scan_ms, e2e_ms, st, clocks = time_search(search, queries, opts, args, dev, world, local)
    # Parity of sampled queries over all n rows: the oracle quantizes every
    # row (regenerated chunk by chunk on rank 0), keeps each chunk's 40 best
    # codes per query, merges them and refines the 40 with the originals.
    gpu_res = gpu_results_host(search, queries, opts)
    parity = None
    if rank == 0 and not args.no_parity:
        from oracle.oracle import IP as OIP
        qids = sample_query_ids(nq, SQ_PARITY_QUERIES)
        qs = queries[torch.as_tensor(qids, device=dev)].cpu().numpy()
        ora, kind = oracle_with_kernels()
        threads = os.cpu_count() or 1
        cand = max(1, int(SQ_K * SQ_SCALE))
        lists = [[] for _ in qids]
        t0 = time.perf_counter()
        for c0 in range(0, n, SQ_CHUNK_ROWS):
            m = min(SQ_CHUNK_ROWS, n - c0)
            rows = sq_rows(torch, scale, c0 // SQ_CHUNK_ROWS, m, dev).cpu().numpy()
            codes, params = ora.quantize_int8_batch(rows, threads)
            keys = np.arange(c0, c0 + m, dtype=np.uint64)
            st_, ok, os_, oc, ost = ora.sq8_search(OIP, codes, params, rows, keys, qs, cand,
                                                   threads=threads)
            if st_ != 0:
                raise RuntimeError(f"oracle SQ8 status {st_}")
            for i in range(len(qids)):
                kk = ok[i, :oc[i]]
                lists[i].append((kk, os_[i, :oc[i]], rows[(kk - c0).astype(np.int64)]))
            del rows, codes, params
        rk, rs, rc = merged_refine(ora, OIP, cand, SQ_K, lists, qs)
        parity = parity_record(gpu_res, (rk, rs, rc), qids, n, kind, time.perf_counter() - t0,
                               "oracle SQ8 Flat IP + refine over all rows (each chunk's 40 best "
                               "codes merged, then the exact refine)")
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        m = min(args.cpu_sample_rows // 10, n)
        sample = sq_rows(torch, scale, 0, m, dev).cpu().numpy()
        cpu = cpu_sq8_qps(sample, queries[:max(8, args.cpu_sample_queries // 8)].cpu().numpy(), n)
    if rank == 0:
        shard = e - b
        ops = 2.0 * nq * shard * SQ_DIM
        achieved = ops / (scan_ms / 1000.0) / 1e12 if scan_ms > 0 else None
        roof = int8_roofline(achieved, dev, "SQ8 code scan",
                             "the scan runs on tcgen05 kind::i8", ops)
        roof["kernel_ms"] = scan_ms
        config = {"workload": SQ_WORKLOAD, "global_batch": nq, "top_k": SQ_K, "base_vectors": n,
                  "dim": SQ_DIM, "metric": "ip", "refine_scale": SQ_SCALE,
                  "parallelism": f"rows sharded over {world} GPU(s), NCCL all-gather + merge",
                  "l2": "inputs larger than L2 (20 GB codes)"}
        line = common_line(nq, ms, e2e_ms, args, world, "i8 codes, f32/f64 scores", config, roof,
                           cpu, clocks, st, SQ_K, SQ_DIM, 4)
        line["parity"] = parity
        print(json.dumps(line), flush=True)
    finish_ranks(world)


# ---------------------------------------------------------------------------
# INT4 scalar-quantized Flat, L2, FP32 refinement: 4,000,000 x 128, N(0,1)
# scaled per dimension by U(0.5, 2); 10,000 queries; top-k 10, ScaleFactor 4.
# The codes (512 MB, one per byte) are larger than L2.
# ---------------------------------------------------------------------------
SQ4_N, SQ4_DIM, SQ4_NQ, SQ4_K, SQ4_SCALE = 4_000_000, 128, 10_000, 10, 4.0
SQ4_WORKLOAD = ("INT4 scalar-quantized Flat L2 search with FP32 refinement, 4,000,000 x 128 "
                "(N(0,1) x per-dimension U(0.5,2)), 10,000 queries, top-k=10, ScaleFactor 4")


def run_sq4(args):
    import numpy as np
    import torch

    import xvec_b200 as xb
    from xvec_b200.sharded import ShardedSearch, shard_range
    world, rank, local, dev = init_ranks(args)
    n = args.n if args.n != N_BASE else SQ4_N
    nq = args.nq if args.nq != N_QUERIES else SQ4_NQ
    g = torch.Generator(device=dev).manual_seed(44)
    scale = torch.rand(SQ4_DIM, generator=g, device=dev) * 1.5 + 0.5
    index = xb.Int4QuantizedFlatIndex(SQ4_DIM, xb.METRIC_L2, device=local)
    b, e = shard_range(n, rank, world, align=SQ_CHUNK_ROWS)
    index.reserve(e - b)
    stream = torch.cuda.current_stream().cuda_stream
    for c0 in range(b, e, SQ_CHUNK_ROWS):
        m = min(SQ_CHUNK_ROWS, e - c0)
        rows = sq_rows(torch, scale, c0 // SQ_CHUNK_ROWS, m, dev).contiguous()
        keys = torch.arange(c0, c0 + m, dtype=torch.int64, device=dev)
        index.add_device(keys.data_ptr(), rows.data_ptr(), m, stream)
        del rows, keys
    queries = sq_rows(torch, scale, 10**6, nq, dev).contiguous()
    torch.cuda.synchronize()
    opts = xb.SearchOptions(top_k=SQ4_K, refine_scale=SQ4_SCALE)
    ms, scan_ms, e2e_ms, st, clocks = time_search(sharded(index, world, local), queries, opts, args, dev,
                                                  world, local)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        from oracle.oracle import L2, Oracle
        ora = Oracle()
        m = min(args.cpu_sample_rows // 10, n)
        sample = sq_rows(torch, scale, 0, m, dev).cpu().numpy()
        qs = queries[:max(8, args.cpu_sample_queries // 4)].cpu().numpy()
        packed, params = ora.quantize_int4_batch(sample)
        threads = os.cpu_count() or 1
        t0 = time.perf_counter()
        ora.sq4_search(L2, packed, params, sample, np.arange(m, dtype=np.uint64), qs, SQ4_K, 0.0,
                       SQ4_SCALE, threads=threads)
        dt = time.perf_counter() - t0
        cpu = {"value": qs.shape[0] / dt * m / n, "unit": "queries/sec", "cores": threads,
               "kind": "port",
               "sample": f"{qs.shape[0]} queries x {m}-row sample, {dt:.1f} s on {threads} "
                         f"threads; QPS scaled by rows/{n}"}
    if rank == 0:
        shard = e - b
        flops = 2.0 * nq * shard * SQ4_DIM
        achieved = flops / (scan_ms / 1000.0) / 1e12 if scan_ms > 0 else None
        roof = int8_roofline(achieved, dev, "INT4 code scan",
                             "the INT4 codes are scanned by tcgen05 kind::i8", flops)
        roof["kernel_ms"] = scan_ms
        config = {"workload": SQ4_WORKLOAD, "global_batch": nq, "top_k": SQ4_K,
                  "base_vectors": n, "dim": SQ4_DIM, "metric": "l2", "refine_scale": SQ4_SCALE,
                  "parallelism": f"rows sharded over {world} GPU(s), NCCL all-gather + merge",
                  "l2": "inputs larger than L2 (512 MB codes)"}
        print(json.dumps(common_line(nq, ms, e2e_ms, args, world, "i4 codes, f32/f64 scores",
                                     config, roof, cpu, clocks, st, SQ4_K, SQ4_DIM, 4)),
              flush=True)
    finish_ranks(world)


# ---------------------------------------------------------------------------
# TrainPQ: 1,000,000 x 128 from the IVF-PQ mixture generator's distribution
# (i.i.d. N(0,1) here), 32 chunks of 4 dimensions, the default 200,000-row
# sample and 12 iterations.  One step is one training; the metric is
# trainings per second.
# ---------------------------------------------------------------------------
PQT_N, PQT_DIM, PQT_CHUNKS = 1_000_000, 128, 32
PQT_WORKLOAD = ("TrainPQ L2, 1,000,000 x 128 N(0,1), 32 chunks x 256 centroids, 200,000-row "
                "sample, 12 Lloyd iterations, KMC2 seeding")


def run_pq_train(args):
    import numpy as np
    import torch

    import xvec_b200 as xb
    world, rank, local, dev = init_ranks(args)
    if world != 1:
        raise SystemExit("pq_train_l2 runs on one GPU (the training is not sharded)")
    n = args.n if args.n != N_BASE else PQT_N
    g = torch.Generator(device=dev).manual_seed(303)
    rows = torch.randn(n, PQT_DIM, generator=g, device=dev)
    offsets = np.zeros(PQT_CHUNKS + 1, np.int32)
    pivots = torch.empty(256, PQT_DIM, device=dev)
    stream = torch.cuda.current_stream().cuda_stream
    lib = xb.library()

    def train():
        import ctypes
        out = ctypes.c_int32()
        st = lib.xvec_gpu_pq_train_device(local, xb.METRIC_L2, rows.data_ptr(), n, PQT_DIM,
                                          PQT_CHUNKS, 200_000, 12, 7, offsets.ctypes.data,
                                          pivots.data_ptr(), ctypes.byref(out), stream)
        if st != 0:
            raise xb.XvecGPUError(st, xb.last_error())

    for _ in range(args.warmup):
        train()
    torch.cuda.synchronize()
    st0 = xb.stats()
    with ClockSampler(local) as clocks:
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        for _ in range(args.steps):
            train()
        end.record()
        torch.cuda.synchronize()
    ms = start.elapsed_time(end) / args.steps
    launches = xb.stats()["kernel_launches"] - st0["kernel_launches"]
    # End to end: host rows in, host pivots out (xvec_gpu_pq_train).
    host = rows[:200_000].cpu().numpy()
    t0 = time.perf_counter()
    for _ in range(max(1, args.steps // 2)):
        xb.pq_train(xb.METRIC_L2, host, PQT_CHUNKS, 200_000, 12, 7, device=local)
    e2e_ms = (time.perf_counter() - t0) * 1000.0 / max(1, args.steps // 2)
    cpu = None
    if not args.no_cpu_baseline:
        from oracle.oracle import L2, Oracle
        ora = Oracle()
        sample_chunks = 4
        sub = np.ascontiguousarray(host[:, :sample_chunks * PQT_DIM // PQT_CHUNKS])
        threads = os.cpu_count() or 1
        t0 = time.perf_counter()
        ora.pq_train(L2, sub, sample_chunks, 200_000, 12, 7, threads=threads)
        dt = (time.perf_counter() - t0) * PQT_CHUNKS / sample_chunks
        cpu = {"value": 1.0 / dt, "unit": "trainings/sec", "cores": threads, "kind": "port",
               "sample": f"{sample_chunks} of {PQT_CHUNKS} chunks trained, time scaled by "
                         f"{PQT_CHUNKS // sample_chunks}"}
    print(json.dumps({
        "metric": "TrainPQ trainings per second", "value": 1000.0 / ms, "unit": "trainings/sec",
        "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32/f64",
        "data": "synthetic",
        "config": {"workload": PQT_WORKLOAD, "base_vectors": n, "dim": PQT_DIM,
                   "chunks": PQT_CHUNKS, "l2": "200,000 x 128 sample (102 MB) re-read per "
                                              "iteration; not flushed"},
        "e2e": {"value": 1000.0 / e2e_ms, "unit": "trainings/sec",
                "h2d_bytes_per_step": 200_000 * PQT_DIM * 4,
                "d2h_bytes_per_step": 256 * PQT_DIM * 4},
        "roofline": None, "cpu_baseline": cpu, "clocks": clocks.summary(),
        "gpu_launches": int(launches)}), flush=True)


def cpu_sq8_qps(sample, queries, n_total):
    import numpy as np

    from oracle.oracle import IP, Oracle
    ora = Oracle()
    codes, params = ora.quantize_int8_batch(sample)
    keys = np.arange(sample.shape[0], dtype=np.uint64)
    threads = os.cpu_count() or 1
    t0 = time.perf_counter()
    ora.sq8_search(IP, codes, params, sample, keys, queries, SQ_K, 0.0, SQ_SCALE, threads=threads)
    dt = time.perf_counter() - t0
    return {"value": queries.shape[0] / dt * sample.shape[0] / n_total, "unit": "queries/sec",
            "cores": threads, "kind": "port",
            "sample": f"{queries.shape[0]} queries x {sample.shape[0]}-row sample, {dt:.1f} s on "
                      f"{threads} threads; QPS scaled by rows/{n_total}"}


# ---------------------------------------------------------------------------
# One-bit RaBitQ, L2, exact FP32 refinement: 10,000,000 x 960 from a
# 1,000-cluster mixture (not normalised); 16 clusters and seeded rotation
# signs; 10,000 queries; top-k 10 with EF 100 (10x over-fetch) and Refine.
# ---------------------------------------------------------------------------
RQ_N, RQ_DIM, RQ_NC, RQ_K, RQ_EF, RQ_CHUNK_ROWS = 10_000_000, 960, 16, 10, 100, 500_000
RQ_PARITY_QUERIES = 16
RQ_WORKLOAD = ("RaBitQ 1-bit L2 search with exact FP32 refinement, 10,000,000 x 960 "
               "(1,000-cluster mixture), 16 clusters, 10,000 queries, top-k=10, EF 100")
# The same data with the reference's default TotalBits 7 (6 extra bits); the
# ExtraScale stands in for TrainRaBitQ's trained value (the scale that maps
# the rotated unit residuals' coordinates, |N(0,1)|/sqrt(960), onto 0..63).
RQ7_BITS, RQ7_SCALE = 7, 620.0
RQ7_WORKLOAD = ("RaBitQ 7-bit (TotalBits 7, ExtraScale 620) L2 search with exact FP32 "
                "refinement, 10,000,000 x 960 (1,000-cluster mixture), 16 clusters, 10,000 "
                "queries, top-k=10, EF 100")


def run_rabitq(args, total_bits=1):
    import numpy as np
    import torch

    import xvec_b200 as xb
    from xvec_b200.sharded import ShardedSearch, shard_range
    world, rank, local, dev = init_ranks(args)
    n = args.n if args.n != N_BASE else RQ_N
    nq = args.nq
    g = torch.Generator(device=dev).manual_seed(960)
    centers = torch.randn(CLUSTERS, RQ_DIM, generator=g, device=dev)
    cents = pq_mixture(torch, centers, 10**6 + 11, RQ_NC, dev).contiguous()
    padded = (RQ_DIM + 63) // 64 * 64
    signs = np.random.default_rng(961).integers(0, 256, 4 * padded // 8, dtype=np.uint8)
    index = xb.RaBitQIndex(RQ_DIM, xb.METRIC_L2, device=local)
    extra_scale = RQ7_SCALE if total_bits > 1 else 0.0
    index.set_model(cents.cpu().numpy(), signs, total_bits, extra_scale)
    b, e = shard_range(n, rank, world, align=RQ_CHUNK_ROWS)
    index.reserve(e - b)
    stream = torch.cuda.current_stream().cuda_stream
    for c0 in range(b, e, RQ_CHUNK_ROWS):
        m = min(RQ_CHUNK_ROWS, e - c0)
        rows = pq_mixture(torch, centers, 2 * 10**6 + c0 // RQ_CHUNK_ROWS, m, dev).contiguous()
        keys = torch.arange(c0, c0 + m, dtype=torch.int64, device=dev)
        index.add_device(keys.data_ptr(), rows.data_ptr(), m, stream)
        del rows, keys
    queries = pq_mixture(torch, centers, 3 * 10**6, nq, dev).contiguous()
    torch.cuda.synchronize()
    opts = xb.SearchOptions(top_k=RQ_K, ef=RQ_EF, refine=True)
    search = sharded(index, world, local)
    ms, scan_ms, e2e_ms, st, clocks = time_search(search, queries, opts, args, dev, world, local)
    sweep = None
    if args.batch_sweep and world == 1:
        sweep = batch_sweep(search, queries, opts, [int(x) for x in args.batch_sweep.split(",")])
    # Parity of sampled queries over all n rows: the oracle encodes every row
    # (regenerated chunk by chunk on rank 0), keeps each chunk's EF best
    # estimates per query, merges them and refines the EF with the originals.
    gpu_res = gpu_results_host(search, queries, opts)
    parity = None
    if rank == 0 and not args.no_parity:
        from oracle.oracle import L2 as OL2
        qids = sample_query_ids(nq, RQ_PARITY_QUERIES)
        qs = queries[torch.as_tensor(qids, device=dev)].cpu().numpy()
        ora, kind = oracle_with_kernels()
        threads = os.cpu_count() or 1
        cents_h = cents.cpu().numpy()
        lists = [[] for _ in qids]
        t0 = time.perf_counter()
        for c0 in range(0, n, RQ_CHUNK_ROWS):
            m = min(RQ_CHUNK_ROWS, n - c0)
            rows = pq_mixture(torch, centers, 2 * 10**6 + c0 // RQ_CHUNK_ROWS, m,
                              dev).cpu().numpy()
            codes, extra, factors = ora.rabitq_encode_rows(OL2, cents_h, signs, rows, total_bits,
                                                           extra_scale, threads)
            keys = np.arange(c0, c0 + m, dtype=np.uint64)
            st_, ok, os_, oc, ost = ora.rabitq_search(OL2, cents_h, signs, codes, factors, rows,
                                                      keys, qs, RQ_EF, RQ_EF, threads=threads,
                                                      refine=False, total_bits=total_bits,
                                                      extra=extra)
            if st_ != 0:
                raise RuntimeError(f"oracle RaBitQ status {st_}")
            for i in range(len(qids)):
                kk = ok[i, :oc[i]]
                lists[i].append((kk, os_[i, :oc[i]], rows[(kk - c0).astype(np.int64)]))
            del rows, codes, extra, factors
        rk, rs, rc = merged_refine(ora, OL2, min(n, max(RQ_K, RQ_EF)), RQ_K, lists, qs)
        parity = parity_record(gpu_res, (rk, rs, rc), qids, n, kind, time.perf_counter() - t0,
                               f"oracle RaBitQ ({total_bits}-bit) linear search + refine over "
                               "all rows (each chunk's EF best estimates merged, then the exact "
                               "refine)")
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        m = min(args.cpu_sample_rows // 50, n)
        sample = pq_mixture(torch, centers, 2 * 10**6, m, dev).cpu().numpy()
        cpu = cpu_rabitq_qps(cents.cpu().numpy(), signs, sample,
                             queries[:max(8, args.cpu_sample_queries // 4)].cpu().numpy(), n,
                             total_bits, extra_scale)
    if rank == 0:
        if total_bits > 1:
            # INT8 MMAs of the code plane v - 128 against the 16-bit integer
            # query's two planes (h, l): 2 x nq x n x (2 padded) integer ops
            # (2 x nq x n x padded algorithmic multiply-adds of the values).
            ops = 2.0 * nq * (e - b) * (2 * padded)
            achieved = ops / (scan_ms / 1000.0) / 1e12 if scan_ms > 0 else None
            roof = int8_roofline(achieved, dev, "RaBitQ multi-bit code-plane scan",
                                 "the scan runs two tcgen05 kind::i8 MMAs per k-step", ops)
            roof["kernel_ms"] = scan_ms
            workload, dtype = RQ7_WORKLOAD, "7-bit codes as an i8 plane, i32 dots, f32/f64 estimates"
            l2note = "inputs larger than L2 (9.6 GB code plane, 19.2 GB code values, 38 GB originals)"
        else:
            # INT8 MMAs over the code planes [127 b | b] against the integer
            # query [h | l]: 2 x nq x n x (2 padded) integer ops.
            ops = 2.0 * nq * (e - b) * (2 * padded)
            achieved = ops / (scan_ms / 1000.0) / 1e12 if scan_ms > 0 else None
            roof = int8_roofline(achieved, dev, "RaBitQ code-plane scan",
                                 "the scan runs on tcgen05 kind::i8", ops)
            roof["kernel_ms"] = scan_ms
            workload, dtype = RQ_WORKLOAD, "1-bit codes as i8 planes, i32 dots, f32/f64 estimates"
            l2note = "inputs larger than L2 (19.2 GB code planes, 38 GB originals)"
        config = {"workload": workload, "global_batch": nq, "top_k": RQ_K, "base_vectors": n,
                  "dim": RQ_DIM, "metric": "l2", "clusters": RQ_NC, "ef": RQ_EF,
                  "total_bits": total_bits,
                  "parallelism": f"rows sharded over {world} GPU(s), NCCL all-gather + merge",
                  "l2": l2note}
        line = common_line(nq, ms, e2e_ms, args, world, dtype, config, roof, cpu, clocks, st,
                           RQ_K, RQ_DIM, 4)
        line["exact_queries"] = int(st["exact_queries"])
        line["parity"] = parity
        if sweep is not None:
            line["batch_sweep"] = sweep
        print(json.dumps(line), flush=True)
    finish_ranks(world)


# HNSW-RaBitQ: the graph walk over a proximity graph built here (level 0: each
# row's 24 nearest rows by the library's FP16 Flat search plus 8 random rows,
# the long links that make a small-world graph navigable; levels drawn as HNSW
# draws them, each upper level's nodes linked to their 32 nearest nodes of that
# level); the same index searched linearly beside it.  The rows have low
# intrinsic dimension (a 1,000-cluster mixture in 16 latent dimensions
# projected to 960, plus noise), on which such a graph is navigable.
RH_N, RH_DEGREE, RH_RANDOM = 1_000_000, 32, 8
RH_WORKLOAD = ("HNSW-RaBitQ 1-bit L2 graph search with exact FP32 refinement, 1,000,000 x 960 "
               "(1,000-cluster mixture in 16 latent dimensions projected to 960, plus noise), "
               "degree-32 proximity graph (24 nearest + 8 random links), 16 clusters, 10,000 "
               "queries, top-k=10, EF 100")


def knn_graph_level(xb, torch, vecs, degree, dev):
    """Each row's `degree` nearest other rows (L2) by the library's Flat
    search over FP16 copies, as int32 positions [n][degree]."""
    n, d = vecs.shape
    idx = xb.DenseFlatIndex(d, xb.METRIC_L2, xb.STORAGE_FP16, device=dev.index or 0)
    h = vecs.half().contiguous()
    keys = torch.arange(n, dtype=torch.int64, device=dev)
    idx.add_device(keys.data_ptr(), h.data_ptr(), n)
    k = min(degree + 1, n)
    out = torch.empty((n, k), dtype=torch.int64, device=dev)
    sc = torch.empty((n, k), dtype=torch.float32, device=dev)
    cnt = torch.empty(n, dtype=torch.int32, device=dev)
    for b in range(0, n, 8192):
        e = min(n, b + 8192)
        idx.search_device(h[b:e].data_ptr(), e - b, xb.SearchOptions(top_k=k),
                          out[b:e].data_ptr(), sc[b:e].data_ptr(), cnt[b:e].data_ptr())
    torch.cuda.synchronize()
    idx.close()
    # Drop the row itself (first, at distance 0, for rows without an equal
    # row of a lower key; otherwise the last neighbour goes).
    own = torch.arange(n, device=dev).unsqueeze(1)
    sel = torch.where(out[:, :1] == own, out[:, 1:], out[:, :-1])[:, :degree]
    return sel.to(torch.int32).cpu().numpy()


def run_rabitq_hnsw(args):
    import numpy as np
    import torch

    import xvec_b200 as xb
    world, rank, local, dev = init_ranks(args)
    if world != 1:
        raise SystemExit("rabitq_hnsw_l2_refine runs on one GPU (the graph is not sharded)")
    n = args.n if args.n != N_BASE else RH_N
    nq = args.nq
    g = torch.Generator(device=dev).manual_seed(960)
    proj = torch.randn(DK_LATENT, RQ_DIM, generator=g, device=dev) / DK_LATENT ** 0.5
    latent = torch.randn(DK_CLUSTERS, DK_LATENT, generator=g, device=dev)

    def gen(tag, m):
        return dk_rows(torch, proj, latent, tag, m, dev)

    cents = gen(10**6 + 11, RQ_NC).contiguous()
    padded = (RQ_DIM + 63) // 64 * 64
    signs = np.random.default_rng(961).integers(0, 256, 4 * padded // 8, dtype=np.uint8)
    rows = torch.cat([gen(2 * 10**6 + c, min(RQ_CHUNK_ROWS, n - c * RQ_CHUNK_ROWS))
                      for c in range((n + RQ_CHUNK_ROWS - 1) // RQ_CHUNK_ROWS)]).contiguous()
    index = xb.RaBitQIndex(RQ_DIM, xb.METRIC_L2, device=local)
    index.set_model(cents.cpu().numpy(), signs)
    keys = torch.arange(n, dtype=torch.int64, device=dev)
    index.add_device(keys.data_ptr(), rows.data_ptr(), n, torch.cuda.current_stream().cuda_stream)
    # The graph: HNSW levels, each level's kNN lists.
    t0 = time.perf_counter()
    rng = np.random.default_rng(7)
    levels = np.floor(-np.log(rng.random(n) + 1e-12) / np.log(RH_DEGREE)).astype(np.int64)
    max_level = int(levels.max())
    offsets = np.zeros((max_level + 1, n + 1), np.int64)
    flat, base = [], 0
    for level in range(max_level + 1):
        nodes = np.nonzero(levels >= level)[0]
        counts = np.zeros(n, np.int64)
        if nodes.size > 1:
            sub = rows[torch.as_tensor(nodes, device=dev)]
            near = RH_DEGREE - RH_RANDOM if level == 0 else RH_DEGREE
            nb = knn_graph_level(xb, torch, sub, min(near, nodes.size - 1), dev)
            lists = nodes[nb]                       # positions
            if level == 0:
                lists = np.concatenate(
                    [lists, rng.integers(0, n, (n, RH_RANDOM)).astype(lists.dtype)], axis=1)
            counts[nodes] = lists.shape[1]
            order = np.zeros((n, lists.shape[1]), np.int32)
            order[nodes] = lists
            flat.append(order[counts > 0].reshape(-1) if lists.shape[1] else np.zeros(0, np.int32))
        else:
            flat.append(np.zeros(0, np.int32))
        offsets[level, 1:] = np.cumsum(counts)
        offsets[level] += base
        base += int(counts.sum())
    entry = int(np.nonzero(levels == max_level)[0][0])
    neighbors = np.concatenate(flat).astype(np.int32)
    index.set_graph(max_level, entry, offsets.reshape(-1), neighbors)
    graph_s = time.perf_counter() - t0
    del rows
    queries = gen(3 * 10**6, nq).contiguous()
    torch.cuda.synchronize()
    opts = xb.SearchOptions(top_k=RQ_K, ef=RQ_EF, refine=True)
    search = sharded(index, world, local)
    ms, walk_ms, e2e_ms, st, clocks = time_search(search, queries, opts, args, dev, world, local)
    lin_opts = xb.SearchOptions(top_k=RQ_K, ef=RQ_EF, refine=True, linear=True)
    lin_ms, _, _, _, _ = time_search(search, queries, lin_opts, args, dev, world, local)
    # Agreement of the walk with the linear scan (recall of the walk's top-10).
    gw = gpu_results_host(search, queries, opts)
    gl = gpu_results_host(search, queries, lin_opts)
    hit = sum(len(set(gw[0][q, :int(gw[2][q])].tolist()) & set(gl[0][q, :int(gl[2][q])].tolist()))
              for q in range(nq))
    recall = hit / float(max(1, int(gl[2].sum())))
    # Parity of sampled queries: the oracle's walk over the same graph, every
    # row regenerated and encoded by the oracle.
    parity = None
    if not args.no_parity:
        from oracle.oracle import L2 as OL2
        qids = sample_query_ids(nq, RQ_PARITY_QUERIES)
        qs = queries[torch.as_tensor(qids, device=dev)].cpu().numpy()
        ora, kind = oracle_with_kernels()
        t0 = time.perf_counter()
        host = np.concatenate([
            gen(2 * 10**6 + c, min(RQ_CHUNK_ROWS, n - c * RQ_CHUNK_ROWS)).cpu().numpy()
            for c in range((n + RQ_CHUNK_ROWS - 1) // RQ_CHUNK_ROWS)])
        cents_h = cents.cpu().numpy()
        codes, _, factors = ora.rabitq_encode_rows(OL2, cents_h, signs, host)
        ost, rk, rs, rc, _ = ora.hnsw_rabitq_search(
            OL2, cents_h, signs, codes, factors, host, np.arange(n, dtype=np.uint64),
            (max_level, entry, offsets.reshape(-1), neighbors), qs, RQ_K, RQ_EF)
        if ost != 0:
            raise RuntimeError(f"oracle HNSW-RaBitQ status {ost}")
        parity = parity_record(gw, (rk, rs, rc), qids, n, kind, time.perf_counter() - t0,
                               "oracle HNSW-RaBitQ walk + refine over the same graph")
        del host, codes, factors
    # Bytes the walk reads per query: codes (padded / 8) + factors (48) per
    # estimate; the walk is latency-bound, so no roofline fraction is claimed.
    roof = {"bound": "latency", "achieved": None, "peak": None, "unit": None, "frac": None,
            "traffic": None, "kernel": "hnsw_rabitq_walk_kernel", "kernel_ms": walk_ms,
            "note": "one warp per query; sequential heap decisions per visited node"}
    config = {"workload": RH_WORKLOAD, "global_batch": nq, "top_k": RQ_K, "base_vectors": n,
              "dim": RQ_DIM, "metric": "l2", "clusters": RQ_NC, "ef": RQ_EF, "degree": RH_DEGREE,
              "graph_levels": max_level + 1, "graph_build_s": graph_s,
              "parallelism": "one GPU", "l2": "inputs larger than L2 (3.8 GB originals)"}
    line = common_line(nq, ms, e2e_ms, args, world, "1-bit codes, f64 estimates", config, roof,
                       None, clocks, st, RQ_K, RQ_DIM, 4)
    line["linear_scan"] = {"ms_per_step": lin_ms, "queries_per_sec": nq / (lin_ms / 1000.0)}
    line["walk_recall_vs_linear"] = recall
    line["parity"] = parity
    print(json.dumps(line), flush=True)
    finish_ranks(world)


# DiskANN with the PQ frontier: 1,000,000 x 128 float32 of low intrinsic
# dimension (a 1,000-cluster mixture in 16 latent dimensions, sigma 0.5,
# projected to 128 by a fixed Gaussian matrix, plus N(0, 0.05^2) noise: the
# shape of descriptor data, on which a nearest-neighbour graph is navigable);
# a degree-32 graph built here (each row's 24 nearest rows by the library's
# FP16 Flat search plus 8 random rows, the entry the row nearest the mean);
# the traversal PQ model TrainPQ's on the GPU (32 chunks); ListSize 100,
# MaxDegree 32 (1 sector per node: read batches of 128 nodes); 10,000
# queries from the same distribution, top-k 10.
DK_N, DK_DIM, DK_DEGREE, DK_RANDOM, DK_CHUNKS, DK_LIST, DK_K = (
    1_000_000, 128, 32, 8, 32, 100, 10)
DK_PARITY_QUERIES, DK_CPU_QUERIES = 16, 2000
DK_LATENT, DK_CLUSTERS, DK_SIGMA, DK_NOISE = 16, 1000, 0.5, 0.05
DK_WORKLOAD = ("DiskANN L2 graph search with the PQ frontier, 1,000,000 x 128 float32 "
               "(1,000-cluster mixture in 16 latent dimensions projected to 128, plus noise), "
               "degree-32 graph (24 nearest + 8 random links), PQ 32 x 256, ListSize 100, "
               "10,000 queries, top-k=10")


def dk_rows(torch, proj, centers, tag, rows, device):
    g = torch.Generator(device=device).manual_seed(11_000_003 + tag)
    idx = torch.randint(0, centers.shape[0], (rows,), generator=g, device=device)
    z = centers[idx] + DK_SIGMA * torch.randn(rows, centers.shape[1], generator=g, device=device)
    return z @ proj + DK_NOISE * torch.randn(rows, proj.shape[1], generator=g, device=device)


def run_diskann(args):
    import numpy as np
    import torch

    import xvec_b200 as xb
    world, rank, local, dev = init_ranks(args)
    if world != 1:
        raise SystemExit("diskann_l2 runs on one GPU (the graph is not sharded)")
    n = args.n if args.n != N_BASE else DK_N
    nq = args.nq
    g = torch.Generator(device=dev).manual_seed(1616)
    proj = torch.randn(DK_LATENT, DK_DIM, generator=g, device=dev) / DK_LATENT ** 0.5
    centers = torch.randn(DK_CLUSTERS, DK_LATENT, generator=g, device=dev)
    rows = torch.cat([dk_rows(torch, proj, centers, c, min(PQ_CHUNK_ROWS, n - c * PQ_CHUNK_ROWS),
                              dev)
                      for c in range((n + PQ_CHUNK_ROWS - 1) // PQ_CHUNK_ROWS)]).contiguous()
    host = rows.cpu().numpy()
    t0 = time.perf_counter()
    chunk_offsets, pivots = xb.pq_train(xb.METRIC_L2, host, chunks=DK_CHUNKS, seed=DK_CHUNKS,
                                        device=local)
    pq_s = time.perf_counter() - t0
    index = xb.DiskANNIndex(DK_DIM, xb.METRIC_L2, device=local)
    index.set_model(pivots, DK_CHUNKS)
    keys = torch.arange(n, dtype=torch.int64, device=dev)
    index.add_device(keys.data_ptr(), rows.data_ptr(), n, torch.cuda.current_stream().cuda_stream)
    t0 = time.perf_counter()
    near = knn_graph_level(xb, torch, rows, DK_DEGREE - DK_RANDOM, dev)
    rng = np.random.default_rng(17)
    nbrs = np.concatenate([near, rng.integers(0, n, (n, DK_RANDOM)).astype(np.int32)], axis=1)
    offsets = np.arange(0, n * DK_DEGREE + 1, DK_DEGREE, dtype=np.int64)
    entry = int(torch.argmin(((rows - rows.mean(dim=0)) ** 2).sum(dim=1)).item())
    index.set_graph(entry, DK_DEGREE, offsets, nbrs.reshape(-1))
    graph_s = time.perf_counter() - t0
    del rows
    queries = dk_rows(torch, proj, centers, 10**6, nq, dev).contiguous()
    torch.cuda.synchronize()
    opts = xb.SearchOptions(top_k=DK_K, ef=DK_LIST)
    search = sharded(index, world, local)
    ms, walk_ms, e2e_ms, st, clocks = time_search(search, queries, opts, args, dev, world, local)
    lin_opts = xb.SearchOptions(top_k=DK_K, linear=True)
    lin_ms, _, _, _, _ = time_search(search, queries, lin_opts, args, dev, world, local)
    gw = gpu_results_host(search, queries, opts)
    gl = gpu_results_host(search, queries, lin_opts)
    hit = sum(len(set(gw[0][q, :int(gw[2][q])].tolist()) & set(gl[0][q, :int(gl[2][q])].tolist()))
              for q in range(nq))
    recall = hit / float(max(1, int(gl[2].sum())))
    parity, cpu = None, None
    if not (args.no_parity and args.no_cpu_baseline):
        from oracle.oracle import L2 as OL2
        ora, kind = oracle_with_kernels()
        threads = os.cpu_count() or 1
        codes = ora.pq_encode_rows(OL2, pivots, chunk_offsets, host, threads)
        norms = np.zeros(n, np.float32)
        beam = 128  # diskANNReadBatchSize of 648-byte node records
        graph = (entry, offsets, nbrs.reshape(-1))
        all_keys = np.arange(n, dtype=np.uint64)
        if not args.no_parity:
            qids = sample_query_ids(nq, DK_PARITY_QUERIES)
            qs = queries[torch.as_tensor(qids, device=dev)].cpu().numpy()
            t0 = time.perf_counter()
            ost, rk, rs, rc, _ = ora.diskann_search(OL2, pivots, chunk_offsets, codes, norms, host,
                                                    all_keys, graph, beam, qs, DK_K, DK_LIST,
                                                    threads=threads)
            if ost != 0:
                raise RuntimeError(f"oracle DiskANN status {ost}")
            parity = parity_record(gw, (rk, rs, rc), qids, n, kind, time.perf_counter() - t0,
                                   "oracle DiskANN traversal over the same graph and PQ model")
        if not args.no_cpu_baseline:
            qs = queries[:min(nq, DK_CPU_QUERIES)].cpu().numpy()
            t0 = time.perf_counter()
            ora.diskann_search(OL2, pivots, chunk_offsets, codes, norms, host, all_keys, graph,
                               beam, qs, DK_K, DK_LIST, threads=threads)
            dt = time.perf_counter() - t0
            cpu = {"value": qs.shape[0] / dt, "unit": "queries/sec", "cores": threads,
                   "kind": "port",
                   "sample": f"{qs.shape[0]} queries over the full index, {dt:.2f} s on "
                             f"{threads} threads (one query per thread)"}
    roof = {"bound": "latency", "achieved": None, "peak": None, "unit": None, "frac": None,
            "traffic": None, "kernel": "diskann_search_kernel", "kernel_ms": walk_ms,
            "note": "one block per query; rounds of up to 128 expansions with a sorted merge"}
    config = {"workload": DK_WORKLOAD, "global_batch": nq, "top_k": DK_K, "base_vectors": n,
              "dim": DK_DIM, "metric": "l2", "pq_chunks": DK_CHUNKS, "list_size": DK_LIST,
              "degree": DK_DEGREE, "read_batch": 128,  # 648-byte node records: 1 sector
              "graph_build_s": graph_s, "pq_train_s": pq_s, "parallelism": "one GPU",
              "l2": "inputs smaller than L2 (512 MB rows, 32 MB codes): a graph walk"}
    line = common_line(nq, ms, e2e_ms, args, world, "f32 rows, u8 PQ codes, f64 sums", config,
                       roof, cpu, clocks, st, DK_K, DK_DIM, 4)
    line["linear_scan"] = {"ms_per_step": lin_ms, "queries_per_sec": nq / (lin_ms / 1000.0)}
    line["recall_vs_exact"] = recall
    line["parity"] = parity
    print(json.dumps(line), flush=True)
    finish_ranks(world)


def cpu_rabitq_qps(cents, signs, sample, queries, n_total, total_bits=1, extra_scale=0.0):
    import numpy as np

    from oracle.oracle import L2, Oracle
    ora = Oracle()
    codes, extra, factors = ora.rabitq_encode_batch(L2, cents, signs, sample, total_bits,
                                                    extra_scale)
    keys = np.arange(sample.shape[0], dtype=np.uint64)
    threads = os.cpu_count() or 1
    t0 = time.perf_counter()
    ora.rabitq_search(L2, cents, signs, codes, factors, sample, keys, queries, RQ_K, RQ_EF,
                      threads=threads, total_bits=total_bits, extra=extra)
    dt = time.perf_counter() - t0
    return {"value": queries.shape[0] / dt * sample.shape[0] / n_total, "unit": "queries/sec",
            "cores": threads, "kind": "port",
            "sample": f"{queries.shape[0]} queries x {sample.shape[0]}-row sample, {dt:.1f} s on "
                      f"{threads} threads; QPS scaled by rows/{n_total}"}


PQ_PARITY_QUERIES = 8


def ivfpq_parity(torch, centers, cents, pivots, labels, queries, gpu_res, n, dev):
    import numpy as np

    from oracle.oracle import L2 as OL2
    ora, kind = oracle_with_kernels()
    threads = os.cpu_count() or 1
    qids = sample_query_ids(queries.shape[0], PQ_PARITY_QUERIES)
    qs = queries[torch.as_tensor(qids, device=dev)].cpu().numpy()
    t0 = time.perf_counter()
    probed = np.unique(np.concatenate([ora.ivf_probe(OL2, cents, q, PQ_NPROBE) for q in qs]))
    pos = np.nonzero(np.isin(labels, probed))[0]
    rows = np.empty((pos.size, PQ_DIM), np.float32)
    for c0 in range(0, n, PQ_CHUNK_ROWS):
        m = min(PQ_CHUNK_ROWS, n - c0)
        lo, hi = np.searchsorted(pos, [c0, c0 + m])
        if hi == lo:
            continue
        chunk = pq_mixture(torch, centers, c0 // PQ_CHUNK_ROWS, m, dev)
        sel = torch.as_tensor(pos[lo:hi] - c0, device=dev)
        rows[lo:hi] = chunk[sel].cpu().numpy()
        del chunk
    offsets = ora.pq_chunk_offsets(PQ_DIM, PQ_CHUNKS)
    codes = ora.pq_encode_rows(OL2, pivots, offsets, rows, threads)
    lab = labels[pos]
    list_offsets = np.zeros(cents.shape[0] + 1, np.int64)
    list_offsets[1:] = np.cumsum(np.bincount(lab, minlength=cents.shape[0]))
    list_positions = np.argsort(lab, kind="stable").astype(np.int64)
    st, rk, rs, rc, ost = ora.ivfpq_search(OL2, cents, pivots, offsets, codes,
                                           pos.astype(np.uint64), list_offsets, list_positions,
                                           qs, PQ_K, PQ_NPROBE, threads=threads)
    if st != 0:
        raise RuntimeError(f"oracle IVF-PQ status {st}")
    return parity_record(gpu_res, (rk, rs, rc), qids, n, kind, time.perf_counter() - t0,
                         f"oracle IVF-PQ search (its own probe of the {cents.shape[0]} centroids, "
                         f"the {pos.size} rows of the probed lists PQ-encoded by the oracle; "
                         "lists from the GPU assignment)")


def cpu_ivfpq_qps(cents, pivots, list_sizes, queries):
    """The oracle's IVF-PQ search over lists of the measured sizes (codes
    drawn at random: the scan's work does not depend on their values)."""
    import numpy as np

    from oracle.oracle import L2, Oracle
    ora = Oracle()
    rng = np.random.default_rng(5)
    n = int(list_sizes.sum())
    offsets = np.zeros(PQ_NLIST + 1, np.int64)
    offsets[1:] = np.cumsum(list_sizes)
    positions = np.arange(n, dtype=np.int64)
    codes = rng.integers(0, 256, (n, PQ_CHUNKS), dtype=np.uint8)
    keys = np.arange(n, dtype=np.uint64)
    w = PQ_DIM // PQ_CHUNKS
    chunk_offsets = np.arange(0, PQ_DIM + 1, w, dtype=np.int32)
    threads = os.cpu_count() or 1
    t0 = time.perf_counter()
    st, *_ = ora.ivfpq_search(L2, cents, pivots, chunk_offsets, codes, keys, offsets, positions,
                              queries, PQ_K, PQ_NPROBE, threads=threads)
    dt = time.perf_counter() - t0
    del codes
    return {"value": queries.shape[0] / dt, "unit": "queries/sec", "cores": threads,
            "kind": "port",
            "sample": f"{queries.shape[0]} queries over the full list structure ({n} codes, list "
                      f"sizes as measured, random code bytes), {dt:.1f} s on {threads} threads"}


def main():
    args = parse()
    if args.impl == "reference":
        return run_reference(args)
    if args.workload == "ivfpq_l2":
        return run_ivfpq(args)
    if args.workload == "sq8_ip_refine":
        return run_sq8(args)
    if args.workload == "flat_l2_fp32":
        return run_flat_fp32(args)
    if args.workload == "ivf_flat_l2":
        return run_ivf_flat(args)
    if args.workload == "ivf_sq8_l2_refine":
        return run_ivf_flat(args, sq8=True)
    if args.workload == "rabitq_l2_refine":
        return run_rabitq(args)
    if args.workload == "rabitq7_l2_refine":
        return run_rabitq(args, total_bits=RQ7_BITS)
    if args.workload == "sq4_l2_refine":
        return run_sq4(args)
    if args.workload == "pq_train_l2":
        return run_pq_train(args)
    if args.workload == "diskann_l2":
        return run_diskann(args)
    if args.workload == "rabitq_hnsw_l2_refine":
        return run_rabitq_hnsw(args)

    import numpy as np
    import torch
    import torch.distributed as dist

    import xvec_b200 as xb
    from xvec_b200.sharded import ShardedSearch

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)

    n, nq, k = args.n, args.nq, TOP_K
    chunks = (n + CHUNK - 1) // CHUNK
    per_rank = (chunks + world - 1) // world
    my_chunks = range(rank * per_rank, min(chunks, (rank + 1) * per_rank))
    centers = mixture_centers(torch, dev)
    index = xb.DenseFlatIndex(DIM, xb.METRIC_COSINE, xb.STORAGE_FP16, device=local)
    index.reserve(sum(min(CHUNK, n - c * CHUNK) for c in my_chunks))
    for c in my_chunks:
        rows = mixture_chunk(torch, centers, c, min(CHUNK, n - c * CHUNK), dev)
        keys = torch.arange(c * CHUNK, c * CHUNK + rows.shape[0], dtype=torch.int64, device=dev)
        index.add_device(keys.data_ptr(), rows.data_ptr(), rows.shape[0],
                         torch.cuda.current_stream().cuda_stream)
        del rows, keys
    queries = make_queries(torch, centers, nq, dev)
    torch.cuda.synchronize()
    search = sharded(index, world, local)
    opts = xb.SearchOptions(top_k=k)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    # --- device-resident timing (value) ---------------------------------------
    for _ in range(args.warmup):
        search.search_device(queries, opts)
    barrier()
    xb.enable_timing(True)
    xb.reset_stats()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        barrier()
        start.record()
        for _ in range(args.steps):
            search.search_device(queries, opts)
        stop.record()
        barrier()
    xb.enable_timing(False)
    st = xb.stats()
    ms = start.elapsed_time(stop) / args.steps
    t = torch.tensor([ms], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    value = nq / (ms / 1000.0)
    launches = int(st["kernel_launches"])
    scan_ms = st["scan_ms"] / max(1, args.steps)

    # --- end to end through the host-buffer API (e2e) ----------------------
    q_host = queries.cpu().pin_memory()
    if world == 1:
        qn = q_host.numpy().view(np.uint16)
        index.search_with_options(qn, opts)  # warm
        barrier()
        t0 = time.perf_counter()
        for _ in range(args.steps):
            index.search_with_options(qn, opts)
        e2e_ms = (time.perf_counter() - t0) * 1000.0 / args.steps
    else:
        search.search(q_host, opts)
        barrier()
        t0 = time.perf_counter()
        for _ in range(args.steps):
            search.search(q_host, opts)
        barrier()
        e2e_ms = (time.perf_counter() - t0) * 1000.0 / args.steps
        t = torch.tensor([e2e_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())
    e2e_value = nq / (e2e_ms / 1000.0)

    # --- parity on the full base (and, at N = 1, the CPU baseline) -----------
    # Every rank takes the same collective step (the search), then rank 0
    # checks the sampled queries against the oracle over all n rows, which it
    # regenerates chunk by chunk; the others wait at the closing barrier.
    gpu_res = gpu_results_host(search, queries, opts)
    cpu, parity = None, None
    if rank == 0 and not args.no_parity:
        from oracle.oracle import COSINE
        qids = sample_query_ids(nq)
        ora, kind = oracle_with_kernels()
        threads = os.cpu_count() or 1
        qsel = queries[torch.as_tensor(qids, device=dev)].float().cpu().numpy()
        rk, rs, rc, secs = oracle_flat_over_chunks(ora, COSINE, host_chunks(torch, centers, n, dev),
                                                   qsel, k, threads)
        parity = parity_record(gpu_res, (rk, rs, rc), qids, n, kind, secs,
                               "oracle Flat cosine over all rows (per-chunk top-k merged by "
                               "MergeSearchResults)")
        if world == 1 and not args.no_cpu_baseline:
            cpu = {"value": len(qids) / secs, "unit": "queries/sec", "cores": threads,
                   "kind": kind,
                   "sample": f"{len(qids)} of the {nq} queries over all {n} rows (float32 "
                             f"decodings of the stored binary16 rows, held in host memory one "
                             f"{CHUNK}-row chunk at a time), {secs:.1f} s of oracle time on "
                             f"{threads} threads; no scaling; distance kernels: "
                             + ("the reference's floats_avx512.c compiled in place"
                                if kind == "reference" else "the oracle's restatement")
                             + "; heap/top-k and merge: the ported Go rules"}

    # Batch-size sweep (one GPU): device latency of one search per batch size;
    # the streaming scan serves the smallest batches, the tensor cores the rest.
    sweep = None
    if args.batch_sweep and world == 1:
        sweep = batch_sweep(search, queries, opts, [int(x) for x in args.batch_sweep.split(",")])
        _, hbm, _ = peaks()
        for e in sweep:
            if e["stream_scans_per_search"] >= 1 and e["scan_ms"] > 0:
                # The streaming scan reads every row once (plus a 1/64 sample).
                gbs = n * DIM * 2 / (e["scan_ms"] / 1000.0) / 1e9
                e["stream_scan_hbm"] = {"achieved_gbs": gbs, "peak_gbs": hbm,
                                        "frac": gbs / hbm,
                                        "bytes": "n x d x 2 (every row once)"}

    if rank == 0:
        bf16_peak, hbm_peak, peak_kind = peaks()
        shard_rows = min(n, per_rank * CHUNK)
        flops = 2.0 * nq * shard_rows * DIM  # one launch of the scan on one shard
        achieved = flops / (scan_ms / 1000.0) / 1e12 if scan_ms > 0 else None
        # DRAM traffic of the scan from the ncu capture of the one-GPU
        # workload, scaled to this shard by its rows (the scan streams its
        # shard's rows once per pass over the query blocks, so its traffic is
        # proportional to the rows it holds).
        traffic = None
        tfile = os.path.join(ROOT, "profiles", "flat_scan_traffic.json")
        if os.path.exists(tfile):
            try:
                tjs = json.load(open(tfile))
                traffic = (tjs["bytes_per_launch_full_workload"] * shard_rows
                           / tjs.get("rows_full_workload", N_BASE))
            except Exception:
                traffic = None
        line = {
            "metric": METRIC, "value": value, "unit": "queries/sec", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f16",
            "data": "synthetic",
            "config": {"workload": WORKLOAD, "global_batch": nq, "top_k": k, "base_vectors": n,
                       "dim": DIM, "metric": "cosine", "storage": "fp16",
                       "parallelism": f"base sharded over {world} GPU(s), NCCL all-gather + merge",
                       "l2": "inputs larger than L2 (15.4 GB base)"},
            "e2e": {"value": e2e_value, "unit": "queries/sec",
                    "h2d_bytes_per_step": nq * DIM * 2,
                    "d2h_bytes_per_step": nq * k * 12 + nq * 4},
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": bf16_peak,
                         "unit": "TFLOP/s", "frac": (achieved / bf16_peak) if achieved else None,
                         "traffic": traffic,
                         "peak_source": f"{peak_kind} sustained bf16 dense GEMM",
                         "kernel": "candidate scan", "kernel_ms": scan_ms,
                         "algorithmic_flops_per_launch": flops},
            "cpu_baseline": cpu,
            "parity": parity,
            "clocks": clocks.summary(),
            "gpu_launches": launches,
            "exact_queries": int(st["exact_queries"]),
        }
        if sweep is not None:
            line["batch_sweep"] = sweep
        print(json.dumps(line), flush=True)
    finish_ranks(world)


if __name__ == "__main__":
    main()
