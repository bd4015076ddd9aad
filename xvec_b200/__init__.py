"""xvec_b200 — Python host binding of the B200 (sm_100a) xvec search library.

The compute lives in ``libxvec_gpu.so`` (CUDA kernels + the C ABI declared in
``include/xvec_gpu.h``).  This module mirrors the reference's Go interfaces for
the search path so that tests read like the reference's own:

  reference (gorse-io/xvec)                      here
  ---------------------------------------------  --------------------------------
  core.NewDenseFlatIndex / Add / SearchWithOptions  DenseFlatIndex (flat.go:79-196)
  core.NewScalarQuantizedFlatIndex (INT8)        ScalarQuantizedFlatIndex
                                                 (quantized_index.go:33-120)
  IVF SearchIVF over PQ codes                    IVFPQIndex (ivf.go:423-493, pq.go:549-595)
  HNSW-RaBitQ linear scan + Refine               RaBitQIndex (hnsw_rabitq.go:539-642)
  core.SearchOptions {TopK, Radius, Filter}      SearchOptions (query.go:39-55)
  core.Result {Key, Score}                       Result / ndarray pairs (topk.go:47-50)
  assignKMeans                                   kmeans_assign (kmeans.go:382-479)
  core.MergeSearchResults                        merge_results_device (query.go:154-191)
  segment fan-out + merge (collection.go:4040-4066)  Comm, sharded_search(_device)

There is no CPU fallback: importing this module fails if the shared library is
missing, and every search runs on a CUDA device.
"""
from __future__ import annotations

import ctypes
import dataclasses
import os
from typing import Callable, Iterable, Optional, Sequence

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libxvec_gpu.so")

METRIC_L2, METRIC_IP, METRIC_COSINE, METRIC_MIPSL2 = 1, 2, 3, 4
INDEX_FLAT, INDEX_SQ8_FLAT, INDEX_IVF_PQ, INDEX_RABITQ, INDEX_IVF_FLAT, INDEX_IVF_SQ8 = (
    1, 2, 3, 4, 5, 6)
INDEX_SQ4_FLAT, INDEX_IVF_SQ4, INDEX_DISKANN = 7, 8, 9
STORAGE_FP32, STORAGE_FP16 = 1, 2

STATUS_NAMES = {
    0: "OK", 1: "INVALID_ARGUMENT", 2: "OUT_OF_MEMORY", 3: "CANCELLED", 4: "TIMEOUT",
    5: "CUDA_ERROR", 6: "NCCL_ERROR", 7: "NON_FINITE", 8: "OVERFLOW", 9: "NOT_FOUND",
    10: "DUPLICATE_KEY", 11: "UNSUPPORTED", 12: "CHECKSUM_MISMATCH",
}
OK, INVALID_ARGUMENT, NON_FINITE, DUPLICATE_KEY, UNSUPPORTED, CANCELLED = 0, 1, 7, 10, 11, 3
NOT_FOUND, CHECKSUM_MISMATCH, OVERFLOW = 9, 12, 8

# Entry points of include/xvec_gpu.h (checked by the CPU test suite).
EXPORTED_SYMBOLS = (
    "xvec_gpu_abi_version", "xvec_gpu_last_error", "xvec_gpu_device_count",
    "xvec_gpu_index_create", "xvec_gpu_index_destroy", "xvec_gpu_index_len",
    "xvec_gpu_index_add", "xvec_gpu_index_add_device", "xvec_gpu_ivfpq_set_model",
    "xvec_gpu_rabitq_set_model", "xvec_gpu_index_search", "xvec_gpu_index_search_device",
    "xvec_gpu_kmeans_assign", "xvec_gpu_kmeans_assign_device", "xvec_gpu_merge_results_device",
    "xvec_gpu_stats_enable_timing", "xvec_gpu_get_stats", "xvec_gpu_reset_stats",
    "xvec_gpu_index_search_noalloc", "xvec_gpu_index_reserve",
    "xvec_gpu_index_candidate_count", "xvec_gpu_index_candidates_device",
    "xvec_gpu_index_refine_device", "xvec_gpu_kmeans_train", "xvec_gpu_kmeans_train_device",
    "xvec_gpu_ivf_set_model", "xvec_gpu_rabitq_set_model_bits", "xvec_gpu_ivf_add_with_lists",
    "xvec_gpu_ivf_file_info", "xvec_gpu_ivf_open", "xvec_gpu_kmeans_train_init_device",
    "xvec_gpu_pq_train", "xvec_gpu_pq_train_device",
    "xvec_gpu_comm_unique_id", "xvec_gpu_comm_init_rank", "xvec_gpu_comm_init_all",
    "xvec_gpu_comm_destroy", "xvec_gpu_comm_abort", "xvec_gpu_comm_size", "xvec_gpu_comm_rank",
    "xvec_gpu_sharded_search_device", "xvec_gpu_sharded_search",
    "xvec_gpu_set_wait_limit_ns",
    "xvec_gpu_rotation_signs", "xvec_gpu_rotate", "xvec_gpu_rotate_device",
    "xvec_gpu_rabitq_set_graph", "xvec_gpu_diskann_set_model", "xvec_gpu_diskann_set_graph",
)


class XvecGPUError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"{STATUS_NAMES.get(status, status)}: {message}")
        self.status = status


class IndexDesc(ctypes.Structure):
    _fields_ = [("kind", ctypes.c_int32), ("dimension", ctypes.c_int32),
                ("metric", ctypes.c_int32), ("storage", ctypes.c_int32),
                ("device", ctypes.c_int32), ("reserved", ctypes.c_int32 * 3)]


class SearchOpts(ctypes.Structure):
    _fields_ = [("top_k", ctypes.c_int32), ("radius", ctypes.c_float),
                ("nprobe", ctypes.c_int32), ("refine_scale", ctypes.c_float),
                ("ef", ctypes.c_int32), ("refine", ctypes.c_int32),
                ("filter_bitmap", ctypes.c_void_p), ("filter_words", ctypes.c_int64),
                ("stream", ctypes.c_void_p), ("cancel_flag", ctypes.c_void_p),
                ("linear", ctypes.c_int32)]


class Stats(ctypes.Structure):
    _fields_ = [("searches", ctypes.c_int64), ("queries", ctypes.c_int64),
                ("kernel_launches", ctypes.c_int64), ("exact_queries", ctypes.c_int64),
                ("scan_ms", ctypes.c_double), ("search_ms", ctypes.c_double),
                ("tensor_scans", ctypes.c_int64), ("stream_scans", ctypes.c_int64)]


def _load() -> ctypes.CDLL:
    if not os.path.exists(LIB_PATH):
        raise ImportError(f"{LIB_PATH} is missing: run `python xvec_b200/build.py` "
                          "(or __graft_entry__.build()) first")
    lib = ctypes.CDLL(LIB_PATH)
    vp, i32, i64 = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64
    lib.xvec_gpu_abi_version.restype = i32
    lib.xvec_gpu_last_error.restype = ctypes.c_size_t
    lib.xvec_gpu_last_error.argtypes = [ctypes.c_char_p, ctypes.c_size_t]
    lib.xvec_gpu_device_count.restype = i32
    lib.xvec_gpu_index_create.argtypes = [ctypes.POINTER(IndexDesc), ctypes.POINTER(vp)]
    lib.xvec_gpu_index_destroy.argtypes = [vp]
    lib.xvec_gpu_index_len.restype = i64
    lib.xvec_gpu_index_len.argtypes = [vp]
    lib.xvec_gpu_index_add.argtypes = [vp, vp, vp, i64]
    lib.xvec_gpu_index_add_device.argtypes = [vp, vp, vp, i64, vp]
    lib.xvec_gpu_ivfpq_set_model.argtypes = [vp, vp, i32, vp, i32]
    lib.xvec_gpu_rabitq_set_model.argtypes = [vp, vp, i32, vp]
    lib.xvec_gpu_rabitq_set_model_bits.argtypes = [vp, vp, i32, vp, i32, ctypes.c_double]
    lib.xvec_gpu_ivf_add_with_lists.argtypes = [vp, vp, vp, vp, i64]
    lib.xvec_gpu_ivf_file_info.argtypes = [ctypes.c_char_p, vp]
    lib.xvec_gpu_ivf_open.argtypes = [ctypes.c_char_p, i32, vp]
    lib.xvec_gpu_ivf_set_model.argtypes = [vp, vp, i32]
    lib.xvec_gpu_index_search.argtypes = [vp, vp, i32, ctypes.POINTER(SearchOpts), vp, vp, vp]
    lib.xvec_gpu_index_search_device.argtypes = [vp, vp, i32, ctypes.POINTER(SearchOpts), vp,
                                                 vp, vp]
    lib.xvec_gpu_kmeans_assign.argtypes = [i32, i32, vp, i64, vp, i32, i32, vp, vp]
    lib.xvec_gpu_kmeans_assign_device.argtypes = [i32, i32, vp, i64, vp, i32, i32, vp, vp, vp]
    lib.xvec_gpu_index_reserve.argtypes = [vp, i64]
    lib.xvec_gpu_merge_results_device.argtypes = [i32, i32, i32, i32, i32, vp, vp, vp, vp, vp,
                                                  vp, vp]
    lib.xvec_gpu_index_search_noalloc.argtypes = [vp, vp, i32, ctypes.POINTER(SearchOpts), vp,
                                                  vp, vp]
    lib.xvec_gpu_kmeans_train.argtypes = [i32, i32, vp, i64, i32, i32, i32, ctypes.c_double,
                                          ctypes.c_uint64, vp, vp, vp, vp, vp, vp]
    lib.xvec_gpu_kmeans_train_device.argtypes = [i32, i32, vp, i64, i32, i32, i32,
                                                 ctypes.c_double, ctypes.c_uint64, vp, vp, vp,
                                                 vp, vp, vp, vp]
    lib.xvec_gpu_kmeans_train_init_device.argtypes = [i32, i32, vp, i64, i32, i32, vp, i32,
                                                      ctypes.c_double, vp, vp, vp, vp, vp, vp]
    lib.xvec_gpu_pq_train.argtypes = [i32, i32, vp, i64, i32, i32, i64, i32, ctypes.c_uint64,
                                      vp, vp, vp]
    lib.xvec_gpu_pq_train_device.argtypes = [i32, i32, vp, i64, i32, i32, i64, i32,
                                             ctypes.c_uint64, vp, vp, vp, vp]
    lib.xvec_gpu_index_candidate_count.restype = i32
    lib.xvec_gpu_index_candidate_count.argtypes = [vp, ctypes.POINTER(SearchOpts)]
    lib.xvec_gpu_index_candidates_device.argtypes = [vp, vp, i32, ctypes.POINTER(SearchOpts), vp,
                                                     vp, vp]
    lib.xvec_gpu_index_refine_device.argtypes = [vp, vp, i32, vp, i32, vp, i32, ctypes.c_float,
                                                 vp, vp, vp, vp]
    lib.xvec_gpu_comm_unique_id.argtypes = [vp]
    lib.xvec_gpu_comm_init_rank.argtypes = [i32, vp, i32, i32, i32, ctypes.POINTER(vp)]
    lib.xvec_gpu_comm_init_all.argtypes = [vp, i32, i32, vp]
    lib.xvec_gpu_comm_destroy.argtypes = [vp]
    lib.xvec_gpu_comm_abort.argtypes = [vp]
    lib.xvec_gpu_comm_size.restype = i32
    lib.xvec_gpu_comm_size.argtypes = [vp]
    lib.xvec_gpu_comm_rank.restype = i32
    lib.xvec_gpu_comm_rank.argtypes = [vp]
    lib.xvec_gpu_sharded_search_device.argtypes = [vp, vp, vp, i32, ctypes.POINTER(SearchOpts),
                                                   vp, vp, vp]
    lib.xvec_gpu_sharded_search.argtypes = [vp, vp, i32, vp, i32, ctypes.POINTER(SearchOpts), vp,
                                            vp, vp]
    lib.xvec_gpu_rabitq_set_graph.argtypes = [vp, i32, i64, vp, vp, i64]
    lib.xvec_gpu_diskann_set_model.argtypes = [vp, vp, i32]
    lib.xvec_gpu_diskann_set_graph.argtypes = [vp, i64, i32, vp, vp, i64]
    lib.xvec_gpu_rotation_signs.argtypes = [ctypes.c_char_p, ctypes.c_char_p, i32, i32, i32, vp,
                                            i64]
    lib.xvec_gpu_rotate.argtypes = [i32, vp, i64, i32, vp, i64, vp, i32]
    lib.xvec_gpu_rotate_device.argtypes = [i32, vp, i64, i32, vp, i64, vp, i32, vp, vp]
    lib.xvec_gpu_set_wait_limit_ns.restype = i64
    lib.xvec_gpu_set_wait_limit_ns.argtypes = [i64]
    lib.xvec_gpu_stats_enable_timing.argtypes = [i32]
    lib.xvec_gpu_get_stats.argtypes = [ctypes.POINTER(Stats)]
    for name in EXPORTED_SYMBOLS:
        if not hasattr(lib, name):
            raise ImportError(f"{LIB_PATH} does not export {name}")
    return lib


_lib = _load()


def library() -> ctypes.CDLL:
    return _lib


def last_error() -> str:
    buf = ctypes.create_string_buffer(1024)
    _lib.xvec_gpu_last_error(buf, 1024)
    return buf.value.decode(errors="replace")


def _check(status: int) -> None:
    if status != OK:
        raise XvecGPUError(status, last_error())


def stats() -> dict:
    """xvec_gpu_get_stats as a dict (kernel launches, queries, device ms)."""
    st = Stats()
    _lib.xvec_gpu_get_stats(ctypes.byref(st))
    return {name: getattr(st, name) for name, _ in Stats._fields_}


def reset_stats() -> None:
    _lib.xvec_gpu_reset_stats()


def enable_timing(on: bool = True) -> None:
    _lib.xvec_gpu_stats_enable_timing(1 if on else 0)


def set_wait_limit_ns(ns: int) -> int:
    """Bound of the tensor-core scans' device-side waits (xvec_gpu_set_wait_limit_ns):
    2 s by default, ns <= 0 restores it; returns the previous bound."""
    return int(_lib.xvec_gpu_set_wait_limit_ns(ns))


def rotation_signs(schema_name: str, field_name: str, dimension: int, index_type: int,
                   quantize: int) -> np.ndarray:
    """collectionReformer's FHT sign state for a collection's vector field
    (collection.go:1981-2000): 4 * ((dimension + 7) / 8) bytes."""
    out = np.zeros(4 * ((dimension + 7) // 8), np.uint8)
    _check(_lib.xvec_gpu_rotation_signs(schema_name.encode(), field_name.encode(), dimension,
                                        index_type, quantize, out.ctypes.data, out.size))
    return out


class RotationReformer:
    """RotationReformer (internal/core/rotation.go:248-280) over an FHT
    rotator's sign state: transform() rotates vectors into index space,
    revert() back, both on the GPU and bit-identical to FHTRotator."""

    def __init__(self, dimension: int, signs, device: int = 0):
        self.dimension, self.device = dimension, device
        self.signs = np.ascontiguousarray(signs, np.uint8)

    def _run(self, vectors, inverse: int) -> np.ndarray:
        v = np.ascontiguousarray(vectors, np.float32)
        one = v.ndim == 1
        v = v.reshape(-1, self.dimension)
        out = np.empty_like(v)
        _check(_lib.xvec_gpu_rotate(self.device, self.signs.ctypes.data, self.signs.size,
                                    self.dimension, v.ctypes.data, v.shape[0], out.ctypes.data,
                                    inverse))
        return out[0] if one else out

    def transform(self, vectors) -> np.ndarray:
        return self._run(vectors, 0)

    def revert(self, vectors) -> np.ndarray:
        return self._run(vectors, 1)

    def transform_device(self, d_vectors: int, n: int, d_out: int, d_failed: int,
                         inverse: bool = False, stream: int = 0) -> None:
        """Device form (xvec_gpu_rotate_device): enqueued on `stream`;
        d_failed (n int32) flags vectors whose input or result is not finite."""
        _check(_lib.xvec_gpu_rotate_device(self.device, self.signs.ctypes.data, self.signs.size,
                                           self.dimension, d_vectors, n, d_out, 1 if inverse else 0,
                                           d_failed, stream or None))


def device_count() -> int:
    return int(_lib.xvec_gpu_device_count())


def _ptr(a: Optional[np.ndarray]):
    return None if a is None else a.ctypes.data


@dataclasses.dataclass
class SearchOptions:
    """core.SearchOptions (internal/core/query.go:39-55) plus the IVF/refine knobs."""
    top_k: int
    radius: float = 0.0
    filter: Optional[np.ndarray] = None  # uint32 bitmap over insertion positions
    nprobe: int = 10                     # DefaultIVFNProbe (ivf.go:380)
    refine_scale: float = 0.0            # > 0: UseRefiner with this ScaleFactor (SQ8)
    ef: int = 300                        # HNSWRaBitQSearchOptions.EF (DefaultHNSWEFSearch)
    refine: bool = True                  # HNSWRaBitQSearchOptions.Refine
    linear: bool = False                 # HNSWRaBitQSearchOptions.Linear (with a graph)


def bitmap_from_predicate(n: int, keys: Sequence[int], predicate: Callable[[int], bool]) -> np.ndarray:
    """Materialises a CandidateFilter (query.go:35) as the position bitmap the ABI takes."""
    words = np.zeros(max(1, (n + 31) // 32), np.uint32)
    for pos in range(n):
        if predicate(int(keys[pos])):
            words[pos >> 5] |= np.uint32(1 << (pos & 31))
    return words


@dataclasses.dataclass
class SearchResults:
    keys: np.ndarray    # [nq, k] uint64
    scores: np.ndarray  # [nq, k] float32
    counts: np.ndarray  # [nq] int32; negative = -(status) of a failed query

    def query(self, q: int):
        c = int(self.counts[q])
        return [(int(self.keys[q, i]), float(self.scores[q, i])) for i in range(max(c, 0))]


class _Index:
    kind = 0

    def __init__(self, dimension: int, metric: int, storage: int = STORAGE_FP32, device: int = 0):
        desc = IndexDesc(self.kind, dimension, metric, storage, device)
        handle = ctypes.c_void_p()
        _check(_lib.xvec_gpu_index_create(ctypes.byref(desc), ctypes.byref(handle)))
        self._h = handle
        self.dimension = dimension
        self.metric = metric
        self.storage = storage
        self.device = device

    def close(self) -> None:
        if getattr(self, "_h", None):
            _lib.xvec_gpu_index_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __len__(self) -> int:
        return int(_lib.xvec_gpu_index_len(self._h))

    def _row_dtype(self):
        return np.uint16 if self.storage == STORAGE_FP16 else np.float32

    def reserve(self, capacity: int) -> None:
        """Pre-sizes the index for `capacity` rows (xvec_gpu_index_reserve)."""
        _check(_lib.xvec_gpu_index_reserve(self._h, capacity))

    def add(self, keys, vectors) -> None:
        """Batch form of DenseFlatIndex.Add (flat.go:122-153)."""
        keys = np.ascontiguousarray(keys, np.uint64)
        vectors = np.ascontiguousarray(vectors, self._row_dtype())
        if vectors.ndim != 2 or vectors.shape[1] != self.dimension or vectors.shape[0] != keys.size:
            raise XvecGPUError(INVALID_ARGUMENT, "core: invalid vector dimension")
        _check(_lib.xvec_gpu_index_add(self._h, _ptr(keys), _ptr(vectors), keys.size))

    def add_device(self, keys_ptr: int, rows_ptr: int, n: int, stream: int = 0) -> None:
        _check(_lib.xvec_gpu_index_add_device(self._h, keys_ptr, rows_ptr, n, stream or None))

    def _opts(self, options: SearchOptions, stream=None, device_filter_ptr=None,
              cancel_flag=None) -> SearchOpts:
        o = SearchOpts()
        o.top_k = options.top_k
        o.radius = options.radius
        o.nprobe = options.nprobe
        o.refine_scale = options.refine_scale
        o.ef = options.ef
        o.refine = 1 if options.refine else 0
        o.linear = 1 if options.linear else 0
        if device_filter_ptr is not None:
            o.filter_bitmap = device_filter_ptr
            o.filter_words = (len(self) + 31) // 32
        elif options.filter is not None:
            f = np.ascontiguousarray(options.filter, np.uint32)
            self._keep_filter = f
            o.filter_bitmap = f.ctypes.data
            o.filter_words = f.size
        o.stream = stream
        o.cancel_flag = cancel_flag
        return o

    def search_with_options(self, queries, options: SearchOptions, raise_on_error: bool = True,
                            cancel_flag: Optional[np.ndarray] = None) -> SearchResults:
        """Batched DenseQuerySearcher.SearchWithOptions (query.go:58-61)."""
        queries = np.ascontiguousarray(queries, self._row_dtype())
        if queries.ndim == 1:
            queries = queries[None, :]
        if queries.shape[1] != self.dimension:
            raise XvecGPUError(INVALID_ARGUMENT, "core: invalid vector dimension")
        nq, k = queries.shape[0], options.top_k
        keys = np.zeros((nq, max(k, 1)), np.uint64)
        scores = np.zeros((nq, max(k, 1)), np.float32)
        counts = np.zeros(nq, np.int32)
        o = self._opts(options, cancel_flag=None if cancel_flag is None else cancel_flag.ctypes.data)
        st = _lib.xvec_gpu_index_search(self._h, _ptr(queries), nq, ctypes.byref(o), _ptr(keys),
                                        _ptr(scores), _ptr(counts))
        # Per-query failures come back as negative counts (the call's status
        # is the first one); anything else failed the whole call.
        if st != OK and (raise_on_error or not (counts < 0).any()):
            raise XvecGPUError(st, last_error())
        return SearchResults(keys[:, :k], scores[:, :k], counts)

    def search(self, queries, k: int) -> SearchResults:
        return self.search_with_options(queries, SearchOptions(top_k=k))

    def search_device(self, queries_ptr: int, nq: int, options: SearchOptions, out_keys_ptr: int,
                      out_scores_ptr: int, out_counts_ptr: int, stream: int = 0,
                      filter_ptr: Optional[int] = None) -> None:
        """Device-memory variant (xvec_gpu_index_search_device)."""
        o = self._opts(options, stream=stream or None, device_filter_ptr=filter_ptr)
        _check(_lib.xvec_gpu_index_search_device(self._h, queries_ptr, nq, ctypes.byref(o),
                                                 out_keys_ptr, out_scores_ptr, out_counts_ptr))

    def candidate_count(self, options: SearchOptions) -> int:
        """Candidates per query of a refined search's approximate stage
        (xvec_gpu_index_candidate_count); 0 without refinement."""
        o = self._opts(options)
        return int(_lib.xvec_gpu_index_candidate_count(self._h, ctypes.byref(o)))

    def candidates_device(self, queries_ptr: int, nq: int, options: SearchOptions,
                          out_keys_ptr: int, out_ranks_ptr: int, out_counts_ptr: int,
                          stream: int = 0, filter_ptr: Optional[int] = None) -> None:
        """The approximate stage of a refined search (xvec_gpu_index_candidates_device):
        keys and ranks at stride candidate_count(options); failed queries have
        negative counts."""
        o = self._opts(options, stream=stream or None, device_filter_ptr=filter_ptr)
        _check(_lib.xvec_gpu_index_candidates_device(self._h, queries_ptr, nq, ctypes.byref(o),
                                                     out_keys_ptr, out_ranks_ptr,
                                                     out_counts_ptr))

    def refine_device(self, queries_ptr: int, nq: int, cand_keys_ptr: int, cand_stride: int,
                      cand_counts_ptr: int, top_k: int, radius: float, out_keys_ptr: int,
                      out_scores_ptr: int, out_counts_ptr: int, stream: int = 0) -> None:
        """DenseRefiner.Refine of given candidate keys (xvec_gpu_index_refine_device):
        exact scores of the keys this index holds, top_k within radius."""
        _check(_lib.xvec_gpu_index_refine_device(self._h, queries_ptr, nq, cand_keys_ptr,
                                                 cand_stride, cand_counts_ptr, top_k, radius,
                                                 stream or None, out_keys_ptr, out_scores_ptr,
                                                 out_counts_ptr))


class _NoAllocMixin:
    def search_device_noalloc(self, queries_ptr: int, nq: int, options: SearchOptions,
                              out_keys_ptr: int, out_scores_ptr: int, out_counts_ptr: int,
                              stream: int = 0) -> None:
        """xvec_gpu_index_search_noalloc: the Flat search without device allocations,
        for callers that cannot allocate while searching (see include/xvec_gpu.h)."""
        o = self._opts(options, stream=stream or None)
        _check(_lib.xvec_gpu_index_search_noalloc(self._h, queries_ptr, nq, ctypes.byref(o),
                                                  out_keys_ptr, out_scores_ptr, out_counts_ptr))


class DenseFlatIndex(_NoAllocMixin, _Index):
    """core.DenseFlatIndex (internal/core/flat.go:70-196) on one B200.

    storage=STORAGE_FP16 keeps rows as binary16 bit patterns (uint16) and takes
    binary16 queries; the arithmetic is float32 on the decoded values, like a
    VectorFP16 field (collection.go:4607-4613)."""
    kind = INDEX_FLAT


class ScalarQuantizedFlatIndex(_Index):
    """core.ScalarQuantizedFlatIndex with QuantizationInt8 (quantized_index.go:28-120)."""
    kind = INDEX_SQ8_FLAT


class Int4QuantizedFlatIndex(_Index):
    """core.ScalarQuantizedFlatIndex with QuantizationInt4 (quantized_index.go:28-120,
    quantization.go:91-103, 267-321): codes in [-8, 7] held one per byte on the
    device, scanned, scored and refined by the INT8 kind's paths; rows and
    queries need an even dimension."""
    kind = INDEX_SQ4_FLAT


FP16_MAX = 65504.0


def quantize_fp16(metric: int, vectors):
    """QuantizeVector(QuantizationFP16, v) per row (quantization.go:240-265)
    after the index's metric.Compute(v, v) validation (quantized_index.go:
    233-235, 264-272): returns (IEEE binary16 bit patterns [n, d] as uint16,
    status per row: OK, NON_FINITE or OVERFLOW).  The conversion rounds to
    nearest even, as utility.Float32ToFloat16Bits does."""
    v = np.ascontiguousarray(vectors, np.float32)
    if v.ndim == 1:
        v = v[None, :]
    status = np.zeros(v.shape[0], np.int32)
    finite = np.isfinite(v).all(axis=1)
    status[~finite] = NON_FINITE
    if metric != METRIC_L2:
        with np.errstate(over="ignore", invalid="ignore"):
            selfdot = np.einsum("ij,ij->i", v.astype(np.float64), v.astype(np.float64))
        status[(status == 0) & ~(selfdot <= np.finfo(np.float32).max)] = NON_FINITE
    with np.errstate(over="ignore", invalid="ignore"):
        half = v.astype(np.float16)
    overflow = np.isinf(half).any(axis=1) & finite
    status[(status == 0) & overflow] = OVERFLOW
    half[status != 0] = 0
    return half.view(np.uint16), status


class FP16QuantizedFlatIndex:
    """core.ScalarQuantizedFlatIndex with QuantizationFP16: rows and queries
    become binary16 (quantize_fp16) and QuantizedDistance decodes both and
    applies metric.Compute (quantization.go:187-191), which is the FLAT kind
    with FP16 storage.  A row that fails conversion fails the add; a query
    that fails it fails alone (negative count)."""

    def __init__(self, dimension: int, metric: int, device: int = 0):
        self._flat = DenseFlatIndex(dimension, metric, STORAGE_FP16, device)
        self.dimension, self.metric, self.device = dimension, metric, device

    def close(self) -> None:
        self._flat.close()

    def __len__(self) -> int:
        return len(self._flat)

    def add(self, keys, vectors) -> None:
        half, status = quantize_fp16(self.metric, vectors)
        bad = np.flatnonzero(status)
        if bad.size:
            raise XvecGPUError(int(status[bad[0]]), f"core: quantize vector {int(bad[0])}")
        self._flat.add(keys, half)

    def search_with_options(self, queries, options: SearchOptions,
                            raise_on_error: bool = True) -> SearchResults:
        half, status = quantize_fp16(self.metric, queries)
        res = self._flat.search_with_options(half, options, raise_on_error=raise_on_error)
        bad = np.flatnonzero(status)
        if bad.size:
            if raise_on_error:
                raise XvecGPUError(int(status[bad[0]]), f"core: quantize query {int(bad[0])}")
            res.counts[bad] = -status[bad]
            res.keys[bad] = 0
            res.scores[bad] = 0
        return res

    def search(self, queries, k: int) -> SearchResults:
        return self.search_with_options(queries, SearchOptions(top_k=k))


class IVFPQIndex(_Index):
    """IVF list scan over 8-bit PQ codes (composition of ivf.go:524-561 and pq.go:549-595)."""
    kind = INDEX_IVF_PQ

    def set_model(self, centroids, pivots, chunks: int) -> None:
        centroids = np.ascontiguousarray(centroids, np.float32)
        pivots = np.ascontiguousarray(pivots, np.float32)
        _check(_lib.xvec_gpu_ivfpq_set_model(self._h, _ptr(centroids), centroids.shape[0],
                                             _ptr(pivots), chunks))


class IvfFileHeader(ctypes.Structure):
    _fields_ = [("count", ctypes.c_int64), ("dimension", ctypes.c_int32),
                ("nlist", ctypes.c_int32), ("metric", ctypes.c_int32),
                ("converged", ctypes.c_int32), ("options_nlist", ctypes.c_int64),
                ("options_iterations", ctypes.c_int64), ("options_workers", ctypes.c_int64),
                ("options_seed", ctypes.c_uint64), ("options_tolerance", ctypes.c_double),
                ("training_cost", ctypes.c_double), ("training_iterations", ctypes.c_int64)]


def ivf_file_info(path: str) -> dict:
    """The header of a verified ZVECIVF file (xvec_gpu_ivf_file_info)."""
    h = IvfFileHeader()
    _check(_lib.xvec_gpu_ivf_file_info(os.fsencode(path), ctypes.byref(h)))
    return {name: getattr(h, name) for name, _ in IvfFileHeader._fields_}


class IVFIndex(_Index):
    """core.IVFIndex (internal/core/ivf.go:214-597): probe the nprobe best
    centroids, exact-score the original rows of those lists."""
    kind = INDEX_IVF_FLAT

    def set_model(self, centroids) -> None:
        centroids = np.ascontiguousarray(centroids, np.float32)
        _check(_lib.xvec_gpu_ivf_set_model(self._h, _ptr(centroids), centroids.shape[0]))

    def add_with_lists(self, keys, vectors, lists) -> None:
        """Rows with their lists given (xvec_gpu_ivf_add_with_lists)."""
        keys = np.ascontiguousarray(keys, np.uint64)
        vectors = np.ascontiguousarray(vectors, np.float32)
        lists = np.ascontiguousarray(lists, np.int32)
        if vectors.ndim != 2 or vectors.shape[1] != self.dimension or \
                vectors.shape[0] != keys.size or lists.size != keys.size:
            raise XvecGPUError(INVALID_ARGUMENT, "core: invalid vector dimension")
        _check(_lib.xvec_gpu_ivf_add_with_lists(self._h, _ptr(keys), _ptr(vectors), _ptr(lists),
                                                keys.size))

    @classmethod
    def open(cls, path: str, device: int = 0) -> "IVFIndex":
        """OpenIVFIndex (ivf.go:815-830) onto the device (xvec_gpu_ivf_open);
        the file holds an exact IVF index."""
        if cls is not IVFIndex:
            raise TypeError("a ZVECIVF file opens as an IVFIndex")
        handle = ctypes.c_void_p()
        _check(_lib.xvec_gpu_ivf_open(os.fsencode(path), device, ctypes.byref(handle)))
        info = ivf_file_info(path)
        self = cls.__new__(cls)
        self._h = handle
        self.dimension = info["dimension"]
        self.metric = info["metric"]
        self.storage = STORAGE_FP32
        self.device = device
        return self


class ScalarQuantizedIVFIndex(IVFIndex):
    """core.ScalarQuantizedIVFIndex (internal/core/ivf_quantized.go:23-192):
    probe the nprobe best centroids with the original metric, score the
    probed lists' rows with INT8 codes (refine_scale > 0: exact rerank of the
    floor(top_k * scale) best codes)."""
    kind = INDEX_IVF_SQ8


class Int4QuantizedIVFIndex(IVFIndex):
    """ScalarQuantizedIVFIndex with QuantizationInt4 (ivf_quantized.go:31-54):
    the INT8 kind's probe, list scan and refine stage over INT4 codes (held
    one per byte on the device)."""
    kind = INDEX_IVF_SQ4


class RaBitQIndex(_Index):
    """HNSWRaBitQIndex search with exact refinement (hnsw_rabitq.go:539-642,
    780-801) over codes of RaBitQModelState.TotalBits bits (one bit:
    EstimateCoarse; more: Estimate on the full codes, rabitq.go:421-446): the
    linear scan, or with a graph (set_graph) the graph walk of
    searchPrepared (hnsw_rabitq.go:589-737)."""
    kind = INDEX_RABITQ

    def set_graph(self, max_level: int, entry: int, offsets, neighbors) -> None:
        """The HNSW graph over the insertion positions (xvec_gpu_rabitq_set_graph):
        node p's level-L neighbours at neighbors[offsets[L (n + 1) + p] ..
        offsets[L (n + 1) + p + 1]); max_level = -1 removes the graph."""
        if max_level < 0:
            _check(_lib.xvec_gpu_rabitq_set_graph(self._h, -1, 0, None, None, 0))
            return
        offsets = np.ascontiguousarray(offsets, np.int64)
        neighbors = np.ascontiguousarray(neighbors, np.int32)
        self._graph = (offsets, neighbors)
        _check(_lib.xvec_gpu_rabitq_set_graph(self._h, max_level, entry, offsets.ctypes.data,
                                              neighbors.ctypes.data if neighbors.size else None,
                                              neighbors.size))

    def set_model(self, centroids, rotation_signs, total_bits: int = 1,
                  extra_scale: float = 0.0) -> None:
        centroids = np.ascontiguousarray(centroids, np.float32)
        signs = np.ascontiguousarray(rotation_signs, np.uint8)
        if total_bits == 1 and extra_scale == 0.0:
            _check(_lib.xvec_gpu_rabitq_set_model(self._h, _ptr(centroids), centroids.shape[0],
                                                  _ptr(signs)))
        else:
            _check(_lib.xvec_gpu_rabitq_set_model_bits(self._h, _ptr(centroids),
                                                       centroids.shape[0], _ptr(signs),
                                                       total_bits, float(extra_scale)))


class DiskANNIndex(_Index):
    """DiskANNIndex graph search with the PQ frontier (diskann.go:472-683):
    set_model (the traversal PQ model) before adding rows, set_graph after.
    SearchOptions.ef is DiskANNSearchOptions.ListSize (0: the default 300),
    SearchOptions.linear its Linear flag."""
    kind = INDEX_DISKANN

    def set_model(self, pivots, chunks: int) -> None:
        pivots = np.ascontiguousarray(pivots, np.float32)
        _check(_lib.xvec_gpu_diskann_set_model(self._h, _ptr(pivots), chunks))

    def set_graph(self, entry: int, max_degree: int, offsets, neighbors) -> None:
        """The graph over the insertion positions: node p's neighbours at
        neighbors[offsets[p] .. offsets[p + 1]); offsets None removes it."""
        if offsets is None:
            _check(_lib.xvec_gpu_diskann_set_graph(self._h, 0, 0, None, None, 0))
            return
        offsets = np.ascontiguousarray(offsets, np.int64)
        neighbors = np.ascontiguousarray(neighbors, np.int32)
        self._graph = (offsets, neighbors)
        _check(_lib.xvec_gpu_diskann_set_graph(self._h, entry, max_degree, offsets.ctypes.data,
                                               neighbors.ctypes.data if neighbors.size else None,
                                               neighbors.size))


def kmeans_assign(metric: int, vectors, centroids, device: int = 0):
    """assignKMeans / assignKMeansCosine (kmeans.go:382-479) on the GPU."""
    vectors = np.ascontiguousarray(vectors, np.float32)
    centroids = np.ascontiguousarray(centroids, np.float32)
    n, d = vectors.shape
    labels = np.zeros(n, np.int32)
    scores = np.zeros(n, np.float32)
    _check(_lib.xvec_gpu_kmeans_assign(device, metric, _ptr(vectors), n, _ptr(centroids),
                                       centroids.shape[0], d, _ptr(labels), _ptr(scores)))
    return labels, scores


def kmeans_assign_device(device: int, metric: int, vectors_ptr: int, n: int, centroids_ptr: int,
                         nc: int, dim: int, labels_ptr: int, scores_ptr: int = 0,
                         stream: int = 0) -> None:
    """assignKMeans on device memory (xvec_gpu_kmeans_assign_device): float32
    vectors [n, dim] and centroids [nc, dim] in, int32 labels [n] (and float32
    scores [n] when scores_ptr is non-zero) out."""
    _check(_lib.xvec_gpu_kmeans_assign_device(device, metric, vectors_ptr, n, centroids_ptr, nc,
                                              dim, labels_ptr, scores_ptr or None,
                                              stream or None))


def kmeans_train(metric: int, vectors, clusters: int, iterations: int = 10,
                 tolerance: float = 1.1920928955078125e-7, seed: int = 0, device: int = 0):
    """TrainKMeans with the IVF builder's options (kmeans.go:83-92, 208-298)
    on the GPU: returns (centroids [min(clusters, n), d], labels [n],
    iterations run, converged, final cost)."""
    vectors = np.ascontiguousarray(vectors, np.float32)
    n, d = vectors.shape
    kc = min(clusters, n)
    cents = np.zeros((max(kc, 1), d), np.float32)
    labels = np.zeros(n, np.int32)
    out = (ctypes.c_int32 * 3)()
    cost = ctypes.c_double()
    _check(_lib.xvec_gpu_kmeans_train(device, metric, _ptr(vectors), n, d, clusters, iterations,
                                      tolerance, seed, _ptr(cents), _ptr(labels),
                                      ctypes.byref(out, 0), ctypes.byref(out, 4),
                                      ctypes.byref(out, 8), ctypes.byref(cost)))
    return cents[:out[0]], labels, int(out[1]), bool(out[2]), float(cost.value)


def kmeans_train_device(device: int, metric: int, vectors_ptr: int, n: int, dim: int,
                        clusters: int, centroids_ptr: int, labels_ptr: int, iterations: int = 10,
                        tolerance: float = 1.1920928955078125e-7, seed: int = 0,
                        stream: int = 0):
    """xvec_gpu_kmeans_train_device: device vectors in, device centroids
    [min(clusters, n), dim] and labels [n] out; returns (clusters,
    iterations, converged, cost)."""
    out = (ctypes.c_int32 * 3)()
    cost = ctypes.c_double()
    _check(_lib.xvec_gpu_kmeans_train_device(device, metric, vectors_ptr, n, dim, clusters,
                                             iterations, tolerance, seed, centroids_ptr,
                                             labels_ptr, ctypes.byref(out, 0),
                                             ctypes.byref(out, 4), ctypes.byref(out, 8),
                                             ctypes.byref(cost), stream or None))
    return int(out[0]), int(out[1]), bool(out[2]), float(cost.value)


def kmeans_train_init_device(device: int, metric: int, vectors_ptr: int, n: int, dim: int,
                             kc: int, initial_ptr: int, centroids_ptr: int, labels_ptr: int,
                             iterations: int = 10, tolerance: float = 1.1920928955078125e-7,
                             stream: int = 0):
    """xvec_gpu_kmeans_train_init_device: TrainKMeans from kc given initial
    centroids (kmeans.go:354-363), device memory in and out; returns
    (iterations, converged, cost)."""
    out = (ctypes.c_int32 * 2)()
    cost = ctypes.c_double()
    _check(_lib.xvec_gpu_kmeans_train_init_device(device, metric, vectors_ptr, n, dim, kc,
                                                  initial_ptr, iterations, tolerance,
                                                  centroids_ptr, labels_ptr,
                                                  ctypes.byref(out, 0), ctypes.byref(out, 4),
                                                  ctypes.byref(cost), stream or None))
    return int(out[0]), bool(out[1]), float(cost.value)


PQ_CENTROIDS = 256


def pq_train(metric: int, vectors, chunks: int = 0, max_train_samples: int = 200_000,
             max_iterations: int = 12, seed: int = 0, device: int = 0):
    """TrainPQ (pq.go:107-179) on the GPU: PQOptions{Metric, Chunks,
    MaxTrainSamples, MaxIterations, Seed}; chunks 0 means dim // 2.  Returns
    PQModelState's (chunk_offsets [chunks + 1], pivots [256, dim]), ready for
    IVFPQIndex.set_model."""
    vectors = np.ascontiguousarray(vectors, np.float32)
    if vectors.ndim != 2:
        raise ValueError("vectors must be [n, dim]")
    n, d = vectors.shape
    offsets = np.zeros(max(chunks if chunks > 0 else d // 2, 1) + 1, np.int32)
    pivots = np.zeros((PQ_CENTROIDS, max(d, 1)), np.float32)
    resolved = ctypes.c_int32()
    _check(_lib.xvec_gpu_pq_train(device, metric, _ptr(vectors), n, d, chunks, max_train_samples,
                                  max_iterations, seed, _ptr(offsets), _ptr(pivots),
                                  ctypes.byref(resolved)))
    return offsets[:resolved.value + 1].copy(), pivots


def merge_results_device(device: int, metric: int, top_k: int, nq: int, parts: int, keys_ptr: int,
                         scores_ptr: int, counts_ptr: int, out_keys_ptr: int,
                         out_scores_ptr: int, out_counts_ptr: int, stream: int = 0) -> None:
    """MergeSearchResults (query.go:154-191) over per-shard lists in device memory."""
    _check(_lib.xvec_gpu_merge_results_device(device, metric, top_k, nq, parts, keys_ptr,
                                              scores_ptr, counts_ptr, out_keys_ptr,
                                              out_scores_ptr, out_counts_ptr, stream or None))


# ---------------------------------------------------------------------------
# Multi-GPU: the library's NCCL communicator and the sharded search.
# ---------------------------------------------------------------------------
COMM_ID_BYTES = 128


def _use_pytorch_nccl() -> None:
    """Points the library at the NCCL that PyTorch links (the nvidia.nccl
    package), unless XVEC_GPU_NCCL_LIBRARY names one: a process holds one
    library of that name, and the first to load decides which, so the two must
    agree whichever loads first."""
    if os.environ.get("XVEC_GPU_NCCL_LIBRARY"):
        return
    try:
        import importlib.util
        spec = importlib.util.find_spec("nvidia.nccl")
    except (ImportError, ValueError):
        return
    for base in (spec.submodule_search_locations or []) if spec else []:
        path = os.path.join(base, "lib", "libnccl.so.2")
        if os.path.exists(path):
            os.environ["XVEC_GPU_NCCL_LIBRARY"] = path
            return


class Comm:
    """A communicator of the library (xvec_gpu_comm_*): one rank per GPU."""

    def __init__(self, handle: ctypes.c_void_p, device: int):
        self._h = handle
        self.device = device

    @staticmethod
    def unique_id() -> bytes:
        """A new communicator id (one rank makes it and sends it to the others)."""
        _use_pytorch_nccl()
        buf = (ctypes.c_uint8 * COMM_ID_BYTES)()
        _check(_lib.xvec_gpu_comm_unique_id(buf))
        return bytes(buf)

    @classmethod
    def init_rank(cls, device: int, comm_id: bytes, nranks: int, rank: int,
                  timeout_ms: int = 60000) -> "Comm":
        """This process's rank on `device` (one process per GPU)."""
        if len(comm_id) != COMM_ID_BYTES:
            raise XvecGPUError(INVALID_ARGUMENT, "communicator id must be 128 bytes")
        _use_pytorch_nccl()
        buf = (ctypes.c_uint8 * COMM_ID_BYTES).from_buffer_copy(comm_id)
        h = ctypes.c_void_p()
        _check(_lib.xvec_gpu_comm_init_rank(device, buf, nranks, rank, timeout_ms,
                                            ctypes.byref(h)))
        return cls(h, device)

    @classmethod
    def init_all(cls, devices: Sequence[int], timeout_ms: int = 60000) -> list:
        """Ranks 0..len(devices)-1 of one process, one per device."""
        _use_pytorch_nccl()
        n = len(devices)
        devs = (ctypes.c_int32 * n)(*devices)
        hs = (ctypes.c_void_p * n)()
        _check(_lib.xvec_gpu_comm_init_all(devs, n, timeout_ms, hs))
        return [cls(ctypes.c_void_p(hs[i]), devices[i]) for i in range(n)]

    @property
    def size(self) -> int:
        return int(_lib.xvec_gpu_comm_size(self._h))

    @property
    def rank(self) -> int:
        return int(_lib.xvec_gpu_comm_rank(self._h))

    def abort(self) -> None:
        _check(_lib.xvec_gpu_comm_abort(self._h))

    def close(self) -> None:
        if getattr(self, "_h", None):
            _lib.xvec_gpu_comm_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def sharded_search_device(comm: Comm, index: _Index, queries_ptr: int, nq: int,
                          options: SearchOptions, out_keys_ptr: int, out_scores_ptr: int,
                          out_counts_ptr: int, stream: int = 0,
                          filter_ptr: Optional[int] = None) -> None:
    """One rank's call of a sharded search (xvec_gpu_sharded_search_device):
    the merged results of every rank's shard in this rank's device outputs."""
    o = index._opts(options, stream=stream or None, device_filter_ptr=filter_ptr)
    _check(_lib.xvec_gpu_sharded_search_device(comm._h, index._h, queries_ptr, nq,
                                               ctypes.byref(o), out_keys_ptr, out_scores_ptr,
                                               out_counts_ptr))


def sharded_search(comms: Sequence[Comm], indexes: Sequence[_Index], queries,
                   options: SearchOptions, raise_on_error: bool = True) -> SearchResults:
    """A sharded search of one process over several GPUs
    (xvec_gpu_sharded_search): host queries in, merged host results out."""
    if options.filter is not None:
        raise XvecGPUError(INVALID_ARGUMENT, "filter a sharded search per rank "
                                             "(sharded_search_device)")
    idx0 = indexes[0]
    queries = np.ascontiguousarray(queries, idx0._row_dtype())
    if queries.ndim == 1:
        queries = queries[None, :]
    nq, k = queries.shape[0], options.top_k
    keys = np.zeros((nq, max(k, 1)), np.uint64)
    scores = np.zeros((nq, max(k, 1)), np.float32)
    counts = np.zeros(nq, np.int32)
    n = len(comms)
    ch = (ctypes.c_void_p * n)(*[c._h.value for c in comms])
    ih = (ctypes.c_void_p * n)(*[i._h.value for i in indexes])
    o = idx0._opts(options)
    st = _lib.xvec_gpu_sharded_search(ch, ih, n, _ptr(queries), nq, ctypes.byref(o), _ptr(keys),
                                      _ptr(scores), _ptr(counts))
    if st != OK and (raise_on_error or not (counts < 0).any()):
        raise XvecGPUError(st, last_error())
    return SearchResults(keys[:, :k], scores[:, :k], counts)
