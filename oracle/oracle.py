"""ctypes front end of the CPU oracle (test infrastructure only).

The oracle restates the xvec search hot path on the CPU (see
``oracle/xvec_oracle.cpp``); only ``tests/``, ``__graft_entry__.smoke()`` and
the CPU-baseline leg of ``bench.py`` import this module, always as the checker
or the reported baseline, never as a code path of the shipped library.

``ReferenceFloats`` loads the reference's own AVX-512/AVX kernels
(``internal/floats/src/floats_avx512.c`` and ``floats_avx.c``), compiled in
place by ``make -C oracle ref`` into ``oracle/_ref/``.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_build", "libxvec_oracle.so")
REF_PATH = os.path.join(HERE, "_ref", "libxvec_floats_ref.so")

L2, IP, COSINE, MIPSL2 = 1, 2, 3, 4
OK, INVALID_ARGUMENT, NON_FINITE, OVERFLOW = 0, 1, 7, 8

_f32p = ctypes.POINTER(ctypes.c_float)
_f64p = ctypes.POINTER(ctypes.c_double)
_u64p = ctypes.POINTER(ctypes.c_uint64)
_i64p = ctypes.POINTER(ctypes.c_int64)
_i32p = ctypes.POINTER(ctypes.c_int32)
_u32p = ctypes.POINTER(ctypes.c_uint32)
_u8p = ctypes.POINTER(ctypes.c_uint8)
_i8p = ctypes.POINTER(ctypes.c_int8)


class SQParams(ctypes.Structure):
    _fields_ = [("inverse_scale", ctypes.c_float), ("offset", ctypes.c_float),
                ("code_sum", ctypes.c_double), ("code_square", ctypes.c_double)]


SQ_PARAMS_DTYPE = np.dtype([("inverse_scale", "<f4"), ("offset", "<f4"),
                            ("code_sum", "<f8"), ("code_square", "<f8")])


class RaBitQFactors(ctypes.Structure):
    _fields_ = [("cluster", ctypes.c_int32), ("pad_", ctypes.c_int32),
                ("coarse_add", ctypes.c_double), ("coarse_rescale", ctypes.c_double),
                ("coarse_error", ctypes.c_double), ("full_add", ctypes.c_double),
                ("full_rescale", ctypes.c_double)]


RABITQ_FACTORS_DTYPE = np.dtype([("cluster", "<i4"), ("pad_", "<i4"), ("coarse_add", "<f8"),
                                 ("coarse_rescale", "<f8"), ("coarse_error", "<f8"),
                                 ("full_add", "<f8"), ("full_rescale", "<f8")])


def collection_rotation_signs(schema: str, field: str, dimension: int, index_type: int,
                              quantize: int) -> np.ndarray:
    """collectionReformer's sign state (collection.go:1981-2000): the bytes of
    SHA-256 over the seed text followed by a little-endian uint64 counter,
    counters 0, 1, ... concatenated until 4 ((dimension + 7) / 8) bytes."""
    import hashlib
    import struct
    seed = ("zvec-go-rotation-v1\x00%s\x00%s\x00%d\x00%d\x00%d"
            % (schema, field, dimension, index_type, quantize)).encode()
    want = 4 * ((dimension + 7) // 8)
    out, counter = b"", 0
    while len(out) < want:
        out += hashlib.sha256(seed + struct.pack("<Q", counter)).digest()
        counter += 1
    return np.frombuffer(out[:want], np.uint8).copy()


def build(reference: str | None = None) -> None:
    """Compile the restatement and, when `reference` (else the XVEC_REFERENCE
    environment variable) names an existing reference checkout, its C kernels."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    reference = reference or os.environ.get("XVEC_REFERENCE")
    if reference and os.path.isdir(reference):
        subprocess.run(["make", "-s", "-C", HERE, "ref", "REFERENCE=" + reference], check=True)


def _ptr(a: np.ndarray | None, typ):
    if a is None:
        return None
    return a.ctypes.data_as(typ)


def _c(a, dtype):
    return np.ascontiguousarray(a, dtype=dtype)


class Oracle:
    def __init__(self, path: str = LIB_PATH):
        if not os.path.exists(path):
            build(reference=False)
        lib = ctypes.CDLL(path)
        self.lib = lib
        lib.xo_l2_squared.restype = ctypes.c_float
        lib.xo_l2_squared.argtypes = [_f32p, _f32p, ctypes.c_int64]
        lib.xo_inner_product.restype = ctypes.c_float
        lib.xo_inner_product.argtypes = [_f32p, _f32p, ctypes.c_int64]
        lib.xo_dot_norms.argtypes = [_f32p, _f32p, ctypes.c_int64, _f32p, _f32p, _f32p]
        lib.xo_metric_compute.argtypes = [ctypes.c_int, _f32p, _f32p, ctypes.c_int64, _f32p]
        lib.xo_f32_to_f16.restype = ctypes.c_uint16
        lib.xo_f32_to_f16.argtypes = [ctypes.c_float]
        lib.xo_f16_to_f32.restype = ctypes.c_float
        lib.xo_f16_to_f32.argtypes = [ctypes.c_uint16]
        search_tail = [_i32p, _u64p, _f32p, _i32p, _i32p]
        lib.xo_flat_search.argtypes = [ctypes.c_int, _f32p, _u64p, ctypes.c_int64, ctypes.c_int32,
                                       _f32p, ctypes.c_int32, ctypes.c_int32, ctypes.c_float,
                                       _u32p, ctypes.c_int32, _u64p, _f32p, _i32p, _i32p]
        lib.xo_merge_results.restype = ctypes.c_int32
        lib.xo_merge_results.argtypes = [ctypes.c_int, ctypes.c_int32, _u64p, _f32p,
                                         ctypes.c_int64, _u64p, _f32p]
        lib.xo_quantize_int8.argtypes = [_f32p, ctypes.c_int32, _i8p, ctypes.POINTER(SQParams)]
        lib.xo_quantize_int4.argtypes = [_f32p, ctypes.c_int32, _u8p, ctypes.POINTER(SQParams)]
        lib.xo_quantized_distance_int8.argtypes = [ctypes.c_int, _i8p, ctypes.POINTER(SQParams),
                                                   _i8p, ctypes.POINTER(SQParams),
                                                   ctypes.c_int32, _f32p]
        lib.xo_quantize_int8_batch.argtypes = [_f32p, ctypes.c_int64, ctypes.c_int32,
                                               ctypes.c_int32, _i8p, ctypes.c_void_p]
        lib.xo_refinement_candidate_count.argtypes = [ctypes.c_int32, ctypes.c_float, _i32p]
        lib.xo_sq8_search.argtypes = [ctypes.c_int, _i8p, ctypes.c_void_p, _f32p, _u64p,
                                      ctypes.c_int64, ctypes.c_int32, _f32p, ctypes.c_int32,
                                      ctypes.c_int32, ctypes.c_float, ctypes.c_float, _u32p,
                                      ctypes.c_int32, _u64p, _f32p, _i32p, _i32p]
        lib.xo_quantize_int4_batch.argtypes = [_f32p, ctypes.c_int64, ctypes.c_int32,
                                               ctypes.c_int32, _u8p, ctypes.c_void_p]
        lib.xo_quantized_distance_int4.argtypes = [ctypes.c_int, _u8p, ctypes.POINTER(SQParams),
                                                   _u8p, ctypes.POINTER(SQParams),
                                                   ctypes.c_int32, _f32p]
        lib.xo_sq4_search.argtypes = [ctypes.c_int, _u8p, ctypes.c_void_p, _f32p, _u64p,
                                      ctypes.c_int64, ctypes.c_int32, _f32p, ctypes.c_int32,
                                      ctypes.c_int32, ctypes.c_float, ctypes.c_float, _u32p,
                                      ctypes.c_int32, _u64p, _f32p, _i32p, _i32p]
        lib.xo_splitmix64_next.restype = ctypes.c_uint64
        lib.xo_splitmix64_next.argtypes = [_u64p]
        lib.xo_kmeans_reservoir.argtypes = [ctypes.c_int64, ctypes.c_int32, ctypes.c_uint64, _i64p]
        lib.xo_kmeans_assign.argtypes = [ctypes.c_int, _f32p, ctypes.c_int64, _f32p,
                                         ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, _i32p,
                                         _f32p]
        lib.xo_kmeans_train.argtypes = [ctypes.c_int, _f32p, ctypes.c_int64, ctypes.c_int32,
                                        ctypes.c_int32, ctypes.c_int32, ctypes.c_double,
                                        ctypes.c_uint64, ctypes.c_int32, _f32p, _i32p, _i32p]
        lib.xo_ivf_probe.restype = ctypes.c_int32
        lib.xo_ivf_probe.argtypes = [ctypes.c_int, _f32p, ctypes.c_int32, ctypes.c_int32, _f32p,
                                     ctypes.c_int32, _i32p]
        lib.xo_ivf_flat_search.argtypes = [ctypes.c_int, _f32p, _u64p, ctypes.c_int64,
                                           ctypes.c_int32, _f32p, ctypes.c_int32, _i64p, _i64p,
                                           _f32p, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
                                           ctypes.c_float, _u32p, ctypes.c_int32, _u64p, _f32p,
                                           _i32p, _i32p]
        lib.xo_ivf_sq8_search.argtypes = [ctypes.c_int, _i8p, ctypes.c_void_p, _f32p, _u64p,
                                          ctypes.c_int64, ctypes.c_int32, _f32p, ctypes.c_int32,
                                          _i64p, _i64p, _f32p, ctypes.c_int32, ctypes.c_int32,
                                          ctypes.c_int32, ctypes.c_float, ctypes.c_float, _u32p,
                                          ctypes.c_int32, _u64p, _f32p, _i32p, _i32p]
        lib.xo_pq_chunk_offsets.argtypes = [ctypes.c_int32, ctypes.c_int32, _i32p]
        lib.xo_kmeans_train_init.argtypes = [ctypes.c_int, _f32p, ctypes.c_int64, ctypes.c_int32,
                                             ctypes.c_int32, _f32p, ctypes.c_int32,
                                             ctypes.c_double, ctypes.c_int32, _f32p, _i32p]
        lib.xo_pq_kmc2.argtypes = [ctypes.c_int, _f32p, ctypes.c_int64, ctypes.c_int32,
                                   ctypes.c_int32, ctypes.c_uint64, _f32p]
        lib.xo_pq_train.argtypes = [ctypes.c_int, _f32p, ctypes.c_int64, ctypes.c_int32,
                                    ctypes.c_int32, ctypes.c_int64, ctypes.c_int32,
                                    ctypes.c_uint64, ctypes.c_int32, _f32p]
        lib.xo_pq_encode.argtypes = [ctypes.c_int, _f32p, _i32p, ctypes.c_int32, ctypes.c_int32,
                                     _f32p, _u8p]
        lib.xo_pq_distance_table.argtypes = [ctypes.c_int, _f32p, _i32p, ctypes.c_int32,
                                             ctypes.c_int32, _f32p, _f32p]
        lib.xo_pq_lookup.argtypes = [_f32p, ctypes.c_int32, _u8p, _f32p]
        lib.xo_ivfpq_search.argtypes = [ctypes.c_int, _f32p, ctypes.c_int32, ctypes.c_int32,
                                        _f32p, _i32p, ctypes.c_int32, _u8p, _u64p, _i64p, _i64p,
                                        _f32p, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
                                        ctypes.c_float, _u32p, ctypes.c_int32, _u64p, _f32p,
                                        _i32p, _i32p]
        lib.xo_fht_rotate.argtypes = [ctypes.c_int32, _u8p, _f32p, _f32p]
        lib.xo_fht_unrotate.argtypes = [ctypes.c_int32, _u8p, _f32p, _f32p]
        lib.xo_rabitq_padded_dimension.restype = ctypes.c_int32
        lib.xo_rabitq_padded_dimension.argtypes = [ctypes.c_int32]
        lib.xo_rabitq_rotate.argtypes = [ctypes.c_int32, _u8p, _f32p, _f32p]
        lib.xo_rabitq_quantize.argtypes = [_f32p, _f32p, ctypes.c_int32, ctypes.c_int32,
                                           ctypes.c_int32, ctypes.c_double, ctypes.c_int32,
                                           _u8p, _u8p, ctypes.POINTER(RaBitQFactors)]
        lib.xo_rabitq_encode1.argtypes = [ctypes.c_int, ctypes.c_int32, _f32p, ctypes.c_int32,
                                          _u8p, _f32p, _u8p, ctypes.POINTER(RaBitQFactors)]
        lib.xo_rabitq_encode.argtypes = [ctypes.c_int, ctypes.c_int32, _f32p, ctypes.c_int32,
                                         _u8p, ctypes.c_int32, ctypes.c_double, _f32p, _u8p,
                                         _u8p, ctypes.POINTER(RaBitQFactors)]
        lib.xo_rabitq_estimate.argtypes = [_f32p, ctypes.c_int32, ctypes.c_double, _f64p, _f64p,
                                           ctypes.c_int32, _u8p, _u8p,
                                           ctypes.POINTER(RaBitQFactors), _f32p]
        lib.xo_rabitq_search_bits.argtypes = [ctypes.c_int, ctypes.c_int32, _f32p,
                                              ctypes.c_int32, _u8p, ctypes.c_int32, _u8p, _u8p,
                                              ctypes.c_void_p, _f32p, _u64p, ctypes.c_int64,
                                              _f32p, ctypes.c_int32, ctypes.c_int32,
                                              ctypes.c_int32, ctypes.c_int32, ctypes.c_float,
                                              _u32p, ctypes.c_int32, _u64p, _f32p, _i32p, _i32p]
        lib.xo_hnsw_rabitq_search.argtypes = [ctypes.c_int, ctypes.c_int32, _f32p,
                                              ctypes.c_int32, _u8p, ctypes.c_int32, _u8p, _u8p,
                                              ctypes.c_void_p, _f32p, _u64p, ctypes.c_int64,
                                              ctypes.c_int32, ctypes.c_int64, _i64p, _i32p,
                                              _f32p, ctypes.c_int32, ctypes.c_int32,
                                              ctypes.c_int32, ctypes.c_int32, ctypes.c_float,
                                              _u32p, ctypes.c_int32, _u64p, _f32p, _i32p, _i32p]
        lib.xo_pq_encode_rows.argtypes = [ctypes.c_int, _f32p, _i32p, ctypes.c_int32,
                                          ctypes.c_int32, _f32p, ctypes.c_int64, ctypes.c_int32,
                                          _u8p]
        lib.xo_rabitq_encode_rows.argtypes = [ctypes.c_int, ctypes.c_int32, _f32p, ctypes.c_int32,
                                              _u8p, ctypes.c_int32, ctypes.c_double, _f32p,
                                              ctypes.c_int64, ctypes.c_int32, _u8p, _u8p,
                                              ctypes.c_int64, ctypes.c_void_p]
        lib.xo_diskann_code_norms.argtypes = [_f32p, _i32p, ctypes.c_int32, ctypes.c_int32,
                                              _u8p, ctypes.c_int64, _f32p]
        lib.xo_diskann_code_norms.restype = None
        lib.xo_diskann_search.argtypes = [ctypes.c_int, ctypes.c_int32, _f32p, _i32p,
                                          ctypes.c_int32, _u8p, _f32p, _f32p, _u64p,
                                          ctypes.c_int64, ctypes.c_int64, _i64p, _i32p,
                                          ctypes.c_int32, _f32p, ctypes.c_int32, ctypes.c_int32,
                                          ctypes.c_int32, ctypes.c_float, _u32p, ctypes.c_int32,
                                          _u64p, _f32p, _i32p, _i32p]
        lib.xo_rabitq_prepare_query.argtypes = [ctypes.c_int, ctypes.c_int32, _f32p,
                                                ctypes.c_int32, _u8p, _f32p, _f32p, _f64p, _f64p,
                                                _f64p]
        lib.xo_rabitq_estimate_coarse.argtypes = [_f32p, ctypes.c_int32, ctypes.c_double, _f64p,
                                                  _f64p, _u8p, ctypes.POINTER(RaBitQFactors),
                                                  _f32p]
        lib.xo_rabitq_search.argtypes = [ctypes.c_int, ctypes.c_int32, _f32p, ctypes.c_int32,
                                         _u8p, _u8p, ctypes.c_void_p, _f32p, _u64p,
                                         ctypes.c_int64, _f32p, ctypes.c_int32, ctypes.c_int32,
                                         ctypes.c_int32, ctypes.c_int32, ctypes.c_float, _u32p,
                                         ctypes.c_int32, _u64p, _f32p, _i32p, _i32p]
        del search_tail
        lib.xo_use_reference_kernels.argtypes = [ctypes.c_void_p] * 6
        self.kernels = "restated"

    def use_reference_kernels(self, ref: "ReferenceFloats | None") -> None:
        """Dispatch the distance kernels to the reference's compiled C (or back)."""
        if ref is None:
            self.lib.xo_use_reference_kernels(None, None, None, None, None, None)
            self.kernels = "restated"
            return
        names = ("xvec_avx512_l2_squared", "xvec_avx512_inner_product", "xvec_avx512_dot_norms",
                 "xvec_avx_l2_squared", "xvec_avx_inner_product", "xvec_avx_dot_norms")
        ptrs = [ctypes.cast(getattr(ref.lib, n), ctypes.c_void_p).value for n in names]
        self.lib.xo_use_reference_kernels(*ptrs)
        self.kernels = "reference"

    # ---- distances ---------------------------------------------------------
    def l2_squared(self, a, b) -> float:
        a, b = _c(a, np.float32), _c(b, np.float32)
        return float(np.float32(self.lib.xo_l2_squared(_ptr(a, _f32p), _ptr(b, _f32p), a.size)))

    def inner_product(self, a, b) -> float:
        a, b = _c(a, np.float32), _c(b, np.float32)
        return float(np.float32(self.lib.xo_inner_product(_ptr(a, _f32p), _ptr(b, _f32p), a.size)))

    def dot_norms(self, a, b):
        a, b = _c(a, np.float32), _c(b, np.float32)
        out = np.zeros(3, np.float32)
        self.lib.xo_dot_norms(_ptr(a, _f32p), _ptr(b, _f32p), a.size, _ptr(out[0:1], _f32p),
                              _ptr(out[1:2], _f32p), _ptr(out[2:3], _f32p))
        return out

    def metric_compute(self, metric: int, a, b):
        """Returns (status, score) like metric.Compute."""
        a, b = _c(a, np.float32), _c(b, np.float32)
        out = np.zeros(1, np.float32)
        st = self.lib.xo_metric_compute(metric, _ptr(a, _f32p), _ptr(b, _f32p), a.size,
                                        _ptr(out, _f32p))
        return st, np.float32(out[0])

    def f32_to_f16(self, values) -> np.ndarray:
        v = np.asarray(values, np.float32).ravel()
        return np.array([self.lib.xo_f32_to_f16(float(x)) for x in v], np.uint16)

    def f16_to_f32(self, bits) -> np.ndarray:
        b = np.asarray(bits, np.uint16).ravel()
        return np.array([self.lib.xo_f16_to_f32(int(x)) for x in b], np.float32)

    # ---- searches ------------------------------------------------------------
    @staticmethod
    def _outs(nq, k):
        return (np.zeros(nq * k, np.uint64), np.zeros(nq * k, np.float32),
                np.zeros(nq, np.int32), np.zeros(nq, np.int32))

    def flat_search(self, metric, rows, keys, queries, k, radius=0.0, bitmap=None, threads=0):
        rows = _c(rows, np.float32)
        queries = _c(queries, np.float32)
        keys = _c(keys, np.uint64)
        n, d = rows.shape
        nq = queries.shape[0]
        ok, os_, oc, ost = self._outs(nq, k)
        bm = None if bitmap is None else _c(bitmap, np.uint32)
        st = self.lib.xo_flat_search(metric, _ptr(rows, _f32p), _ptr(keys, _u64p), n, d,
                                     _ptr(queries, _f32p), nq, k, radius, _ptr(bm, _u32p),
                                     threads or os.cpu_count(), _ptr(ok, _u64p),
                                     _ptr(os_, _f32p), _ptr(oc, _i32p), _ptr(ost, _i32p))
        return st, ok.reshape(nq, k), os_.reshape(nq, k), oc, ost

    def merge_results(self, metric, k, keys, scores):
        keys = _c(keys, np.uint64)
        scores = _c(scores, np.float32)
        ok = np.zeros(max(k, 1), np.uint64)
        os_ = np.zeros(max(k, 1), np.float32)
        c = self.lib.xo_merge_results(metric, k, _ptr(keys, _u64p), _ptr(scores, _f32p),
                                      keys.size, _ptr(ok, _u64p), _ptr(os_, _f32p))
        return ok[:c], os_[:c]

    def quantize_int8(self, v):
        v = _c(v, np.float32)
        codes = np.zeros(v.size, np.int8)
        p = SQParams()
        st = self.lib.xo_quantize_int8(_ptr(v, _f32p), v.size, _ptr(codes, _i8p), ctypes.byref(p))
        return st, codes, p

    def quantize_int8_batch(self, rows, threads=0):
        rows = _c(rows, np.float32)
        n, d = rows.shape
        codes = np.zeros((n, d), np.int8)
        params = np.zeros(n, SQ_PARAMS_DTYPE)
        st = self.lib.xo_quantize_int8_batch(_ptr(rows, _f32p), n, d, threads or os.cpu_count(),
                                             _ptr(codes, _i8p), params.ctypes.data)
        if st != OK:
            raise ValueError(f"quantize rows: status {st}")
        return codes, params

    def quantize_int4(self, v):
        v = _c(v, np.float32)
        packed = np.zeros(v.size // 2, np.uint8)
        p = SQParams()
        st = self.lib.xo_quantize_int4(_ptr(v, _f32p), v.size, _ptr(packed, _u8p), ctypes.byref(p))
        return st, packed, p

    def quantize_int4_batch(self, rows, threads=0):
        """QuantizeVector(QuantizationInt4, row) per row: packed [n, d / 2]."""
        rows = _c(rows, np.float32)
        n, d = rows.shape
        packed = np.zeros((n, d // 2), np.uint8)
        params = np.zeros(n, SQ_PARAMS_DTYPE)
        st = self.lib.xo_quantize_int4_batch(_ptr(rows, _f32p), n, d, threads or os.cpu_count(),
                                             _ptr(packed, _u8p), params.ctypes.data)
        if st != OK:
            raise ValueError(f"quantize rows: status {st}")
        return packed, params

    def quantized_distance_int4(self, metric, lcodes, lp, rcodes, rp, d):
        lcodes, rcodes = _c(lcodes, np.uint8), _c(rcodes, np.uint8)
        out = np.zeros(1, np.float32)
        st = self.lib.xo_quantized_distance_int4(metric, _ptr(lcodes, _u8p), ctypes.byref(lp),
                                                 _ptr(rcodes, _u8p), ctypes.byref(rp), d,
                                                 _ptr(out, _f32p))
        return st, np.float32(out[0])

    def quantized_distance_int8(self, metric, lcodes, lp, rcodes, rp):
        lcodes, rcodes = _c(lcodes, np.int8), _c(rcodes, np.int8)
        out = np.zeros(1, np.float32)
        st = self.lib.xo_quantized_distance_int8(metric, _ptr(lcodes, _i8p), ctypes.byref(lp),
                                                 _ptr(rcodes, _i8p), ctypes.byref(rp),
                                                 lcodes.size, _ptr(out, _f32p))
        return st, np.float32(out[0])

    def refinement_candidate_count(self, k, scale):
        out = np.zeros(1, np.int32)
        st = self.lib.xo_refinement_candidate_count(k, scale, _ptr(out, _i32p))
        return st, int(out[0])

    def sq8_search(self, metric, codes, params, originals, keys, queries, k, radius=0.0,
                   refine_scale=0.0, bitmap=None, threads=0):
        codes = _c(codes, np.int8)
        params = np.ascontiguousarray(params, SQ_PARAMS_DTYPE)
        originals = _c(originals, np.float32)
        keys = _c(keys, np.uint64)
        queries = _c(queries, np.float32)
        n, d = codes.shape
        nq = queries.shape[0]
        ok, os_, oc, ost = self._outs(nq, k)
        bm = None if bitmap is None else _c(bitmap, np.uint32)
        st = self.lib.xo_sq8_search(metric, _ptr(codes, _i8p), params.ctypes.data,
                                    _ptr(originals, _f32p), _ptr(keys, _u64p), n, d,
                                    _ptr(queries, _f32p), nq, k, radius, refine_scale,
                                    _ptr(bm, _u32p), threads or os.cpu_count(), _ptr(ok, _u64p),
                                    _ptr(os_, _f32p), _ptr(oc, _i32p), _ptr(ost, _i32p))
        return st, ok.reshape(nq, k), os_.reshape(nq, k), oc, ost

    def sq4_search(self, metric, packed, params, originals, keys, queries, k, radius=0.0,
                   refine_scale=0.0, bitmap=None, threads=0):
        """xo_sq4_search: the SQ-Flat search over INT4 codes (packed [n, d / 2])."""
        packed = _c(packed, np.uint8)
        params = np.ascontiguousarray(params, SQ_PARAMS_DTYPE)
        originals = _c(originals, np.float32)
        keys = _c(keys, np.uint64)
        queries = _c(queries, np.float32)
        n, d = originals.shape[0], queries.shape[1]
        nq = queries.shape[0]
        ok, os_, oc, ost = self._outs(nq, k)
        bm = None if bitmap is None else _c(bitmap, np.uint32)
        st = self.lib.xo_sq4_search(metric, _ptr(packed, _u8p), params.ctypes.data,
                                    _ptr(originals, _f32p), _ptr(keys, _u64p), n, d,
                                    _ptr(queries, _f32p), nq, k, radius, refine_scale,
                                    _ptr(bm, _u32p), threads or os.cpu_count(), _ptr(ok, _u64p),
                                    _ptr(os_, _f32p), _ptr(oc, _i32p), _ptr(ost, _i32p))
        return st, ok.reshape(nq, k), os_.reshape(nq, k), oc, ost

    def splitmix64(self, seed: int, count: int) -> np.ndarray:
        state = np.array([seed], np.uint64)
        return np.array([self.lib.xo_splitmix64_next(_ptr(state, _u64p)) for _ in range(count)],
                        np.uint64)

    def kmeans_reservoir(self, n, clusters, seed):
        out = np.zeros(clusters, np.int64)
        self.lib.xo_kmeans_reservoir(n, clusters, seed, _ptr(out, _i64p))
        return out

    def kmeans_assign(self, metric, vectors, centroids, threads=0):
        vectors = _c(vectors, np.float32)
        centroids = _c(centroids, np.float32)
        n, d = vectors.shape
        labels = np.zeros(n, np.int32)
        scores = np.zeros(n, np.float32)
        st = self.lib.xo_kmeans_assign(metric, _ptr(vectors, _f32p), n, _ptr(centroids, _f32p),
                                       centroids.shape[0], d, threads or os.cpu_count(),
                                       _ptr(labels, _i32p), _ptr(scores, _f32p))
        return st, labels, scores

    def kmeans_train(self, metric, vectors, clusters, iterations=10,
                     tolerance=1.1920928955078125e-7, seed=0, threads=0):
        vectors = _c(vectors, np.float32)
        n, d = vectors.shape
        cents = np.zeros((clusters, d), np.float32)
        kc = np.zeros(1, np.int32)
        labels = np.zeros(n, np.int32)
        st = self.lib.xo_kmeans_train(metric, _ptr(vectors, _f32p), n, d, clusters, iterations,
                                      tolerance, seed, threads or os.cpu_count(),
                                      _ptr(cents, _f32p), _ptr(kc, _i32p), _ptr(labels, _i32p))
        return st, cents[: int(kc[0])], labels

    def ivf_probe(self, metric, centroids, query, nprobe):
        centroids = _c(centroids, np.float32)
        query = _c(query, np.float32)
        lists = np.zeros(min(nprobe, centroids.shape[0]), np.int32)
        c = self.lib.xo_ivf_probe(metric, _ptr(centroids, _f32p), centroids.shape[0],
                                  centroids.shape[1], _ptr(query, _f32p), nprobe,
                                  _ptr(lists, _i32p))
        return lists[:c]

    def ivf_flat_search(self, metric, rows, keys, centroids, list_offsets, list_positions,
                        queries, k, nprobe, radius=0.0, bitmap=None, threads=0):
        rows = _c(rows, np.float32)
        keys = _c(keys, np.uint64)
        centroids = _c(centroids, np.float32)
        lo = _c(list_offsets, np.int64)
        lp = _c(list_positions, np.int64)
        queries = _c(queries, np.float32)
        n, d = rows.shape
        nq = queries.shape[0]
        ok, os_, oc, ost = self._outs(nq, k)
        bm = None if bitmap is None else _c(bitmap, np.uint32)
        st = self.lib.xo_ivf_flat_search(metric, _ptr(rows, _f32p), _ptr(keys, _u64p), n, d,
                                         _ptr(centroids, _f32p), centroids.shape[0],
                                         _ptr(lo, _i64p), _ptr(lp, _i64p), _ptr(queries, _f32p),
                                         nq, k, nprobe, radius, _ptr(bm, _u32p),
                                         threads or os.cpu_count(), _ptr(ok, _u64p),
                                         _ptr(os_, _f32p), _ptr(oc, _i32p), _ptr(ost, _i32p))
        return st, ok.reshape(nq, k), os_.reshape(nq, k), oc, ost

    def ivf_sq8_search(self, metric, codes, params, originals, keys, centroids, list_offsets,
                       list_positions, queries, k, nprobe, radius=0.0, refine_scale=0.0,
                       bitmap=None, threads=0):
        codes = _c(codes, np.int8)
        params = np.ascontiguousarray(params, SQ_PARAMS_DTYPE)
        originals = _c(originals, np.float32)
        keys = _c(keys, np.uint64)
        centroids = _c(centroids, np.float32)
        lo = _c(list_offsets, np.int64)
        lp = _c(list_positions, np.int64)
        queries = _c(queries, np.float32)
        n, d = codes.shape
        nq = queries.shape[0]
        ok, os_, oc, ost = self._outs(nq, k)
        bm = None if bitmap is None else _c(bitmap, np.uint32)
        st = self.lib.xo_ivf_sq8_search(metric, _ptr(codes, _i8p), params.ctypes.data,
                                        _ptr(originals, _f32p), _ptr(keys, _u64p), n, d,
                                        _ptr(centroids, _f32p), centroids.shape[0],
                                        _ptr(lo, _i64p), _ptr(lp, _i64p), _ptr(queries, _f32p),
                                        nq, k, nprobe, radius, refine_scale, _ptr(bm, _u32p),
                                        threads or os.cpu_count(), _ptr(ok, _u64p),
                                        _ptr(os_, _f32p), _ptr(oc, _i32p), _ptr(ost, _i32p))
        return st, ok.reshape(nq, k), os_.reshape(nq, k), oc, ost

    def pq_kmc2(self, metric, vectors, clusters, seed):
        """initializePQKMC2 (pq.go:410-459)."""
        vectors = _c(vectors, np.float32)
        n, d = vectors.shape
        out = np.zeros((clusters, d), np.float32)
        st = self.lib.xo_pq_kmc2(metric, _ptr(vectors, _f32p), n, d, clusters, seed,
                                 _ptr(out, _f32p))
        return st, out

    def kmeans_train_init(self, metric, vectors, initial, iterations,
                          tolerance=1.1920928955078125e-7, threads=0):
        vectors = _c(vectors, np.float32)
        initial = _c(initial, np.float32)
        n, d = vectors.shape
        kc = initial.shape[0]
        cents = np.zeros((kc, d), np.float32)
        labels = np.zeros(n, np.int32)
        st = self.lib.xo_kmeans_train_init(metric, _ptr(vectors, _f32p), n, d, kc,
                                           _ptr(initial, _f32p), iterations, tolerance,
                                           threads or os.cpu_count(), _ptr(cents, _f32p),
                                           _ptr(labels, _i32p))
        return st, cents, labels

    def pq_train(self, metric, vectors, chunks, max_train_samples=200_000, max_iterations=12,
                 seed=0, threads=0):
        """TrainPQ (pq.go:107-179): pivots [256][d]."""
        vectors = _c(vectors, np.float32)
        n, d = vectors.shape
        pivots = np.zeros((256, d), np.float32)
        st = self.lib.xo_pq_train(metric, _ptr(vectors, _f32p), n, d, chunks, max_train_samples,
                                  max_iterations, seed, threads or os.cpu_count(),
                                  _ptr(pivots, _f32p))
        return st, pivots

    def pq_chunk_offsets(self, d, chunks):
        out = np.zeros(chunks + 1, np.int32)
        self.lib.xo_pq_chunk_offsets(d, chunks, _ptr(out, _i32p))
        return out

    def pq_encode(self, metric, pivots, offsets, v):
        pivots = _c(pivots, np.float32)
        offsets = _c(offsets, np.int32)
        v = _c(v, np.float32)
        chunks = offsets.size - 1
        code = np.zeros(chunks, np.uint8)
        st = self.lib.xo_pq_encode(metric, _ptr(pivots, _f32p), _ptr(offsets, _i32p), chunks,
                                   v.size, _ptr(v, _f32p), _ptr(code, _u8p))
        return st, code

    def pq_distance_table(self, metric, pivots, offsets, query):
        pivots = _c(pivots, np.float32)
        offsets = _c(offsets, np.int32)
        query = _c(query, np.float32)
        chunks = offsets.size - 1
        table = np.zeros(chunks * 256, np.float32)
        st = self.lib.xo_pq_distance_table(metric, _ptr(pivots, _f32p), _ptr(offsets, _i32p),
                                           chunks, query.size, _ptr(query, _f32p),
                                           _ptr(table, _f32p))
        return st, table

    def pq_lookup(self, table, code):
        table = _c(table, np.float32)
        code = _c(code, np.uint8)
        out = np.zeros(1, np.float32)
        st = self.lib.xo_pq_lookup(_ptr(table, _f32p), code.size, _ptr(code, _u8p),
                                   _ptr(out, _f32p))
        return st, np.float32(out[0])

    def ivfpq_search(self, metric, centroids, pivots, offsets, codes, keys, list_offsets,
                     list_positions, queries, k, nprobe, radius=0.0, bitmap=None, threads=0):
        centroids = _c(centroids, np.float32)
        pivots = _c(pivots, np.float32)
        offsets = _c(offsets, np.int32)
        codes = _c(codes, np.uint8)
        keys = _c(keys, np.uint64)
        lo = _c(list_offsets, np.int64)
        lp = _c(list_positions, np.int64)
        queries = _c(queries, np.float32)
        nq, d = queries.shape
        ok, os_, oc, ost = self._outs(nq, k)
        bm = None if bitmap is None else _c(bitmap, np.uint32)
        st = self.lib.xo_ivfpq_search(metric, _ptr(centroids, _f32p), centroids.shape[0], d,
                                      _ptr(pivots, _f32p), _ptr(offsets, _i32p), offsets.size - 1,
                                      _ptr(codes, _u8p), _ptr(keys, _u64p), _ptr(lo, _i64p),
                                      _ptr(lp, _i64p), _ptr(queries, _f32p), nq, k, nprobe,
                                      radius, _ptr(bm, _u32p), threads or os.cpu_count(),
                                      _ptr(ok, _u64p), _ptr(os_, _f32p), _ptr(oc, _i32p),
                                      _ptr(ost, _i32p))
        return st, ok.reshape(nq, k), os_.reshape(nq, k), oc, ost

    def fht_rotate(self, signs, v):
        signs = _c(signs, np.uint8)
        v = _c(v, np.float32)
        out = np.zeros_like(v)
        st = self.lib.xo_fht_rotate(v.size, _ptr(signs, _u8p), _ptr(v, _f32p), _ptr(out, _f32p))
        return st, out

    def fht_unrotate(self, signs, v):
        signs = _c(signs, np.uint8)
        v = _c(v, np.float32)
        out = np.zeros_like(v)
        st = self.lib.xo_fht_unrotate(v.size, _ptr(signs, _u8p), _ptr(v, _f32p),
                                      _ptr(out, _f32p))
        return st, out

    def rabitq_padded_dimension(self, d):
        return int(self.lib.xo_rabitq_padded_dimension(d))

    def rabitq_rotate(self, d, signs, v):
        signs = _c(signs, np.uint8)
        v = _c(v, np.float32)
        out = np.zeros(self.rabitq_padded_dimension(d), np.float32)
        st = self.lib.xo_rabitq_rotate(d, _ptr(signs, _u8p), _ptr(v, _f32p), _ptr(out, _f32p))
        return st, out

    def rabitq_quantize(self, rotated, rotated_centroid, cluster, total_bits, extra_scale, ip):
        rotated = _c(rotated, np.float32)
        rc = _c(rotated_centroid, np.float32)
        padded = rotated.size
        binary = np.zeros(padded // 8, np.uint8)
        extra = np.zeros(max(1, (padded * (total_bits - 1) + 7) // 8), np.uint8)
        f = RaBitQFactors()
        st = self.lib.xo_rabitq_quantize(_ptr(rotated, _f32p), _ptr(rc, _f32p), padded, cluster,
                                         total_bits, extra_scale, int(ip), _ptr(binary, _u8p),
                                         _ptr(extra, _u8p), ctypes.byref(f))
        return st, binary, extra[: (padded * (total_bits - 1) + 7) // 8], f

    def rabitq_encode1_batch(self, metric, centroids, signs, rows):
        centroids = _c(centroids, np.float32)
        signs = _c(signs, np.uint8)
        rows = _c(rows, np.float32)
        n, d = rows.shape
        padded = self.rabitq_padded_dimension(d)
        codes = np.zeros((n, padded // 8), np.uint8)
        factors = np.zeros(n, RABITQ_FACTORS_DTYPE)
        for i in range(n):
            f = RaBitQFactors()
            st = self.lib.xo_rabitq_encode1(metric, d, _ptr(centroids, _f32p), centroids.shape[0],
                                            _ptr(signs, _u8p), _ptr(rows[i], _f32p),
                                            _ptr(codes[i], _u8p), ctypes.byref(f))
            if st != OK:
                raise ValueError(f"encode row {i}: status {st}")
            factors[i] = (f.cluster, 0, f.coarse_add, f.coarse_rescale, f.coarse_error,
                          f.full_add, f.full_rescale)
        return codes, factors

    def rabitq_extra_bytes(self, d, total_bits):
        padded = self.rabitq_padded_dimension(d)
        return (padded * (total_bits - 1) + 7) // 8

    def rabitq_encode_batch(self, metric, centroids, signs, rows, total_bits, extra_scale):
        """RaBitQModel.Encode of every row with TotalBits / ExtraScale: (sign
        bits [n][padded/8], extra codes [n][extra bytes], factors)."""
        centroids = _c(centroids, np.float32)
        signs = _c(signs, np.uint8)
        rows = _c(rows, np.float32)
        n, d = rows.shape
        padded = self.rabitq_padded_dimension(d)
        xb = max(1, self.rabitq_extra_bytes(d, total_bits))
        codes = np.zeros((n, padded // 8), np.uint8)
        extra = np.zeros((n, xb), np.uint8)
        factors = np.zeros(n, RABITQ_FACTORS_DTYPE)
        for i in range(n):
            f = RaBitQFactors()
            st = self.lib.xo_rabitq_encode(metric, d, _ptr(centroids, _f32p), centroids.shape[0],
                                           _ptr(signs, _u8p), total_bits, extra_scale,
                                           _ptr(rows[i], _f32p), _ptr(codes[i], _u8p),
                                           _ptr(extra[i], _u8p), ctypes.byref(f))
            if st != OK:
                raise ValueError(f"encode row {i}: status {st}")
            factors[i] = (f.cluster, 0, f.coarse_add, f.coarse_rescale, f.coarse_error,
                          f.full_add, f.full_rescale)
        return codes, extra[:, :self.rabitq_extra_bytes(d, total_bits)].copy(), factors

    def pq_encode_rows(self, metric, pivots, offsets, rows, threads=0):
        """PQModel.EncodeBatch (pq.go:303-330) of every row, threaded."""
        pivots = _c(pivots, np.float32)
        offsets = _c(offsets, np.int32)
        rows = _c(rows, np.float32)
        n, d = rows.shape
        chunks = offsets.size - 1
        codes = np.zeros((n, chunks), np.uint8)
        st = self.lib.xo_pq_encode_rows(metric, _ptr(pivots, _f32p), _ptr(offsets, _i32p), chunks,
                                        d, _ptr(rows, _f32p), n, threads or os.cpu_count(),
                                        _ptr(codes, _u8p))
        if st != OK:
            raise ValueError(f"encode rows: status {st}")
        return codes

    def rabitq_encode_rows(self, metric, centroids, signs, rows, total_bits=1, extra_scale=0.0,
                           threads=0):
        """rabitq_encode_batch over `threads` workers."""
        centroids = _c(centroids, np.float32)
        signs = _c(signs, np.uint8)
        rows = _c(rows, np.float32)
        n, d = rows.shape
        padded = self.rabitq_padded_dimension(d)
        xbytes = self.rabitq_extra_bytes(d, total_bits)
        stride = max(1, xbytes)
        codes = np.zeros((n, padded // 8), np.uint8)
        extra = np.zeros((n, stride), np.uint8)
        factors = np.zeros(n, RABITQ_FACTORS_DTYPE)
        st = self.lib.xo_rabitq_encode_rows(metric, d, _ptr(centroids, _f32p), centroids.shape[0],
                                            _ptr(signs, _u8p), total_bits, extra_scale,
                                            _ptr(rows, _f32p), n, threads or os.cpu_count(),
                                            _ptr(codes, _u8p), _ptr(extra, _u8p), stride,
                                            factors.ctypes.data)
        if st != OK:
            raise ValueError(f"encode rows: status {st}")
        return codes, extra[:, :xbytes].copy(), factors

    def rabitq_estimate(self, rotated, qsum, gadd, gerr, total_bits, code, extra, factors_row):
        rotated = _c(rotated, np.float32)
        gadd = _c(gadd, np.float64)
        gerr = None if gerr is None else _c(gerr, np.float64)
        code = _c(code, np.uint8)
        extra = None if extra is None else _c(extra, np.uint8)
        f = RaBitQFactors(int(factors_row["cluster"]), 0, float(factors_row["coarse_add"]),
                          float(factors_row["coarse_rescale"]), float(factors_row["coarse_error"]),
                          float(factors_row["full_add"]), float(factors_row["full_rescale"]))
        out = np.zeros(1, np.float32)
        st = self.lib.xo_rabitq_estimate(_ptr(rotated, _f32p), rotated.size, qsum,
                                         _ptr(gadd, _f64p), _ptr(gerr, _f64p), total_bits,
                                         _ptr(code, _u8p), _ptr(extra, _u8p), ctypes.byref(f),
                                         _ptr(out, _f32p))
        return st, np.float32(out[0])

    def rabitq_prepare_query(self, metric, centroids, signs, query):
        centroids = _c(centroids, np.float32)
        signs = _c(signs, np.uint8)
        query = _c(query, np.float32)
        d = query.size
        nc = centroids.shape[0]
        rot = np.zeros(self.rabitq_padded_dimension(d), np.float32)
        s = np.zeros(1, np.float64)
        gadd = np.zeros(nc, np.float64)
        gerr = np.zeros(nc, np.float64)
        st = self.lib.xo_rabitq_prepare_query(metric, d, _ptr(centroids, _f32p), nc,
                                              _ptr(signs, _u8p), _ptr(query, _f32p),
                                              _ptr(rot, _f32p), _ptr(s, _f64p),
                                              _ptr(gadd, _f64p), _ptr(gerr, _f64p))
        return st, rot, float(s[0]), gadd, gerr

    def rabitq_estimate_coarse(self, rotated, qsum, gadd, code, factors_row, gerr=None):
        rotated = _c(rotated, np.float32)
        gadd = _c(gadd, np.float64)
        gerr = None if gerr is None else _c(gerr, np.float64)
        code = _c(code, np.uint8)
        f = RaBitQFactors(int(factors_row["cluster"]), 0, float(factors_row["coarse_add"]),
                          float(factors_row["coarse_rescale"]), float(factors_row["coarse_error"]),
                          float(factors_row["full_add"]), float(factors_row["full_rescale"]))
        out = np.zeros(1, np.float32)
        st = self.lib.xo_rabitq_estimate_coarse(_ptr(rotated, _f32p), rotated.size, qsum,
                                                _ptr(gadd, _f64p), _ptr(gerr, _f64p),
                                                _ptr(code, _u8p),
                                                ctypes.byref(f), _ptr(out, _f32p))
        return st, np.float32(out[0])

    def rabitq_search(self, metric, centroids, signs, codes, factors, originals, keys, queries,
                      k, candidate_count, radius=0.0, bitmap=None, threads=0, refine=True,
                      total_bits=1, extra=None):
        """Linear RaBitQ search; candidate_count plays HNSWRaBitQSearchOptions.EF."""
        if total_bits > 1:
            return self._rabitq_search_bits(metric, centroids, signs, codes, extra, factors,
                                            originals, keys, queries, k, candidate_count,
                                            radius, bitmap, threads, refine, total_bits)
        centroids = _c(centroids, np.float32)
        signs = _c(signs, np.uint8)
        codes = _c(codes, np.uint8)
        factors = np.ascontiguousarray(factors, RABITQ_FACTORS_DTYPE)
        originals = _c(originals, np.float32)
        keys = _c(keys, np.uint64)
        queries = _c(queries, np.float32)
        n, d = originals.shape
        nq = queries.shape[0]
        ok, os_, oc, ost = self._outs(nq, k)
        bm = None if bitmap is None else _c(bitmap, np.uint32)
        st = self.lib.xo_rabitq_search(metric, d, _ptr(centroids, _f32p), centroids.shape[0],
                                       _ptr(signs, _u8p), _ptr(codes, _u8p), factors.ctypes.data,
                                       _ptr(originals, _f32p), _ptr(keys, _u64p), n,
                                       _ptr(queries, _f32p), nq, k, candidate_count,
                                       1 if refine else 0, radius,
                                       _ptr(bm, _u32p), threads or os.cpu_count(),
                                       _ptr(ok, _u64p), _ptr(os_, _f32p), _ptr(oc, _i32p),
                                       _ptr(ost, _i32p))
        return st, ok.reshape(nq, k), os_.reshape(nq, k), oc, ost


    def _rabitq_search_bits(self, metric, centroids, signs, codes, extra, factors, originals,
                            keys, queries, k, candidate_count, radius, bitmap, threads, refine,
                            total_bits):
        centroids = _c(centroids, np.float32)
        signs = _c(signs, np.uint8)
        codes = _c(codes, np.uint8)
        extra = _c(extra, np.uint8)
        factors = np.ascontiguousarray(factors, RABITQ_FACTORS_DTYPE)
        originals = _c(originals, np.float32)
        keys = _c(keys, np.uint64)
        queries = _c(queries, np.float32)
        n, d = originals.shape
        assert extra.shape == (n, self.rabitq_extra_bytes(d, total_bits))
        nq = queries.shape[0]
        ok, os_, oc, ost = self._outs(nq, k)
        bm = None if bitmap is None else _c(bitmap, np.uint32)
        st = self.lib.xo_rabitq_search_bits(metric, d, _ptr(centroids, _f32p), centroids.shape[0],
                                            _ptr(signs, _u8p), total_bits, _ptr(codes, _u8p),
                                            _ptr(extra, _u8p), factors.ctypes.data,
                                            _ptr(originals, _f32p), _ptr(keys, _u64p), n,
                                            _ptr(queries, _f32p), nq, k, candidate_count,
                                            1 if refine else 0, radius, _ptr(bm, _u32p),
                                            threads or os.cpu_count(), _ptr(ok, _u64p),
                                            _ptr(os_, _f32p), _ptr(oc, _i32p), _ptr(ost, _i32p))
        return st, ok.reshape(nq, k), os_.reshape(nq, k), oc, ost


    def hnsw_rabitq_search(self, metric, centroids, signs, codes, factors, originals, keys,
                           graph, queries, k, ef, radius=0.0, bitmap=None, refine=True,
                           total_bits=1, extra=None, threads=0):
        """HNSW-RaBitQ search (hnsw_rabitq.go:589-801) over `graph` =
        (max_level, entry, offsets [(max_level + 1) (n + 1)] int64, neighbors
        int32): node p's level-L neighbours at neighbors[offsets[L (n + 1) + p]
        .. offsets[L (n + 1) + p + 1])."""
        max_level, entry, offsets, nbrs = graph
        centroids = _c(centroids, np.float32)
        signs = _c(signs, np.uint8)
        codes = _c(codes, np.uint8)
        factors = np.ascontiguousarray(factors, RABITQ_FACTORS_DTYPE)
        originals = _c(originals, np.float32)
        keys = _c(keys, np.uint64)
        queries = _c(queries, np.float32)
        offsets = _c(offsets, np.int64)
        nbrs = _c(nbrs, np.int32)
        n, d = originals.shape
        if total_bits > 1:
            extra = _c(extra, np.uint8)
            assert extra.shape == (n, self.rabitq_extra_bytes(d, total_bits))
        nq = queries.shape[0]
        ok, os_, oc, ost = self._outs(nq, k)
        bm = None if bitmap is None else _c(bitmap, np.uint32)
        st = self.lib.xo_hnsw_rabitq_search(
            metric, d, _ptr(centroids, _f32p), centroids.shape[0], _ptr(signs, _u8p), total_bits,
            _ptr(codes, _u8p), _ptr(extra, _u8p) if total_bits > 1 else None, factors.ctypes.data,
            _ptr(originals, _f32p), _ptr(keys, _u64p), n, max_level, entry,
            _ptr(offsets, _i64p), _ptr(nbrs, _i32p), _ptr(queries, _f32p), nq, k, ef,
            1 if refine else 0, radius, _ptr(bm, _u32p), threads or os.cpu_count(),
            _ptr(ok, _u64p), _ptr(os_, _f32p), _ptr(oc, _i32p), _ptr(ost, _i32p))
        return st, ok.reshape(nq, k), os_.reshape(nq, k), oc, ost

    # DiskANN ----------------------------------------------------------------
    @staticmethod
    def diskann_traversal_metric(metric):
        """diskANNTraversalMetric (diskann.go:276-281)."""
        return L2 if metric in (COSINE, MIPSL2) else metric

    @staticmethod
    def diskann_read_batch(d, max_degree):
        """diskANNReadBatchSize (diskann.go:685-691) for the node layout of
        NewDiskANNLayout (diskann_storage.go:61-100): 128 sectors per read,
        ceil(record / 4096) sectors per node when a record exceeds a
        sector."""
        record = 4 * d + 4 + 4 * max_degree + 4
        sectors = 1 if record <= 4096 else (record + 4095) // 4096
        return max(1, 128 // sectors)

    def diskann_prepare(self, metric, rows):
        """prepareDiskANNPQVectors (diskann.go:258-274): cosine rows
        normalised as normalizeRaBitQVector (rabitq.go:514-526)."""
        rows = _c(rows, np.float32)
        if metric != COSINE:
            return rows.copy()
        out = rows.copy()
        for i in range(rows.shape[0]):
            ns = 0.0
            for x in rows[i].astype(np.float64):
                ns += x * x
            if ns != 0:
                out[i] = rows[i] * np.float32(1.0 / np.sqrt(ns))
        return out

    def diskann_encode(self, metric, pivots, offsets, rows):
        """The DiskANN build's PQ codes (diskann.go:224-243): EncodeBatch of
        the prepared rows under the traversal metric, and for MIPSL2 the code
        norms."""
        tm = self.diskann_traversal_metric(metric)
        prepared = self.diskann_prepare(metric, rows)
        offsets = _c(offsets, np.int32)
        chunks = offsets.size - 1
        codes = np.zeros((rows.shape[0], chunks), np.uint8)
        for i in range(rows.shape[0]):
            st, codes[i] = self.pq_encode(tm, pivots, offsets, prepared[i])
            assert st == OK
        norms = np.zeros(rows.shape[0], np.float32)
        if metric == MIPSL2:
            pivots = _c(pivots, np.float32)
            self.lib.xo_diskann_code_norms(_ptr(pivots, _f32p), _ptr(offsets, _i32p), chunks,
                                           rows.shape[1], _ptr(codes, _u8p), rows.shape[0],
                                           _ptr(norms, _f32p))
        return codes, norms

    def diskann_search(self, metric, pivots, offsets, codes, code_norms, vectors, keys, graph,
                       beam, queries, k, list_size, radius=0.0, bitmap=None, threads=0):
        """DiskANNIndex.SearchDiskANN (diskann.go:472-525, 559-683) with
        Linear false over `graph` = (entry, offsets [n + 1] int64, neighbors
        int32)."""
        entry, goff, nbrs = graph
        pivots = _c(pivots, np.float32)
        offsets = _c(offsets, np.int32)
        codes = _c(codes, np.uint8)
        code_norms = _c(code_norms, np.float32)
        vectors = _c(vectors, np.float32)
        keys = _c(keys, np.uint64)
        queries = _c(queries, np.float32)
        goff = _c(goff, np.int64)
        nbrs = _c(nbrs, np.int32)
        n, d = vectors.shape
        nq = queries.shape[0]
        ok, os_, oc, ost = self._outs(nq, k)
        bm = None if bitmap is None else _c(bitmap, np.uint32)
        st = self.lib.xo_diskann_search(
            metric, d, _ptr(pivots, _f32p), _ptr(offsets, _i32p), offsets.size - 1,
            _ptr(codes, _u8p), _ptr(code_norms, _f32p), _ptr(vectors, _f32p), _ptr(keys, _u64p),
            n, entry, _ptr(goff, _i64p), _ptr(nbrs, _i32p), beam, _ptr(queries, _f32p), nq, k,
            list_size, radius, _ptr(bm, _u32p), threads or os.cpu_count(), _ptr(ok, _u64p),
            _ptr(os_, _f32p), _ptr(oc, _i32p), _ptr(ost, _i32p))
        return st, ok.reshape(nq, k), os_.reshape(nq, k), oc, ost


def diskann_test_graph(vectors, degree=16, seed=0):
    """A single-level proximity graph for the DiskANN tests (any graph
    defines the search): every node linked to its `degree` - 3 nearest nodes
    (L2, ties to the lower position), two random ones and the next position
    (so every node is reachable), at most `degree` in all; the entry the node
    nearest the mean.  Returns (entry, offsets [n + 1], neighbors) in the
    layout of diskann_search."""
    rng = np.random.default_rng(seed)
    n = vectors.shape[0]
    v = vectors.astype(np.float64)
    sq = (v * v).sum(axis=1)
    near = max(0, min(degree - 3, n - 1))
    adj = []
    for start in range(0, n, 512):
        blk = v[start:start + 512]
        m = blk.shape[0]
        dist = sq[start:start + m, None] + sq[None, :] - 2.0 * blk @ v.T
        dist[np.arange(m), start + np.arange(m)] = np.inf
        if near > 0:
            part = np.argpartition(dist, near - 1, axis=1)[:, :near] if near < n else \
                np.tile(np.arange(n), (m, 1))
        for i in range(m):
            p = start + i
            if near > 0:
                cand = part[i]
                cand = cand[np.lexsort((cand, dist[i, cand]))]
                cand = [int(c) for c in cand if c != p]
            else:
                cand = []
            extra = [int(x) for x in rng.integers(0, n, 2)] if n > 1 else []
            seen, row = set(), []
            for c in cand + extra + ([(p + 1) % n] if n > 1 else []):
                if c != p and c not in seen:
                    seen.add(c)
                    row.append(c)
            adj.append(np.asarray(row[:degree], np.int32))
    offsets = np.zeros(n + 1, np.int64)
    offsets[1:] = np.cumsum([a.size for a in adj])
    nbrs = np.concatenate(adj) if n else np.zeros(0, np.int32)
    entry = int(np.argmin(((v - v.mean(axis=0)) ** 2).sum(axis=1))) if n else 0
    return entry, offsets, nbrs.astype(np.int32)


def hnsw_test_graph(vectors, degree=12, seed=0, ml=None):
    """A layered proximity graph for the graph-search tests (any graph
    defines the search): node levels drawn as HNSW draws them (floor of
    -ln(U) / ln(degree)), on each level every node linked to its `degree`
    nearest nodes of that level (L2, ties to the lower position) plus two
    random ones, and on level 0 also to the next position (so every node is
    reachable), the entry the first node of the top level.  Returns
    (max_level, entry, offsets, neighbors) in the layout of
    hnsw_rabitq_search."""
    rng = np.random.default_rng(seed)
    n = vectors.shape[0]
    ml = ml if ml is not None else 1.0 / np.log(max(degree, 2))
    levels = np.floor(-np.log(rng.random(n) + 1e-12) * ml).astype(np.int64)
    max_level = int(levels.max())
    v = vectors.astype(np.float64)
    sq = (v * v).sum(axis=1)
    offsets = np.zeros((max_level + 1, n + 1), np.int64)
    lists = []
    for level in range(max_level + 1):
        nodes = np.nonzero(levels >= level)[0]
        adj = [np.zeros(0, np.int32) for _ in range(n)]
        if nodes.size > 1:
            for start in range(0, nodes.size, 2048):
                blk = nodes[start:start + 2048]
                dist = sq[blk][:, None] + sq[nodes][None, :] - 2.0 * v[blk] @ v[nodes].T
                for i, p in enumerate(blk):
                    dist[i, start + i] = np.inf
                    take = min(degree, nodes.size - 1)
                    near = nodes[np.lexsort((nodes, dist[i]))[:take]]
                    extra = rng.choice(nodes, size=min(2, nodes.size), replace=False)
                    if level == 0:
                        extra = np.append(extra, (p + 1) % n)
                    extra = extra[(extra != p) & ~np.isin(extra, near)]
                    adj[p] = np.concatenate([near, extra]).astype(np.int32)
        counts = np.array([a.size for a in adj], np.int64)
        offsets[level, 1:] = np.cumsum(counts)
        lists.append(np.concatenate(adj) if counts.sum() else np.zeros(0, np.int32))
    base = 0
    flat = []
    for level in range(max_level + 1):
        offsets[level] += base
        base += lists[level].size
        flat.append(lists[level])
    entry = int(np.nonzero(levels == max_level)[0][0])
    return max_level, entry, offsets.reshape(-1), np.concatenate(flat).astype(np.int32)


class ReferenceFloats:
    """The reference's own float kernels (floats_avx512.c / floats_avx.c) from oracle/_ref."""

    def __init__(self, path: str = REF_PATH):
        lib = ctypes.CDLL(path)
        self.lib = lib
        for name in ("xvec_avx512_l2_squared", "xvec_avx512_inner_product",
                     "xvec_avx_l2_squared", "xvec_avx_inner_product"):
            getattr(lib, name).argtypes = [_f32p, _f32p, ctypes.c_int64, _f32p]
        for name in ("xvec_avx512_dot_norms", "xvec_avx_dot_norms"):
            getattr(lib, name).argtypes = [_f32p, _f32p, ctypes.c_int64, _f32p, _f32p, _f32p]

    @staticmethod
    def available() -> bool:
        if not os.path.exists(REF_PATH):
            return False
        try:
            with open("/proc/cpuinfo") as f:
                flags = f.read()
        except OSError:
            return False
        return "avx512f" in flags and " fma" in flags

    def _binary(self, name, a, b):
        a, b = _c(a, np.float32), _c(b, np.float32)
        out = np.zeros(1, np.float32)
        getattr(self.lib, name)(_ptr(a, _f32p), _ptr(b, _f32p), a.size, _ptr(out, _f32p))
        return np.float32(out[0])

    def l2_squared(self, a, b):
        """Go dispatch (floats_amd64.go:59-91) over the reference kernels."""
        a = np.asarray(a, np.float32)
        if a.size >= 16:
            return self._binary("xvec_avx512_l2_squared", a, b)
        if a.size >= 8:
            return self._binary("xvec_avx_l2_squared", a, b)
        return None

    def inner_product(self, a, b):
        a = np.asarray(a, np.float32)
        if a.size >= 16:
            return self._binary("xvec_avx512_inner_product", a, b)
        if a.size >= 8:
            return self._binary("xvec_avx_inner_product", a, b)
        return None

    def dot_norms(self, a, b):
        a, b = _c(a, np.float32), _c(b, np.float32)
        name = "xvec_avx512_dot_norms" if a.size >= 16 else "xvec_avx_dot_norms"
        out = np.zeros(3, np.float32)
        getattr(self.lib, name)(_ptr(a, _f32p), _ptr(b, _f32p), a.size, _ptr(out[0:1], _f32p),
                                _ptr(out[1:2], _f32p), _ptr(out[2:3], _f32p))
        return out
