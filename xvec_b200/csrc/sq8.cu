// sq8.cu — INT8 scalar-quantized Flat search (+ exact float32 refinement).
//
// Reference: ScalarQuantizedFlatIndex (internal/core/quantized_index.go:28-120,
// 182-335) with QuantizationInt8 (quantization.go:79-105, 267-321),
// QuantizedDistance (quantization.go:171-235) and, when a refine scale is
// given, the collection's refinement (collection.go:1606-1631,
// refiner.go:66-129).
//
// Per row the index keeps the float32 original, the int8 codes and the
// quantization parameters (inverse scale, offset, code sum and code sum of
// squares).  A search quantizes each query with the same rule, scans the
// int8 codes with the shared FFMA tile kernel (the int8 dot products are
// exact in float32 for d <= 1040), ranks in float32 within a bound eps of the
// reference's float64 formula, rescores the candidates exactly (integer dot,
// float64 formula in the reference's operation order with explicit
// round-to-nearest intrinsics) and selects the k (or refine-count) best.
#include <algorithm>
#include <cmath>
#include <mutex>
#include <vector>

#include "capi_internal.h"
#include "common.cuh"
#include "flat_kernels.cuh"
#include "flat_tc.cuh"
#include "index_kernels.cuh"
#include "ivf_scan.cuh"
#include "pipeline.cuh"
#include "refine.cuh"

namespace xvec {

struct SQParams {
  float inv_scale;
  float offset;
  double code_sum;
  double code_square;
};

namespace {

constexpr float kU = 5.9604645e-8f;  // 2^-24

// quantizeInteger (quantization.go:267-321) for INT8, one warp per vector.
// Returns false on ErrQuantizationOverflow.  Writes codes and params.
__device__ bool warp_quantize_int8(const float* v, int d, int8_t* codes, SQParams* p) {
  const int lane = threadIdx.x & 31;
  float mn = v[0], mx = v[0];
  for (int i = lane; i < d; i += 32) {
    mn = go_min_zero(mn, v[i]);
    mx = go_max_zero(mx, v[i]);
  }
  for (int o = 16; o > 0; o >>= 1) {
    mn = go_min_zero(mn, __shfl_xor_sync(kFullMask, mn, o));
    mx = go_max_zero(mx, __shfl_xor_sync(kFullMask, mx, o));
  }
  if (mn == mx) {
    for (int i = lane; i < d; i += 32) codes[i] = 0;
    if (lane == 0) *p = SQParams{0.f, mn, 0.0, 0.0};
    return true;
  }
  const float eps32 = 1.1920928955078125e-7f;
  const float span = __fsub_rn(mx, mn);
  const float scale = __fdiv_rn(254.f, go_maxf(span, eps32));
  const float bias = __fadd_rn(__fmul_rn(-mn, scale), -127.f);
  const float inv = __fdiv_rn(1.f, scale);
  const float off = __fdiv_rn(-bias, scale);
  if (!finite_f(inv) || !finite_f(off)) return false;
  long long sum = 0, sq = 0;
  for (int i = lane; i < d; i += 32) {
    const float t = __fadd_rn(__fmul_rn(v[i], scale), bias);
    int c = (int)round((double)t);
    c = min(127, max(-127, c));
    codes[i] = (int8_t)c;
    sum += c;
    sq += c * c;
  }
  for (int o = 16; o > 0; o >>= 1) {
    sum += __shfl_xor_sync(kFullMask, sum, o);
    sq += __shfl_xor_sync(kFullMask, sq, o);
  }
  if (lane == 0) *p = SQParams{inv, off, (double)sum, (double)sq};
  return true;
}

// quantizeInteger (quantization.go:267-321) for INT4 ([-8, 7]), one warp per
// vector of even dimension, a lane per element pair.  The codes are written
// one per byte (the reference packs two per byte; the values, code sums and
// scores are the same).
__device__ bool warp_quantize_int4(const float* v, int d, int8_t* codes, SQParams* p) {
  const int lane = threadIdx.x & 31;
  float mn = v[0], mx = v[0];
  for (int i = lane; i < d; i += 32) {
    mn = go_min_zero(mn, v[i]);
    mx = go_max_zero(mx, v[i]);
  }
  for (int o = 16; o > 0; o >>= 1) {
    mn = go_min_zero(mn, __shfl_xor_sync(kFullMask, mn, o));
    mx = go_max_zero(mx, __shfl_xor_sync(kFullMask, mx, o));
  }
  const int half = d >> 1;
  if (mn == mx) {
    for (int j = lane; j < half; j += 32) codes[2 * j] = codes[2 * j + 1] = 0;
    if (lane == 0) *p = SQParams{0.f, mn, 0.0, 0.0};
    return true;
  }
  const float eps32 = 1.1920928955078125e-7f;
  const float span = __fsub_rn(mx, mn);
  const float scale = __fdiv_rn(15.f, go_maxf(span, eps32));
  const float bias = __fadd_rn(__fmul_rn(-mn, scale), -8.f);
  const float inv = __fdiv_rn(1.f, scale);
  const float off = __fdiv_rn(-bias, scale);
  if (!finite_f(inv) || !finite_f(off)) return false;
  long long sum = 0, sq = 0;
  for (int j = lane; j < half; j += 32) {
    int c[2];
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const float t = __fadd_rn(__fmul_rn(v[2 * j + e], scale), bias);
      c[e] = min(7, max(-8, (int)round((double)t)));
      sum += c[e];
      sq += c[e] * c[e];
    }
    codes[2 * j] = (int8_t)c[0];
    codes[2 * j + 1] = (int8_t)c[1];
  }
  for (int o = 16; o > 0; o >>= 1) {
    sum += __shfl_xor_sync(kFullMask, sum, o);
    sq += __shfl_xor_sync(kFullMask, sq, o);
  }
  if (lane == 0) *p = SQParams{inv, off, (double)sum, (double)sq};
  return true;
}

// The squared norm of the decoded vector, float64 in the reference order
// (leftNorm / rightNorm of quantization.go:205-208).
__device__ __forceinline__ double sq_norm64(const SQParams& p, int d) {
  const double s = (double)p.inv_scale, o = (double)p.offset;
  return __dadd_rn(__dadd_rn(__dmul_rn(__dmul_rn(s, s), p.code_square),
                             __dmul_rn(__dmul_rn(__dmul_rn(2.0, s), o), p.code_sum)),
                   __dmul_rn(__dmul_rn((double)d, o), o));
}

// QuantizedDistance (quantization.go:196-235) from the exact integer code dot;
// left = stored row, right = query.
__device__ float sq_reference_score(int metric, double dot, const SQParams& l, const SQParams& r,
                                    int d) {
  const double ls = (double)l.inv_scale, rs = (double)r.inv_scale;
  const double lo = (double)l.offset, ro = (double)r.offset;
  const double dim = (double)d;
  const double inner =
      __dadd_rn(__dadd_rn(__dadd_rn(__dmul_rn(__dmul_rn(ls, rs), dot),
                                    __dmul_rn(__dmul_rn(lo, rs), r.code_sum)),
                          __dmul_rn(__dmul_rn(ro, ls), l.code_sum)),
                __dmul_rn(__dmul_rn(dim, lo), ro));
  const double ln = sq_norm64(l, d), rn = sq_norm64(r, d);
  double s;
  if (metric == kMetricL2) {
    s = __dsub_rn(__dadd_rn(ln, rn), __dmul_rn(2.0, inner));
    if (s < 0 && s > __dmul_rn(-1e-6, go_maxd(1.0, __dadd_rn(ln, rn)))) s = 0;
  } else if (metric == kMetricIP) {
    s = inner;
  } else if (metric == kMetricCosine) {
    if (ln == 0 && rn == 0) {
      s = 0;
    } else if (ln == 0 || rn == 0) {
      s = 1;
    } else {
      double c = __ddiv_rn(inner, __dsqrt_rn(__dmul_rn(ln, rn)));
      c = go_mind(1.0, go_maxd(-1.0, c));
      s = __dsub_rn(1.0, c);
    }
  } else {
    const double den = go_maxd(ln, rn);
    s = den == 0 ? 0.0 : __dsub_rn(2.0, __ddiv_rn(__dmul_rn(2.0, inner), den));
  }
  // finiteQuantizedScore (quantization.go:387-393)
  const float f = __double2float_rn(s);
  if (isnan(s) || isinf(s) || !finite_f(f)) return __int_as_float(0x7fc00000);
  return f;
}

// Rows: quantize, fast-rank terms and the index-wide error-bound maxima.
// d int8 codes per row for either width (INT4 codes in [-8, 7], one per
// byte, so both widths share the tcgen05 kind::i8 scan).
template <int BITS>
__global__ void sq8_encode_rows_kernel(const float* __restrict__ rows, int64_t n, int d,
                                       uint8_t* __restrict__ codes, SQParams* __restrict__ params,
                                       float4* __restrict__ fast, unsigned* __restrict__ bounds,
                                       int* __restrict__ err) {
  const int64_t w = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (w >= n) return;
  SQParams p;
  __shared__ SQParams sp[8];
  const int wl = threadIdx.x >> 5;
  int8_t* row_codes = reinterpret_cast<int8_t*>(codes) + w * d;
  const bool ok = BITS == 8 ? warp_quantize_int8(rows + w * d, d, row_codes, &sp[wl])
                            : warp_quantize_int4(rows + w * d, d, row_codes, &sp[wl]);
  if (!ok) {
    if (lane == 0) atomicExch(err, XVEC_GPU_OVERFLOW);
    return;
  }
  __syncwarp();
  p = sp[wl];
  if (lane == 0) {
    params[w] = p;
    const float ln = __double2float_rn(sq_norm64(p, d));
    fast[w] = make_float4(p.inv_scale, p.offset, (float)p.code_sum, ln);
    const float U = fabsf(p.inv_scale) * sqrtf((float)p.code_square);
    const float V = fabsf(p.inv_scale * (float)p.code_sum);
    const float W = fabsf(p.offset);
    atomicMax(&bounds[0], float_to_ordered(U));
    atomicMax(&bounds[1], float_to_ordered(V));
    atomicMax(&bounds[2], float_to_ordered(W));
    atomicMax(&bounds[3], float_to_ordered(ln));
  }
}

// Queries: validation (metric.Compute(q, q), quantized_index.go:264-272),
// quantization, the float codes for the scan, the fast-rank constants and
// eps (bound on |fast rank - reference rank|, see sq8.cu header).  qcodes
// hold d int8 codes per query for either width (INT4 codes unpacked); an odd
// dimension fails every INT4 query (ErrOddInt4Dimension, quantization.go:91-93).
template <int BITS>
__global__ void sq8_prep_queries_kernel(const float* __restrict__ q, int nq, int d, int metric,
                                        const unsigned* __restrict__ bounds,
                                        int8_t* __restrict__ qcodes, SQParams* __restrict__ qparams,
                                        float* __restrict__ qf, float4* __restrict__ qinfo,
                                        float* __restrict__ q_eps, int* __restrict__ q_status) {
  const int w = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (w >= nq) return;
  const float* v = q + (int64_t)w * d;
  bool finite = true;
  for (int i = lane; i < d; i += 32) finite &= finite_f(v[i]);
  finite = __all_sync(kFullMask, finite);
  float s0, s1, s2;
  warp_reference_sums<1>(v, v, d, &s0, &s1, &s2);
  int st = 0;
  if (!finite || (metric != kMetricL2 && !finite_f(s0))) st = XVEC_GPU_NON_FINITE;
  __shared__ SQParams sp[8];
  const int wl = threadIdx.x >> 5;
  if (st == 0 && BITS == 4 && (d & 1)) st = XVEC_GPU_INVALID_ARGUMENT;
  if (st == 0 &&
      !(BITS == 8 ? warp_quantize_int8(v, d, qcodes + (int64_t)w * d, &sp[wl])
                  : warp_quantize_int4(v, d, qcodes + (int64_t)w * d, &sp[wl])))
    st = XVEC_GPU_OVERFLOW;
  __syncwarp();
  if (st != 0) {
    if (lane == 0) q_status[w] = st;
    for (int i = lane; i < d; i += 32) qf[(int64_t)w * d + i] = 0.f;
    return;
  }
  for (int i = lane; i < d; i += 32) qf[(int64_t)w * d + i] = (float)qcodes[(int64_t)w * d + i];
  if (lane == 0) {
    const SQParams p = sp[wl];
    qparams[w] = p;
    const double rs = p.inv_scale, ro = p.offset;
    const float A = p.inv_scale, B = p.offset;
    const float C = __double2float_rn(rs * p.code_sum + (double)d * ro);
    const double rn64 = sq_norm64(p, d);
    const float rn = __double2float_rn(rn64);
    qinfo[w] = make_float4(A, B, C, rn);
    const float maxU = ordered_to_float(bounds[0]), maxV = ordered_to_float(bounds[1]);
    const float maxW = ordered_to_float(bounds[2]), maxLn = ordered_to_float(bounds[3]);
    const float a = fabsf(A) * sqrtf((float)p.code_square);
    const float b = fabsf(A * (float)p.code_sum);
    const float c = fabsf(B);
    const float e = (float)d * fabsf(B);
    float ei = 8.f * kU * (a * maxU + c * maxV + (b + e) * maxW) + kU * sqrtf(maxLn * rn);
    float eps;
    if (metric == kMetricL2)
      eps = 2.f * ei + 5.f * kU * (maxLn + rn);
    else
      eps = ei;
    q_eps[w] = 1.25f * eps + 1e-30f;
    q_status[w] = 0;
  }
}

struct SQ8Ranker {
  int metric;
  const float4* row_fast;
  const float4* q_info;
  using RowInfo = float4;
  using QueryInfo = float4;
  __device__ QueryInfo query(int qi) const { return q_info[qi]; }
  __device__ RowInfo row(int64_t r) const { return row_fast[r]; }
  // inner ~ ls * (rs*dot + ro*sum_l) + lo * (rs*sum_r + d*ro)
  __device__ float rank(float dot, const RowInfo& r, const QueryInfo& q) const {
    const float t = fmaf(q.x, dot, q.y * r.z);
    const float inner = fmaf(r.x, t, r.y * q.z);
    if (metric == kMetricIP) return -inner;
    return (r.w + q.w) - 2.f * inner;  // L2
  }
};

struct SQ8Scorer {
  int metric;
  const uint8_t* codes;
  const SQParams* params;
  const int8_t* qcodes;
  const SQParams* qparams;
  const float* q_eps;
  int d;
  __device__ float score(int qi, int64_t row) const {
    const int lane = threadIdx.x & 31;
    const int8_t* b = qcodes + (int64_t)qi * d;
    int dot = 0;
    const int8_t* a = reinterpret_cast<const int8_t*>(codes) + row * d;
    if ((d & 3) == 0) {
      // Rows of d % 4 == 0 codes are 4-byte aligned: four codes per load and
      // dp4a (the integer dot is exact in any order).
      const int* a4 = reinterpret_cast<const int*>(a);
      const int* b4 = reinterpret_cast<const int*>(b);
#pragma unroll 4
      for (int i = lane; i < (d >> 2); i += 32) dot = __dp4a(a4[i], b4[i], dot);
    } else {
      for (int i = lane; i < d; i += 32) dot += (int)a[i] * (int)b[i];
    }
    for (int o = 16; o > 0; o >>= 1) dot += __shfl_xor_sync(kFullMask, dot, o);
    return sq_reference_score(metric, (double)dot, params[row], qparams[qi], d);
  }
  __device__ float eps(int qi) const { return q_eps[qi]; }
  __device__ bool half_warp() const { return false; }
  __device__ int error_flag(float) const { return 4; }
  __device__ float output(float r) const { return score_from_rank(metric, r); }
  __device__ bool keep(float out, float radius) const { return within_radius(metric, out, radius); }
};

__global__ void sq8_status_kernel(const int* q_status, const int* q_flags, int nq,
                                  int* out_counts) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= nq) return;
  int st = q_status[i];
  if (st == 0 && (q_flags[i] & 4)) st = XVEC_GPU_NON_FINITE;
  if (st != 0) out_counts[i] = -st;
}

__global__ void sq8_clear_flags(const int* ids, int n, int* q_flags) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) q_flags[ids[i]] &= ~3;
}

inline unsigned blocks_of(int64_t n, int t = 256) { return (unsigned)((n + t - 1) / t); }

int sq8_kp(int k) {
  int want = k + std::max(8, k / 4);
  int kp = 32;
  while (kp < want) kp <<= 1;
  return kp;
}

// The IVF list scan over INT8 codes (ivf_scan.cuh): the exact integer dot of
// the row's codes with the query's codes (staged in shared memory, dp4a on
// 4-byte groups), ranked with SQ8Ranker; the reference score as SQ8Scorer.
struct Sq8IvfPolicy {
  int metric;
  const int8_t* codes;
  const SQParams* params;
  const float4* row_fast;
  const int4* list_codes;    // list-major interleaved codes (d % 16 == 0), or null
  const float4* list_fast;   // rank terms in list order (with list_codes)
  const int8_t* qcodes;
  const SQParams* qparams;
  const float4* q_info;
  int d;
  __host__ __device__ int smem_bytes(int dim) const { return (dim + 15) / 16 * 16; }
  __device__ void stage(int q, unsigned char* smem) const {
    int8_t* sq = reinterpret_cast<int8_t*>(smem);
    for (int i = threadIdx.x; i < d; i += blockDim.x) sq[i] = qcodes[(int64_t)q * d + i];
  }
  __device__ float fast_rank(int q, int64_t idx, uint32_t pos, const unsigned char* smem) const {
    const int8_t* a = codes + (int64_t)pos * d;
    int dot = 0;
    if (list_codes) {
      // Chunk c of list entry idx: coalesced across the warp's 32 entries.
      const int C = d / 16;
      const int4* src = list_codes + (idx >> 5) * C * 32 + (idx & 31);
      const int4* b16 = reinterpret_cast<const int4*>(smem);
      for (int c = 0; c < C; ++c) {
        const int4 x = __ldg(src + c * 32), y = b16[c];
        dot = __dp4a(x.x, y.x, dot);
        dot = __dp4a(x.y, y.y, dot);
        dot = __dp4a(x.z, y.z, dot);
        dot = __dp4a(x.w, y.w, dot);
      }
      const SQ8Ranker rk{metric, row_fast, q_info};
      return rk.rank((float)dot, __ldg(list_fast + idx), q_info[q]);
    }
    if ((d & 15) == 0) {
      // 16-byte loads: the lane's code row in d/16 requests.
      const int4* a16 = reinterpret_cast<const int4*>(a);
      const int4* b16 = reinterpret_cast<const int4*>(smem);
      for (int i = 0; i < d / 16; ++i) {
        const int4 x = __ldg(a16 + i), y = b16[i];
        dot = __dp4a(x.x, y.x, dot);
        dot = __dp4a(x.y, y.y, dot);
        dot = __dp4a(x.z, y.z, dot);
        dot = __dp4a(x.w, y.w, dot);
      }
    } else if ((d & 3) == 0) {
      const int* a4 = reinterpret_cast<const int*>(a);
      const int* b4 = reinterpret_cast<const int*>(smem);
      for (int i = 0; i < d / 4; ++i) dot = __dp4a(__ldg(a4 + i), b4[i], dot);
    } else {
      const int8_t* b = reinterpret_cast<const int8_t*>(smem);
      for (int i = 0; i < d; ++i) dot += (int)__ldg(a + i) * (int)b[i];
    }
    const SQ8Ranker rk{metric, row_fast, q_info};
    return rk.rank((float)dot, row_fast[pos], q_info[q]);
  }
  __device__ float exact_score(int q, uint32_t pos, const unsigned char* smem) const {
    const int lane = threadIdx.x & 31;
    const int8_t* a = codes + (int64_t)pos * d;
    const int8_t* b = reinterpret_cast<const int8_t*>(smem);
    int dot = 0;
    for (int i = lane; i < d; i += 32) dot += (int)a[i] * (int)b[i];
    for (int o = 16; o > 0; o >>= 1) dot += __shfl_xor_sync(kFullMask, dot, o);
    return sq_reference_score(metric, (double)dot, params[pos], qparams[q], d);
  }
};

}  // namespace

// ---------------------------------------------------------------------------
// Insertion hooks.
// ---------------------------------------------------------------------------
// Code bytes per row: d for both widths (INT4 codes are kept one per byte).
inline size_t sq_row_bytes(const xvec_gpu_index* idx) { return (size_t)idx->desc.dimension; }

xvec_gpu_status sq8_reserve(xvec_gpu_index* idx, int64_t cap, cudaStream_t s) {
  const size_t rb = sq_row_bytes(idx);
  const int64_t n = idx->n;
  xvec_gpu_status st;
  if ((st = idx->sq_codes.reserve((size_t)cap * rb, (size_t)n * rb, s)) ||
      (st = idx->sq_params.reserve((size_t)cap * sizeof(SQParams), (size_t)n * sizeof(SQParams), s)) ||
      (st = idx->sq_fast.reserve((size_t)cap * 16, (size_t)n * 16, s)))
    return st;
  if (!idx->sq_bounds.ptr) {
    if ((st = idx->sq_bounds.reserve(16, 0, s))) return st;
    XVEC_CUDA(cudaMemsetAsync(idx->sq_bounds.ptr, 0, 16, s));
  }
  return XVEC_GPU_OK;
}

xvec_gpu_status sq8_commit(xvec_gpu_index* idx, int64_t old_n, int64_t m, cudaStream_t s) {
  const int d = idx->desc.dimension;
  // metric.Compute(vector, vector) must be finite (quantized_index.go:233-235).
  if (idx->desc.metric != XVEC_METRIC_L2) {
    std::vector<float> n2(m);
    XVEC_CUDA(cudaMemcpyAsync(n2.data(), idx->row_n2.as<float>() + old_n, (size_t)m * 4,
                              cudaMemcpyDeviceToHost, s));
    XVEC_CUDA(cudaStreamSynchronize(s));
    for (int64_t i = 0; i < m; ++i)
      if (!std::isfinite(n2[i]))
        return set_error("core: validate scalar-quantized vector %lld: non-finite",
                         (long long)(old_n + i)),
               XVEC_GPU_NON_FINITE;
  }
  const bool int4 =
      idx->desc.kind == XVEC_INDEX_SQ4_FLAT || idx->desc.kind == XVEC_INDEX_IVF_SQ4;
  if (int4 && (d & 1))
    return set_error("core: quantize vector %lld: core: INT4 quantization requires an even "
                     "dimension: got %d",
                     (long long)old_n, d),
           XVEC_GPU_INVALID_ARGUMENT;
  Scratch err, bounds;
  xvec_gpu_status st;
  if ((st = err.alloc(4, s)) || (st = bounds.alloc(16, s))) return st;
  XVEC_CUDA(cudaMemsetAsync(err.ptr, 0, 4, s));
  XVEC_CUDA(cudaMemcpyAsync(bounds.ptr, idx->sq_bounds.ptr, 16, cudaMemcpyDeviceToDevice, s));
  uint8_t* codes = idx->sq_codes.as<uint8_t>() + old_n * sq_row_bytes(idx);
  if (int4)
    sq8_encode_rows_kernel<4><<<blocks_of(m * 32), 256, 0, s>>>(
        idx->rows.as<float>() + old_n * d, m, d, codes, idx->sq_params.as<SQParams>() + old_n,
        idx->sq_fast.as<float4>() + old_n, bounds.as<unsigned>(), err.as<int>());
  else
    sq8_encode_rows_kernel<8><<<blocks_of(m * 32), 256, 0, s>>>(
        idx->rows.as<float>() + old_n * d, m, d, codes, idx->sq_params.as<SQParams>() + old_n,
        idx->sq_fast.as<float4>() + old_n, bounds.as<unsigned>(), err.as<int>());
  XVEC_LAUNCHED();
  XVEC_CUDA(cudaGetLastError());
  int h_err = 0;
  XVEC_CUDA(cudaMemcpyAsync(&h_err, err.ptr, 4, cudaMemcpyDeviceToHost, s));
  XVEC_CUDA(cudaStreamSynchronize(s));
  if (h_err) return set_error("core: value overflows quantized representation"), XVEC_GPU_OVERFLOW;
  XVEC_CUDA(cudaMemcpyAsync(idx->sq_bounds.ptr, bounds.ptr, 16, cudaMemcpyDeviceToDevice, s));
  return XVEC_GPU_OK;
}

// ---------------------------------------------------------------------------
// Search.
// ---------------------------------------------------------------------------
int sq8_candidate_count(const xvec_gpu_search_opts& o) {
  if (!(o.refine_scale > 0) || std::isinf(o.refine_scale)) return 0;
  return std::max(1, (int)std::floor((double)o.top_k * (double)o.refine_scale));
}

xvec_gpu_status sq8_search_impl(xvec_gpu_index* idx, const float* d_q, int nq,
                                const xvec_gpu_search_opts& o, const uint32_t* d_bitmap,
                                uint64_t* d_keys, float* d_scores, int* d_counts, cudaStream_t s,
                                std::vector<int>* statuses, bool candidates_only) {
  EventTimer timer(s);
  timer.mark(0);
  const int d = idx->desc.dimension, metric = idx->desc.metric;
  const int64_t n = idx->n;
  const bool refine = o.refine_scale > 0;
  if (candidates_only && !refine)
    return set_error("candidates of a search without refinement"), XVEC_GPU_INVALID_ARGUMENT;
  int stage_k = o.top_k;
  if (refine) {
    if (!(o.refine_scale > 0) || std::isinf(o.refine_scale))
      return set_error("core: refiner scale factor must be finite and positive"),
             XVEC_GPU_INVALID_ARGUMENT;
    const double product = (double)o.top_k * (double)o.refine_scale;
    if (product >= 1024.0 + 1.0)
      return set_error("refinement candidate count %.0f exceeds 1024", std::floor(product)),
             XVEC_GPU_INVALID_ARGUMENT;
    stage_k = std::max(1, (int)std::floor(product));  // RefinementCandidateCount (refiner.go:112-129)
  }
  const float stage_radius = refine ? 0.f : o.radius;  // collection.go:1623
  const int kp = sq8_kp(stage_k);
  xvec_gpu_status st;
  Scratch qcodes, qparams, qf, qinfo, qeps, qstatus, qflags;
  if ((st = qcodes.alloc((size_t)nq * d, s)) ||
      (st = qparams.alloc((size_t)nq * sizeof(SQParams), s)) ||
      (st = qf.alloc((size_t)nq * d * 4, s)) || (st = qinfo.alloc((size_t)nq * 16, s)) ||
      (st = qeps.alloc((size_t)nq * 4, s)) || (st = qstatus.alloc((size_t)nq * 4, s)) ||
      (st = qflags.alloc((size_t)nq * 4, s)))
    return st;
  XVEC_CUDA(cudaMemsetAsync(qflags.ptr, 0, (size_t)nq * 4, s));
  XVEC_CUDA(cudaMemsetAsync(qstatus.ptr, 0, (size_t)nq * 4, s));
  const bool int4 = idx->desc.kind == XVEC_INDEX_SQ4_FLAT;
  if (int4)
    sq8_prep_queries_kernel<4><<<blocks_of((int64_t)nq * 32), 256, 0, s>>>(
        d_q, nq, d, metric, idx->sq_bounds.as<unsigned>(), qcodes.as<int8_t>(),
        qparams.as<SQParams>(), qf.as<float>(), qinfo.as<float4>(), qeps.as<float>(),
        qstatus.as<int>());
  else
    sq8_prep_queries_kernel<8><<<blocks_of((int64_t)nq * 32), 256, 0, s>>>(
        d_q, nq, d, metric, idx->sq_bounds.as<unsigned>(), qcodes.as<int8_t>(),
        qparams.as<SQParams>(), qf.as<float>(), qinfo.as<float4>(), qeps.as<float>(),
        qstatus.as<int>());
  XVEC_LAUNCHED();
  XVEC_CUDA(cudaGetLastError());
  // Stage outputs: the final outputs, or scratch when a refine stage follows.
  Scratch skeys, sscores, scounts, spos;
  uint64_t* o_keys = d_keys;
  float* o_scores = d_scores;
  int* o_counts = d_counts;
  if ((st = spos.alloc((size_t)nq * stage_k * 4, s))) return st;
  if (refine && !candidates_only) {
    if ((st = skeys.alloc((size_t)nq * stage_k * 8, s)) ||
        (st = sscores.alloc((size_t)nq * stage_k * 4, s)) ||
        (st = scounts.alloc((size_t)nq * 4, s)))
      return st;
    o_keys = skeys.as<uint64_t>();
    o_scores = sscores.as<float>();
    o_counts = scounts.as<int>();
  }
  XVEC_CUDA(cudaMemsetAsync(o_counts, 0, (size_t)nq * 4, s));
  SQ8Scorer sc{metric, idx->sq_codes.as<uint8_t>(), idx->sq_params.as<SQParams>(),
               qcodes.as<int8_t>(), qparams.as<SQParams>(), qeps.as<float>(), d};
  const bool ranked = n > 0 && (metric == XVEC_METRIC_IP || metric == XVEC_METRIC_L2);
  // INT8 tensor cores (tcgen05 kind::i8) when the layout allows, else FFMA.
  const bool use_tc = ranked && kp + 128 <= flat_tc_cap() && n < (1ll << 31) - 256 &&
                      sq8_tc_supported(d, idx->sq_codes.ptr, qcodes.ptr);
  const bool fast = use_tc || (ranked && simt_cap_for(kp) <= 512);
  if (use_tc) {
    Scratch pkeys, pcounts, psat, kstatus, gthr_keep;
    int lists = 0;
    if ((st = kstatus.alloc(4, s))) return st;
    XVEC_CUDA(cudaMemsetAsync(kstatus.ptr, 0, 4, s));
    timer.mark(1);
    st = tc_seeded_scan(
        idx->device, nq, n, kp, s,
        [&](int64_t b, int64_t e, int p, int list0, int nlists, unsigned long long* gthr,
            uint64_t* cand, int* counts, uint64_t* sat) {
          return launch_sq8_scan_tc(metric, qcodes.as<int8_t>(), nq,
                                    idx->sq_codes.as<int8_t>() + b * d, e - b, d,
                                    idx->sq_fast.as<float4>() + b,
                                    idx->keyrank.as<uint32_t>() + b, qinfo.as<float4>(), gthr,
                                    d_bitmap ? d_bitmap + b / 32 : nullptr, p, kp, list0, nlists,
                                    cand, counts, sat, qflags.as<int>(), kstatus.as<int>(), s);
        },
        pkeys, pcounts, psat, &lists, &gthr_keep);
    if (st) return st;
    timer.mark(2);
    XVEC_LAUNCHED();
    count_tensor_scan();
    XVEC_CUDA(launch_merge_rescore(sc, idx->pos_of_kr.as<uint32_t>(), idx->keys.as<uint64_t>(),
                                   nullptr, nq, stage_k, stage_radius, 0, pkeys.as<uint64_t>(),
                                   pcounts.as<int>(), psat.as<uint64_t>(), lists, flat_tc_cap(),
                                   o_keys, o_scores, o_counts, spos.as<uint32_t>(),
                                   qflags.as<int>(), s,
                                   gthr_keep.as<unsigned long long>()));
    XVEC_LAUNCHED();
    int h_kstatus = 0;
    XVEC_CUDA(cudaMemcpyAsync(&h_kstatus, kstatus.ptr, 4, cudaMemcpyDeviceToHost, s));
    XVEC_CUDA(cudaStreamSynchronize(s));
    if (h_kstatus != 0)
      return set_error("tensor-core scan: a bounded device wait expired (code %d)", h_kstatus),
             XVEC_GPU_TIMEOUT;
  } else if (fast) {
    const int qtiles = (nq + 31) / 32;
    int parts = (int)std::max<int64_t>(
        1, std::min<int64_t>((592 + qtiles - 1) / qtiles, (n + 1023) / 1024));
    parts = std::min(parts, std::max(1, flat_merge_capacity() / kp));
    Scratch pkeys, pcounts, psat;
    if ((st = pkeys.alloc((size_t)nq * parts * kp * 8, s)) ||
        (st = pcounts.alloc((size_t)nq * parts * 4, s)) ||
        (st = psat.alloc((size_t)nq * parts * 8, s)))
      return st;
    const SQ8Ranker rk{metric, idx->sq_fast.as<float4>(), qinfo.as<float4>()};
    timer.mark(1);
    XVEC_CUDA(launch_scan_simt(idx->sq_codes.as<int8_t>(), n, d, idx->keyrank.as<uint32_t>(),
                               qf.as<float>(), nq, d_bitmap, rk, parts, kp, pkeys.as<uint64_t>(),
                               pcounts.as<int>(), psat.as<uint64_t>(), qflags.as<int>(), s));
    timer.mark(2);
    XVEC_CUDA(launch_merge_rescore(sc, idx->pos_of_kr.as<uint32_t>(), idx->keys.as<uint64_t>(),
                                   nullptr, nq, stage_k, stage_radius, 0, pkeys.as<uint64_t>(),
                                   pcounts.as<int>(), psat.as<uint64_t>(), parts, kp, o_keys,
                                   o_scores, o_counts, spos.as<uint32_t>(), qflags.as<int>(), s));
    count_launches(2);
  }
  std::vector<int> h_status(nq), h_flags(nq);
  XVEC_CUDA(cudaMemcpyAsync(h_status.data(), qstatus.ptr, (size_t)nq * 4, cudaMemcpyDeviceToHost,
                            s));
  XVEC_CUDA(cudaMemcpyAsync(h_flags.data(), qflags.ptr, (size_t)nq * 4, cudaMemcpyDeviceToHost, s));
  XVEC_CUDA(cudaStreamSynchronize(s));
  std::vector<int> exact_list;
  if (n > 0)
    for (int q = 0; q < nq; ++q)
      if (h_status[q] == 0 && (!fast || (h_flags[q] & 3))) exact_list.push_back(q);
  if (!exact_list.empty()) {
    const int nl = (int)exact_list.size();
    int parts = (int)std::max<int64_t>(1, std::min<int64_t>((592 + nl - 1) / nl, (n + 1023) / 1024));
    parts = std::min(parts, std::max(1, flat_merge_capacity() / kp));
    Scratch ids, pkeys, pcounts, psat;
    if ((st = ids.alloc((size_t)nl * 4, s)) || (st = pkeys.alloc((size_t)nl * parts * kp * 8, s)) ||
        (st = pcounts.alloc((size_t)nl * parts * 4, s)) ||
        (st = psat.alloc((size_t)nl * parts * 8, s)))
      return st;
    XVEC_CUDA(cudaMemcpyAsync(ids.ptr, exact_list.data(), (size_t)nl * 4, cudaMemcpyHostToDevice, s));
    sq8_clear_flags<<<blocks_of(nl), 256, 0, s>>>(ids.as<int>(), nl, qflags.as<int>());
    XVEC_CUDA(launch_scan_exact(sc, n, idx->keyrank.as<uint32_t>(), ids.as<int>(), nl, d_bitmap,
                                parts, kp, pkeys.as<uint64_t>(), pcounts.as<int>(),
                                psat.as<uint64_t>(), qflags.as<int>(), s));
    XVEC_CUDA(launch_merge_rescore(sc, idx->pos_of_kr.as<uint32_t>(), idx->keys.as<uint64_t>(),
                                   ids.as<int>(), nl, stage_k, stage_radius, 1,
                                   pkeys.as<uint64_t>(), pcounts.as<int>(), psat.as<uint64_t>(),
                                   parts, kp, o_keys, o_scores, o_counts, spos.as<uint32_t>(),
                                   qflags.as<int>(), s));
    count_launches(3);
    XVEC_CUDA(cudaMemcpyAsync(h_flags.data(), qflags.ptr, (size_t)nq * 4, cudaMemcpyDeviceToHost, s));
    XVEC_CUDA(cudaStreamSynchronize(s));
    for (int q : exact_list)
      if (h_flags[q] & 2) return set_error("exact scan could not complete query %d", q), XVEC_GPU_CUDA_ERROR;
  }
  if (candidates_only) {
    // The approximate stage's candidates are the output.
  } else if (refine && n > 0) {
    // The approximate stage's failures are final; the refine stage sees
    // counts >= 0 only for healthy queries.
    sq8_status_kernel<<<blocks_of(nq), 256, 0, s>>>(qstatus.as<int>(), qflags.as<int>(), nq,
                                                    o_counts);
    XVEC_CUDA(cudaMemsetAsync(d_counts, 0, (size_t)nq * 4, s));
    XVEC_CUDA(launch_refine(idx->rows.as<float>(), d, metric, d_q, nq, spos.as<uint32_t>(),
                            o_counts, stage_k, idx->keyrank.as<uint32_t>(),
                            idx->pos_of_kr.as<uint32_t>(), idx->keys.as<uint64_t>(), o.top_k,
                            o.radius, d_keys, d_scores, d_counts, qflags.as<int>(), s));
    count_launches(2);
  } else if (refine) {
    XVEC_CUDA(cudaMemsetAsync(d_counts, 0, (size_t)nq * 4, s));
  }
  sq8_status_kernel<<<blocks_of(nq), 256, 0, s>>>(qstatus.as<int>(), qflags.as<int>(), nq,
                                                  d_counts);
  XVEC_LAUNCHED();
  if (candidates_only && metric == XVEC_METRIC_IP) {
    scores_to_ranks_kernel<<<blocks_of((int64_t)nq * stage_k), 256, 0, s>>>(
        d_scores, d_counts, nq, stage_k, metric);
    XVEC_LAUNCHED();
  }
  XVEC_CUDA(cudaGetLastError());
  XVEC_CUDA(cudaMemcpyAsync(h_flags.data(), qflags.ptr, (size_t)nq * 4, cudaMemcpyDeviceToHost, s));
  timer.mark(3);
  XVEC_CUDA(cudaStreamSynchronize(s));
  count_search(nq, (int64_t)exact_list.size(), timer.ms(1, 2), timer.ms(0, 3));
  if (statuses) {
    statuses->resize(nq);
    for (int q = 0; q < nq; ++q) {
      int sq = h_status[q];
      if (sq == 0 && (h_flags[q] & 4)) sq = XVEC_GPU_NON_FINITE;
      (*statuses)[q] = sq;
    }
  }
  return XVEC_GPU_OK;
}

// ---------------------------------------------------------------------------
// IVF over INT8 codes: ScalarQuantizedIVFIndex.search (ivf_quantized.go:
// 135-192): the query's INT8 code first (quantizedQuery: validation, then
// quantization), the IVF probe with the original metric (ivf_probe, shared
// with the exact IVF), then the scalar-quantized scoring of the probed
// lists' positions (searchWithCode, quantized_index.go:313-335), and the
// refine stage when a refine scale is given (refiner.go:66-129).
// ---------------------------------------------------------------------------
xvec_gpu_status ivf_sq8_search_impl(xvec_gpu_index* idx, const float* d_q, int nq,
                                    const xvec_gpu_search_opts& o, const uint32_t* d_bitmap,
                                    uint64_t* d_keys, float* d_scores, int* d_counts,
                                    cudaStream_t s, std::vector<int>* statuses,
                                    bool candidates_only) {
  if (!idx->has_model) return set_error("IVF index has no model"), XVEC_GPU_INVALID_ARGUMENT;
  if (o.nprobe <= 0) return set_error("core: IVF NProbe must be positive"), XVEC_GPU_INVALID_ARGUMENT;
  EventTimer timer(s);
  timer.mark(0);
  const int d = idx->desc.dimension, metric = idx->desc.metric;
  const int64_t n = idx->n;
  const bool refine = o.refine_scale > 0;
  if (candidates_only && !refine)
    return set_error("candidates of a search without refinement"), XVEC_GPU_INVALID_ARGUMENT;
  int stage_k = o.top_k;
  if (refine) {
    if (std::isinf(o.refine_scale))
      return set_error("core: refiner scale factor must be finite and positive"),
             XVEC_GPU_INVALID_ARGUMENT;
    const double product = (double)o.top_k * (double)o.refine_scale;
    if (product >= 1024.0 + 1.0)
      return set_error("refinement candidate count %.0f exceeds 1024", std::floor(product)),
             XVEC_GPU_INVALID_ARGUMENT;
    stage_k = std::max(1, (int)std::floor(product));  // RefinementCandidateCount
  }
  const float stage_radius = refine ? 0.f : o.radius;  // collection.go:1623
  xvec_gpu_status st;
  {
    static std::mutex rebuild_mu;
    std::lock_guard<std::mutex> g(rebuild_mu);
    if (idx->lists_dirty && n > 0 && (st = rebuild_lists(idx, s))) return st;
  }
  const int nprobe = std::min(o.nprobe, idx->nlist);
  const int kp = sq8_kp(stage_k);
  if ((int64_t)kIvfWarps * kp > flat_merge_capacity())
    return set_error("top_k %d exceeds the merge capacity", stage_k), XVEC_GPU_INVALID_ARGUMENT;
  // The probe's query terms (metric.Compute validation, cosine magnitudes).
  Scratch pf, pn2, paux, pstatus, pkeys, pscores, pcounts;
  if ((st = pf.alloc((size_t)nq * d * 4, s)) || (st = pn2.alloc((size_t)nq * 4, s)) ||
      (st = paux.alloc((size_t)nq * 4, s)) || (st = pstatus.alloc((size_t)nq * 4, s)) ||
      (st = pkeys.alloc((size_t)nq * nprobe * 8, s)) ||
      (st = pscores.alloc((size_t)nq * nprobe * 4, s)) || (st = pcounts.alloc((size_t)nq * 4, s)))
    return st;
  // The scalar-quantized query.
  Scratch qcodes, qparams, qf, qinfo, qeps, qstatus, qflags;
  if ((st = qcodes.alloc((size_t)nq * d, s)) ||
      (st = qparams.alloc((size_t)nq * sizeof(SQParams), s)) ||
      (st = qf.alloc((size_t)nq * d * 4, s)) || (st = qinfo.alloc((size_t)nq * 16, s)) ||
      (st = qeps.alloc((size_t)nq * 4, s)) || (st = qstatus.alloc((size_t)nq * 4, s)) ||
      (st = qflags.alloc((size_t)nq * 4, s)))
    return st;
  XVEC_CUDA(cudaMemsetAsync(qflags.ptr, 0, (size_t)nq * 4, s));
  XVEC_CUDA(cudaMemsetAsync(qstatus.ptr, 0, (size_t)nq * 4, s));
  if (idx->desc.kind == XVEC_INDEX_IVF_SQ4)
    sq8_prep_queries_kernel<4><<<blocks_of((int64_t)nq * 32), 256, 0, s>>>(
        d_q, nq, d, metric, idx->sq_bounds.as<unsigned>(), qcodes.as<int8_t>(),
        qparams.as<SQParams>(), qf.as<float>(), qinfo.as<float4>(), qeps.as<float>(),
        qstatus.as<int>());
  else
    sq8_prep_queries_kernel<8><<<blocks_of((int64_t)nq * 32), 256, 0, s>>>(
        d_q, nq, d, metric, idx->sq_bounds.as<unsigned>(), qcodes.as<int8_t>(),
        qparams.as<SQParams>(), qf.as<float>(), qinfo.as<float4>(), qeps.as<float>(),
        qstatus.as<int>());
  XVEC_LAUNCHED();
  launch_prep_queries<float>(d_q, nq, d, metric, pf.as<float>(), pn2.as<float>(),
                             paux.as<float>(), pstatus.as<int>(), s);
  XVEC_LAUNCHED();
  std::vector<int> h_probe(nq), h_sq(nq);
  if ((st = ivf_probe(idx, d_q, nq, nprobe, pf.as<float>(), pn2.as<float>(), pstatus.as<int>(),
                      pkeys.as<uint64_t>(), pscores.as<float>(), pcounts.as<int>(),
                      qflags.as<int>(), &h_probe, s)))
    return st;
  XVEC_CUDA(cudaMemcpyAsync(h_sq.data(), qstatus.ptr, (size_t)nq * 4, cudaMemcpyDeviceToHost, s));
  XVEC_CUDA(cudaStreamSynchronize(s));
  // Per-query status before the scan: the quantization's, then the probe's.
  std::vector<int> h_status(nq);
  for (int q = 0; q < nq; ++q) h_status[q] = h_sq[q] ? h_sq[q] : h_probe[q];
  XVEC_CUDA(cudaMemcpyAsync(qstatus.ptr, h_status.data(), (size_t)nq * 4, cudaMemcpyHostToDevice,
                            s));
  // Stage outputs: the final outputs, or scratch when a refine stage follows.
  Scratch skeys, sscores, scounts, spos;
  uint64_t* o_keys = d_keys;
  float* o_scores = d_scores;
  int* o_counts = d_counts;
  if ((st = spos.alloc((size_t)nq * stage_k * 4, s))) return st;
  if (refine && !candidates_only) {
    if ((st = skeys.alloc((size_t)nq * stage_k * 8, s)) ||
        (st = sscores.alloc((size_t)nq * stage_k * 4, s)) ||
        (st = scounts.alloc((size_t)nq * 4, s)))
      return st;
    o_keys = skeys.as<uint64_t>();
    o_scores = sscores.as<float>();
    o_counts = scounts.as<int>();
  }
  XVEC_CUDA(cudaMemsetAsync(o_counts, 0, (size_t)nq * 4, s));
  int exact_count = 0;
  if (n > 0) {
    Scratch lkeys, lcounts, lsat;
    const size_t lists = (size_t)nq * kIvfWarps;
    if ((st = lkeys.alloc(lists * kp * 8, s)) || (st = lcounts.alloc(lists * 4, s)) ||
        (st = lsat.alloc(lists * 8, s)))
      return st;
    const SQ8Scorer sc{metric, idx->sq_codes.as<uint8_t>(), idx->sq_params.as<SQParams>(),
                       qcodes.as<int8_t>(), qparams.as<SQParams>(), qeps.as<float>(), d};
    const Sq8IvfPolicy pol{metric,
                           idx->sq_codes.as<int8_t>(),
                           idx->sq_params.as<SQParams>(),
                           idx->sq_fast.as<float4>(),
                           idx->list_sq_codes.ptr ? idx->list_sq_codes.as<int4>() : nullptr,
                           idx->list_sq_codes.ptr ? idx->list_sq_fast.as<float4>() : nullptr,
                           qcodes.as<int8_t>(),
                           qparams.as<SQParams>(),
                           qinfo.as<float4>(),
                           d};
    auto scan = [&](bool exact, const int* ids, int count) -> xvec_gpu_status {
      cudaError_t e =
          exact ? launch_ivf_list_scan<true>(pol, d, pkeys.as<uint64_t>(), pcounts.as<int>(),
                                             nprobe, idx->list_offsets.as<int64_t>(),
                                             idx->list_rows.as<uint32_t>(),
                                             idx->list_keyrank.as<uint32_t>(), d_bitmap, ids,
                                             count, kp, lkeys.as<uint64_t>(), lcounts.as<int>(),
                                             lsat.as<uint64_t>(), qflags.as<int>(), s)
                : launch_ivf_list_scan<false>(pol, d, pkeys.as<uint64_t>(), pcounts.as<int>(),
                                              nprobe, idx->list_offsets.as<int64_t>(),
                                              idx->list_rows.as<uint32_t>(),
                                              idx->list_keyrank.as<uint32_t>(), d_bitmap, ids,
                                              count, kp, lkeys.as<uint64_t>(), lcounts.as<int>(),
                                              lsat.as<uint64_t>(), qflags.as<int>(), s);
      if (e == cudaErrorInvalidValue)
        return set_error("top_k %d or dimension %d too large for the IVF scan", stage_k, d),
               XVEC_GPU_UNSUPPORTED;
      XVEC_CUDA(e);
      XVEC_LAUNCHED();
      XVEC_CUDA(launch_merge_rescore(sc, idx->pos_of_kr.as<uint32_t>(), idx->keys.as<uint64_t>(),
                                     ids, count, stage_k, stage_radius, exact ? 1 : 0,
                                     lkeys.as<uint64_t>(), lcounts.as<int>(), lsat.as<uint64_t>(),
                                     kIvfWarps, kp, o_keys, o_scores, o_counts,
                                     spos.as<uint32_t>(), qflags.as<int>(), s));
      XVEC_LAUNCHED();
      return XVEC_GPU_OK;
    };
    // Inner product and L2 have a fast rank; cosine and MIPS are scored in
    // reference order from the start.
    const bool ranked = metric == XVEC_METRIC_IP || metric == XVEC_METRIC_L2;
    timer.mark(1);
    std::vector<int> exact_list;
    if (ranked) {
      if ((st = scan(false, nullptr, nq))) return st;
      std::vector<int> h_fl(nq);
      XVEC_CUDA(cudaMemcpyAsync(h_fl.data(), qflags.ptr, (size_t)nq * 4, cudaMemcpyDeviceToHost,
                                s));
      XVEC_CUDA(cudaStreamSynchronize(s));
      for (int q = 0; q < nq; ++q)
        if (h_status[q] == 0 && (h_fl[q] & 3)) exact_list.push_back(q);
    } else {
      for (int q = 0; q < nq; ++q)
        if (h_status[q] == 0) exact_list.push_back(q);
    }
    timer.mark(2);
    if (!exact_list.empty()) {
      const int nl = (int)exact_list.size();
      Scratch ids;
      if ((st = ids.alloc((size_t)nl * 4, s))) return st;
      XVEC_CUDA(cudaMemcpyAsync(ids.ptr, exact_list.data(), (size_t)nl * 4,
                                cudaMemcpyHostToDevice, s));
      sq8_clear_flags<<<blocks_of(nl), 256, 0, s>>>(ids.as<int>(), nl, qflags.as<int>());
      XVEC_LAUNCHED();
      if ((st = scan(true, ids.as<int>(), nl))) return st;
      exact_count = nl;
      std::vector<int> h_fl(nq);
      XVEC_CUDA(cudaMemcpyAsync(h_fl.data(), qflags.ptr, (size_t)nq * 4, cudaMemcpyDeviceToHost,
                                s));
      XVEC_CUDA(cudaStreamSynchronize(s));
      for (int q : exact_list)
        if (h_fl[q] & 2)
          return set_error("exact scan could not complete query %d", q), XVEC_GPU_CUDA_ERROR;
    }
  }
  if (candidates_only) {
    // The approximate stage's candidates are the output.
  } else if (refine && n > 0) {
    // The approximate stage's failures are final; the refine stage sees
    // counts >= 0 only for healthy queries.
    sq8_status_kernel<<<blocks_of(nq), 256, 0, s>>>(qstatus.as<int>(), qflags.as<int>(), nq,
                                                    o_counts);
    XVEC_CUDA(cudaMemsetAsync(d_counts, 0, (size_t)nq * 4, s));
    XVEC_CUDA(launch_refine(idx->rows.as<float>(), d, metric, d_q, nq, spos.as<uint32_t>(),
                            o_counts, stage_k, idx->keyrank.as<uint32_t>(),
                            idx->pos_of_kr.as<uint32_t>(), idx->keys.as<uint64_t>(), o.top_k,
                            o.radius, d_keys, d_scores, d_counts, qflags.as<int>(), s));
    count_launches(2);
  } else if (refine) {
    XVEC_CUDA(cudaMemsetAsync(d_counts, 0, (size_t)nq * 4, s));
  }
  sq8_status_kernel<<<blocks_of(nq), 256, 0, s>>>(qstatus.as<int>(), qflags.as<int>(), nq,
                                                  d_counts);
  XVEC_LAUNCHED();
  if (candidates_only && metric == XVEC_METRIC_IP) {
    scores_to_ranks_kernel<<<blocks_of((int64_t)nq * stage_k), 256, 0, s>>>(
        d_scores, d_counts, nq, stage_k, metric);
    XVEC_LAUNCHED();
  }
  XVEC_CUDA(cudaGetLastError());
  std::vector<int> h_flags(nq);
  XVEC_CUDA(cudaMemcpyAsync(h_flags.data(), qflags.ptr, (size_t)nq * 4, cudaMemcpyDeviceToHost, s));
  timer.mark(3);
  XVEC_CUDA(cudaStreamSynchronize(s));
  count_search(nq, exact_count, timer.ms(1, 2), timer.ms(0, 3));
  if (statuses) {
    statuses->resize(nq);
    for (int q = 0; q < nq; ++q) {
      int sq = h_status[q];
      if (sq == 0 && (h_flags[q] & 4)) sq = XVEC_GPU_NON_FINITE;
      (*statuses)[q] = sq;
    }
  }
  return XVEC_GPU_OK;
}

}  // namespace xvec
