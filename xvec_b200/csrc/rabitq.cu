// rabitq.cu — one-bit RaBitQ linear scan with exact float32 refinement.
//
// Reference: the HNSW-RaBitQ index's linear scan and refine
// (internal/core/hnsw_rabitq.go:539-642, 739-801) over RaBitQModel codes with
// TotalBits = 1 (internal/core/rabitq.go:297-327, 372-430;
// rabitq_quantize.go:99-262, 302-310; rotation.go:123-153; fht.go:28-101).
//
//   model    centroids, rotation signs; the centroids are rotated once.
//   insert   prepare (cosine: normalise, float64 norm in index order), the
//            nearest centroid (L2, or IP for IP/cosine; ties to the lower
//            index, through a Flat index over the centroids), the FHT-Kac
//            rotation of the zero-padded vector (shared memory, each butterfly
//            elementwise so the float32 results are the reference's), the
//            sign bits of the residual and the float64 factors (sums in index
//            order, explicit round-to-nearest operations).
//   query    PrepareQuery: rotated query, float64 sum, per-centroid gAdd and
//            gError (sequential float64 sums).
//   scan     fast estimate: the bit-plane x query dot as an exact integer
//            dot product on INT8 tensor cores (flat_tc.cu; the query rounded
//            to integers with a per-query scale and an exact bound on that
//            rounding), or in float32 on the shared FFMA tile kernel; the
//            estimate formula in float32 within a bound eps of the reference;
//            candidates are rescored with EstimateCoarse's float64 masked sum
//            in index order.
//   refine   the k best by metric.Compute on the original rows among the
//            candidate_count best estimates (refine.cuh).
#include <algorithm>
#include <cmath>
#include <vector>

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "capi_internal.h"
#include "common.cuh"
#include "flat_kernels.cuh"
#include "fht.cuh"
#include "flat_tc.cuh"
#include "index_kernels.cuh"
#include "pipeline.cuh"
#include "refine.cuh"

namespace xvec {

xvec_gpu_status add_device_locked(xvec_gpu_index* idx, const uint64_t* d_keys, const void* d_rows,
                                  int64_t m, cudaStream_t s);

struct RaBitQFactors {
  double add;           // coarse (one-bit) factors
  double rescale;
  double error;
  double full_add;      // multi-bit factors (equal to the coarse ones for one bit)
  double full_rescale;
  int32_t cluster;
  int32_t pad_;
};

// A row of packed sign bits seen by the FFMA tile kernel as 0/1 elements.
struct BitElem {
  uint8_t raw;
};
__device__ __forceinline__ float load_elem(const BitElem* p, int64_t i) {
  const uint8_t* b = reinterpret_cast<const uint8_t*>(p);
  return (float)((b[i >> 3] >> (i & 7)) & 1u);
}
// Multi-bit code values as 16-bit floats (bfloat16 up to 8 bits, binary16
// for 9), seen by the FFMA tile kernel and the exact scorer.
struct Bf16Value {
  __nv_bfloat16 v;
};
struct HalfValue {
  __half v;
};
__device__ __forceinline__ float load_elem(const Bf16Value* p, int64_t i) {
  return __bfloat162float(p[i].v);
}
__device__ __forceinline__ float load_elem(const HalfValue* p, int64_t i) {
  return __half2float(p[i].v);
}
// The value at coordinate i of a row of the 16-bit plane.
__device__ __forceinline__ double rabitq_value(const uint16_t* row, int i, bool half) {
  const uint16_t raw = row[i];
  return half ? (double)__half2float(__ushort_as_half(raw))
              : (double)__bfloat162float(__ushort_as_bfloat16(raw));
}

namespace {

constexpr double kU = 5.9604644775390625e-8;  // 2^-24
// q_flags bits of this file (bits 1 and 2 belong to the pipeline, 4 to refine).
constexpr int kRaBitQInvalid = 8;      // ErrInvalidRaBitQCode
constexpr int kRaBitQOverflow = 16;    // ErrQuantizationOverflow
constexpr int kRaBitQFullCheck = 32;   // estimates may fail: check every row
constexpr int kRaBitQGraphFull = 64;   // the graph walk's frontier outgrew its buffer
// DefaultHNSWBruteForceThreshold (hnsw.go:592): indexes of at most this many
// rows are scanned linearly even with a graph.
constexpr int64_t kHNSWBruteForce = 1000;
inline unsigned blocks_of(int64_t n, int t = 256) { return (unsigned)((n + t - 1) / t); }

// normalizeRaBitQVector (rabitq.go:514-526) of v[0, d) in shared memory.
__device__ void block_normalize(float* v, int d) {
  __shared__ float s_inv;
  __shared__ int s_skip;
  if (threadIdx.x == 0) {
    double ns = 0.0;
    for (int i = 0; i < d; ++i) ns = __dadd_rn(ns, __dmul_rn((double)v[i], (double)v[i]));
    s_skip = ns == 0.0;
    s_inv = s_skip ? 0.f : __double2float_rn(__ddiv_rn(1.0, __dsqrt_rn(ns)));
  }
  __syncthreads();
  if (!s_skip)
    for (int i = threadIdx.x; i < d; i += blockDim.x) v[i] = __fmul_rn(v[i], s_inv);
  __syncthreads();
}

// Loads v (d floats) zero-padded to `padded`, optionally normalises, rotates.
__device__ bool block_prepare_rotate(const float* src, int d, int padded, int truncated,
                                     const uint8_t* signs, float inv, bool normalize, float* v) {
  for (int i = threadIdx.x; i < padded; i += blockDim.x) v[i] = i < d ? src[i] : 0.f;
  __syncthreads();
  if (normalize) block_normalize(v, d);
  block_fht_rotate(v, padded, truncated, signs, inv);  // FHTRotator.Rotate
  __shared__ int s_bad;
  if (threadIdx.x == 0) s_bad = 0;
  __syncthreads();
  for (int i = threadIdx.x; i < padded; i += blockDim.x)
    if (!finite_f(v[i])) s_bad = 1;
  __syncthreads();
  return !s_bad;
}

// Rotated model centroids (RestoreRaBitQModel, rabitq.go:224-230).
__global__ void rabitq_rotate_centroids_kernel(const float* centroids, int d, int padded,
                                               int truncated, const uint8_t* signs, float inv,
                                               float* out, int* err) {
  extern __shared__ float v[];
  if (!block_prepare_rotate(centroids + (int64_t)blockIdx.x * d, d, padded, truncated, signs, inv,
                            false, v) &&
      threadIdx.x == 0)
    atomicExch(err, XVEC_GPU_NON_FINITE);
  for (int i = threadIdx.x; i < padded; i += blockDim.x) out[(int64_t)blockIdx.x * padded + i] = v[i];
}

// prepareRaBitQVector for rows that are assigned before rotation.
__global__ void rabitq_prepare_kernel(const float* rows, int64_t n, int d, bool normalize,
                                      float* out) {
  extern __shared__ float v[];
  const float* src = rows + (int64_t)blockIdx.x * d;
  for (int i = threadIdx.x; i < d; i += blockDim.x) v[i] = src[i];
  __syncthreads();
  if (normalize) block_normalize(v, d);
  for (int i = threadIdx.x; i < d; i += blockDim.x) out[(int64_t)blockIdx.x * d + i] = v[i];
}

// raBitQFactors (rabitq_quantize.go:210-262) from its five float64 sums
// (index order); ok = false where the reference returns an error.
__device__ bool rabitq_factor_formula(double ns, double cns, double rcd, double ccd, double rcent,
                                      int padded, int inner_product, double* add,
                                      double* rescale, double* errf) {
  if (ns == 0) {
    *add = inner_product ? 1.0 : 0.0;
    *rescale = 0.0;
    *errf = 0.0;
    return true;
  }
  if (!(rcd > 0) || isinf(rcd)) return false;
  double ratio = __dsub_rn(__ddiv_rn(__dmul_rn(ns, cns), __dmul_rn(rcd, rcd)), 1.0);
  if (ratio < 0 && ratio > -1e-12) ratio = 0;
  if (ratio < 0 || isnan(ratio) || isinf(ratio)) return false;
  const double norm = __dsqrt_rn(ns);
  const double te =
      __dmul_rn(__dmul_rn(norm, 1.9), __dsqrt_rn(__ddiv_rn(ratio, (double)(padded - 1))));
  if (inner_product) {
    *add = __dadd_rn(__dsub_rn(1.0, rcent), __ddiv_rn(__dmul_rn(ns, ccd), rcd));
    *rescale = __ddiv_rn(-ns, rcd);
    *errf = te;
  } else {
    *add = __dadd_rn(ns, __ddiv_rn(__dmul_rn(__dmul_rn(2.0, ns), ccd), rcd));
    *rescale = __ddiv_rn(__dmul_rn(-2.0, ns), rcd);
    *errf = __dmul_rn(2.0, te);
  }
  return isfinite(*add) && isfinite(*rescale) && isfinite(*errf);
}

// The extra-bit quantization of one coordinate (quantizeRaBitQVector,
// rabitq_quantize.go:140-180): an = |r| / norm, q = int(scale an + 1e-5)
// clamped to [0, 2^eb - 1], the extra value (mirrored for r < 0), the factor
// value extra | (r >= 0) << eb and the code value extra | (r > 0) << eb.
struct RaBitQExtra {
  double an;
  int q, factor_value, code_value;
};
__device__ __forceinline__ RaBitQExtra rabitq_extra(double res, double norm, double extra_scale,
                                                    int eb) {
  RaBitQExtra x{0.0, 0, 0, 0};
  if (!(norm > 0)) return x;  // the reference leaves every value zero
  const int max_extra = (1 << eb) - 1;
  x.an = __ddiv_rn(fabs(res), norm);
  int q = __double2int_rz(__dadd_rn(__dmul_rn(extra_scale, x.an), 1e-5));
  q = min(max(q, 0), max_extra);
  x.q = q;
  const int e = res < 0 ? max_extra - q : q;
  x.factor_value = e | ((res >= 0 ? 1 : 0) << eb);
  x.code_value = e | ((res > 0 ? 1 : 0) << eb);
  return x;
}

// quantizeRaBitQVector (rabitq_quantize.go:99-200) and raBitQFactors
// (rabitq_quantize.go:210-262), one block per row: the sign bits, the coarse
// factors and, for TotalBits > 1, the full code values (16-bit floats) and the
// full factors (full rescale = -norm / ip (IP) or -2 norm / ip, ip = sum of
// (q + 1/2) an in index order).
__global__ void rabitq_encode_kernel(const float* prepared, int64_t n, int d, int padded,
                                     int truncated, const uint8_t* signs, float inv,
                                     const float* rot_centroids, const int32_t* labels,
                                     int inner_product, int total_bits, double extra_scale,
                                     uint8_t* codes, uint16_t* values, RaBitQFactors* factors,
                                     float4* fast, unsigned* bounds, int* err) {
  extern __shared__ float smem[];
  float* v = smem;                 // [padded] rotated row
  __shared__ double s_sum[4];
  __shared__ double s_full[4];
  const int eb = total_bits - 1;
  const int64_t r = blockIdx.x;
  if (!block_prepare_rotate(prepared + r * d, d, padded, truncated, signs, inv, false, v)) {
    if (threadIdx.x == 0) atomicExch(err, XVEC_GPU_NON_FINITE);
    return;
  }
  const int c = labels[r];
  const float* cen = rot_centroids + (int64_t)c * padded;
  // Sign bits of the residual, LSB first (setRaBitQBit).
  for (int byte = threadIdx.x; byte < padded / 8; byte += blockDim.x) {
    uint8_t b = 0;
    for (int j = 0; j < 8; ++j) {
      const int i = byte * 8 + j;
      const double res = __dsub_rn((double)v[i], (double)cen[i]);
      if (res > 0) b |= (uint8_t)(1u << j);
    }
    codes[r * (padded / 8) + byte] = b;
  }
  // The four float64 sums of raBitQFactors, each in index order.
  if (threadIdx.x < 4) {
    double acc = 0.0;
    for (int i = 0; i < padded; ++i) {
      const double res = __dsub_rn((double)v[i], (double)cen[i]);
      const double cc = res > 0 ? 0.5 : -0.5;  // value + center, center = -(2^1 - 1)/2
      const double ce = (double)cen[i];
      double t;
      if (threadIdx.x == 0) t = __dmul_rn(res, res);        // normSquared
      else if (threadIdx.x == 1) t = __dmul_rn(res, cc);    // residualCodeDot
      else if (threadIdx.x == 2) t = __dmul_rn(ce, cc);     // centroidCodeDot
      else t = __dmul_rn(res, ce);                          // residualCentroidDot
      acc = __dadd_rn(acc, t);
    }
    s_sum[threadIdx.x] = acc;
  }
  __syncthreads();
  const double norm = __dsqrt_rn(s_sum[0]);
  if (eb > 0) {
    // The code values (any order), then the full sums (index order): ip of
    // the extra quantization, and the code norm, residual and centroid dots
    // of the factor values (center -(2^TotalBits - 1)/2).
    const bool half = total_bits > 8;
    for (int i = threadIdx.x; i < padded; i += blockDim.x) {
      const double res = __dsub_rn((double)v[i], (double)cen[i]);
      const float cv = (float)rabitq_extra(res, norm, extra_scale, eb).code_value;
      values[r * padded + i] = half ? __half_as_ushort(__float2half_rn(cv))
                                    : __bfloat16_as_ushort(__float2bfloat16_rn(cv));
    }
    if (threadIdx.x < 4) {
      const double center = -((double)(1 << total_bits) - 1.0) / 2.0;
      double acc = 0.0;
      for (int i = 0; i < padded; ++i) {
        const double res = __dsub_rn((double)v[i], (double)cen[i]);
        const RaBitQExtra x = rabitq_extra(res, norm, extra_scale, eb);
        const double cc = __dadd_rn((double)x.factor_value, center);
        double t;
        if (threadIdx.x == 0) {
          if (!(norm > 0)) continue;
          t = __dmul_rn(__dadd_rn((double)x.q, 0.5), x.an);  // ip of the quantization
        } else if (threadIdx.x == 1) {
          t = __dmul_rn(cc, cc);                    // codeNormSquared
        } else if (threadIdx.x == 2) {
          t = __dmul_rn(res, cc);                   // residualCodeDot
        } else {
          t = __dmul_rn((double)cen[i], cc);        // centroidCodeDot
        }
        acc = __dadd_rn(acc, t);
      }
      s_full[threadIdx.x] = acc;
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    const double ns = s_sum[0], rcd = s_sum[1], ccd = s_sum[2], rcent = s_sum[3];
    const double cns = 0.25 * (double)padded;  // sum of 0.25 over padded terms, exact
    double add, rescale, errf;
    bool ok = rabitq_factor_formula(ns, cns, rcd, ccd, rcent, padded, inner_product, &add,
                                    &rescale, &errf);
    double fadd = add, frescale = rescale, ferr_scaled = errf;
    if (ok && eb > 0) {
      double unused;
      ok = rabitq_factor_formula(ns, s_full[1], s_full[2], s_full[3], rcent, padded,
                                 inner_product, &fadd, &frescale, &unused);
      const double ipn = s_full[0];
      const double inv_ip = (norm > 0 && ipn > 0 && isfinite(ipn)) ? __ddiv_rn(1.0, ipn) : 1.0;
      frescale = inner_product ? __dmul_rn(-norm, inv_ip) : __dmul_rn(__dmul_rn(-2.0, norm), inv_ip);
      ferr_scaled = ldexp(errf, -eb);  // Estimate's error bound over 2^extra bits
    }
    if (!ok) {
      atomicExch(err, XVEC_GPU_OVERFLOW);
      return;
    }
    factors[r] = RaBitQFactors{add, rescale, errf, fadd, frescale, c, 0};
    fast[r] = make_float4(__double2float_rn(fadd), __double2float_rn(frescale), __int_as_float(c),
                          0.f);
    atomicMax(&bounds[0], float_to_ordered(fabsf(__double2float_rn(fadd))));
    atomicMax(&bounds[1], float_to_ordered(fabsf(__double2float_rn(frescale))));
    atomicMax(&bounds[2], float_to_ordered(__double2float_ru(ferr_scaled)));
  }
}

// The sign bits as the tensor-core scan's int8 planes: row r holds
// [127 b_0 .. 127 b_{padded-1} | b_0 .. b_{padded-1}], one thread per code byte.
__global__ void rabitq_planes_kernel(const uint8_t* __restrict__ codes, int64_t bytes_total,
                                     int padded, int8_t* __restrict__ planes) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= bytes_total) return;
  const int bpr = padded / 8;
  const int64_t r = i / bpr;
  const int col = (int)(i - r * bpr) * 8;
  const uint32_t b = codes[i];
  uint32_t lo = 0, hi = 0;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    lo |= ((b >> j) & 1u) << (8 * j);
    hi |= ((b >> (j + 4)) & 1u) << (8 * j);
  }
  int8_t* row = planes + r * 2 * padded;
  *reinterpret_cast<uint2*>(row + col) = make_uint2(lo * 127u, hi * 127u);
  *reinterpret_cast<uint2*>(row + padded + col) = make_uint2(lo, hi);
}

// Multi-bit code values (TotalBits <= 8, bfloat16, exact) as the INT8
// tensor-core operand v - 128, and the row's 128 sum(v - 128) into the w slot
// of its fast terms (one warp per row).
__global__ void rabitq_vplane_kernel(const uint16_t* __restrict__ values, int64_t m, int padded,
                                     int8_t* __restrict__ plane, float4* __restrict__ fast) {
  const int64_t r = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (r >= m) return;
  int sum = 0;
  for (int i = lane; i < padded; i += 32) {
    const int v = (int)__bfloat162float(__ushort_as_bfloat16(values[r * padded + i]));
    plane[r * padded + i] = (int8_t)(v - 128);
    sum += v - 128;
  }
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(kFullMask, sum, o);
  if (lane == 0) fast[r].w = 128.f * (float)sum;
}

// Estimate's center, -(2^(TotalBits-1) - 1/2).
__device__ __forceinline__ double center_of(int total_bits) {
  return -(ldexp(1.0, total_bits - 1) - 0.5);
}

// The query of the multi-bit INT8 scan: w = round(v / scale) with
// |w| <= 32767 (scale = max |v| / 32767), as w = 256 h + l + 128 with h, l
// signed bytes.
constexpr int kRaBitQInt16Max = 32767;

// The query as the integers of the tensor-core scan: w = round(v / scale)
// with |w| <= kRaBitQIntMax, written as w = 127 h + l (|h| <= 127, |l| <= 63).
constexpr int kRaBitQIntMax = 127 * 127 + 63;
__device__ __forceinline__ int rabitq_query_int(float v, float scale) {
  if (!(scale > 0.f)) return 0;
  const double w = rint((double)v / (double)scale);
  return (int)fmin(fmax(w, -(double)kRaBitQIntMax), (double)kRaBitQIntMax);
}

// PrepareQuery (rabitq.go:372-408) + the fast-estimate constants and eps.
__global__ void rabitq_prep_query_kernel(const float* queries, int nq, int d, int padded,
                                         int truncated, const uint8_t* signs, float inv,
                                         int normalize, int metric, const float* rot_centroids,
                                         int nc, const unsigned* bounds, float* q_rot,
                                         double* q_sum, double* g_add, double* g_error,
                                         float* q_fast_sum, float* q_fast_gadd, float* q_eps,
                                         int* q_exact, int* q_status, int* q_flags,
                                         int8_t* q_int, float2* q_terms, int total_bits,
                                         int8_t* q_planes8) {
  // total_bits > 1: q_int is unused; q_planes8 (optional, the multi-bit INT8
  // tensor-core scan): the 16-bit integer query as planes [2][nq][padded]
  // (h, then l); q_terms and q_eps then follow that form, else the FFMA
  // scan's.
  const bool multi = total_bits > 1;
  const bool int8_form = multi && q_planes8 != nullptr;
  const double vmax = (double)((1 << total_bits) - 1);  // largest code value
  extern __shared__ float v[];
  __shared__ double s_sum;
  __shared__ float s_abs;
  const int q = blockIdx.x;
  const float* src = queries + (int64_t)q * d;
  __shared__ int s_bad;
  if (threadIdx.x == 0) s_bad = 0;
  __syncthreads();
  for (int i = threadIdx.x; i < d; i += blockDim.x)
    if (!finite_f(src[i])) s_bad = 1;
  __syncthreads();
  // A query PrepareQuery rejects gets neutral values (it is never scored).
  auto reject = [&]() {
    for (int i = threadIdx.x; i < padded; i += blockDim.x) {
      q_rot[(int64_t)q * padded + i] = 0.f;
      if (multi) {
        if (int8_form) {
          q_planes8[(int64_t)q * padded + i] = 0;
          q_planes8[((int64_t)nq + q) * padded + i] = 0;
        }
      } else {
        q_int[(int64_t)q * 2 * padded + i] = 0;
        q_int[(int64_t)q * 2 * padded + padded + i] = 0;
      }
    }
    for (int c = threadIdx.x; c < nc; c += blockDim.x) {
      g_add[(int64_t)q * nc + c] = 0.0;
      g_error[(int64_t)q * nc + c] = 0.0;
      q_fast_gadd[(int64_t)q * nc + c] = 0.f;
    }
    if (threadIdx.x == 0) {
      q_sum[q] = 0.0;
      q_fast_sum[q] = 0.f;
      q_terms[q] = make_float2(0.f, 0.f);
      q_eps[q] = 0.f;
      q_exact[q] = 1;
      q_status[q] = XVEC_GPU_NON_FINITE;
    }
  };
  if (s_bad) {
    reject();
    return;
  }
  if (!block_prepare_rotate(src, d, padded, truncated, signs, inv, normalize != 0, v)) {
    reject();
    return;
  }
  for (int i = threadIdx.x; i < padded; i += blockDim.x) q_rot[(int64_t)q * padded + i] = v[i];
  __shared__ float s_maxabs, s_scale;
  __shared__ double s_resid, s_wsum, s_wabs;
  if (threadIdx.x == 0) {
    double s = 0.0, a = 0.0;
    float mx = 0.f;
    int g = 1 << 20;  // least exponent of an ulp among the non-zero values
    for (int i = 0; i < padded; ++i) {
      s = __dadd_rn(s, (double)v[i]);
      a = __dadd_rn(a, fabs((double)v[i]));
      mx = fmaxf(mx, fabsf(v[i]));
      if (v[i] != 0.f) {
        const int e = (int)((float_bits(v[i]) >> 23) & 0xffu);
        g = min(g, e == 0 ? -149 : e - 150);
      }
    }
    s_sum = s;
    s_abs = (float)a;
    s_maxabs = mx;
    q_sum[q] = s;
    q_fast_sum[q] = __double2float_rn(s);
    // The scale of the tensor-core scan's integer query.
    const float scale = mx > 0.f ? mx / (float)kRaBitQIntMax : 0.f;
    s_scale = int8_form ? (mx > 0.f ? mx / (float)kRaBitQInt16Max : 0.f) : scale;
    s_resid = 0.0;
    s_wsum = 0.0;
    s_wabs = 0.0;
    // Multi-bit: -(center sum), center = -(2^(TotalBits-1) - 1/2) (Estimate);
    // the INT8 form's terms are set once sum(w) is known (below).
    const double center = multi ? center_of(total_bits) : -0.5;
    q_terms[q] = multi ? make_float2(-__double2float_rn(__dmul_rn(center, s)), 0.f)
                       : make_float2(0.5f * __double2float_rn(s), scale);
    // Every value is a multiple of 2^g, so is every product with a code value
    // (at most vmax), and every partial sum of such products is at most
    // vmax a in magnitude; below 2^(52+g) all of them are exact in float64,
    // so the sums may be taken in any order.
    q_exact[q] = (g == (1 << 20)) || __dmul_ru(a, vmax) <= ldexp(1.0, min(1000, 52 + g));
  }
  for (int c = threadIdx.x; c < nc; c += blockDim.x) {
    const float* cen = rot_centroids + (int64_t)c * padded;
    double sq = 0.0, dot = 0.0;
    for (int i = 0; i < padded; ++i) {
      const double diff = __dsub_rn((double)v[i], (double)cen[i]);
      sq = __dadd_rn(sq, __dmul_rn(diff, diff));
      dot = __dadd_rn(dot, __dmul_rn((double)v[i], (double)cen[i]));
    }
    g_error[(int64_t)q * nc + c] = __dsqrt_rn(sq);
    const double ga = metric == kMetricL2 ? sq : -dot;
    g_add[(int64_t)q * nc + c] = ga;
    q_fast_gadd[(int64_t)q * nc + c] = __double2float_rn(ga);
  }
  __syncthreads();
  if (multi) {
    if (int8_form) {
      // w = round(v / scale), |w| <= 32767, as h = floor(w / 256) and
      // l = (w mod 256) - 128; sum w, sum |w| and the rounding bound
      // sum |v - scale w| (each term exact in float64).
      const float scale = s_scale;
      int8_t* ph = q_planes8 + (int64_t)q * padded;
      int8_t* pl = q_planes8 + ((int64_t)nq + q) * padded;
      double resid = 0.0, wsum = 0.0, wabs = 0.0;
      for (int i = threadIdx.x; i < padded; i += blockDim.x) {
        int w = 0;
        if (scale > 0.f) {
          const double t = rint((double)v[i] / (double)scale);
          w = (int)fmin(fmax(t, -(double)kRaBitQInt16Max), (double)kRaBitQInt16Max);
        }
        ph[i] = (int8_t)(w >> 8);
        pl[i] = (int8_t)((w & 255) - 128);
        resid += fabs((double)v[i] - (double)scale * (double)w);
        wsum += (double)w;
        wabs += fabs((double)w);
      }
      for (int o = 16; o > 0; o >>= 1) {
        resid += __shfl_xor_sync(0xffffffffu, resid, o);
        wsum += __shfl_xor_sync(0xffffffffu, wsum, o);
        wabs += __shfl_xor_sync(0xffffffffu, wabs, o);
      }
      if ((threadIdx.x & 31) == 0) {
        atomicAdd(&s_resid, resid);
        atomicAdd(&s_wsum, wsum);
        atomicAdd(&s_wabs, wabs);
      }
    }
  } else {
    // The integer query and the bound on its rounding, sum |v_i - scale w_i|
    // (each term exact in float64; the sum is only a bound).
    const float scale = s_scale;
    int8_t* qi = q_int + (int64_t)q * 2 * padded;
    double resid = 0.0;
    for (int i = threadIdx.x; i < padded; i += blockDim.x) {
      const int w = rabitq_query_int(v[i], scale);
      const int h = (int)rintf((float)w / 127.f);
      qi[i] = (int8_t)h;
      qi[padded + i] = (int8_t)(w - 127 * h);
      resid += fabs((double)v[i] - (double)scale * (double)w);
    }
    for (int o = 16; o > 0; o >>= 1) resid += __shfl_xor_sync(0xffffffffu, resid, o);
    if ((threadIdx.x & 31) == 0) atomicAdd(&s_resid, resid);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    double maxg = 0.0, maxge = 0.0;
    for (int c = 0; c < nc; ++c) {
      maxg = fmax(maxg, fabs(g_add[(int64_t)q * nc + c]));
      maxge = fmax(maxge, g_error[(int64_t)q * nc + c]);
    }
    const double maxA = ordered_to_float(bounds[0]), maxR = ordered_to_float(bounds[1]);
    const double maxE = ordered_to_float(bounds[2]);
    const double S1 = (double)s_abs * 1.001;
    const double sumd = fabs(s_sum);
    // Multi-bit: |dot + center sum| <= vmax S1 + |center sum|.
    const double csum = multi ? (ldexp(1.0, total_bits - 1) - 0.5) * sumd : 0.5 * sumd;
    // |estimate| and its error bound over every row; far below MaxFloat32 no
    // row can fail makeRaBitQEstimate and the float32 fast rank is finite.
    const double reach = maxA + maxg + maxR * (vmax * S1 + csum) + maxE * maxge;
    if (!(reach < 1e37)) q_flags[q] |= 1 | kRaBitQFullCheck;
    // Bound on |fast rank - float32(estimate)|: the float32 sum of up to
    // padded terms (FFMA scan) or the integer query's rounding plus the
    // float32 conversion and scaling of the exact integer dot product
    // (tensor-core scan), the float32 roundings of the inputs and of each
    // operation.
    double e;
    if (int8_form) {
      // The exact integer dots leave the query's rounding, vmax sum |v - s w|,
      // and the float32 evaluation of dp = 256 A_h + A_l + 128 sum(v - 128)
      // (each |term| <= 128 (sum |w| + 384 padded), the row term <= 2^14
      // padded; the int32-to-float conversions, the fma and the add) and of
      // s dp - x (one fma).
      const double scale = (double)s_scale;
      const double dpmag = 128.0 * (s_wabs + 384.0 * padded) + 16384.0 * padded;
      const double x = fabs(-__dmul_rn(center_of(total_bits), s_sum) -
                            scale * 128.0 * s_wsum);
      const double dot_err = vmax * s_resid * 1.0001 +
                             kU * (5.0 * scale * dpmag + x) * 1.01;
      e = maxR * (dot_err + kU * csum) + 6.0 * kU * (maxA + maxg + maxR * (vmax * S1 + csum));
    } else if (multi) {
      // The FFMA scan (TotalBits 9, or clusters beyond the tensor-core
      // epilogue's table): a float32 sum of padded products of exact 16-bit
      // code values with the float32 query, bounded here with a margin for
      // any accumulation order (2 padded + 8 roundings, plus 2^-16 relative
      // and the underflow of each term), then the float32 roundings of the
      // terms and of the formula.
      const double dot_err =
          vmax * (S1 * (ldexp(1.0, -16) + (2.0 * padded + 8.0) * ldexp(1.0, -23) * 1.01) +
                  (double)padded * ldexp(1.0, -126));
      e = maxR * (dot_err + kU * csum) + 6.0 * kU * (maxA + maxg + maxR * (vmax * S1 + csum));
    } else {
      const double resid = s_resid * 1.0001;
      const double dot_err = fmax((double)(padded + 2) * kU * S1,
                                  resid + 3.0 * kU * (S1 + resid));
      e = maxR * dot_err + 6.0 * kU * (maxA + maxg + maxR * (S1 + 0.5 * sumd));
    }
    q_eps[q] = (float)(2.5 * e) + 1e-30f;
    if (int8_form) {
      // {-(center sum) - scale 128 sum(w), scale}: s dp - x = s sum(v w)
      // + center sum (sum(v w) = dp + 128 sum(w)).
      const double scale = (double)s_scale;
      q_terms[q] = make_float2(
          __double2float_rn(-__dmul_rn(center_of(total_bits), s_sum) - scale * 128.0 * s_wsum),
          s_scale);
    }
    // Magnitudes whose scale would lose precision go to the exact scan.
    if (!(s_maxabs < 1e30f) || (s_maxabs > 0.f && s_maxabs < 1e-30f)) q_flags[q] |= 1;
    q_status[q] = 0;
  }
}

__host__ __device__ inline int rabitq_query_status(int prep, int flags, int refine_status) {
  if (prep) return prep;
  if (flags & kRaBitQInvalid) return XVEC_GPU_INVALID_ARGUMENT;
  if (flags & kRaBitQOverflow) return XVEC_GPU_OVERFLOW;
  if (flags & kRaBitQGraphFull) return XVEC_GPU_UNSUPPORTED;
  if (refine_status) return refine_status;
  if (flags & 4) return XVEC_GPU_NON_FINITE;
  return 0;
}

// FULL: the multi-bit estimate, dot - q_terms.x with q_terms.x = -(center sum).
template <bool FULL>
struct RaBitQRanker {
  const float4* fast;
  const float* q_fast_sum;
  const float* q_fast_gadd;
  int nc;
  const float2* q_terms;
  struct RowInfo {
    float add, rescale;
    int cluster;
  };
  struct QueryInfo {
    int qi;
    float half_sum;
  };
  __device__ QueryInfo query(int qi) const {
    if constexpr (FULL) return {qi, q_terms[qi].x};
    return {qi, 0.5f * q_fast_sum[qi]};
  }
  __device__ RowInfo row(int64_t r) const {
    const float4 f = fast[r];
    return {f.x, f.y, __float_as_int(f.z)};
  }
  __device__ float rank(float dot, const RowInfo& r, const QueryInfo& q) const {
    return fmaf(r.rescale, dot - q.half_sum, r.add + q_fast_gadd[(int64_t)q.qi * nc + r.cluster]);
  }
};

// EstimateCoarse (rabitq.go:421-430) + makeRaBitQEstimate (rabitq.go:464-476).
// The masked sum is the reference's float64 sum in index order: taken by the
// whole warp when every partial sum is exact for this query (q_exact), else
// sequentially by lane 0.  An invalid estimate scores NaN, an overflowing one
// +inf (error_flag tells them apart).
struct RaBitQScorer {
  int metric;         // ordering: estimates rank ascending for every metric
  int public_metric;  // the index metric, for the reported score without refine
  const uint8_t* codes;
  const RaBitQFactors* factors;
  const float* q_rot;
  const double* q_sum;
  const double* g_add;
  const double* g_error;
  const float* q_eps;
  const int* q_exact;
  int padded, nc;
  int total_bits;          // > 1: Estimate on the full code values
  const uint16_t* values;  // [n][padded] 16-bit floats (multi-bit)
  __device__ float score(int qi, int64_t row) const {
    const int lane = threadIdx.x & 31;
    const uint8_t* b = codes + row * (padded / 8);
    const float* q = q_rot + (int64_t)qi * padded;
    const bool multi = total_bits > 1, half = total_bits > 8;
    const uint16_t* vrow = multi ? values + row * padded : nullptr;
    // raBitQBinaryDot / raBitQFullCodeDot: float64 sum in index order (or in
    // any order when every partial sum is exact for this query).
    auto term = [&](int i) -> double {
      if (multi) return __dmul_rn(rabitq_value(vrow, i, half), (double)q[i]);
      return (b[i >> 3] & (1u << (i & 7))) ? (double)q[i] : 0.0;
    };
    double dot = 0.0;
    if (q_exact[qi]) {
      for (int i = lane; i < padded; i += 32) dot = __dadd_rn(dot, term(i));
      for (int o = 16; o > 0; o >>= 1) dot = __dadd_rn(dot, __shfl_xor_sync(kFullMask, dot, o));
    } else {
      if (lane == 0)
        for (int i = 0; i < padded; ++i) {
          const double t = term(i);
          if (multi || t != 0.0 || (b[i >> 3] & (1u << (i & 7)))) dot = __dadd_rn(dot, t);
        }
      dot = __shfl_sync(kFullMask, dot, 0);
    }
    const RaBitQFactors f = factors[row];
    double dist, eb;
    if (multi) {
      // Estimate (rabitq.go:434-446).
      const double center = -(ldexp(1.0, total_bits - 1) - 0.5);
      dist = __dadd_rn(__dadd_rn(f.full_add, g_add[(int64_t)qi * nc + f.cluster]),
                       __dmul_rn(f.full_rescale, __dadd_rn(dot, __dmul_rn(center, q_sum[qi]))));
      eb = __ddiv_rn(__dmul_rn(f.error, g_error[(int64_t)qi * nc + f.cluster]),
                     ldexp(1.0, total_bits - 1));
    } else {
      const double centered = __dsub_rn(dot, __dmul_rn(0.5, q_sum[qi]));
      dist = __dadd_rn(__dadd_rn(f.add, g_add[(int64_t)qi * nc + f.cluster]),
                       __dmul_rn(f.rescale, centered));
      eb = __dmul_rn(f.error, g_error[(int64_t)qi * nc + f.cluster]);
    }
    constexpr double kMaxF = 3.40282346638528859811704183484516925440e+38;
    if (isnan(dist) || isinf(dist) || isnan(eb) || isinf(eb) || eb < 0)
      return __int_as_float(0x7fc00000);
    if (fabs(dist) > kMaxF || eb > kMaxF) return __int_as_float(0x7f800000);
    if (__dsub_rn(dist, eb) < -kMaxF || __dadd_rn(dist, eb) > kMaxF)
      return __int_as_float(0x7f800000);
    return __double2float_rn(dist);
  }
  __device__ float eps(int qi) const { return q_eps[qi]; }
  __device__ int error_flag(float s) const { return isnan(s) ? kRaBitQInvalid : kRaBitQOverflow; }
  __device__ bool half_warp() const { return false; }
  // Without refinement the reported score is the public one
  // (publicRaBitQScore, hnsw_rabitq.go:746-751) and the radius applies to it
  // (acceptRaBitQNode, hnsw_rabitq.go:753-757).
  __device__ float output(float r) const {
    return public_metric == kMetricIP ? __fsub_rn(1.f, r) : r;
  }
  __device__ bool keep(float out, float radius) const {
    return within_radius(public_metric, out, radius);
  }
};

// ---------------------------------------------------------------------------
// HNSW-RaBitQ graph walk (HNSWRaBitQIndex.searchPrepared,
// hnsw_rabitq.go:589-612): the descent through the upper levels
// (searchRaBitQLayer, :644-671, coarse estimates) and the base-layer search
// (searchRaBitQBase, :673-737) over a graph the caller uploaded
// (xvec_gpu_rabitq_set_graph).  One warp per query: the warp computes the
// estimates of a neighbour list 32 at a time (lane j the j-th neighbour's,
// a float64 sum in index order, or in four interleaved parts when the
// query's sums are exact), and lane 0 then
// applies the reference's decisions to the neighbours in list order, with
// the frontier (best first) and the accepted set (worst first) as binary
// heaps in shared memory.  A node is the packed key (order-preserving
// estimate << 32 | key rank), so the heaps' order is raBitQNodeBetter
// (:739-744).  Full estimates are computed ahead for every unvisited
// neighbour (they are pure functions), but a failure counts only where the
// reference computes that estimate.
// ---------------------------------------------------------------------------

struct WalkArgs {
  const uint8_t* codes;
  const RaBitQFactors* factors;
  const float* q_rot;
  const double* q_sum;
  const double* g_add;
  const double* g_error;
  const int* q_exact;
  int padded, nc, total_bits;
  const uint16_t* values;
  int64_t n;
  int max_level;
  int64_t entry;
  const int64_t* offsets;  // [(max_level + 1) (n + 1)]
  const int32_t* nbrs;
  const uint64_t* keys;
  const uint32_t* keyrank;
  const uint32_t* pos_of_kr;
  const uint32_t* bitmap;
  int capacity, top, refine, public_metric;
  float radius;
  int fcap;                 // frontier entries per warp
  uint32_t* visited;        // [slots][words]
  int64_t words;
  int32_t* vlist;           // [slots][vcap]
  int vcap;
  int nq;
  const int* qids;          // the queries to walk (null: 0 .. nq - 1)
  int stride;               // output entries per query
  uint64_t* o_keys;
  float* o_scores;
  int* o_counts;
  uint32_t* o_pos;
  int* q_flags;
};

__device__ int walk_finish(const WalkArgs& a, int qi, int64_t row, bool multi, double dot,
                           float* dist, float* lower);

// EstimateCoarse (full = false) or Estimate (rabitq.go:421-446) of `row`
// for query qi with makeRaBitQEstimate's checks (:464-476): 0, or the
// failure flag.  Every lane gets the result.
__device__ int walk_estimate(const WalkArgs& a, int qi, int64_t row, bool full, float* dist,
                             float* lower) {
  const int lane = threadIdx.x & 31;
  const uint8_t* b = a.codes + row * (a.padded / 8);
  const float* q = a.q_rot + (int64_t)qi * a.padded;
  const bool multi = full && a.total_bits > 1, half = a.total_bits > 8;
  const uint16_t* vrow = multi ? a.values + row * a.padded : nullptr;
  auto term = [&](int i) -> double {
    if (multi) return __dmul_rn(rabitq_value(vrow, i, half), (double)q[i]);
    return (b[i >> 3] & (1u << (i & 7))) ? (double)q[i] : 0.0;
  };
  double dot = 0.0;
  if (a.q_exact[qi]) {
    for (int i = lane; i < a.padded; i += 32) dot = __dadd_rn(dot, term(i));
    for (int o = 16; o > 0; o >>= 1) dot = __dadd_rn(dot, __shfl_xor_sync(kFullMask, dot, o));
  } else {
    if (lane == 0)
      for (int i = 0; i < a.padded; ++i) {
        const double t = term(i);
        if (multi || t != 0.0 || (b[i >> 3] & (1u << (i & 7)))) dot = __dadd_rn(dot, t);
      }
    dot = __shfl_sync(kFullMask, dot, 0);
  }
  return walk_finish(a, qi, row, multi, dot, dist, lower);
}

// One lane's dot of `row` with the query (the other lanes take other rows):
// the float64 sum in index order, or (ANY_ORDER: the query's sums are exact)
// in four interleaved parts.  ANY_ORDER is a template parameter so that the
// four parts stay in registers.
template <bool ANY_ORDER>
__device__ __noinline__ double walk_dot_lane(const WalkArgs& a, const float* q, int64_t row, bool multi,
                                bool half) {
  double acc0 = 0.0, acc1 = 0.0, acc2 = 0.0, acc3 = 0.0;
  auto add = [&](int part, double t) {
    if (!ANY_ORDER || part == 0) acc0 = __dadd_rn(acc0, t);
    else if (part == 1) acc1 = __dadd_rn(acc1, t);
    else if (part == 2) acc2 = __dadd_rn(acc2, t);
    else acc3 = __dadd_rn(acc3, t);
  };
  // The query is read four floats at a time (every lane reads the same
  // address: one broadcast per warp).
  const float4* q4 = reinterpret_cast<const float4*>(q);
  if (multi) {
    const uint16_t* vrow = a.values + row * a.padded;
    for (int i = 0; i < a.padded; i += 8) {
      const uint4 raw = *reinterpret_cast<const uint4*>(vrow + i);
      const float4 qa = __ldg(q4 + (i >> 2)), qb = __ldg(q4 + (i >> 2) + 1);
      const float qv[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
      const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const uint16_t v16 = (uint16_t)(w[j >> 1] >> (16 * (j & 1)));
        const double v = half ? (double)__half2float(__ushort_as_half(v16))
                              : (double)__bfloat162float(__ushort_as_bfloat16(v16));
        add(j & 3, __dmul_rn(v, (double)qv[j]));
      }
    }
  } else {
    const uint2* pairs = reinterpret_cast<const uint2*>(a.codes + row * (a.padded / 8));
    for (int wi = 0; wi < a.padded / 32; ++wi) {
      const uint2 pw = pairs[wi >> 1];
      const uint32_t word = (wi & 1) ? pw.y : pw.x;
#pragma unroll
      for (int g = 0; g < 8; ++g) {
        const float4 v = __ldg(q4 + wi * 8 + g);
        const float qv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          // An unset bit adds +0, which leaves the sum unchanged (it is
          // never -0: it starts at +0).
          add(u, ((word >> (g * 4 + u)) & 1u) ? (double)qv[u] : 0.0);
        }
      }
    }
  }
  return ANY_ORDER ? __dadd_rn(__dadd_rn(acc0, acc1), __dadd_rn(acc2, acc3)) : acc0;
}

// One lane's estimate of `row`: the dot (walk_dot_lane), then walk_finish.
__device__ int walk_estimate_lane(const WalkArgs& a, int qi, int64_t row, bool full, float* dist,
                                  float* lower) {
  const float* q = a.q_rot + (int64_t)qi * a.padded;
  const bool multi = full && a.total_bits > 1, half = a.total_bits > 8;
  // The row's lines are requested up front (each lane reads its own row, so
  // the loads below would otherwise wait on L2 one after another).
  {
    const char* rb = multi ? reinterpret_cast<const char*>(a.values + row * a.padded)
                           : reinterpret_cast<const char*>(a.codes + row * (a.padded / 8));
    const int bytes = multi ? a.padded * 2 : a.padded / 8;
    const uintptr_t first = reinterpret_cast<uintptr_t>(rb) & ~(uintptr_t)127;
    for (uintptr_t l = first; l < reinterpret_cast<uintptr_t>(rb) + bytes; l += 128)
      asm volatile("prefetch.global.L1 [%0];" ::"l"(l));
    asm volatile("prefetch.global.L1 [%0];" ::"l"(a.factors + row));
  }
  const double dot = a.q_exact[qi] ? walk_dot_lane<true>(a, q, row, multi, half)
                                   : walk_dot_lane<false>(a, q, row, multi, half);
  return walk_finish(a, qi, row, multi, dot, dist, lower);
}

// makeRaBitQEstimate's formula and checks (rabitq.go:434-476) given the dot.
__device__ int walk_finish(const WalkArgs& a, int qi, int64_t row, bool multi, double dot,
                           float* dist, float* lower) {
  const RaBitQFactors f = a.factors[row];
  const int64_t gi = (int64_t)qi * a.nc + f.cluster;
  double d, eb;
  if (multi) {
    const double center = -(ldexp(1.0, a.total_bits - 1) - 0.5);
    d = __dadd_rn(__dadd_rn(f.full_add, a.g_add[gi]),
                  __dmul_rn(f.full_rescale, __dadd_rn(dot, __dmul_rn(center, a.q_sum[qi]))));
    eb = __ddiv_rn(__dmul_rn(f.error, a.g_error[gi]), ldexp(1.0, a.total_bits - 1));
  } else {
    const double centered = __dsub_rn(dot, __dmul_rn(0.5, a.q_sum[qi]));
    d = __dadd_rn(__dadd_rn(f.add, a.g_add[gi]), __dmul_rn(f.rescale, centered));
    eb = __dmul_rn(f.error, a.g_error[gi]);
  }
  constexpr double kMaxF = 3.40282346638528859811704183484516925440e+38;
  if (isnan(d) || isinf(d) || isnan(eb) || isinf(eb) || eb < 0) return kRaBitQInvalid;
  if (fabs(d) > kMaxF || eb > kMaxF) return kRaBitQOverflow;
  const double lo = __dsub_rn(d, eb), hi = __dadd_rn(d, eb);
  if (lo < -kMaxF || hi > kMaxF) return kRaBitQOverflow;
  *dist = __double2float_rn(d);
  *lower = __double2float_rn(lo);
  return 0;
}

__device__ __forceinline__ uint64_t walk_key(float score, uint32_t kr) {
  return ((uint64_t)float_to_ordered(score) << 32) | kr;
}

// Binary heaps of packed keys in shared memory (lane 0 only): MIN = true
// keeps the smallest key on top (the frontier), false the largest (the
// accepted set).
template <bool MIN>
__device__ __forceinline__ bool heap_before(uint64_t a, uint64_t b) {
  return MIN ? a < b : a > b;
}
template <bool MIN>
__device__ void heap_push(uint64_t* h, int& size, uint64_t v) {
  int i = size++;
  while (i > 0) {
    const int p = (i - 1) >> 1;
    if (!heap_before<MIN>(v, h[p])) break;
    h[i] = h[p];
    i = p;
  }
  h[i] = v;
}
template <bool MIN>
__device__ uint64_t heap_pop(uint64_t* h, int& size) {
  const uint64_t top = h[0];
  const uint64_t v = h[--size];
  int i = 0;
  for (;;) {
    const int l = 2 * i + 1;
    if (l >= size) break;
    int c = l;
    if (l + 1 < size && heap_before<MIN>(h[l + 1], h[l])) c = l + 1;
    if (!heap_before<MIN>(h[c], v)) break;
    h[i] = h[c];
    i = c;
  }
  if (size > 0) h[i] = v;
  return top;
}
template <bool MIN>
__device__ void heap_build(uint64_t* h, int size) {
  for (int s = size / 2 - 1; s >= 0; --s) {
    const uint64_t v = h[s];
    int i = s;
    for (;;) {
      const int l = 2 * i + 1;
      if (l >= size) break;
      int c = l;
      if (l + 1 < size && heap_before<MIN>(h[l + 1], h[l])) c = l + 1;
      if (!heap_before<MIN>(h[c], v)) break;
      h[i] = h[c];
      i = c;
    }
    h[i] = v;
  }
}

// Sorts a[0, m) ascending with the warp (bitonic over the next power of two,
// padded with all-ones keys; a has room for it).
__device__ void warp_sort_keys(uint64_t* a, int m) {
  const int lane = threadIdx.x & 31;
  int p = 1;
  while (p < m) p <<= 1;
  for (int i = m + lane; i < p; i += 32) a[i] = kEmptyKey;
  __syncwarp();
  for (int k = 2; k <= p; k <<= 1)
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = lane; i < p; i += 32) {
        const int x = i ^ j;
        if (x > i) {
          const uint64_t u = a[i], w = a[x];
          const bool up = (i & k) == 0;
          if ((u > w) == up) {
            a[i] = w;
            a[x] = u;
          }
        }
      }
      __syncwarp();
    }
}

constexpr int kWalkStage = 96;  // uint64 slots per warp for the staged neighbour values

__global__ void __launch_bounds__(256) hnsw_rabitq_walk_kernel(WalkArgs a) {
  extern __shared__ __align__(16) unsigned char walk_smem[];
  const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5, wpb = blockDim.x >> 5;
  // Per warp: frontier [fcap], accepted [pow2 >= capacity].
  int acap2 = 1;
  while (acap2 < a.capacity + 1) acap2 <<= 1;
  uint64_t* frontier =
      reinterpret_cast<uint64_t*>(walk_smem) + (size_t)wib * (a.fcap + acap2 + kWalkStage);
  uint64_t* accepted = frontier + a.fcap;
  // A neighbour list's values for lane 0's decisions (lane j's in slot j).
  uint32_t* st_kr = reinterpret_cast<uint32_t*>(accepted + acap2);
  float* st_l = reinterpret_cast<float*>(st_kr + 32);
  float* st_f = st_l + 32;
  int* st_c1 = reinterpret_cast<int*>(st_f + 32);
  int* st_c2 = st_c1 + 32;
  int* st_acc = st_c2 + 32;
  const int slot = blockIdx.x * wpb + wib, slots = gridDim.x * wpb;
  uint32_t* vis = a.visited + (int64_t)slot * a.words;
  int32_t* vl = a.vlist + (int64_t)slot * a.vcap;
  for (int t = slot; t < a.nq; t += slots) {
    const int qi = a.qids ? a.qids[t] : t;
    int fail = 0;
    int nvis = 0;  // visited nodes recorded (lane 0's count is the truth)
    // Marks node p visited; true when it was not yet (every lane calls it
    // with its own p or -1).
    auto mark = [&](int64_t p) -> bool {
      bool fresh = false;
      if (p >= 0) {
        const uint32_t bit = 1u << (p & 31);
        fresh = !(atomicOr(&vis[p >> 5], bit) & bit);
      }
      const unsigned m = __ballot_sync(kFullMask, fresh);
      if (fresh) {
        const int at = nvis + __popc(m & ((1u << lane) - 1));
        if (at < a.vcap) vl[at] = (int32_t)p;
      }
      nvis += __popc(m);
      return fresh;
    };
    // ---- upper levels: greedy descent on coarse estimates ----
    int64_t cur = a.entry;
    float cur_d = 0.f, lo = 0.f;
    for (int level = a.max_level; level > 0 && !fail; --level) {
      fail = walk_estimate(a, qi, cur, false, &cur_d, &lo);
      bool changed = !fail;
      while (changed && !fail) {
        changed = false;
        const int64_t* off = a.offsets + (int64_t)level * (a.n + 1);
        const int64_t first = off[cur], last = off[cur + 1];
        for (int64_t e0 = first; e0 < last && !fail; e0 += 32) {
          const int cnt = (int)min((int64_t)32, last - e0);
          const int64_t nb = lane < cnt ? (int64_t)a.nbrs[e0 + lane] : -1;
          float nd = 0.f, nl = 0.f;
          int nst = 0;
          if (lane < cnt) nst = walk_estimate_lane(a, qi, nb, false, &nd, &nl);
          __syncwarp();
          for (int j = 0; j < cnt; ++j) {
            const int64_t p = __shfl_sync(kFullMask, nb, j);
            const float dj = __shfl_sync(kFullMask, nd, j);
            const int sj = __shfl_sync(kFullMask, nst, j);
            if (sj) {
              fail = sj;
              break;
            }
            if (dj < cur_d || (dj == cur_d && p < cur)) {
              cur = p;
              cur_d = dj;
              changed = true;
            }
          }
        }
      }
    }
    // ---- base layer ----
    int fsize = 0, asize = 0;
    auto accept = [&](int64_t p, float score) {
      if (!bitmap_pass(a.bitmap, p)) return false;
      if (a.refine) return true;
      const float pub = a.public_metric == kMetricIP ? __fsub_rn(1.f, score) : score;
      return within_radius(a.public_metric, pub, a.radius);
    };
    if (!fail) {
      float sd, sl;
      fail = walk_estimate(a, qi, cur, true, &sd, &sl);
      mark(cur);
      if (!fail && lane == 0) {
        const uint64_t s = walk_key(sd, a.keyrank[cur]);
        heap_push<true>(frontier, fsize, s);
        if (accept(cur, sd)) heap_push<false>(accepted, asize, s);
      }
    }
    fsize = __shfl_sync(kFullMask, fsize, 0);
    asize = __shfl_sync(kFullMask, asize, 0);
    __syncwarp();
    while (fsize > 0 && !fail) {
      uint64_t c = 0;
      if (lane == 0) c = heap_pop<true>(frontier, fsize);
      c = __shfl_sync(kFullMask, c, 0);
      fsize = __shfl_sync(kFullMask, fsize, 0);
      const uint64_t worst0 = __shfl_sync(kFullMask, asize > 0 ? accepted[0] : 0ull, 0);
      if (asize >= a.capacity && asize > 0 && worst0 < c) break;
      const int64_t cpos = a.pos_of_kr[(uint32_t)c];
      const int64_t first = a.offsets[cpos], last = a.offsets[cpos + 1];
      for (int64_t e0 = first; e0 < last && !fail; e0 += 32) {
        const int cnt = (int)min((int64_t)32, last - e0);
        int64_t nb = lane < cnt ? (int64_t)a.nbrs[e0 + lane] : -1;
        // A node listed twice is taken at its first place (the reference's
        // later occurrence finds it visited).
        const unsigned same = __match_any_sync(kFullMask, nb);
        if (nb >= 0 && lane != __ffs(same) - 1) nb = -2;  // a repeat within the chunk
        const bool fresh = mark(nb >= 0 ? nb : -1);
        float cd = 0.f, cl = 0.f, fd = 0.f;
        int cst = 0, fst = 0;
        const unsigned fm = __ballot_sync(kFullMask, fresh);
        // Each unvisited neighbour's estimates by its own lane.
        if (fresh) {
          cst = walk_estimate_lane(a, qi, nb, false, &cd, &cl);
          if (a.total_bits > 1) {
            float unused;
            fst = walk_estimate_lane(a, qi, nb, true, &fd, &unused);
          } else {
            fd = cd;
          }
        }
        __syncwarp();
        // The reference's decisions, in list order, by lane 0 (which holds
        // the heaps) from the values each lane staged for its neighbour.
        if (fresh) {
          st_kr[lane] = a.keyrank[nb];
          st_l[lane] = cl;
          st_f[lane] = fd;
          st_c1[lane] = cst;
          st_c2[lane] = fst;
          st_acc[lane] = accept(nb, fd) ? 1 : 0;
        }
        __syncwarp();
        int lfail = 0;
        if (lane == 0) {
          for (unsigned m = fm; m; m &= m - 1) {
            const int j = __ffs(m) - 1;
            if (st_c1[j]) {
              lfail = st_c1[j];
              break;
            }
            const bool full_set = asize >= a.capacity && asize > 0;
            if (full_set && st_l[j] >= rank_of(accepted[0])) continue;  // pruned
            if (st_c2[j]) {
              lfail = st_c2[j];
              break;
            }
            const uint64_t v = walk_key(st_f[j], st_kr[j]);
            if (asize < a.capacity || asize == 0 || v < accepted[0]) {
              if (fsize == a.fcap && asize >= a.capacity && asize > 0) {
                // Frontier entries worse than the worst accepted node only
                // end the walk when popped: drop them.
                int keep = 0;
                for (int i = 0; i < fsize; ++i)
                  if (frontier[i] < accepted[0]) frontier[keep++] = frontier[i];
                fsize = keep;
                heap_build<true>(frontier, fsize);
              }
              if (fsize == a.fcap) {
                lfail = kRaBitQGraphFull;
                break;
              }
              heap_push<true>(frontier, fsize, v);
              if (st_acc[j]) {
                heap_push<false>(accepted, asize, v);
                if (asize > a.capacity) heap_pop<false>(accepted, asize);
              }
            }
          }
        }
        fail = __shfl_sync(kFullMask, lfail, 0);
        fsize = __shfl_sync(kFullMask, fsize, 0);
        asize = __shfl_sync(kFullMask, asize, 0);
        __syncwarp();
      }
    }
    // ---- results: the accepted nodes best first, the first `top` of them ----
    __syncwarp();
    int count = 0;
    if (!fail) {
      warp_sort_keys(accepted, asize);
      count = min(asize, a.top);
      for (int i = lane; i < count; i += 32) {
        const uint64_t v = accepted[i];
        const uint32_t pos = a.pos_of_kr[(uint32_t)v];
        const float est = rank_of(v);
        a.o_keys[(int64_t)qi * a.stride + i] = a.keys[pos];
        a.o_scores[(int64_t)qi * a.stride + i] =
            (!a.refine && a.public_metric == kMetricIP) ? __fsub_rn(1.f, est) : est;
        if (a.o_pos) a.o_pos[(int64_t)qi * a.stride + i] = pos;
      }
    }
    if (lane == 0) {
      a.o_counts[qi] = count;
      if (fail) atomicOr(&a.q_flags[qi], fail);
    }
    // Clear this query's visited marks (the whole bitmap when the record
    // overflowed).
    __syncwarp();
    if (nvis <= a.vcap) {
      for (int i = lane; i < nvis; i += 32) {
        const int32_t p = vl[i];
        atomicAnd(&vis[p >> 5], ~(1u << (p & 31)));
      }
    } else {
      for (int64_t w = lane; w < a.words; w += 32) vis[w] = 0u;
    }
    __syncwarp();
  }
}

__global__ void clear_flag_bits_kernel(const int* ids, int n, int bit, int* q_flags) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) q_flags[ids[i]] &= ~bit;
}

// Launches the walk for nq queries: the approximate stage's `top` nodes
// (refine: the candidate count cc, else k) per query into o_* (stride cc).
xvec_gpu_status rabitq_graph_walk(xvec_gpu_index* idx, int nq, int k, int ef, int cc,
                                  bool refine, float radius, const uint32_t* d_bitmap,
                                  const RaBitQScorer& sc, uint64_t* o_keys, float* o_scores,
                                  int* o_counts, uint32_t* o_pos, int* q_flags, cudaStream_t s) {
  const int64_t n = idx->n;
  const int top = refine ? cc : k;
  const int capacity = std::max(ef, top);
  int acap2 = 1;
  while (acap2 < capacity + 1) acap2 <<= 1;
  int sms = 148;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, idx->device);
  const int64_t words = (n + 31) / 32;
  const int vcap = 65536;
  WalkArgs a{};
  a.codes = sc.codes;
  a.factors = sc.factors;
  a.q_rot = sc.q_rot;
  a.q_sum = sc.q_sum;
  a.g_add = sc.g_add;
  a.g_error = sc.g_error;
  a.q_exact = sc.q_exact;
  a.padded = sc.padded;
  a.nc = sc.nc;
  a.total_bits = sc.total_bits;
  a.values = sc.values;
  a.n = n;
  a.max_level = idx->hnsw_max_level;
  a.entry = idx->hnsw_entry;
  a.offsets = idx->hnsw_offsets.as<int64_t>();
  a.nbrs = idx->hnsw_nbrs.as<int32_t>();
  a.keys = idx->keys.as<uint64_t>();
  a.keyrank = idx->keyrank.as<uint32_t>();
  a.pos_of_kr = idx->pos_of_kr.as<uint32_t>();
  a.bitmap = d_bitmap;
  a.capacity = capacity;
  a.top = top;
  a.refine = refine ? 1 : 0;
  a.public_metric = idx->desc.metric;
  a.radius = radius;
  a.vcap = vcap;
  a.stride = cc;
  a.o_keys = o_keys;
  a.o_scores = o_scores;
  a.o_counts = o_counts;
  a.o_pos = o_pos;
  a.q_flags = q_flags;
  // One launch over `count` queries (qids: their ids, or null for all) with
  // `warps` warps per block and a frontier of fcap entries per warp; the
  // blocks fill the SMs (several per SM when the frontier is small).
  auto launch = [&](int count, const int* qids, int warps, int fcap) -> xvec_gpu_status {
    const size_t smem = (size_t)warps * (fcap + acap2 + kWalkStage) * 8;
    XVEC_CUDA(cudaFuncSetAttribute(hnsw_rabitq_walk_kernel,
                                   cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    int per_sm = 0;
    XVEC_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, hnsw_rabitq_walk_kernel,
                                                            warps * 32, smem));
    int64_t slots = std::min<int64_t>((int64_t)sms * std::max(1, per_sm) * warps,
                                      ((int64_t)count + warps - 1) / warps * warps);
    // The per-warp visited bitmaps stay within 2 GB.
    while (slots > warps && slots * words * 4 > (2ll << 30)) slots -= warps;
    Scratch vis, vlist;
    xvec_gpu_status st;
    if ((st = vis.alloc((size_t)slots * words * 4, s)) ||
        (st = vlist.alloc((size_t)slots * vcap * 4, s)))
      return st;
    XVEC_CUDA(cudaMemsetAsync(vis.ptr, 0, (size_t)slots * words * 4, s));
    a.fcap = fcap;
    a.visited = vis.as<uint32_t>();
    a.words = words;
    a.vlist = vlist.as<int32_t>();
    a.nq = count;
    a.qids = qids;
    hnsw_rabitq_walk_kernel<<<(unsigned)(slots / warps), warps * 32, smem, s>>>(a);
    XVEC_LAUNCHED();
    XVEC_CUDA(cudaGetLastError());
    return XVEC_GPU_OK;
  };
  // The large frontier: 200 KB of shared memory per SM.
  const int big_warps = capacity <= 256 ? 8 : capacity <= 1024 ? 4 : 2;
  const int big_fcap = (200 * 1024 / 8) / big_warps - acap2 - kWalkStage;
  if (big_fcap < 2 * capacity)
    return set_error("HNSW-RaBitQ walk: capacity %d is beyond the supported maximum", capacity),
           XVEC_GPU_INVALID_ARGUMENT;
  // First a frontier of max(1024, 4 capacity) entries, so that several
  // blocks share an SM; the queries whose frontier outgrew it walk again with
  // the large one (a walk's result does not depend on the buffer it used).
  const int small_fcap = std::max(1024, 4 * capacity);
  int small_warps = 8;
  while (small_warps > 1 &&
         (size_t)small_warps * (small_fcap + acap2 + kWalkStage) * 8 > 75 * 1024)
    small_warps >>= 1;
  const bool small_fits =
      (size_t)small_warps * (small_fcap + acap2 + kWalkStage) * 8 <= 75 * 1024;
  if (!small_fits || small_fcap >= big_fcap || nq == 0)
    return launch(nq, nullptr, big_warps, big_fcap);
  xvec_gpu_status st = launch(nq, nullptr, small_warps, small_fcap);
  if (st) return st;
  std::vector<int> flags(nq);
  XVEC_CUDA(cudaMemcpyAsync(flags.data(), q_flags, (size_t)nq * 4, cudaMemcpyDeviceToHost, s));
  XVEC_CUDA(cudaStreamSynchronize(s));
  std::vector<int> again;
  for (int q = 0; q < nq; ++q)
    if (flags[q] & kRaBitQGraphFull) again.push_back(q);
  if (again.empty()) return XVEC_GPU_OK;
  Scratch dq;
  if ((st = dq.alloc(again.size() * 4, s))) return st;
  XVEC_CUDA(cudaMemcpyAsync(dq.ptr, again.data(), again.size() * 4, cudaMemcpyHostToDevice, s));
  clear_flag_bits_kernel<<<(unsigned)((again.size() + 255) / 256), 256, 0, s>>>(
      dq.as<int>(), (int)again.size(), kRaBitQGraphFull, q_flags);
  XVEC_LAUNCHED();
  st = launch((int)again.size(), dq.as<int>(), big_warps, big_fcap);
  if (st) return st;
  XVEC_CUDA(cudaStreamSynchronize(s));
  return XVEC_GPU_OK;
}

// Per-query status: PrepareQuery's, then the scan's, then the refine's.
__global__ void rabitq_status_kernel(const int* q_status, const int* q_flags,
                                     const int* refine_status, int nq, int* out_counts) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= nq) return;
  const int st = rabitq_query_status(q_status[i], q_flags[i], refine_status ? refine_status[i] : 0);
  if (st != 0) out_counts[i] = -st;
}
__global__ void rabitq_clear_flags(const int* ids, int n, int* q_flags) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) q_flags[ids[i]] &= ~3;
}

// Small batches: a scan of the sign bits (n x padded/8 bytes) instead of
// the tensor-core operand planes (16 x larger).  One block of 32 warps per
// (row part, query), one part per SM.  The block's query is a byte table in
// shared memory: entry (b, pos) = the float32 sum of q[8 pos + i] over the
// set bits i of b, stored at column (pos mod 4) * 32 + pos / 4 of row b (128
// columns, zero past padded/8).  Steps of 512 rows are staged in shared
// memory (coalesced 8-byte loads held in registers while the block scores
// the previous step, rows padded with zeros to 128 bytes); two lanes score a
// row, each over 16 of its 32 code words read in a rotated order, so the
// code reads (bank w) and the four table reads of a word (column j * 32 + w,
// bank w) of the 32 lanes all hit different banks.  A row's dot is a float32 sum of at most `padded` terms (within the
// FFMA term of q_eps); ranks use the RaBitQRanker formula; keys below the
// block's threshold go to one block list, compacted to the KP best by a
// block sort when full.  The parts' lists are then reduced to one list per
// query (reduce_lists_kernel) for the merge.
constexpr int kLutThreads = 1024;
constexpr int kLutRows = 512;       // rows per step (two threads per row)
constexpr int kLutCap = 2048;       // block list entries (kp + one step's appends)
constexpr int kLutMaxBytes = 128;   // padded / 8 (padded <= 1024)

__global__ void __launch_bounds__(kLutThreads, 1) rabitq_lut_scan_kernel(
    const uint8_t* __restrict__ codes, int64_t n, int padded, const float4* __restrict__ fast,
    const uint32_t* __restrict__ keyrank, const uint32_t* __restrict__ bitmap,
    const float* __restrict__ q_rot, const float* __restrict__ q_fast_sum,
    const float* __restrict__ q_fast_gadd, int nc, int64_t rows_per_part, int kp,
    uint64_t* __restrict__ part_keys, int* __restrict__ part_counts,
    uint64_t* __restrict__ part_sat, int* __restrict__ q_flags) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  float* lut = reinterpret_cast<float*>(smem_raw);                          // [256][128]
  uint32_t* stage = reinterpret_cast<uint32_t*>(lut + 256 * kLutMaxBytes);  // [512][32]
  uint64_t* list = reinterpret_cast<uint64_t*>(stage + kLutRows * 32);      // [kLutCap]
  float* gadd = reinterpret_cast<float*>(list + kLutCap);                   // [nc]
  __shared__ int s_count, s_bad;
  __shared__ unsigned long long s_thr;
  const int part = blockIdx.x, q = blockIdx.y, parts = gridDim.x;
  const int tid = threadIdx.x, lane = tid & 31;
  const int bytes = padded / 8, words8 = bytes / 8;  // 8-byte words per row
  const float* qr = q_rot + (int64_t)q * padded;
  // Table: thread pos < 128 fills column col(pos) for every byte value b,
  // entry b = entry (b without its highest set bit) + that bit's value.
  if (tid < kLutMaxBytes) {
    const int pos = tid, col = (pos & 3) * 32 + (pos >> 2);
    float v[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = pos < bytes ? qr[pos * 8 + i] : 0.f;
    // Entry 2^i + j is entry j plus bit i's value (i unrolled, so v stays in
    // registers).
    lut[col] = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i)
      for (int j = 0; j < (1 << i); ++j)
        lut[((1 << i) + j) * kLutMaxBytes + col] = lut[j * kLutMaxBytes + col] + v[i];
  }
  // Zero padding of the staged rows (bytes past padded/8, never overwritten).
  for (int i = tid; i < kLutRows * 32; i += kLutThreads)
    if ((i & 31) >= bytes / 4) stage[i] = 0u;
  for (int c = tid; c < nc; c += kLutThreads) gadd[c] = q_fast_gadd[(int64_t)q * nc + c];
  if (tid == 0) {
    s_count = 0;
    s_bad = 0;
    s_thr = kEmptyKey;
  }
  const float half_sum = 0.5f * q_fast_sum[q];
  const int64_t begin = (int64_t)part * rows_per_part;
  const int64_t end = min(n, begin + rows_per_part);
  const int steps = end > begin ? (int)((end - begin + kLutRows - 1) / kLutRows) : 0;
  // Step i's rows [begin + 512 i, ...) as 8-byte words: thread t takes words
  // t, t + 1024, ... of the step's contiguous bytes.
  const int per_step = kLutRows * words8;
  constexpr int kMaxLoads = kLutRows * (kLutMaxBytes / 8) / kLutThreads;  // per thread
  uint2 pre[kMaxLoads];
  auto load_step = [&](int i) {
    const int64_t r0 = begin + (int64_t)i * kLutRows;
    const int64_t words_avail = (min(end, r0 + kLutRows) - r0) * words8;
    const uint2* src = reinterpret_cast<const uint2*>(codes + r0 * bytes);
#pragma unroll
    for (int k = 0; k < kMaxLoads; ++k) {
      const int u = tid + k * kLutThreads;
      pre[k] = (u < per_step && u < words_avail) ? __ldg(src + u) : make_uint2(0u, 0u);
    }
  };
  // Row of word u: u / words8 through a float reciprocal (u < 2^13, so
  // (u + 0.5) / words8 is at least 1/32 away from an integer and the product
  // rounds to the right side).
  const float inv_words8 = 1.0f / (float)words8;
  auto store_step = [&]() {
#pragma unroll
    for (int k = 0; k < kMaxLoads; ++k) {
      const int u = tid + k * kLutThreads;
      if (u < per_step) {
        const int r = (int)(((float)u + 0.5f) * inv_words8), w = u - r * words8;
        *reinterpret_cast<uint2*>(stage + r * 32 + w * 2) = pre[k];
      }
    }
  };
  // Warp w scores rows 16 w .. 16 w + 15 of a step: lane l takes row
  // 16 w + (l mod 16) and its words 16 (l / 16) .. 16 (l / 16) + 15; the two
  // halves are added by a shuffle and the lower half ranks the row.
  const int row_local = (tid >> 5) * 16 + (lane & 15), half = lane >> 4;
  // The row terms of this thread's row in a step, loaded a step ahead.
  float4 nf = make_float4(0.f, 0.f, 0.f, 0.f);
  uint32_t nkr = 0;
  bool nok = false;
  auto load_terms = [&](int i) {
    const int64_t row = begin + (int64_t)i * kLutRows + row_local;
    nok = half == 0 && row < end && bitmap_pass(bitmap, row);
    if (nok) {
      nf = fast[row];
      nkr = keyrank[row];
    }
  };
  if (steps > 0) {
    load_step(0);
    load_terms(0);
    store_step();
  }
  __syncthreads();
  bool saturated = false;
  for (int i = 0; i < steps; ++i) {
    const bool ok = nok;
    const float4 f = nf;
    const uint32_t kr = nkr;
    // The next step's codes and row terms stay in flight (in registers)
    // while this step is scored from the stage.
    if (i + 1 < steps) {
      load_step(i + 1);
      load_terms(i + 1);
    }
    const uint32_t* mine = stage + row_local * 32 + half * 16;
    const float* lut_h = lut + half * 16;
    float acc0 = 0.f, acc1 = 0.f, acc2 = 0.f, acc3 = 0.f;
    // Byte j of word w selects row (byte) of column j * 32 + w: the float
    // offset byte * 128 is the byte shifted into bits 7..14.  The words of a
    // half are read in the order (g + l) mod 16, so the 32 lanes' code and
    // table reads hit 32 different banks.
#pragma unroll 8
    for (int g = 0; g < 16; ++g) {
      const uint32_t w = (uint32_t)(g + lane) & 15u;
      const uint32_t word = mine[w];
      const float* col = lut_h + w;
      acc0 += col[(word << 7) & 0x7f80u];
      acc1 += col[((word >> 1) & 0x7f80u) + 32];
      acc2 += col[((word >> 9) & 0x7f80u) + 64];
      acc3 += col[((word >> 17) & 0x7f80u) + 96];
    }
    float dot = (acc0 + acc1) + (acc2 + acc3);
    dot += __shfl_xor_sync(kFullMask, dot, 16);
    if (ok) {
      const float rank = fmaf(f.y, dot - half_sum, f.x + gadd[__float_as_int(f.z)]);
      if (!finite_f(rank)) {
        s_bad = 1;
      } else {
        const uint64_t key = pack_rank(rank, kr);
        if (key < *(volatile unsigned long long*)&s_thr) {
          const int slot = atomicAdd(&s_count, 1);
          list[slot] = key;
        }
      }
    }
    __syncthreads();  // the stage is read and the appends are in
    if (i + 1 < steps) store_step();
    // Room for the next step's appends: compact to the KP best.
    if (s_count > kLutCap - kLutRows) {
      const int cnt = s_count;
      block_sort_u64<kLutCap>(list, cnt);
      __syncthreads();
      if (tid == 0) {
        if (cnt > kp) saturated = true;
        s_thr = list[kp - 1];
        s_count = kp;
      }
    }
    __syncthreads();
  }
  __syncthreads();
  const int cnt = s_count;
  block_sort_u64_fit<kLutCap>(list, cnt);
  __syncthreads();
  const int out = min(cnt, kp);
  const int64_t slot = (int64_t)q * parts + part;
  for (int i = tid; i < out; i += kLutThreads) part_keys[slot * kp + i] = list[i];
  if (tid == 0) {
    part_counts[slot] = out;
    // Every dropped key is at or above the KP-th kept one.
    part_sat[slot] = (saturated || cnt > kp || s_thr != kEmptyKey) && cnt >= kp ? list[kp - 1]
                                                                               : kEmptyKey;
    if (s_bad) atomicOr(&q_flags[q], 1);
  }
}

int floor_pow2(int v) {
  int r = 1;
  while (r <= v / 2) r *= 2;
  return r;
}
float inv_sqrt_size(int truncated) {
  return 1.0f / (float)std::sqrt((double)(float)truncated);
}

// Entries kept per (query, part): the candidate count plus a margin for the
// eps band, a multiple of 32 (the accumulators take any such size).
int rabitq_kp(int cc) { return (cc + std::max(8, cc / 4) + 31) / 32 * 32; }

}  // namespace

// ---------------------------------------------------------------------------
// Index hooks.
// ---------------------------------------------------------------------------
xvec_gpu_status rabitq_reserve(xvec_gpu_index* idx, int64_t cap, cudaStream_t s) {
  const int64_t n = idx->n;
  const int bytes = idx->padded / 8;
  xvec_gpu_status st;
  // One bit: the int8 code planes [127 b | b]; multi-bit: the 16-bit code
  // values; both 2 padded bytes per row.
  DeviceBuffer& plane = idx->rq_total_bits > 1 ? idx->rq_values : idx->rq_planes;
  if ((st = idx->rq_codes.reserve((size_t)cap * bytes, (size_t)n * bytes, s)) ||
      (st = idx->rq_factors.reserve((size_t)cap * sizeof(RaBitQFactors),
                                    (size_t)n * sizeof(RaBitQFactors), s)) ||
      (st = idx->rq_fast.reserve((size_t)cap * 16, (size_t)n * 16, s)) ||
      (st = plane.reserve((size_t)cap * idx->padded * 2, (size_t)n * idx->padded * 2, s)))
    return st;
  if (idx->rq_total_bits > 1 && idx->rq_total_bits <= 8 &&
      (st = idx->rq_vplane.reserve((size_t)cap * idx->padded, (size_t)n * idx->padded, s)))
    return st;
  if (!idx->rq_bounds.ptr) {
    if ((st = idx->rq_bounds.reserve(16, 0, s))) return st;
    XVEC_CUDA(cudaMemsetAsync(idx->rq_bounds.ptr, 0, 16, s));
  }
  return XVEC_GPU_OK;
}

xvec_gpu_status rabitq_commit(xvec_gpu_index* idx, int64_t old_n, int64_t m, cudaStream_t s) {
  const int d = idx->desc.dimension, padded = idx->padded, metric = idx->desc.metric;
  const int truncated = floor_pow2(d);
  const float inv = inv_sqrt_size(truncated);
  xvec_gpu_status st;
  Scratch prepared, labels, err, bounds;
  if ((st = prepared.alloc((size_t)m * d * 4, s)) || (st = labels.alloc((size_t)m * 4, s)) ||
      (st = err.alloc(4, s)) || (st = bounds.alloc(16, s)))
    return st;
  XVEC_CUDA(cudaMemsetAsync(err.ptr, 0, 4, s));
  XVEC_CUDA(cudaMemcpyAsync(bounds.ptr, idx->rq_bounds.ptr, 16, cudaMemcpyDeviceToDevice, s));
  rabitq_prepare_kernel<<<(unsigned)m, 256, d * 4, s>>>(idx->rows.as<float>() + old_n * d, m, d,
                                                       metric == XVEC_METRIC_COSINE,
                                                       prepared.as<float>());
  XVEC_LAUNCHED();
  // Nearest centroid (L2, or IP for IP and cosine), ties to the lower index.
  extern xvec_gpu_status rabitq_assign(xvec_gpu_index*, const float*, int64_t, int32_t*,
                                       cudaStream_t);
  if ((st = rabitq_assign(idx, prepared.as<float>(), m, labels.as<int32_t>(), s))) return st;
  rabitq_encode_kernel<<<(unsigned)m, 256, padded * 4, s>>>(
      prepared.as<float>(), m, d, padded, truncated, idx->rq_signs.as<uint8_t>(), inv,
      idx->rq_rot_centroids.as<float>(), labels.as<int32_t>(), metric != XVEC_METRIC_L2,
      idx->rq_total_bits, idx->rq_extra_scale, idx->rq_codes.as<uint8_t>() + old_n * (padded / 8),
      idx->rq_total_bits > 1 ? idx->rq_values.as<uint16_t>() + old_n * padded : nullptr,
      idx->rq_factors.as<RaBitQFactors>() + old_n, idx->rq_fast.as<float4>() + old_n,
      bounds.as<unsigned>(), err.as<int>());
  XVEC_LAUNCHED();
  XVEC_CUDA(cudaGetLastError());
  int h = 0;
  XVEC_CUDA(cudaMemcpyAsync(&h, err.ptr, 4, cudaMemcpyDeviceToHost, s));
  XVEC_CUDA(cudaStreamSynchronize(s));
  if (h) return set_error("core: invalid RaBitQ code (status %d)", h), (xvec_gpu_status)h;
  if (idx->rq_total_bits > 1 && idx->rq_total_bits <= 8) {
    rabitq_vplane_kernel<<<blocks_of(m * 32), 256, 0, s>>>(
        idx->rq_values.as<uint16_t>() + old_n * padded, m, padded,
        idx->rq_vplane.as<int8_t>() + old_n * padded, idx->rq_fast.as<float4>() + old_n);
    XVEC_LAUNCHED();
    XVEC_CUDA(cudaGetLastError());
  }
  if (idx->rq_total_bits == 1) {
  const int64_t code_bytes = m * (padded / 8);
  rabitq_planes_kernel<<<blocks_of(code_bytes), 256, 0, s>>>(
      idx->rq_codes.as<uint8_t>() + old_n * (padded / 8), code_bytes, padded,
      idx->rq_planes.as<int8_t>() + old_n * 2 * padded);
  XVEC_LAUNCHED();
  XVEC_CUDA(cudaGetLastError());
  }
  XVEC_CUDA(cudaMemcpyAsync(idx->rq_bounds.ptr, bounds.ptr, 16, cudaMemcpyDeviceToDevice, s));
  return XVEC_GPU_OK;
}

xvec_gpu_status rabitq_assign(xvec_gpu_index* idx, const float* prepared, int64_t m,
                              int32_t* labels, cudaStream_t s) {
  xvec_gpu_search_opts o{};
  o.top_k = 1;
  Scratch keys, scores, counts;
  xvec_gpu_status st;
  const int64_t batch = std::min<int64_t>(m, 65536);
  if ((st = keys.alloc((size_t)batch * 8, s)) || (st = scores.alloc((size_t)batch * 4, s)) ||
      (st = counts.alloc((size_t)batch * 4, s)))
    return st;
  const int d = idx->desc.dimension;
  for (int64_t b = 0; b < m; b += batch) {
    const int cnt = (int)std::min<int64_t>(batch, m - b);
    std::vector<int> statuses;
    NestedSearch nested;
    st = search_device_locked(idx->probe_index, prepared + b * d, cnt, o, nullptr,
                              keys.as<uint64_t>(), scores.as<float>(), counts.as<int>(), s,
                              &statuses);
    if (st) return st;
    std::vector<uint64_t> hk(cnt);
    XVEC_CUDA(cudaMemcpyAsync(hk.data(), keys.ptr, (size_t)cnt * 8, cudaMemcpyDeviceToHost, s));
    XVEC_CUDA(cudaStreamSynchronize(s));
    std::vector<int32_t> hl(cnt);
    for (int i = 0; i < cnt; ++i) {
      if (statuses[i]) return set_error("assign row: status %d", statuses[i]), (xvec_gpu_status)statuses[i];
      hl[i] = (int32_t)hk[i];
    }
    XVEC_CUDA(cudaMemcpyAsync(labels + b, hl.data(), (size_t)cnt * 4, cudaMemcpyHostToDevice, s));
    XVEC_CUDA(cudaStreamSynchronize(s));
  }
  return XVEC_GPU_OK;
}

int rabitq_candidate_count(const xvec_gpu_search_opts& o) {
  return o.refine ? std::max(o.top_k, o.ef) : 0;
}

xvec_gpu_status rabitq_search_impl(xvec_gpu_index* idx, const float* d_q, int nq,
                                   const xvec_gpu_search_opts& o, const uint32_t* d_bitmap,
                                   uint64_t* d_keys, float* d_scores, int* d_counts,
                                   cudaStream_t s, std::vector<int>* statuses,
                                   bool candidates_only) {
  EventTimer timer(s);
  timer.mark(0);
  // hnsw_rabitq.go:548-550, 573-579.
  if (o.ef <= 0 || o.ef > 2048)
    return set_error("core: invalid HNSW ef %d (want 1..2048)", o.ef), XVEC_GPU_INVALID_ARGUMENT;
  if (!idx->has_model) return set_error("RaBitQ index has no model"), XVEC_GPU_INVALID_ARGUMENT;
  const int d = idx->desc.dimension, padded = idx->padded, metric = idx->desc.metric;
  const int nc = idx->rq_clusters;
  const int64_t n = idx->n;
  const int k = o.top_k;
  const bool refine = o.refine != 0;
  if (candidates_only && !refine)
    return set_error("candidates of a search without refinement"), XVEC_GPU_INVALID_ARGUMENT;
  const int cc = refine ? (int)std::min<int64_t>(std::max<int64_t>(n, 1), std::max(k, o.ef)) : k;
  const int kp = rabitq_kp(cc);
  if (exact_cap_for(kp) > 8192)
    return set_error("top_k %d exceeds the supported maximum for RaBitQ", k),
           XVEC_GPU_INVALID_ARGUMENT;
  const int truncated = floor_pow2(d);
  const float inv = inv_sqrt_size(truncated);
  xvec_gpu_status st;
  const int total_bits = idx->rq_total_bits;
  const bool multi = total_bits > 1;
  Scratch qrot, qsum, gadd, gerr, qfs, qfg, qeps, qexact, qstatus, qflags, qint, qterms, q8;
  // Multi-bit with TotalBits <= 8: the INT8 tensor-core scan on the int8
  // code plane and the 16-bit integer query (its eps is that form's).
  const bool want8 = multi && total_bits <= 8 && idx->rq_vplane.ptr != nullptr;
  if ((st = qint.alloc((size_t)nq * padded * 2, s)) || (st = qterms.alloc((size_t)nq * 8, s)) ||
      (want8 && (st = q8.alloc((size_t)nq * padded * 2, s))))
    return st;
  const int64_t n_all = idx->n;
  const bool small_batch = !multi && n_all > 0 && nq <= 8 && padded <= 8 * kLutMaxBytes &&
                           kp <= 256 && nc <= 4096;
  const bool graph_walk = idx->hnsw_max_level >= 0 && !o.linear && n_all > kHNSWBruteForce;
  if (graph_walk && idx->hnsw_n != n_all)
    return set_error("the HNSW graph covers %lld rows, the index holds %lld: set the graph "
                     "again after adding rows",
                     (long long)idx->hnsw_n, (long long)n_all),
           XVEC_GPU_INVALID_ARGUMENT;
  const bool tc8 = !graph_walk && want8 && !small_batch && n_all > 0 &&
                   nc <= rabitq_tc_max_clusters() &&
                   kp + 128 <= flat_tc_cap() && n_all < (1ll << 31) - 256 &&
                   rabitq8_tc_supported(padded, idx->rq_vplane.ptr, q8.ptr);
  if ((st = qrot.alloc((size_t)nq * padded * 4, s)) || (st = qsum.alloc((size_t)nq * 8, s)) ||
      (st = gadd.alloc((size_t)nq * nc * 8, s)) || (st = gerr.alloc((size_t)nq * nc * 8, s)) ||
      (st = qfs.alloc((size_t)nq * 4, s)) || (st = qfg.alloc((size_t)nq * nc * 4, s)) ||
      (st = qeps.alloc((size_t)nq * 4, s)) || (st = qexact.alloc((size_t)nq * 4, s)) ||
      (st = qstatus.alloc((size_t)nq * 4, s)) || (st = qflags.alloc((size_t)nq * 4, s)))
    return st;
  XVEC_CUDA(cudaMemsetAsync(qflags.ptr, 0, (size_t)nq * 4, s));
  rabitq_prep_query_kernel<<<nq, 256, padded * 4, s>>>(
      d_q, nq, d, padded, truncated, idx->rq_signs.as<uint8_t>(), inv,
      metric == XVEC_METRIC_COSINE, metric, idx->rq_rot_centroids.as<float>(), nc,
      idx->rq_bounds.as<unsigned>(), qrot.as<float>(), qsum.as<double>(), gadd.as<double>(),
      gerr.as<double>(), qfs.as<float>(), qfg.as<float>(), qeps.as<float>(), qexact.as<int>(),
      qstatus.as<int>(), qflags.as<int>(), qint.as<int8_t>(), qterms.as<float2>(), total_bits,
      tc8 ? q8.as<int8_t>() : nullptr);
  XVEC_LAUNCHED();
  // The approximate stage writes the final results, or the candidates of the
  // refine stage (no radius there: hnsw_rabitq.go:584).
  Scratch skeys, sscores, scounts, spos;
  if ((st = skeys.alloc((size_t)nq * cc * 8, s)) || (st = sscores.alloc((size_t)nq * cc * 4, s)) ||
      (st = scounts.alloc((size_t)nq * 4, s)) || (st = spos.alloc((size_t)nq * cc * 4, s)))
    return st;
  uint64_t* o_keys = refine ? skeys.as<uint64_t>() : d_keys;
  float* o_scores = refine ? sscores.as<float>() : d_scores;
  int* o_counts = refine ? scounts.as<int>() : d_counts;
  XVEC_CUDA(cudaMemsetAsync(o_counts, 0, (size_t)nq * 4, s));
  // The candidates-only form reports the estimates themselves (ranks).
  const RaBitQScorer sc{kMetricL2, candidates_only ? kMetricL2 : metric,
                        idx->rq_codes.as<uint8_t>(),
                        idx->rq_factors.as<RaBitQFactors>(), qrot.as<float>(),
                        qsum.as<double>(), gadd.as<double>(), gerr.as<double>(),
                        qeps.as<float>(), qexact.as<int>(), padded, nc, total_bits,
                        multi ? idx->rq_values.as<uint16_t>() : nullptr};
  const float stage_radius = refine ? 0.f : o.radius;
  // Small batches: the sign bits through a byte table (the tensor-core scan
  // streams 16x more bytes and fills few SMs at this size).
  // An uploaded graph: the HNSW-RaBitQ walk unless the caller asks for the
  // linear scan or the index is small (searchPrepared, hnsw_rabitq.go:589-591).
  const bool walk = graph_walk;
  const bool small = !walk && small_batch;
  // INT8 tensor cores on the code planes (one bit) or on the int8 code-value
  // plane (up to 8 bits), when the layout allows, else FFMA.
  const bool use_tc = !walk && !small && n > 0 && nc <= rabitq_tc_max_clusters() &&
                      kp + 128 <= flat_tc_cap() && n < (1ll << 31) - 256 &&
                      (multi ? tc8 : rabitq_tc_supported(padded, idx->rq_planes.ptr, qint.ptr));
  const bool fast = walk || small || use_tc || (n > 0 && simt_cap_for(kp) <= 512);
  if (walk) {
    timer.mark(1);
    if ((st = rabitq_graph_walk(idx, nq, k, o.ef, cc, refine, o.radius, d_bitmap, sc, o_keys,
                                o_scores, o_counts, spos.as<uint32_t>(), qflags.as<int>(), s)))
      return st;
    timer.mark(2);
  } else if (small) {
    // One part per SM (each block keeps its kp best), then one list per
    // query for the merge.
    int sms = 148;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, idx->device);
    int parts = (int)std::max<int64_t>(1, std::min<int64_t>(sms, (n + 4095) / 4096));
    while (parts > 1 && !reduce_lists_supported(parts, kp)) --parts;
    const int64_t rows_per_part = ((n + parts - 1) / parts + kLutRows - 1) / kLutRows * kLutRows;
    parts = (int)((n + rows_per_part - 1) / rows_per_part);
    const int lstride = reduce_lists_out_cap(kp);
    Scratch pkeys, pcounts, psat, lkeys, lcounts, lsat;
    if ((st = pkeys.alloc((size_t)nq * parts * kp * 8, s)) ||
        (st = pcounts.alloc((size_t)nq * parts * 4, s)) ||
        (st = psat.alloc((size_t)nq * parts * 8, s)) ||
        (st = lkeys.alloc((size_t)nq * lstride * 8, s)) ||
        (st = lcounts.alloc((size_t)nq * 4, s)) || (st = lsat.alloc((size_t)nq * 8, s)))
      return st;
    const int smem = kLutMaxBytes * 256 * 4 + kLutRows * 128 + kLutCap * 8 + nc * 4;
    cudaFuncSetAttribute(rabitq_lut_scan_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         smem);
    timer.mark(1);
    rabitq_lut_scan_kernel<<<dim3(parts, nq), kLutThreads, smem, s>>>(
        idx->rq_codes.as<uint8_t>(), n, padded, idx->rq_fast.as<float4>(),
        idx->keyrank.as<uint32_t>(), d_bitmap, qrot.as<float>(), qfs.as<float>(),
        qfg.as<float>(), nc, rows_per_part, kp, pkeys.as<uint64_t>(), pcounts.as<int>(),
        psat.as<uint64_t>(), qflags.as<int>());
    XVEC_LAUNCHED();
    XVEC_CUDA(cudaGetLastError());
    XVEC_CUDA(launch_reduce_lists(pkeys.as<uint64_t>(), pcounts.as<int>(), psat.as<uint64_t>(),
                                  nq, parts, kp, lstride, nullptr, lkeys.as<uint64_t>(),
                                  lcounts.as<int>(), lsat.as<uint64_t>(), s));
    XVEC_LAUNCHED();
    timer.mark(2);
    XVEC_CUDA(launch_merge_rescore(sc, idx->pos_of_kr.as<uint32_t>(), idx->keys.as<uint64_t>(),
                                   nullptr, nq, cc, stage_radius, 0, lkeys.as<uint64_t>(),
                                   lcounts.as<int>(), lsat.as<uint64_t>(), 1, lstride, o_keys,
                                   o_scores, o_counts, spos.as<uint32_t>(), qflags.as<int>(), s));
    XVEC_LAUNCHED();
  } else if (use_tc) {
    Scratch pkeys, pcounts, psat, kstatus, gthr_keep;
    int lists = 0;
    if ((st = kstatus.alloc(4, s))) return st;
    XVEC_CUDA(cudaMemsetAsync(kstatus.ptr, 0, 4, s));
    timer.mark(1);
    st = tc_seeded_scan(
        idx->device, nq, n, kp, s,
        [&](int64_t b, int64_t e, int p, int list0, int nlists, unsigned long long* gthr,
            uint64_t* cand, int* counts, uint64_t* sat) {
          if (multi)
            return launch_rabitq8_scan_tc(
                q8.as<int8_t>(), nq, idx->rq_vplane.as<int8_t>() + b * padded, e - b, padded,
                idx->rq_fast.as<float4>() + b, idx->keyrank.as<uint32_t>() + b,
                qterms.as<float2>(), qfg.as<float>(), nc, gthr,
                d_bitmap ? d_bitmap + b / 32 : nullptr, p, kp, list0, nlists, cand, counts, sat,
                qflags.as<int>(), kstatus.as<int>(), s);
          return launch_rabitq_scan_tc(
              qint.as<int8_t>(), nq, idx->rq_planes.as<int8_t>() + b * 2 * padded, e - b,
              padded, idx->rq_fast.as<float4>() + b, idx->keyrank.as<uint32_t>() + b,
              qterms.as<float2>(), qfg.as<float>(), nc, gthr, d_bitmap ? d_bitmap + b / 32 : nullptr,
              p, kp, list0, nlists, cand, counts, sat, qflags.as<int>(), kstatus.as<int>(), s);
        },
        pkeys, pcounts, psat, &lists, &gthr_keep);
    if (st) return st;
    timer.mark(2);
    XVEC_LAUNCHED();
    count_tensor_scan();
    XVEC_CUDA(launch_merge_rescore(sc, idx->pos_of_kr.as<uint32_t>(), idx->keys.as<uint64_t>(),
                                   nullptr, nq, cc, stage_radius, 0, pkeys.as<uint64_t>(),
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
    const RaBitQRanker<false> rk{idx->rq_fast.as<float4>(), qfs.as<float>(), qfg.as<float>(),
                                 nc, nullptr};
    const RaBitQRanker<true> rkf{idx->rq_fast.as<float4>(), qfs.as<float>(), qfg.as<float>(),
                                 nc, qterms.as<float2>()};
    timer.mark(1);
    if (!multi)
      XVEC_CUDA(launch_scan_simt(reinterpret_cast<const BitElem*>(idx->rq_codes.ptr), n, padded,
                                 idx->keyrank.as<uint32_t>(), qrot.as<float>(), nq, d_bitmap, rk,
                                 parts, kp, pkeys.as<uint64_t>(), pcounts.as<int>(),
                                 psat.as<uint64_t>(), qflags.as<int>(), s));
    else if (total_bits <= 8)
      XVEC_CUDA(launch_scan_simt(reinterpret_cast<const Bf16Value*>(idx->rq_values.ptr), n,
                                 padded, idx->keyrank.as<uint32_t>(), qrot.as<float>(), nq,
                                 d_bitmap, rkf, parts, kp, pkeys.as<uint64_t>(), pcounts.as<int>(),
                                 psat.as<uint64_t>(), qflags.as<int>(), s));
    else
      XVEC_CUDA(launch_scan_simt(reinterpret_cast<const HalfValue*>(idx->rq_values.ptr), n,
                                 padded, idx->keyrank.as<uint32_t>(), qrot.as<float>(), nq,
                                 d_bitmap, rkf, parts, kp, pkeys.as<uint64_t>(), pcounts.as<int>(),
                                 psat.as<uint64_t>(), qflags.as<int>(), s));
    timer.mark(2);
    XVEC_CUDA(launch_merge_rescore(sc, idx->pos_of_kr.as<uint32_t>(), idx->keys.as<uint64_t>(),
                                   nullptr, nq, cc, stage_radius, 0, pkeys.as<uint64_t>(),
                                   pcounts.as<int>(), psat.as<uint64_t>(), parts, kp, o_keys,
                                   o_scores, o_counts, spos.as<uint32_t>(), qflags.as<int>(), s));
    count_launches(2);
  }
  std::vector<int> h_status(nq), h_flags(nq);
  XVEC_CUDA(cudaMemcpyAsync(h_status.data(), qstatus.ptr, (size_t)nq * 4, cudaMemcpyDeviceToHost, s));
  XVEC_CUDA(cudaMemcpyAsync(h_flags.data(), qflags.ptr, (size_t)nq * 4, cudaMemcpyDeviceToHost, s));
  XVEC_CUDA(cudaStreamSynchronize(s));
  // Exact pass: queries the fast pass could not settle, every query when the
  // candidate count is beyond the fast accumulators, and queries whose
  // estimates may fail (scanRaBitQCodes stops at the first failing row,
  // filtered or not, so those are first scored over every row).
  std::vector<int> exact_list, check_list;
  if (n > 0)
    for (int q = 0; q < nq; ++q) {
      if (h_status[q] != 0) continue;
      if (!fast || (h_flags[q] & 3)) exact_list.push_back(q);
      // (The graph walk meets failing estimates where the reference does.)
      if ((h_flags[q] & kRaBitQFullCheck) && d_bitmap && !walk) check_list.push_back(q);
    }
  auto exact_pass = [&](const std::vector<int>& list, const uint32_t* bitmap,
                        bool write) -> xvec_gpu_status {
    const int nl = (int)list.size();
    int parts = (int)std::max<int64_t>(1, std::min<int64_t>((592 + nl - 1) / nl, (n + 1023) / 1024));
    parts = std::min(parts, std::max(1, flat_merge_capacity() / kp));
    Scratch ids, pkeys, pcounts, psat, dk, ds, dc, dp;
    xvec_gpu_status e;
    if ((e = ids.alloc((size_t)nl * 4, s)) || (e = pkeys.alloc((size_t)nl * parts * kp * 8, s)) ||
        (e = pcounts.alloc((size_t)nl * parts * 4, s)) ||
        (e = psat.alloc((size_t)nl * parts * 8, s)))
      return e;
    XVEC_CUDA(cudaMemcpyAsync(ids.ptr, list.data(), (size_t)nl * 4, cudaMemcpyHostToDevice, s));
    rabitq_clear_flags<<<blocks_of(nl), 256, 0, s>>>(ids.as<int>(), nl, qflags.as<int>());
    XVEC_CUDA(launch_scan_exact(sc, n, idx->keyrank.as<uint32_t>(), ids.as<int>(), nl, bitmap,
                                parts, kp, pkeys.as<uint64_t>(), pcounts.as<int>(),
                                psat.as<uint64_t>(), qflags.as<int>(), s));
    count_launches(2);
    if (!write) return XVEC_GPU_OK;
    XVEC_CUDA(launch_merge_rescore(sc, idx->pos_of_kr.as<uint32_t>(), idx->keys.as<uint64_t>(),
                                   ids.as<int>(), nl, cc, stage_radius, 1, pkeys.as<uint64_t>(),
                                   pcounts.as<int>(), psat.as<uint64_t>(), parts, kp, o_keys,
                                   o_scores, o_counts, spos.as<uint32_t>(), qflags.as<int>(), s));
    XVEC_LAUNCHED();
    XVEC_CUDA(cudaMemcpyAsync(h_flags.data(), qflags.ptr, (size_t)nq * 4, cudaMemcpyDeviceToHost, s));
    XVEC_CUDA(cudaStreamSynchronize(s));
    for (int q : list)
      if (h_flags[q] & 2)
        return set_error("exact scan could not complete query %d", q), XVEC_GPU_CUDA_ERROR;
    return XVEC_GPU_OK;
  };
  if (!check_list.empty() && (st = exact_pass(check_list, nullptr, false))) return st;
  if (!exact_list.empty() && (st = exact_pass(exact_list, d_bitmap, true))) return st;

  Scratch rstatus;
  if (candidates_only) {
    // The approximate stage's candidates, at stride max(top_k, ef).
    const int stride = rabitq_candidate_count(o);
    rabitq_status_kernel<<<blocks_of(nq), 256, 0, s>>>(qstatus.as<int>(), qflags.as<int>(),
                                                       nullptr, nq, o_counts);
    XVEC_LAUNCHED();
    XVEC_CUDA(cudaMemcpy2DAsync(d_keys, (size_t)stride * 8, o_keys, (size_t)cc * 8,
                                (size_t)cc * 8, nq, cudaMemcpyDeviceToDevice, s));
    XVEC_CUDA(cudaMemcpy2DAsync(d_scores, (size_t)stride * 4, o_scores, (size_t)cc * 4,
                                (size_t)cc * 4, nq, cudaMemcpyDeviceToDevice, s));
    XVEC_CUDA(cudaMemcpyAsync(d_counts, o_counts, (size_t)nq * 4, cudaMemcpyDeviceToDevice, s));
  } else if (refine) {
    // refinePrepared (hnsw_rabitq.go:780-801) -> topKCandidatesWithOptions:
    // metric.Compute(q, q) on the raw query first (topk.go:92-94).
    Scratch qf, qn2, qaux;
    if ((st = rstatus.alloc((size_t)nq * 4, s)) || (st = qf.alloc((size_t)nq * d * 4, s)) ||
        (st = qn2.alloc((size_t)nq * 4, s)) || (st = qaux.alloc((size_t)nq * 4, s)))
      return st;
    launch_prep_queries<float>(d_q, nq, d, metric, qf.as<float>(), qn2.as<float>(),
                               qaux.as<float>(), rstatus.as<int>(), s);
    XVEC_LAUNCHED();
    rabitq_status_kernel<<<blocks_of(nq), 256, 0, s>>>(qstatus.as<int>(), qflags.as<int>(),
                                                       rstatus.as<int>(), nq, o_counts);
    XVEC_CUDA(cudaMemsetAsync(d_counts, 0, (size_t)nq * 4, s));
    if (n > 0) {
      XVEC_CUDA(launch_refine(idx->rows.as<float>(), d, metric, d_q, nq, spos.as<uint32_t>(),
                              o_counts, cc, idx->keyrank.as<uint32_t>(),
                              idx->pos_of_kr.as<uint32_t>(), idx->keys.as<uint64_t>(), k,
                              o.radius, d_keys, d_scores, d_counts, qflags.as<int>(), s));
      count_launches(2);
    }
  }
  const int* rs = (refine && !candidates_only && n > 0) ? rstatus.as<int>() : nullptr;
  rabitq_status_kernel<<<blocks_of(nq), 256, 0, s>>>(qstatus.as<int>(), qflags.as<int>(), rs, nq,
                                                     d_counts);
  XVEC_LAUNCHED();
  XVEC_CUDA(cudaGetLastError());
  std::vector<int> h_rs(nq, 0);
  XVEC_CUDA(cudaMemcpyAsync(h_flags.data(), qflags.ptr, (size_t)nq * 4, cudaMemcpyDeviceToHost, s));
  if (rs) XVEC_CUDA(cudaMemcpyAsync(h_rs.data(), rs, (size_t)nq * 4, cudaMemcpyDeviceToHost, s));
  timer.mark(3);
  XVEC_CUDA(cudaStreamSynchronize(s));
  count_search(nq, (int64_t)exact_list.size(), timer.ms(1, 2), timer.ms(0, 3));
  if (statuses) {
    statuses->resize(nq);
    for (int q = 0; q < nq; ++q) (*statuses)[q] = rabitq_query_status(h_status[q], h_flags[q], h_rs[q]);
  }
  return XVEC_GPU_OK;
}

}  // namespace xvec

using namespace xvec;

extern "C" xvec_gpu_status xvec_gpu_rabitq_set_graph(xvec_gpu_index* idx, int32_t max_level,
                                                     int64_t entry, const int64_t* offsets,
                                                     const int32_t* neighbors,
                                                     int64_t total_neighbors) {
  if (!idx) return set_error("nil index"), XVEC_GPU_INVALID_ARGUMENT;
  if (idx->desc.kind != XVEC_INDEX_RABITQ)
    return set_error("a graph belongs to a RaBitQ index"), XVEC_GPU_INVALID_ARGUMENT;
  std::unique_lock<std::shared_mutex> lock(idx->mu);
  if (max_level < 0) {
    idx->hnsw_max_level = -1;
    idx->hnsw_n = 0;
    return XVEC_GPU_OK;
  }
  const int64_t n = idx->n;
  if (max_level > 64) return set_error("graph level %d out of range", max_level), XVEC_GPU_INVALID_ARGUMENT;
  if (n <= 0 || entry < 0 || entry >= n)
    return set_error("graph entry %lld outside the index's %lld rows", (long long)entry,
                     (long long)n),
           XVEC_GPU_INVALID_ARGUMENT;
  if (!offsets || total_neighbors < 0 || (total_neighbors > 0 && !neighbors))
    return set_error("nil graph arrays"), XVEC_GPU_INVALID_ARGUMENT;
  const int64_t levels = (int64_t)max_level + 1;
  for (int64_t l = 0; l < levels; ++l) {
    const int64_t* off = offsets + l * (n + 1);
    if (off[0] < 0 || off[n] > total_neighbors)
      return set_error("graph level %lld: offsets outside the neighbour array", (long long)l),
             XVEC_GPU_INVALID_ARGUMENT;
    for (int64_t p = 0; p < n; ++p)
      if (off[p + 1] < off[p])
        return set_error("graph level %lld: offsets decrease at node %lld", (long long)l,
                         (long long)p),
               XVEC_GPU_INVALID_ARGUMENT;
  }
  for (int64_t e = 0; e < total_neighbors; ++e)
    if (neighbors[e] < 0 || neighbors[e] >= n)
      return set_error("graph neighbour %lld: position %d outside the index", (long long)e,
                       neighbors[e]),
             XVEC_GPU_INVALID_ARGUMENT;
  XVEC_CUDA(cudaSetDevice(idx->device));
  cudaStream_t s = nullptr;
  xvec_gpu_status st;
  const size_t obytes = (size_t)levels * (n + 1) * 8, nbytes = (size_t)total_neighbors * 4;
  if ((st = idx->hnsw_offsets.reserve(obytes, 0, s)) ||
      (st = idx->hnsw_nbrs.reserve(std::max<size_t>(nbytes, 4), 0, s)))
    return st;
  XVEC_CUDA(cudaMemcpy(idx->hnsw_offsets.ptr, offsets, obytes, cudaMemcpyHostToDevice));
  if (nbytes) XVEC_CUDA(cudaMemcpy(idx->hnsw_nbrs.ptr, neighbors, nbytes, cudaMemcpyHostToDevice));
  idx->hnsw_max_level = max_level;
  idx->hnsw_entry = entry;
  idx->hnsw_n = n;
  return XVEC_GPU_OK;
}

extern "C" xvec_gpu_status xvec_gpu_rabitq_set_model(xvec_gpu_index* idx, const float* centroids,
                                                     int32_t nclusters,
                                                     const uint8_t* rotation_signs) {
  return xvec_gpu_rabitq_set_model_bits(idx, centroids, nclusters, rotation_signs, 1, 0.0);
}

extern "C" xvec_gpu_status xvec_gpu_rabitq_set_model_bits(xvec_gpu_index* idx,
                                                          const float* centroids,
                                                          int32_t nclusters,
                                                          const uint8_t* rotation_signs,
                                                          int32_t total_bits,
                                                          double extra_scale) {
  if (!idx || !centroids || !rotation_signs) return set_error("nil argument"), XVEC_GPU_INVALID_ARGUMENT;
  if (idx->desc.kind != XVEC_INDEX_RABITQ) return set_error("not a RaBitQ index"), XVEC_GPU_INVALID_ARGUMENT;
  // RestoreRaBitQModel (rabitq.go:196-211).
  if (total_bits < 1 || total_bits > 9)
    return set_error("core: invalid RaBitQ model: TotalBits must be in [1,9]"),
           XVEC_GPU_INVALID_ARGUMENT;
  if (nclusters <= 0) return set_error("core: invalid RaBitQ model: no centroids"), XVEC_GPU_INVALID_ARGUMENT;
  if (total_bits == 1 && extra_scale != 0)
    return set_error("core: invalid RaBitQ model: one-bit model must have zero ExtraScale"),
           XVEC_GPU_INVALID_ARGUMENT;
  if (total_bits > 1 && !(extra_scale > 0 && std::isfinite(extra_scale)))
    return set_error("core: invalid RaBitQ model: ExtraScale must be finite and positive"),
           XVEC_GPU_INVALID_ARGUMENT;
  const int d = idx->desc.dimension, padded = idx->padded;
  std::unique_lock<std::shared_mutex> lock(idx->mu);
  if (idx->n > 0) return set_error("set the model before adding rows"), XVEC_GPU_INVALID_ARGUMENT;
  for (int64_t i = 0; i < (int64_t)nclusters * d; ++i)
    if (!std::isfinite(centroids[i])) return set_error("non-finite centroid"), XVEC_GPU_NON_FINITE;
  cudaSetDevice(idx->device);
  cudaStream_t s = nullptr;
  xvec_gpu_status st;
  const size_t sign_bytes = (size_t)4 * padded / 8;
  if ((st = idx->rq_centroids.reserve((size_t)nclusters * d * 4, 0, s)) ||
      (st = idx->rq_rot_centroids.reserve((size_t)nclusters * padded * 4, 0, s)) ||
      (st = idx->rq_signs.reserve(sign_bytes, 0, s)))
    return st;
  // The bound maxima start at zero: a search of an empty index reads them.
  if (!idx->rq_bounds.ptr) {
    if ((st = idx->rq_bounds.reserve(16, 0, s))) return st;
    XVEC_CUDA(cudaMemset(idx->rq_bounds.ptr, 0, 16));
  }
  XVEC_CUDA(cudaMemcpy(idx->rq_centroids.ptr, centroids, (size_t)nclusters * d * 4,
                       cudaMemcpyHostToDevice));
  XVEC_CUDA(cudaMemcpy(idx->rq_signs.ptr, rotation_signs, sign_bytes, cudaMemcpyHostToDevice));
  Scratch err;
  if ((st = err.alloc(4, s))) return st;
  XVEC_CUDA(cudaMemsetAsync(err.ptr, 0, 4, s));
  const int truncated = floor_pow2(d);
  rabitq_rotate_centroids_kernel<<<nclusters, 256, padded * 4, s>>>(
      idx->rq_centroids.as<float>(), d, padded, truncated, idx->rq_signs.as<uint8_t>(),
      inv_sqrt_size(truncated), idx->rq_rot_centroids.as<float>(), err.as<int>());
  XVEC_CUDA(cudaGetLastError());
  int h = 0;
  XVEC_CUDA(cudaMemcpy(&h, err.ptr, 4, cudaMemcpyDeviceToHost));
  if (h) return set_error("core: invalid RaBitQ model: rotated centroid is not finite"), XVEC_GPU_NON_FINITE;
  // Nearest-centroid index: L2 for L2, IP for IP and cosine (rabitq.go:309-313).
  if (idx->probe_index) {
    xvec_gpu_index_destroy(idx->probe_index);
    idx->probe_index = nullptr;
  }
  xvec_gpu_index_desc desc{};
  desc.kind = XVEC_INDEX_FLAT;
  desc.dimension = d;
  desc.metric = idx->desc.metric == XVEC_METRIC_L2 ? XVEC_METRIC_L2 : XVEC_METRIC_IP;
  desc.storage = XVEC_STORAGE_FP32;
  desc.device = idx->device;
  if ((st = xvec_gpu_index_create(&desc, &idx->probe_index))) return st;
  std::vector<uint64_t> ids(nclusters);
  for (int i = 0; i < nclusters; ++i) ids[i] = (uint64_t)i;
  Scratch dk;
  if ((st = dk.alloc((size_t)nclusters * 8, s))) return st;
  XVEC_CUDA(cudaMemcpy(dk.ptr, ids.data(), (size_t)nclusters * 8, cudaMemcpyHostToDevice));
  if ((st = add_device_locked(idx->probe_index, dk.as<uint64_t>(), idx->rq_centroids.ptr,
                              nclusters, s)))
    return st;
  idx->rq_clusters = nclusters;
  idx->rq_total_bits = total_bits;
  idx->rq_extra_scale = extra_scale;
  idx->has_model = true;
  return XVEC_GPU_OK;
}
