// common.cuh — shared device helpers of the xvec B200 search library.
//
// Two kinds of arithmetic live here:
//   * "fast" arithmetic used to rank candidates (tensor cores or FFMA in any
//     order), always paired with a rigorous error bound (see fast_eps_*);
//   * "reference" arithmetic that reproduces, bit for bit, the float32
//     accumulation order of the reference's distance kernels:
//       internal/floats/floats_amd64.go:59-91 dispatch —
//         d >= 16 : floats_avx512.c (16 lanes, fused lane updates, lanes summed
//                   in order from 0, fused scalar tail),
//         d >= 8  : floats_avx.c   (8 lanes, unfused, unfused tail),
//         d <  8  : floats.go:47-70 (sequential, unfused);
//     and the Go formulas around them (internal/ailego/math/distance.go).
//     Every operation uses an explicit _rn intrinsic so nvcc cannot contract
//     or reorder it.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

namespace xvec {

constexpr int kMetricL2 = 1;
constexpr int kMetricIP = 2;
constexpr int kMetricCosine = 3;
constexpr int kMetricMIPS = 4;

constexpr unsigned kFullMask = 0xffffffffu;

// ---------------------------------------------------------------------------
// Total order on (float rank, uint32 position) packed into one uint64 so a
// plain unsigned sort orders by rank, then position.  Lower rank = better.
// ---------------------------------------------------------------------------
__host__ __device__ __forceinline__ uint32_t float_bits(float f) {
#ifdef __CUDA_ARCH__
  return __float_as_uint(f);
#else
  uint32_t b;
  memcpy(&b, &f, 4);
  return b;
#endif
}
__host__ __device__ __forceinline__ float bits_float(uint32_t b) {
#ifdef __CUDA_ARCH__
  return __uint_as_float(b);
#else
  float f;
  memcpy(&f, &b, 4);
  return f;
#endif
}
__host__ __device__ __forceinline__ uint32_t float_to_ordered(float f) {
  uint32_t b = float_bits(f);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
__host__ __device__ __forceinline__ float ordered_to_float(uint32_t o) {
  uint32_t b = (o & 0x80000000u) ? (o & 0x7fffffffu) : ~o;
  return bits_float(b);
}
__host__ __device__ __forceinline__ uint64_t pack_rank(float r, uint32_t pos) {
  return ((uint64_t)float_to_ordered(r) << 32) | pos;
}
__host__ __device__ __forceinline__ float rank_of(uint64_t key) {
  return ordered_to_float((uint32_t)(key >> 32));
}
__host__ __device__ __forceinline__ uint32_t pos_of(uint64_t key) { return (uint32_t)key; }
constexpr uint64_t kEmptyKey = 0xffffffffffffffffull;

// ---------------------------------------------------------------------------
// Row element loads (float32 rows or binary16 rows decoded exactly).
// ---------------------------------------------------------------------------
__device__ __forceinline__ float load_elem(const float* p, int64_t i) { return p[i]; }
__device__ __forceinline__ float load_elem(const __half* p, int64_t i) { return __half2float(p[i]); }
__device__ __forceinline__ float load_elem(const int8_t* p, int64_t i) { return (float)p[i]; }

// Go's min/max built-ins on floats propagate NaN.
__device__ __forceinline__ float go_minf(float a, float b) {
  if (a != a || b != b) return __int_as_float(0x7fc00000);
  return a < b ? a : b;
}
__device__ __forceinline__ float go_maxf(float a, float b) {
  if (a != a || b != b) return __int_as_float(0x7fc00000);
  return a > b ? a : b;
}
__device__ __forceinline__ double go_mind(double a, double b) {
  if (a != a || b != b) return __longlong_as_double(0x7ff8000000000000ll);
  return a < b ? a : b;
}
__device__ __forceinline__ double go_maxd(double a, double b) {
  if (a != a || b != b) return __longlong_as_double(0x7ff8000000000000ll);
  return a > b ? a : b;
}
__device__ __forceinline__ bool finite_f(float v) { return isfinite(v); }
// Go's min/max on float32 also order the zeros: min(-0, +0) = -0, max = +0.
__device__ __forceinline__ float go_min_zero(float a, float b) {
  return (a < b || (a == b && signbit(a))) ? a : b;
}
__device__ __forceinline__ float go_max_zero(float a, float b) {
  return (a > b || (a == b && !signbit(a))) ? a : b;
}

// ---------------------------------------------------------------------------
// Reference-order accumulation, evaluated by one warp (all 32 lanes call it;
// the result is returned on every lane).
//   MODE 0: sum (x-q)^2                     (xvec_avx512_l2_squared)
//   MODE 1: sum x*q                         (xvec_avx512_inner_product)
//   MODE 2: sum x*q, sum x*x, sum q*q       (xvec_avx512_dot_norms)
// For d >= 16 each half-warp evaluates the row its own lanes pass: the two
// halves may pass two different rows (two candidates per warp) or the same
// one.  Lane j of a half holds the AVX-512 accumulator lane j; its loads are
// issued kRefBatch 16-element blocks at a time so that their latencies
// overlap, and its fused multiply-adds keep the reference's order.
// ---------------------------------------------------------------------------
constexpr int kRefBatch = 8;

template <int MODE, typename RowT>
__device__ __forceinline__ void warp_reference_sums(const RowT* x, const float* q, int d,
                                                    float* s0, float* s1, float* s2) {
  const int lane = threadIdx.x & 31;
  float r0 = 0.f, r1 = 0.f, r2 = 0.f;
  if (d >= 16) {
    const int blocks = d >> 4;
    const int j = lane & 15;
    float a0 = 0.f, a1 = 0.f, a2 = 0.f;
    for (int v0 = 0; v0 < blocks; v0 += kRefBatch) {
      float xv[kRefBatch], qv[kRefBatch];
#pragma unroll
      for (int u = 0; u < kRefBatch; ++u) {
        const bool in = v0 + u < blocks;
        xv[u] = in ? load_elem(x, (int64_t)(v0 + u) * 16 + j) : 0.f;
        qv[u] = in ? q[(int64_t)(v0 + u) * 16 + j] : 0.f;
      }
#pragma unroll
      for (int u = 0; u < kRefBatch; ++u) {
        if (v0 + u >= blocks) break;
        if (MODE == 0) {
          const float df = __fsub_rn(xv[u], qv[u]);
          a0 = __fmaf_rn(df, df, a0);
        } else {
          a0 = __fmaf_rn(xv[u], qv[u], a0);
          if (MODE == 2) {
            a1 = __fmaf_rn(xv[u], xv[u], a1);
            a2 = __fmaf_rn(qv[u], qv[u], a2);
          }
        }
      }
    }
    // reduce512: lanes added in index order to a zero start (within each
    // half-warp).
    for (int t = 0; t < 16; ++t) {
      r0 = __fadd_rn(r0, __shfl_sync(kFullMask, a0, t, 16));
      if (MODE == 2) {
        r1 = __fadd_rn(r1, __shfl_sync(kFullMask, a1, t, 16));
        r2 = __fadd_rn(r2, __shfl_sync(kFullMask, a2, t, 16));
      }
    }
    // Fused scalar tail (the AVX-512 file is compiled with -mfma).
    for (int i = blocks * 16; i < d; ++i) {
      const float xv = load_elem(x, i), qv = q[i];
      if (MODE == 0) {
        const float df = __fsub_rn(xv, qv);
        r0 = __fmaf_rn(df, df, r0);
      } else {
        r0 = __fmaf_rn(xv, qv, r0);
        if (MODE == 2) {
          r1 = __fmaf_rn(xv, xv, r1);
          r2 = __fmaf_rn(qv, qv, r2);
        }
      }
    }
  } else if (d >= 8) {
    // floats_avx.c: one 8-lane block (d < 16), unfused.
    float a0 = 0.f, a1 = 0.f, a2 = 0.f;
    if (lane < 8) {
      const float xv = load_elem(x, lane), qv = q[lane];
      if (MODE == 0) {
        const float df = __fsub_rn(xv, qv);
        a0 = __fadd_rn(0.f, __fmul_rn(df, df));
      } else {
        a0 = __fadd_rn(0.f, __fmul_rn(xv, qv));
        if (MODE == 2) {
          a1 = __fadd_rn(0.f, __fmul_rn(xv, xv));
          a2 = __fadd_rn(0.f, __fmul_rn(qv, qv));
        }
      }
    }
    for (int j = 0; j < 8; ++j) {
      r0 = __fadd_rn(r0, __shfl_sync(kFullMask, a0, j));
      if (MODE == 2) {
        r1 = __fadd_rn(r1, __shfl_sync(kFullMask, a1, j));
        r2 = __fadd_rn(r2, __shfl_sync(kFullMask, a2, j));
      }
    }
    for (int i = 8; i < d; ++i) {
      const float xv = load_elem(x, i), qv = q[i];
      if (MODE == 0) {
        const float df = __fsub_rn(xv, qv);
        r0 = __fadd_rn(r0, __fmul_rn(df, df));
      } else {
        r0 = __fadd_rn(r0, __fmul_rn(xv, qv));
        if (MODE == 2) {
          r1 = __fadd_rn(r1, __fmul_rn(xv, xv));
          r2 = __fadd_rn(r2, __fmul_rn(qv, qv));
        }
      }
    }
  } else {
    // floats.go scalar loops (Go on amd64 does not fuse).
    for (int i = 0; i < d; ++i) {
      const float xv = load_elem(x, i), qv = q[i];
      if (MODE == 0) {
        const float df = __fsub_rn(xv, qv);
        r0 = __fadd_rn(r0, __fmul_rn(df, df));
      } else {
        r0 = __fadd_rn(r0, __fmul_rn(xv, qv));
        if (MODE == 2) {
          r1 = __fadd_rn(r1, __fmul_rn(xv, xv));
          r2 = __fadd_rn(r2, __fmul_rn(qv, qv));
        }
      }
    }
  }
  *s0 = r0;
  *s1 = r1;
  *s2 = r2;
}

// The same reference order evaluated by a single thread (short vectors: PQ
// chunk scores).  MODE 0: sum (x-q)^2, MODE 1: sum x*q.
template <int MODE>
__device__ __forceinline__ float thread_reference_sum(const float* x, const float* q, int d) {
  float r = 0.f;
  if (d >= 16) {
    float lanes[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) lanes[j] = 0.f;
    const int blocks = d >> 4;
    for (int v = 0; v < blocks; ++v) {
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const float xv = x[v * 16 + j], qv = q[v * 16 + j];
        if (MODE == 0) {
          const float df = __fsub_rn(xv, qv);
          lanes[j] = __fmaf_rn(df, df, lanes[j]);
        } else {
          lanes[j] = __fmaf_rn(xv, qv, lanes[j]);
        }
      }
    }
#pragma unroll
    for (int j = 0; j < 16; ++j) r = __fadd_rn(r, lanes[j]);
    for (int i = blocks * 16; i < d; ++i) {
      if (MODE == 0) {
        const float df = __fsub_rn(x[i], q[i]);
        r = __fmaf_rn(df, df, r);
      } else {
        r = __fmaf_rn(x[i], q[i], r);
      }
    }
  } else if (d >= 8) {
    float lanes[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      if (MODE == 0) {
        const float df = __fsub_rn(x[j], q[j]);
        lanes[j] = __fadd_rn(0.f, __fmul_rn(df, df));
      } else {
        lanes[j] = __fadd_rn(0.f, __fmul_rn(x[j], q[j]));
      }
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) r = __fadd_rn(r, lanes[j]);
    for (int i = 8; i < d; ++i) {
      if (MODE == 0) {
        const float df = __fsub_rn(x[i], q[i]);
        r = __fadd_rn(r, __fmul_rn(df, df));
      } else {
        r = __fadd_rn(r, __fmul_rn(x[i], q[i]));
      }
    }
  } else {
    for (int i = 0; i < d; ++i) {
      if (MODE == 0) {
        const float df = __fsub_rn(x[i], q[i]);
        r = __fadd_rn(r, __fmul_rn(df, df));
      } else {
        r = __fadd_rn(r, __fmul_rn(x[i], q[i]));
      }
    }
  }
  return r;
}

// cosineDistance (distance.go:65-81) from DotNorms output.
__device__ __forceinline__ float reference_cosine(float inner, float ln, float rn) {
  if (ln == 0.f && rn == 0.f) return 0.f;
  if (ln == 0.f || rn == 0.f) return 1.f;
  const float lm = __double2float_rn(__dsqrt_rn((double)ln));
  const float rm = __double2float_rn(__dsqrt_rn((double)rn));
  float c = __fdiv_rn(inner, __fmul_rn(lm, rm));
  c = go_minf(1.f, go_maxf(-1.f, c));
  return __fsub_rn(1.f, c);
}

// mipsL2Squared (distance.go:93-100) from DotNorms output.
__device__ __forceinline__ float reference_mips(float inner, float ln, float rn) {
  const float den = go_maxf(ln, rn);
  if (den == 0.f) return 0.f;
  return __fsub_rn(2.f, __fdiv_rn(__fmul_rn(2.f, inner), den));
}

// metric.Compute(row, query) with the reference's rounding; returns the
// score on every lane.  The caller checks finiteness (finiteScore).
template <typename RowT>
__device__ __forceinline__ float warp_reference_score(int metric, const RowT* x, const float* q,
                                                      int d) {
  float s0, s1, s2;
  if (metric == kMetricL2) {
    warp_reference_sums<0>(x, q, d, &s0, &s1, &s2);
    return s0;
  }
  if (metric == kMetricIP) {
    warp_reference_sums<1>(x, q, d, &s0, &s1, &s2);
    return s0;
  }
  warp_reference_sums<2>(x, q, d, &s0, &s1, &s2);
  return metric == kMetricCosine ? reference_cosine(s0, s1, s2) : reference_mips(s0, s1, s2);
}

// Fast rank of a (row, query) pair from its dot product and the exact
// squared norms (see fast_eps for the bound on |fast - reference|).
__device__ __forceinline__ float fast_rank(int metric, float dot, float xn2, float qn2) {
  switch (metric) {
    case kMetricL2: return (xn2 + qn2) - 2.f * dot;
    case kMetricIP: return -dot;
    case kMetricCosine:
      if (xn2 == 0.f && qn2 == 0.f) return 0.f;
      if (xn2 == 0.f || qn2 == 0.f) return 1.f;
      return 1.f - dot * rsqrtf(xn2) * rsqrtf(qn2);
    default: {
      const float den = fmaxf(xn2, qn2);
      if (den == 0.f) return 0.f;
      return 2.f - 2.f * dot / den;
    }
  }
}

// Rank (lower = better) from a metric score: IP ranks by -score.
__device__ __forceinline__ float rank_from_score(int metric, float s) {
  return metric == kMetricIP ? -s : s;
}
__device__ __forceinline__ float score_from_rank(int metric, float r) {
  return metric == kMetricIP ? -r : r;
}

// scoreWithinRadius (query.go:193-201).
__device__ __forceinline__ bool within_radius(int metric, float score, float radius) {
  if (radius == 0.f) return true;
  if (metric == kMetricIP) return score >= radius;
  return score <= radius;
}

__device__ __forceinline__ bool bitmap_pass(const uint32_t* bitmap, int64_t pos) {
  return bitmap == nullptr || ((bitmap[pos >> 5] >> (pos & 31)) & 1u);
}

}  // namespace xvec
