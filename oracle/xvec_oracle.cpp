// xvec_oracle.cpp — CPU restatement of the xvec search hot path.
//
// TEST INFRASTRUCTURE ONLY (the oracle).  It is the checker for the CUDA
// library under xvec_b200/csrc and the CPU baseline for bench.py; no shipped
// code path links or calls it.  Each function names the reference file:line
// (paths relative to the gorse-io/xvec module root) whose behaviour it
// restates, including the float32-vs-float64 accumulation, the operation
// order and the tie rules.
//
// Floating-point contract: this file is compiled with -ffp-contract=off so
// that every fused multiply-add is explicit (fmaf), matching the reference:
//   * Go code (amd64, GOAMD64=v1) never fuses x*y+z;
//   * the AVX-512 kernels fuse their lane updates (_mm512_fmadd_ps) and,
//     being compiled with -mfma, their scalar tails;
//   * the AVX kernels are compiled without -mfma and never fuse.
#include "xvec_oracle.h"

#include <algorithm>
#include <queue>
#include <atomic>
#include <cmath>
#include <cstring>
#include <limits>
#include <thread>
#include <vector>

namespace {

// ---------------------------------------------------------------------------
// internal/floats — three accumulation orders and the amd64 dispatch.
// ---------------------------------------------------------------------------

// floats.go:47-70 (scalar Go loops; no fusion on amd64).
float l2_scalar(const float* a, const float* b, int64_t n) {
  float sum = 0.0f;
  for (int64_t i = 0; i < n; ++i) {
    float diff = a[i] - b[i];
    sum = sum + diff * diff;
  }
  return sum;
}
float ip_scalar(const float* a, const float* b, int64_t n) {
  float sum = 0.0f;
  for (int64_t i = 0; i < n; ++i) sum = sum + a[i] * b[i];
  return sum;
}
void dn_scalar(const float* a, const float* b, int64_t n, float* dot, float* ln, float* rn) {
  float d = 0.0f, l = 0.0f, r = 0.0f;
  for (int64_t i = 0; i < n; ++i) {
    d = d + a[i] * b[i];
    l = l + a[i] * a[i];
    r = r + b[i] * b[i];
  }
  *dot = d;
  *ln = l;
  *rn = r;
}

// Sequential lane reduction: reduce256 / reduce512 (floats_avx.c:18-26,
// floats_avx512.c:19-27) add the stored lanes in index order starting at 0.
template <int L>
float reduce_lanes(const float* lanes) {
  float sum = 0.0f;
  for (int i = 0; i < L; ++i) sum = sum + lanes[i];
  return sum;
}

// floats_avx.c:28-90: 8 lanes, unfused lane update sum + x*y, unfused tail.
float l2_avx(const float* a, const float* b, int64_t n) {
  float lanes[8] = {0};
  int64_t blocks = n / 8;
  for (int64_t v = 0; v < blocks; ++v)
    for (int j = 0; j < 8; ++j) {
      float diff = a[v * 8 + j] - b[v * 8 + j];
      lanes[j] = lanes[j] + diff * diff;
    }
  float result = reduce_lanes<8>(lanes);
  for (int64_t i = blocks * 8; i < n; ++i) {
    float diff = a[i] - b[i];
    result = result + diff * diff;
  }
  return result;
}
float ip_avx(const float* a, const float* b, int64_t n) {
  float lanes[8] = {0};
  int64_t blocks = n / 8;
  for (int64_t v = 0; v < blocks; ++v)
    for (int j = 0; j < 8; ++j) lanes[j] = lanes[j] + a[v * 8 + j] * b[v * 8 + j];
  float result = reduce_lanes<8>(lanes);
  for (int64_t i = blocks * 8; i < n; ++i) result = result + a[i] * b[i];
  return result;
}
void dn_avx(const float* a, const float* b, int64_t n, float* dot, float* ln, float* rn) {
  float dl[8] = {0}, ll[8] = {0}, rl[8] = {0};
  int64_t blocks = n / 8;
  for (int64_t v = 0; v < blocks; ++v)
    for (int j = 0; j < 8; ++j) {
      float x = a[v * 8 + j], y = b[v * 8 + j];
      dl[j] = dl[j] + x * y;
      ll[j] = ll[j] + x * x;
      rl[j] = rl[j] + y * y;
    }
  float d = reduce_lanes<8>(dl), l = reduce_lanes<8>(ll), r = reduce_lanes<8>(rl);
  for (int64_t i = blocks * 8; i < n; ++i) {
    d = d + a[i] * b[i];
    l = l + a[i] * a[i];
    r = r + b[i] * b[i];
  }
  *dot = d;
  *ln = l;
  *rn = r;
}

// floats_avx512.c:29-90: 16 lanes updated with FMA, sequential reduce,
// tail fused (the file is built with -mfma; `result += x*y` contracts).
float l2_avx512(const float* a, const float* b, int64_t n) {
  float lanes[16] = {0};
  int64_t blocks = n / 16;
  for (int64_t v = 0; v < blocks; ++v)
    for (int j = 0; j < 16; ++j) {
      float diff = a[v * 16 + j] - b[v * 16 + j];
      lanes[j] = std::fmaf(diff, diff, lanes[j]);
    }
  float result = reduce_lanes<16>(lanes);
  for (int64_t i = blocks * 16; i < n; ++i) {
    float diff = a[i] - b[i];
    result = std::fmaf(diff, diff, result);
  }
  return result;
}
float ip_avx512(const float* a, const float* b, int64_t n) {
  float lanes[16] = {0};
  int64_t blocks = n / 16;
  for (int64_t v = 0; v < blocks; ++v)
    for (int j = 0; j < 16; ++j) lanes[j] = std::fmaf(a[v * 16 + j], b[v * 16 + j], lanes[j]);
  float result = reduce_lanes<16>(lanes);
  for (int64_t i = blocks * 16; i < n; ++i) result = std::fmaf(a[i], b[i], result);
  return result;
}
void dn_avx512(const float* a, const float* b, int64_t n, float* dot, float* ln, float* rn) {
  float dl[16] = {0}, ll[16] = {0}, rl[16] = {0};
  int64_t blocks = n / 16;
  for (int64_t v = 0; v < blocks; ++v)
    for (int j = 0; j < 16; ++j) {
      float x = a[v * 16 + j], y = b[v * 16 + j];
      dl[j] = std::fmaf(x, y, dl[j]);
      ll[j] = std::fmaf(x, x, ll[j]);
      rl[j] = std::fmaf(y, y, rl[j]);
    }
  float d = reduce_lanes<16>(dl), l = reduce_lanes<16>(ll), r = reduce_lanes<16>(rl);
  for (int64_t i = blocks * 16; i < n; ++i) {
    d = std::fmaf(a[i], b[i], d);
    l = std::fmaf(a[i], a[i], l);
    r = std::fmaf(b[i], b[i], r);
  }
  *dot = d;
  *ln = l;
  *rn = r;
}

// Optional: the reference's own compiled kernels (oracle/_ref), installed by
// xo_use_reference_kernels; they produce the same bits as the restatement
// above (tests/test_oracle_golden.py checks it) and are what the CPU
// baseline times.
typedef void (*binary_kernel)(float*, float*, int64_t, float*);
typedef void (*products_kernel)(float*, float*, int64_t, float*, float*, float*);
binary_kernel g_ref_l2_512 = nullptr, g_ref_ip_512 = nullptr, g_ref_l2_256 = nullptr,
              g_ref_ip_256 = nullptr;
products_kernel g_ref_dn_512 = nullptr, g_ref_dn_256 = nullptr;

}  // namespace

extern "C" void xo_use_reference_kernels(void* l2_512, void* ip_512, void* dn_512, void* l2_256,
                                         void* ip_256, void* dn_256) {
  g_ref_l2_512 = (binary_kernel)l2_512;
  g_ref_ip_512 = (binary_kernel)ip_512;
  g_ref_dn_512 = (products_kernel)dn_512;
  g_ref_l2_256 = (binary_kernel)l2_256;
  g_ref_ip_256 = (binary_kernel)ip_256;
  g_ref_dn_256 = (products_kernel)dn_256;
}

// floats_amd64.go:27-91 on an AVX-512F+FMA host: >=16 → AVX-512 kernel,
// >=8 → AVX kernel, otherwise the scalar Go loop.
extern "C" float xo_l2_squared(const float* a, const float* b, int64_t n) {
  float r;
  if (n >= 16) {
    if (g_ref_l2_512) return g_ref_l2_512((float*)a, (float*)b, n, &r), r;
    return l2_avx512(a, b, n);
  }
  if (n >= 8) {
    if (g_ref_l2_256) return g_ref_l2_256((float*)a, (float*)b, n, &r), r;
    return l2_avx(a, b, n);
  }
  return l2_scalar(a, b, n);
}
extern "C" float xo_inner_product(const float* a, const float* b, int64_t n) {
  float r;
  if (n >= 16) {
    if (g_ref_ip_512) return g_ref_ip_512((float*)a, (float*)b, n, &r), r;
    return ip_avx512(a, b, n);
  }
  if (n >= 8) {
    if (g_ref_ip_256) return g_ref_ip_256((float*)a, (float*)b, n, &r), r;
    return ip_avx(a, b, n);
  }
  return ip_scalar(a, b, n);
}
extern "C" void xo_dot_norms(const float* a, const float* b, int64_t n, float* dot, float* ln,
                             float* rn) {
  if (n >= 16) {
    if (g_ref_dn_512) return g_ref_dn_512((float*)a, (float*)b, n, dot, ln, rn);
    return dn_avx512(a, b, n, dot, ln, rn);
  }
  if (n >= 8) {
    if (g_ref_dn_256) return g_ref_dn_256((float*)a, (float*)b, n, dot, ln, rn);
    return dn_avx(a, b, n, dot, ln, rn);
  }
  return dn_scalar(a, b, n, dot, ln, rn);
}

namespace {

// ---------------------------------------------------------------------------
// internal/ailego/math/distance.go + metric.go
// ---------------------------------------------------------------------------

inline bool finite32(float v) { return std::isfinite(v); }  // distance.go:167-176

// finiteScore (distance.go:178-184).
inline int finite_score(double value, float* out) {
  float s = (float)value;
  if (std::isnan(value) || std::isinf(value) || !finite32(s)) return XO_NON_FINITE;
  *out = s;
  return XO_OK;
}

// Go's built-in min/max on floats propagate NaN.
inline float go_min(float a, float b) {
  if (std::isnan(a) || std::isnan(b)) return std::numeric_limits<float>::quiet_NaN();
  return a < b ? a : b;
}
inline float go_max(float a, float b) {
  if (std::isnan(a) || std::isnan(b)) return std::numeric_limits<float>::quiet_NaN();
  return a > b ? a : b;
}
inline double go_maxd(double a, double b) {
  if (std::isnan(a) || std::isnan(b)) return std::numeric_limits<double>::quiet_NaN();
  return a > b ? a : b;
}
inline double go_mind(double a, double b) {
  if (std::isnan(a) || std::isnan(b)) return std::numeric_limits<double>::quiet_NaN();
  return a < b ? a : b;
}

// cosineDistance (distance.go:65-81).
float cosine_distance(const float* a, const float* b, int64_t n) {
  float inner, ln, rn;
  xo_dot_norms(a, b, n, &inner, &ln, &rn);
  if (ln == 0 && rn == 0) return 0;
  if (ln == 0 || rn == 0) return 1;
  float lm = (float)std::sqrt((double)ln);
  float rm = (float)std::sqrt((double)rn);
  float c = inner / (lm * rm);
  c = go_min(1.0f, go_max(-1.0f, c));
  return 1.0f - c;
}

// mipsL2Squared (distance.go:93-100).
float mips_l2(const float* a, const float* b, int64_t n) {
  float inner, ln, rn;
  xo_dot_norms(a, b, n, &inner, &ln, &rn);
  float den = go_max(ln, rn);
  if (den == 0) return 0;
  float t = 2.0f * inner;
  t = t / den;
  return 2.0f - t;
}

// Metric.PrevalidatedDistance (metric.go:52-65): score without validation.
inline int prevalidated(int metric, const float* a, const float* b, int64_t n, float* out) {
  switch (metric) {
    case XO_L2: return finite_score((double)xo_l2_squared(a, b, n), out);
    case XO_IP: return finite_score((double)xo_inner_product(a, b, n), out);
    case XO_COSINE: return finite_score((double)cosine_distance(a, b, n), out);
    case XO_MIPSL2: return finite_score((double)mips_l2(a, b, n), out);
    default: return XO_INVALID_ARGUMENT;
  }
}

// Metric.Better (metric.go:68-73).
inline bool better(int metric, float a, float b) { return metric == XO_IP ? a > b : a < b; }

// scoreWithinRadius (query.go:193-201).
inline bool within_radius(int metric, float score, float radius) {
  if (radius == 0) return true;
  if (metric == XO_IP) return score >= radius;
  return score <= radius;
}

struct Result {
  uint64_t key;
  float score;
};

// resultBetter (topk.go:271-276).
inline bool result_better(int metric, const Result& l, const Result& r) {
  if (l.score == r.score) return l.key < r.key;
  return better(metric, l.score, r.score);
}

// container.Heap (internal/ailego/container/heap.go) with the worst-first
// comparator of topk.go:117-122: the root is the worst retained result.
struct WorstFirstHeap {
  int metric;
  std::vector<Result> v;
  bool less(const Result& a, const Result& b) const {  // "a is worse than b"
    if (a.score == b.score) return a.key > b.key;
    return better(metric, b.score, a.score);
  }
  void push(const Result& r) {  // heap.go:45-49, siftUp heap.go:94-103
    v.push_back(r);
    size_t i = v.size() - 1;
    while (i > 0) {
      size_t p = (i - 1) / 2;
      if (!less(v[i], v[p])) return;
      std::swap(v[i], v[p]);
      i = p;
    }
  }
  void replace(const Result& r) {  // heap.go:79-90, siftDown heap.go:105-122
    v[0] = r;
    size_t i = 0;
    for (;;) {
      size_t l = 2 * i + 1;
      if (l >= v.size()) return;
      size_t best = l, rr = l + 1;
      if (rr < v.size() && less(v[rr], v[l])) best = rr;
      if (!less(v[best], v[i])) return;
      std::swap(v[i], v[best]);
      i = best;
    }
  }
  // Offer one result to a heap bounded at k (topk.go:146-153).
  void offer(const Result& r, size_t k) {
    if (v.size() < k) {
      push(r);
      return;
    }
    if (result_better(metric, r, v[0])) replace(r);
  }
  // Final best-first sort (topk.go:155-165).
  std::vector<Result> sorted() const {
    std::vector<Result> out = v;
    int m = metric;
    std::sort(out.begin(), out.end(),
              [m](const Result& a, const Result& b) { return result_better(m, a, b); });
    return out;
  }
};

inline bool filter_pass(const uint32_t* bitmap, int64_t position) {
  if (!bitmap) return true;
  return (bitmap[position >> 5] >> (position & 31)) & 1u;
}

// parallel.ParallelFor (internal/ailego/parallel/thread_pool.go:29-73): an
// atomic-counter work queue over `threads` workers.
template <typename F>
void parallel_for(int64_t count, int32_t threads, F fn) {
  if (threads <= 1 || count <= 1) {
    for (int64_t i = 0; i < count; ++i) fn(i);
    return;
  }
  std::atomic<int64_t> next{0};
  std::vector<std::thread> pool;
  int32_t workers = (int32_t)std::min<int64_t>(threads, count);
  for (int32_t w = 0; w < workers; ++w)
    pool.emplace_back([&]() {
      for (;;) {
        int64_t i = next.fetch_add(1);
        if (i >= count) return;
        fn(i);
      }
    });
  for (auto& t : pool) t.join();
}

// SearchOptions.Validate (query.go:47-55).
inline int validate_options(int32_t k, float radius) {
  if (k <= 0) return XO_INVALID_ARGUMENT;
  if (radius < 0 || std::isnan(radius) || std::isinf(radius)) return XO_INVALID_ARGUMENT;
  return XO_OK;
}

void write_results(const std::vector<Result>& res, int32_t k, int32_t q, uint64_t* out_keys,
                   float* out_scores, int32_t* out_counts) {
  int32_t c = (int32_t)std::min<size_t>(res.size(), (size_t)k);
  for (int32_t i = 0; i < c; ++i) {
    out_keys[(int64_t)q * k + i] = res[i].key;
    out_scores[(int64_t)q * k + i] = res[i].score;
  }
  out_counts[q] = c;
}

// topKPrevalidatedCandidatesWithOptions (topk.go:105-166) over a generic
// candidate accessor; `score_at` returns a status.
template <typename ScoreAt>
int topk_scan(int metric, int64_t count, int32_t top_k, float radius, const uint32_t* bitmap,
              const uint64_t* keys, const int64_t* positions, ScoreAt score_at,
              std::vector<Result>* out) {
  out->clear();
  if (top_k == 0 || count == 0) return XO_OK;
  size_t k = (size_t)std::min<int64_t>(top_k, count);
  WorstFirstHeap heap{metric, {}};
  heap.v.reserve(k);
  for (int64_t i = 0; i < count; ++i) {
    int64_t pos = positions ? positions[i] : i;
    if (!filter_pass(bitmap, pos)) continue;
    float s;
    int st = score_at(pos, &s);
    if (st != XO_OK) return st;
    if (!within_radius(metric, s, radius)) continue;
    heap.offer(Result{keys[pos], s}, k);
  }
  *out = heap.sorted();
  return XO_OK;
}

}  // namespace

extern "C" int xo_metric_compute(int metric, const float* a, const float* b, int64_t n,
                                 float* score) {
  // validateDensePair / validateDenseFinite (distance.go:132-150) then the
  // metric kernel (metric.go:35-48).
  if (n <= 0) return XO_INVALID_ARGUMENT;
  for (int64_t i = 0; i < n; ++i)
    if (!finite32(a[i]) || !finite32(b[i])) return XO_NON_FINITE;
  return prevalidated(metric, a, b, n, score);
}

// CosineDistanceWithMagnitudesPrevalidated (distance_prevalidated.go:57-68).
extern "C" int xo_cosine_with_magnitudes(const float* a, const float* b, int64_t n, float lm,
                                         float rm, float* score) {
  if (lm == 0 && rm == 0) {
    *score = 0;
    return XO_OK;
  }
  if (lm == 0 || rm == 0) {
    *score = 1;
    return XO_OK;
  }
  float c = xo_inner_product(a, b, n) / (lm * rm);
  c = go_min(1.0f, go_max(-1.0f, c));
  return finite_score((double)(1.0f - c), score);
}

// L2MagnitudePrevalidated (distance_prevalidated.go:46-55).
extern "C" int xo_l2_magnitude(const float* v, int64_t n, float* mag) {
  float norm = xo_inner_product(v, v, n);
  if (norm < 0) norm = 0;
  return finite_score(std::sqrt((double)norm), mag);
}

// ---------------------------------------------------------------------------
// internal/ailego/utility/float_helper.go:21-96 (binary16, round to nearest
// even; NaN payload kept non-zero).
// ---------------------------------------------------------------------------
extern "C" uint16_t xo_f32_to_f16(float value) {
  uint32_t bits;
  std::memcpy(&bits, &value, 4);
  uint16_t sign = (uint16_t)((bits >> 16) & 0x8000u);
  int exponent32 = (int)((bits >> 23) & 0xffu);
  uint32_t mantissa = bits & 0x7fffffu;
  if (exponent32 == 0xff) {
    if (mantissa == 0) return sign | 0x7c00u;
    uint16_t payload = (uint16_t)(mantissa >> 13);
    if (payload == 0) payload = 1;
    return sign | 0x7c00u | payload;
  }
  int exponent16 = exponent32 - 127 + 15;
  if (exponent16 >= 31) return sign | 0x7c00u;
  if (exponent16 <= 0) {
    if (exponent16 < -10) return sign;
    mantissa |= 0x800000u;
    uint32_t shift = (uint32_t)(14 - exponent16);
    uint32_t rounded = mantissa >> shift;
    uint32_t remainder = mantissa & ((1u << shift) - 1u);
    uint32_t halfway = 1u << (shift - 1);
    if (remainder > halfway || (remainder == halfway && (rounded & 1u))) rounded++;
    return sign | (uint16_t)rounded;
  }
  uint32_t rounded = mantissa >> 13;
  uint32_t remainder = mantissa & 0x1fffu;
  if (remainder > 0x1000u || (remainder == 0x1000u && (rounded & 1u))) {
    rounded++;
    if (rounded == 0x400u) {
      rounded = 0;
      exponent16++;
      if (exponent16 >= 31) return sign | 0x7c00u;
    }
  }
  return sign | (uint16_t)(exponent16 << 10) | (uint16_t)rounded;
}

extern "C" float xo_f16_to_f32(uint16_t bits) {
  uint32_t sign = (uint32_t)(bits & 0x8000u) << 16;
  uint32_t exponent = (bits >> 10) & 0x1fu;
  uint32_t mantissa = bits & 0x3ffu;
  uint32_t out;
  if (exponent == 0) {
    if (mantissa == 0) {
      out = sign;
    } else {
      int32_t e = 127 - 14;
      while ((mantissa & 0x400u) == 0) {
        mantissa <<= 1;
        e--;
      }
      mantissa &= 0x3ffu;
      out = sign | ((uint32_t)e << 23) | (mantissa << 13);
    }
  } else if (exponent == 0x1f) {
    out = sign | 0x7f800000u | (mantissa << 13);
  } else {
    out = sign | ((exponent + (127 - 15)) << 23) | (mantissa << 13);
  }
  float f;
  std::memcpy(&f, &out, 4);
  return f;
}

// ---------------------------------------------------------------------------
// Flat search: DenseFlatIndex.search (flat.go:179-196) →
// topKCandidatesWithOptions (topk.go:77-103) with requirePositiveTopK, run
// per query like core.BatchTopK (topk.go:242-269).
// ---------------------------------------------------------------------------
namespace {
// Query validation: metric.Compute(query, query) (topk.go:92-94).
int validate_query(int metric, const float* q, int32_t d) {
  float s;
  return xo_metric_compute(metric, q, q, d, &s);
}
}  // namespace

extern "C" int xo_flat_search(int metric, const float* rows, const uint64_t* keys, int64_t n,
                              int32_t d, const float* queries, int32_t nq, int32_t k,
                              float radius, const uint32_t* bitmap, int32_t threads,
                              uint64_t* out_keys, float* out_scores, int32_t* out_counts,
                              int32_t* out_status) {
  if (d <= 0 || metric < XO_L2 || metric > XO_MIPSL2) return XO_INVALID_ARGUMENT;
  int st0 = validate_options(k, radius);
  if (st0 != XO_OK) return st0;
  std::vector<int32_t> status(nq, XO_OK);
  parallel_for(nq, threads, [&](int64_t q) {
    const float* query = queries + q * d;
    int st = validate_query(metric, query, d);
    std::vector<Result> res;
    if (st == XO_OK)
      st = topk_scan(metric, n, k, radius, bitmap, keys, nullptr,
                     [&](int64_t pos, float* s) {
                       return prevalidated(metric, rows + pos * d, query, d, s);
                     },
                     &res);
    status[q] = st;
    if (st != XO_OK) res.clear();
    write_results(res, k, (int32_t)q, out_keys, out_scores, out_counts);
  });
  int first = XO_OK;
  for (int32_t q = 0; q < nq; ++q) {
    if (out_status) out_status[q] = status[q];
    if (first == XO_OK) first = status[q];
  }
  return first;
}

// MergeSearchResults (query.go:154-191).
extern "C" int32_t xo_merge_results(int metric, int32_t k, const uint64_t* keys,
                                    const float* scores, int64_t count, uint64_t* out_keys,
                                    float* out_scores) {
  if (k <= 0) return 0;
  WorstFirstHeap heap{metric, {}};
  for (int64_t i = 0; i < count; ++i) heap.offer(Result{keys[i], scores[i]}, (size_t)k);
  std::vector<Result> res = heap.sorted();
  for (size_t i = 0; i < res.size(); ++i) {
    out_keys[i] = res[i].key;
    out_scores[i] = res[i].score;
  }
  return (int32_t)res.size();
}

// ---------------------------------------------------------------------------
// Scalar quantization (internal/core/quantization.go).
// ---------------------------------------------------------------------------
namespace {
// quantizeInteger (quantization.go:267-321).  `store` receives each code.
template <typename Store>
int quantize_integer(const float* v, int32_t d, int lower, int upper, xo_sq_params* p,
                     Store store) {
  if (d <= 0) return XO_INVALID_ARGUMENT;
  for (int32_t i = 0; i < d; ++i)  // QuantizeVector finite check (quantization.go:86-90)
    if (!finite32(v[i])) return XO_NON_FINITE;
  float minimum = v[0], maximum = v[0];
  for (int32_t i = 1; i < d; ++i) {
    minimum = go_min(minimum, v[i]);
    maximum = go_max(maximum, v[i]);
  }
  p->code_sum = 0;
  p->code_square = 0;
  if (minimum == maximum) {
    p->inverse_scale = 0;
    p->offset = minimum;
    for (int32_t i = 0; i < d; ++i) store(i, 0);
    return XO_OK;
  }
  const float eps32 = 1.1920928955078125e-7f;
  float span = maximum - minimum;
  float scale = (float)(upper - lower) / go_max(span, eps32);
  float bias = (-minimum) * scale + (float)lower;
  float inverse_scale = 1.0f / scale;
  float offset = (-bias) / scale;
  if (!finite32(inverse_scale) || !finite32(offset)) return XO_OVERFLOW;
  p->inverse_scale = inverse_scale;
  p->offset = offset;
  for (int32_t i = 0; i < d; ++i) {
    float t = v[i] * scale + bias;  // two roundings: Go does not fuse on amd64
    int code = (int)std::round((double)t);
    code = std::min(upper, std::max(lower, code));
    p->code_sum += (double)code;
    p->code_square += (double)(code * code);
    store(i, code);
  }
  return XO_OK;
}
}  // namespace

extern "C" int xo_quantize_int8(const float* v, int32_t d, int8_t* codes, xo_sq_params* p) {
  return quantize_integer(v, d, -127, 127, p, [&](int32_t i, int c) { codes[i] = (int8_t)c; });
}

// QuantizeVector(QuantizationInt8, row) for each of n rows (threads > 1:
// rows split across threads; the per-row result does not depend on it).
// Returns the first failing row's status.
extern "C" int xo_quantize_int8_batch(const float* rows, int64_t n, int32_t d, int32_t threads,
                                      int8_t* codes, xo_sq_params* params) {
  std::vector<int> status(n > 0 ? (size_t)n : 1, XO_OK);
  parallel_for(n, threads, [&](int64_t i) {
    status[i] = xo_quantize_int8(rows + i * d, d, codes + i * d, &params[i]);
  });
  for (int64_t i = 0; i < n; ++i)
    if (status[i] != XO_OK) return status[i];
  return XO_OK;
}

extern "C" int xo_quantize_int4(const float* v, int32_t d, uint8_t* packed, xo_sq_params* p) {
  if (d % 2 != 0) return XO_INVALID_ARGUMENT;  // ErrOddInt4Dimension
  std::memset(packed, 0, (size_t)d / 2);
  return quantize_integer(v, d, -8, 7, p, [&](int32_t i, int c) {
    if (i % 2 == 0)
      packed[i / 2] = (uint8_t)((uint8_t)c & 0x0f);
    else
      packed[i / 2] |= (uint8_t)(((uint8_t)c & 0x0f) << 4);
  });
}

// xo_quantize_int4 over n rows (packed d / 2 bytes each).
extern "C" int xo_quantize_int4_batch(const float* rows, int64_t n, int32_t d, int32_t threads,
                                      uint8_t* packed, xo_sq_params* params) {
  if (d % 2 != 0) return XO_INVALID_ARGUMENT;
  std::vector<int> status(n > 0 ? (size_t)n : 1, XO_OK);
  parallel_for(n, threads, [&](int64_t i) {
    status[i] = xo_quantize_int4(rows + i * d, d, packed + i * (d / 2), &params[i]);
  });
  for (int64_t i = 0; i < n; ++i)
    if (status[i] != XO_OK) return status[i];
  return XO_OK;
}

namespace {
// finiteQuantizedScore (quantization.go:387-393).
inline int finite_quantized(double value, float* out) { return finite_score(value, out); }

// QuantizedDistance for integer kinds (quantization.go:171-235) given the
// exact integer code dot.  `left` is the stored code, `right` the query.
int quantized_formula(int metric, double dot_codes, const xo_sq_params& l,
                      const xo_sq_params& r, int32_t d, float* score) {
  double ls = (double)l.inverse_scale, rs = (double)r.inverse_scale;
  double lo = (double)l.offset, ro = (double)r.offset;
  double dim = (double)d;
  double inner = ls * rs * dot_codes + lo * rs * r.code_sum + ro * ls * l.code_sum + dim * lo * ro;
  double ln = ls * ls * l.code_square + 2 * ls * lo * l.code_sum + dim * lo * lo;
  double rn = rs * rs * r.code_square + 2 * rs * ro * r.code_sum + dim * ro * ro;
  double s = 0;
  switch (metric) {
    case XO_L2:
      s = ln + rn - 2 * inner;
      if (s < 0 && s > -1e-6 * go_maxd(1, ln + rn)) s = 0;
      break;
    case XO_IP: s = inner; break;
    case XO_COSINE:
      if (ln == 0 && rn == 0)
        s = 0;
      else if (ln == 0 || rn == 0)
        s = 1;
      else {
        double c = inner / std::sqrt(ln * rn);
        c = go_mind(1, go_maxd(-1, c));
        s = 1 - c;
      }
      break;
    case XO_MIPSL2: {
      double den = go_maxd(ln, rn);
      s = den == 0 ? 0 : 2 - 2 * inner / den;
      break;
    }
    default: return XO_INVALID_ARGUMENT;
  }
  return finite_quantized(s, score);
}

// integerCodeDot (quantization.go:358-366): float64 sum of int products in
// index order (exact while |sum| < 2^53).
double int8_code_dot(const int8_t* a, const int8_t* b, int32_t d) {
  double dot = 0;
  for (int32_t i = 0; i < d; ++i) dot += (double)((int)a[i] * (int)b[i]);
  return dot;
}
}  // namespace

extern "C" int xo_quantized_distance_int8(int metric, const int8_t* left, const xo_sq_params* lp,
                                          const int8_t* right, const xo_sq_params* rp, int32_t d,
                                          float* score) {
  return quantized_formula(metric, int8_code_dot(left, right, d), *lp, *rp, d, score);
}

namespace {
// QuantizedVector.integerCode for INT4 (quantization.go:368-383).
inline int int4_code(const uint8_t* packed, int32_t i) {
  int v = (i % 2 == 0) ? (packed[i / 2] & 0x0f) : (packed[i / 2] >> 4);
  if (v & 0x08) v -= 16;
  return v;
}
}  // namespace

// QuantizedDistance on two INT4 codes (packed d / 2 bytes each).
extern "C" int xo_quantized_distance_int4(int metric, const uint8_t* left, const xo_sq_params* lp,
                                          const uint8_t* right, const xo_sq_params* rp,
                                          int32_t d, float* score) {
  double dot = 0;
  for (int32_t i = 0; i < d; ++i) dot += (double)(int4_code(left, i) * int4_code(right, i));
  return quantized_formula(metric, dot, *lp, *rp, d, score);
}

// RefinementCandidateCount (refiner.go:112-129).
extern "C" int xo_refinement_candidate_count(int32_t top_k, float scale, int32_t* count) {
  if (top_k <= 0) return XO_INVALID_ARGUMENT;
  if (scale <= 0 || std::isnan(scale) || std::isinf(scale)) return XO_INVALID_ARGUMENT;
  double product = (double)top_k * (double)scale;
  if (product >= 2147483647.0) return XO_INVALID_ARGUMENT;
  int64_t c = (int64_t)std::floor(product);
  if (c < 1) c = 1;
  *count = (int32_t)c;
  return XO_OK;
}

namespace {
// OriginalVectorRefiner.Refine (refiner.go:66-108): dedup by key in input
// order, drop filtered keys, exact metric over originals, top-k with radius.
int refine_exact(int metric, const float* query, int32_t d, const std::vector<Result>& cands,
                 const std::vector<int64_t>& cand_positions, const float* originals,
                 const uint64_t* keys, int32_t k, float radius, const uint32_t* bitmap,
                 std::vector<Result>* out) {
  std::vector<int64_t> exact;
  std::vector<uint64_t> seen;
  for (size_t i = 0; i < cands.size(); ++i) {
    uint64_t key = cands[i].key;
    if (std::find(seen.begin(), seen.end(), key) != seen.end()) continue;
    seen.push_back(key);
    if (!filter_pass(bitmap, cand_positions[i])) continue;
    exact.push_back(cand_positions[i]);
  }
  return topk_scan(metric, (int64_t)exact.size(), k, radius, nullptr, keys, exact.data(),
                   [&](int64_t pos, float* s) {
                     return prevalidated(metric, originals + pos * d, query, d, s);
                   },
                   out);
}
}  // namespace

// SQ-Flat search with optional refinement.  Quantized stage:
// scalarQuantizedVectors.search → searchWithCode (quantized_index.go:296-335):
// every accepted (filter, radius) score, then MergeSearchResults.
static int sq_flat_search(int bits, int metric, const uint8_t* codes, const xo_sq_params* params,
                             const float* originals, const uint64_t* keys, int64_t n, int32_t d,
                             const float* queries, int32_t nq, int32_t k, float radius,
                             float refine_scale, const uint32_t* bitmap, int32_t threads,
                             uint64_t* out_keys, float* out_scores, int32_t* out_counts,
                             int32_t* out_status) {
  int st0 = validate_options(k, radius);
  if (st0 != XO_OK) return st0;
  int32_t stage_k = k;
  float stage_radius = radius;
  bool refine = refine_scale > 0;
  if (refine) {
    st0 = xo_refinement_candidate_count(k, refine_scale, &stage_k);
    if (st0 != XO_OK) return st0;
    stage_radius = 0;  // executeCollectionDenseSearch drops the radius (collection.go:1623)
  }
  std::vector<int32_t> status(nq, XO_OK);
  parallel_for(nq, threads, [&](int64_t q) {
    const float* query = queries + q * d;
    std::vector<Result> res;
    int st = validate_query(metric, query, d);  // validateQuery (quantized_index.go:264-272)
    std::vector<uint8_t> qcode(bits == 4 ? d / 2 + 1 : d);
    xo_sq_params qp;
    if (st == XO_OK)
      st = bits == 4 ? xo_quantize_int4(query, d, qcode.data(), &qp)
                     : xo_quantize_int8(query, d, reinterpret_cast<int8_t*>(qcode.data()), &qp);
    std::vector<Result> stage;
    std::vector<int64_t> stage_pos;
    if (st == XO_OK) {
      // searchWithCode accepts every candidate then keeps the best stage_k
      // with MergeSearchResults; a bounded heap yields the same set.
      WorstFirstHeap heap{metric, {}};
      for (int64_t pos = 0; pos < n && st == XO_OK; ++pos) {
        if (!filter_pass(bitmap, pos)) continue;
        float s;
        st = bits == 4
                 ? xo_quantized_distance_int4(metric, codes + pos * (d / 2), &params[pos],
                                              qcode.data(), &qp, d, &s)
                 : xo_quantized_distance_int8(
                       metric, reinterpret_cast<const int8_t*>(codes) + pos * d, &params[pos],
                       reinterpret_cast<const int8_t*>(qcode.data()), &qp, d, &s);
        if (st != XO_OK) break;
        if (!within_radius(metric, s, stage_radius)) continue;
        heap.offer(Result{keys[pos], s}, (size_t)stage_k);
      }
      if (st == XO_OK) stage = heap.sorted();
    }
    if (st == XO_OK && refine) {
      // Keys are unique and equal to positions' keys; recover positions.
      stage_pos.resize(stage.size());
      for (size_t i = 0; i < stage.size(); ++i) {
        int64_t pos = -1;
        for (int64_t p = 0; p < n; ++p)
          if (keys[p] == stage[i].key) {
            pos = p;
            break;
          }
        stage_pos[i] = pos;
      }
      st = refine_exact(metric, query, d, stage, stage_pos, originals, keys, k, radius, bitmap,
                        &res);
    } else if (st == XO_OK) {
      res = stage;
    }
    status[q] = st;
    if (st != XO_OK) res.clear();
    write_results(res, k, (int32_t)q, out_keys, out_scores, out_counts);
  });
  int first = XO_OK;
  for (int32_t q = 0; q < nq; ++q) {
    if (out_status) out_status[q] = status[q];
    if (first == XO_OK) first = status[q];
  }
  return first;
}

extern "C" int xo_sq8_search(int metric, const int8_t* codes, const xo_sq_params* params,
                             const float* originals, const uint64_t* keys, int64_t n, int32_t d,
                             const float* queries, int32_t nq, int32_t k, float radius,
                             float refine_scale, const uint32_t* bitmap, int32_t threads,
                             uint64_t* out_keys, float* out_scores, int32_t* out_counts,
                             int32_t* out_status) {
  return sq_flat_search(8, metric, reinterpret_cast<const uint8_t*>(codes), params, originals,
                        keys, n, d, queries, nq, k, radius, refine_scale, bitmap, threads,
                        out_keys, out_scores, out_counts, out_status);
}

// The same search over INT4 codes (QuantizationInt4; packed d / 2 bytes per
// row).  An odd d fails every query in quantizeVector (ErrOddInt4Dimension).
extern "C" int xo_sq4_search(int metric, const uint8_t* codes, const xo_sq_params* params,
                             const float* originals, const uint64_t* keys, int64_t n, int32_t d,
                             const float* queries, int32_t nq, int32_t k, float radius,
                             float refine_scale, const uint32_t* bitmap, int32_t threads,
                             uint64_t* out_keys, float* out_scores, int32_t* out_counts,
                             int32_t* out_status) {
  return sq_flat_search(4, metric, codes, params, originals, keys, n, d, queries, nq, k, radius,
                        refine_scale, bitmap, threads, out_keys, out_scores, out_counts,
                        out_status);
}

// ---------------------------------------------------------------------------
// k-means (internal/core/kmeans.go, internal/ailego/algorithm).
// ---------------------------------------------------------------------------

// splitMix64.next (kmeans.go:607-613).
extern "C" uint64_t xo_splitmix64_next(uint64_t* state) {
  *state += 0x9e3779b97f4a7c15ULL;
  uint64_t v = *state;
  v = (v ^ (v >> 30)) * 0xbf58476d1ce4e5b9ULL;
  v = (v ^ (v >> 27)) * 0x94d049bb133111ebULL;
  return v ^ (v >> 31);
}

namespace {
// splitMix64.intn (kmeans.go:615-628): rejection sampling.
int64_t splitmix_intn(uint64_t* state, int64_t limit) {
  if (limit <= 1) return 0;
  uint64_t bound = (uint64_t)limit;
  uint64_t threshold = (0 - bound) % bound;
  for (;;) {
    uint64_t v = xo_splitmix64_next(state);
    if (v >= threshold) return (int64_t)(v % bound);
  }
}

// nearestCentroidContext (kmeans.go:485-509): metric.Compute over centroids,
// strictly Better replaces, so the lower index wins ties.
int nearest_centroid(int metric, const float* centroids, int32_t nc, int32_t d, const float* v,
                     int32_t* label, float* score) {
  if (nc <= 0) return XO_INVALID_ARGUMENT;
  float best;
  int st = xo_metric_compute(metric, centroids, v, d, &best);
  if (st != XO_OK) return st;
  int32_t bi = 0;
  for (int32_t c = 1; c < nc; ++c) {
    float s;
    st = xo_metric_compute(metric, centroids + (int64_t)c * d, v, d, &s);
    if (st != XO_OK) return st;
    if (better(metric, s, best)) {
      bi = c;
      best = s;
    }
  }
  *label = bi;
  *score = best;
  return XO_OK;
}
}  // namespace

// algorithm.InitializeReservoir (internal/ailego/algorithm/kmeans.go:25-56)
// with splitMix64{Seed}.intn (kmeans.go:365-367).
extern "C" int xo_kmeans_reservoir(int64_t n, int32_t clusters, uint64_t seed, int64_t* indices) {
  uint64_t state = seed;
  for (int32_t i = 0; i < clusters; ++i) indices[i] = i;
  for (int64_t i = clusters; i < n; ++i) {
    int64_t selected = splitmix_intn(&state, i + 1);
    if (selected < clusters) indices[selected] = i;
  }
  return XO_OK;
}

// assignKMeans (kmeans.go:382-411) and assignKMeansCosine (kmeans.go:413-479).
extern "C" int xo_kmeans_assign(int metric, const float* vectors, int64_t n,
                                const float* centroids, int32_t nc, int32_t d, int32_t threads,
                                int32_t* labels, float* scores) {
  if (nc <= 0 || d <= 0) return XO_INVALID_ARGUMENT;
  std::vector<float> cmag;
  if (metric == XO_COSINE) {
    cmag.resize(nc);
    for (int32_t c = 0; c < nc; ++c) {
      int st = xo_l2_magnitude(centroids + (int64_t)c * d, d, &cmag[c]);
      if (st != XO_OK) return st;
    }
  }
  std::atomic<int> err{XO_OK};
  parallel_for(n, threads, [&](int64_t i) {
    const float* v = vectors + i * d;
    int st;
    if (metric == XO_COSINE) {  // nearestCosineCentroidContext (kmeans.go:445-479)
      float vm;
      st = xo_l2_magnitude(v, d, &vm);
      if (st == XO_OK) {
        float best;
        st = xo_cosine_with_magnitudes(centroids, v, d, cmag[0], vm, &best);
        int32_t bi = 0;
        for (int32_t c = 1; c < nc && st == XO_OK; ++c) {
          float s;
          st = xo_cosine_with_magnitudes(centroids + (int64_t)c * d, v, d, cmag[c], vm, &s);
          if (st == XO_OK && s < best) {
            bi = c;
            best = s;
          }
        }
        labels[i] = bi;
        scores[i] = best;
      }
    } else {
      st = nearest_centroid(metric, centroids, nc, d, v, &labels[i], &scores[i]);
    }
    if (st != XO_OK) err = st;
  });
  return err.load();
}

// trainKMeansWithAssignments (kmeans.go:208-298) with the default options of
// DefaultKMeansOptions (kmeans.go:83-92): reservoir initialisation,
// EmptyReseedFarthest, non-spherical; LloydUpdate (lloyd_cluster.go:53-138).
// Lloyd iterations of TrainKMeans (kmeans.go:240-298) from kc initial
// centroids (cents, updated in place).
static int kmeans_lloyd(int metric, const float* vectors, int64_t n, int32_t d, int32_t kc,
                        std::vector<float>& cents, int32_t max_iterations, double tolerance,
                        int32_t threads, float* centroids_out, int32_t* labels_out) {
  std::vector<int32_t> labels(n);
  std::vector<float> scores(n);
  double previous = 0;
  for (int32_t it = 0; it < max_iterations; ++it) {
    int st = xo_kmeans_assign(metric, vectors, n, cents.data(), kc, d, threads, labels.data(),
                              scores.data());
    if (st != XO_OK) return st;
    // LloydUpdate: float64 sums in input order.
    std::vector<int64_t> counts(kc, 0);
    std::vector<double> sums((size_t)kc * d, 0.0);
    for (int64_t i = 0; i < n; ++i) {
      int32_t l = labels[i];
      counts[l]++;
      for (int32_t j = 0; j < d; ++j) sums[(size_t)l * d + j] += (double)vectors[i * d + j];
    }
    std::vector<float> next((size_t)kc * d);
    std::vector<int32_t> empty;
    for (int32_t c = 0; c < kc; ++c) {
      if (counts[c] == 0) {
        empty.push_back(c);
        std::memcpy(&next[(size_t)c * d], &cents[(size_t)c * d], sizeof(float) * d);
        continue;
      }
      for (int32_t j = 0; j < d; ++j)
        next[(size_t)c * d + j] = (float)(sums[(size_t)c * d + j] / (double)counts[c]);
    }
    bool changed = false;
    // EmptyReseedFarthest (lloyd_cluster.go:100-117, worstAssignedVector :140-160).
    std::vector<char> used(n, 0);
    for (int32_t c : empty) {
      int64_t sel = -1;
      for (int64_t i = 0; i < n; ++i) {
        if (used[i]) continue;
        if (sel < 0 || better(metric, scores[sel], scores[i])) sel = i;
      }
      if (sel < 0) break;
      used[sel] = 1;
      std::memcpy(&next[(size_t)c * d], vectors + sel * d, sizeof(float) * d);
      changed = true;
    }
    // kMeansObjective (kmeans.go:537-552).
    double cost = 0;
    for (int64_t i = 0; i < n; ++i) cost += metric == XO_IP ? -(double)scores[i] : (double)scores[i];
    cents.swap(next);
    if (!changed && std::fabs(cost - previous) < tolerance) break;
    previous = cost;
  }
  int st = xo_kmeans_assign(metric, vectors, n, cents.data(), kc, d, threads, labels_out,
                            scores.data());
  if (st != XO_OK) return st;
  std::memcpy(centroids_out, cents.data(), sizeof(float) * cents.size());
  return XO_OK;
}

extern "C" int xo_kmeans_train(int metric, const float* vectors, int64_t n, int32_t d,
                               int32_t clusters, int32_t max_iterations, double tolerance,
                               uint64_t seed, int32_t threads, float* centroids_out,
                               int32_t* clusters_out, int32_t* labels_out) {
  if (n <= 0 || d <= 0 || clusters <= 0 || max_iterations <= 0) return XO_INVALID_ARGUMENT;
  int32_t kc = (int32_t)std::min<int64_t>(clusters, n);
  std::vector<int64_t> idx(kc);
  xo_kmeans_reservoir(n, kc, seed, idx.data());
  std::vector<float> cents((size_t)kc * d);
  for (int32_t c = 0; c < kc; ++c)
    std::memcpy(&cents[(size_t)c * d], vectors + idx[c] * d, sizeof(float) * d);
  int st = kmeans_lloyd(metric, vectors, n, d, kc, cents, max_iterations, tolerance, threads,
                        centroids_out, labels_out);
  if (st != XO_OK) return st;
  *clusters_out = kc;
  return XO_OK;
}

// TrainKMeans with KMeansOptions.InitialCentroids (kmeans.go:354-363): kc =
// min(clusters, n) given centroids, then the Lloyd iterations.
extern "C" int xo_kmeans_train_init(int metric, const float* vectors, int64_t n, int32_t d,
                                    int32_t kc, const float* initial, int32_t max_iterations,
                                    double tolerance, int32_t threads, float* centroids_out,
                                    int32_t* labels_out) {
  if (n <= 0 || d <= 0 || kc <= 0 || kc > n || max_iterations <= 0) return XO_INVALID_ARGUMENT;
  std::vector<float> cents(initial, initial + (size_t)kc * d);
  for (float v : cents)
    if (!finite32(v)) return XO_INVALID_ARGUMENT;
  return kmeans_lloyd(metric, vectors, n, d, kc, cents, max_iterations, tolerance, threads,
                      centroids_out, labels_out);
}

// splitMix64.float64 (kmeans.go:630-632).
static double splitmix_float64(uint64_t* state) {
  return (double)(xo_splitmix64_next(state) >> 11) * (1.0 / 9007199254740992.0);
}

// pqUniformSampleIndices (pq.go:461-476): `sample` of `count` indices in
// increasing order, index i kept with odds remaining / (count - i).
static std::vector<int64_t> pq_uniform_sample(int64_t count, int64_t sample, uint64_t* state) {
  std::vector<int64_t> out;
  int64_t remaining = sample;
  for (int64_t i = 0; i < count && remaining > 0; ++i)
    if (splitmix_intn(state, count - i) < remaining) {
      out.push_back(i);
      --remaining;
    }
  return out;
}

// initializePQKMC2 (pq.go:410-459): the first centroid uniformly, then each
// next one by a Markov chain over min(32, n) uniform candidates scored by
// their nearest centroid (metric.Compute; IP negated), accepting a candidate
// when the current score is 0 or score * float32(U) < candidate score.
extern "C" int xo_pq_kmc2(int metric, const float* vectors, int64_t n, int32_t d,
                          int32_t clusters, uint64_t seed, float* centroids_out) {
  if (clusters <= 0 || clusters > n) return XO_INVALID_ARGUMENT;
  uint64_t state = seed;
  std::vector<int64_t> first = pq_uniform_sample(n, 1, &state);
  std::vector<const float*> chosen{vectors + first[0] * d};
  while ((int32_t)chosen.size() < clusters) {
    std::vector<int64_t> cand = pq_uniform_sample(n, std::min<int64_t>(32, n), &state);
    std::vector<float> scores(cand.size());
    for (size_t ci = 0; ci < cand.size(); ++ci) {
      float best = 3.40282346638528859811704183484516925440e+38f;
      for (const float* c : chosen) {
        float sc;
        int st = xo_metric_compute(metric, c, vectors + cand[ci] * d, d, &sc);
        if (st != XO_OK) return st;
        if (metric == XO_IP) sc = -sc;
        if (sc < best) best = sc;
      }
      scores[ci] = best;
    }
    float sel_score = scores[0];
    size_t sel = 0;
    for (size_t ci = 1; ci < scores.size(); ++ci) {
      // The draw happens only when the current score is not 0 (|| short-circuits).
      if (sel_score == 0 || sel_score * (float)splitmix_float64(&state) < scores[ci]) {
        sel_score = scores[ci];
        sel = ci;
      }
    }
    chosen.push_back(vectors + cand[sel] * d);
  }
  for (int32_t c = 0; c < clusters; ++c)
    std::memcpy(centroids_out + (int64_t)c * d, chosen[c], sizeof(float) * d);
  return XO_OK;
}

// TrainPQ (pq.go:107-179): per contiguous chunk (pqChunkOffsets), the first
// min(n, max_train_samples) rows' sub-vectors, KMC2 seeding and TrainKMeans
// with 256 clusters, seed ^ (0x70716b6d00000000 + chunk), max_iterations and
// the default tolerance; pivots [256][d] centroid-major, rows past the
// trained centroids repeating centroid 0.
extern "C" int xo_pq_train(int metric, const float* vectors, int64_t n, int32_t d, int32_t chunks,
                           int64_t max_train_samples, int32_t max_iterations, uint64_t seed,
                           int32_t threads, float* pivots_out) {
  if (n <= 0 || d <= 0 || chunks <= 0 || chunks > d || max_train_samples <= 0 ||
      max_iterations <= 0 || (metric != XO_L2 && metric != XO_IP))
    return XO_INVALID_ARGUMENT;
  std::vector<int32_t> offsets(chunks + 1);
  xo_pq_chunk_offsets(d, chunks, offsets.data());
  const int64_t samples = std::min<int64_t>(n, max_train_samples);
  for (int32_t chunk = 0; chunk < chunks; ++chunk) {
    const int32_t start = offsets[chunk], width = offsets[chunk + 1] - offsets[chunk];
    std::vector<float> training((size_t)samples * width);
    for (int64_t i = 0; i < samples; ++i)
      std::memcpy(&training[(size_t)i * width], vectors + i * d + start, sizeof(float) * width);
    const uint64_t cseed = seed ^ (0x70716b6d00000000ULL + (uint64_t)chunk);
    const int32_t kc = (int32_t)std::min<int64_t>(256, samples);
    std::vector<float> init((size_t)kc * width), cents((size_t)kc * width);
    std::vector<int32_t> labels(samples);
    int st = xo_pq_kmc2(metric, training.data(), samples, width, kc, cseed, init.data());
    if (st != XO_OK) return st;
    st = xo_kmeans_train_init(metric, training.data(), samples, width, kc, init.data(),
                              max_iterations, 1.1920928955078125e-7, threads, cents.data(),
                              labels.data());
    if (st != XO_OK) return st;
    for (int32_t c = 0; c < 256; ++c) {
      const float* src = &cents[(size_t)(c < kc ? c : 0) * width];
      std::memcpy(pivots_out + (int64_t)c * d + start, src, sizeof(float) * width);
    }
  }
  return XO_OK;
}

// ---------------------------------------------------------------------------
// IVF probe and exact list scan (internal/core/ivf.go).
// ---------------------------------------------------------------------------

// probedListsLocked (ivf.go:524-561) for the non-cosine metrics: TopK over
// centroids keyed by centroid index (ties → lower index); for cosine the
// magnitude-cached distance of distance_prevalidated.go:57-68.
extern "C" int32_t xo_ivf_probe(int metric, const float* centroids, int32_t nlist, int32_t d,
                                const float* query, int32_t nprobe, int32_t* lists) {
  if (nlist <= 0 || nprobe <= 0) return 0;
  std::vector<uint64_t> ids(nlist);
  for (int32_t c = 0; c < nlist; ++c) ids[c] = (uint64_t)c;
  std::vector<float> cmag;
  float qmag = 0;
  if (metric == XO_COSINE) {
    cmag.resize(nlist);
    for (int32_t c = 0; c < nlist; ++c) xo_l2_magnitude(centroids + (int64_t)c * d, d, &cmag[c]);
    xo_l2_magnitude(query, d, &qmag);
  }
  std::vector<Result> res;
  int32_t count = std::min(nprobe, nlist);
  int st = topk_scan(metric, nlist, count, 0, nullptr, ids.data(), nullptr,
                     [&](int64_t c, float* s) {
                       if (metric == XO_COSINE)
                         return xo_cosine_with_magnitudes(centroids + c * d, query, d, cmag[c],
                                                          qmag, s);
                       return xo_metric_compute(metric, centroids + c * d, query, d, s);
                     },
                     &res);
  if (st != XO_OK) return -st;
  for (size_t i = 0; i < res.size(); ++i) lists[i] = (int32_t)res[i].key;
  return (int32_t)res.size();
}

// searchIVF (ivf.go:427-493): probe, then topKPrevalidatedCandidateBatches
// (topk.go:171-237) over the probed lists in probe order.
extern "C" int xo_ivf_flat_search(int metric, const float* rows, const uint64_t* keys, int64_t n,
                                  int32_t d, const float* centroids, int32_t nlist,
                                  const int64_t* list_offsets, const int64_t* list_positions,
                                  const float* queries, int32_t nq, int32_t k, int32_t nprobe,
                                  float radius, const uint32_t* bitmap, int32_t threads,
                                  uint64_t* out_keys, float* out_scores, int32_t* out_counts,
                                  int32_t* out_status) {
  int st0 = validate_options(k, radius);
  if (st0 != XO_OK) return st0;
  if (nprobe <= 0) return XO_INVALID_ARGUMENT;
  std::vector<float> rmag;
  if (metric == XO_COSINE) {
    rmag.resize(n);
    for (int64_t p = 0; p < n; ++p) xo_l2_magnitude(rows + p * d, d, &rmag[p]);
  }
  std::vector<int32_t> status(nq, XO_OK);
  parallel_for(nq, threads, [&](int64_t q) {
    const float* query = queries + q * d;
    int st = validate_query(metric, query, d);
    std::vector<Result> res;
    if (st == XO_OK && n > 0) {
      std::vector<int32_t> lists(std::min(nprobe, nlist));
      int32_t np = xo_ivf_probe(metric, centroids, nlist, d, query, nprobe, lists.data());
      if (np < 0) st = -np;
      float qmag = 0;
      if (metric == XO_COSINE) xo_l2_magnitude(query, d, &qmag);
      std::vector<int64_t> pos;
      for (int32_t i = 0; i < np; ++i)
        for (int64_t j = list_offsets[lists[i]]; j < list_offsets[lists[i] + 1]; ++j)
          pos.push_back(list_positions[j]);
      if (st == XO_OK)
        st = topk_scan(metric, (int64_t)pos.size(), k, radius, bitmap, keys, pos.data(),
                       [&](int64_t p, float* s) {
                         if (metric == XO_COSINE)
                           return xo_cosine_with_magnitudes(rows + p * d, query, d, rmag[p], qmag,
                                                            s);
                         return prevalidated(metric, rows + p * d, query, d, s);
                       },
                       &res);
    }
    status[q] = st;
    if (st != XO_OK) res.clear();
    write_results(res, k, (int32_t)q, out_keys, out_scores, out_counts);
  });
  int first = XO_OK;
  for (int32_t q = 0; q < nq; ++q) {
    if (out_status) out_status[q] = status[q];
    if (first == XO_OK) first = status[q];
  }
  return first;
}

// ScalarQuantizedIVFIndex.search (ivf_quantized.go:135-192): quantizedQuery
// first (validation, then the INT8 code), then the probe with the original
// metric, then searchWithCode (quantized_index.go:313-335) over the probed
// lists' positions; with refine_scale > 0 the refine stage of xo_sq8_search.
extern "C" int xo_ivf_sq8_search(int metric, const int8_t* codes, const xo_sq_params* params,
                                 const float* originals, const uint64_t* keys, int64_t n,
                                 int32_t d, const float* centroids, int32_t nlist,
                                 const int64_t* list_offsets, const int64_t* list_positions,
                                 const float* queries, int32_t nq, int32_t k, int32_t nprobe,
                                 float radius, float refine_scale, const uint32_t* bitmap,
                                 int32_t threads, uint64_t* out_keys, float* out_scores,
                                 int32_t* out_counts, int32_t* out_status) {
  int st0 = validate_options(k, radius);
  if (st0 != XO_OK) return st0;
  if (nprobe <= 0) return XO_INVALID_ARGUMENT;
  int32_t stage_k = k;
  float stage_radius = radius;
  const bool refine = refine_scale > 0;
  if (refine) {
    st0 = xo_refinement_candidate_count(k, refine_scale, &stage_k);
    if (st0 != XO_OK) return st0;
    stage_radius = 0;
  }
  std::vector<int32_t> status(nq, XO_OK);
  parallel_for(nq, threads, [&](int64_t q) {
    const float* query = queries + q * d;
    std::vector<Result> res;
    int st = validate_query(metric, query, d);
    std::vector<int8_t> qcode(d);
    xo_sq_params qp;
    if (st == XO_OK) st = xo_quantize_int8(query, d, qcode.data(), &qp);
    std::vector<Result> stage;
    std::vector<int64_t> pos;
    if (st == XO_OK && n > 0) {
      std::vector<int32_t> lists(std::min(nprobe, nlist));
      int32_t np = xo_ivf_probe(metric, centroids, nlist, d, query, nprobe, lists.data());
      if (np < 0) st = -np;
      for (int32_t i = 0; i < np; ++i)
        for (int64_t j = list_offsets[lists[i]]; j < list_offsets[lists[i] + 1]; ++j)
          pos.push_back(list_positions[j]);
      WorstFirstHeap heap{metric, {}};
      for (size_t i = 0; i < pos.size() && st == XO_OK; ++i) {
        const int64_t p = pos[i];
        if (!filter_pass(bitmap, p)) continue;
        float sc;
        st = xo_quantized_distance_int8(metric, codes + p * d, &params[p], qcode.data(), &qp, d,
                                        &sc);
        if (st != XO_OK) break;
        if (!within_radius(metric, sc, stage_radius)) continue;
        heap.offer(Result{keys[p], sc}, (size_t)stage_k);
      }
      if (st == XO_OK) stage = heap.sorted();
    }
    if (st == XO_OK && refine) {
      std::vector<int64_t> stage_pos(stage.size(), -1);
      for (size_t i = 0; i < stage.size(); ++i)
        for (int64_t p : pos)
          if (keys[p] == stage[i].key) {
            stage_pos[i] = p;
            break;
          }
      st = refine_exact(metric, query, d, stage, stage_pos, originals, keys, k, radius, bitmap,
                        &res);
    } else if (st == XO_OK) {
      res = stage;
    }
    status[q] = st;
    if (st != XO_OK) res.clear();
    write_results(res, k, (int32_t)q, out_keys, out_scores, out_counts);
  });
  int first = XO_OK;
  for (int32_t q = 0; q < nq; ++q) {
    if (out_status) out_status[q] = status[q];
    if (first == XO_OK) first = status[q];
  }
  return first;
}

// ---------------------------------------------------------------------------
// Product quantization (internal/core/pq.go).
// ---------------------------------------------------------------------------

// pqChunkOffsets (pq.go:395-406): contiguous chunks, wider chunks first.
extern "C" void xo_pq_chunk_offsets(int32_t d, int32_t chunks, int32_t* offsets) {
  int32_t base = d / chunks, larger = d % chunks;
  offsets[0] = 0;
  for (int32_t c = 0; c < chunks; ++c) offsets[c + 1] = offsets[c] + base + (c < larger ? 1 : 0);
}

namespace {
// subspaceScore (pq.go:373-381): metric.Compute on the chunk slices.
inline int subspace_score(int metric, const float* pivots, int32_t d, const float* v,
                          int32_t centroid, int32_t start, int32_t end, float* s) {
  return xo_metric_compute(metric, v + start, pivots + (int64_t)centroid * d + start, end - start,
                           s);
}
}  // namespace

// Encode (pq.go:274-301): per chunk argmin by Better, ties → lower id.
extern "C" int xo_pq_encode(int metric, const float* pivots, const int32_t* offsets,
                            int32_t chunks, int32_t d, const float* v, uint8_t* code) {
  for (int32_t c = 0; c < chunks; ++c) {
    float best;
    int st = subspace_score(metric, pivots, d, v, 0, offsets[c], offsets[c + 1], &best);
    if (st != XO_OK) return st;
    int32_t bi = 0;
    for (int32_t p = 1; p < 256; ++p) {
      float s;
      st = subspace_score(metric, pivots, d, v, p, offsets[c], offsets[c + 1], &s);
      if (st != XO_OK) return st;
      if (better(metric, s, best)) {
        bi = p;
        best = s;
      }
    }
    code[c] = (uint8_t)bi;
  }
  return XO_OK;
}

// DistanceTable (pq.go:549-571): chunk-major [chunks][256].
extern "C" int xo_pq_distance_table(int metric, const float* pivots, const int32_t* offsets,
                                    int32_t chunks, int32_t d, const float* query, float* table) {
  for (int32_t c = 0; c < chunks; ++c)
    for (int32_t p = 0; p < 256; ++p) {
      int st = subspace_score(metric, pivots, d, query, p, offsets[c], offsets[c + 1],
                              &table[(int64_t)c * 256 + p]);
      if (st != XO_OK) return st;
    }
  return XO_OK;
}

// Lookup (pq.go:574-595): float64 sum in chunk order, overflow-checked.
extern "C" int xo_pq_lookup(const float* table, int32_t chunks, const uint8_t* code, float* score) {
  double s = 0;
  for (int32_t c = 0; c < chunks; ++c) s += (double)table[(int64_t)c * 256 + code[c]];
  if (std::isnan(s) || std::isinf(s) || s > 3.4028234663852886e38 || s < -3.4028234663852886e38)
    return XO_OVERFLOW;
  *score = (float)s;
  return XO_OK;
}

// IVF-PQ, composed from reference primitives (no single reference type):
//   probe   = probedListsLocked (ivf.go:524-561) over the IVF centroids;
//   scoring = PQDistanceTable.Lookup (pq.go:574-595) of the per-query table
//             (pq.go:549-571) on each probed position's raw-vector PQ code;
//   ranking = topKPrevalidatedCandidateBatchesWithOptions (topk.go:171-237):
//             filter before scoring, radius, worst-first heap, ties → key.
extern "C" int xo_ivfpq_search(int metric, const float* centroids, int32_t nlist, int32_t d,
                               const float* pivots, const int32_t* offsets, int32_t chunks,
                               const uint8_t* codes, const uint64_t* keys,
                               const int64_t* list_offsets, const int64_t* list_positions,
                               const float* queries, int32_t nq, int32_t k, int32_t nprobe,
                               float radius, const uint32_t* bitmap, int32_t threads,
                               uint64_t* out_keys, float* out_scores, int32_t* out_counts,
                               int32_t* out_status) {
  int st0 = validate_options(k, radius);
  if (st0 != XO_OK) return st0;
  if (nprobe <= 0 || (metric != XO_L2 && metric != XO_IP)) return XO_INVALID_ARGUMENT;
  std::vector<int32_t> status(nq, XO_OK);
  parallel_for(nq, threads, [&](int64_t q) {
    const float* query = queries + q * d;
    int st = validate_query(metric, query, d);
    std::vector<Result> res;
    if (st == XO_OK) {
      std::vector<int32_t> lists(std::min(nprobe, nlist));
      int32_t np = xo_ivf_probe(metric, centroids, nlist, d, query, nprobe, lists.data());
      if (np < 0) st = -np;
      std::vector<float> table((size_t)chunks * 256);
      if (st == XO_OK) st = xo_pq_distance_table(metric, pivots, offsets, chunks, d, query,
                                                 table.data());
      std::vector<int64_t> pos;
      for (int32_t i = 0; i < np && st == XO_OK; ++i)
        for (int64_t j = list_offsets[lists[i]]; j < list_offsets[lists[i] + 1]; ++j)
          pos.push_back(list_positions[j]);
      if (st == XO_OK)
        st = topk_scan(metric, (int64_t)pos.size(), k, radius, bitmap, keys, pos.data(),
                       [&](int64_t p, float* s) {
                         return xo_pq_lookup(table.data(), chunks, codes + p * chunks, s);
                       },
                       &res);
    }
    status[q] = st;
    if (st != XO_OK) res.clear();
    write_results(res, k, (int32_t)q, out_keys, out_scores, out_counts);
  });
  int first = XO_OK;
  for (int32_t q = 0; q < nq; ++q) {
    if (out_status) out_status[q] = status[q];
    if (first == XO_OK) first = status[q];
  }
  return first;
}

// ---------------------------------------------------------------------------
// RaBitQ: FHT rotation (rotation.go:123-153, fht.go:28-101) and the 1-bit
// estimator (rabitq.go, rabitq_quantize.go).
// ---------------------------------------------------------------------------
namespace {
// FHTFlipSigns (fht.go:28-39).
void fht_flip(const uint8_t* signs, float* data, int32_t n) {
  for (int32_t i = 0; i < n; ++i)
    if (signs[i / 8] & (1u << (i % 8))) data[i] = -data[i];
}
// FHTInPlace (fht.go:41-57).
void fht_inplace(float* data, int32_t n) {
  for (int32_t w = 1; w < n; w <<= 1)
    for (int32_t b = 0; b < n; b += w << 1)
      for (int32_t i = b; i < b + w; ++i) {
        float l = data[i], r = data[i + w];
        data[i] = l + r;
        data[i + w] = l - r;
      }
}
// FHTKacWalk (fht.go:59-76).
void fht_kac(float* data, int32_t n) {
  int32_t half = n / 2, base = n % 2, off = base + half;
  for (int32_t i = 0; i < half; ++i) {
    float l = data[i], r = data[i + off];
    data[i] = l + r;
    data[i + off] = l - r;
  }
  if (base != 0) data[half] *= (float)std::sqrt(2.0);
}
void scale(float* data, int32_t n, float f) {  // ScaleFloat32 (fht.go:97-101)
  for (int32_t i = 0; i < n; ++i) data[i] *= f;
}
int32_t floor_pow2(int32_t v) {  // floorPowerOfTwo (rotation.go:239-245)
  int32_t r = 1;
  while (r <= v / 2) r *= 2;
  return r;
}
// FHTRotator.Rotate (rotation.go:123-153) for a rotator of `dimension` whose
// FHT window is `truncated` (newRaBitQPaddedRotator sets truncated from the
// unpadded dimension, rabitq.go:555-567).
int rotate(int32_t dimension, int32_t truncated, const uint8_t* signs, const float* in, float* out) {
  int32_t bpr = (dimension + 7) / 8;
  float inv = 1.0f / (float)std::sqrt((double)(float)truncated);
  std::memcpy(out, in, sizeof(float) * dimension);
  for (int32_t i = 0; i < dimension; ++i)
    if (!finite32(in[i])) return XO_NON_FINITE;
  if (truncated == dimension) {
    for (int r = 0; r < 4; ++r) {
      fht_flip(signs + r * bpr, out, dimension);
      fht_inplace(out, dimension);
      scale(out, dimension, inv);
    }
  } else {
    int32_t start = dimension - truncated;
    for (int r = 0; r < 4; ++r) {
      fht_flip(signs + r * bpr, out, dimension);
      float* window = (r % 2 != 0) ? out + start : out;
      fht_inplace(window, truncated);
      scale(window, truncated, inv);
      fht_kac(out, dimension);
    }
    scale(out, dimension, 0.25f);
  }
  for (int32_t i = 0; i < dimension; ++i)
    if (!finite32(out[i])) return XO_NON_FINITE;
  return XO_OK;
}
}  // namespace

extern "C" int xo_fht_rotate(int32_t dimension, const uint8_t* signs, const float* in, float* out) {
  if (dimension <= 0) return XO_INVALID_ARGUMENT;
  return rotate(dimension, floor_pow2(dimension), signs, in, out);
}

namespace {
// FHTInverseKacWalk (fht.go:78-94).
void fht_inverse_kac(float* data, int32_t n) {
  int32_t half = n / 2, base = n % 2, off = base + half;
  if (base != 0) data[half] *= (float)std::sqrt(0.5);
  for (int32_t i = 0; i < half; ++i) {
    float l = data[i], r = data[i + off];
    data[i] = (l + r) * 0.5f;
    data[i + off] = (l - r) * 0.5f;
  }
}
}  // namespace

// FHTRotator.Unrotate (rotation.go:155-185): the rounds of Rotate undone in
// reverse order.
extern "C" int xo_fht_unrotate(int32_t dimension, const uint8_t* signs, const float* in,
                               float* out) {
  if (dimension <= 0) return XO_INVALID_ARGUMENT;
  const int32_t truncated = floor_pow2(dimension);
  const int32_t bpr = (dimension + 7) / 8;
  const float inv = 1.0f / (float)std::sqrt((double)(float)truncated);
  for (int32_t i = 0; i < dimension; ++i)
    if (!finite32(in[i])) return XO_NON_FINITE;
  std::memcpy(out, in, sizeof(float) * dimension);
  if (truncated == dimension) {
    for (int r = 3; r >= 0; --r) {
      fht_inplace(out, dimension);
      scale(out, dimension, inv);
      fht_flip(signs + r * bpr, out, dimension);
    }
  } else {
    scale(out, dimension, 4.0f);
    const int32_t start = dimension - truncated;
    for (int r = 3; r >= 0; --r) {
      fht_inverse_kac(out, dimension);
      float* window = (r % 2 != 0) ? out + start : out;
      fht_inplace(window, truncated);
      scale(window, truncated, inv);
      fht_flip(signs + r * bpr, out, dimension);
    }
  }
  for (int32_t i = 0; i < dimension; ++i)
    if (!finite32(out[i])) return XO_NON_FINITE;
  return XO_OK;
}

// roundUpRaBitQDimension (rabitq.go:579-581).
extern "C" int32_t xo_rabitq_padded_dimension(int32_t d) { return (d + 63) / 64 * 64; }

// rotateRaBitQVector (rabitq.go:570-577) with newRaBitQPaddedRotator.
extern "C" int xo_rabitq_rotate(int32_t d, const uint8_t* signs, const float* in, float* out) {
  int32_t padded = xo_rabitq_padded_dimension(d);
  std::vector<float> tmp(padded, 0.0f);
  std::memcpy(tmp.data(), in, sizeof(float) * d);
  return rotate(padded, floor_pow2(d), signs, tmp.data(), out);
}

namespace {
// raBitQFactors (rabitq_quantize.go:210-262).
int rabitq_factors(const std::vector<double>& residual, const float* centroid,
                   const std::vector<uint16_t>& values, int levels_bits, bool ip, double* add,
                   double* rescale, double* err) {
  size_t n = residual.size();
  if (n < 2) return XO_INVALID_ARGUMENT;
  double center = -((double)(1ULL << levels_bits) - 1) / 2;
  double ns = 0, cns = 0, rcd = 0, ccd = 0, rcent = 0;
  for (size_t i = 0; i < n; ++i) {
    double cc = (double)values[i] + center;
    double rv = residual[i];
    ns += rv * rv;
    cns += cc * cc;
    rcd += rv * cc;
    ccd += (double)centroid[i] * cc;
    rcent += rv * (double)centroid[i];
  }
  if (ns == 0) {
    *add = ip ? 1 : 0;
    *rescale = 0;
    *err = 0;
    return XO_OK;
  }
  if (rcd <= 0 || std::isnan(rcd) || std::isinf(rcd)) return XO_INVALID_ARGUMENT;
  double ratio = ns * cns / (rcd * rcd) - 1;
  if (ratio < 0 && ratio > -1e-12) ratio = 0;
  if (ratio < 0 || std::isnan(ratio) || std::isinf(ratio)) return XO_INVALID_ARGUMENT;
  double norm = std::sqrt(ns);
  double te = norm * 1.9 * std::sqrt(ratio / (double)(n - 1));
  if (ip) {
    *add = 1 - rcent + ns * ccd / rcd;
    *rescale = -ns / rcd;
    *err = te;
  } else {
    *add = ns + 2 * ns * ccd / rcd;
    *rescale = -2 * ns / rcd;
    *err = 2 * te;
  }
  if (!std::isfinite(*add) || !std::isfinite(*rescale) || !std::isfinite(*err)) return XO_OVERFLOW;
  return XO_OK;
}
}  // namespace

// quantizeRaBitQVector (rabitq_quantize.go:99-200).
extern "C" int xo_rabitq_quantize(const float* vec, const float* cen, int32_t padded,
                                  int32_t cluster, int32_t total_bits, double extra_scale,
                                  int32_t inner_product, uint8_t* binary_code, uint8_t* extra_code,
                                  xo_rabitq_factors* f) {
  if (padded <= 0 || padded % 64 != 0 || total_bits < 1 || total_bits > 9 || cluster < 0)
    return XO_INVALID_ARGUMENT;
  int extra_bits = total_bits - 1;
  std::vector<double> residual(padded);
  std::vector<uint16_t> bin(padded, 0);
  std::memset(binary_code, 0, padded / 8);
  double rns = 0;
  for (int32_t i = 0; i < padded; ++i) {
    if (!finite32(vec[i]) || !finite32(cen[i])) return XO_NON_FINITE;
    double v = (double)vec[i] - (double)cen[i];
    residual[i] = v;
    rns += v * v;
    if (v > 0) {
      bin[i] = 1;
      binary_code[i / 8] |= (uint8_t)(1u << (i % 8));
    }
  }
  f->cluster = cluster;
  int st = rabitq_factors(residual, cen, bin, 1, inner_product != 0, &f->coarse_add,
                          &f->coarse_rescale, &f->coarse_error);
  if (st != XO_OK) return st;
  if (extra_bits == 0) {
    f->full_add = f->coarse_add;
    f->full_rescale = f->coarse_rescale;
    return XO_OK;
  }
  double norm = std::sqrt(rns);
  std::vector<uint16_t> extra(padded, 0), factor_values(padded, 0);
  uint16_t max_extra = (uint16_t)((1u << extra_bits) - 1);
  double inv_ip = 1;
  if (norm > 0) {
    double ipn = 0;
    for (int32_t i = 0; i < padded; ++i) {
      double an = std::fabs(residual[i]) / norm;
      int qv = (int)(extra_scale * an + 1e-5);
      if (qv < 0) qv = 0;
      if (qv > (int)max_extra) qv = max_extra;
      ipn += ((double)qv + .5) * an;
      uint16_t e = (uint16_t)qv;
      if (residual[i] < 0) e = max_extra - e;
      extra[i] = e;
      uint16_t fs = residual[i] >= 0 ? 1 : 0;
      factor_values[i] = (uint16_t)(e | (fs << extra_bits));
    }
    if (ipn > 0 && std::isfinite(ipn)) inv_ip = 1 / ipn;
  }
  // packRaBitQValues (rabitq_quantize.go:265-280).
  size_t packed_len = ((size_t)padded * extra_bits + 7) / 8;
  std::memset(extra_code, 0, packed_len);
  for (int32_t i = 0; i < padded; ++i)
    for (int b = 0; b < extra_bits; ++b)
      if (extra[i] & (1u << b)) {
        size_t p = (size_t)i * extra_bits + b;
        extra_code[p / 8] |= (uint8_t)(1u << (p % 8));
      }
  double dummy;
  st = rabitq_factors(residual, cen, factor_values, total_bits, inner_product != 0, &f->full_add,
                      &f->full_rescale, &dummy);
  if (st != XO_OK) return st;
  f->full_rescale = inner_product ? -norm * inv_ip : -2 * norm * inv_ip;
  return XO_OK;
}

namespace {
// prepareRaBitQVector / normalizeRaBitQVector (rabitq.go:503-526).
std::vector<float> prepare_vector(const float* v, int32_t d, int metric) {
  std::vector<float> out(v, v + d);
  if (metric == XO_COSINE) {
    double ns = 0;
    for (int32_t i = 0; i < d; ++i) ns += (double)out[i] * (double)out[i];
    if (ns != 0) {
      float inv = (float)(1 / std::sqrt(ns));
      for (int32_t i = 0; i < d; ++i) out[i] *= inv;
    }
  }
  return out;
}
}  // namespace

// RaBitQModel.Encode (rabitq.go:297-327): nearest centroid under L2 (IP for
// IP/cosine), rotate, quantize against the rotated centroid with the model's
// TotalBits and ExtraScale (RestoreRaBitQModel rotates centroids,
// rabitq.go:224-230).  extra_code: (padded (total_bits - 1) + 7) / 8 bytes.
extern "C" int xo_rabitq_encode(int metric, int32_t d, const float* centroids, int32_t nc,
                                const uint8_t* signs, int32_t total_bits, double extra_scale,
                                const float* v, uint8_t* binary_code, uint8_t* extra_code,
                                xo_rabitq_factors* f) {
  for (int32_t i = 0; i < d; ++i)
    if (!finite32(v[i])) return XO_NON_FINITE;
  std::vector<float> prepared = prepare_vector(v, d, metric);
  int cmetric = metric == XO_COSINE ? XO_IP : metric;
  int32_t cluster;
  float s;
  int st = nearest_centroid(cmetric, centroids, nc, d, prepared.data(), &cluster, &s);
  if (st != XO_OK) return st;
  int32_t padded = xo_rabitq_padded_dimension(d);
  std::vector<float> rot(padded), rcen(padded);
  st = xo_rabitq_rotate(d, signs, prepared.data(), rot.data());
  if (st != XO_OK) return st;
  st = xo_rabitq_rotate(d, signs, centroids + (int64_t)cluster * d, rcen.data());
  if (st != XO_OK) return st;
  return xo_rabitq_quantize(rot.data(), rcen.data(), padded, cluster, total_bits, extra_scale,
                            metric != XO_L2, binary_code, extra_code, f);
}

// The TotalBits = 1 encoding.
extern "C" int xo_rabitq_encode1(int metric, int32_t d, const float* centroids, int32_t nc,
                                 const uint8_t* signs, const float* v, uint8_t* binary_code,
                                 xo_rabitq_factors* f) {
  return xo_rabitq_encode(metric, d, centroids, nc, signs, 1, 0, v, binary_code, nullptr, f);
}

// PrepareQuery (rabitq.go:372-408).
extern "C" int xo_rabitq_prepare_query(int metric, int32_t d, const float* centroids, int32_t nc,
                                       const uint8_t* signs, const float* query, float* rotated,
                                       double* sum, double* g_add, double* g_error) {
  for (int32_t i = 0; i < d; ++i)
    if (!finite32(query[i])) return XO_NON_FINITE;
  std::vector<float> prepared = prepare_vector(query, d, metric);
  int32_t padded = xo_rabitq_padded_dimension(d);
  int st = xo_rabitq_rotate(d, signs, prepared.data(), rotated);
  if (st != XO_OK) return st;
  double s = 0;
  for (int32_t i = 0; i < padded; ++i) s += (double)rotated[i];
  *sum = s;
  std::vector<float> rc(padded);
  for (int32_t c = 0; c < nc; ++c) {
    st = xo_rabitq_rotate(d, signs, centroids + (int64_t)c * d, rc.data());
    if (st != XO_OK) return st;
    double sq = 0, dot = 0;
    for (int32_t i = 0; i < padded; ++i) {
      double diff = (double)rotated[i] - (double)rc[i];
      sq += diff * diff;
      dot += (double)rotated[i] * (double)rc[i];
    }
    g_error[c] = std::sqrt(sq);
    g_add[c] = metric == XO_L2 ? sq : -dot;
  }
  return XO_OK;
}

// EstimateCoarse (rabitq.go:421-430), raBitQBinaryDot (rabitq_quantize.go:
// 302-310) and makeRaBitQEstimate (rabitq.go:464-476); g_error may be null
// (then the error bound is taken as 0).
extern "C" int xo_rabitq_estimate_coarse(const float* rotated, int32_t padded, double sum,
                                         const double* g_add, const double* g_error,
                                         const uint8_t* bits, const xo_rabitq_factors* f,
                                         float* distance) {
  double dot = 0;
  for (int32_t i = 0; i < padded; ++i)
    if (bits[i / 8] & (1u << (i % 8))) dot += (double)rotated[i];
  double centered = dot - .5 * sum;
  double dist = f->coarse_add + g_add[f->cluster] + f->coarse_rescale * centered;
  double eb = g_error ? f->coarse_error * g_error[f->cluster] : 0.0;
  const double maxf = 3.40282346638528859811704183484516925440e+38;
  if (std::isnan(dist) || std::isinf(dist) || std::isnan(eb) || std::isinf(eb) || eb < 0)
    return XO_INVALID_ARGUMENT;
  if (std::fabs(dist) > maxf || eb > maxf) return XO_OVERFLOW;
  if (dist - eb < -maxf || dist + eb > maxf) return XO_OVERFLOW;
  *distance = (float)dist;
  return XO_OK;
}

// Estimate (rabitq.go:434-446): EstimateCoarse for one bit, else the full
// code dot raBitQFullCodeDot (rabitq_quantize.go:312-323: value = extra |
// sign bit << extra bits, float64 products summed in index order) with
// center -(2^extra - 1/2), and the coarse error over 2^extra.
extern "C" int xo_rabitq_estimate(const float* rotated, int32_t padded, double sum,
                                  const double* g_add, const double* g_error, int32_t total_bits,
                                  const uint8_t* bits, const uint8_t* extra,
                                  const xo_rabitq_factors* f, float* distance) {
  if (total_bits <= 1)
    return xo_rabitq_estimate_coarse(rotated, padded, sum, g_add, g_error, bits, f, distance);
  const int eb = total_bits - 1;
  double dot = 0;
  for (int32_t i = 0; i < padded; ++i) {
    uint32_t q = 0;
    for (int b = 0; b < eb; ++b) {
      const size_t p = (size_t)i * eb + b;
      if (extra[p / 8] & (1u << (p % 8))) q |= 1u << b;
    }
    if (bits[i / 8] & (1u << (i % 8))) q |= 1u << eb;
    dot += (double)q * (double)rotated[i];
  }
  const double center = -((double)(1ull << eb) - .5);
  double dist = f->full_add + g_add[f->cluster] + f->full_rescale * (dot + center * sum);
  double eb_err = g_error ? f->coarse_error * g_error[f->cluster] / (double)(1ull << eb) : 0.0;
  const double maxf = 3.40282346638528859811704183484516925440e+38;
  if (std::isnan(dist) || std::isinf(dist) || std::isnan(eb_err) || std::isinf(eb_err) ||
      eb_err < 0)
    return XO_INVALID_ARGUMENT;
  if (std::fabs(dist) > maxf || eb_err > maxf) return XO_OVERFLOW;
  if (dist - eb_err < -maxf || dist + eb_err > maxf) return XO_OVERFLOW;
  *distance = (float)dist;
  return XO_OK;
}

// Composed RaBitQ linear search (hnsw_rabitq.go:539-586) over every code
// (scanRaBitQCodes, :615-642: first failing estimate fails the query, then
// acceptRaBitQNode :753-757, filter and radius on the public score, and a
// heap with raBitQNodeBetter :739-744, lower estimate, ties to the lower key).
//   refine != 0: the scan keeps min(n, candidate_count) estimates without the
//     radius (:579-584) and refinePrepared (:780-801) returns the exact fp32
//     top-k of those (metric.Compute on the originals, query validated first).
//   refine == 0: the k best estimates with publicRaBitQScore (:746-751).
// total_bits > 1: Estimate on the full codes (extra_codes: per row
// (padded (total_bits - 1) + 7) / 8 bytes).
extern "C" int xo_rabitq_search_bits(int metric, int32_t d, const float* centroids, int32_t nc,
                                     const uint8_t* signs, int32_t total_bits,
                                     const uint8_t* binary_codes, const uint8_t* extra_codes,
                                     const xo_rabitq_factors* factors, const float* originals,
                                     const uint64_t* keys, int64_t n, const float* queries,
                                     int32_t nq, int32_t k, int32_t candidate_count,
                                     int32_t refine, float radius, const uint32_t* bitmap,
                                     int32_t threads, uint64_t* out_keys, float* out_scores,
                                     int32_t* out_counts, int32_t* out_status) {
  int st0 = validate_options(k, radius);
  if (st0 != XO_OK) return st0;
  if (total_bits < 1 || total_bits > 9) return XO_INVALID_ARGUMENT;
  int32_t padded = xo_rabitq_padded_dimension(d);
  int32_t bytes = padded / 8;
  const int64_t xbytes = ((int64_t)padded * (total_bits - 1) + 7) / 8;
  std::vector<int32_t> status(nq, XO_OK);
  auto public_score = [&](float dist) { return metric == XO_IP ? 1.0f - dist : dist; };
  parallel_for(nq, threads, [&](int64_t q) {
    const float* query = queries + q * d;
    std::vector<float> rot(padded);
    std::vector<double> gadd(nc), gerr(nc);
    double sum;
    int st = xo_rabitq_prepare_query(metric, d, centroids, nc, signs, query, rot.data(), &sum,
                                     gadd.data(), gerr.data());
    std::vector<Result> res;
    if (st == XO_OK && n > 0) {
      int32_t cc = refine ? (int32_t)std::min<int64_t>(n, std::max(k, candidate_count)) : k;
      // Estimates rank lower-is-better for every metric: the L2 heap order.
      WorstFirstHeap heap{XO_L2, {}};
      for (int64_t p = 0; p < n && st == XO_OK; ++p) {
        float est;
        st = xo_rabitq_estimate(rot.data(), padded, sum, gadd.data(), gerr.data(), total_bits,
                                binary_codes + p * bytes,
                                total_bits > 1 ? extra_codes + p * xbytes : nullptr, &factors[p],
                                &est);
        if (st != XO_OK) break;
        if (!filter_pass(bitmap, p)) continue;
        if (!refine && !within_radius(metric, public_score(est), radius)) continue;
        heap.offer(Result{keys[p], est}, (size_t)cc);
      }
      if (st == XO_OK) {
        std::vector<Result> cands = heap.sorted();
        if (!refine) {
          for (auto& r : cands) r.score = public_score(r.score);
          res = cands;
        } else {
          std::vector<int64_t> cpos(cands.size());
          for (size_t i = 0; i < cands.size(); ++i) {
            int64_t pos = -1;
            for (int64_t pp = 0; pp < n; ++pp)
              if (keys[pp] == cands[i].key) {
                pos = pp;
                break;
              }
            cpos[i] = pos;
          }
          st = validate_query(metric, query, d);
          if (st == XO_OK)
            st = topk_scan(metric, (int64_t)cpos.size(), k, radius, nullptr, keys, cpos.data(),
                           [&](int64_t pos, float* s) {
                             return prevalidated(metric, originals + pos * d, query, d, s);
                           },
                           &res);
        }
      }
    }
    status[q] = st;
    if (st != XO_OK) res.clear();
    write_results(res, k, (int32_t)q, out_keys, out_scores, out_counts);
  });
  int first = XO_OK;
  for (int32_t q = 0; q < nq; ++q) {
    if (out_status) out_status[q] = status[q];
    if (first == XO_OK) first = status[q];
  }
  return first;
}

extern "C" int xo_rabitq_search(int metric, int32_t d, const float* centroids, int32_t nc,
                                const uint8_t* signs, const uint8_t* binary_codes,
                                const xo_rabitq_factors* factors, const float* originals,
                                const uint64_t* keys, int64_t n, const float* queries, int32_t nq,
                                int32_t k, int32_t candidate_count, int32_t refine, float radius,
                                const uint32_t* bitmap, int32_t threads, uint64_t* out_keys,
                                float* out_scores, int32_t* out_counts, int32_t* out_status) {
  return xo_rabitq_search_bits(metric, d, centroids, nc, signs, 1, binary_codes, nullptr, factors,
                               originals, keys, n, queries, nq, k, candidate_count, refine,
                               radius, bitmap, threads, out_keys, out_scores, out_counts,
                               out_status);
}

// ---------------------------------------------------------------------------
// HNSW-RaBitQ graph search (hnsw_rabitq.go:589-612 searchPrepared, :644-671
// searchRaBitQLayer, :673-737 searchRaBitQBase, :739-757 node order and
// acceptance, :780-801 refinePrepared) over a given graph.  The graph: levels
// 0..max_level, node p's level-L neighbours at
// neighbors[offsets[L (n + 1) + p] .. offsets[L (n + 1) + p + 1]).
// ---------------------------------------------------------------------------
namespace {
struct GraphNode {
  float score;
  uint64_t key;
  int64_t pos;
};
// raBitQNodeBetter (:739-744): lower estimate, ties to the lower key.
inline bool node_better(const GraphNode& a, const GraphNode& b) {
  if (a.score == b.score) return a.key < b.key;
  return a.score < b.score;
}
struct BestOnTop {
  bool operator()(const GraphNode& a, const GraphNode& b) const { return node_better(b, a); }
};
struct WorstOnTop {
  bool operator()(const GraphNode& a, const GraphNode& b) const { return node_better(a, b); }
};
// EstimateCoarse with its lower bound (rabitq.go:421-430, 464-476).
int coarse_with_lower(const float* rot, int32_t padded, double sum, const double* gadd,
                      const double* gerr, const uint8_t* bits, const xo_rabitq_factors* f,
                      float* dist, float* lower) {
  double dot = 0;
  for (int32_t i = 0; i < padded; ++i)
    if (bits[i / 8] & (1u << (i % 8))) dot += (double)rot[i];
  const double centered = dot - .5 * sum;
  const double d = f->coarse_add + gadd[f->cluster] + f->coarse_rescale * centered;
  const double eb = f->coarse_error * gerr[f->cluster];
  const double maxf = 3.40282346638528859811704183484516925440e+38;
  if (std::isnan(d) || std::isinf(d) || std::isnan(eb) || std::isinf(eb) || eb < 0)
    return XO_INVALID_ARGUMENT;
  if (std::fabs(d) > maxf || eb > maxf) return XO_OVERFLOW;
  if (d - eb < -maxf || d + eb > maxf) return XO_OVERFLOW;
  *dist = (float)d;
  *lower = (float)(d - eb);
  return XO_OK;
}
}  // namespace

extern "C" int xo_hnsw_rabitq_search(
    int metric, int32_t d, const float* centroids, int32_t nc, const uint8_t* signs,
    int32_t total_bits, const uint8_t* binary_codes, const uint8_t* extra_codes,
    const xo_rabitq_factors* factors, const float* originals, const uint64_t* keys, int64_t n,
    int32_t max_level, int64_t entry, const int64_t* offsets, const int32_t* neighbors,
    const float* queries, int32_t nq, int32_t k, int32_t ef, int32_t refine, float radius,
    const uint32_t* bitmap, int32_t threads, uint64_t* out_keys, float* out_scores,
    int32_t* out_counts, int32_t* out_status) {
  int st0 = validate_options(k, radius);
  if (st0 != XO_OK) return st0;
  if (ef <= 0 || ef > 2048) return XO_INVALID_ARGUMENT;
  const int32_t padded = xo_rabitq_padded_dimension(d);
  const int32_t bytes = padded / 8;
  const int64_t xbytes = ((int64_t)padded * (total_bits - 1) + 7) / 8;
  std::vector<int32_t> status(nq, XO_OK);
  auto public_score = [&](float dist) { return metric == XO_IP ? 1.0f - dist : dist; };
  parallel_for(nq, threads, [&](int64_t q) {
    const float* query = queries + q * d;
    std::vector<float> rot(padded);
    std::vector<double> gadd(nc), gerr(nc);
    double sum;
    int st = xo_rabitq_prepare_query(metric, d, centroids, nc, signs, query, rot.data(), &sum,
                                     gadd.data(), gerr.data());
    std::vector<Result> res;
    auto full = [&](int64_t p, float* dist) {
      return xo_rabitq_estimate(rot.data(), padded, sum, gadd.data(), gerr.data(), total_bits,
                                binary_codes + p * bytes,
                                total_bits > 1 ? extra_codes + p * xbytes : nullptr,
                                &factors[p], dist);
    };
    auto coarse = [&](int64_t p, float* dist, float* lower) {
      return coarse_with_lower(rot.data(), padded, sum, gadd.data(), gerr.data(),
                               binary_codes + p * bytes, &factors[p], dist, lower);
    };
    if (st == XO_OK && n > 0) {
      // The approximate stage's size: candidateCount with refine (:579),
      // else TopK; the base layer keeps max(ef, that).
      const int64_t top = refine ? std::min<int64_t>(n, std::max(k, ef)) : k;
      const int64_t capacity = std::max<int64_t>(ef, top);
      // acceptRaBitQNode (:753-757): the filter, and without refine the radius
      // on the public score.
      auto accept = [&](const GraphNode& v) {
        if (!filter_pass(bitmap, v.pos)) return false;
        return refine ? true : within_radius(metric, public_score(v.score), radius);
      };
      // searchRaBitQLayer on levels max_level .. 1 (coarse estimates).
      int64_t cur = entry;
      float cur_dist = 0, lo = 0;
      for (int32_t level = max_level; level > 0 && st == XO_OK; --level) {
        st = coarse(cur, &cur_dist, &lo);
        bool changed = true;
        while (st == XO_OK && changed) {
          changed = false;
          // Go's range takes the list of the node the pass starts from, even
          // when the pass moves on to a neighbour.
          const int64_t* off = offsets + (int64_t)level * (n + 1);
          const int64_t first = off[cur], last = off[cur + 1];
          for (int64_t e = first; e < last && st == XO_OK; ++e) {
            const int64_t nb = neighbors[e];
            float cd, cl;
            st = coarse(nb, &cd, &cl);
            if (st != XO_OK) break;
            if (cd < cur_dist || (cd == cur_dist && nb < cur)) {
              cur = nb;
              cur_dist = cd;
              changed = true;
            }
          }
        }
      }
      std::vector<GraphNode> nodes;
      if (st == XO_OK) {
        // searchRaBitQBase (:673-737).
        std::vector<uint8_t> visited((size_t)n, 0);
        std::priority_queue<GraphNode, std::vector<GraphNode>, BestOnTop> frontier;
        std::priority_queue<GraphNode, std::vector<GraphNode>, WorstOnTop> accepted;
        float sd;
        st = full(cur, &sd);
        if (st == XO_OK) {
          GraphNode start{sd, keys[cur], cur};
          visited[cur] = 1;
          frontier.push(start);
          if (accept(start)) accepted.push(start);
          const int64_t* off0 = offsets;
          while (!frontier.empty() && st == XO_OK) {
            GraphNode c = frontier.top();
            frontier.pop();
            if ((int64_t)accepted.size() >= capacity && !accepted.empty() &&
                node_better(accepted.top(), c))
              break;
            for (int64_t e = off0[c.pos]; e < off0[c.pos + 1]; ++e) {
              const int64_t nb = neighbors[e];
              if (visited[nb]) continue;
              visited[nb] = 1;
              float cd, cl;
              st = coarse(nb, &cd, &cl);
              if (st != XO_OK) break;
              if ((int64_t)accepted.size() >= capacity && !accepted.empty() &&
                  cl >= accepted.top().score)
                continue;
              float fd;
              st = full(nb, &fd);
              if (st != XO_OK) break;
              GraphNode v{fd, keys[nb], nb};
              if ((int64_t)accepted.size() < capacity || accepted.empty() ||
                  node_better(v, accepted.top())) {
                frontier.push(v);
                if (accept(v)) {
                  accepted.push(v);
                  if ((int64_t)accepted.size() > capacity) accepted.pop();
                }
              }
            }
          }
        }
        while (!accepted.empty()) {
          nodes.push_back(accepted.top());
          accepted.pop();
        }
        std::reverse(nodes.begin(), nodes.end());  // best first
        if ((int64_t)nodes.size() > top) nodes.resize((size_t)top);
      }
      if (st == XO_OK) {
        if (!refine) {
          for (auto& v : nodes) res.push_back(Result{v.key, public_score(v.score)});
        } else {
          // refinePrepared: exact fp32 top-k of the candidates' originals.
          std::vector<int64_t> cpos;
          for (auto& v : nodes) cpos.push_back(v.pos);
          st = validate_query(metric, query, d);
          if (st == XO_OK)
            st = topk_scan(metric, (int64_t)cpos.size(), k, radius, nullptr, keys, cpos.data(),
                           [&](int64_t pos, float* s) {
                             return prevalidated(metric, originals + pos * d, query, d, s);
                           },
                           &res);
        }
      }
    }
    status[q] = st;
    if (st != XO_OK) res.clear();
    write_results(res, k, (int32_t)q, out_keys, out_scores, out_counts);
  });
  int first = XO_OK;
  for (int32_t q = 0; q < nq; ++q) {
    if (out_status) out_status[q] = status[q];
    if (first == XO_OK) first = status[q];
  }
  return first;
}

// ---------------------------------------------------------------------------
// DiskANN graph search with the PQ frontier (DiskANNIndex.searchDiskANNGraph,
// diskann.go:559-651; diskANNApproximateScore :653-683) over a given graph:
// node p's neighbours at neighbors[offsets[p] .. offsets[p + 1]), node p's
// vector at vectors[p d], its PQ code (of the prepared vector, under the
// traversal metric) at codes[p chunks].
// ---------------------------------------------------------------------------
namespace {
struct DiskNode {
  float score;
  uint32_t id;
};
// diskANNTraversalMetric (diskann.go:276-281).
inline int diskann_traversal(int metric) {
  return (metric == XO_COSINE || metric == XO_MIPSL2) ? XO_L2 : metric;
}
// The queue order of searchDiskANNGraph (:571-576): the traversal metric's
// Better, ties to the lower node id.
struct DiskBetter {
  int traversal;
  bool operator()(const DiskNode& a, const DiskNode& b) const {
    if (a.score == b.score) return a.id < b.id;
    return better(traversal, a.score, b.score);
  }
};
}  // namespace

// diskANNPQCodeNorms (diskann.go:292-323): per code, the float64 sum of the
// squares of its pivots' chunk components in chunk order, as float32.
extern "C" void xo_diskann_code_norms(const float* pivots, const int32_t* offsets, int32_t chunks,
                                      int32_t d, const uint8_t* codes, int64_t n, float* norms) {
  for (int64_t p = 0; p < n; ++p) {
    double norm = 0;
    for (int32_t c = 0; c < chunks; ++c) {
      const float* pv = pivots + (int64_t)codes[p * chunks + c] * d;
      for (int32_t i = offsets[c]; i < offsets[c + 1]; ++i) norm += (double)pv[i] * (double)pv[i];
    }
    norms[p] = (float)norm;
  }
}

// diskANNApproximateScore (diskann.go:653-676).
static int diskann_approx(int metric, const float* table, int32_t chunks, const uint8_t* codes,
                          const float* code_norms, uint32_t id, double query_norm, float* out) {
  float score;
  int st = xo_pq_lookup(table, chunks, codes + (int64_t)id * chunks, &score);
  if (st != XO_OK) return st;
  if (metric != XO_MIPSL2) {
    *out = score;
    return XO_OK;
  }
  const double cn = (double)code_norms[id];
  const double inner = (query_norm + cn - (double)score) / 2;
  const double den = go_maxd(query_norm, cn);
  if (den == 0) {
    *out = 0;
    return XO_OK;
  }
  const double converted = 2 - 2 * inner / den;
  if (std::isnan(converted) || std::isinf(converted) || converted > 3.4028234663852886e38 ||
      converted < -3.4028234663852886e38)
    return XO_OVERFLOW;
  *out = (float)converted;
  return XO_OK;
}

// DiskANNIndex.SearchDiskANN (diskann.go:472-525) with Linear = false:
// validation, then searchDiskANNGraph; `beam` is diskANNReadBatchSize
// (:685-691).
extern "C" int xo_diskann_search(int metric, int32_t d, const float* pivots,
                                 const int32_t* offsets, int32_t chunks, const uint8_t* codes,
                                 const float* code_norms, const float* vectors,
                                 const uint64_t* keys, int64_t n, int64_t entry,
                                 const int64_t* graph_offsets, const int32_t* neighbors,
                                 int32_t beam, const float* queries, int32_t nq, int32_t k,
                                 int32_t list_size, float radius, const uint32_t* bitmap,
                                 int32_t threads, uint64_t* out_keys, float* out_scores,
                                 int32_t* out_counts, int32_t* out_status) {
  if (list_size <= 0) return XO_INVALID_ARGUMENT;  // ErrInvalidDiskANNListSize
  int st0 = validate_options(k, radius);
  if (st0 != XO_OK) return st0;
  if (beam <= 0) return XO_INVALID_ARGUMENT;
  const int traversal = diskann_traversal(metric);
  const DiskBetter node_better{traversal};
  std::vector<int32_t> status(nq, XO_OK);
  parallel_for(nq, threads, [&](int64_t q) {
    const float* query = queries + q * d;
    std::vector<Result> res;
    int st = validate_query(metric, query, d);
    if (st == XO_OK && n > 0) {
      // prepareDiskANNPQQuery (:283-289), the table, diskANNVectorNormSquared.
      std::vector<float> prepared = prepare_vector(query, d, metric);
      std::vector<float> table((size_t)chunks * 256);
      st = xo_pq_distance_table(traversal, pivots, offsets, chunks, d, prepared.data(),
                                table.data());
      double qnorm = 0;
      for (int32_t i = 0; i < d; ++i) qnorm += (double)prepared[i] * (double)prepared[i];
      const int64_t capacity = std::min<int64_t>(n, std::max(k, list_size));
      auto approx = [&](uint32_t id, float* s) {
        return diskann_approx(metric, table.data(), chunks, codes, code_norms, id, qnorm, s);
      };
      // frontier: best on top; retained: worst on top.
      auto best_top = [&](const DiskNode& a, const DiskNode& b) { return node_better(b, a); };
      auto worst_top = [&](const DiskNode& a, const DiskNode& b) { return node_better(a, b); };
      std::priority_queue<DiskNode, std::vector<DiskNode>, decltype(best_top)> frontier(best_top);
      std::priority_queue<DiskNode, std::vector<DiskNode>, decltype(worst_top)> retained(
          worst_top);
      std::vector<uint8_t> visited((size_t)n, 0), member((size_t)n, 0), expanded((size_t)n, 0);
      WorstFirstHeap collector{metric, {}};
      float es = 0;
      if (st == XO_OK) st = approx((uint32_t)entry, &es);
      if (st == XO_OK) {
        const DiskNode start{es, (uint32_t)entry};
        frontier.push(start);
        retained.push(start);
        visited[entry] = member[entry] = 1;
      }
      while (st == XO_OK && !frontier.empty()) {
        std::vector<DiskNode> batch;
        while (!frontier.empty() && (int32_t)batch.size() < beam) {
          const DiskNode c = frontier.top();
          frontier.pop();
          if (!member[c.id] || expanded[c.id]) continue;
          expanded[c.id] = 1;
          batch.push_back(c);
        }
        if (batch.empty()) break;
        for (const DiskNode& node : batch) {
          float exact;
          st = xo_metric_compute(metric, query, vectors + (int64_t)node.id * d, d, &exact);
          if (st != XO_OK) break;
          // diskANNResultCollector.Add (:709-721): filter, radius, top-k.
          if (filter_pass(bitmap, node.id) && within_radius(metric, exact, radius))
            collector.offer(Result{keys[node.id], exact}, (size_t)k);
          for (int64_t e = graph_offsets[node.id]; e < graph_offsets[node.id + 1]; ++e) {
            const uint32_t nb = (uint32_t)neighbors[e];
            if (visited[nb]) continue;
            visited[nb] = 1;
            float s;
            st = approx(nb, &s);
            if (st != XO_OK) break;
            const DiskNode cand{s, nb};
            if ((int64_t)retained.size() < capacity) {
              retained.push(cand);
              member[nb] = 1;
              frontier.push(cand);
              continue;
            }
            if (node_better(cand, retained.top())) {
              member[retained.top().id] = 0;
              retained.pop();
              retained.push(cand);
              member[nb] = 1;
              frontier.push(cand);
            }
          }
          if (st != XO_OK) break;
        }
      }
      if (st == XO_OK) res = collector.sorted();
    }
    status[q] = st;
    if (st != XO_OK) res.clear();
    write_results(res, k, (int32_t)q, out_keys, out_scores, out_counts);
  });
  int first = XO_OK;
  for (int32_t q = 0; q < nq; ++q) {
    if (out_status) out_status[q] = status[q];
    if (first == XO_OK) first = status[q];
  }
  return first;
}

// ---------------------------------------------------------------------------
// Batch encoders for the full-size checks: PQModel.EncodeBatch (pq.go:303-330)
// and RaBitQModel.Encode (rabitq.go:297-327) of n rows over `threads`
// workers; a row's code does not depend on the split.  The first failing
// row's status is returned.
// ---------------------------------------------------------------------------
extern "C" int xo_pq_encode_rows(int metric, const float* pivots, const int32_t* offsets,
                                 int32_t chunks, int32_t d, const float* rows, int64_t n,
                                 int32_t threads, uint8_t* codes) {
  std::vector<int> st(n > 0 ? (size_t)n : 1, XO_OK);
  parallel_for(n, threads, [&](int64_t i) {
    st[i] = xo_pq_encode(metric, pivots, offsets, chunks, d, rows + i * d, codes + i * chunks);
  });
  for (int64_t i = 0; i < n; ++i)
    if (st[i] != XO_OK) return st[i];
  return XO_OK;
}

extern "C" int xo_rabitq_encode_rows(int metric, int32_t d, const float* centroids, int32_t nc,
                                     const uint8_t* signs, int32_t total_bits, double extra_scale,
                                     const float* rows, int64_t n, int32_t threads,
                                     uint8_t* binary_codes, uint8_t* extra_codes,
                                     int64_t extra_stride, xo_rabitq_factors* factors) {
  const int32_t bytes = xo_rabitq_padded_dimension(d) / 8;
  std::vector<int> st(n > 0 ? (size_t)n : 1, XO_OK);
  parallel_for(n, threads, [&](int64_t i) {
    st[i] = xo_rabitq_encode(metric, d, centroids, nc, signs, total_bits, extra_scale,
                             rows + i * d, binary_codes + i * bytes,
                             extra_codes + i * extra_stride, &factors[i]);
  });
  for (int64_t i = 0; i < n; ++i)
    if (st[i] != XO_OK) return st[i];
  return XO_OK;
}
