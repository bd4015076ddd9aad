// ivfpq.cu — IVF list scan over 8-bit PQ codes, and k-means assignment.
//
// The reference has no IVF-PQ type; the path is composed from its parts
// (the same composition the oracle restates in xo_ivfpq_search):
//   probe   probedListsLocked (internal/core/ivf.go:524-561): the nprobe best
//           centroids under the index metric, ties to the lower index.  Done
//           by an internal Flat index over the centroids keyed by centroid
//           index, so the probe is the Flat path (exact, reference order).
//   table   PQModel.DistanceTable (internal/core/pq.go:549-571): per query,
//           chunk-major [chunks][256] of metric.Compute(query chunk, pivot
//           chunk) in the reference's float32 order (thread_reference_sum).
//   scan    PQDistanceTable.Lookup (pq.go:574-595) of every code of every
//           probed list: a float64 sum in chunk order, rounded to float32
//           with the overflow check; filter before scoring, ties by key.
//           The fast scan ranks the codes by a float32 sum (one code per
//           lane, each code's bytes rotated so that the 32 look-ups of a warp
//           hit 32 different shared-memory banks) and the merge rescores
//           the candidates within its error bound with that float64 sum; the
//           exact scan (float64 sums throughout) takes the queries the fast
//           pass cannot settle, and layouts it does not cover.
//   insert  KMeansModel.Nearest (kmeans.go:169-175) for the list and
//           PQModel.Encode (pq.go:274-301) for the code: per chunk the best
//           of the 256 pivots, ties to the lower id.
// The exact scan's scores are the reference scores, so its per-list
// selections are merged in exact mode.
#include <cub/device/device_radix_sort.cuh>
#include <cub/device/device_scan.cuh>

#include <algorithm>
#include <cmath>
#include <utility>
#include <vector>

#include "capi_internal.h"
#include "common.cuh"
#include "flat_kernels.cuh"
#include "index_kernels.cuh"
#include "pipeline.cuh"

namespace xvec {

xvec_gpu_status add_device_locked(xvec_gpu_index* idx, const uint64_t* d_keys, const void* d_rows,
                                  int64_t m, cudaStream_t s);

namespace {

inline unsigned blocks_of(int64_t n, int t = 256) { return (unsigned)((n + t - 1) / t); }
constexpr int kAssignBatch = 131072;  // rows per nearest-centroid search

__global__ void keys_to_labels_kernel(const uint64_t* keys, const int* counts, int64_t n,
                                      int32_t* labels, int* err) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  if (counts[i] != 1) {
    atomicExch(err, counts[i] < 0 ? -counts[i] : XVEC_GPU_INVALID_ARGUMENT);
    labels[i] = 0;
    return;
  }
  labels[i] = (int32_t)keys[i];
}

// PQModel.Encode: block per row, thread per pivot.
__global__ void __launch_bounds__(256) pq_encode_kernel(const float* __restrict__ rows, int64_t n,
                                                        int d, int metric,
                                                        const float* __restrict__ pivots,
                                                        const int* __restrict__ offsets,
                                                        int chunks, uint8_t* __restrict__ codes,
                                                        int* __restrict__ err) {
  const int64_t r = blockIdx.x;
  if (r >= n) return;
  __shared__ float s_score[8];
  __shared__ int s_id[8];
  const int c = threadIdx.x, warp = c >> 5, lane = c & 31;
  const float* x = rows + r * d;
  for (int ch = 0; ch < chunks; ++ch) {
    const int start = offsets[ch], w = offsets[ch + 1] - start;
    float s = metric == kMetricL2 ? thread_reference_sum<0>(x + start, pivots + (int64_t)c * d + start, w)
                                  : thread_reference_sum<1>(x + start, pivots + (int64_t)c * d + start, w);
    if (!finite_f(s)) atomicExch(err, XVEC_GPU_NON_FINITE);
    // Best (metric Better), ties to the lower pivot id.
    int id = c;
    for (int o = 16; o > 0; o >>= 1) {
      const float os = __shfl_xor_sync(kFullMask, s, o);
      const int oid = __shfl_xor_sync(kFullMask, id, o);
      const bool take = metric == kMetricIP ? (os > s || (os == s && oid < id))
                                            : (os < s || (os == s && oid < id));
      if (take) {
        s = os;
        id = oid;
      }
    }
    if (lane == 0) {
      s_score[warp] = s;
      s_id[warp] = id;
    }
    __syncthreads();
    if (c == 0) {
      float bs = s_score[0];
      int bi = s_id[0];
      for (int i = 1; i < 8; ++i) {
        const bool take = metric == kMetricIP ? (s_score[i] > bs || (s_score[i] == bs && s_id[i] < bi))
                                              : (s_score[i] < bs || (s_score[i] == bs && s_id[i] < bi));
        if (take) {
          bs = s_score[i];
          bi = s_id[i];
        }
      }
      codes[r * chunks + ch] = (uint8_t)bi;
    }
    __syncthreads();
  }
}

// PQModel.DistanceTable: block per query, thread per pivot.
__global__ void __launch_bounds__(256) pq_table_kernel(const float* __restrict__ queries, int nq,
                                                       int d, int metric,
                                                       const float* __restrict__ pivots,
                                                       const int* __restrict__ offsets,
                                                       int chunks, float* __restrict__ table,
                                                       int* __restrict__ q_flags) {
  const int q = blockIdx.x;
  const int c = threadIdx.x;
  const float* x = queries + (int64_t)q * d;
  for (int ch = 0; ch < chunks; ++ch) {
    const int start = offsets[ch], w = offsets[ch + 1] - start;
    const float s = metric == kMetricL2
                        ? thread_reference_sum<0>(x + start, pivots + (int64_t)c * d + start, w)
                        : thread_reference_sum<1>(x + start, pivots + (int64_t)c * d + start, w);
    if (!finite_f(s)) atomicOr(&q_flags[q], 4);
    table[((int64_t)q * chunks + ch) * 256 + c] = s;
  }
}

// PQDistanceTable.Lookup: float64 sum in chunk order, float32 result, or
// false on overflow (ErrPQScoreOverflow).
__device__ __forceinline__ bool pq_lookup(const float* table, const uint8_t* code, int chunks,
                                          float* out) {
  double s = 0.0;
  for (int c = 0; c < chunks; ++c) s = __dadd_rn(s, (double)table[c * 256 + code[c]]);
  if (isnan(s) || isinf(s) || s > 3.4028234663852886e38 || s < -3.4028234663852886e38) return false;
  *out = __double2float_rn(s);
  return true;
}

// Byte c (compile-time) of a 32-byte code held as two 16-byte vectors.
__device__ __forceinline__ uint32_t code_byte(const uint4& lo, const uint4& hi, int c) {
  const uint4& v = c < 16 ? lo : hi;
  const int w = (c >> 2) & 3;
  const uint32_t word = w == 0 ? v.x : w == 1 ? v.y : w == 2 ? v.z : v.w;
  return (word >> (8 * (c & 3))) & 0xffu;
}

// One block (16 warps) per query: the query's table is staged once in shared
// memory as LutT (float64 when it fits, so the float64 sums need no
// conversions) and the block walks every probed list; the warps split each
// list in 64-code steps and work without block barriers.  Each warp keeps its
// own candidate list (ballot appends, warp compaction to the KP best keys)
// and the warps share the lowest list threshold through shared memory; the
// 16 lists of a query are merged in exact mode.  Codes and key ranks are read
// in list-major order (contiguous per list; positions only for the filter).
// Each lane scores kPer codes per step with their float64 sums interleaved,
// each still in chunk order, so every score is the reference's, and loads a
// row's key rank only when its score can enter the list.
constexpr int kScanWarps = 16;

template <int CAPW, typename LutT>
__global__ void __launch_bounds__(kScanWarps * 32, 2) ivfpq_scan_kernel(
    const float* __restrict__ table, int chunks, const uint8_t* __restrict__ list_codes,
    const uint64_t* __restrict__ probe_lists, const int* __restrict__ probe_counts, int nprobe,
    const int64_t* __restrict__ list_offsets, const uint32_t* __restrict__ list_rows,
    const uint32_t* __restrict__ list_keyrank, const uint32_t* __restrict__ bitmap, int metric,
    int kp, const int* __restrict__ query_ids, uint64_t* __restrict__ part_keys,
    int* __restrict__ part_counts, uint64_t* __restrict__ part_sat, int* __restrict__ q_flags) {
  constexpr int kPer = 2;
  constexpr int kStep = 32 * kPer;  // codes per warp step
  extern __shared__ __align__(16) unsigned char smem_raw[];
  LutT* slut = reinterpret_cast<LutT*>(smem_raw);                       // [chunks][256]
  uint64_t* wbuf = reinterpret_cast<uint64_t*>(slut + chunks * 256);    // [warps][CAPW]
  __shared__ AccumState wst[kScanWarps];
  __shared__ unsigned long long s_thr;
  const int q = query_ids ? query_ids[blockIdx.x] : blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int i = threadIdx.x; i < chunks * 256; i += blockDim.x)
    slut[i] = (LutT)table[(int64_t)q * chunks * 256 + i];
  if (lane == 0) {
    wst[warp].count = 0;
    wst[warp].saturated = 0;
    wst[warp].thr = kEmptyKey;
  }
  if (threadIdx.x == 0) s_thr = kEmptyKey;
  __syncthreads();
  uint64_t* buf = wbuf + warp * CAPW;
  AccumState* st = &wst[warp];
  int cnt = 0;               // warp-uniform copies of st
  uint64_t wthr = kEmptyKey;
  const bool wide = chunks == 32;  // two 16-byte loads per code
  const int nl = probe_counts[q];
  for (int j = 0; j < nl; ++j) {
    const uint64_t list = probe_lists[(int64_t)q * nprobe + j];
    const int64_t begin = list_offsets[list], end = list_offsets[list + 1];
    for (int64_t base = begin + (int64_t)warp * kStep; base < end;
         base += (int64_t)kScanWarps * kStep) {
      int64_t idx[kPer];
      bool valid[kPer];
      double sum[kPer];
#pragma unroll
      for (int u = 0; u < kPer; ++u) {
        idx[u] = base + u * 32 + lane;
        valid[u] = idx[u] < end;
        if (bitmap && valid[u]) valid[u] = bitmap_pass(bitmap, list_rows[idx[u]]);
        if (!valid[u]) idx[u] = begin;
        sum[u] = 0.0;
      }
      if (wide) {
        uint4 lo[kPer], hi[kPer];
#pragma unroll
        for (int u = 0; u < kPer; ++u) {
          const uint4* cp = reinterpret_cast<const uint4*>(list_codes + idx[u] * 32);
          lo[u] = __ldg(cp);
          hi[u] = __ldg(cp + 1);
        }
#pragma unroll
        for (int c = 0; c < 32; ++c)
#pragma unroll
          for (int u = 0; u < kPer; ++u)
            sum[u] = __dadd_rn(sum[u], (double)slut[c * 256 + code_byte(lo[u], hi[u], c)]);
      } else {
#pragma unroll
        for (int u = 0; u < kPer; ++u) {
          const uint8_t* code = list_codes + idx[u] * chunks;
          for (int c = 0; c < chunks; ++c)
            sum[u] = __dadd_rn(sum[u], (double)slut[c * 256 + code[c]]);
        }
      }
      const uint64_t shared_thr = *(volatile unsigned long long*)&s_thr;
      const uint64_t thr = shared_thr < wthr ? shared_thr : wthr;
#pragma unroll
      for (int u = 0; u < kPer; ++u) {
        bool take = false;
        uint64_t key = 0;
        if (valid[u]) {
          const double sv = sum[u];
          if (isnan(sv) || isinf(sv) || sv > 3.4028234663852886e38 ||
              sv < -3.4028234663852886e38) {
            atomicOr(&q_flags[q], 8);  // ErrPQScoreOverflow
          } else {
            const uint32_t ord = float_to_ordered(rank_from_score(metric, __double2float_rn(sv)));
            if (ord <= (uint32_t)(thr >> 32)) {
              key = ((uint64_t)ord << 32) | list_keyrank[idx[u]];
              take = key < thr;
            }
          }
        }
        const unsigned m = __ballot_sync(kFullMask, take);
        if (take) buf[cnt + __popc(m & ((1u << lane) - 1))] = key;
        cnt += __popc(m);
      }
      if (cnt > CAPW - kStep) {
        __syncwarp();
        if (lane == 0) st->count = cnt;
        __syncwarp();
        warp_compact<CAPW>(buf, st, kp);
        cnt = st->count;
        wthr = st->thr;
        if (lane == 0 && wthr != kEmptyKey) atomicMin(&s_thr, (unsigned long long)wthr);
      }
    }
  }
  __syncwarp();
  if (lane == 0) st->count = cnt;
  __syncwarp();
  warp_compact<CAPW>(buf, st, kp);
  const int out = min(st->count, kp);
  const int64_t slot = (int64_t)blockIdx.x * kScanWarps + warp;
  for (int i = lane; i < out; i += 32) part_keys[slot * kp + i] = buf[i];
  if (lane == 0) {
    part_counts[slot] = out;
    part_sat[slot] = st->thr;
  }
}

// Fast scan: the same block-per-query structure on a float32 rank, one
// code per lane and no cross-lane reduction.  The table is staged as rows
// of W = 32 G + 32 entries, T2[e][s] = T[e][s mod 32 G] (zero past
// `chunks`), and each code of a list is stored with its 32 G chunk bytes
// rotated by its position in the list mod 32, so lane l reads byte t of its
// code and looks up chunk (l + t) mod 32 G at T2[e][l + t]: the 32 lanes of
// a look-up always hit 32 different banks.  Four float32 accumulators per
// lane (terms t mod 4); the rank is within q_eps of the reference's float64
// sum rounded to float32 (8 G - 1 sequential additions per accumulator, two
// combining levels, one rounding of the reference's result, over terms
// bounded by the per-chunk maxima).  A warp walks its 32-code blocks of all
// probed lists in order with the next block's codes loaded ahead into
// registers.  A non-finite or near-overflow rank sends the query to the
// exact scan (q_flags bit 2); the merge rescores the candidates in reference
// order.
template <int G>
__device__ __forceinline__ void load_code(const uint8_t* codes_t, int64_t idx, bool ok,
                                          uint4 (&c)[2 * G]) {
  const uint4* p = reinterpret_cast<const uint4*>(codes_t + idx * (32 * G));
#pragma unroll
  for (int i = 0; i < 2 * G; ++i) c[i] = ok ? __ldg(p + i) : make_uint4(0u, 0u, 0u, 0u);
}
// Byte t of the code as an integer (one PRMT).
template <int G>
__device__ __forceinline__ uint32_t rot_byte(const uint4 (&c)[2 * G], int t) {
  const uint4& v = c[t >> 4];
  const int w = (t >> 2) & 3;
  const uint32_t word = w == 0 ? v.x : w == 1 ? v.y : w == 2 ? v.z : v.w;
  return __byte_perm(word, 0u, 0x4440u | (uint32_t)(t & 3));
}
// ld.shared.f32 at addr + OFF (OFF an immediate of the instruction).
template <int OFF>
__device__ __forceinline__ float lds_f32(uint32_t addr) {
  float v;
  asm volatile("ld.shared.f32 %0, [%1+%2];" : "=f"(v) : "r"(addr), "n"(OFF));
  return v;
}
// The 32 G look-ups of one code: term t = T2[byte t][lane + t], summed into
// accumulator t mod 4.
template <int G, int W, int... T>
__device__ __forceinline__ void pq_lookups(const uint4 (&code)[2 * G], uint32_t lbase,
                                           float (&acc)[4], std::integer_sequence<int, T...>) {
  ((acc[T & 3] += lds_f32<T * 4>(rot_byte<G>(code, T) * (uint32_t)(W * 4) + lbase)), ...);
}

// Two CTAs per SM where the shared memory allows (32 G + 32 table columns
// plus the lists: G = 1 with lists of <= 256 keys).
template <int CAPW, int G>
constexpr int fast_min_blocks() { return (G == 1 && CAPW <= 256) ? 2 : 1; }

template <int CAPW, int G>
__global__ void __launch_bounds__(kScanWarps * 32, (fast_min_blocks<CAPW, G>())) ivfpq_fast_kernel(
    const float* __restrict__ table, int chunks, const uint8_t* __restrict__ codes_t,
    const uint64_t* __restrict__ probe_lists, const int* __restrict__ probe_counts, int nprobe,
    const int64_t* __restrict__ list_offsets, const uint32_t* __restrict__ list_rows,
    const uint32_t* __restrict__ list_keyrank, const uint32_t* __restrict__ bitmap, int metric,
    int kp, uint64_t* __restrict__ part_keys, int* __restrict__ part_counts,
    uint64_t* __restrict__ part_sat, float* __restrict__ q_eps, int* __restrict__ q_flags) {
  constexpr int kSlots = 32 * G;
  constexpr int W = kSlots + 32;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  float* lut = reinterpret_cast<float*>(smem_raw);                            // [256][W]
  uint64_t* wbuf = reinterpret_cast<uint64_t*>(lut + 256 * W);              // [warps][CAPW]
  __shared__ AccumState wst[kScanWarps];
  __shared__ unsigned long long s_thr;
  __shared__ float s_cmax[kSlots];
  const int q = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const float* tq = table + (int64_t)q * chunks * 256;
  for (int i = threadIdx.x; i < 256 * W; i += blockDim.x) {
    const int e = i / W, c = (i % W) % kSlots;
    lut[i] = c < chunks ? __ldg(tq + c * 256 + e) : 0.f;
  }
  // Per-chunk maxima |T[.][c]| for the error bound.
  for (int c = warp; c < kSlots; c += kScanWarps) {
    float m = 0.f;
    if (c < chunks)
      for (int e = lane; e < 256; e += 32) m = fmaxf(m, fabsf(__ldg(tq + c * 256 + e)));
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(kFullMask, m, o));
    if (lane == 0) s_cmax[c] = m;
  }
  if (lane == 0) {
    wst[warp].count = 0;
    wst[warp].saturated = 0;
    wst[warp].thr = kEmptyKey;
  }
  if (threadIdx.x == 0) s_thr = kEmptyKey;
  __syncthreads();
  if (threadIdx.x == 0) {
    double sum = 0.0;
    for (int c = 0; c < kSlots; ++c) sum += (double)s_cmax[c];
    q_eps[q] = __double2float_ru((double)(8 * G + 3) * 5.9604644775390625e-8 * 1.001 * sum);
  }
  uint64_t* buf = wbuf + warp * CAPW;
  AccumState* st = &wst[warp];
  int cnt = 0;
  uint64_t wthr = kEmptyKey;
  // Shared-memory address of this lane's column of the table.
  const uint32_t lbase = (uint32_t)__cvta_generic_to_shared(lut + lane);
  const int nl = probe_counts[q];

  // Cursor over this warp's blocks: list cj, block cbb of the list; it
  // starts before list 0, so the first next_block() enters it.
  int cj = -1, cbb = 0, cnb = 0;
  int64_t cbegin = 0, cend = 0;
  auto next_block = [&]() {
    cbb += kScanWarps;
    while (cbb >= cnb) {
      if (++cj >= nl) return;
      const uint64_t list = probe_lists[(int64_t)q * nprobe + cj];
      cbegin = list_offsets[list];
      cend = list_offsets[list + 1];
      cnb = (int)((cend - cbegin + 31) >> 5);
      cbb = warp;
    }
  };
  next_block();
  bool have = cj < nl;
  int64_t idx = have ? cbegin + (int64_t)cbb * 32 + lane : 0;
  int64_t lend = cend;
  uint4 code[2 * G];
  load_code<G>(codes_t, idx, have && idx < lend, code);
  while (have) {
    // The next block's codes, in flight while this one is scored.
    next_block();
    const bool have_next = cj < nl;
    const int64_t nidx = have_next ? cbegin + (int64_t)cbb * 32 + lane : 0;
    const int64_t nend = cend;
    uint4 ncode[2 * G];
    load_code<G>(codes_t, nidx, have_next && nidx < nend, ncode);
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    pq_lookups<G, W>(code, lbase, acc, std::make_integer_sequence<int, kSlots>{});
    const float fast = (acc[0] + acc[1]) + (acc[2] + acc[3]);
    const uint64_t shared_thr = *(volatile unsigned long long*)&s_thr;
    const uint64_t thr = shared_thr < wthr ? shared_thr : wthr;
    // Common case first: no lane's rank can enter the list (the float bound
    // is NaN, accepting everything, until a list is full).
    const float rank = rank_from_score(metric, fast);
    const bool in_list = idx < lend;
    const bool maybe = in_list && (!(rank > rank_of(thr)) || !(fabsf(fast) < 3.0e38f));
    if (__any_sync(kFullMask, maybe)) {
      bool valid = in_list;
      if (bitmap && valid) valid = bitmap_pass(bitmap, list_rows[idx]);
      bool take = false;
      uint64_t key = 0;
      if (valid) {
        if (!(fabsf(fast) < 3.0e38f)) {
          atomicOr(&q_flags[q], 2);
        } else {
          const uint32_t ord = float_to_ordered(rank);
          if (ord <= (uint32_t)(thr >> 32)) {
            key = ((uint64_t)ord << 32) | list_keyrank[idx];
            take = key < thr;
          }
        }
      }
      const unsigned m = __ballot_sync(kFullMask, take);
      if (take) buf[cnt + __popc(m & ((1u << lane) - 1))] = key;
      cnt += __popc(m);
      if (cnt > CAPW - 32) {
        __syncwarp();
        if (lane == 0) st->count = cnt;
        __syncwarp();
        warp_compact<CAPW>(buf, st, kp);
        cnt = st->count;
        wthr = st->thr;
        if (lane == 0 && wthr != kEmptyKey) atomicMin(&s_thr, (unsigned long long)wthr);
      }
    }
    have = have_next;
    idx = nidx;
    lend = nend;
#pragma unroll
    for (int i = 0; i < 2 * G; ++i) code[i] = ncode[i];
  }
  __syncwarp();
  if (lane == 0) st->count = cnt;
  __syncwarp();
  warp_compact<CAPW>(buf, st, kp);
  const int out = min(st->count, kp);
  const int64_t slot = (int64_t)q * kScanWarps + warp;
  for (int i = lane; i < out; i += 32) part_keys[slot * kp + i] = buf[i];
  if (lane == 0) {
    part_counts[slot] = out;
    part_sat[slot] = st->thr;
  }
}

struct PQScorer {
  int metric;
  const float* table;
  const uint8_t* codes;
  int chunks;
  const float* q_eps;  // fast-rank error bound per query (null: exact lists)
  __device__ float score(int qi, int64_t row) const {
    float s;
    if (!pq_lookup(table + (int64_t)qi * chunks * 256, codes + row * chunks, chunks, &s))
      return __int_as_float(0x7fc00000);
    return s;
  }
  __device__ float eps(int qi) const { return q_eps ? q_eps[qi] : 0.f; }
  __device__ bool half_warp() const { return false; }
  __device__ int error_flag(float) const { return 8; }
  __device__ float output(float r) const { return score_from_rank(metric, r); }
  __device__ bool keep(float out, float radius) const { return within_radius(metric, out, radius); }
};

__global__ void ivfpq_status_kernel(const int* q_status, const int* q_flags, int nq,
                                    int* out_counts) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= nq) return;
  int st = q_status[i];
  if (st == 0 && (q_flags[i] & 4)) st = XVEC_GPU_NON_FINITE;
  if (st == 0 && (q_flags[i] & 8)) st = XVEC_GPU_OVERFLOW;
  if (st != 0) out_counts[i] = -st;
}

__global__ void clear_flag_kernel(const int* ids, int n, int bit, int* q_flags) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) q_flags[ids[i]] &= ~bit;
}

__global__ void count_lists_kernel(const int32_t* row_list, int64_t n, int64_t* counts) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) atomicAdd((unsigned long long*)&counts[row_list[i]], 1ull);
}
__global__ void iota32_kernel(uint32_t* out, int64_t n) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) out[i] = (uint32_t)i;
}

}  // namespace

cudaError_t launch_pq_encode(const float* rows, int64_t n, int d, int metric, const float* pivots,
                             const int* offsets, int chunks, uint8_t* codes, int* err,
                             cudaStream_t s) {
  if (n <= 0) return cudaSuccess;
  pq_encode_kernel<<<(unsigned)n, 256, 0, s>>>(rows, n, d, metric, pivots, offsets, chunks, codes,
                                                err);
  XVEC_LAUNCHED();
  return cudaGetLastError();
}

cudaError_t launch_pq_table(const float* queries, int nq, int d, int metric, const float* pivots,
                            const int* offsets, int chunks, float* table, int* q_flags,
                            cudaStream_t s) {
  if (nq <= 0) return cudaSuccess;
  pq_table_kernel<<<nq, 256, 0, s>>>(queries, nq, d, metric, pivots, offsets, chunks, table,
                                     q_flags);
  XVEC_LAUNCHED();
  return cudaGetLastError();
}


// Nearest centroid of each row through a Flat index over the centroids
// (keys = centroid index): top-1 under the metric, ties to the lower index.
xvec_gpu_status assign_rows(xvec_gpu_index* probe, const float* d_rows, int64_t n, int d,
                            int32_t* d_labels, float* d_scores, cudaStream_t s) {
  xvec_gpu_search_opts o{};
  o.top_k = 1;
  xvec_gpu_status st;
  Scratch keys, scores, counts, err;
  const int64_t batch = std::min<int64_t>(n, kAssignBatch);
  if ((st = keys.alloc((size_t)batch * 8, s)) || (st = scores.alloc((size_t)batch * 4, s)) ||
      (st = counts.alloc((size_t)batch * 4, s)) || (st = err.alloc(4, s)))
    return st;
  XVEC_CUDA(cudaMemsetAsync(err.ptr, 0, 4, s));
  for (int64_t b = 0; b < n; b += kAssignBatch) {
    const int m = (int)std::min<int64_t>(kAssignBatch, n - b);
    std::vector<int> statuses;
    NestedSearch nested;
    st = search_device_locked(probe, d_rows + b * d, m, o, nullptr, keys.as<uint64_t>(),
                              d_scores ? d_scores + b : scores.as<float>(), counts.as<int>(), s,
                              &statuses);
    if (st) return st;
    for (int i = 0; i < m; ++i)
      if (statuses[i]) return set_error("assign row %lld: status %d", (long long)(b + i), statuses[i]),
                              (xvec_gpu_status)statuses[i];
    keys_to_labels_kernel<<<blocks_of(m), 256, 0, s>>>(keys.as<uint64_t>(), counts.as<int>(), m,
                                                        d_labels + b, err.as<int>());
    XVEC_LAUNCHED();
  }
  int h = 0;
  XVEC_CUDA(cudaMemcpyAsync(&h, err.ptr, 4, cudaMemcpyDeviceToHost, s));
  XVEC_CUDA(cudaStreamSynchronize(s));
  if (h) return set_error("k-means assignment failed (status %d)", h), (xvec_gpu_status)h;
  return XVEC_GPU_OK;
}

xvec_gpu_status make_probe_index(int device, int metric, int d, const float* d_centroids,
                                 int nlist, cudaStream_t s, xvec_gpu_index** out) {
  xvec_gpu_index_desc desc{};
  desc.kind = XVEC_INDEX_FLAT;
  desc.dimension = d;
  desc.metric = metric;
  desc.storage = XVEC_STORAGE_FP32;
  desc.device = device;
  xvec_gpu_index* p = nullptr;
  xvec_gpu_status st = xvec_gpu_index_create(&desc, &p);
  if (st) return st;
  std::vector<uint64_t> ids(nlist);
  for (int i = 0; i < nlist; ++i) ids[i] = (uint64_t)i;
  Scratch dk;
  if ((st = dk.alloc((size_t)nlist * 8, s))) {
    xvec_gpu_index_destroy(p);
    return st;
  }
  cudaMemcpyAsync(dk.ptr, ids.data(), (size_t)nlist * 8, cudaMemcpyHostToDevice, s);
  st = add_device_locked(p, dk.as<uint64_t>(), d_centroids, nlist, s);
  if (st) {
    xvec_gpu_index_destroy(p);
    return st;
  }
  *out = p;
  return XVEC_GPU_OK;
}


// ---------------------------------------------------------------------------
// Index hooks.
// ---------------------------------------------------------------------------
xvec_gpu_status ivfpq_reserve(xvec_gpu_index* idx, int64_t cap, cudaStream_t s) {
  xvec_gpu_status st;
  const int64_t n = idx->n;
  const int chunks = std::max(1, idx->chunks);
  if ((st = idx->pq_codes.reserve((size_t)cap * chunks, (size_t)n * chunks, s)) ||
      (st = idx->row_list.reserve((size_t)cap * 4, (size_t)n * 4, s)))
    return st;
  return XVEC_GPU_OK;
}

xvec_gpu_status ivfpq_commit(xvec_gpu_index* idx, int64_t old_n, int64_t m, cudaStream_t s) {
  const int d = idx->desc.dimension;
  xvec_gpu_status st =
      assign_rows(idx->probe_index, idx->rows.as<float>() + old_n * d, m, d,
                  idx->row_list.as<int32_t>() + old_n, nullptr, s);
  if (st) return st;
  Scratch err;
  if ((st = err.alloc(4, s))) return st;
  XVEC_CUDA(cudaMemsetAsync(err.ptr, 0, 4, s));
  pq_encode_kernel<<<(unsigned)m, 256, 0, s>>>(idx->rows.as<float>() + old_n * d, m, d,
                                                idx->desc.metric, idx->pivots.as<float>(),
                                                idx->chunk_offsets.as<int>(), idx->chunks,
                                                idx->pq_codes.as<uint8_t>() + old_n * idx->chunks,
                                                err.as<int>());
  XVEC_LAUNCHED();
  XVEC_CUDA(cudaGetLastError());
  int h = 0;
  XVEC_CUDA(cudaMemcpyAsync(&h, err.ptr, 4, cudaMemcpyDeviceToHost, s));
  XVEC_CUDA(cudaStreamSynchronize(s));
  if (h) return set_error("PQ encoding produced a non-finite score"), (xvec_gpu_status)h;
  idx->lists_dirty = true;
  return XVEC_GPU_OK;
}

// CSR of positions per list; positions keep insertion order within a list
// (ivf.go:193-201 appends in position order; the radix sort is stable).
// List-major copies of the codes and key ranks, so a list scan streams
// contiguous memory instead of gathering rows scattered in insertion order.
__global__ void gather_list_major_kernel(const uint32_t* __restrict__ list_rows, int64_t n,
                                         int chunks, const uint8_t* __restrict__ codes,
                                         const uint32_t* __restrict__ keyrank,
                                         uint8_t* __restrict__ list_codes,
                                         uint32_t* __restrict__ list_keyrank) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const uint32_t pos = list_rows[i];
  list_keyrank[i] = keyrank[pos];
  if (chunks % 16 == 0) {
    const uint4* src = reinterpret_cast<const uint4*>(codes + (int64_t)pos * chunks);
    uint4* dst = reinterpret_cast<uint4*>(list_codes + i * chunks);
    for (int c = 0; c < chunks / 16; ++c) dst[c] = src[c];
  } else {
    for (int c = 0; c < chunks; ++c) list_codes[i * chunks + c] = codes[(int64_t)pos * chunks + c];
  }
}

// IVF-SQ8's list-major codes, one thread per (list entry, 16-byte chunk):
// chunk c of entry i goes to ((i / 32) C + c) 32 + i mod 32 (C = d / 16), so a
// warp reading chunk c of 32 consecutive entries reads 512 contiguous bytes;
// the entry's float4 rank terms follow in list order.
__global__ void gather_sq8_list_kernel(const uint32_t* __restrict__ list_rows, int64_t n, int d,
                                       const uint4* __restrict__ codes,
                                       const float4* __restrict__ fast,
                                       uint4* __restrict__ list_codes,
                                       float4* __restrict__ list_fast) {
  const int C = d / 16;
  const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= n * C) return;
  const int64_t i = t / C;
  const int c = (int)(t - i * C);
  const uint32_t pos = list_rows[i];
  list_codes[((i >> 5) * C + c) * 32 + (i & 31)] = codes[(int64_t)pos * C + c];
  if (c == 0) list_fast[i] = fast[pos];
}

// IVF-Flat's list-major rows, one thread per (list entry, float4 chunk), in
// the same interleaved order; the entry's ||x||^2 follows in list order.
__global__ void gather_flat_list_kernel(const uint32_t* __restrict__ list_rows, int64_t n, int d,
                                        const float4* __restrict__ rows,
                                        const float* __restrict__ row_n2,
                                        float4* __restrict__ list_rows_f,
                                        float* __restrict__ list_n2) {
  const int C = d / 4;
  const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= n * C) return;
  const int64_t i = t / C;
  const int c = (int)(t - i * C);
  const uint32_t pos = list_rows[i];
  list_rows_f[((i >> 5) * C + c) * 32 + (i & 31)] = rows[(int64_t)pos * C + c];
  if (c == 0) list_n2[i] = row_n2[pos];
}

// The fast scan's code layout (list_codes_t), one CTA per list: code i of
// the list holds at byte t its chunk (i mod 32 + t) mod slots (zero past
// `chunks`).
__global__ void rotate_list_codes_kernel(const int64_t* __restrict__ list_offsets, int chunks,
                                         int slots, const uint8_t* __restrict__ list_codes,
                                         uint8_t* __restrict__ codes_t) {
  const int l = blockIdx.x;
  const int64_t begin = list_offsets[l], len = list_offsets[l + 1] - begin;
  for (int64_t x = threadIdx.x; x < len * slots; x += blockDim.x) {
    const int64_t i = x / slots;
    const int t = (int)(x - i * slots);
    const int c = ((int)(i & 31) + t) % slots;
    codes_t[(begin + i) * slots + t] = c < chunks ? list_codes[(begin + i) * chunks + c] : (uint8_t)0;
  }
}

// Chunk slots of the fast scan (0: the layout does not apply).
int fast_slots(int chunks) { return chunks <= 32 ? 32 : chunks <= 64 ? 64 : 0; }

xvec_gpu_status rebuild_lists(xvec_gpu_index* idx, cudaStream_t s) {
  const int64_t n = idx->n;
  const int nlist = idx->nlist;
  xvec_gpu_status st;
  if ((st = idx->list_offsets.reserve((size_t)(nlist + 1) * 8, 0, s)) ||
      (st = idx->list_rows.reserve((size_t)std::max<int64_t>(n, 1) * 4, 0, s)))
    return st;
  Scratch counts, iota, sorted_lists, temp;
  if ((st = counts.alloc((size_t)(nlist + 1) * 8, s)) || (st = iota.alloc((size_t)n * 4, s)) ||
      (st = sorted_lists.alloc((size_t)n * 4, s)))
    return st;
  XVEC_CUDA(cudaMemsetAsync(counts.ptr, 0, (size_t)(nlist + 1) * 8, s));
  count_lists_kernel<<<blocks_of(n), 256, 0, s>>>(idx->row_list.as<int32_t>(), n,
                                                  counts.as<int64_t>());
  iota32_kernel<<<blocks_of(n), 256, 0, s>>>(iota.as<uint32_t>(), n);
  size_t tb = 0, tb2 = 0;
  XVEC_CUDA(cub::DeviceRadixSort::SortPairs(nullptr, tb, idx->row_list.as<uint32_t>(),
                                            sorted_lists.as<uint32_t>(), iota.as<uint32_t>(),
                                            idx->list_rows.as<uint32_t>(), n, 0, 32, s));
  XVEC_CUDA(cub::DeviceScan::ExclusiveSum(nullptr, tb2, counts.as<int64_t>(),
                                          idx->list_offsets.as<int64_t>(), nlist + 1, s));
  if ((st = temp.alloc(std::max(tb, tb2), s))) return st;
  XVEC_CUDA(cub::DeviceRadixSort::SortPairs(temp.ptr, tb, idx->row_list.as<uint32_t>(),
                                            sorted_lists.as<uint32_t>(), iota.as<uint32_t>(),
                                            idx->list_rows.as<uint32_t>(), n, 0, 32, s));
  XVEC_CUDA(cub::DeviceScan::ExclusiveSum(temp.ptr, tb2, counts.as<int64_t>(),
                                          idx->list_offsets.as<int64_t>(), nlist + 1, s));
  // IVF-PQ: list-major codes (and their rotated copy); every IVF kind: the
  // key ranks in list order.
  const int chunks = idx->desc.kind == XVEC_INDEX_IVF_PQ ? idx->chunks : 0;
  if ((st = idx->list_codes.reserve((size_t)std::max<int64_t>(n, 1) * std::max(chunks, 1), 0, s)) ||
      (st = idx->list_keyrank.reserve((size_t)std::max<int64_t>(n, 1) * 4, 0, s)))
    return st;
  gather_list_major_kernel<<<blocks_of(n), 256, 0, s>>>(
      idx->list_rows.as<uint32_t>(), n, chunks, idx->pq_codes.as<uint8_t>(),
      idx->keyrank.as<uint32_t>(), idx->list_codes.as<uint8_t>(),
      idx->list_keyrank.as<uint32_t>());
  XVEC_LAUNCHED();
  XVEC_CUDA(cudaGetLastError());
  const int slots = fast_slots(chunks);
  if (chunks > 0 && slots > 0) {
    const size_t bytes = (size_t)std::max<int64_t>(n, 1) * slots;
    if ((st = idx->list_codes_t.reserve(bytes, 0, s))) return st;
    rotate_list_codes_kernel<<<nlist, 256, 0, s>>>(idx->list_offsets.as<int64_t>(), chunks, slots,
                                                   idx->list_codes.as<uint8_t>(),
                                                   idx->list_codes_t.as<uint8_t>());
    XVEC_LAUNCHED();
    XVEC_CUDA(cudaGetLastError());
  }
  if ((idx->desc.kind == XVEC_INDEX_IVF_SQ8 || idx->desc.kind == XVEC_INDEX_IVF_SQ4) &&
      idx->desc.dimension % 16 == 0) {
    const int d = idx->desc.dimension;
    const int64_t padded = (n + 31) / 32 * 32;
    if ((st = idx->list_sq_codes.reserve((size_t)padded * d, 0, s)) ||
        (st = idx->list_sq_fast.reserve((size_t)padded * 16, 0, s)))
      return st;
    gather_sq8_list_kernel<<<blocks_of(n * (d / 16)), 256, 0, s>>>(
        idx->list_rows.as<uint32_t>(), n, d, idx->sq_codes.as<uint4>(),
        idx->sq_fast.as<float4>(), idx->list_sq_codes.as<uint4>(),
        idx->list_sq_fast.as<float4>());
    XVEC_LAUNCHED();
    XVEC_CUDA(cudaGetLastError());
  }
  if (idx->desc.kind == XVEC_INDEX_IVF_FLAT && idx->desc.dimension % 4 == 0) {
    const int d = idx->desc.dimension;
    const int64_t padded = (n + 31) / 32 * 32;
    if ((st = idx->list_rows_f.reserve((size_t)padded * d * 4, 0, s)) ||
        (st = idx->list_n2.reserve((size_t)padded * 4, 0, s)))
      return st;
    gather_flat_list_kernel<<<blocks_of(n * (d / 4)), 256, 0, s>>>(
        idx->list_rows.as<uint32_t>(), n, d, idx->rows.as<float4>(), idx->row_n2.as<float>(),
        idx->list_rows_f.as<float4>(), idx->list_n2.as<float>());
    XVEC_LAUNCHED();
    XVEC_CUDA(cudaGetLastError());
  }
  XVEC_CUDA(cudaStreamSynchronize(s));
  idx->lists_dirty = false;
  return XVEC_GPU_OK;
}

xvec_gpu_status ivfpq_search_impl(xvec_gpu_index* idx, const float* d_q, int nq,
                                  const xvec_gpu_search_opts& o, const uint32_t* d_bitmap,
                                  uint64_t* d_keys, float* d_scores, int* d_counts,
                                  cudaStream_t s, std::vector<int>* statuses) {
  if (!idx->has_model) return set_error("IVF-PQ index has no model"), XVEC_GPU_INVALID_ARGUMENT;
  if (o.nprobe <= 0) return set_error("core: IVF NProbe must be positive"), XVEC_GPU_INVALID_ARGUMENT;
  const int d = idx->desc.dimension, metric = idx->desc.metric, k = o.top_k;
  const int64_t n = idx->n;
  const int chunks = idx->chunks;
  xvec_gpu_status st;
  EventTimer timer(s);
  timer.mark(0);
  // The lists are rebuilt under the shared lock: only one searcher may do it.
  {
    static std::mutex rebuild_mu;
    std::lock_guard<std::mutex> g(rebuild_mu);
    if (idx->lists_dirty && n > 0 && (st = rebuild_lists(idx, s))) return st;
  }
  const int nprobe = std::min(o.nprobe, idx->nlist);
  int kp = 32;
  while (kp < k + std::max(8, k / 4)) kp <<= 1;
  if ((int64_t)kScanWarps * kp > flat_merge_capacity())
    return set_error("top_k %d exceeds the merge capacity", k), XVEC_GPU_INVALID_ARGUMENT;
  // Probe: the Flat path over the centroids (validates the queries too).
  Scratch pkeys_probe, pscores_probe, pcounts_probe, table, qflags, qstatus;
  if ((st = pkeys_probe.alloc((size_t)nq * nprobe * 8, s)) ||
      (st = pscores_probe.alloc((size_t)nq * nprobe * 4, s)) ||
      (st = pcounts_probe.alloc((size_t)nq * 4, s)) ||
      (st = table.alloc((size_t)nq * chunks * 256 * 4, s)) ||
      (st = qflags.alloc((size_t)nq * 4, s)) || (st = qstatus.alloc((size_t)nq * 4, s)))
    return st;
  xvec_gpu_search_opts po{};
  po.top_k = nprobe;
  std::vector<int> probe_status;
  {
    NestedSearch nested;
    st = search_device_locked(idx->probe_index, d_q, nq, po, nullptr, pkeys_probe.as<uint64_t>(),
                              pscores_probe.as<float>(), pcounts_probe.as<int>(), s,
                              &probe_status);
  }
  if (st) return st;
  XVEC_CUDA(cudaMemcpyAsync(qstatus.ptr, probe_status.data(), (size_t)nq * 4,
                            cudaMemcpyHostToDevice, s));
  XVEC_CUDA(cudaMemsetAsync(qflags.ptr, 0, (size_t)nq * 4, s));
  XVEC_CUDA(cudaMemsetAsync(d_counts, 0, (size_t)nq * 4, s));
  pq_table_kernel<<<nq, 256, 0, s>>>(d_q, nq, d, metric, idx->pivots.as<float>(),
                                     idx->chunk_offsets.as<int>(), chunks, table.as<float>(),
                                     qflags.as<int>());
  XVEC_LAUNCHED();
  int exact_count = 0;
  if (n > 0) {
    int capw = 128;
    while (capw < kp + 64) capw <<= 1;
    if (capw > 1024) return set_error("top_k %d too large for the IVF-PQ scan", k), XVEC_GPU_INVALID_ARGUMENT;
    Scratch lkeys, lcounts, lsat, qeps;
    const size_t lists = (size_t)nq * kScanWarps;
    if ((st = lkeys.alloc(lists * kp * 8, s)) || (st = lcounts.alloc(lists * 4, s)) ||
        (st = lsat.alloc(lists * 8, s)) || (st = qeps.alloc((size_t)nq * 4, s)))
      return st;
    const size_t bufs = (size_t)kScanWarps * capw * 8;
    // Exact scan: the table as float64 in shared memory when it fits next
    // to the buffers.
    auto exact_scan = [&](const int* ids, int count) -> xvec_gpu_status {
      const bool lut64 = (size_t)chunks * 256 * 8 + bufs <= 200 * 1024;
      const size_t smem = (size_t)chunks * 256 * (lut64 ? 8 : 4) + bufs;
      if (smem > 220 * 1024) return set_error("too many PQ chunks for the scan"), XVEC_GPU_UNSUPPORTED;
#define XVEC_PQ_CASE(C, T)                                                                     \
  if (capw == C && lut64 == (sizeof(T) == 8)) {                                                \
    auto kern = ivfpq_scan_kernel<C, T>;                                                       \
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);        \
    kern<<<count, kScanWarps * 32, smem, s>>>(                                                 \
        table.as<float>(), chunks, idx->list_codes.as<uint8_t>(), pkeys_probe.as<uint64_t>(),  \
        pcounts_probe.as<int>(), nprobe, idx->list_offsets.as<int64_t>(),                      \
        idx->list_rows.as<uint32_t>(), idx->list_keyrank.as<uint32_t>(), d_bitmap, metric, kp, \
        ids, lkeys.as<uint64_t>(), lcounts.as<int>(), lsat.as<uint64_t>(), qflags.as<int>());  \
  }
      XVEC_PQ_CASE(128, double)
      XVEC_PQ_CASE(256, double)
      XVEC_PQ_CASE(512, double)
      XVEC_PQ_CASE(1024, double)
      XVEC_PQ_CASE(128, float)
      XVEC_PQ_CASE(256, float)
      XVEC_PQ_CASE(512, float)
      XVEC_PQ_CASE(1024, float)
#undef XVEC_PQ_CASE
      XVEC_LAUNCHED();
      XVEC_CUDA(cudaGetLastError());
      PQScorer sc{metric, table.as<float>(), idx->pq_codes.as<uint8_t>(), chunks, nullptr};
      XVEC_CUDA(launch_merge_rescore(sc, idx->pos_of_kr.as<uint32_t>(), idx->keys.as<uint64_t>(),
                                     ids, count, k, o.radius, 1, lkeys.as<uint64_t>(),
                                     lcounts.as<int>(), lsat.as<uint64_t>(), kScanWarps, kp,
                                     d_keys, d_scores, d_counts, nullptr, qflags.as<int>(), s));
      XVEC_LAUNCHED();
      return XVEC_GPU_OK;
    };
    // Fast scan: the widened table and the warps' lists.
    const int slots = fast_slots(chunks);
    const size_t fast_smem = (size_t)256 * (slots + 32) * 4 + bufs;
    const bool fast = slots > 0 && fast_smem <= 220 * 1024;
    timer.mark(1);
    if (fast) {
      bool launched = false;
#define XVEC_PQ_FAST(C, G)                                                                     \
  if (capw == C && slots == 32 * G) {                                                          \
    auto kern = ivfpq_fast_kernel<C, G>;                                                       \
    launched = true;                                                                           \
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)fast_smem);   \
    kern<<<nq, kScanWarps * 32, fast_smem, s>>>(                                               \
        table.as<float>(), chunks, idx->list_codes_t.as<uint8_t>(), pkeys_probe.as<uint64_t>(), \
        pcounts_probe.as<int>(), nprobe, idx->list_offsets.as<int64_t>(), idx->list_rows.as<uint32_t>(),                \
        idx->list_keyrank.as<uint32_t>(), d_bitmap, metric, kp, lkeys.as<uint64_t>(),          \
        lcounts.as<int>(), lsat.as<uint64_t>(), qeps.as<float>(), qflags.as<int>());           \
  }
      XVEC_PQ_FAST(128, 1)
      XVEC_PQ_FAST(256, 1)
      XVEC_PQ_FAST(512, 1)
      XVEC_PQ_FAST(1024, 1)
      XVEC_PQ_FAST(128, 2)
      XVEC_PQ_FAST(256, 2)
      XVEC_PQ_FAST(512, 2)
#undef XVEC_PQ_FAST
      if (!launched) return set_error("no fast IVF-PQ scan for this layout"), XVEC_GPU_UNSUPPORTED;
      timer.mark(2);
      XVEC_LAUNCHED();
      XVEC_CUDA(cudaGetLastError());
      PQScorer sc{metric, table.as<float>(), idx->pq_codes.as<uint8_t>(), chunks, qeps.as<float>()};
      XVEC_CUDA(launch_merge_rescore(sc, idx->pos_of_kr.as<uint32_t>(), idx->keys.as<uint64_t>(),
                                     nullptr, nq, k, o.radius, 0, lkeys.as<uint64_t>(),
                                     lcounts.as<int>(), lsat.as<uint64_t>(), kScanWarps, kp,
                                     d_keys, d_scores, d_counts, nullptr, qflags.as<int>(), s));
      XVEC_LAUNCHED();
      // Queries the fast pass could not settle go through the exact scan.
      std::vector<int> h_fl(nq), exact_list;
      XVEC_CUDA(cudaMemcpyAsync(h_fl.data(), qflags.ptr, (size_t)nq * 4, cudaMemcpyDeviceToHost, s));
      XVEC_CUDA(cudaStreamSynchronize(s));
      for (int q = 0; q < nq; ++q)
        if (probe_status[q] == 0 && (h_fl[q] & 2)) exact_list.push_back(q);
      if (!exact_list.empty()) {
        const int nl = (int)exact_list.size();
        Scratch ids;
        if ((st = ids.alloc((size_t)nl * 4, s))) return st;
        XVEC_CUDA(cudaMemcpyAsync(ids.ptr, exact_list.data(), (size_t)nl * 4,
                                  cudaMemcpyHostToDevice, s));
        clear_flag_kernel<<<blocks_of(nl), 256, 0, s>>>(ids.as<int>(), nl, 2, qflags.as<int>());
        XVEC_LAUNCHED();
        if ((st = exact_scan(ids.as<int>(), nl))) return st;
        XVEC_CUDA(cudaStreamSynchronize(s));
        exact_count = nl;
      }
    } else {
      if ((st = exact_scan(nullptr, nq))) return st;
      timer.mark(2);
      exact_count = nq;
    }
  }
  ivfpq_status_kernel<<<blocks_of(nq), 256, 0, s>>>(qstatus.as<int>(), qflags.as<int>(), nq,
                                                    d_counts);
  XVEC_LAUNCHED();
  XVEC_CUDA(cudaGetLastError());
  std::vector<int> h_flags(nq);
  XVEC_CUDA(cudaMemcpyAsync(h_flags.data(), qflags.ptr, (size_t)nq * 4, cudaMemcpyDeviceToHost, s));
  timer.mark(3);
  XVEC_CUDA(cudaStreamSynchronize(s));
  count_search(nq, exact_count, timer.ms(1, 2), timer.ms(0, 3));
  if (statuses) {
    statuses->resize(nq);
    for (int q = 0; q < nq; ++q) {
      int sq = probe_status[q];
      if (sq == 0 && (h_flags[q] & 4)) sq = XVEC_GPU_NON_FINITE;
      if (sq == 0 && (h_flags[q] & 8)) sq = XVEC_GPU_OVERFLOW;
      (*statuses)[q] = sq;
    }
  }
  return XVEC_GPU_OK;
}

}  // namespace xvec

using namespace xvec;

extern "C" xvec_gpu_status xvec_gpu_ivfpq_set_model(xvec_gpu_index* idx, const float* centroids,
                                                    int32_t nlist, const float* pivots,
                                                    int32_t chunks) {
  if (!idx || !centroids || !pivots) return set_error("nil argument"), XVEC_GPU_INVALID_ARGUMENT;
  if (idx->desc.kind != XVEC_INDEX_IVF_PQ)
    return set_error("not an IVF-PQ index"), XVEC_GPU_INVALID_ARGUMENT;
  const int d = idx->desc.dimension;
  if (nlist <= 0 || chunks <= 0 || chunks > d)
    return set_error("core: invalid PQ options: resolved Chunks must be in [1,%d]", d),
           XVEC_GPU_INVALID_ARGUMENT;
  std::unique_lock<std::shared_mutex> lock(idx->mu);
  if (idx->n > 0) return set_error("set the model before adding rows"), XVEC_GPU_INVALID_ARGUMENT;
  for (int64_t i = 0; i < (int64_t)nlist * d; ++i)
    if (!std::isfinite(centroids[i])) return set_error("non-finite centroid"), XVEC_GPU_NON_FINITE;
  for (int64_t i = 0; i < (int64_t)256 * d; ++i)
    if (!std::isfinite(pivots[i])) return set_error("non-finite PQ pivot"), XVEC_GPU_NON_FINITE;
  cudaSetDevice(idx->device);
  cudaStream_t s = nullptr;
  // pqChunkOffsets (pq.go:395-406): contiguous chunks, wider chunks first.
  std::vector<int> offsets(chunks + 1, 0);
  const int base = d / chunks, larger = d % chunks;
  for (int c = 0; c < chunks; ++c) offsets[c + 1] = offsets[c] + base + (c < larger ? 1 : 0);
  xvec_gpu_status st;
  if ((st = idx->centroids.reserve((size_t)nlist * d * 4, 0, s)) ||
      (st = idx->pivots.reserve((size_t)256 * d * 4, 0, s)) ||
      (st = idx->chunk_offsets.reserve((size_t)(chunks + 1) * 4, 0, s)))
    return st;
  XVEC_CUDA(cudaMemcpy(idx->centroids.ptr, centroids, (size_t)nlist * d * 4, cudaMemcpyHostToDevice));
  XVEC_CUDA(cudaMemcpy(idx->pivots.ptr, pivots, (size_t)256 * d * 4, cudaMemcpyHostToDevice));
  XVEC_CUDA(cudaMemcpy(idx->chunk_offsets.ptr, offsets.data(), (size_t)(chunks + 1) * 4,
                       cudaMemcpyHostToDevice));
  if (idx->probe_index) {
    xvec_gpu_index_destroy(idx->probe_index);
    idx->probe_index = nullptr;
  }
  if ((st = make_probe_index(idx->device, idx->desc.metric, d, idx->centroids.as<float>(), nlist,
                             s, &idx->probe_index)))
    return st;
  idx->nlist = nlist;
  idx->chunks = chunks;
  idx->has_model = true;
  idx->lists_dirty = true;
  return XVEC_GPU_OK;
}

extern "C" xvec_gpu_status xvec_gpu_kmeans_assign_device(int32_t device, int32_t metric,
                                                         const float* d_vectors, int64_t n,
                                                         const float* d_centroids, int32_t nc,
                                                         int32_t dim, int32_t* d_labels,
                                                         float* d_scores, void* stream) {
  if (nc <= 0 || dim <= 0 || n < 0) return set_error("invalid k-means arguments"), XVEC_GPU_INVALID_ARGUMENT;
  if (n == 0) return XVEC_GPU_OK;
  cudaSetDevice(device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  xvec_gpu_index* probe = nullptr;
  xvec_gpu_status st = make_probe_index(device, metric, dim, d_centroids, nc, s, &probe);
  if (st) return st;
  st = assign_rows(probe, d_vectors, n, dim, d_labels, d_scores, s);
  xvec_gpu_index_destroy(probe);
  return st;
}

extern "C" xvec_gpu_status xvec_gpu_kmeans_assign(int32_t device, int32_t metric,
                                                  const float* vectors, int64_t n,
                                                  const float* centroids, int32_t nc, int32_t dim,
                                                  int32_t* labels, float* scores) {
  if (nc <= 0 || dim <= 0 || n < 0 || !vectors || !centroids || !labels)
    return set_error("invalid k-means arguments"), XVEC_GPU_INVALID_ARGUMENT;
  if (n == 0) return XVEC_GPU_OK;
  cudaSetDevice(device);
  cudaStream_t s = nullptr;
  Scratch dv, dc, dl, ds;
  xvec_gpu_status st;
  if ((st = dv.alloc((size_t)n * dim * 4, s)) || (st = dc.alloc((size_t)nc * dim * 4, s)) ||
      (st = dl.alloc((size_t)n * 4, s)) || (st = ds.alloc((size_t)n * 4, s)))
    return st;
  XVEC_CUDA(cudaMemcpyAsync(dv.ptr, vectors, (size_t)n * dim * 4, cudaMemcpyHostToDevice, s));
  XVEC_CUDA(cudaMemcpyAsync(dc.ptr, centroids, (size_t)nc * dim * 4, cudaMemcpyHostToDevice, s));
  st = xvec_gpu_kmeans_assign_device(device, metric, dv.as<float>(), n, dc.as<float>(), nc, dim,
                                     dl.as<int32_t>(), ds.as<float>(), s);
  if (st) return st;
  XVEC_CUDA(cudaMemcpyAsync(labels, dl.ptr, (size_t)n * 4, cudaMemcpyDeviceToHost, s));
  if (scores) XVEC_CUDA(cudaMemcpyAsync(scores, ds.ptr, (size_t)n * 4, cudaMemcpyDeviceToHost, s));
  XVEC_CUDA(cudaStreamSynchronize(s));
  return XVEC_GPU_OK;
}
