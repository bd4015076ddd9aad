// flat_kernels.cu — Flat exact search kernels (CUDA cores).
//
// Reference path: DenseFlatIndex.search (internal/core/flat.go:179-196) →
// topKPrevalidatedCandidatesWithOptions (internal/core/topk.go:105-166) with
// metric.Compute (internal/core/metric/metric.go:35-48).
//
// Pipeline per batch of queries:
//   1. prep_queries: decode queries to float32, reference-order ||q||^2 and
//      the query validation of topk.go:92-94 (metric.Compute(q, q) finite).
//   2. scan (fast):  FFMA tiles of 64 rows x 32 queries; the rank of each
//      pair goes into a per-(query, part) accumulator of the KP best packed
//      keys (select.cuh).  Filter before scoring (topk.go:134-136).
//   3. merge_rescore: per query, the kth best fast key over all parts, the
//      candidate set {rank <= F_k + 2*eps} (eps bounds |fast - reference|),
//      reference-order rescoring of the candidates, final (score, key) sort,
//      radius (query.go:193-201) and top-k.
//   4. scan (exact) + merge in exact mode for the rare query whose candidate
//      set cannot be proven complete, and for large k.
#include <algorithm>

#include "flat_kernels.cuh"
#include "pipeline.cuh"

namespace xvec {

// ---------------------------------------------------------------------------
// Query preparation.
// ---------------------------------------------------------------------------
template <typename QT>
__global__ void prep_queries_kernel(const QT* __restrict__ q_in, int nq, int d, int metric,
                                    float* __restrict__ qf, float* __restrict__ q_n2,
                                    float* __restrict__ q_aux, int* __restrict__ q_status) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= nq) return;
  const QT* src = q_in + (int64_t)warp * d;
  float* dst = qf + (int64_t)warp * d;
  bool finite = true;
  for (int i = lane; i < d; i += 32) {
    const float v = load_elem(src, i);
    dst[i] = v;
    finite &= finite_f(v);
  }
  finite = __all_sync(kFullMask, finite);
  __syncwarp();
  float s0, s1, s2;
  warp_reference_sums<1>(dst, dst, d, &s0, &s1, &s2);  // InnerProduct(q, q)
  if (lane == 0) {
    q_n2[warp] = s0;
    // Tensor-core epilogue operand: 1/||q|| for cosine, ||q||^2 otherwise.
    q_aux[warp] = metric == kMetricCosine ? (s0 > 0.f ? rsqrtf(s0) : 0.f) : s0;
    // metric.Compute(q, q): L2 is always 0 for finite input; IP, cosine and
    // MIPS become non-finite exactly when ||q||^2 overflows.
    int st = 0;
    if (!finite) st = 7;
    else if (metric != kMetricL2 && !finite_f(s0)) st = 7;
    q_status[warp] = st;
  }
}

// Reference-order ||x||^2 of stored rows (InnerProduct(x, x)); used by the
// fast L2 / cosine / MIPS ranks and the error bounds.
template <typename RowT>
__global__ void row_norms_kernel(const RowT* __restrict__ rows, int64_t n, int d,
                                 float* __restrict__ n2, float* __restrict__ inv_mag,
                                 unsigned* __restrict__ max_n2_ordered,
                                 int* __restrict__ nonfinite) {
  const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= n) return;
  const RowT* x = rows + warp * d;
  bool finite = true;
  for (int i = lane; i < d; i += 32) finite &= finite_f(load_elem(x, i));
  finite = __all_sync(kFullMask, finite);
  float s0 = 0.f;
  if (finite) {
    // InnerProduct(x, x) in the reference order (fp16 rows decode exactly).
    float a0 = 0.f, r0 = 0.f;
    if (d >= 16) {
      if (lane < 16)
        for (int v = 0; v < (d >> 4); ++v) {
          const float xv = load_elem(x, v * 16 + lane);
          a0 = __fmaf_rn(xv, xv, a0);
        }
      for (int j = 0; j < 16; ++j) r0 = __fadd_rn(r0, __shfl_sync(kFullMask, a0, j));
      for (int i = (d >> 4) * 16; i < d; ++i) {
        const float xv = load_elem(x, i);
        r0 = __fmaf_rn(xv, xv, r0);
      }
    } else if (d >= 8) {
      if (lane < 8) {
        const float xv = load_elem(x, lane);
        a0 = __fadd_rn(0.f, __fmul_rn(xv, xv));
      }
      for (int j = 0; j < 8; ++j) r0 = __fadd_rn(r0, __shfl_sync(kFullMask, a0, j));
      for (int i = 8; i < d; ++i) {
        const float xv = load_elem(x, i);
        r0 = __fadd_rn(r0, __fmul_rn(xv, xv));
      }
    } else {
      for (int i = 0; i < d; ++i) {
        const float xv = load_elem(x, i);
        r0 = __fadd_rn(r0, __fmul_rn(xv, xv));
      }
    }
    s0 = r0;
  }
  if (lane == 0) {
    n2[warp] = s0;
    inv_mag[warp] = s0 > 0.f ? rsqrtf(s0) : 0.f;
    if (!finite) atomicExch(nonfinite, 1);
    else if (finite_f(s0)) atomicMax(max_n2_ordered, float_to_ordered(s0));
    else atomicMax(max_n2_ordered, float_to_ordered(3.0e38f));
  }
}

// Bound on |fast rank - reference rank| for a query (both accumulate d
// exact-or-rounded products in float32; factor 4 covers both sides and a
// non round-to-nearest accumulator).
// split: the fast dot came from bfloat16 high/low parts (three products per
// element, x = hi + lo to 2^-18 |x|, the lo·lo product dropped) accumulated
// in fp32 by the tensor cores, whose additions may truncate: a relative
// bound of 3.2·2^-18 + (3d + 8)·2u on top.
__device__ __forceinline__ float fast_eps(int metric, int d, float qn2, float max_xn2,
                                          int split = 0) {
  const float u = 5.9604645e-8f;  // 2^-24
  const float g = 4.f * (float)(d + 8) * u +
                  (split ? 2.f * (3.2f * 3.8146973e-6f + (float)(3 * d + 8) * 2.f * u) : 0.f);
  const float qn = sqrtf(qn2), xn = sqrtf(max_xn2);
  switch (metric) {
    case kMetricL2: return g * (xn + qn) * (xn + qn) * 1.0001f;
    case kMetricIP: return g * xn * qn * 1.0001f + 1e-30f;
    case kMetricCosine: return g * 2.f;
    default: return g * 4.f;
  }
}

// ---------------------------------------------------------------------------
// Flat ranker / scorer for the generic pipeline (pipeline.cuh).
// ---------------------------------------------------------------------------
struct FlatRanker {
  int metric;
  const float* row_n2;
  const float* q_n2;
  struct RowInfo {
    float n2;
  };
  struct QueryInfo {
    float n2;
  };
  __device__ QueryInfo query(int qi) const { return {q_n2[qi]}; }
  __device__ RowInfo row(int64_t r) const { return {row_n2[r]}; }
  __device__ float rank(float dot, const RowInfo& r, const QueryInfo& q) const {
    return fast_rank(metric, dot, r.n2, q.n2);
  }
};

template <typename RowT>
struct FlatScorer {
  int metric;
  const RowT* rows;
  const float* qf;
  int d;
  const float* q_n2;
  const unsigned* max_n2_ordered;
  int split;  // fast ranks from the bfloat16-split tensor-core scan
  __device__ float score(int qi, int64_t row) const {
    return warp_reference_score(metric, rows + row * d, qf + (int64_t)qi * d, d);
  }
  __device__ float eps(int qi) const {
    return fast_eps(metric, d, q_n2[qi], ordered_to_float(*max_n2_ordered), split);
  }
  __device__ bool half_warp() const { return d >= 16; }
  __device__ int error_flag(float) const { return 4; }
  __device__ float output(float r) const { return score_from_rank(metric, r); }
  __device__ bool keep(float out, float radius) const { return within_radius(metric, out, radius); }
};

// ---------------------------------------------------------------------------
// Host launchers.
// ---------------------------------------------------------------------------
template <typename QT>
void launch_prep_queries(const QT* q, int nq, int d, int metric, float* qf, float* q_n2,
                         float* q_aux, int* q_status, cudaStream_t stream) {
  const int warps_per_block = 8;
  const int blocks = (nq + warps_per_block - 1) / warps_per_block;
  if (blocks > 0)
    prep_queries_kernel<QT><<<blocks, warps_per_block * 32, 0, stream>>>(q, nq, d, metric, qf,
                                                                         q_n2, q_aux, q_status);
}
template void launch_prep_queries<float>(const float*, int, int, int, float*, float*, float*,
                                         int*, cudaStream_t);
template void launch_prep_queries<__half>(const __half*, int, int, int, float*, float*, float*,
                                          int*, cudaStream_t);

template <typename RowT>
void launch_row_norms(const RowT* rows, int64_t n, int d, float* n2, float* inv_mag,
                      unsigned* max_n2, int* nonfinite, cudaStream_t stream) {
  const int64_t blocks = (n + 7) / 8;
  if (blocks > 0)
    row_norms_kernel<RowT><<<(unsigned)blocks, 256, 0, stream>>>(rows, n, d, n2, inv_mag, max_n2,
                                                                 nonfinite);
}
template void launch_row_norms<float>(const float*, int64_t, int, float*, float*, unsigned*,
                                      int*, cudaStream_t);
template void launch_row_norms<__half>(const __half*, int64_t, int, float*, float*, unsigned*,
                                       int*, cudaStream_t);

int flat_merge_capacity() { return kMergeSmemEntries; }

// One block per query: gather the seed lists, radix-select the kp-th key.
__global__ void __launch_bounds__(256) seed_thresholds_kernel(
    const uint64_t* __restrict__ cand, const int* __restrict__ counts, int num_lists,
    int seed_lists, int cap, int kp, unsigned long long* __restrict__ gthr) {
  extern __shared__ __align__(16) unsigned char seed_smem[];
  uint64_t* keys = reinterpret_cast<uint64_t*>(seed_smem);  // [seed_lists * kp]
  __shared__ int hist[256];
  const int q = blockIdx.x;
  // Published lists hold at most kp keys each, so the buffer holds them all.
  const int total = gather_union(cand, counts, (int64_t)q * num_lists, seed_lists, cap,
                                 kEmptyKey, keys, seed_lists * kp);
  if (total < kp) return;
  const uint64_t kth = smem_radix_select(keys, min(total, seed_lists * kp), kp, 0, hist);
  if (threadIdx.x == 0) atomicMin(&gthr[q], (unsigned long long)kth);
}

cudaError_t launch_seed_thresholds(const uint64_t* cand, const int* counts, int nq, int num_lists,
                                   int seed_lists, int cap, int kp, unsigned long long* gthr,
                                   cudaStream_t stream) {
  if (nq <= 0 || seed_lists <= 0) return cudaSuccess;
  if (seed_lists > 64 || seed_lists * kp > kMergeSmemEntries) return cudaErrorInvalidValue;
  const int smem = seed_lists * kp * 8;
  cudaFuncSetAttribute(seed_thresholds_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  seed_thresholds_kernel<<<nq, 256, smem, stream>>>(cand, counts, num_lists, seed_lists, cap, kp,
                                                    gthr);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// Sample seeding of the tensor-core scan's shared thresholds.
//
// Before its first launch the scan's candidate lists have no threshold, so
// each list accepts every row of its first tiles and then compacts them, a
// cost per (query, list) that dominates a launch over few rows.  Instead,
// for every query: the FP32 Flat fast ranks (fast_rank, the SIMT scan's) of
// `samples` rows evenly spaced over the base, their kp-th best R, and the
// bound t = R + eps_sample + eps_scan rounded up.  The kp sample rows ranked
// at or below R have reference ranks within eps_sample of their sample ranks
// (the fast_eps bound holds for any float32 accumulation order) and scan
// ranks within eps_scan of their reference ranks, so at least kp rows have
// scan keys at or below pack(t, max key rank): an upper bound on the query's
// kp-th best scan key over all rows, which is all that the scan (a list
// drops only keys above it) and the merge's coverage check ask of gthr.
// Rows the filter excludes are not sampled.
// ---------------------------------------------------------------------------
constexpr int kSmpTile = 64;  // queries and sample rows per block
constexpr int kSmpK = 32;     // dimensions per shared-memory chunk
constexpr uint32_t kSmpNone = 0xffffffffu;

// ranks[q][s]: the ordered fast rank of query q against sample row s
// (kSmpNone: filtered out or not finite).  Block: a 64 x 64 tile, each
// thread 4 queries x 4 sample rows accumulated with FFMA over 32-dimension
// chunks staged in shared memory.
template <typename RowT>
__global__ void __launch_bounds__(256) sample_rank_kernel(
    const RowT* __restrict__ rows, int64_t n, int d, const float* __restrict__ row_n2,
    const uint32_t* __restrict__ bitmap, const float* __restrict__ qf,
    const float* __restrict__ q_n2, int nq, int metric, int samples,
    uint32_t* __restrict__ ranks) {
  __shared__ __align__(16) float qs[kSmpK][kSmpTile + 4];
  __shared__ __align__(16) float xs[kSmpK][kSmpTile + 4];
  __shared__ int64_t srow[kSmpTile];
  const int tid = threadIdx.x;
  const int q0 = blockIdx.x * kSmpTile, s0 = blockIdx.y * kSmpTile;
  if (tid < kSmpTile) srow[tid] = s0 + tid < samples ? (int64_t)(s0 + tid) * n / samples : -1;
  __syncthreads();
  const int tq = (tid >> 4) * 4, ts = (tid & 15) * 4;
  const int kk = tid & 31, rr = tid >> 5;  // loader: dimension kk of tile rows rr + 8 i
  float acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;
  for (int k0 = 0; k0 < d; k0 += kSmpK) {
    const int k = k0 + kk;
#pragma unroll
    for (int i = 0; i < kSmpTile / 8; ++i) {
      const int r = rr + 8 * i;
      const int q = q0 + r;
      qs[kk][r] = (q < nq && k < d) ? qf[(int64_t)q * d + k] : 0.f;
      const int64_t row = srow[r];
      xs[kk][r] = (row >= 0 && k < d) ? load_elem(rows, row * d + k) : 0.f;
    }
    __syncthreads();
#pragma unroll 8
    for (int c = 0; c < kSmpK; ++c) {
      const float4 a = *reinterpret_cast<const float4*>(&qs[c][tq]);
      const float4 b = *reinterpret_cast<const float4*>(&xs[c][ts]);
      const float av[4] = {a.x, a.y, a.z, a.w};
      const float bv[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int q = q0 + tq + i;
    if (q >= nq) continue;
    const float qn2 = q_n2[q];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int s = s0 + ts + j;
      if (s >= samples) continue;
      const int64_t row = srow[ts + j];
      uint32_t o = kSmpNone;
      if (bitmap_pass(bitmap, row)) {
        const float r = fast_rank(metric, acc[i][j], row_n2[row], qn2);
        if (finite_f(r)) o = float_to_ordered(r);
      }
      ranks[(int64_t)q * samples + s] = o;
    }
  }
}

// One warp per query: the kp-th smallest of its sample ranks (a radix
// select over the 32-bit ordered ranks, 8 bits per pass), then gthr[q] =
// min(gthr[q], pack(t, max key rank)) with t the bound above.
__global__ void __launch_bounds__(256) sample_seed_select_kernel(
    const uint32_t* __restrict__ ranks, int nq, int samples, int kp, int metric, int d,
    const float* __restrict__ q_n2, const unsigned* __restrict__ max_n2, int split,
    unsigned long long* __restrict__ gthr) {
  __shared__ int hist_all[8][256];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int q = blockIdx.x * 8 + warp;
  if (q >= nq) return;  // whole warps; nothing below synchronises the block
  int* hist = hist_all[warp];
  const uint32_t* v = ranks + (int64_t)q * samples;
  int cnt = 0;
  for (int i = lane; i < samples; i += 32) cnt += v[i] != kSmpNone;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) cnt += __shfl_xor_sync(kFullMask, cnt, o);
  if (cnt < kp) return;  // too few finite sample ranks: no seed
  uint32_t prefix = 0;
  int kth = kp;
#pragma unroll 1
  for (int shift = 24; shift >= 0; shift -= 8) {
    for (int b = lane; b < 256; b += 32) hist[b] = 0;
    __syncwarp();
    const uint32_t mask = shift == 24 ? 0u : (~0u << (shift + 8));
    for (int i = lane; i < samples; i += 32) {
      const uint32_t x = v[i];
      if ((x & mask) == prefix) atomicAdd(&hist[(x >> shift) & 0xff], 1);
    }
    __syncwarp();
    // Lane l owns bins 8 l .. 8 l + 7: the bin where the running count
    // reaches kth holds the next digit.
    int local[8], sum = 0;
#pragma unroll
    for (int b = 0; b < 8; ++b) {
      local[b] = hist[lane * 8 + b];
      sum += local[b];
    }
    int incl = sum;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int t = __shfl_up_sync(kFullMask, incl, o);
      if (lane >= o) incl += t;
    }
    const int excl = incl - sum;
    const unsigned owner = __ballot_sync(kFullMask, excl < kth && kth <= incl);
    const int src = __ffs(owner) - 1;
    int digit = 0, rem = kth - excl;
#pragma unroll
    for (int b = 0; b < 8; ++b) {
      if (rem > 0 && rem <= local[b]) {
        digit = lane * 8 + b;
        rem = -rem;  // found: later bins leave it alone
      } else if (rem > 0) {
        rem -= local[b];
      }
    }
    digit = __shfl_sync(kFullMask, digit, src);
    kth = -__shfl_sync(kFullMask, rem, src);
    prefix |= (uint32_t)digit << shift;
    __syncwarp();
  }
  // prefix is the kp-th smallest rank; kp <= cnt finite ranks sort before
  // every kSmpNone, so it is finite.
  if (lane == 0) {
    const float qn2 = q_n2[q], xn2 = ordered_to_float(*max_n2);
    const float e = __fadd_ru(fast_eps(metric, d, qn2, xn2, 0), fast_eps(metric, d, qn2, xn2, split));
    const float t = __fadd_ru(ordered_to_float(prefix), e);
    if (finite_f(t)) atomicMin(&gthr[q], (unsigned long long)pack_rank(t, 0xffffffffu));
  }
}

int flat_sample_seed_rows(int64_t n, int kp) {
  const int s = std::min(2048, std::max(1024, 8 * kp));
  return n >= 16 * (int64_t)s ? s : 0;
}

template <typename RowT>
cudaError_t launch_flat_sample_seed(const RowT* rows, int64_t n, int d, const float* row_n2,
                                    const uint32_t* bitmap, const float* qf, const float* q_n2,
                                    int nq, int metric, int kp, const unsigned* max_n2, int split,
                                    int samples, uint32_t* ranks, unsigned long long* gthr,
                                    cudaStream_t stream) {
  if (nq <= 0 || samples <= 0 || kp > samples) return cudaSuccess;
  const dim3 grid((unsigned)((nq + kSmpTile - 1) / kSmpTile),
                  (unsigned)((samples + kSmpTile - 1) / kSmpTile));
  sample_rank_kernel<RowT><<<grid, 256, 0, stream>>>(rows, n, d, row_n2, bitmap, qf, q_n2, nq,
                                                     metric, samples, ranks);
  sample_seed_select_kernel<<<(unsigned)((nq + 7) / 8), 256, 0, stream>>>(
      ranks, nq, samples, kp, metric, d, q_n2, max_n2, split, gthr);
  return cudaGetLastError();
}
template cudaError_t launch_flat_sample_seed<float>(const float*, int64_t, int, const float*,
                                                    const uint32_t*, const float*, const float*,
                                                    int, int, int, const unsigned*, int, int,
                                                    uint32_t*, unsigned long long*, cudaStream_t);
template cudaError_t launch_flat_sample_seed<__half>(const __half*, int64_t, int, const float*,
                                                     const uint32_t*, const float*, const float*,
                                                     int, int, int, const unsigned*, int, int,
                                                     uint32_t*, unsigned long long*, cudaStream_t);

int simt_cap_for(int kp) {
  // CAP must hold KP retained entries plus two tiles of appends.
  int need = kp + 2 * kSimtRT;
  int cap = 256;
  while (cap < need) cap <<= 1;
  return cap;
}

template <typename RowT>
cudaError_t launch_flat_scan_simt(const RowT* rows, int64_t n, int d, const float* row_n2,
                                  const uint32_t* keyrank, const float* qf, const float* q_n2,
                                  int nq, const uint32_t* bitmap, int metric, int num_parts,
                                  int kp, uint64_t* part_keys, int* part_counts,
                                  uint64_t* part_sat, int* q_flags, cudaStream_t stream) {
  return launch_scan_simt<RowT, FlatRanker>(rows, n, d, keyrank, qf, nq, bitmap,
                                            FlatRanker{metric, row_n2, q_n2}, num_parts, kp,
                                            part_keys, part_counts, part_sat, q_flags, stream);
}
template cudaError_t launch_flat_scan_simt<float>(const float*, int64_t, int, const float*,
                                                  const uint32_t*, const float*, const float*, int,
                                                  const uint32_t*, int, int, int, uint64_t*, int*,
                                                  uint64_t*, int*, cudaStream_t);
template cudaError_t launch_flat_scan_simt<__half>(const __half*, int64_t, int, const float*,
                                                   const uint32_t*, const float*, const float*,
                                                   int, const uint32_t*, int, int, int, uint64_t*,
                                                   int*, uint64_t*, int*, cudaStream_t);

int exact_cap_for(int kp) {
  int need = kp + 2 * 128;
  int cap = 512;
  while (cap < need) cap <<= 1;
  return cap;
}

template <typename RowT>
cudaError_t launch_flat_scan_exact(const RowT* rows, int64_t n, int d, const uint32_t* keyrank,
                                   const float* qf, const int* query_ids, int nlist,
                                   const uint32_t* bitmap, int metric, int num_parts, int kp,
                                   uint64_t* part_keys, int* part_counts, uint64_t* part_sat,
                                   int* q_flags, cudaStream_t stream) {
  FlatScorer<RowT> sc{metric, rows, qf, d, nullptr, nullptr};
  return launch_scan_exact(sc, n, keyrank, query_ids, nlist, bitmap, num_parts, kp, part_keys,
                           part_counts, part_sat, q_flags, stream);
}
template cudaError_t launch_flat_scan_exact<float>(const float*, int64_t, int, const uint32_t*,
                                                   const float*, const int*, int, const uint32_t*,
                                                   int, int, int, uint64_t*, int*, uint64_t*,
                                                   int*, cudaStream_t);
template cudaError_t launch_flat_scan_exact<__half>(const __half*, int64_t, int, const uint32_t*,
                                                    const float*, const int*, int,
                                                    const uint32_t*, int, int, int, uint64_t*,
                                                    int*, uint64_t*, int*, cudaStream_t);

template <typename RowT>
cudaError_t launch_flat_merge_rescore(const RowT* rows, int d, const uint32_t* pos_of_keyrank,
                                      const uint64_t* keys, const float* qf, const float* q_n2,
                                      const unsigned* max_n2, const int* query_ids, int nlist,
                                      int metric, int k, float radius, int exact_mode,
                                      const uint64_t* part_keys, const int* part_counts,
                                      const uint64_t* part_sat, int num_parts, int stride,
                                      uint64_t* out_keys, float* out_scores, int* out_counts,
                                      int* q_flags, cudaStream_t stream, int split_eps,
                                      const unsigned long long* gthr, const float* band) {
  FlatScorer<RowT> sc{metric, rows, qf, d, q_n2, max_n2, split_eps};
  return launch_merge_rescore(sc, pos_of_keyrank, keys, query_ids, nlist, k, radius, exact_mode,
                              part_keys, part_counts, part_sat, num_parts, stride, out_keys,
                              out_scores, out_counts, nullptr, q_flags, stream, gthr, band);
}
#define XVEC_FLAT_MERGE_INST(T)                                                                 \
  template cudaError_t launch_flat_merge_rescore<T>(                                            \
      const T*, int, const uint32_t*, const uint64_t*, const float*, const float*,              \
      const unsigned*, const int*, int, int, int, float, int, const uint64_t*, const int*,      \
      const uint64_t*, int, int, uint64_t*, float*, int*, int*, cudaStream_t, int,               \
      const unsigned long long*, const float*);
XVEC_FLAT_MERGE_INST(float)
XVEC_FLAT_MERGE_INST(__half)
#undef XVEC_FLAT_MERGE_INST

template <typename RowT>
cudaError_t launch_flat_band_prepare(const RowT* rows, int d, const float* qf, const float* q_n2,
                                     const unsigned* max_n2, int nq, int metric, int k,
                                     const uint64_t* part_keys, const int* part_counts,
                                     int num_parts, int stride, const unsigned long long* gthr,
                                     float* out, cudaStream_t stream, int split_eps) {
  FlatScorer<RowT> sc{metric, rows, qf, d, q_n2, max_n2, split_eps};
  return launch_band_prepare(sc, nq, k, part_keys, part_counts, num_parts, stride, gthr, out,
                             stream);
}
template cudaError_t launch_flat_band_prepare<float>(const float*, int, const float*,
                                                     const float*, const unsigned*, int, int, int,
                                                     const uint64_t*, const int*, int, int,
                                                     const unsigned long long*, float*,
                                                     cudaStream_t, int);
template cudaError_t launch_flat_band_prepare<__half>(const __half*, int, const float*,
                                                      const float*, const unsigned*, int, int, int,
                                                      const uint64_t*, const int*, int, int,
                                                      const unsigned long long*, float*,
                                                      cudaStream_t, int);

// Second half: from every shard's k best fast ranks and eps (recv [nranks]
// blocks of nq * (k + 1) floats), the query's band limit on this shard:
// F_k over all shards + the largest eps + this shard's eps (rounded up).
// Any k rows with fast rank <= F_k have reference scores <= F_k + max eps,
// so every row of the global top-k has a fast rank within the limit on its
// own shard.  Fewer than k finite ranks in all: NaN (no band).
__global__ void __launch_bounds__(256) band_limit_kernel(const float* __restrict__ recv,
                                                         int nranks, int nq, int k,
                                                         const float* __restrict__ own,
                                                         float* __restrict__ band) {
  extern __shared__ __align__(16) unsigned char limit_smem[];
  uint64_t* keys = reinterpret_cast<uint64_t*>(limit_smem);  // [nranks * k]
  __shared__ int hist[256];
  __shared__ int s_n;
  __shared__ unsigned s_eps;
  const int q = blockIdx.x;
  if (threadIdx.x == 0) {
    s_n = 0;
    s_eps = 0u;
  }
  __syncthreads();
  for (int r = 0; r < nranks; ++r) {
    const float* src = recv + ((int64_t)r * nq + q) * (k + 1);
    for (int i = threadIdx.x; i < k; i += blockDim.x) {
      const float v = src[i];
      if (v < INFINITY) keys[atomicAdd(&s_n, 1)] = (uint64_t)float_to_ordered(v) << 32;
    }
    if (threadIdx.x == 0) atomicMax(&s_eps, float_to_ordered(src[k]));
  }
  __syncthreads();
  const int m = s_n;
  if (m < k) {
    if (threadIdx.x == 0) band[q] = NAN;
    return;
  }
  const uint64_t fk = smem_radix_select(keys, m, k, 32, hist);
  if (threadIdx.x == 0) {
    const float eps_max = ordered_to_float(s_eps);
    const float eps_own = own[(int64_t)q * (k + 1) + k];
    band[q] = __fadd_ru(ordered_to_float((unsigned)(fk >> 32)), __fadd_ru(eps_max, eps_own));
  }
}

static cudaError_t launch_band_limit(const float* recv, int nranks, int nq, int k,
                                     const float* own, float* band, cudaStream_t stream) {
  if (nq <= 0) return cudaSuccess;
  if (!flat_band_supported(nranks, k)) return cudaErrorInvalidValue;
  const int smem = nranks * k * 8;
  cudaFuncSetAttribute(band_limit_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  band_limit_kernel<<<nq, 256, smem, stream>>>(recv, nranks, nq, k, own, band);
  return cudaGetLastError();
}

bool flat_band_supported(int nranks, int k) {
  return nranks >= 1 && k >= 1 && (int64_t)nranks * k <= kMergeSmemEntries;
}

cudaError_t launch_flat_band_limit(const float* recv, int nranks, int nq, int k,
                                   const float* own, float* band, cudaStream_t stream) {
  return launch_band_limit(recv, nranks, nq, k, own, band, stream);
}

}  // namespace xvec
