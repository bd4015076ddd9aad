// refine.cuh — exact float32 re-ranking of a small candidate list per query.
//
// OriginalVectorRefiner.Refine (internal/core/refiner.go:66-108): the
// candidates of the approximate stage (distinct keys, already filtered) are
// rescored with metric.Compute on the original float32 rows, then the k best
// under (score by metric, ties by ascending key) within the radius are kept.
// Used by the SQ8 refine stage and the RaBitQ refine stage.
#pragma once

#include "common.cuh"
#include "select.cuh"

namespace xvec {

constexpr int kRefineMax = 2048;  // candidates per query (MaxHNSWEFSearch)

// Scores of a stage's output rows turned into ranks (lower is better) in
// place: -score for inner product, unchanged otherwise.
static __global__ void scores_to_ranks_kernel(float* scores, const int* counts, int nq,
                                              int stride, int metric) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (int64_t)nq * stride) return;
  const int q = (int)(i / stride), j = (int)(i - (int64_t)q * stride);
  if (j < counts[q]) scores[i] = rank_from_score(metric, scores[i]);
}

// One block (256 threads) per query; N >= the candidate count, a power of two.
// stage_pos/stage_counts: per query the positions of the approximate stage's
// results (stride `stage_k`).
template <int N>
__global__ void __launch_bounds__(256) refine_kernel(
    const float* __restrict__ rows, int d, int metric, const float* __restrict__ queries,
    const uint32_t* __restrict__ stage_pos, const int* __restrict__ stage_counts, int stage_k,
    const uint32_t* __restrict__ keyrank, const uint32_t* __restrict__ pos_of_keyrank,
    const uint64_t* __restrict__ keys, int k, float radius,
    uint64_t* __restrict__ out_keys, float* __restrict__ out_scores, int* __restrict__ out_counts,
    int* __restrict__ q_flags) {
  __shared__ uint64_t cand[N];
  const int qi = blockIdx.x;
  const int c = stage_counts[qi];
  if (c <= 0) {
    if (threadIdx.x == 0 && c == 0) out_counts[qi] = 0;
    return;
  }
  const int n = min(c, N);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const float* q = queries + (int64_t)qi * d;
  // d >= 16: each half-warp scores its own candidate (an odd last one is
  // scored by both halves and written by one).
  const bool pairs = d >= 16;
  const int step = pairs ? 2 : 1;
  for (int i0 = warp * step; i0 < n; i0 += (blockDim.x >> 5) * step) {
    const int i = pairs ? min(i0 + (lane >> 4), n - 1) : i0;
    const uint32_t pos = stage_pos[(int64_t)qi * stage_k + i];
    const float s = warp_reference_score(metric, rows + (int64_t)pos * d, q, d);
    if ((lane & (pairs ? 15 : 31)) == 0 && (!pairs || i0 + (lane >> 4) < n)) {
      if (!finite_f(s)) atomicOr(&q_flags[qi], 4);
      cand[i] = pack_rank(rank_from_score(metric, s), keyrank[pos]);
    }
  }
  __syncthreads();
  // (rank, key rank) ascending is the reference order.
  block_sort_u64<N>(cand, n);
  if (threadIdx.x < 32) {
    int count = 0;
    for (int base = 0; base < n && count < k; base += 32) {
      const int i = base + lane;
      bool in = i < n;
      float s = 0.f;
      if (in) {
        s = score_from_rank(metric, rank_of(cand[i]));
        in = within_radius(metric, s, radius);
      }
      const unsigned m = __ballot_sync(kFullMask, in);
      const int run = (m == kFullMask) ? 32 : __ffs(~m) - 1;
      if (lane < run && count + lane < k) {
        const uint32_t pos = pos_of_keyrank[pos_of(cand[i])];
        out_keys[(int64_t)qi * k + count + lane] = keys[pos];
        out_scores[(int64_t)qi * k + count + lane] = s;
      }
      count = min(k, count + run);
      if (run < 32) break;
    }
    if (lane == 0) out_counts[qi] = count;
  }
}

// Launches refine_kernel with the smallest shared buffer that holds
// `stage_k` (<= kRefineMax) candidates.
inline cudaError_t launch_refine(const float* rows, int d, int metric, const float* queries,
                                 int nq, const uint32_t* stage_pos, const int* stage_counts,
                                 int stage_k, const uint32_t* keyrank,
                                 const uint32_t* pos_of_keyrank, const uint64_t* keys, int k,
                                 float radius, uint64_t* out_keys, float* out_scores,
                                 int* out_counts, int* q_flags, cudaStream_t s) {
  if (nq <= 0) return cudaSuccess;
#define XVEC_REFINE_CASE(NN)                                                                  \
  if (stage_k <= NN) {                                                                        \
    refine_kernel<NN><<<nq, 256, 0, s>>>(rows, d, metric, queries, stage_pos, stage_counts,   \
                                         stage_k, keyrank, pos_of_keyrank, keys, k, radius,   \
                                         out_keys, out_scores, out_counts, q_flags);          \
    return cudaGetLastError();                                                                \
  }
  XVEC_REFINE_CASE(128)
  XVEC_REFINE_CASE(512)
  XVEC_REFINE_CASE(1024)
  XVEC_REFINE_CASE(2048)
#undef XVEC_REFINE_CASE
  return cudaErrorInvalidValue;
}

}  // namespace xvec
