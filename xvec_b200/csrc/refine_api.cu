// refine_api.cu — the two halves of a refined search as separate calls, for
// refined searches over several shards.
//
// RefinedSearch (internal/core/refiner.go:133-166) takes the approximate
// stage's RefinementCandidateCount best candidates over the whole index and
// rescores exactly those with DenseRefiner.Refine (refiner.go:30-33, 66-108);
// the HNSW-RaBitQ search does the same with its max(TopK, EF) best estimates
// (hnsw_rabitq.go:584, 780-801).  With the rows split over shards the global
// candidate list is the merge of the shards' candidate lists, so a sharded
// refined search is: candidates on every shard, one exchange and merge (by
// rank, ties by key), the refine of the merged list on every shard (each
// shard scores the keys it holds), a second exchange and merge.
//
//   xvec_gpu_index_candidates_device  the approximate stage: keys and ranks
//   xvec_gpu_index_refine_device      exact float32 scores of given keys
#include <algorithm>
#include <vector>

#include "capi_internal.h"
#include "common.cuh"
#include "flat_kernels.cuh"
#include "index_kernels.cuh"
#include "refine.cuh"

namespace xvec {

xvec_gpu_status validate_search(xvec_gpu_index* idx, int nq, const xvec_gpu_search_opts* o);

namespace {

// Positions of the candidate keys this index holds, per query (one block per
// query): a binary search over the keys in ascending order (key rank r is at
// position pos_of_kr[r]).  Failed queries (negative counts) pass through.
__global__ void keys_to_positions_kernel(const uint64_t* __restrict__ cand_keys, int stride,
                                         const int* __restrict__ cand_counts,
                                         const uint64_t* __restrict__ keys,
                                         const uint32_t* __restrict__ pos_of_kr, int64_t n,
                                         uint32_t* __restrict__ positions,
                                         int* __restrict__ counts) {
  __shared__ int s_count;
  const int q = blockIdx.x;
  const int c = cand_counts[q];
  if (threadIdx.x == 0) s_count = 0;
  __syncthreads();
  for (int i = threadIdx.x; i < c && i < stride; i += blockDim.x) {
    const uint64_t key = cand_keys[(int64_t)q * stride + i];
    int64_t lo = 0, hi = n;
    while (lo < hi) {
      const int64_t mid = (lo + hi) >> 1;
      if (keys[pos_of_kr[mid]] < key) lo = mid + 1;
      else hi = mid;
    }
    if (lo < n && keys[pos_of_kr[lo]] == key) {
      const int slot = atomicAdd(&s_count, 1);
      positions[(int64_t)q * stride + slot] = pos_of_kr[lo];
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) counts[q] = c < 0 ? c : s_count;
}

// Final per-query status: the candidates' (negative counts), then the
// query's validation (metric.Compute(q, q)), then a non-finite exact score.
__global__ void refine_status_kernel(const int* cand_counts, const int* q_status,
                                     const int* q_flags, int nq, int* out_counts) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= nq) return;
  if (cand_counts[i] < 0) out_counts[i] = cand_counts[i];
  else if (q_status[i]) out_counts[i] = -q_status[i];
  else if (q_flags[i] & 4) out_counts[i] = -(int)XVEC_GPU_NON_FINITE;
}

bool has_float_rows(const xvec_gpu_index* idx) {
  return !(idx->desc.kind == XVEC_INDEX_FLAT && idx->desc.storage == XVEC_STORAGE_FP16);
}

}  // namespace
}  // namespace xvec

using namespace xvec;

extern "C" int32_t xvec_gpu_index_candidate_count(const xvec_gpu_index* idx,
                                                  const xvec_gpu_search_opts* opts) {
  if (!idx || !opts) return 0;
  switch (idx->desc.kind) {
    case XVEC_INDEX_SQ8_FLAT:
    case XVEC_INDEX_SQ4_FLAT:
    case XVEC_INDEX_IVF_SQ8:
    case XVEC_INDEX_IVF_SQ4:
      return sq8_candidate_count(*opts);
    default:
      break;
  }
  if (idx->desc.kind == XVEC_INDEX_RABITQ) return rabitq_candidate_count(*opts);
  return 0;
}

extern "C" xvec_gpu_status xvec_gpu_index_candidates_device(xvec_gpu_index* idx,
                                                            const void* d_queries, int32_t nq,
                                                            const xvec_gpu_search_opts* opts,
                                                            uint64_t* d_keys, float* d_ranks,
                                                            int32_t* d_counts) {
  xvec_gpu_status st = validate_search(idx, nq, opts);
  if (st) return st;
  const int c = xvec_gpu_index_candidate_count(idx, opts);
  if (c <= 0)
    return set_error("the options ask for no refinement of this index kind"),
           XVEC_GPU_INVALID_ARGUMENT;
  if (nq == 0) return XVEC_GPU_OK;
  if (!d_queries || !d_keys || !d_ranks || !d_counts)
    return set_error("nil buffer"), XVEC_GPU_INVALID_ARGUMENT;
  std::shared_lock<std::shared_mutex> lock(idx->mu);
  cudaSetDevice(idx->device);
  cudaStream_t s = static_cast<cudaStream_t>(opts->stream);
  std::vector<int> statuses;
  const float* q = static_cast<const float*>(d_queries);
  if (idx->desc.kind == XVEC_INDEX_SQ8_FLAT || idx->desc.kind == XVEC_INDEX_SQ4_FLAT)
    return sq8_search_impl(idx, q, nq, *opts, opts->filter_bitmap, d_keys, d_ranks, d_counts, s,
                           &statuses, true);
  if (idx->desc.kind == XVEC_INDEX_IVF_SQ8 || idx->desc.kind == XVEC_INDEX_IVF_SQ4)
    return ivf_sq8_search_impl(idx, q, nq, *opts, opts->filter_bitmap, d_keys, d_ranks,
                               d_counts, s, &statuses, true);
  return rabitq_search_impl(idx, q, nq, *opts, opts->filter_bitmap, d_keys, d_ranks, d_counts, s,
                            &statuses, true);
}

extern "C" xvec_gpu_status xvec_gpu_index_refine_device(
    xvec_gpu_index* idx, const float* d_queries, int32_t nq, const uint64_t* d_cand_keys,
    int32_t cand_stride, const int32_t* d_cand_counts, int32_t top_k, float radius,
    void* stream, uint64_t* d_keys, float* d_scores, int32_t* d_counts) {
  if (!idx) return set_error("nil index"), XVEC_GPU_INVALID_ARGUMENT;
  if (nq < 0 || top_k <= 0 || top_k > 1024 || cand_stride <= 0 || cand_stride > kRefineMax)
    return set_error("invalid refine arguments (top_k %d, candidate stride %d)", top_k,
                     cand_stride),
           XVEC_GPU_INVALID_ARGUMENT;
  if (!(radius >= 0) || std::isinf(radius))
    return set_error("core: radius must be finite and non-negative"), XVEC_GPU_INVALID_ARGUMENT;
  if (!has_float_rows(idx))
    return set_error("refinement needs float32 original rows"), XVEC_GPU_UNSUPPORTED;
  if (nq == 0) return XVEC_GPU_OK;
  if (!d_queries || !d_cand_keys || !d_cand_counts || !d_keys || !d_scores || !d_counts)
    return set_error("nil buffer"), XVEC_GPU_INVALID_ARGUMENT;
  std::shared_lock<std::shared_mutex> lock(idx->mu);
  cudaSetDevice(idx->device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int d = idx->desc.dimension, metric = idx->desc.metric;
  xvec_gpu_status st;
  Scratch pos, pcounts, qf, qn2, qaux, qstatus, qflags;
  if ((st = pos.alloc((size_t)nq * cand_stride * 4, s)) ||
      (st = pcounts.alloc((size_t)nq * 4, s)) || (st = qf.alloc((size_t)nq * d * 4, s)) ||
      (st = qn2.alloc((size_t)nq * 4, s)) || (st = qaux.alloc((size_t)nq * 4, s)) ||
      (st = qstatus.alloc((size_t)nq * 4, s)) || (st = qflags.alloc((size_t)nq * 4, s)))
    return st;
  XVEC_CUDA(cudaMemsetAsync(qflags.ptr, 0, (size_t)nq * 4, s));
  XVEC_CUDA(cudaMemsetAsync(d_counts, 0, (size_t)nq * 4, s));
  // metric.Compute(q, q) must be finite (topk.go:92-94).
  launch_prep_queries<float>(d_queries, nq, d, metric, qf.as<float>(), qn2.as<float>(),
                             qaux.as<float>(), qstatus.as<int>(), s);
  XVEC_LAUNCHED();
  if (idx->n > 0) {
    keys_to_positions_kernel<<<nq, 256, 0, s>>>(d_cand_keys, cand_stride, d_cand_counts,
                                                idx->keys.as<uint64_t>(),
                                                idx->pos_of_kr.as<uint32_t>(), idx->n,
                                                pos.as<uint32_t>(), pcounts.as<int>());
    XVEC_LAUNCHED();
    XVEC_CUDA(launch_refine(idx->rows.as<float>(), d, metric, d_queries, nq, pos.as<uint32_t>(),
                            pcounts.as<int>(), cand_stride, idx->keyrank.as<uint32_t>(),
                            idx->pos_of_kr.as<uint32_t>(), idx->keys.as<uint64_t>(), top_k,
                            radius, d_keys, d_scores, d_counts, qflags.as<int>(), s));
    count_launches(1);
  }
  refine_status_kernel<<<(nq + 255) / 256, 256, 0, s>>>(d_cand_counts, qstatus.as<int>(),
                                                        qflags.as<int>(), nq, d_counts);
  XVEC_LAUNCHED();
  XVEC_CUDA(cudaGetLastError());
  XVEC_CUDA(cudaStreamSynchronize(s));
  return XVEC_GPU_OK;
}
