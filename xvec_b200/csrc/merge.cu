// merge.cu — cross-shard merge of per-shard top-k lists and library counters.
//
// MergeSearchResults (internal/core/query.go:154-191): the k best results of
// all lists under resultBetter (topk.go:271-276: score by metric, ties by the
// ascending key).  Used after the NCCL allgather of a sharded search.
#include <atomic>
#include <mutex>

#include "capi_internal.h"
#include "common.cuh"

namespace xvec {

namespace {
std::atomic<int64_t> g_searches{0}, g_queries{0}, g_launches{0}, g_exact{0}, g_tensor{0},
    g_stream{0};
std::mutex g_ms_mu;
double g_scan_ms = 0, g_search_ms = 0;
std::atomic<int> g_timing{0};
}  // namespace

void count_launches(int64_t n) { g_launches.fetch_add(n, std::memory_order_relaxed); }
void count_tensor_scan() { g_tensor.fetch_add(1); }
void count_stream_scan() { g_stream.fetch_add(1); }
thread_local int g_nested = 0;
void nested_search_enter() { ++g_nested; }
void nested_search_leave() { --g_nested; }

void count_search(int64_t queries, int64_t exact_queries, double scan_ms, double search_ms) {
  if (g_nested > 0) return;
  g_searches.fetch_add(1);
  g_queries.fetch_add(queries);
  g_exact.fetch_add(exact_queries);
  if (scan_ms > 0 || search_ms > 0) {
    std::lock_guard<std::mutex> lock(g_ms_mu);
    g_scan_ms += scan_ms;
    g_search_ms += search_ms;
  }
}
bool timing_enabled() { return g_timing.load() != 0; }

// One block per query: gather the valid entries of every part, bitonic-sort
// them by (ordered rank, key) and keep the first top_k.  Part p's lists start
// p * key_stride / score_stride / count_stride elements into keys / scores /
// counts (query q's list at q * k inside its part).
__global__ void merge_results_kernel(int metric, int k, int nq, int parts, int n_pow2,
                                     const uint64_t* __restrict__ keys, int64_t key_stride,
                                     const float* __restrict__ scores, int64_t score_stride,
                                     const int* __restrict__ counts, int64_t count_stride,
                                     uint64_t* __restrict__ out_keys,
                                     float* __restrict__ out_scores, int* __restrict__ out_counts) {
  extern __shared__ __align__(16) unsigned char smem[];
  uint64_t* skey = reinterpret_cast<uint64_t*>(smem);
  uint32_t* srank = reinterpret_cast<uint32_t*>(skey + n_pow2);
  float* sscore = reinterpret_cast<float*>(srank + n_pow2);
  __shared__ int s_n, s_err;
  const int q = blockIdx.x;
  if (threadIdx.x == 0) {
    s_n = 0;
    // A query that failed on a shard (count = -status) fails as a whole; the
    // shards validate a query the same way, so the first one's status stands.
    s_err = 0;
    for (int p = 0; p < parts && s_err == 0; ++p) {
      const int c = counts[(int64_t)p * count_stride + q];
      if (c < 0) s_err = c;
    }
    if (s_err) out_counts[q] = s_err;
  }
  __syncthreads();
  if (s_err) return;
  for (int i = threadIdx.x; i < parts * k; i += blockDim.x) {
    const int p = i / k, j = i - p * k;
    const int c = counts[(int64_t)p * count_stride + q];
    if (j < c) {
      const int64_t src = (int64_t)q * k + j;
      const int slot = atomicAdd(&s_n, 1);
      const float sc = scores[(int64_t)p * score_stride + src];
      skey[slot] = keys[(int64_t)p * key_stride + src];
      sscore[slot] = sc;
      // + 0.f: -0 and +0 rank equal (the reference compares scores with ==).
      srank[slot] = float_to_ordered(rank_from_score(metric, sc) + 0.f);
    }
  }
  __syncthreads();
  const int n = s_n;
  for (int i = n + threadIdx.x; i < n_pow2; i += blockDim.x) {
    skey[i] = ~0ull;
    srank[i] = 0xffffffffu;
    sscore[i] = 0.f;
  }
  __syncthreads();
  for (int kk = 2; kk <= n_pow2; kk <<= 1) {
    for (int jj = kk >> 1; jj > 0; jj >>= 1) {
      for (int i = threadIdx.x; i < n_pow2; i += blockDim.x) {
        const int ixj = i ^ jj;
        if (ixj > i) {
          const bool up = (i & kk) == 0;
          const bool gt = srank[i] != srank[ixj] ? srank[i] > srank[ixj] : skey[i] > skey[ixj];
          if (gt == up) {
            uint32_t r = srank[i]; srank[i] = srank[ixj]; srank[ixj] = r;
            uint64_t kv = skey[i]; skey[i] = skey[ixj]; skey[ixj] = kv;
            float sv = sscore[i]; sscore[i] = sscore[ixj]; sscore[ixj] = sv;
          }
        }
      }
      __syncthreads();
    }
  }
  const int c = min(n, k);
  for (int i = threadIdx.x; i < c; i += blockDim.x) {
    out_keys[(int64_t)q * k + i] = skey[i];
    out_scores[(int64_t)q * k + i] = sscore[i];
  }
  if (threadIdx.x == 0) out_counts[q] = c;
}

xvec_gpu_status launch_merge_results(int metric, int top_k, int nq, int parts,
                                     const uint64_t* keys, int64_t key_stride,
                                     const float* scores, int64_t score_stride,
                                     const int* counts, int64_t count_stride,
                                     uint64_t* out_keys, float* out_scores, int* out_counts,
                                     cudaStream_t stream) {
  if (metric < XVEC_METRIC_L2 || metric > XVEC_METRIC_MIPSL2 || top_k <= 0 || nq < 0 ||
      parts <= 0)
    return set_error("invalid merge arguments"), XVEC_GPU_INVALID_ARGUMENT;
  int64_t entries = (int64_t)parts * top_k;
  int n_pow2 = 1;
  while (n_pow2 < entries) n_pow2 <<= 1;
  if (n_pow2 > 8192)
    return set_error("merge of %lld entries per query exceeds 8192", (long long)entries),
           XVEC_GPU_INVALID_ARGUMENT;
  if (nq == 0) return XVEC_GPU_OK;
  const size_t smem = (size_t)n_pow2 * 16;
  cudaFuncSetAttribute(merge_results_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                       (int)smem);
  merge_results_kernel<<<nq, 256, smem, stream>>>(metric, top_k, nq, parts, n_pow2, keys,
                                                  key_stride, scores, score_stride, counts,
                                                  count_stride, out_keys, out_scores,
                                                  out_counts);
  XVEC_LAUNCHED();
  XVEC_CUDA(cudaGetLastError());
  return XVEC_GPU_OK;
}

}  // namespace xvec

using namespace xvec;

extern "C" void xvec_gpu_stats_enable_timing(int32_t enabled) { g_timing.store(enabled ? 1 : 0); }

extern "C" void xvec_gpu_get_stats(xvec_gpu_stats* out) {
  if (!out) return;
  out->searches = g_searches.load();
  out->queries = g_queries.load();
  out->kernel_launches = g_launches.load();
  out->exact_queries = g_exact.load();
  out->tensor_scans = g_tensor.load();
  out->stream_scans = g_stream.load();
  std::lock_guard<std::mutex> lock(g_ms_mu);
  out->scan_ms = g_scan_ms;
  out->search_ms = g_search_ms;
}

extern "C" void xvec_gpu_reset_stats(void) {
  g_searches = 0;
  g_queries = 0;
  g_launches = 0;
  g_exact = 0;
  g_tensor = 0;
  g_stream = 0;
  std::lock_guard<std::mutex> lock(g_ms_mu);
  g_scan_ms = 0;
  g_search_ms = 0;
}

extern "C" xvec_gpu_status xvec_gpu_merge_results_device(int32_t device, int32_t metric,
                                                         int32_t top_k, int32_t nq, int32_t parts,
                                                         const uint64_t* d_keys,
                                                         const float* d_scores,
                                                         const int32_t* d_counts,
                                                         uint64_t* d_out_keys, float* d_out_scores,
                                                         int32_t* d_out_counts, void* stream) {
  if (nq > 0 && parts > 0 && top_k > 0) cudaSetDevice(device);
  return launch_merge_results(metric, top_k, nq, parts, d_keys, (int64_t)nq * top_k, d_scores,
                              (int64_t)nq * top_k, d_counts, nq, d_out_keys, d_out_scores,
                              d_out_counts, static_cast<cudaStream_t>(stream));
}
