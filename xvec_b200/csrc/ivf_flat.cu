// ivf_flat.cu — IVF search that exact-scores the original rows of the probed
// lists (the IVFIndex of internal/core/ivf.go).
//
//   probe   probedListsLocked (ivf.go:524-561): the nprobe best centroids
//           under the index metric, ties to the lower index; the Flat path
//           over the centroids, except for cosine, whose probe uses the
//           cached magnitudes (CosineDistanceWithMagnitudesPrevalidated,
//           distance_prevalidated.go:57-68) and is scored exactly here.
//   scan    searchIVF (ivf.go:427-493) → topKPrevalidatedCandidateBatches-
//           WithOptions (topk.go:171-237) over the positions of the probed
//           lists: the prevalidated metric, or for cosine the cached-
//           magnitude formula (ivf.go:469-478, magnitudes as
//           L2MagnitudePrevalidated, distance_prevalidated.go:46-53); filter
//           before scoring, ties by key.
//   insert  the nearest centroid (KMeansModel.Nearest, kmeans.go:169-175).
// The list scan (ivf_scan.cuh, shared with the INT8 IVF of sq8.cu) is one
// 16-warp block per query over its probed lists (positions in list order,
// rows gathered by position): each lane ranks one row with a float32 dot
// product (the fast rank of the Flat path, within the
// Flat error bound of the reference score), keys below the lists' shared
// threshold go to per-warp lists, and the merge rescores the candidates in
// the reference's arithmetic.  Queries the fast pass cannot settle are
// rescanned with reference-order scores (a warp per row).
#include <algorithm>
#include <cmath>
#include <mutex>
#include <vector>

#include "capi_internal.h"
#include "common.cuh"
#include "flat_kernels.cuh"
#include "index_kernels.cuh"
#include "ivf_scan.cuh"
#include "pipeline.cuh"

namespace xvec {


namespace {

inline unsigned blocks_of(int64_t n, int t = 256) { return (unsigned)((n + t - 1) / t); }

// L2MagnitudePrevalidated from the reference-order InnerProduct(v, v).
__device__ __forceinline__ float ivf_magnitude(float n2) {
  return __double2float_rn(__dsqrt_rn((double)fmaxf(n2, 0.f)));
}

// CosineDistanceWithMagnitudesPrevalidated from InnerProduct(left, right).
__device__ __forceinline__ float ivf_cosine(float inner, float lm, float rm) {
  if (lm == 0.f && rm == 0.f) return 0.f;
  if (lm == 0.f || rm == 0.f) return 1.f;
  float c = __fdiv_rn(inner, __fmul_rn(lm, rm));
  c = go_minf(1.f, go_maxf(-1.f, c));
  return __fsub_rn(1.f, c);
}

// The IVF score of one (row, query) pair on every lane of the warp.
__device__ __forceinline__ float ivf_reference_score(int metric, const float* x, float x_n2,
                                                     const float* q, float q_n2, int d) {
  if (metric == kMetricCosine) {
    float s0, s1, s2;
    warp_reference_sums<1>(x, q, d, &s0, &s1, &s2);
    return ivf_cosine(s0, ivf_magnitude(x_n2), ivf_magnitude(q_n2));
  }
  return warp_reference_score(metric, x, q, d);
}

struct IvfFlatScorer {
  int metric;
  const float* rows;
  const float* row_n2;
  const float* qf;
  const float* q_n2;
  const unsigned* max_n2_ordered;
  int d;
  __device__ float score(int qi, int64_t pos) const {
    return ivf_reference_score(metric, rows + pos * d, row_n2[pos], qf + (int64_t)qi * d,
                               q_n2[qi], d);
  }
  __device__ bool half_warp() const { return d >= 16; }
  __device__ float eps(int qi) const {
    // The Flat bound covers the float32 dot against either cosine formula.
    const float u = 5.9604645e-8f, g = 4.f * (float)(d + 8) * u;
    const float qn = sqrtf(q_n2[qi]), xn = sqrtf(ordered_to_float(*max_n2_ordered));
    switch (metric) {
      case kMetricL2: return g * (xn + qn) * (xn + qn) * 1.0001f;
      case kMetricIP: return g * xn * qn * 1.0001f + 1e-30f;
      case kMetricCosine: return g * 2.f;
      default: return g * 4.f;
    }
  }
  __device__ int error_flag(float) const { return 4; }
  __device__ float output(float r) const { return score_from_rank(metric, r); }
  __device__ bool keep(float out, float radius) const { return within_radius(metric, out, radius); }
};

// The cosine probe: every (query, centroid) scored with the cached-magnitude
// formula, a warp per pair; keys are centroid indexes, ranks the distances
// themselves (lower is better).
struct IvfProbeScorer {
  int metric;  // kMetricL2: the ordering of the ranks
  const float* cents;
  const float* cent_n2;
  const float* qf;
  const float* q_n2;
  int d;
  __device__ float score(int qi, int64_t c) const {
    return ivf_reference_score(kMetricCosine, cents + c * d, cent_n2[c], qf + (int64_t)qi * d,
                               q_n2[qi], d);
  }
  __device__ bool half_warp() const { return d >= 16; }
  __device__ float eps(int) const { return 0.f; }
  __device__ int error_flag(float) const { return 4; }
  __device__ float output(float r) const { return r; }
  __device__ bool keep(float, float) const { return true; }
};

// The IVF list scan over float32 rows (ivf_scan.cuh): the query staged in
// shared memory, the fast rank of the Flat path (a float32 dot product), the
// IVF reference score.
struct IvfFlatPolicy {
  int metric;
  const float* rows;
  const float* row_n2;
  const float4* list_rows;  // list-major interleaved rows (d % 4 == 0), or null
  const float* list_n2;     // ||x||^2 in list order (with list_rows)
  const float* qf;
  const float* q_n2;
  int d;
  __host__ __device__ int smem_bytes(int dim) const { return dim * 4; }
  __device__ void stage(int q, unsigned char* smem) const {
    float* sq = reinterpret_cast<float*>(smem);
    const float* qv = qf + (int64_t)q * d;
    for (int i = threadIdx.x; i < d; i += blockDim.x) sq[i] = qv[i];
  }
  __device__ float fast_rank(int q, int64_t idx, uint32_t pos, const unsigned char* smem) const {
    const float* x = rows + (int64_t)pos * d;
    const float* sq = reinterpret_cast<const float*>(smem);
    float dot = 0.f;
    if (list_rows) {
      // Chunk c of list entry idx: coalesced across the warp's 32 entries.
      const int C = d / 4;
      const float4* src = list_rows + (idx >> 5) * C * 32 + (idx & 31);
      const float4* q4 = reinterpret_cast<const float4*>(sq);
      float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
      for (int c = 0; c < C; ++c) {
        const float4 xv = __ldg(src + c * 32), qq = q4[c];
        a0 = fmaf(xv.x, qq.x, a0);
        a1 = fmaf(xv.y, qq.y, a1);
        a2 = fmaf(xv.z, qq.z, a2);
        a3 = fmaf(xv.w, qq.w, a3);
      }
      dot = (a0 + a1) + (a2 + a3);
      return ::xvec::fast_rank(metric, dot, __ldg(list_n2 + idx), q_n2[q]);
    }
    if ((d & 3) == 0) {
      const float4* x4 = reinterpret_cast<const float4*>(x);
      const float4* q4 = reinterpret_cast<const float4*>(sq);
      float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
      for (int i = 0; i < d / 4; ++i) {
        const float4 xv = __ldg(x4 + i), qq = q4[i];
        a0 = fmaf(xv.x, qq.x, a0);
        a1 = fmaf(xv.y, qq.y, a1);
        a2 = fmaf(xv.z, qq.z, a2);
        a3 = fmaf(xv.w, qq.w, a3);
      }
      dot = (a0 + a1) + (a2 + a3);
    } else {
      for (int i = 0; i < d; ++i) dot = fmaf(__ldg(x + i), sq[i], dot);
    }
    return ::xvec::fast_rank(metric, dot, row_n2[pos], q_n2[q]);
  }
  __device__ float exact_score(int q, uint32_t pos, const unsigned char* smem) const {
    return ivf_reference_score(metric, rows + (int64_t)pos * d, row_n2[pos],
                               reinterpret_cast<const float*>(smem), q_n2[q], d);
  }
};

__global__ void iota64_kernel(uint64_t* keys, uint32_t* ranks, int n) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) {
    keys[i] = (uint64_t)i;
    ranks[i] = (uint32_t)i;
  }
}

__global__ void clear_bits_kernel(const int* ids, int n, int bits, int* q_flags) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) q_flags[ids[i]] &= ~bits;
}

__global__ void ivf_status_kernel(const int* q_status, const int* q_flags, int nq,
                                  int* out_counts) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= nq) return;
  int st = q_status[i];
  if (st == 0 && (q_flags[i] & 4)) st = XVEC_GPU_NON_FINITE;
  if (st != 0) out_counts[i] = -st;
}

}  // namespace

// ---------------------------------------------------------------------------
// Index hooks.
// ---------------------------------------------------------------------------
xvec_gpu_status ivf_flat_reserve(xvec_gpu_index* idx, int64_t cap, cudaStream_t s) {
  return idx->row_list.reserve((size_t)cap * 4, (size_t)idx->n * 4, s);
}

xvec_gpu_status ivf_flat_commit(xvec_gpu_index* idx, int64_t old_n, int64_t m, cudaStream_t s) {
  const int d = idx->desc.dimension;
  if (idx->given_lists) {
    // Lists given by the caller (checked against nlist on the host).
    XVEC_CUDA(cudaMemcpyAsync(idx->row_list.as<int32_t>() + old_n, idx->given_lists,
                              (size_t)m * 4, cudaMemcpyDeviceToDevice, s));
  } else {
    const xvec_gpu_status st = assign_rows(idx->probe_index, idx->rows.as<float>() + old_n * d,
                                           m, d, idx->row_list.as<int32_t>() + old_n, nullptr, s);
    if (st) return st;
  }
  idx->lists_dirty = true;
  return XVEC_GPU_OK;
}

// The probe of the IVF kinds (probedListsLocked, ivf.go:524-561): per query
// the nprobe best centroid indexes (pkeys [nq][nprobe], pcounts [nq]) and the
// per-query status so far (h_status).  qf / qn2 / q_status: launch_prep_queries
// of the raw queries (the cosine probe scores them with the cached
// magnitudes; a non-finite probe score sets flag 4 of the query).
xvec_gpu_status ivf_probe(xvec_gpu_index* idx, const float* d_q, int nq, int nprobe,
                          const float* qf, const float* qn2, const int* q_status,
                          uint64_t* pkeys, float* pscores, int* pcounts, int* q_flags,
                          std::vector<int>* h_status, cudaStream_t s) {
  const int d = idx->desc.dimension, metric = idx->desc.metric, nlist = idx->nlist;
  xvec_gpu_status st;
  h_status->resize(nq);
  if (metric == XVEC_METRIC_COSINE) {
    const xvec_gpu_index* pi = idx->probe_index;
    Scratch ckeys, cranks, lkeys, lcounts, lsat;
    const int parts = std::max(1, std::min(flat_merge_capacity() / std::max(nprobe, 32),
                                           (nlist + 255) / 256));
    int pkp = 32;
    while (pkp < nprobe) pkp <<= 1;
    if ((int64_t)parts * pkp > flat_merge_capacity() || exact_cap_for(pkp) > 8192)
      return set_error("nprobe %d too large for the cosine probe", nprobe), XVEC_GPU_UNSUPPORTED;
    if ((st = ckeys.alloc((size_t)nlist * 8, s)) || (st = cranks.alloc((size_t)nlist * 4, s)) ||
        (st = lkeys.alloc((size_t)nq * parts * pkp * 8, s)) ||
        (st = lcounts.alloc((size_t)nq * parts * 4, s)) ||
        (st = lsat.alloc((size_t)nq * parts * 8, s)))
      return st;
    iota64_kernel<<<blocks_of(nlist), 256, 0, s>>>(ckeys.as<uint64_t>(), cranks.as<uint32_t>(),
                                                   nlist);
    XVEC_LAUNCHED();
    const IvfProbeScorer msc{kMetricL2, pi->rows.as<float>(), pi->row_n2.as<float>(), qf, qn2, d};
    XVEC_CUDA(launch_scan_exact(msc, nlist, cranks.as<uint32_t>(), nullptr, nq, nullptr, parts,
                                pkp, lkeys.as<uint64_t>(), lcounts.as<int>(),
                                lsat.as<uint64_t>(), q_flags, s));
    XVEC_CUDA(launch_merge_rescore(msc, cranks.as<uint32_t>(), ckeys.as<uint64_t>(), nullptr, nq,
                                   nprobe, 0.f, 1, lkeys.as<uint64_t>(), lcounts.as<int>(),
                                   lsat.as<uint64_t>(), parts, pkp, pkeys, pscores, pcounts,
                                   nullptr, q_flags, s));
    count_launches(2);
    XVEC_CUDA(cudaMemcpyAsync(h_status->data(), q_status, (size_t)nq * 4, cudaMemcpyDeviceToHost,
                              s));
    XVEC_CUDA(cudaStreamSynchronize(s));
    return XVEC_GPU_OK;
  }
  xvec_gpu_search_opts po{};
  po.top_k = nprobe;
  NestedSearch nested;
  return search_device_locked(idx->probe_index, d_q, nq, po, nullptr, pkeys, pscores, pcounts, s,
                              h_status);
}

xvec_gpu_status ivf_flat_search_impl(xvec_gpu_index* idx, const float* d_q, int nq,
                                     const xvec_gpu_search_opts& o, const uint32_t* d_bitmap,
                                     uint64_t* d_keys, float* d_scores, int* d_counts,
                                     cudaStream_t s, std::vector<int>* statuses) {
  if (!idx->has_model) return set_error("IVF index has no model"), XVEC_GPU_INVALID_ARGUMENT;
  if (o.nprobe <= 0) return set_error("core: IVF NProbe must be positive"), XVEC_GPU_INVALID_ARGUMENT;
  const int d = idx->desc.dimension, metric = idx->desc.metric, k = o.top_k;
  const int64_t n = idx->n;
  xvec_gpu_status st;
  EventTimer timer(s);
  timer.mark(0);
  {
    static std::mutex rebuild_mu;
    std::lock_guard<std::mutex> g(rebuild_mu);
    if (idx->lists_dirty && n > 0 && (st = rebuild_lists(idx, s))) return st;
  }
  const int nprobe = std::min(o.nprobe, idx->nlist);
  int kp = 32;
  while (kp < k + std::max(8, k / 4)) kp <<= 1;
  if ((int64_t)kIvfWarps * kp > flat_merge_capacity())
    return set_error("top_k %d exceeds the merge capacity", k), XVEC_GPU_INVALID_ARGUMENT;
  Scratch qf, qn2, qaux, qstatus, qflags, pkeys, pscores, pcounts;
  if ((st = qf.alloc((size_t)nq * d * 4, s)) || (st = qn2.alloc((size_t)nq * 4, s)) ||
      (st = qaux.alloc((size_t)nq * 4, s)) || (st = qstatus.alloc((size_t)nq * 4, s)) ||
      (st = qflags.alloc((size_t)nq * 4, s)) || (st = pkeys.alloc((size_t)nq * nprobe * 8, s)) ||
      (st = pscores.alloc((size_t)nq * nprobe * 4, s)) || (st = pcounts.alloc((size_t)nq * 4, s)))
    return st;
  XVEC_CUDA(cudaMemsetAsync(qflags.ptr, 0, (size_t)nq * 4, s));
  XVEC_CUDA(cudaMemsetAsync(d_counts, 0, (size_t)nq * 4, s));
  // metric.Compute(q, q) validation and the query terms.
  launch_prep_queries<float>(d_q, nq, d, metric, qf.as<float>(), qn2.as<float>(),
                             qaux.as<float>(), qstatus.as<int>(), s);
  XVEC_LAUNCHED();
  std::vector<int> h_status(nq);
  if ((st = ivf_probe(idx, d_q, nq, nprobe, qf.as<float>(), qn2.as<float>(), qstatus.as<int>(),
                      pkeys.as<uint64_t>(), pscores.as<float>(), pcounts.as<int>(),
                      qflags.as<int>(), &h_status, s)))
    return st;
  int exact_count = 0;
  if (n > 0) {
    Scratch lkeys, lcounts, lsat;
    const size_t lists = (size_t)nq * kIvfWarps;
    if ((st = lkeys.alloc(lists * kp * 8, s)) || (st = lcounts.alloc(lists * 4, s)) ||
        (st = lsat.alloc(lists * 8, s)))
      return st;
    const IvfFlatScorer sc{metric,           idx->rows.as<float>(), idx->row_n2.as<float>(),
                           qf.as<float>(),   qn2.as<float>(),       idx->max_n2.as<unsigned>(),
                           d};
    const bool lm = idx->list_rows_f.ptr != nullptr;
    const IvfFlatPolicy pol{metric,
                            idx->rows.as<float>(),
                            idx->row_n2.as<float>(),
                            lm ? idx->list_rows_f.as<float4>() : nullptr,
                            lm ? idx->list_n2.as<float>() : nullptr,
                            qf.as<float>(),
                            qn2.as<float>(),
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
        return set_error("top_k %d or dimension %d too large for the IVF scan", k, d),
               XVEC_GPU_UNSUPPORTED;
      XVEC_CUDA(e);
      XVEC_LAUNCHED();
      XVEC_CUDA(launch_merge_rescore(sc, idx->pos_of_kr.as<uint32_t>(), idx->keys.as<uint64_t>(),
                                     ids, count, k, o.radius, exact ? 1 : 0, lkeys.as<uint64_t>(),
                                     lcounts.as<int>(), lsat.as<uint64_t>(), kIvfWarps, kp,
                                     d_keys, d_scores, d_counts, nullptr, qflags.as<int>(), s));
      XVEC_LAUNCHED();
      return XVEC_GPU_OK;
    };
    timer.mark(1);
    if ((st = scan(false, nullptr, nq))) return st;
    timer.mark(2);
    std::vector<int> h_fl(nq), exact_list;
    XVEC_CUDA(cudaMemcpyAsync(h_fl.data(), qflags.ptr, (size_t)nq * 4, cudaMemcpyDeviceToHost, s));
    XVEC_CUDA(cudaStreamSynchronize(s));
    for (int q = 0; q < nq; ++q)
      if (h_status[q] == 0 && (h_fl[q] & 3)) exact_list.push_back(q);
    if (!exact_list.empty()) {
      const int nl = (int)exact_list.size();
      Scratch ids;
      if ((st = ids.alloc((size_t)nl * 4, s))) return st;
      XVEC_CUDA(cudaMemcpyAsync(ids.ptr, exact_list.data(), (size_t)nl * 4,
                                cudaMemcpyHostToDevice, s));
      clear_bits_kernel<<<blocks_of(nl), 256, 0, s>>>(ids.as<int>(), nl, 3, qflags.as<int>());
      XVEC_LAUNCHED();
      if ((st = scan(true, ids.as<int>(), nl))) return st;
      exact_count = nl;
    }
  }
  XVEC_CUDA(cudaMemcpyAsync(qstatus.ptr, h_status.data(), (size_t)nq * 4, cudaMemcpyHostToDevice,
                            s));
  ivf_status_kernel<<<blocks_of(nq), 256, 0, s>>>(qstatus.as<int>(), qflags.as<int>(), nq,
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
      int sq = h_status[q];
      if (sq == 0 && (h_flags[q] & 4)) sq = XVEC_GPU_NON_FINITE;
      (*statuses)[q] = sq;
    }
  }
  return XVEC_GPU_OK;
}

}  // namespace xvec

using namespace xvec;

extern "C" xvec_gpu_status xvec_gpu_ivf_set_model(xvec_gpu_index* idx, const float* centroids,
                                                  int32_t nlist) {
  if (!idx || !centroids) return set_error("nil argument"), XVEC_GPU_INVALID_ARGUMENT;
  if (idx->desc.kind != XVEC_INDEX_IVF_FLAT && idx->desc.kind != XVEC_INDEX_IVF_SQ8 &&
      idx->desc.kind != XVEC_INDEX_IVF_SQ4)
    return set_error("not an IVF index"), XVEC_GPU_INVALID_ARGUMENT;
  if (nlist <= 0) return set_error("core: IVF NList must be positive"), XVEC_GPU_INVALID_ARGUMENT;
  const int d = idx->desc.dimension;
  std::unique_lock<std::shared_mutex> lock(idx->mu);
  if (idx->n > 0) return set_error("set the model before adding rows"), XVEC_GPU_INVALID_ARGUMENT;
  for (int64_t i = 0; i < (int64_t)nlist * d; ++i)
    if (!std::isfinite(centroids[i])) return set_error("non-finite centroid"), XVEC_GPU_NON_FINITE;
  cudaSetDevice(idx->device);
  cudaStream_t s = nullptr;
  xvec_gpu_status st;
  if ((st = idx->centroids.reserve((size_t)nlist * d * 4, 0, s))) return st;
  XVEC_CUDA(cudaMemcpy(idx->centroids.ptr, centroids, (size_t)nlist * d * 4,
                       cudaMemcpyHostToDevice));
  if (idx->probe_index) {
    xvec_gpu_index_destroy(idx->probe_index);
    idx->probe_index = nullptr;
  }
  if ((st = make_probe_index(idx->device, idx->desc.metric, d, idx->centroids.as<float>(), nlist,
                             s, &idx->probe_index)))
    return st;
  idx->nlist = nlist;
  idx->chunks = 0;
  idx->has_model = true;
  idx->lists_dirty = true;
  return XVEC_GPU_OK;
}
