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
// The list scan is one 16-warp block per query over its probed lists
// (positions in list order, rows gathered by position): each lane ranks one
// row with a float32 dot product (the fast rank of the Flat path, within the
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
#include "pipeline.cuh"

namespace xvec {

xvec_gpu_status search_device_locked(xvec_gpu_index* idx, const void* d_q, int nq,
                                     const xvec_gpu_search_opts& o, const uint32_t* d_bitmap,
                                     uint64_t* d_keys, float* d_scores, int* d_counts,
                                     cudaStream_t s, std::vector<int>* statuses);

namespace {

inline unsigned blocks_of(int64_t n, int t = 256) { return (unsigned)((n + t - 1) / t); }
constexpr int kIvfWarps = 16;

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
  __device__ float eps(int) const { return 0.f; }
  __device__ int error_flag(float) const { return 4; }
  __device__ float output(float r) const { return r; }
  __device__ bool keep(float, float) const { return true; }
};

// One block per query (query_ids[blockIdx.x] when given) over its probed
// lists; EXACT: reference-order scores, a warp per row.
template <int CAPW, bool EXACT>
__global__ void __launch_bounds__(kIvfWarps * 32, 1) ivf_flat_scan_kernel(
    const float* __restrict__ rows, int d, const float* __restrict__ row_n2,
    const uint64_t* __restrict__ probe_lists, const int* __restrict__ probe_counts, int nprobe,
    const int64_t* __restrict__ list_offsets, const uint32_t* __restrict__ list_rows,
    const uint32_t* __restrict__ list_keyrank, const uint32_t* __restrict__ bitmap, int metric,
    const float* __restrict__ qf, const float* __restrict__ q_n2,
    const int* __restrict__ query_ids, int kp, uint64_t* __restrict__ part_keys,
    int* __restrict__ part_counts, uint64_t* __restrict__ part_sat, int* __restrict__ q_flags) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  uint64_t* wbuf = reinterpret_cast<uint64_t*>(smem_raw);         // [warps][CAPW]
  float* sq = reinterpret_cast<float*>(wbuf + kIvfWarps * CAPW);  // [d] the query
  __shared__ AccumState wst[kIvfWarps];
  __shared__ unsigned long long s_thr;
  const int q = query_ids ? query_ids[blockIdx.x] : blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const float* qv = qf + (int64_t)q * d;
  for (int i = threadIdx.x; i < d; i += blockDim.x) sq[i] = qv[i];
  if (lane == 0) {
    wst[warp].count = 0;
    wst[warp].saturated = 0;
    wst[warp].thr = kEmptyKey;
  }
  if (threadIdx.x == 0) s_thr = kEmptyKey;
  __syncthreads();
  const float qn2 = q_n2[q];
  uint64_t* buf = wbuf + warp * CAPW;
  AccumState* st = &wst[warp];
  int cnt = 0;
  uint64_t wthr = kEmptyKey;
  const bool vec4 = (d & 3) == 0;
  const int nl = probe_counts[q];
  for (int j = 0; j < nl; ++j) {
    const uint64_t list = probe_lists[(int64_t)q * nprobe + j];
    const int64_t begin = list_offsets[list], end = list_offsets[list + 1];
    for (int64_t base = begin + (int64_t)warp * 32; base < end; base += kIvfWarps * 32) {
      const int64_t idx = base + lane;
      bool valid = idx < end;
      uint32_t pos = 0;
      if (valid) {
        pos = list_rows[idx];
        valid = bitmap_pass(bitmap, pos);
      }
      float rank = 0.f;
      if constexpr (EXACT) {
        // Reference scores, one row per warp step.
        const unsigned vm = __ballot_sync(kFullMask, valid);
        for (int r = 0; r < 32; ++r) {
          if (!((vm >> r) & 1u)) continue;
          const uint32_t p = __shfl_sync(kFullMask, pos, r);
          const float sc =
              ivf_reference_score(metric, rows + (int64_t)p * d, row_n2[p], sq, qn2, d);
          if (lane == r) rank = rank_from_score(metric, sc);
        }
      } else if (valid) {
        const float* x = rows + (int64_t)pos * d;
        float dot = 0.f;
        if (vec4) {
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
        rank = fast_rank(metric, dot, row_n2[pos], qn2);
      }
      const uint64_t shared_thr = *(volatile unsigned long long*)&s_thr;
      const uint64_t thr = shared_thr < wthr ? shared_thr : wthr;
      bool take = false;
      uint64_t key = 0;
      if (valid) {
        if (!finite_f(rank)) {
          atomicOr(&q_flags[q], EXACT ? 4 : 1);
        } else {
          key = pack_rank(rank, list_keyrank[idx]);
          take = key < thr;
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
  }
  __syncwarp();
  if (lane == 0) st->count = cnt;
  __syncwarp();
  warp_compact<CAPW>(buf, st, kp);
  const int out = min(st->count, kp);
  const int64_t slot = (int64_t)blockIdx.x * kIvfWarps + warp;
  for (int i = lane; i < out; i += 32) part_keys[slot * kp + i] = buf[i];
  if (lane == 0) {
    part_counts[slot] = out;
    part_sat[slot] = st->thr;
  }
}

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
  xvec_gpu_status st = assign_rows(idx->probe_index, idx->rows.as<float>() + old_n * d, m, d,
                                   idx->row_list.as<int32_t>() + old_n, nullptr, s);
  if (st) return st;
  idx->lists_dirty = true;
  return XVEC_GPU_OK;
}

xvec_gpu_status ivf_flat_search_impl(xvec_gpu_index* idx, const float* d_q, int nq,
                                     const xvec_gpu_search_opts& o, const uint32_t* d_bitmap,
                                     uint64_t* d_keys, float* d_scores, int* d_counts,
                                     cudaStream_t s, std::vector<int>* statuses) {
  if (!idx->has_model) return set_error("IVF index has no model"), XVEC_GPU_INVALID_ARGUMENT;
  if (o.nprobe <= 0) return set_error("core: IVF NProbe must be positive"), XVEC_GPU_INVALID_ARGUMENT;
  const int d = idx->desc.dimension, metric = idx->desc.metric, k = o.top_k;
  const int64_t n = idx->n;
  const int nlist = idx->nlist;
  xvec_gpu_status st;
  EventTimer timer(s);
  timer.mark(0);
  {
    static std::mutex rebuild_mu;
    std::lock_guard<std::mutex> g(rebuild_mu);
    if (idx->lists_dirty && n > 0 && (st = rebuild_lists(idx, s))) return st;
  }
  const int nprobe = std::min(o.nprobe, nlist);
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
  // Probe.
  if (metric == XVEC_METRIC_COSINE) {
    const xvec_gpu_index* pi = idx->probe_index;
    Scratch ckeys, cranks, lkeys, lcounts, lsat;
    const int parts = std::max(1, std::min(flat_merge_capacity() / std::max(nprobe, 32),
                                           (nlist + 255) / 256));
    int pkp = 32;
    while (pkp < nprobe) pkp <<= 1;
    if ((st = ckeys.alloc((size_t)nlist * 8, s)) || (st = cranks.alloc((size_t)nlist * 4, s)) ||
        (st = lkeys.alloc((size_t)nq * parts * pkp * 8, s)) ||
        (st = lcounts.alloc((size_t)nq * parts * 4, s)) ||
        (st = lsat.alloc((size_t)nq * parts * 8, s)))
      return st;
    if ((int64_t)parts * pkp > flat_merge_capacity() || exact_cap_for(pkp) > 8192)
      return set_error("nprobe %d too large for the cosine probe", nprobe), XVEC_GPU_UNSUPPORTED;
    iota64_kernel<<<blocks_of(nlist), 256, 0, s>>>(ckeys.as<uint64_t>(), cranks.as<uint32_t>(),
                                                   nlist);
    XVEC_LAUNCHED();
    const IvfProbeScorer msc{kMetricL2,      pi->rows.as<float>(), pi->row_n2.as<float>(),
                             qf.as<float>(), qn2.as<float>(),      d};
    XVEC_CUDA(launch_scan_exact(msc, nlist, cranks.as<uint32_t>(), nullptr, nq, nullptr, parts,
                                pkp, lkeys.as<uint64_t>(), lcounts.as<int>(),
                                lsat.as<uint64_t>(), qflags.as<int>(), s));
    XVEC_CUDA(launch_merge_rescore(msc, cranks.as<uint32_t>(), ckeys.as<uint64_t>(), nullptr, nq,
                                   nprobe, 0.f, 1, lkeys.as<uint64_t>(), lcounts.as<int>(),
                                   lsat.as<uint64_t>(), parts, pkp, pkeys.as<uint64_t>(),
                                   pscores.as<float>(), pcounts.as<int>(), nullptr,
                                   qflags.as<int>(), s));
    count_launches(2);
    // A non-finite probe score fails the query (flag 4 stays set).
    XVEC_CUDA(cudaMemcpyAsync(h_status.data(), qstatus.ptr, (size_t)nq * 4,
                              cudaMemcpyDeviceToHost, s));
    XVEC_CUDA(cudaStreamSynchronize(s));
  } else {
    xvec_gpu_search_opts po{};
    po.top_k = nprobe;
    NestedSearch nested;
    st = search_device_locked(idx->probe_index, d_q, nq, po, nullptr, pkeys.as<uint64_t>(),
                              pscores.as<float>(), pcounts.as<int>(), s, &h_status);
    if (st) return st;
  }
  int exact_count = 0;
  if (n > 0) {
    int capw = 128;
    while (capw < kp + 64) capw <<= 1;
    if (capw > 1024) return set_error("top_k %d too large for the IVF scan", k), XVEC_GPU_INVALID_ARGUMENT;
    Scratch lkeys, lcounts, lsat;
    const size_t lists = (size_t)nq * kIvfWarps;
    if ((st = lkeys.alloc(lists * kp * 8, s)) || (st = lcounts.alloc(lists * 4, s)) ||
        (st = lsat.alloc(lists * 8, s)))
      return st;
    const size_t smem = (size_t)kIvfWarps * capw * 8 + (size_t)d * 4;
    if (smem > 220 * 1024) return set_error("dimension too large for the IVF scan"), XVEC_GPU_UNSUPPORTED;
    const IvfFlatScorer sc{metric,           idx->rows.as<float>(), idx->row_n2.as<float>(),
                           qf.as<float>(),   qn2.as<float>(),       idx->max_n2.as<unsigned>(),
                           d};
    auto scan = [&](bool exact, const int* ids, int count) -> xvec_gpu_status {
#define XVEC_IVF_CASE(C, E)                                                                    \
  if (capw == C && exact == E) {                                                               \
    auto kern = ivf_flat_scan_kernel<C, E>;                                                    \
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);        \
    kern<<<count, kIvfWarps * 32, smem, s>>>(                                                  \
        idx->rows.as<float>(), d, idx->row_n2.as<float>(), pkeys.as<uint64_t>(),               \
        pcounts.as<int>(), nprobe, idx->list_offsets.as<int64_t>(),                            \
        idx->list_rows.as<uint32_t>(), idx->list_keyrank.as<uint32_t>(), d_bitmap, metric,     \
        qf.as<float>(), qn2.as<float>(), ids, kp, lkeys.as<uint64_t>(), lcounts.as<int>(),     \
        lsat.as<uint64_t>(), qflags.as<int>());                                                \
  }
      XVEC_IVF_CASE(128, false)
      XVEC_IVF_CASE(256, false)
      XVEC_IVF_CASE(512, false)
      XVEC_IVF_CASE(1024, false)
      XVEC_IVF_CASE(128, true)
      XVEC_IVF_CASE(256, true)
      XVEC_IVF_CASE(512, true)
      XVEC_IVF_CASE(1024, true)
#undef XVEC_IVF_CASE
      XVEC_LAUNCHED();
      XVEC_CUDA(cudaGetLastError());
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
  if (idx->desc.kind != XVEC_INDEX_IVF_FLAT)
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
