// noalloc.cu — Flat search that allocates no memory during the call.
//
// For callers that cannot allocate device memory while they search: a
// process that owns a fixed device-memory budget and plans every byte up
// front (an arena shared with other work, so a surprise allocation could fail
// or fragment it), or a latency-critical caller that must not enter the CUDA
// allocator, which can block or synchronise the device.  The regular entry
// point takes its per-call scratch from the stream-ordered allocator; this one
// takes it from one file-scope device array instead.
//
// The array is kNoAllocScratchBytes (32 MiB) on every GPU that loads the
// library, held until the process exits.  Requests whose scratch would not
// fit are rejected with XVEC_GPU_INVALID_ARGUMENT; so are more than
// kNoAllocMaxQueries queries per call and top-k above 100.
//
// All calls share the array and it keeps the last call's contents, so the
// parts that must start at zero are cleared on every call, and calls whose
// GPU work overlaps (for example from two host threads on two streams of the
// same device) race on it.  Calls are serialised on the host by a mutex, and
// each call waits for its GPU work before returning, on its error paths too,
// so the array is idle whenever the mutex is released.  The caller's cancel
// flag is polled between launches and the library's counters are updated,
// as for the regular search.
//
// Set-up: the first call on a device looks up the device address of the
// array with cudaGetSymbolAddress (with that device current) and keeps it;
// that first call should come before any stream capture begins.
#include <algorithm>
#include <cmath>
#include <cstring>
#include <mutex>

#include "capi_internal.h"
#include "common.cuh"
#include "flat_kernels.cuh"

namespace xvec {

constexpr size_t kNoAllocScratchBytes = 32u << 20;
constexpr int kNoAllocMaxQueries = 4096;
constexpr int kNoAllocMaxDevices = 64;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

namespace {

std::mutex g_noalloc_mu;
void* g_noalloc_ptr[kNoAllocMaxDevices] = {};

// Device address of the scratch array on `device` (current), looked up once.
xvec_gpu_status noalloc_scratch(int device, unsigned char** out) {
  if (device < 0 || device >= kNoAllocMaxDevices)
    return set_error("device %d out of range", device), XVEC_GPU_INVALID_ARGUMENT;
  if (!g_noalloc_ptr[device]) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p) {
      cudaGetLastError();
      set_error("cudaGetSymbolAddress(scratch) failed on device %d: %s", device,
                cudaGetErrorString(e));
      return XVEC_GPU_CUDA_ERROR;
    }
    g_noalloc_ptr[device] = p;
  }
  *out = static_cast<unsigned char*>(g_noalloc_ptr[device]);
  return XVEC_GPU_OK;
}

// Bump allocator over the static array (no memory is allocated).
struct Carve {
  unsigned char* base;
  size_t used = 0;
  template <typename T>
  T* take(size_t count) {
    used = (used + 255) & ~size_t(255);
    T* p = reinterpret_cast<T*>(base + used);
    used += count * sizeof(T);
    return p;
  }
};

__global__ void noalloc_clear_flags(const int* ids, int n, int* q_flags) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) q_flags[ids[i]] &= ~3;
}
__global__ void noalloc_apply_status(const int* q_status, const int* q_flags, int nq,
                                     int* out_counts) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= nq) return;
  int st = q_status[i];
  if (st == 0 && (q_flags[i] & 4)) st = XVEC_GPU_NON_FINITE;
  if (st != 0) out_counts[i] = -st;
}

int noalloc_kp(int k) {
  int want = k + std::max(8, k / 4);
  int kp = 32;
  while (kp < want) kp <<= 1;
  return kp;
}

template <typename RowT>
xvec_gpu_status noalloc_search(xvec_gpu_index* idx, const void* d_q, int nq,
                               const xvec_gpu_search_opts& o, uint64_t* d_keys_out,
                               float* d_scores_out, int* d_counts_out, unsigned char* scratch,
                               cudaStream_t s) {
  const int d = idx->desc.dimension, metric = idx->desc.metric, k = o.top_k;
  const int64_t n = idx->n;
  const RowT* rows = idx->rows.as<RowT>();
  const int kp = noalloc_kp(k);
  const int qtiles = (nq + 31) / 32;
  int parts = (int)std::max<int64_t>(
      1, std::min<int64_t>((592 + qtiles - 1) / qtiles, (n + 1023) / 1024));
  parts = std::min(parts, std::max(1, flat_merge_capacity() / kp));
  // The exact pass reuses the part-list region, so size it for either pass:
  // the exact pass takes nl <= nq queries with at most ceil(592 / nl) parts
  // each, i.e. fewer than 592 + nq lists.
  const size_t fast_lists = (size_t)nq * parts;
  const size_t exact_lists =
      std::min((size_t)592 + nq, (size_t)nq * std::max(1, flat_merge_capacity() / kp));
  const size_t lists = std::max(fast_lists, exact_lists);
  // Scratch layout (256-byte aligned pieces).
  const size_t need = 256 * 12 + (size_t)nq * d * 4 + (size_t)nq * 4 * 6 + lists * (size_t)kp * 8 +
                      lists * 12;
  if (need > kNoAllocScratchBytes)
    return set_error("no-allocation search needs %zu bytes of scratch; the limit is %zu "
                     "(use fewer queries per call)",
                     need, kNoAllocScratchBytes),
           XVEC_GPU_INVALID_ARGUMENT;
  Carve c{scratch};
  float* qf = c.take<float>((size_t)nq * d);
  float* qn2 = c.take<float>(nq);
  float* qaux = c.take<float>(nq);
  int* qstatus = c.take<int>(nq);
  int* qflags = c.take<int>(nq);
  int* ids = c.take<int>(nq);
  uint64_t* pkeys = c.take<uint64_t>(lists * kp);
  int* pcounts = c.take<int>(lists);
  uint64_t* psat = c.take<uint64_t>(lists);

  XVEC_CUDA(cudaMemsetAsync(qflags, 0, (size_t)nq * 4, s));
  XVEC_CUDA(cudaMemsetAsync(d_counts_out, 0, (size_t)nq * 4, s));
  launch_prep_queries<RowT>(static_cast<const RowT*>(d_q), nq, d, metric, qf, qn2, qaux, qstatus,
                            s);
  XVEC_LAUNCHED();
  XVEC_CUDA(cudaGetLastError());
  if (n > 0) {
    if (is_cancelled(o)) return set_error("cancelled"), XVEC_GPU_CANCELLED;
    XVEC_CUDA(launch_flat_scan_simt<RowT>(rows, n, d, idx->row_n2.as<float>(),
                                          idx->keyrank.as<uint32_t>(), qf, qn2, nq, nullptr,
                                          metric, parts, kp, pkeys, pcounts, psat, qflags, s));
    XVEC_LAUNCHED();
    if (is_cancelled(o)) return set_error("cancelled"), XVEC_GPU_CANCELLED;
    XVEC_CUDA(launch_flat_merge_rescore<RowT>(rows, d, idx->pos_of_kr.as<uint32_t>(),
                                              idx->keys.as<uint64_t>(), qf, qn2,
                                              idx->max_n2.as<unsigned>(), nullptr, nq, metric, k,
                                              o.radius, 0, pkeys, pcounts, psat, parts, kp,
                                              d_keys_out, d_scores_out, d_counts_out, qflags, s));
    XVEC_LAUNCHED();
  }
  int h_status[kNoAllocMaxQueries], h_flags[kNoAllocMaxQueries], h_ids[kNoAllocMaxQueries];
  XVEC_CUDA(cudaMemcpyAsync(h_status, qstatus, (size_t)nq * 4, cudaMemcpyDeviceToHost, s));
  XVEC_CUDA(cudaMemcpyAsync(h_flags, qflags, (size_t)nq * 4, cudaMemcpyDeviceToHost, s));
  XVEC_CUDA(cudaStreamSynchronize(s));
  int nl = 0;
  if (n > 0)
    for (int q = 0; q < nq; ++q)
      if (h_status[q] == 0 && (h_flags[q] & 3)) h_ids[nl++] = q;
  if (nl > 0) {
    if (is_cancelled(o)) return set_error("cancelled"), XVEC_GPU_CANCELLED;
    int eparts = (int)std::max<int64_t>(1, std::min<int64_t>((592 + nl - 1) / nl, (n + 1023) / 1024));
    eparts = std::min(eparts, std::max(1, flat_merge_capacity() / kp));
    if ((size_t)nl * eparts > lists)
      eparts = std::max(1, (int)(lists / (size_t)nl));
    XVEC_CUDA(cudaMemcpyAsync(ids, h_ids, (size_t)nl * 4, cudaMemcpyHostToDevice, s));
    noalloc_clear_flags<<<(nl + 255) / 256, 256, 0, s>>>(ids, nl, qflags);
    XVEC_LAUNCHED();
    XVEC_CUDA(launch_flat_scan_exact<RowT>(rows, n, d, idx->keyrank.as<uint32_t>(), qf, ids, nl,
                                           nullptr, metric, eparts, kp, pkeys, pcounts, psat,
                                           qflags, s));
    XVEC_CUDA(launch_flat_merge_rescore<RowT>(rows, d, idx->pos_of_kr.as<uint32_t>(),
                                              idx->keys.as<uint64_t>(), qf, qn2,
                                              idx->max_n2.as<unsigned>(), ids, nl, metric, k,
                                              o.radius, 1, pkeys, pcounts, psat, eparts, kp,
                                              d_keys_out, d_scores_out, d_counts_out, qflags, s));
    count_launches(2);
    XVEC_CUDA(cudaMemcpyAsync(h_flags, qflags, (size_t)nq * 4, cudaMemcpyDeviceToHost, s));
    XVEC_CUDA(cudaStreamSynchronize(s));
    for (int i = 0; i < nl; ++i)
      if (h_flags[h_ids[i]] & 2) {
        set_error("exact scan could not complete query %d", h_ids[i]);
        return XVEC_GPU_CUDA_ERROR;
      }
  }
  noalloc_apply_status<<<(nq + 255) / 256, 256, 0, s>>>(qstatus, qflags, nq, d_counts_out);
  XVEC_LAUNCHED();
  XVEC_CUDA(cudaGetLastError());
  XVEC_CUDA(cudaStreamSynchronize(s));
  count_search(nq, nl, 0.0, 0.0);
  for (int q = 0; q < nq; ++q) {
    int st = h_status[q];
    if (st == 0 && (h_flags[q] & 4)) st = XVEC_GPU_NON_FINITE;
    if (st) {
      set_error("query %d failed with status %d", q, st);
      return (xvec_gpu_status)st;
    }
  }
  return XVEC_GPU_OK;
}

}  // namespace
}  // namespace xvec

using namespace xvec;

extern "C" xvec_gpu_status xvec_gpu_index_search_noalloc(xvec_gpu_index* idx, const void* d_q,
                                                         int32_t nq,
                                                         const xvec_gpu_search_opts* opts,
                                                         uint64_t* d_keys, float* d_scores,
                                                         int32_t* d_counts) {
  if (!idx || !opts) return set_error("nil index or options"), XVEC_GPU_INVALID_ARGUMENT;
  if (idx->desc.kind != XVEC_INDEX_FLAT)
    return set_error("the no-allocation search serves Flat indexes only"),
           XVEC_GPU_INVALID_ARGUMENT;
  if (nq < 0 || nq > kNoAllocMaxQueries)
    return set_error("no-allocation search takes at most %d queries per call, got %d",
                     kNoAllocMaxQueries, nq),
           XVEC_GPU_INVALID_ARGUMENT;
  if (opts->top_k <= 0) return set_error("core: top-k must be positive"), XVEC_GPU_INVALID_ARGUMENT;
  if (opts->top_k > 100)
    return set_error("no-allocation search takes top-k up to 100, got %d", opts->top_k),
           XVEC_GPU_INVALID_ARGUMENT;
  if (!(opts->radius >= 0) || std::isinf(opts->radius))
    return set_error("core: radius must be finite and non-negative"), XVEC_GPU_INVALID_ARGUMENT;
  if (opts->filter_bitmap)
    return set_error("the no-allocation search takes no filter bitmap"),
           XVEC_GPU_INVALID_ARGUMENT;
  if (nq == 0) return XVEC_GPU_OK;
  std::lock_guard<std::mutex> host_lock(g_noalloc_mu);
  std::shared_lock<std::shared_mutex> lock(idx->mu);
  if (cudaSetDevice(idx->device) != cudaSuccess) {
    cudaGetLastError();
    return set_error("cudaSetDevice(%d) failed", idx->device), XVEC_GPU_CUDA_ERROR;
  }
  unsigned char* scratch = nullptr;
  xvec_gpu_status st = noalloc_scratch(idx->device, &scratch);
  if (st) return st;
  cudaStream_t s = static_cast<cudaStream_t>(opts->stream);
  if (is_cancelled(*opts)) return set_error("cancelled"), XVEC_GPU_CANCELLED;
  st = idx->desc.storage == XVEC_STORAGE_FP16
           ? noalloc_search<__half>(idx, d_q, nq, *opts, d_keys, d_scores, d_counts, scratch, s)
           : noalloc_search<float>(idx, d_q, nq, *opts, d_keys, d_scores, d_counts, scratch, s);
  // On an early return work may still be queued on the array: wait for it
  // before the next call may take the array.
  if (st != XVEC_GPU_OK) cudaStreamSynchronize(s);
  return st;
}
