// capi.cu — the C ABI (include/xvec_gpu.h): index objects, device memory,
// insertion bookkeeping and the search orchestration.
#include <cub/device/device_radix_sort.cuh>

#include <algorithm>
#include <type_traits>
#include <cmath>
#include <cstring>

#include "capi_internal.h"
#include "common.cuh"
#include "flat_kernels.cuh"
#include "flat_tc.cuh"
#include "index_kernels.cuh"

namespace xvec {

namespace {
thread_local std::string g_last_error;
}

void set_error(const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
}

xvec_gpu_status DeviceBuffer::reserve(size_t need, size_t keep, cudaStream_t stream) {
  if (need <= bytes) return XVEC_GPU_OK;
  void* fresh = nullptr;
  cudaError_t e = cudaMalloc(&fresh, need);
  if (e != cudaSuccess) {
    cudaGetLastError();
    set_error("cudaMalloc(%zu bytes): %s", need, cudaGetErrorString(e));
    return XVEC_GPU_OUT_OF_MEMORY;
  }
  if (ptr && keep) {
    e = cudaMemcpyAsync(fresh, ptr, std::min(keep, bytes), cudaMemcpyDeviceToDevice, stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
    if (e != cudaSuccess) {
      cudaFree(fresh);
      set_error("grow copy: %s", cudaGetErrorString(e));
      return XVEC_GPU_CUDA_ERROR;
    }
  }
  if (ptr) cudaFree(ptr);
  ptr = fresh;
  bytes = need;
  return XVEC_GPU_OK;
}

xvec_gpu_status Scratch::alloc(size_t nbytes, cudaStream_t s) {
  stream = s;
  if (nbytes == 0) nbytes = 16;
  cudaError_t e = cudaMallocAsync(&ptr, nbytes, s);
  if (e != cudaSuccess) {
    cudaGetLastError();
    ptr = nullptr;
    set_error("cudaMallocAsync(%zu bytes): %s", nbytes, cudaGetErrorString(e));
    return XVEC_GPU_OUT_OF_MEMORY;
  }
  return XVEC_GPU_OK;
}

// ---------------------------------------------------------------------------
// Small bookkeeping kernels.
// ---------------------------------------------------------------------------
__global__ void iota_u32_kernel(uint32_t* out, int64_t n) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) out[i] = (uint32_t)i;
}
__global__ void scatter_keyrank_kernel(const uint32_t* pos_of_kr, uint32_t* keyrank, int64_t n) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) keyrank[pos_of_kr[i]] = (uint32_t)i;
}
__global__ void adjacent_equal_kernel(const uint64_t* sorted, int64_t n, int* flag) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i + 1 < n && sorted[i] == sorted[i + 1]) atomicExch(flag, 1);
}
__global__ void clear_flags_kernel(const int* ids, int n, int* q_flags, int mask) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) q_flags[ids[i]] &= ~mask;
}
__global__ void apply_status_kernel(const int* q_status, const int* q_flags, int nq,
                                    int* out_counts) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= nq) return;
  int st = q_status[i];
  if (st == 0 && (q_flags[i] & 4)) st = XVEC_GPU_NON_FINITE;
  if (st == 0 && (q_flags[i] & 8)) st = XVEC_GPU_OVERFLOW;
  if (st != 0) out_counts[i] = -st;
}

inline unsigned blocks_for(int64_t n, int t = 256) { return (unsigned)((n + t - 1) / t); }

// Rebuilds the key-rank permutation for rows [0, n) and rejects duplicate
// keys (ErrDuplicateKey, flat.go:140-142).  Nothing is committed on error.
xvec_gpu_status rebuild_keyrank(xvec_gpu_index* idx, int64_t n, cudaStream_t s) {
  if (n == 0) return XVEC_GPU_OK;
  if (n > 0xffffffffll) {
    set_error("more than 2^32 rows per index are not supported");
    return XVEC_GPU_INVALID_ARGUMENT;
  }
  Scratch iota, sorted_keys, sorted_pos, flag, temp;
  xvec_gpu_status st;
  if ((st = iota.alloc(n * 4, s)) || (st = sorted_keys.alloc(n * 8, s)) ||
      (st = sorted_pos.alloc(n * 4, s)) || (st = flag.alloc(4, s)))
    return st;
  iota_u32_kernel<<<blocks_for(n), 256, 0, s>>>(iota.as<uint32_t>(), n);
  size_t temp_bytes = 0;
  XVEC_CUDA(cub::DeviceRadixSort::SortPairs(nullptr, temp_bytes, idx->keys.as<uint64_t>(),
                                            sorted_keys.as<uint64_t>(), iota.as<uint32_t>(),
                                            sorted_pos.as<uint32_t>(), (int64_t)n, 0, 64, s));
  if ((st = temp.alloc(temp_bytes, s))) return st;
  XVEC_CUDA(cub::DeviceRadixSort::SortPairs(temp.ptr, temp_bytes, idx->keys.as<uint64_t>(),
                                            sorted_keys.as<uint64_t>(), iota.as<uint32_t>(),
                                            sorted_pos.as<uint32_t>(), (int64_t)n, 0, 64, s));
  XVEC_CUDA(cudaMemsetAsync(flag.ptr, 0, 4, s));
  adjacent_equal_kernel<<<blocks_for(n), 256, 0, s>>>(sorted_keys.as<uint64_t>(), n,
                                                      flag.as<int>());
  int dup = 0;
  XVEC_CUDA(cudaMemcpyAsync(&dup, flag.ptr, 4, cudaMemcpyDeviceToHost, s));
  XVEC_CUDA(cudaStreamSynchronize(s));
  if (dup) {
    set_error("duplicate vector key");
    return XVEC_GPU_DUPLICATE_KEY;
  }
  XVEC_CUDA(cudaMemcpyAsync(idx->pos_of_kr.ptr, sorted_pos.ptr, n * 4, cudaMemcpyDeviceToDevice,
                            s));
  scatter_keyrank_kernel<<<blocks_for(n), 256, 0, s>>>(idx->pos_of_kr.as<uint32_t>(),
                                                       idx->keyrank.as<uint32_t>(), n);
  XVEC_CUDA(cudaGetLastError());
  return XVEC_GPU_OK;
}

cudaStream_t thread_stream(int device) {
  thread_local cudaStream_t streams[64] = {};
  if (device < 0 || device >= 64) return nullptr;
  if (!streams[device]) cudaStreamCreateWithFlags(&streams[device], cudaStreamNonBlocking);
  return streams[device];
}

bool is_cancelled(const xvec_gpu_search_opts& o) {
  return o.cancel_flag && *o.cancel_flag != 0;
}


int choose_kp(int k) {
  int want = k + std::max(8, k / 4);
  int kp = 32;
  while (kp < want) kp <<= 1;
  return kp;
}

// ---------------------------------------------------------------------------
// Tensor-core candidate scan in launches over growing row prefixes.
// ---------------------------------------------------------------------------
xvec_gpu_status tc_seeded_scan(int device, int nq, int64_t n, int kp, cudaStream_t s,
                               const TcScanLaunch& scan, Scratch& pkeys, Scratch& pcounts,
                               Scratch& psat, int* lists_out, Scratch* gthr_out,
                               const TcPreseed& preseed) {
  // Parts: pick the row split whose CTA count best fills whole waves of
  // one CTA per SM, keeping at least 16 tiles of 256 rows per part.
  int sms = 148;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
  // Query blocks of 128; CTA pairs take them two at a time.
  const int qblocks = flat_tc_pairs(nq) ? ((nq + 127) / 128 + 1) / 2 * 2 : (nq + 127) / 128;
  auto best_parts = [&](int64_t max_parts) {
    int parts = 1;
    double best = -1;
    for (int p = 1; p <= max_parts; ++p) {
      const int64_t ctas = (int64_t)qblocks * p;
      const int64_t waves = (ctas + sms - 1) / sms;
      const double eff = (double)ctas / (double)(waves * sms);
      if (eff > best + 1e-9) {
        best = eff;
        parts = p;
      }
    }
    return parts;
  };
  const int lpp = flat_tc_lists_per_part();
  // The merge gathers every list of a query in shared memory.
  const int64_t merge_lists = flat_merge_capacity() / kp;
  // Seeding: launches over growing prefixes of the rows (1/256, then up to
  // 1/16); after each, the kp-th best key of every query over all lists
  // so far lowers its shared threshold, so the lists of the next launch
  // filter from their first tile instead of each collecting kp entries.
  std::vector<int64_t> ends;  // row ends of the seeding launches
  if (n >= (int64_t)1 << 16) {
    const int64_t e0 = n / 256 / 256 * 256, e1 = n / 16 / 256 * 256;
    if (e0 >= 4096) ends.push_back(e0);
    ends.push_back(e1);
  }
  std::vector<int> seed_parts;
  int64_t prev = 0;
  int used = 0;
  for (int64_t e : ends) {
    const int64_t lim = std::min<int64_t>(
        std::min<int64_t>(16, (merge_lists / 2 - used * lpp) / lpp), (e - prev) / 4096);
    const int p = best_parts(std::max<int64_t>(1, lim));
    seed_parts.push_back(p);
    used += p;
    prev = e;
  }
  const int64_t seed_rows = ends.empty() ? 0 : ends.back();
  const int64_t rest = n - seed_rows;
  const int parts = best_parts(std::max<int64_t>(
      1, std::min<int64_t>(std::min<int64_t>(64, merge_lists / lpp - used), rest / 4096)));
  const int cap = flat_tc_cap();
  const int lists = (used + parts) * lpp;
  Scratch gthr_local;
  Scratch& gthr = gthr_out ? *gthr_out : gthr_local;
  xvec_gpu_status st;
  if ((st = pkeys.alloc((size_t)nq * lists * cap * 8, s)) ||
      (st = pcounts.alloc((size_t)nq * lists * 4, s)) ||
      (st = psat.alloc((size_t)nq * lists * 8, s)) || (st = gthr.alloc((size_t)nq * 8, s)))
    return st;
  XVEC_CUDA(cudaMemsetAsync(gthr.ptr, 0xff, (size_t)nq * 8, s));
  if (preseed && !ends.empty()) {
    XVEC_CUDA(preseed(gthr.as<unsigned long long>()));
    count_launches(2);
  }
  prev = 0;
  int list0 = 0;
  for (size_t i = 0; i < ends.size(); ++i) {
    XVEC_CUDA(scan(prev, ends[i], seed_parts[i], list0, lists, gthr.as<unsigned long long>(),
                   pkeys.as<uint64_t>(), pcounts.as<int>(), psat.as<uint64_t>()));
    list0 += seed_parts[i] * lpp;
    XVEC_CUDA(launch_seed_thresholds(pkeys.as<uint64_t>(), pcounts.as<int>(), nq, lists, list0,
                                     cap, kp, gthr.as<unsigned long long>(), s));
    count_launches(2);
    prev = ends[i];
  }
  XVEC_CUDA(scan(seed_rows, n, parts, list0, lists, gthr.as<unsigned long long>(),
                 pkeys.as<uint64_t>(), pcounts.as<int>(), psat.as<uint64_t>()));
  *lists_out = lists;
  return XVEC_GPU_OK;
}

// ---------------------------------------------------------------------------
// Flat search (device memory in and out).
// ---------------------------------------------------------------------------
template <typename RowT>
xvec_gpu_status flat_search_impl(xvec_gpu_index* idx, const void* d_q, int nq,
                                 const xvec_gpu_search_opts& o, const uint32_t* d_bitmap,
                                 uint64_t* d_keys_out, float* d_scores_out, int* d_counts_out,
                                 cudaStream_t s, std::vector<int>* statuses,
                                 BandExchange* band) {
  const int d = idx->desc.dimension;
  const int metric = idx->desc.metric;
  const int k = o.top_k;
  const int64_t n = idx->n;
  const RowT* rows = idx->rows.as<RowT>();
  xvec_gpu_status st;
  Scratch qf, qn2, qaux, qstatus, qflags, kstatus;
  if ((st = qf.alloc((size_t)nq * d * 4, s)) || (st = qn2.alloc((size_t)nq * 4, s)) ||
      (st = qaux.alloc((size_t)nq * 4, s)) || (st = qstatus.alloc((size_t)nq * 4, s)) ||
      (st = qflags.alloc((size_t)nq * 4, s)) || (st = kstatus.alloc(4, s)))
    return st;
  XVEC_CUDA(cudaMemsetAsync(kstatus.ptr, 0, 4, s));
  EventTimer timer(s);
  timer.mark(0);
  XVEC_CUDA(cudaMemsetAsync(qflags.ptr, 0, (size_t)nq * 4, s));
  launch_prep_queries<RowT>(static_cast<const RowT*>(d_q), nq, d, metric, qf.as<float>(),
                            qn2.as<float>(), qaux.as<float>(), qstatus.as<int>(), s);
  XVEC_LAUNCHED();
  XVEC_CUDA(cudaGetLastError());
  XVEC_CUDA(cudaMemsetAsync(d_counts_out, 0, (size_t)nq * 4, s));

  // Sharded search: every shard's k best fast ranks and eps, exchanged once,
  // give each query a rank limit that every row of the global top-k meets on
  // its own shard, so a shard rescores about k / nranks candidates instead
  // of all within its own F_k + 2 eps (pipeline.cuh, band_limit_kernel).
  Scratch band_limit;
  auto run_band = [&](const uint64_t* lkeys, const int* lcounts, int nlists, int stride,
                      const unsigned long long* gthr, int split) -> xvec_gpu_status {
    if (!band) return XVEC_GPU_OK;
    band->used = true;
    const size_t w = (size_t)nq * (k + 1);
    Scratch bsend, brecv;
    xvec_gpu_status bst;
    if ((bst = bsend.alloc(w * 4, s)) || (bst = brecv.alloc(w * 4 * band->nranks, s)) ||
        (bst = band_limit.alloc((size_t)nq * 4, s)))
      return bst;
    XVEC_CUDA(launch_flat_band_prepare<RowT>(rows, d, qf.as<float>(), qn2.as<float>(),
                                             idx->max_n2.as<unsigned>(), nq, metric, k, lkeys,
                                             lcounts, nlists, stride, gthr, bsend.as<float>(), s,
                                             split));
    XVEC_LAUNCHED();
    if ((bst = band->allgather(bsend.as<float>(), brecv.as<float>(), w, s))) return bst;
    XVEC_CUDA(launch_flat_band_limit(brecv.as<float>(), band->nranks, nq, k, bsend.as<float>(),
                                     band_limit.as<float>(), s));
    XVEC_LAUNCHED();
    return XVEC_GPU_OK;
  };

  std::vector<int> h_status(nq), h_flags(nq);
  const int kp = choose_kp(k);
  // FP32 rows: the tensor-core scan on bfloat16 high/low parts of the rows
  // (kept beside them) and of the queries.
  constexpr bool kSplit = std::is_same<RowT, float>::value;
  Scratch qhi, qlo;
  // A few queries: the streaming scan (one pass over the rows at HBM speed).
  const bool use_stream = flat_stream_supported<RowT>(nq, n, d, kp, rows, d_q);
  const bool tc_layout = !use_stream && n > 0 && n < (1ll << 31) - 256 &&
                         kp + 128 <= flat_tc_cap() && d % 8 == 0 && d >= 64;
  if (kSplit && tc_layout) {
    if ((st = qhi.alloc((size_t)nq * d * 2, s)) || (st = qlo.alloc((size_t)nq * d * 2, s)))
      return st;
    XVEC_CUDA(launch_split_bf16(static_cast<const float*>(d_q), (int64_t)nq * d,
                                qhi.as<__nv_bfloat16>(), qlo.as<__nv_bfloat16>(), s));
    XVEC_LAUNCHED();
  }
  const bool use_tc =
      tc_layout && (kSplit ? flat_tc_supported(d, idx->rows_bhi.ptr, qhi.ptr) &&
                                 flat_tc_supported(d, idx->rows_blo.ptr, qlo.ptr)
                           : flat_tc_supported(d, rows, d_q));
  const bool fast = use_stream || use_tc || (simt_cap_for(kp) <= 512 && n > 0);
  if (use_stream) {
    if (is_cancelled(o)) return set_error("cancelled"), XVEC_GPU_CANCELLED;
    Scratch lkeys, lcounts, lsat;
    timer.mark(1);
    if ((st = flat_stream_scan<RowT>(idx->device, rows, n, d, idx->row_n2.as<float>(),
                                     idx->keyrank.as<uint32_t>(), qf.as<float>(), qn2.as<float>(),
                                     nq, metric, d_bitmap, kp, s, lkeys, lcounts, lsat,
                                     qflags.as<int>())))
      return st;
    timer.mark(2);
    count_stream_scan();
    if (is_cancelled(o)) return set_error("cancelled"), XVEC_GPU_CANCELLED;
    const int lstride = flat_stream_list_stride(kp);
    if ((st = run_band(lkeys.as<uint64_t>(), lcounts.as<int>(), 1, lstride, nullptr, 0)))
      return st;
    XVEC_CUDA(launch_flat_merge_rescore<RowT>(
        rows, d, idx->pos_of_kr.as<uint32_t>(), idx->keys.as<uint64_t>(), qf.as<float>(),
        qn2.as<float>(), idx->max_n2.as<unsigned>(), nullptr, nq, metric, k, o.radius, 0,
        lkeys.as<uint64_t>(), lcounts.as<int>(), lsat.as<uint64_t>(), 1, lstride, d_keys_out,
        d_scores_out, d_counts_out, qflags.as<int>(), s, 0, nullptr,
        band ? band_limit.as<float>() : nullptr));
    XVEC_LAUNCHED();
  } else if (use_tc) {
    if (is_cancelled(o)) return set_error("cancelled"), XVEC_GPU_CANCELLED;
    const int cap = flat_tc_cap();
    const float* row_aux =
        metric == XVEC_METRIC_COSINE ? idx->row_inv.as<float>() : idx->row_n2.as<float>();
    const __half* hrows = reinterpret_cast<const __half*>(rows);
    Scratch pkeys, pcounts, psat, gthr_keep, seed_ranks;
    int lists = 0;
    timer.mark(1);
    st = tc_seeded_scan(idx->device, nq, n, kp, s,
                        [&](int64_t b, int64_t e, int p, int list0, int nlists,
                            unsigned long long* gthr, uint64_t* cand, int* counts,
                            uint64_t* sat) {
                          if (kSplit)
                            return launch_flat_scan_tc_split(
                                metric, qhi.as<__nv_bfloat16>(), qlo.as<__nv_bfloat16>(), nq,
                                idx->rows_bhi.as<__nv_bfloat16>() + b * d,
                                idx->rows_blo.as<__nv_bfloat16>() + b * d, e - b, d, row_aux + b,
                                idx->keyrank.as<uint32_t>() + b, qaux.as<float>(),
                                qn2.as<float>(), gthr, d_bitmap ? d_bitmap + b / 32 : nullptr, p,
                                kp, list0, nlists, cand, counts, sat, qflags.as<int>(),
                                kstatus.as<int>(), s);
                          return launch_flat_scan_tc(
                              metric, static_cast<const __half*>(d_q), nq, hrows + b * d, e - b,
                              d, d, row_aux + b, idx->keyrank.as<uint32_t>() + b,
                              qaux.as<float>(), qn2.as<float>(), gthr,
                              d_bitmap ? d_bitmap + b / 32 : nullptr, p, kp, list0, nlists, cand,
                              counts, sat, qflags.as<int>(), kstatus.as<int>(), s);
                        },
                        pkeys, pcounts, psat, &lists, &gthr_keep,
                        [&](unsigned long long* gthr) -> cudaError_t {
                          const int samples = flat_sample_seed_rows(n, kp);
                          if (samples == 0) return cudaSuccess;
                          if (seed_ranks.alloc((size_t)nq * samples * 4, s) != XVEC_GPU_OK)
                            return cudaErrorMemoryAllocation;
                          return launch_flat_sample_seed<RowT>(
                              rows, n, d, idx->row_n2.as<float>(), d_bitmap, qf.as<float>(),
                              qn2.as<float>(), nq, metric, kp, idx->max_n2.as<unsigned>(),
                              kSplit ? 1 : 0, samples, seed_ranks.as<uint32_t>(), gthr, s);
                        });
    if (st) return st;
    timer.mark(2);
    XVEC_LAUNCHED();
    count_tensor_scan();
    if (is_cancelled(o)) return set_error("cancelled"), XVEC_GPU_CANCELLED;
    const unsigned long long* gthr = gthr_keep.as<unsigned long long>();
    if ((st = run_band(pkeys.as<uint64_t>(), pcounts.as<int>(), lists, cap, gthr,
                       kSplit ? 1 : 0)))
      return st;
    XVEC_CUDA(launch_flat_merge_rescore<RowT>(
        rows, d, idx->pos_of_kr.as<uint32_t>(), idx->keys.as<uint64_t>(), qf.as<float>(),
        qn2.as<float>(), idx->max_n2.as<unsigned>(), nullptr, nq, metric, k, o.radius, 0,
        pkeys.as<uint64_t>(), pcounts.as<int>(), psat.as<uint64_t>(), lists, cap, d_keys_out,
        d_scores_out, d_counts_out, qflags.as<int>(), s, kSplit ? 1 : 0, gthr,
        band ? band_limit.as<float>() : nullptr));
    XVEC_LAUNCHED();
  } else if (fast) {
    if (is_cancelled(o)) return set_error("cancelled"), XVEC_GPU_CANCELLED;
    const int qtiles = (nq + 31) / 32;
    int parts = (int)std::max<int64_t>(
        1, std::min<int64_t>((592 + qtiles - 1) / qtiles, (n + 1023) / 1024));
    parts = std::min(parts, std::max(1, flat_merge_capacity() / kp));
    Scratch pkeys, pcounts, psat;
    if ((st = pkeys.alloc((size_t)nq * parts * kp * 8, s)) ||
        (st = pcounts.alloc((size_t)nq * parts * 4, s)) ||
        (st = psat.alloc((size_t)nq * parts * 8, s)))
      return st;
    timer.mark(1);
    XVEC_CUDA(launch_flat_scan_simt<RowT>(rows, n, d, idx->row_n2.as<float>(),
                                          idx->keyrank.as<uint32_t>(), qf.as<float>(),
                                          qn2.as<float>(), nq, d_bitmap, metric, parts, kp,
                                          pkeys.as<uint64_t>(), pcounts.as<int>(),
                                          psat.as<uint64_t>(), qflags.as<int>(), s));
    timer.mark(2);
    XVEC_LAUNCHED();
    count_tensor_scan();
    if (is_cancelled(o)) return set_error("cancelled"), XVEC_GPU_CANCELLED;
    if ((st = run_band(pkeys.as<uint64_t>(), pcounts.as<int>(), parts, kp, nullptr, 0)))
      return st;
    XVEC_CUDA(launch_flat_merge_rescore<RowT>(
        rows, d, idx->pos_of_kr.as<uint32_t>(), idx->keys.as<uint64_t>(), qf.as<float>(),
        qn2.as<float>(), idx->max_n2.as<unsigned>(), nullptr, nq, metric, k, o.radius, 0,
        pkeys.as<uint64_t>(), pcounts.as<int>(), psat.as<uint64_t>(), parts, kp, d_keys_out,
        d_scores_out, d_counts_out, qflags.as<int>(), s, 0, nullptr,
        band ? band_limit.as<float>() : nullptr));
    XVEC_LAUNCHED();
  }
  XVEC_CUDA(cudaMemcpyAsync(h_status.data(), qstatus.ptr, (size_t)nq * 4, cudaMemcpyDeviceToHost,
                            s));
  XVEC_CUDA(cudaMemcpyAsync(h_flags.data(), qflags.ptr, (size_t)nq * 4, cudaMemcpyDeviceToHost,
                            s));
  int h_kstatus = 0;
  XVEC_CUDA(cudaMemcpyAsync(&h_kstatus, kstatus.ptr, 4, cudaMemcpyDeviceToHost, s));
  XVEC_CUDA(cudaStreamSynchronize(s));
  if (h_kstatus != 0)
    return set_error("tensor-core scan: a bounded device wait expired (code %d)", h_kstatus),
           XVEC_GPU_TIMEOUT;
  // Exact path: queries whose candidate set was not provably complete (or
  // that saw a non-finite fast rank), and every query when k is large.
  std::vector<int> exact_list;
  if (n > 0)
    for (int q = 0; q < nq; ++q)
      if (h_status[q] == 0 && (!fast || (h_flags[q] & 3))) exact_list.push_back(q);
  if (!exact_list.empty()) {
    if (is_cancelled(o)) return set_error("cancelled"), XVEC_GPU_CANCELLED;
    const int nl = (int)exact_list.size();
    if (exact_cap_for(kp) > 8192 || k > 1024) {
      set_error("top_k %d exceeds the supported maximum of 1024", k);
      return XVEC_GPU_INVALID_ARGUMENT;
    }
    int parts = (int)std::max<int64_t>(1, std::min<int64_t>((592 + nl - 1) / nl, (n + 1023) / 1024));
    parts = std::min(parts, std::max(1, flat_merge_capacity() / kp));
    Scratch ids, pkeys, pcounts, psat;
    if ((st = ids.alloc((size_t)nl * 4, s)) || (st = pkeys.alloc((size_t)nl * parts * kp * 8, s)) ||
        (st = pcounts.alloc((size_t)nl * parts * 4, s)) ||
        (st = psat.alloc((size_t)nl * parts * 8, s)))
      return st;
    XVEC_CUDA(cudaMemcpyAsync(ids.ptr, exact_list.data(), (size_t)nl * 4, cudaMemcpyHostToDevice, s));
    // The fast pass's coverage bit does not apply to the exact pass.
    clear_flags_kernel<<<blocks_for(nl), 256, 0, s>>>(ids.as<int>(), nl, qflags.as<int>(), 3);
    XVEC_LAUNCHED();
    XVEC_CUDA(launch_flat_scan_exact<RowT>(rows, n, d, idx->keyrank.as<uint32_t>(), qf.as<float>(),
                                           ids.as<int>(), nl, d_bitmap, metric, parts, kp,
                                           pkeys.as<uint64_t>(), pcounts.as<int>(),
                                           psat.as<uint64_t>(), qflags.as<int>(), s));
    XVEC_CUDA(launch_flat_merge_rescore<RowT>(
        rows, d, idx->pos_of_kr.as<uint32_t>(), idx->keys.as<uint64_t>(), qf.as<float>(),
        qn2.as<float>(), idx->max_n2.as<unsigned>(), ids.as<int>(), nl, metric, k, o.radius, 1,
        pkeys.as<uint64_t>(), pcounts.as<int>(), psat.as<uint64_t>(), parts, kp, d_keys_out,
        d_scores_out, d_counts_out, qflags.as<int>(), s));
    count_launches(2);
    XVEC_CUDA(cudaMemcpyAsync(h_flags.data(), qflags.ptr, (size_t)nq * 4, cudaMemcpyDeviceToHost,
                              s));
    XVEC_CUDA(cudaStreamSynchronize(s));
    // The exact path selects exactly k keys per part and never fails its
    // coverage check; a failure here is an internal error, not a result.
    for (int q : exact_list) {
      if (h_flags[q] & 2) {
        set_error("exact scan could not complete query %d", q);
        return XVEC_GPU_CUDA_ERROR;
      }
    }
  }
  apply_status_kernel<<<blocks_for(nq), 256, 0, s>>>(qstatus.as<int>(), qflags.as<int>(), nq,
                                                     d_counts_out);
  XVEC_LAUNCHED();
  XVEC_CUDA(cudaGetLastError());
  timer.mark(3);
  XVEC_CUDA(cudaStreamSynchronize(s));
  count_search(nq, (int64_t)exact_list.size(), timer.ms(1, 2), timer.ms(0, 3));
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

xvec_gpu_status validate_search(xvec_gpu_index* idx, int nq, const xvec_gpu_search_opts* o) {
  if (!idx || !o) return set_error("nil index or options"), XVEC_GPU_INVALID_ARGUMENT;
  if (nq < 0) return set_error("negative query count"), XVEC_GPU_INVALID_ARGUMENT;
  if (o->top_k <= 0) return set_error("core: top-k must be positive"), XVEC_GPU_INVALID_ARGUMENT;
  if (o->top_k > 1024)
    return set_error("top_k %d exceeds the supported maximum of 1024", o->top_k),
           XVEC_GPU_INVALID_ARGUMENT;
  if (!(o->radius >= 0) || std::isinf(o->radius))
    return set_error("core: radius must be finite and non-negative"), XVEC_GPU_INVALID_ARGUMENT;
  if (o->filter_bitmap && o->filter_words * 32 < idx->n)
    return set_error("filter bitmap has %lld words, need %lld", (long long)o->filter_words,
                     (long long)((idx->n + 31) / 32)),
           XVEC_GPU_INVALID_ARGUMENT;
  return XVEC_GPU_OK;
}

xvec_gpu_status search_device_locked(xvec_gpu_index* idx, const void* d_q, int nq,
                                     const xvec_gpu_search_opts& o, const uint32_t* d_bitmap,
                                     uint64_t* d_keys, float* d_scores, int* d_counts,
                                     cudaStream_t s, std::vector<int>* statuses,
                                     BandExchange* band) {
  switch (idx->desc.kind) {
    case XVEC_INDEX_FLAT:
      if (idx->desc.storage == XVEC_STORAGE_FP16)
        return flat_search_impl<__half>(idx, d_q, nq, o, d_bitmap, d_keys, d_scores, d_counts, s,
                                        statuses, band);
      return flat_search_impl<float>(idx, d_q, nq, o, d_bitmap, d_keys, d_scores, d_counts, s,
                                     statuses, band);
    case XVEC_INDEX_SQ8_FLAT:
    case XVEC_INDEX_SQ4_FLAT:
      return sq8_search_impl(idx, static_cast<const float*>(d_q), nq, o, d_bitmap, d_keys,
                             d_scores, d_counts, s, statuses);
    case XVEC_INDEX_IVF_PQ:
      return ivfpq_search_impl(idx, static_cast<const float*>(d_q), nq, o, d_bitmap, d_keys,
                               d_scores, d_counts, s, statuses);
    case XVEC_INDEX_RABITQ:
      return rabitq_search_impl(idx, static_cast<const float*>(d_q), nq, o, d_bitmap, d_keys,
                                d_scores, d_counts, s, statuses);
    case XVEC_INDEX_IVF_FLAT:
      return ivf_flat_search_impl(idx, static_cast<const float*>(d_q), nq, o, d_bitmap, d_keys,
                                  d_scores, d_counts, s, statuses);
    case XVEC_INDEX_IVF_SQ8:
    case XVEC_INDEX_IVF_SQ4:
      return ivf_sq8_search_impl(idx, static_cast<const float*>(d_q), nq, o, d_bitmap, d_keys,
                                 d_scores, d_counts, s, statuses);
    case XVEC_INDEX_DISKANN:
      // searchDiskANN (diskann.go:476-525): ListSize (opts.ef; 0 =
      // DefaultDiskANNQueryList) must be positive; Linear scans every node
      // exactly (searchDiskANNLinear :527-557, the Flat search's result).
      if (o.ef < 0)
        return set_error("core: invalid DiskANN list size"), XVEC_GPU_INVALID_ARGUMENT;
      if (o.linear)
        return flat_search_impl<float>(idx, d_q, nq, o, d_bitmap, d_keys, d_scores, d_counts, s,
                                       statuses, band);
      return diskann_search_impl(idx, static_cast<const float*>(d_q), nq, o, d_bitmap, d_keys,
                                 d_scores, d_counts, s, statuses);
    default: return set_error("invalid index kind"), XVEC_GPU_INVALID_ARGUMENT;
  }
}

size_t query_elem_bytes(const xvec_gpu_index* idx) {
  return (idx->desc.kind == XVEC_INDEX_FLAT && idx->desc.storage == XVEC_STORAGE_FP16) ? 2 : 4;
}

// ---------------------------------------------------------------------------
// Insertion.
// ---------------------------------------------------------------------------
// Grows every per-row buffer to `cap` rows, keeping the rows already stored
// (each buffer briefly exists twice while it is copied).
static xvec_gpu_status grow_locked(xvec_gpu_index* idx, int64_t cap, cudaStream_t s) {
  const int64_t old_n = idx->n;
  const size_t in_row_bytes = (size_t)idx->desc.dimension * query_elem_bytes(idx);
  xvec_gpu_status st;
  if ((st = idx->rows.reserve((size_t)cap * in_row_bytes, (size_t)old_n * in_row_bytes, s)) ||
      (st = idx->keys.reserve((size_t)cap * 8, (size_t)old_n * 8, s)) ||
      (st = idx->row_n2.reserve((size_t)cap * 4, (size_t)old_n * 4, s)) ||
      (st = idx->row_inv.reserve((size_t)cap * 4, (size_t)old_n * 4, s)) ||
      (st = idx->keyrank.reserve((size_t)cap * 4, (size_t)old_n * 4, s)) ||
      (st = idx->pos_of_kr.reserve((size_t)cap * 4, (size_t)old_n * 4, s)))
    return st;
  if ((st = extra_reserve(idx, cap, s))) return st;
  idx->capacity = cap;
  return XVEC_GPU_OK;
}

xvec_gpu_status add_device_locked(xvec_gpu_index* idx, const uint64_t* d_keys, const void* d_rows,
                                  int64_t m, cudaStream_t s) {
  const int d = idx->desc.dimension;
  const int64_t old_n = idx->n, new_n = old_n + m;
  if (m == 0) return XVEC_GPU_OK;
  if (new_n > 0xffffffffll) return set_error("index capacity exceeded"), XVEC_GPU_INVALID_ARGUMENT;
  const size_t in_row_bytes = (size_t)d * query_elem_bytes(idx);
  if (new_n > idx->capacity) {
    xvec_gpu_status st =
        grow_locked(idx, std::max<int64_t>(new_n, idx->capacity + idx->capacity / 2), s);
    if (st) return st;
  }
  if (!idx->max_n2.ptr) {
    xvec_gpu_status st = idx->max_n2.reserve(4, 0, s);
    if (st) return st;
    XVEC_CUDA(cudaMemsetAsync(idx->max_n2.ptr, 0, 4, s));
  }
  XVEC_CUDA(cudaMemcpyAsync(idx->rows.as<char>() + (size_t)old_n * in_row_bytes, d_rows,
                            (size_t)m * in_row_bytes, cudaMemcpyDeviceToDevice, s));
  XVEC_CUDA(cudaMemcpyAsync(idx->keys.as<uint64_t>() + old_n, d_keys, (size_t)m * 8,
                            cudaMemcpyDeviceToDevice, s));
  // Finite check and reference-order norms of the new rows
  // (mathutil.L2Squared(vector, vector) validation, flat.go:134-136).
  Scratch nonfinite;
  xvec_gpu_status st = nonfinite.alloc(4, s);
  if (st) return st;
  XVEC_CUDA(cudaMemsetAsync(nonfinite.ptr, 0, 4, s));
  // Norms go to a scratch max first so a rejected batch leaves no trace.
  Scratch max_new;
  if ((st = max_new.alloc(4, s))) return st;
  XVEC_CUDA(cudaMemcpyAsync(max_new.ptr, idx->max_n2.ptr, 4, cudaMemcpyDeviceToDevice, s));
  if (idx->desc.kind == XVEC_INDEX_FLAT && idx->desc.storage == XVEC_STORAGE_FP16)
    launch_row_norms<__half>(idx->rows.as<__half>() + (size_t)old_n * d, m, d,
                             idx->row_n2.as<float>() + old_n, idx->row_inv.as<float>() + old_n,
                             max_new.as<unsigned>(), nonfinite.as<int>(), s);
  else
    launch_row_norms<float>(idx->rows.as<float>() + (size_t)old_n * d, m, d,
                            idx->row_n2.as<float>() + old_n, idx->row_inv.as<float>() + old_n,
                            max_new.as<unsigned>(), nonfinite.as<int>(), s);
  XVEC_CUDA(cudaGetLastError());
  int h_nonfinite = 0;
  XVEC_CUDA(cudaMemcpyAsync(&h_nonfinite, nonfinite.ptr, 4, cudaMemcpyDeviceToHost, s));
  XVEC_CUDA(cudaStreamSynchronize(s));
  if (h_nonfinite) return set_error("ailego: vector contains a non-finite value"), XVEC_GPU_NON_FINITE;
  if ((st = extra_validate(idx, old_n, m, s))) return st;
  if ((st = rebuild_keyrank(idx, new_n, s))) {
    // keyrank of the old rows was not touched; restore nothing else.
    return st;
  }
  if ((st = extra_commit(idx, old_n, m, s))) {
    rebuild_keyrank(idx, old_n, s);
    return st;
  }
  XVEC_CUDA(cudaMemcpyAsync(idx->max_n2.ptr, max_new.ptr, 4, cudaMemcpyDeviceToDevice, s));
  XVEC_CUDA(cudaStreamSynchronize(s));
  idx->n = new_n;
  return XVEC_GPU_OK;
}

}  // namespace xvec

using namespace xvec;

// ---------------------------------------------------------------------------
// Exported entry points.
// ---------------------------------------------------------------------------
extern "C" int32_t xvec_gpu_abi_version(void) { return XVEC_GPU_ABI_VERSION; }

extern "C" size_t xvec_gpu_last_error(char* buffer, size_t length) {
  const std::string& e = g_last_error;
  if (buffer && length) {
    size_t c = std::min(length - 1, e.size());
    memcpy(buffer, e.data(), c);
    buffer[c] = 0;
  }
  return e.size();
}

extern "C" int32_t xvec_gpu_device_count(void) {
  int count = 0;
  if (cudaGetDeviceCount(&count) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  int usable = 0;
  for (int i = 0; i < count; ++i) {
    cudaDeviceProp p;
    if (cudaGetDeviceProperties(&p, i) == cudaSuccess && p.major == 10 && p.minor == 0) ++usable;
  }
  return usable;
}

extern "C" xvec_gpu_status xvec_gpu_index_create(const xvec_gpu_index_desc* desc,
                                                 xvec_gpu_index** out) {
  if (!desc || !out) return set_error("nil argument"), XVEC_GPU_INVALID_ARGUMENT;
  *out = nullptr;
  if (desc->dimension <= 0)
    return set_error("core: invalid vector dimension: got %d", desc->dimension),
           XVEC_GPU_INVALID_ARGUMENT;
  if (desc->metric < XVEC_METRIC_L2 || desc->metric > XVEC_METRIC_MIPSL2)
    return set_error("core: invalid metric"), XVEC_GPU_INVALID_ARGUMENT;
  switch (desc->kind) {
    case XVEC_INDEX_FLAT:
      if (desc->storage != XVEC_STORAGE_FP32 && desc->storage != XVEC_STORAGE_FP16)
        return set_error("invalid storage"), XVEC_GPU_INVALID_ARGUMENT;
      break;
    case XVEC_INDEX_SQ8_FLAT:
    case XVEC_INDEX_SQ4_FLAT:
    case XVEC_INDEX_IVF_SQ8:
    case XVEC_INDEX_IVF_SQ4:
      if (desc->dimension > 65535)
        return set_error("core: invalid vector dimension: got %d", desc->dimension),
               XVEC_GPU_INVALID_ARGUMENT;
      break;
    case XVEC_INDEX_IVF_PQ:
      if (desc->metric != XVEC_METRIC_L2 && desc->metric != XVEC_METRIC_IP)
        return set_error("core: invalid PQ options: core: PQ supports L2 and IP only"),
               XVEC_GPU_INVALID_ARGUMENT;
      break;
    case XVEC_INDEX_RABITQ:
      if (desc->metric == XVEC_METRIC_MIPSL2)
        return set_error("core: RaBitQ supports L2, IP, and cosine only"),
               XVEC_GPU_INVALID_ARGUMENT;
      if (desc->dimension < 64 || desc->dimension > 4095)
        return set_error("core: invalid RaBitQ options: dimension must be in [64,4095]"),
               XVEC_GPU_INVALID_ARGUMENT;
      break;
    case XVEC_INDEX_IVF_FLAT:
      break;
    case XVEC_INDEX_DISKANN:
      // NewDiskANNLayout (diskann_storage.go:68-70).
      if (desc->dimension > 65535)
        return set_error("core: invalid DiskANN layout: dimension must be in [1,65535]"),
               XVEC_GPU_INVALID_ARGUMENT;
      if (desc->storage != XVEC_STORAGE_FP32)
        return set_error("DiskANN node vectors are float32"), XVEC_GPU_INVALID_ARGUMENT;
      break;
    default: return set_error("invalid index kind %d", desc->kind), XVEC_GPU_INVALID_ARGUMENT;
  }
  int count = 0;
  if (cudaGetDeviceCount(&count) != cudaSuccess || desc->device < 0 || desc->device >= count) {
    cudaGetLastError();
    return set_error("CUDA device %d is not available", desc->device), XVEC_GPU_UNSUPPORTED;
  }
  cudaDeviceProp p;
  if (cudaGetDeviceProperties(&p, desc->device) != cudaSuccess || p.major != 10 || p.minor != 0)
    return set_error("device %d is not an sm_100 (B200) device", desc->device),
           XVEC_GPU_UNSUPPORTED;
  cudaSetDevice(desc->device);
  // Keep freed stream-ordered scratch in the pool between searches.
  cudaMemPool_t pool;
  if (cudaDeviceGetDefaultMemPool(&pool, desc->device) == cudaSuccess) {
    uint64_t threshold = UINT64_MAX;
    cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &threshold);
  }
  xvec_gpu_index* idx = new (std::nothrow) xvec_gpu_index();
  if (!idx) return set_error("out of host memory"), XVEC_GPU_OUT_OF_MEMORY;
  idx->desc = *desc;
  idx->device = desc->device;
  if (desc->kind == XVEC_INDEX_RABITQ) idx->padded = (desc->dimension + 63) / 64 * 64;
  *out = idx;
  return XVEC_GPU_OK;
}

extern "C" xvec_gpu_status xvec_gpu_index_destroy(xvec_gpu_index* idx) {
  if (!idx) return XVEC_GPU_OK;
  cudaSetDevice(idx->device);
  cudaDeviceSynchronize();
  delete idx;
  return XVEC_GPU_OK;
}

extern "C" int64_t xvec_gpu_index_len(const xvec_gpu_index* idx) { return idx ? idx->n : 0; }

extern "C" xvec_gpu_status xvec_gpu_index_reserve(xvec_gpu_index* idx, int64_t capacity) {
  if (!idx || capacity < 0 || capacity > 0xffffffffll)
    return set_error("invalid reserve arguments"), XVEC_GPU_INVALID_ARGUMENT;
  std::unique_lock<std::shared_mutex> lock(idx->mu);
  if (capacity <= idx->capacity) return XVEC_GPU_OK;
  cudaSetDevice(idx->device);
  xvec_gpu_status st = grow_locked(idx, capacity, nullptr);
  cudaStreamSynchronize(nullptr);
  return st;
}

extern "C" xvec_gpu_status xvec_gpu_index_add_device(xvec_gpu_index* idx, const uint64_t* d_keys,
                                                     const void* d_rows, int64_t n,
                                                     void* stream) {
  if (!idx || n < 0 || (n > 0 && (!d_keys || !d_rows)))
    return set_error("invalid add arguments"), XVEC_GPU_INVALID_ARGUMENT;
  std::unique_lock<std::shared_mutex> lock(idx->mu);
  cudaSetDevice(idx->device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  xvec_gpu_status st = add_device_locked(idx, d_keys, d_rows, n, s);
  cudaStreamSynchronize(s);
  return st;
}

extern "C" xvec_gpu_status xvec_gpu_index_add(xvec_gpu_index* idx, const uint64_t* keys,
                                              const void* rows, int64_t n) {
  if (!idx || n < 0 || (n > 0 && (!keys || !rows)))
    return set_error("invalid add arguments"), XVEC_GPU_INVALID_ARGUMENT;
  if (n == 0) return XVEC_GPU_OK;
  std::unique_lock<std::shared_mutex> lock(idx->mu);
  cudaSetDevice(idx->device);
  cudaStream_t s = thread_stream(idx->device);
  const size_t row_bytes = (size_t)idx->desc.dimension * query_elem_bytes(idx);
  Scratch dk, dr;
  xvec_gpu_status st;
  if ((st = dk.alloc((size_t)n * 8, s)) || (st = dr.alloc((size_t)n * row_bytes, s))) return st;
  XVEC_CUDA(cudaMemcpyAsync(dk.ptr, keys, (size_t)n * 8, cudaMemcpyHostToDevice, s));
  XVEC_CUDA(cudaMemcpyAsync(dr.ptr, rows, (size_t)n * row_bytes, cudaMemcpyHostToDevice, s));
  st = add_device_locked(idx, dk.as<uint64_t>(), dr.ptr, n, s);
  cudaStreamSynchronize(s);
  return st;
}

extern "C" xvec_gpu_status xvec_gpu_index_search_device(xvec_gpu_index* idx, const void* d_q,
                                                        int32_t nq,
                                                        const xvec_gpu_search_opts* opts,
                                                        uint64_t* d_keys, float* d_scores,
                                                        int32_t* d_counts) {
  xvec_gpu_status st = validate_search(idx, nq, opts);
  if (st) return st;
  if (nq == 0) return XVEC_GPU_OK;
  std::shared_lock<std::shared_mutex> lock(idx->mu);
  cudaSetDevice(idx->device);
  cudaStream_t s = static_cast<cudaStream_t>(opts->stream);
  std::vector<int> statuses;
  st = search_device_locked(idx, d_q, nq, *opts, opts->filter_bitmap, d_keys, d_scores, d_counts,
                            s, &statuses);
  if (st) return st;
  for (int q = 0; q < nq; ++q)
    if (statuses[q]) {
      set_error("query %d failed with status %d", q, statuses[q]);
      return (xvec_gpu_status)statuses[q];
    }
  return XVEC_GPU_OK;
}

extern "C" xvec_gpu_status xvec_gpu_index_search(xvec_gpu_index* idx, const void* queries,
                                                 int32_t nq, const xvec_gpu_search_opts* opts,
                                                 uint64_t* out_keys, float* out_scores,
                                                 int32_t* out_counts) {
  xvec_gpu_status st = validate_search(idx, nq, opts);
  if (st) return st;
  if (nq == 0) return XVEC_GPU_OK;
  if (!queries || !out_keys || !out_scores || !out_counts)
    return set_error("nil buffer"), XVEC_GPU_INVALID_ARGUMENT;
  std::shared_lock<std::shared_mutex> lock(idx->mu);
  cudaSetDevice(idx->device);
  cudaStream_t s = thread_stream(idx->device);
  const int k = opts->top_k;
  const size_t qbytes = (size_t)nq * idx->desc.dimension * query_elem_bytes(idx);
  Scratch dq, dk, ds, dc, dbm;
  if ((st = dq.alloc(qbytes, s)) || (st = dk.alloc((size_t)nq * k * 8, s)) ||
      (st = ds.alloc((size_t)nq * k * 4, s)) || (st = dc.alloc((size_t)nq * 4, s)))
    return st;
  XVEC_CUDA(cudaMemcpyAsync(dq.ptr, queries, qbytes, cudaMemcpyHostToDevice, s));
  const uint32_t* d_bitmap = nullptr;
  if (opts->filter_bitmap) {
    const size_t words = (size_t)std::max<int64_t>(1, (idx->n + 31) / 32);
    if ((st = dbm.alloc(words * 4, s))) return st;
    XVEC_CUDA(cudaMemcpyAsync(dbm.ptr, opts->filter_bitmap, words * 4, cudaMemcpyHostToDevice, s));
    d_bitmap = dbm.as<uint32_t>();
  }
  std::vector<int> statuses;
  st = search_device_locked(idx, dq.ptr, nq, *opts, d_bitmap, dk.as<uint64_t>(), ds.as<float>(),
                            dc.as<int>(), s, &statuses);
  if (st) return st;
  XVEC_CUDA(cudaMemcpyAsync(out_keys, dk.ptr, (size_t)nq * k * 8, cudaMemcpyDeviceToHost, s));
  XVEC_CUDA(cudaMemcpyAsync(out_scores, ds.ptr, (size_t)nq * k * 4, cudaMemcpyDeviceToHost, s));
  XVEC_CUDA(cudaMemcpyAsync(out_counts, dc.ptr, (size_t)nq * 4, cudaMemcpyDeviceToHost, s));
  XVEC_CUDA(cudaStreamSynchronize(s));
  for (int q = 0; q < nq; ++q)
    if (statuses[q]) {
      set_error("query %d failed with status %d", q, statuses[q]);
      return (xvec_gpu_status)statuses[q];
    }
  return XVEC_GPU_OK;
}
