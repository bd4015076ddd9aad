// flat_stream.cu — streaming candidate scan for Flat search over a few queries.
//
// The reference's Flat query is one query against every row
// (Collection.Query, collection.go:3830, into topKPrevalidatedCandidatesWithOptions,
// internal/core/topk.go:105-166).  For one to a few queries the work is a pass over
// the rows in HBM, not a GEMM: the tensor-core scan would compute a 128-query tile
// to use one of its rows.  This scan reads every row once with 128-bit loads and
// ranks it against the batch with FFMA, so it runs at HBM speed.
//
//   CTA = 16 warps, one CTA per SM, each CTA a contiguous range of rows.  A group
//   of 8 lanes owns a row: lane j of the group loads 16-byte chunks j, j + 8, ...
//   of it (up to 12 chunks in flight per lane), multiplies them by the queries (float32,
//   in shared memory) and the group sums its partial dots with three shuffles.
//   Lane j of the group then ranks the row for query j (the Flat fast rank of the
//   other scans), and appends its packed key (rank << 32 | key rank) to the warp's
//   list for query j (shared memory) when it is below the warp's threshold.  A
//   full list is compacted to its kp best keys by the warp, which lowers the
//   threshold.  At the end the CTA merges its warps' lists into one list of at
//   most kp keys per query (global memory).
//
// A search runs the scan twice: first over every 64th row (a sample whose kp best
// keys per query bound the kp-th best key of all rows from above), then over all
// rows with that bound as every warp's starting threshold, so only about
// kp x 64 rows per query are appended.  reduce_lists_kernel (pipeline.cuh) turns the CTA lists
// into the bound (sample) or into the one candidate list per query (main) that
// the common merge rescores in the reference's order (pipeline.cuh).  The sample's
// lists are only used for the bound, so no row is listed twice.
//
// Coverage: each list records the key below which it kept everything (its
// saturation); the merge sends a query to the exact scan when a saturation
// lies within its candidate limit.
#include <algorithm>
#include <cstdlib>

#include "capi_internal.h"
#include "flat_kernels.cuh"
#include "pipeline.cuh"

namespace xvec {

namespace {

constexpr int kStreamWarps = 16;
constexpr int kStreamThreads = kStreamWarps * 32;
constexpr int kStreamMaxQ = 4;      // queries per launch
constexpr int kStreamMaxKp = 128;   // candidate list length (kp) the scan serves
constexpr int kStreamSlack = 32;    // list entries beyond kp before a compaction
constexpr int kSampleStep = 64;     // the sample pass reads every 64th row

// The queries in shared memory with 4 floats of padding after every 32: the
// 16-byte chunk loads of a lane group (chunks j, j + 1, ... of one query)
// then fall on distinct banks.  A chunk (8 FP16 or 4 FP32 elements) never
// straddles the padding.
__host__ __device__ __forceinline__ int qpad(int i) { return i + (i >> 5) * 4; }
__host__ __device__ __forceinline__ int qstride(int d) { return qpad(d) + 4; }

// 16 bytes of a row as floats.
__device__ __forceinline__ void unpack16(const uint4& v, float* x, const __half*) {
  const __half2* h = reinterpret_cast<const __half2*>(&v);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __half22float2(h[i]);
    x[2 * i] = f.x;
    x[2 * i + 1] = f.y;
  }
}
__device__ __forceinline__ void unpack16(const uint4& v, float* x, const float*) {
  x[0] = __uint_as_float(v.x);
  x[1] = __uint_as_float(v.y);
  x[2] = __uint_as_float(v.z);
  x[3] = __uint_as_float(v.w);
}

__device__ __forceinline__ uint4 ldg_stream(const uint4* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

// Keeps the kp smallest of the cnt keys of a shared-memory list (the warp
// calls it together) and returns the kp-th smallest.  Keys are unique.
__device__ uint64_t warp_compact_smem(uint64_t* list, int cnt, int kp, int* hist) {
  const int lane = threadIdx.x & 31;
  __syncwarp();
  uint64_t prefix = 0;
  int kth = kp;
#pragma unroll 1
  for (int shift = 56; shift >= 0; shift -= 8) {
    for (int b = lane; b < 256; b += 32) hist[b] = 0;
    __syncwarp();
    const uint64_t mask = shift == 56 ? 0ull : (~0ull << (shift + 8));
    for (int i = lane; i < cnt; i += 32) {
      const uint64_t key = list[i];
      if ((key & mask) == prefix) atomicAdd(&hist[(key >> shift) & 0xff], 1);
    }
    __syncwarp();
    int local[8], sum = 0;
#pragma unroll
    for (int b = 0; b < 8; ++b) {
      local[b] = hist[lane * 8 + b];
      sum += local[b];
    }
    int incl = sum;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(kFullMask, incl, o);
      if (lane >= o) incl += v;
    }
    const int excl = incl - sum;
    const unsigned owner = __ballot_sync(kFullMask, excl < kth && kth <= incl);
    const int src = __ffs(owner) - 1;
    int digit = 0, rem = kth - excl;
#pragma unroll
    for (int b = 0; b < 8; ++b) {
      if (rem > 0 && rem <= local[b]) {
        digit = lane * 8 + b;
        rem = -rem;
      } else if (rem > 0) {
        rem -= local[b];
      }
    }
    digit = __shfl_sync(kFullMask, digit, src);
    kth = -__shfl_sync(kFullMask, rem, src);
    prefix |= (uint64_t)digit << shift;
    __syncwarp();
  }
  // Keep the keys <= prefix (exactly kp of them), in slot order.
  int out = 0;
  for (int base = 0; base < cnt; base += 32) {
    const int i = base + lane;
    const uint64_t key = i < cnt ? list[i] : kEmptyKey;
    const bool keep = i < cnt && key <= prefix;
    const unsigned m = __ballot_sync(kFullMask, keep);
    __syncwarp();
    if (keep) list[out + __popc(m & ((1u << lane) - 1))] = key;
    out += __popc(m);
    __syncwarp();
  }
  return prefix;
}

// rows [cta_begin, cta_end) of this CTA, visited at a stride of row_step.
// CPL: 16-byte chunks a lane loads at once (a whole row of d <= 64 CPL
// FP16 or 32 CPL FP32 elements per round of loads).
template <typename RowT, int CPL>
__global__ void __launch_bounds__(kStreamThreads, 1) flat_stream_kernel(
    const RowT* __restrict__ rows, int64_t n, int d, const float* __restrict__ row_n2,
    const uint32_t* __restrict__ keyrank, const float* __restrict__ qf,
    const float* __restrict__ q_n2, int nq, int metric, const uint32_t* __restrict__ bitmap,
    int64_t rows_per_cta, int row_step, int kp, const unsigned long long* __restrict__ gthr,
    uint64_t* __restrict__ out_keys, int* __restrict__ out_counts,
    uint64_t* __restrict__ out_sat, int* __restrict__ q_flags) {
  extern __shared__ __align__(16) unsigned char stream_smem[];
  const int lcap = kp + kStreamSlack;
  const int qst = qstride(d);
  float* qs = reinterpret_cast<float*>(stream_smem);                     // [nq][qst], padded
  uint64_t* lists = reinterpret_cast<uint64_t*>(qs + (size_t)kStreamMaxQ * qst);  // [W][nq][lcap]
  uint64_t* mbuf = lists + (size_t)kStreamWarps * kStreamMaxQ * lcap;         // [W * lcap]
  int* hists = reinterpret_cast<int*>(mbuf + (size_t)kStreamWarps * lcap);   // [W][256]
  __shared__ int s_cnt[kStreamWarps][kStreamMaxQ];
  __shared__ uint64_t s_thr[kStreamWarps][kStreamMaxQ];
  __shared__ int s_off[kStreamWarps + 1];
  __shared__ int s_nonfinite[kStreamMaxQ];

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 3, j = lane & 7;  // row group of the warp step, lane in group
  const int cta = blockIdx.x, num_ctas = gridDim.x;
  const int64_t cta_begin = (int64_t)cta * rows_per_cta;
  const int64_t cta_end = min(n, cta_begin + rows_per_cta);
  const int elems = 16 / (int)sizeof(RowT);
  const int nchunks = d / elems;

  for (int i = threadIdx.x; i < nq * d; i += kStreamThreads) {
    const int q = i / d, e = i - q * d;
    qs[q * qst + qpad(e)] = qf[i];
  }
  if (threadIdx.x < kStreamMaxQ) s_nonfinite[threadIdx.x] = 0;
  __syncthreads();

  const bool qlane = j < nq;  // this lane ranks the group's row for query j
  const float qn2_j = qlane ? q_n2[j] : 0.f;
  uint64_t thr = (qlane && gthr) ? (uint64_t)gthr[j] : kEmptyKey;
  int cnt = 0;
  int nonfinite = 0;
  uint64_t* my_list = lists + ((size_t)warp * kStreamMaxQ + (qlane ? j : 0)) * lcap;
  int* hist = hists + warp * 256;

  // Visits t = 0, 1, ... of this CTA: row = cta_begin + t * row_step.
  const int64_t visits = cta_end > cta_begin ? (cta_end - cta_begin + row_step - 1) / row_step : 0;
  for (int64_t t0 = (int64_t)warp * 4; t0 < visits; t0 += (int64_t)kStreamWarps * 4) {
    const int64_t t = t0 + g;
    const bool valid = t < visits;
    const int64_t row = valid ? cta_begin + t * row_step : cta_begin;
    const bool pass_filter = valid && bitmap_pass(bitmap, row);
    // Row metadata first: its latency overlaps the row's loads.
    const float xn2 = pass_filter ? row_n2[row] : 0.f;
    const uint32_t kr = pass_filter ? keyrank[row] : 0u;
    const uint4* src = reinterpret_cast<const uint4*>(rows + row * d);
    float acc[kStreamMaxQ];
#pragma unroll
    for (int q = 0; q < kStreamMaxQ; ++q) acc[q] = 0.f;
    for (int c0 = j; c0 < nchunks; c0 += 8 * CPL) {
      uint4 v[CPL];
#pragma unroll
      for (int u = 0; u < CPL; ++u) {
        const int c = c0 + 8 * u;
        v[u] = (pass_filter && c < nchunks) ? ldg_stream(src + c) : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int u = 0; u < CPL; ++u) {
        const int c = c0 + 8 * u;
        if (c < nchunks) {
          float x[16 / sizeof(RowT)];
          unpack16(v[u], x, static_cast<const RowT*>(nullptr));
#pragma unroll
          for (int q = 0; q < kStreamMaxQ; ++q) {
            if (q < nq) {
              // 16-byte aligned: d and qpad keep multiples of 4 floats.
              const float4* qq =
                  reinterpret_cast<const float4*>(qs + (size_t)q * qst + qpad(c * elems));
#pragma unroll
              for (int e4 = 0; e4 < 4 / (int)sizeof(RowT); ++e4) {  // float4s per chunk
                const float4 w = qq[e4];
                acc[q] = fmaf(x[4 * e4], w.x, acc[q]);
                acc[q] = fmaf(x[4 * e4 + 1], w.y, acc[q]);
                acc[q] = fmaf(x[4 * e4 + 2], w.z, acc[q]);
                acc[q] = fmaf(x[4 * e4 + 3], w.w, acc[q]);
              }
            }
          }
        }
      }
    }
#pragma unroll
    for (int q = 0; q < kStreamMaxQ; ++q) {
      acc[q] += __shfl_xor_sync(kFullMask, acc[q], 1);
      acc[q] += __shfl_xor_sync(kFullMask, acc[q], 2);
      acc[q] += __shfl_xor_sync(kFullMask, acc[q], 4);
    }
    float dot = acc[0];
#pragma unroll
    for (int q = 1; q < kStreamMaxQ; ++q)
      if (j == q) dot = acc[q];
    bool pass = false;
    uint64_t key = kEmptyKey;
    if (qlane && pass_filter) {
      const float r = fast_rank(metric, dot, xn2, qn2_j);
      if (!isfinite(r)) {
        nonfinite = 1;
      } else {
        key = pack_rank(r, kr);
        pass = key < thr;
      }
    }
    const unsigned m = __ballot_sync(kFullMask, pass);
    if (m != 0u) {
      const unsigned same = m & (0x01010101u << j);
      if (pass) my_list[cnt + __popc(same & ((1u << lane) - 1))] = key;
      cnt += __popc(same);
      // Compact a list that may not hold the next step's appends.
      unsigned full = __ballot_sync(kFullMask, qlane && cnt > lcap - 4) & 0xffu;
      while (full) {
        const int q = __ffs(full) - 1;
        full &= full - 1;
        const int qcnt = __shfl_sync(kFullMask, cnt, q);
        uint64_t* ql = lists + ((size_t)warp * kStreamMaxQ + q) * lcap;
        const uint64_t kth = warp_compact_smem(ql, qcnt, kp, hist);
        if (j == q) {
          cnt = kp;
          if (kth < thr) thr = kth;
        }
      }
    }
  }
  if (nonfinite && qlane) atomicOr(&s_nonfinite[j], 1);
  if (g == 0 && qlane) {
    s_cnt[warp][j] = cnt;
    s_thr[warp][j] = thr;
  }
  __syncthreads();
  // The CTA's list per query: the kp best keys of its warps' lists; its
  // saturation is the lowest warp threshold (every warp dropped only keys
  // at or above its own) and, when keys were left out here, the kp-th key.
  for (int q = 0; q < nq; ++q) {
    if (threadIdx.x == 0) {
      int off = 0;
      for (int w = 0; w < kStreamWarps; ++w) {
        s_off[w] = off;
        off += s_cnt[w][q];
      }
      s_off[kStreamWarps] = off;
    }
    __syncthreads();
    const int total = s_off[kStreamWarps];
    for (int w = warp; w < kStreamWarps; w += kStreamWarps) {
      const uint64_t* wl = lists + ((size_t)w * kStreamMaxQ + q) * lcap;
      for (int i = lane; i < s_cnt[w][q]; i += 32) mbuf[s_off[w] + i] = wl[i];
    }
    __syncthreads();
    uint64_t sat = kEmptyKey;
    for (int w = 0; w < kStreamWarps; ++w) sat = min(sat, s_thr[w][q]);
    uint64_t kth = kEmptyKey;
    if (total > kp) {
      kth = smem_radix_select(mbuf, total, kp, 0, hists);
      sat = min(sat, kth);
    }
    uint64_t* dst = out_keys + ((int64_t)q * num_ctas + cta) * kp;
    __shared__ int s_n;
    if (threadIdx.x == 0) s_n = 0;
    __syncthreads();
    for (int i = threadIdx.x; i < total; i += kStreamThreads) {
      const uint64_t key = mbuf[i];
      if (key <= kth) dst[atomicAdd(&s_n, 1)] = key;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      out_counts[(int64_t)q * num_ctas + cta] = s_n;
      out_sat[(int64_t)q * num_ctas + cta] = sat;
      if (s_nonfinite[q]) atomicOr(&q_flags[q], 1);
    }
    __syncthreads();
  }
}

template <typename RowT>
size_t stream_smem_bytes(int d, int kp) {
  const int lcap = kp + kStreamSlack;
  return (size_t)kStreamMaxQ * qstride(d) * 4 + (size_t)kStreamWarps * kStreamMaxQ * lcap * 8 +
         (size_t)kStreamWarps * lcap * 8 + (size_t)kStreamWarps * 256 * 4;
}

}  // namespace

int flat_stream_list_stride(int kp) { return reduce_lists_out_cap(kp); }

int flat_stream_max_batch() {
  static const int limit = [] {
    const char* e = std::getenv("XVEC_GPU_STREAM_MAX_BATCH");
    int v = e ? std::atoi(e) : kStreamMaxQ;
    return std::max(0, std::min(v, kStreamMaxQ));
  }();
  return limit;
}

template <typename RowT>
bool flat_stream_supported(int nq, int64_t n, int d, int kp, const void* rows, const void* q) {
  const int elems = 16 / (int)sizeof(RowT);
  if (nq < 1 || nq > flat_stream_max_batch() || kp > kStreamMaxKp || d % elems != 0) return false;
  if (n < 4096 || n >= (1ll << 31)) return false;
  if (reinterpret_cast<uintptr_t>(rows) % 16 != 0) return false;
  (void)q;
  return stream_smem_bytes<RowT>(d, kp) <= 200 * 1024;
}
template bool flat_stream_supported<float>(int, int64_t, int, int, const void*, const void*);
template bool flat_stream_supported<__half>(int, int64_t, int, int, const void*, const void*);

template <typename RowT>
xvec_gpu_status flat_stream_scan(int device, const RowT* rows, int64_t n, int d,
                                 const float* row_n2, const uint32_t* keyrank, const float* qf,
                                 const float* q_n2, int nq, int metric, const uint32_t* bitmap,
                                 int kp, cudaStream_t s, Scratch& lkeys, Scratch& lcounts,
                                 Scratch& lsat, int* q_flags) {
  int sms = 148;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
  const int ctas = sms;
  const size_t smem = stream_smem_bytes<RowT>(d, kp);
  const int cpl_need = (d / (16 / (int)sizeof(RowT)) + 7) / 8;
  auto kern = cpl_need <= 1   ? flat_stream_kernel<RowT, 1>
              : cpl_need <= 2 ? flat_stream_kernel<RowT, 2>
              : cpl_need <= 4 ? flat_stream_kernel<RowT, 4>
              : cpl_need <= 8 ? flat_stream_kernel<RowT, 8>
                              : flat_stream_kernel<RowT, 12>;
  XVEC_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  Scratch ckeys, ccounts, csat, gthr;
  xvec_gpu_status st;
  if ((st = ckeys.alloc((size_t)nq * ctas * kp * 8, s)) ||
      (st = ccounts.alloc((size_t)nq * ctas * 4, s)) ||
      (st = csat.alloc((size_t)nq * ctas * 8, s)) || (st = gthr.alloc((size_t)nq * 8, s)) ||
      (st = lkeys.alloc((size_t)nq * reduce_lists_out_cap(kp) * 8, s)) ||
      (st = lcounts.alloc((size_t)nq * 4, s)) ||
      (st = lsat.alloc((size_t)nq * 8, s)))
    return st;
  XVEC_CUDA(cudaMemsetAsync(gthr.ptr, 0xff, (size_t)nq * 8, s));
  // Sample pass: every 64th row, for the starting thresholds.
  const int64_t per_cta = (n + ctas - 1) / ctas;
  if (n / kSampleStep >= kp) {
    kern<<<ctas, kStreamThreads, smem, s>>>(rows, n, d, row_n2, keyrank, qf, q_n2, nq, metric,
                                            bitmap, per_cta, kSampleStep, kp, nullptr,
                                            ckeys.as<uint64_t>(), ccounts.as<int>(),
                                            csat.as<uint64_t>(), q_flags);
    XVEC_CUDA(cudaGetLastError());
    XVEC_CUDA(launch_reduce_lists(ckeys.as<uint64_t>(), ccounts.as<int>(), csat.as<uint64_t>(),
                                  nq, ctas, kp, kp, gthr.as<unsigned long long>(), nullptr,
                                  nullptr, nullptr, s));
    count_launches(2);
  }
  kern<<<ctas, kStreamThreads, smem, s>>>(rows, n, d, row_n2, keyrank, qf, q_n2, nq, metric,
                                          bitmap, per_cta, 1, kp, gthr.as<unsigned long long>(),
                                          ckeys.as<uint64_t>(), ccounts.as<int>(),
                                          csat.as<uint64_t>(), q_flags);
  XVEC_CUDA(cudaGetLastError());
  XVEC_CUDA(launch_reduce_lists(ckeys.as<uint64_t>(), ccounts.as<int>(), csat.as<uint64_t>(), nq,
                                ctas, kp, reduce_lists_out_cap(kp), nullptr,
                                lkeys.as<uint64_t>(), lcounts.as<int>(), lsat.as<uint64_t>(), s));
  count_launches(2);
  return XVEC_GPU_OK;
}
template xvec_gpu_status flat_stream_scan<float>(int, const float*, int64_t, int, const float*,
                                                 const uint32_t*, const float*, const float*, int,
                                                 int, const uint32_t*, int, cudaStream_t,
                                                 Scratch&, Scratch&, Scratch&, int*);
template xvec_gpu_status flat_stream_scan<__half>(int, const __half*, int64_t, int, const float*,
                                                  const uint32_t*, const float*, const float*,
                                                  int, int, const uint32_t*, int, cudaStream_t,
                                                  Scratch&, Scratch&, Scratch&, int*);

}  // namespace xvec
