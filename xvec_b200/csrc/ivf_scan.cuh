// ivf_scan.cuh — the IVF list scan shared by the IVF kinds that score rows
// of the probed lists (exact float32 rows: ivf_flat.cu; INT8 codes:
// sq8.cu).
//
// One 16-warp block per query (query_ids[blockIdx.x] when given) over its
// probed lists (positions in list order): each lane ranks one row with the
// policy's fast rank (within the policy's error bound of the reference
// score); keys below the lists' shared threshold go to per-warp lists
// (ballot appends, warp compaction to the KP best, the lowest list threshold
// shared through shared memory), one list per warp for the merge.  EXACT:
// the policy's reference score, a warp per row (for queries the fast pass
// cannot settle, and for metrics without a fast rank).
//
// Policy:  int smem_bytes(int d)                     -- per-query staging
//          void stage(int q, unsigned char* smem)   -- called by the block
//          float fast_rank(int q, int64_t idx, uint32_t pos,
//                          const unsigned char* smem)  -- one lane, one row
//                                                       (idx: list order)
//          float exact_score(int q, uint32_t pos, const unsigned char* smem)
//                                                    -- the whole warp
//          int metric                               (ranking order)
#pragma once

#include "common.cuh"
#include "select.cuh"

namespace xvec {

constexpr int kIvfWarps = 16;

template <int CAPW, bool EXACT, typename Policy>
__global__ void __launch_bounds__(kIvfWarps * 32, 1) ivf_list_scan_kernel(
    Policy pol, const uint64_t* __restrict__ probe_lists, const int* __restrict__ probe_counts,
    int nprobe, const int64_t* __restrict__ list_offsets, const uint32_t* __restrict__ list_rows,
    const uint32_t* __restrict__ list_keyrank, const uint32_t* __restrict__ bitmap,
    const int* __restrict__ query_ids, int kp, uint64_t* __restrict__ part_keys,
    int* __restrict__ part_counts, uint64_t* __restrict__ part_sat, int* __restrict__ q_flags) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  uint64_t* wbuf = reinterpret_cast<uint64_t*>(smem_raw);  // [warps][CAPW]
  unsigned char* qsmem = reinterpret_cast<unsigned char*>(wbuf + kIvfWarps * CAPW);
  __shared__ AccumState wst[kIvfWarps];
  __shared__ unsigned long long s_thr;
  const int q = query_ids ? query_ids[blockIdx.x] : blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  pol.stage(q, qsmem);
  if (lane == 0) {
    wst[warp].count = 0;
    wst[warp].saturated = 0;
    wst[warp].thr = kEmptyKey;
  }
  if (threadIdx.x == 0) s_thr = kEmptyKey;
  __syncthreads();
  uint64_t* buf = wbuf + warp * CAPW;
  AccumState* st = &wst[warp];
  int cnt = 0;
  uint64_t wthr = kEmptyKey;
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
          const float sc = pol.exact_score(q, p, qsmem);
          if (lane == r) rank = rank_from_score(pol.metric, sc);
        }
      } else if (valid) {
        rank = pol.fast_rank(q, idx, pos, qsmem);
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

// Launches the scan for `count` query slots with the smallest per-warp list
// capacity that holds KP keys plus a step of appends.  cudaErrorInvalidValue:
// KP or the policy's staging does not fit.
template <bool EXACT, typename Policy>
cudaError_t launch_ivf_list_scan(const Policy& pol, int d, const uint64_t* probe_lists,
                                 const int* probe_counts, int nprobe, const int64_t* list_offsets,
                                 const uint32_t* list_rows, const uint32_t* list_keyrank,
                                 const uint32_t* bitmap, const int* query_ids, int count, int kp,
                                 uint64_t* part_keys, int* part_counts, uint64_t* part_sat,
                                 int* q_flags, cudaStream_t s) {
  int capw = 128;
  while (capw < kp + 64) capw <<= 1;
  const size_t smem = (size_t)kIvfWarps * capw * 8 + (size_t)pol.smem_bytes(d);
  if (capw > 1024 || smem > 220 * 1024) return cudaErrorInvalidValue;
  if (count <= 0) return cudaSuccess;
#define XVEC_IVF_CASE(C)                                                                     \
  if (capw == C) {                                                                           \
    auto kern = ivf_list_scan_kernel<C, EXACT, Policy>;                                      \
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);      \
    kern<<<count, kIvfWarps * 32, smem, s>>>(pol, probe_lists, probe_counts, nprobe,         \
                                             list_offsets, list_rows, list_keyrank, bitmap,  \
                                             query_ids, kp, part_keys, part_counts, part_sat, \
                                             q_flags);                                       \
    return cudaGetLastError();                                                               \
  }
  XVEC_IVF_CASE(128)
  XVEC_IVF_CASE(256)
  XVEC_IVF_CASE(512)
  XVEC_IVF_CASE(1024)
#undef XVEC_IVF_CASE
  return cudaErrorInvalidValue;
}

}  // namespace xvec
