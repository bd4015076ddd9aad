// select.cuh — candidate accumulation and selection primitives.
//
// Every scan kernel ranks (query, row) pairs by a packed 64-bit key:
//   high 32 bits: the rank value (lower = better) as an order-preserving
//                 uint32 (float_to_ordered);
//   low 32 bits : the row's key-rank, i.e. the position of its uint64 key in
//                 ascending key order.
// Packed keys are unique per query, and their unsigned order is exactly the
// reference's resultBetter order (score by metric, ties by ascending key;
// internal/core/topk.go:271-276) whenever the rank value is the reference
// score.  Each (query, part) keeps the KP smallest keys it has seen in a
// shared-memory buffer of CAP entries (CAP >= KP + 2 * appends per round).
#pragma once

#include "common.cuh"

namespace xvec {

// Bitonic sort of N (power of two) uint64 keys in shared memory by one warp.
template <int N>
__device__ __forceinline__ void warp_sort_u64(uint64_t* a) {
  const int lane = threadIdx.x & 31;
#pragma unroll 1
  for (int k = 2; k <= N; k <<= 1) {
#pragma unroll 1
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = lane; i < N; i += 32) {
        const int ixj = i ^ j;
        if (ixj > i) {
          const uint64_t x = a[i], y = a[ixj];
          const bool up = (i & k) == 0;
          if ((x > y) == up) {
            a[i] = y;
            a[ixj] = x;
          }
        }
      }
      __syncwarp();
    }
  }
}

// Bitonic sort of n <= N keys by the whole block (pads with kEmptyKey).
template <int N>
__device__ __forceinline__ void block_sort_u64(uint64_t* a, int n) {
  for (int i = n + threadIdx.x; i < N; i += blockDim.x) a[i] = kEmptyKey;
  __syncthreads();
#pragma unroll 1
  for (int k = 2; k <= N; k <<= 1) {
#pragma unroll 1
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = threadIdx.x; i < N; i += blockDim.x) {
        const int ixj = i ^ j;
        if (ixj > i) {
          const uint64_t x = a[i], y = a[ixj];
          const bool up = (i & k) == 0;
          if ((x > y) == up) {
            a[i] = y;
            a[ixj] = x;
          }
        }
      }
      __syncthreads();
    }
  }
}

// Per-query accumulator state in shared memory.
struct AccumState {
  int count;       // entries in buf
  int saturated;   // set once an entry was dropped
  uint64_t thr;    // an entry is appended only if key < thr
};

// Compact one query's buffer to its KP best keys (one warp).
template <int CAP>
__device__ __forceinline__ void warp_compact(uint64_t* buf, AccumState* st, int kp) {
  const int lane = threadIdx.x & 31;
  const int cnt = st->count;
  for (int i = cnt + lane; i < CAP; i += 32) buf[i] = kEmptyKey;
  __syncwarp();
  warp_sort_u64<CAP>(buf);
  if (lane == 0) {
    if (cnt >= kp) {
      st->thr = buf[kp - 1];
      if (cnt > kp) st->saturated = 1;
      st->count = kp;
    }
  }
  __syncwarp();
}

// block_sort_u64 over the smallest power of two >= n (at least 64, at most N).
template <int N>
__device__ __forceinline__ void block_sort_u64_fit(uint64_t* a, int n) {
  if (N >= 64 && n <= 64) return block_sort_u64<(N < 64 ? N : 64)>(a, n);
  if (N >= 256 && n <= 256) return block_sort_u64<(N < 256 ? N : 256)>(a, n);
  if (N >= 1024 && n <= 1024) return block_sort_u64<(N < 1024 ? N : 1024)>(a, n);
  block_sort_u64<N>(a, n);
}

}  // namespace xvec
