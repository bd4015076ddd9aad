// fht.cuh — block-wide FHT rotation (FHTRotator) of one vector.
//
// FHTRotator.Rotate (internal/core/rotation.go:123-153) and Unrotate
// (rotation.go:155-185) over the FHT primitives of internal/ailego/math/fht.go
// (FHTFlipSigns 28-39, FHTInPlace 41-57, FHTKacWalk 59-76, FHTInverseKacWalk
// 78-94, ScaleFloat32 97-101).  Every operation is a float32 add, subtract or
// multiply rounded to nearest, as the reference evaluates them, so the result
// is bit-identical to it.  The vector lives in memory the whole block reads
// and writes (shared, or the block's own row of global memory); every pass is
// followed by __syncthreads.  signs: 4 rounds of (dim + 7) / 8 bytes, bit i of
// a round's bytes (LSB first) negates element i.
#pragma once

#include "common.cuh"

namespace xvec {

// FHTInPlace on data[0, n), n a power of two.
__device__ inline void block_fht(float* data, int n) {
  for (int w = 1; w < n; w <<= 1) {
    for (int t = threadIdx.x; t < n / 2; t += blockDim.x) {
      const int idx = (t / w) * 2 * w + (t % w);
      const float l = data[idx], r = data[idx + w];
      data[idx] = __fadd_rn(l, r);
      data[idx + w] = __fsub_rn(l, r);
    }
    __syncthreads();
  }
}

__device__ inline void block_fht_flip(float* v, int n, const uint8_t* sg) {
  for (int i = threadIdx.x; i < n; i += blockDim.x)
    if (sg[i >> 3] & (1u << (i & 7))) v[i] = -v[i];
  __syncthreads();
}

__device__ inline void block_fht_scale(float* w, int n, float f) {
  for (int i = threadIdx.x; i < n; i += blockDim.x) w[i] = __fmul_rn(w[i], f);
  __syncthreads();
}

// FHTKacWalk: pairs (i, i + half + n mod 2); an odd length's middle element
// is multiplied by float32(sqrt 2).
__device__ inline void block_fht_kac(float* v, int n) {
  const int half = n / 2, off = half + (n & 1);
  for (int t = threadIdx.x; t < half; t += blockDim.x) {
    const float l = v[t], r = v[t + off];
    v[t] = __fadd_rn(l, r);
    v[t + off] = __fsub_rn(l, r);
  }
  if ((n & 1) && threadIdx.x == 0) v[half] = __fmul_rn(v[half], (float)1.4142135623730951);
  __syncthreads();
}

// FHTInverseKacWalk: the middle element times float32(sqrt 0.5) first, then
// each pair to ((l + r) 0.5, (l - r) 0.5).
__device__ inline void block_fht_inverse_kac(float* v, int n) {
  const int half = n / 2, off = half + (n & 1);
  if ((n & 1) && threadIdx.x == 0) v[half] = __fmul_rn(v[half], (float)0.7071067811865476);
  __syncthreads();
  for (int t = threadIdx.x; t < half; t += blockDim.x) {
    const float l = v[t], r = v[t + off];
    v[t] = __fmul_rn(__fadd_rn(l, r), 0.5f);
    v[t + off] = __fmul_rn(__fsub_rn(l, r), 0.5f);
  }
  __syncthreads();
}

// FHTRotator.Rotate of v[0, dim); truncated = the largest power of two <= dim,
// inv = float32(1 / sqrt(float32(truncated))).
__device__ inline void block_fht_rotate(float* v, int dim, int truncated, const uint8_t* signs,
                                        float inv) {
  const int bpr = (dim + 7) / 8;
  if (truncated == dim) {
    for (int r = 0; r < 4; ++r) {
      block_fht_flip(v, dim, signs + r * bpr);
      block_fht(v, dim);
      block_fht_scale(v, dim, inv);
    }
    return;
  }
  const int start = dim - truncated;
  for (int r = 0; r < 4; ++r) {
    block_fht_flip(v, dim, signs + r * bpr);
    float* window = (r % 2 != 0) ? v + start : v;
    block_fht(window, truncated);
    block_fht_scale(window, truncated, inv);
    block_fht_kac(v, dim);
  }
  block_fht_scale(v, dim, 0.25f);
}

// FHTRotator.Unrotate of v[0, dim): Rotate's rounds undone in reverse order.
__device__ inline void block_fht_unrotate(float* v, int dim, int truncated, const uint8_t* signs,
                                          float inv) {
  const int bpr = (dim + 7) / 8;
  if (truncated == dim) {
    for (int r = 3; r >= 0; --r) {
      block_fht(v, dim);
      block_fht_scale(v, dim, inv);
      block_fht_flip(v, dim, signs + r * bpr);
    }
    return;
  }
  block_fht_scale(v, dim, 4.0f);
  const int start = dim - truncated;
  for (int r = 3; r >= 0; --r) {
    block_fht_inverse_kac(v, dim);
    float* window = (r % 2 != 0) ? v + start : v;
    block_fht(window, truncated);
    block_fht_scale(window, truncated, inv);
    block_fht_flip(v, dim, signs + r * bpr);
  }
}

}  // namespace xvec
