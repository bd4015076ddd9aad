// flat_kernels.cu — Flat exact search kernels (CUDA cores).
//
// Reference path: DenseFlatIndex.search (internal/core/flat.go:179-196) →
// topKPrevalidatedCandidatesWithOptions (internal/core/topk.go:105-166) with
// metric.Compute (internal/core/metric/metric.go:35-48).
//
// Pipeline per batch of queries:
//   1. prep_queries: decode queries to float32, reference-order ||q||^2 and
//      the query validation of topk.go:92-94 (metric.Compute(q, q) finite).
//   2. scan (fast):  FFMA tiles of 64 rows x 32 queries; the rank of each
//      pair goes into a per-(query, part) accumulator of the KP best packed
//      keys (select.cuh).  Filter before scoring (topk.go:134-136).
//   3. merge_rescore: per query, the kth best fast key over all parts, the
//      candidate set {rank <= F_k + 2*eps} (eps bounds |fast - reference|),
//      reference-order rescoring of the candidates, final (score, key) sort,
//      radius (query.go:193-201) and top-k.
//   4. scan (exact) + merge in exact mode for the rare query whose candidate
//      set cannot be proven complete, and for large k.
#include "flat_kernels.cuh"
#include "select.cuh"

namespace xvec {

// ---------------------------------------------------------------------------
// Query preparation.
// ---------------------------------------------------------------------------
template <typename QT>
__global__ void prep_queries_kernel(const QT* __restrict__ q_in, int nq, int d, int metric,
                                    float* __restrict__ qf, float* __restrict__ q_n2,
                                    float* __restrict__ q_aux, int* __restrict__ q_status) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= nq) return;
  const QT* src = q_in + (int64_t)warp * d;
  float* dst = qf + (int64_t)warp * d;
  bool finite = true;
  for (int i = lane; i < d; i += 32) {
    const float v = load_elem(src, i);
    dst[i] = v;
    finite &= finite_f(v);
  }
  finite = __all_sync(kFullMask, finite);
  __syncwarp();
  float s0, s1, s2;
  warp_reference_sums<1>(dst, dst, d, &s0, &s1, &s2);  // InnerProduct(q, q)
  if (lane == 0) {
    q_n2[warp] = s0;
    // Tensor-core epilogue operand: 1/||q|| for cosine, ||q||^2 otherwise.
    q_aux[warp] = metric == kMetricCosine ? (s0 > 0.f ? rsqrtf(s0) : 0.f) : s0;
    // metric.Compute(q, q): L2 is always 0 for finite input; IP, cosine and
    // MIPS become non-finite exactly when ||q||^2 overflows.
    int st = 0;
    if (!finite) st = 7;
    else if (metric != kMetricL2 && !finite_f(s0)) st = 7;
    q_status[warp] = st;
  }
}

// Reference-order ||x||^2 of stored rows (InnerProduct(x, x)); used by the
// fast L2 / cosine / MIPS ranks and the error bounds.
template <typename RowT>
__global__ void row_norms_kernel(const RowT* __restrict__ rows, int64_t n, int d,
                                 float* __restrict__ n2, float* __restrict__ inv_mag,
                                 unsigned* __restrict__ max_n2_ordered,
                                 int* __restrict__ nonfinite) {
  const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= n) return;
  const RowT* x = rows + warp * d;
  bool finite = true;
  for (int i = lane; i < d; i += 32) finite &= finite_f(load_elem(x, i));
  finite = __all_sync(kFullMask, finite);
  float s0 = 0.f;
  if (finite) {
    // InnerProduct(x, x) in the reference order (fp16 rows decode exactly).
    float a0 = 0.f, r0 = 0.f;
    if (d >= 16) {
      if (lane < 16)
        for (int v = 0; v < (d >> 4); ++v) {
          const float xv = load_elem(x, v * 16 + lane);
          a0 = __fmaf_rn(xv, xv, a0);
        }
      for (int j = 0; j < 16; ++j) r0 = __fadd_rn(r0, __shfl_sync(kFullMask, a0, j));
      for (int i = (d >> 4) * 16; i < d; ++i) {
        const float xv = load_elem(x, i);
        r0 = __fmaf_rn(xv, xv, r0);
      }
    } else if (d >= 8) {
      if (lane < 8) {
        const float xv = load_elem(x, lane);
        a0 = __fadd_rn(0.f, __fmul_rn(xv, xv));
      }
      for (int j = 0; j < 8; ++j) r0 = __fadd_rn(r0, __shfl_sync(kFullMask, a0, j));
      for (int i = 8; i < d; ++i) {
        const float xv = load_elem(x, i);
        r0 = __fadd_rn(r0, __fmul_rn(xv, xv));
      }
    } else {
      for (int i = 0; i < d; ++i) {
        const float xv = load_elem(x, i);
        r0 = __fadd_rn(r0, __fmul_rn(xv, xv));
      }
    }
    s0 = r0;
  }
  if (lane == 0) {
    n2[warp] = s0;
    inv_mag[warp] = s0 > 0.f ? rsqrtf(s0) : 0.f;
    if (!finite) atomicExch(nonfinite, 1);
    else if (finite_f(s0)) atomicMax(max_n2_ordered, float_to_ordered(s0));
    else atomicMax(max_n2_ordered, float_to_ordered(3.0e38f));
  }
}

// Fast rank of a (row, query) pair from its dot product and the exact
// squared norms (see fast_eps for the bound on |fast - reference|).
__device__ __forceinline__ float fast_rank(int metric, float dot, float xn2, float qn2) {
  switch (metric) {
    case kMetricL2: return (xn2 + qn2) - 2.f * dot;
    case kMetricIP: return -dot;
    case kMetricCosine:
      if (xn2 == 0.f && qn2 == 0.f) return 0.f;
      if (xn2 == 0.f || qn2 == 0.f) return 1.f;
      return 1.f - dot * rsqrtf(xn2) * rsqrtf(qn2);
    default: {
      const float den = fmaxf(xn2, qn2);
      if (den == 0.f) return 0.f;
      return 2.f - 2.f * dot / den;
    }
  }
}

// Bound on |fast rank - reference rank| for a query (both accumulate d
// exact-or-rounded products in float32; factor 4 covers both sides and a
// non round-to-nearest accumulator).
__device__ __forceinline__ float fast_eps(int metric, int d, float qn2, float max_xn2) {
  const float u = 5.9604645e-8f;  // 2^-24
  const float g = 4.f * (float)(d + 8) * u;
  const float qn = sqrtf(qn2), xn = sqrtf(max_xn2);
  switch (metric) {
    case kMetricL2: return g * (xn + qn) * (xn + qn) * 1.0001f;
    case kMetricIP: return g * xn * qn * 1.0001f + 1e-30f;
    case kMetricCosine: return g * 2.f;
    default: return g * 4.f;
  }
}

// ---------------------------------------------------------------------------
// Fast FFMA scan: block = 256 threads, tile = 64 rows x 32 queries, k-step 32.
// Thread (ty, tx) owns rows ty*4..ty*4+3 and queries tx*2, tx*2+1.
// ---------------------------------------------------------------------------
constexpr int kSimtQT = 32;
constexpr int kSimtRT = 64;
constexpr int kSimtKT = 32;

template <typename RowT, int CAP>
__global__ void __launch_bounds__(256) flat_scan_simt_kernel(
    const RowT* __restrict__ rows, int64_t n, int d, const float* __restrict__ row_n2,
    const uint32_t* __restrict__ keyrank, const float* __restrict__ qf,
    const float* __restrict__ q_n2, int nq, const uint32_t* __restrict__ bitmap, int metric,
    int64_t rows_per_part, int kp, uint64_t* __restrict__ part_keys,
    int* __restrict__ part_counts, uint64_t* __restrict__ part_sat, int* __restrict__ q_flags) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  uint64_t* buf = reinterpret_cast<uint64_t*>(smem_raw);                       // [QT][CAP]
  float* xs = reinterpret_cast<float*>(buf + kSimtQT * CAP);                    // [KT][RT+4]
  float* qs = xs + kSimtKT * (kSimtRT + 4);                                     // [KT][QT+4]
  __shared__ AccumState st[kSimtQT];

  const int tid = threadIdx.x;
  const int tx = tid & 15, ty = tid >> 4;
  const int q0 = blockIdx.x * kSimtQT;
  const int part = blockIdx.y;
  const int num_parts = gridDim.y;
  const int64_t row_begin = (int64_t)part * rows_per_part;
  const int64_t row_end = min(n, row_begin + rows_per_part);

  if (tid < kSimtQT) {
    st[tid].count = 0;
    st[tid].saturated = 0;
    st[tid].thr = kEmptyKey;
  }
  float qn2_reg[2];
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    const int qi = q0 + tx * 2 + j;
    qn2_reg[j] = qi < nq ? q_n2[qi] : 0.f;
  }
  __syncthreads();

  for (int64_t tile = row_begin; tile < row_end; tile += kSimtRT) {
    float acc[4][2];
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[i][0] = acc[i][1] = 0.f;
    for (int k0 = 0; k0 < d; k0 += kSimtKT) {
      __syncthreads();
      for (int e = tid; e < kSimtRT * kSimtKT; e += 256) {
        const int r = e / kSimtKT, kk = e % kSimtKT;
        const int64_t row = tile + r;
        const int k = k0 + kk;
        xs[kk * (kSimtRT + 4) + r] = (row < row_end && k < d) ? load_elem(rows, row * d + k) : 0.f;
      }
      for (int e = tid; e < kSimtQT * kSimtKT; e += 256) {
        const int qq = e / kSimtKT, kk = e % kSimtKT;
        const int qi = q0 + qq;
        const int k = k0 + kk;
        qs[kk * (kSimtQT + 4) + qq] = (qi < nq && k < d) ? qf[(int64_t)qi * d + k] : 0.f;
      }
      __syncthreads();
#pragma unroll 8
      for (int kk = 0; kk < kSimtKT; ++kk) {
        const float4 a = *reinterpret_cast<const float4*>(&xs[kk * (kSimtRT + 4) + ty * 4]);
        const float2 b = *reinterpret_cast<const float2*>(&qs[kk * (kSimtQT + 4) + tx * 2]);
        acc[0][0] = fmaf(a.x, b.x, acc[0][0]);
        acc[0][1] = fmaf(a.x, b.y, acc[0][1]);
        acc[1][0] = fmaf(a.y, b.x, acc[1][0]);
        acc[1][1] = fmaf(a.y, b.y, acc[1][1]);
        acc[2][0] = fmaf(a.z, b.x, acc[2][0]);
        acc[2][1] = fmaf(a.z, b.y, acc[2][1]);
        acc[3][0] = fmaf(a.w, b.x, acc[3][0]);
        acc[3][1] = fmaf(a.w, b.y, acc[3][1]);
      }
    }
    // Epilogue: rank, filter, append.
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int64_t row = tile + ty * 4 + i;
      if (row >= row_end || !bitmap_pass(bitmap, row)) continue;
      const float xn2 = row_n2[row];
      const uint32_t kr = keyrank[row];
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int ql = tx * 2 + j;
        const int qi = q0 + ql;
        if (qi >= nq) continue;
        const float r = fast_rank(metric, acc[i][j], xn2, qn2_reg[j]);
        if (!finite_f(r)) {
          atomicOr(&q_flags[qi], 1);
          continue;
        }
        const uint64_t key = pack_rank(r, kr);
        if (key < st[ql].thr) {
          const int slot = atomicAdd(&st[ql].count, 1);
          buf[ql * CAP + slot] = key;
        }
      }
    }
    __syncthreads();
    // Keep room for one more tile of appends per query.
    const int warp = tid >> 5;
    for (int ql = warp; ql < kSimtQT; ql += 8)
      if (st[ql].count > CAP - kSimtRT) warp_compact<CAP>(buf + ql * CAP, &st[ql], kp);
    __syncthreads();
  }
  // Final compaction and write-out of this part's sorted list.
  const int warp = tid >> 5, lane = tid & 31;
  for (int ql = warp; ql < kSimtQT; ql += 8) {
    const int qi = q0 + ql;
    if (qi >= nq) continue;
    warp_compact<CAP>(buf + ql * CAP, &st[ql], kp);
    // warp_compact only trims when count >= kp; sort happened regardless.
    const int cnt = min(st[ql].count, kp);
    const int64_t base = ((int64_t)qi * num_parts + part) * kp;
    for (int i = lane; i < cnt; i += 32) part_keys[base + i] = buf[ql * CAP + i];
    if (lane == 0) {
      part_counts[(int64_t)qi * num_parts + part] = cnt;
      part_sat[(int64_t)qi * num_parts + part] = st[ql].thr;
    }
  }
}

// ---------------------------------------------------------------------------
// Exact scan: reference-order scores for one query per block (8 warps, each
// scoring rows in turn).  Used when the fast candidate set cannot be proven
// complete, and for top-k beyond the fast scan's capacity.
// ---------------------------------------------------------------------------
template <typename RowT, int CAP>
__global__ void __launch_bounds__(256) flat_scan_exact_kernel(
    const RowT* __restrict__ rows, int64_t n, int d, const uint32_t* __restrict__ keyrank,
    const float* __restrict__ qf, const int* __restrict__ query_ids,
    const uint32_t* __restrict__ bitmap, int metric, int64_t rows_per_part, int kp,
    uint64_t* __restrict__ part_keys, int* __restrict__ part_counts,
    uint64_t* __restrict__ part_sat, int* __restrict__ q_flags) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  uint64_t* buf = reinterpret_cast<uint64_t*>(smem_raw);
  __shared__ AccumState st;
  constexpr int kRowsPerRound = 8 * 16;
  const int qi = query_ids[blockIdx.x];
  const int slot_q = blockIdx.x;  // part buffers are indexed by list slot
  const int part = blockIdx.y, num_parts = gridDim.y;
  const int64_t row_begin = (int64_t)part * rows_per_part;
  const int64_t row_end = min(n, row_begin + rows_per_part);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const float* q = qf + (int64_t)qi * d;
  if (threadIdx.x == 0) {
    st.count = 0;
    st.saturated = 0;
    st.thr = kEmptyKey;
  }
  __syncthreads();
  for (int64_t round = row_begin; round < row_end; round += kRowsPerRound) {
    for (int j = 0; j < 16; ++j) {
      const int64_t row = round + j * 8 + warp;
      if (row >= row_end || !bitmap_pass(bitmap, row)) continue;
      const float s = warp_reference_score(metric, rows + row * d, q, d);
      if (lane == 0) {
        if (!finite_f(s)) {
          atomicOr(&q_flags[qi], 4);
        } else {
          const uint64_t key = pack_rank(rank_from_score(metric, s), keyrank[row]);
          if (key < st.thr) {
            const int slot = atomicAdd(&st.count, 1);
            buf[slot] = key;
          }
        }
      }
    }
    __syncthreads();
    if (warp == 0 && st.count > CAP - kRowsPerRound) warp_compact<CAP>(buf, &st, kp);
    __syncthreads();
  }
  if (warp == 0) {
    warp_compact<CAP>(buf, &st, kp);
    const int cnt = min(st.count, kp);
    const int64_t base = ((int64_t)slot_q * num_parts + part) * kp;
    for (int i = lane; i < cnt; i += 32) part_keys[base + i] = buf[i];
    if (lane == 0) {
      part_counts[(int64_t)slot_q * num_parts + part] = cnt;
      part_sat[(int64_t)slot_q * num_parts + part] = st.thr;
    }
  }
}

// ---------------------------------------------------------------------------
// Merge + reference rescoring.  One block (256 threads) per query.
// exact_mode: the part keys already hold reference ranks; the candidates are
// exactly the k best keys.
// ---------------------------------------------------------------------------
constexpr int kMaxCandidates = 1024;
constexpr int kMergeSmemEntries = 12288;  // union entries gathered in shared memory

// Radix select over keys[0, m) in shared memory: the kth smallest (1-based)
// considering bits [low_bit, 64) only; returns those high bits (low bits 0).
__device__ uint64_t smem_radix_select(const uint64_t* keys, int m, int kth, int low_bit,
                                      int* hist) {
  __shared__ uint64_t s_prefix;
  __shared__ int s_kth;
  if (threadIdx.x == 0) {
    s_prefix = 0;
    s_kth = kth;
  }
  __syncthreads();
#pragma unroll 1
  for (int shift = 56; shift >= low_bit; shift -= 8) {
    for (int i = threadIdx.x; i < 256; i += blockDim.x) hist[i] = 0;
    __syncthreads();
    const uint64_t prefix = s_prefix;
    const uint64_t mask = (shift == 56) ? 0ull : (~0ull << (shift + 8));
    for (int i = threadIdx.x; i < m; i += blockDim.x) {
      const uint64_t key = keys[i];
      if ((key & mask) == prefix) atomicAdd(&hist[(key >> shift) & 0xff], 1);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      int remaining = s_kth, digit = 0;
      for (; digit < 255; ++digit) {
        if (remaining <= hist[digit]) break;
        remaining -= hist[digit];
      }
      s_kth = remaining;
      s_prefix = prefix | ((uint64_t)digit << shift);
    }
    __syncthreads();
  }
  return s_prefix;
}

template <typename RowT>
__global__ void __launch_bounds__(256) flat_merge_rescore_kernel(
    const RowT* __restrict__ rows, int d, const uint32_t* __restrict__ pos_of_keyrank,
    const uint64_t* __restrict__ keys, const float* __restrict__ qf,
    const float* __restrict__ q_n2, const unsigned* __restrict__ max_n2_ordered,
    const int* __restrict__ query_ids, int metric, int k, float radius, int exact_mode,
    const uint64_t* __restrict__ part_keys, const int* __restrict__ part_counts,
    const uint64_t* __restrict__ part_sat, int num_parts, int stride,
    uint64_t* __restrict__ out_keys, float* __restrict__ out_scores, int* __restrict__ out_counts,
    int* __restrict__ q_flags) {
  extern __shared__ __align__(16) unsigned char merge_smem[];
  uint64_t* ukeys = reinterpret_cast<uint64_t*>(merge_smem);  // [kMergeSmemEntries]
  __shared__ int hist[256];
  __shared__ uint64_t cand[kMaxCandidates];
  __shared__ int s_offsets[1025];
  __shared__ int s_ncand, s_fail;
  const int slot_q = blockIdx.x;
  const int qi = query_ids ? query_ids[blockIdx.x] : blockIdx.x;
  const int64_t pbase = (int64_t)slot_q * num_parts;

  // Prefix sums of the list counts (num_parts <= 1024).
  if (threadIdx.x == 0) {
    int total = 0;
    for (int p = 0; p < num_parts; ++p) {
      s_offsets[p] = total;
      total += part_counts[pbase + p];
    }
    s_offsets[num_parts] = total;
    s_ncand = 0;
    s_fail = 0;
  }
  __syncthreads();
  const int total = s_offsets[num_parts];
  if (total == 0) {
    if (threadIdx.x == 0) out_counts[qi] = 0;
    return;
  }
  if (total > kMergeSmemEntries) {
    // Cannot happen with the list sizes the scans produce; route to the
    // exact path rather than read past the shared buffer.
    if (threadIdx.x == 0) {
      atomicOr(&q_flags[qi], 2);
      out_counts[qi] = 0;
    }
    return;
  }
  // Gather the union (one warp per list).
  {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int p = warp; p < num_parts; p += blockDim.x >> 5) {
      const int off = s_offsets[p], c = s_offsets[p + 1] - off;
      const uint64_t* src = part_keys + (pbase + p) * stride;
      for (int j = lane; j < c; j += 32) ukeys[off + j] = src[j];
    }
  }
  __syncthreads();
  const int kth = min(k, total);
  uint64_t limit;
  if (exact_mode) {
    limit = smem_radix_select(ukeys, total, kth, 0, hist);
  } else {
    const uint64_t kr = smem_radix_select(ukeys, total, kth, 32, hist);
    const float eps = fast_eps(metric, d, q_n2[qi], ordered_to_float(*max_n2_ordered));
    const float t = __fadd_ru(rank_of(kr), 2.f * eps);
    limit = ((uint64_t)float_to_ordered(t) << 32) | 0xffffffffull;
    // Coverage: a list dropped only keys above its saturation key.
    for (int p = threadIdx.x; p < num_parts; p += blockDim.x) {
      const uint64_t sat = part_sat[pbase + p];
      if (sat != kEmptyKey && sat <= limit) atomicExch(&s_fail, 1);
    }
  }
  for (int i = threadIdx.x; i < total; i += blockDim.x) {
    const uint64_t key = ukeys[i];
    if (key <= limit) {
      const int slot = atomicAdd(&s_ncand, 1);
      if (slot < kMaxCandidates) cand[slot] = key;
    }
  }
  __syncthreads();
  if (s_fail || s_ncand > kMaxCandidates) {
    if (threadIdx.x == 0) {
      atomicOr(&q_flags[qi], 2);
      out_counts[qi] = 0;
    }
    return;
  }
  const int ncand = s_ncand;
  // Reference rescoring: one warp per candidate.
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const float* q = qf + (int64_t)qi * d;
  for (int c = warp; c < ncand; c += blockDim.x >> 5) {
    const uint32_t kr = pos_of(cand[c]);
    const uint32_t pos = pos_of_keyrank[kr];
    const float s = warp_reference_score(metric, rows + (int64_t)pos * d, q, d);
    if (lane == 0) {
      if (!finite_f(s)) atomicOr(&q_flags[qi], 4);
      cand[c] = pack_rank(rank_from_score(metric, s), kr);
    }
  }
  __syncthreads();
  block_sort_u64<kMaxCandidates>(cand, ncand);
  // Final top-k (radius is monotone in the sorted order).
  if (threadIdx.x < 32) {
    // Count the prefix within radius with a warp scan over chunks.
    int count = 0;
    for (int base = 0; base < ncand && count < k; base += 32) {
      const int i = base + lane;
      bool in = i < ncand;
      float s = 0.f;
      if (in) {
        s = score_from_rank(metric, rank_of(cand[i]));
        in = within_radius(metric, s, radius);
      }
      const unsigned m = __ballot_sync(kFullMask, in);
      const int run = (m == kFullMask) ? 32 : __ffs(~m) - 1;  // leading in-radius run
      if (lane < run && count + lane < k) {
        const uint32_t pos = pos_of_keyrank[pos_of(cand[i])];
        out_keys[(int64_t)qi * k + count + lane] = keys[pos];
        out_scores[(int64_t)qi * k + count + lane] = s;
      }
      count = min(k, count + run);
      if (run < 32) break;
    }
    if (lane == 0) out_counts[qi] = count;
  }
}

// ---------------------------------------------------------------------------
// Host launchers.
// ---------------------------------------------------------------------------
template <typename QT>
void launch_prep_queries(const QT* q, int nq, int d, int metric, float* qf, float* q_n2,
                         float* q_aux, int* q_status, cudaStream_t stream) {
  const int warps_per_block = 8;
  const int blocks = (nq + warps_per_block - 1) / warps_per_block;
  if (blocks > 0)
    prep_queries_kernel<QT><<<blocks, warps_per_block * 32, 0, stream>>>(q, nq, d, metric, qf,
                                                                         q_n2, q_aux, q_status);
}
template void launch_prep_queries<float>(const float*, int, int, int, float*, float*, float*,
                                         int*, cudaStream_t);
template void launch_prep_queries<__half>(const __half*, int, int, int, float*, float*, float*,
                                          int*, cudaStream_t);

template <typename RowT>
void launch_row_norms(const RowT* rows, int64_t n, int d, float* n2, float* inv_mag,
                      unsigned* max_n2, int* nonfinite, cudaStream_t stream) {
  const int64_t blocks = (n + 7) / 8;
  if (blocks > 0)
    row_norms_kernel<RowT><<<(unsigned)blocks, 256, 0, stream>>>(rows, n, d, n2, inv_mag, max_n2,
                                                                 nonfinite);
}
template void launch_row_norms<float>(const float*, int64_t, int, float*, float*, unsigned*,
                                      int*, cudaStream_t);
template void launch_row_norms<__half>(const __half*, int64_t, int, float*, float*, unsigned*,
                                       int*, cudaStream_t);

int flat_merge_capacity() { return kMergeSmemEntries; }

int simt_cap_for(int kp) {
  // CAP must hold KP retained entries plus two tiles of appends.
  int need = kp + 2 * kSimtRT;
  int cap = 256;
  while (cap < need) cap <<= 1;
  return cap;
}

template <typename RowT>
cudaError_t launch_flat_scan_simt(const RowT* rows, int64_t n, int d, const float* row_n2,
                                  const uint32_t* keyrank, const float* qf, const float* q_n2,
                                  int nq, const uint32_t* bitmap, int metric, int num_parts,
                                  int kp, uint64_t* part_keys, int* part_counts,
                                  uint64_t* part_sat, int* q_flags, cudaStream_t stream) {
  const int cap = simt_cap_for(kp);
  const int64_t rows_per_part = ((n + num_parts - 1) / num_parts + kSimtRT - 1) / kSimtRT * kSimtRT;
  dim3 grid((nq + kSimtQT - 1) / kSimtQT, num_parts);
  const size_t tiles = (size_t)(kSimtKT * (kSimtRT + 4) + kSimtKT * (kSimtQT + 4)) * sizeof(float);
  if (cap == 256) {
    const size_t smem = (size_t)kSimtQT * 256 * 8 + tiles;
    auto kern = flat_scan_simt_kernel<RowT, 256>;
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    kern<<<grid, 256, smem, stream>>>(rows, n, d, row_n2, keyrank, qf, q_n2, nq, bitmap, metric,
                                      rows_per_part, kp, part_keys, part_counts, part_sat,
                                      q_flags);
  } else if (cap == 512) {
    const size_t smem = (size_t)kSimtQT * 512 * 8 + tiles;
    auto kern = flat_scan_simt_kernel<RowT, 512>;
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    kern<<<grid, 256, smem, stream>>>(rows, n, d, row_n2, keyrank, qf, q_n2, nq, bitmap, metric,
                                      rows_per_part, kp, part_keys, part_counts, part_sat,
                                      q_flags);
  } else {
    return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}
template cudaError_t launch_flat_scan_simt<float>(const float*, int64_t, int, const float*,
                                                  const uint32_t*, const float*, const float*, int,
                                                  const uint32_t*, int, int, int, uint64_t*, int*,
                                                  uint64_t*, int*, cudaStream_t);
template cudaError_t launch_flat_scan_simt<__half>(const __half*, int64_t, int, const float*,
                                                   const uint32_t*, const float*, const float*,
                                                   int, const uint32_t*, int, int, int, uint64_t*,
                                                   int*, uint64_t*, int*, cudaStream_t);

int exact_cap_for(int kp) {
  int need = kp + 2 * 128;
  int cap = 512;
  while (cap < need) cap <<= 1;
  return cap;
}

template <typename RowT>
cudaError_t launch_flat_scan_exact(const RowT* rows, int64_t n, int d, const uint32_t* keyrank,
                                   const float* qf, const int* query_ids, int nlist,
                                   const uint32_t* bitmap, int metric, int num_parts, int kp,
                                   uint64_t* part_keys, int* part_counts, uint64_t* part_sat,
                                   int* q_flags, cudaStream_t stream) {
  const int cap = exact_cap_for(kp);
  const int64_t rows_per_part = (n + num_parts - 1) / num_parts;
  dim3 grid(nlist, num_parts);
  const size_t smem = (size_t)cap * 8;
#define XVEC_EXACT_CASE(C)                                                                     \
  if (cap == C) {                                                                              \
    auto kern = flat_scan_exact_kernel<RowT, C>;                                               \
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);        \
    kern<<<grid, 256, smem, stream>>>(rows, n, d, keyrank, qf, query_ids, bitmap, metric,      \
                                      rows_per_part, kp, part_keys, part_counts, part_sat,     \
                                      q_flags);                                                \
    return cudaGetLastError();                                                                 \
  }
  XVEC_EXACT_CASE(512)
  XVEC_EXACT_CASE(1024)
  XVEC_EXACT_CASE(2048)
  XVEC_EXACT_CASE(4096)
  XVEC_EXACT_CASE(8192)
#undef XVEC_EXACT_CASE
  return cudaErrorInvalidValue;
}
template cudaError_t launch_flat_scan_exact<float>(const float*, int64_t, int, const uint32_t*,
                                                   const float*, const int*, int, const uint32_t*,
                                                   int, int, int, uint64_t*, int*, uint64_t*,
                                                   int*, cudaStream_t);
template cudaError_t launch_flat_scan_exact<__half>(const __half*, int64_t, int, const uint32_t*,
                                                    const float*, const int*, int,
                                                    const uint32_t*, int, int, int, uint64_t*,
                                                    int*, uint64_t*, int*, cudaStream_t);

template <typename RowT>
cudaError_t launch_flat_merge_rescore(const RowT* rows, int d, const uint32_t* pos_of_keyrank,
                                      const uint64_t* keys, const float* qf, const float* q_n2,
                                      const unsigned* max_n2, const int* query_ids, int nlist,
                                      int metric, int k, float radius, int exact_mode,
                                      const uint64_t* part_keys, const int* part_counts,
                                      const uint64_t* part_sat, int num_parts, int stride,
                                      uint64_t* out_keys, float* out_scores, int* out_counts,
                                      int* q_flags, cudaStream_t stream) {
  if (nlist <= 0) return cudaSuccess;
  if (num_parts > 1024) return cudaErrorInvalidValue;
  const int smem = kMergeSmemEntries * 8;
  cudaFuncSetAttribute(flat_merge_rescore_kernel<RowT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                       smem);
  flat_merge_rescore_kernel<RowT><<<nlist, 256, smem, stream>>>(
      rows, d, pos_of_keyrank, keys, qf, q_n2, max_n2, query_ids, metric, k, radius, exact_mode,
      part_keys, part_counts, part_sat, num_parts, stride, out_keys, out_scores, out_counts,
      q_flags);
  return cudaGetLastError();
}
template cudaError_t launch_flat_merge_rescore<float>(const float*, int, const uint32_t*,
                                                      const uint64_t*, const float*, const float*,
                                                      const unsigned*, const int*, int, int, int,
                                                      float, int, const uint64_t*, const int*,
                                                      const uint64_t*, int, int, uint64_t*, float*,
                                                      int*, int*, cudaStream_t);
template cudaError_t launch_flat_merge_rescore<__half>(const __half*, int, const uint32_t*,
                                                       const uint64_t*, const float*,
                                                       const float*, const unsigned*, const int*,
                                                       int, int, int, float, int, const uint64_t*,
                                                       const int*, const uint64_t*, int, int,
                                                       uint64_t*, float*, int*, int*,
                                                       cudaStream_t);

}  // namespace xvec
