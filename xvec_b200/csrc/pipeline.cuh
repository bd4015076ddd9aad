// pipeline.cuh — the candidate pipeline shared by every index kind.
//
//   scan (fast)   : a Ranker turns a dot product into a fast rank; each
//                   (query, row part) keeps its KP best packed keys.
//   scan (exact)  : a Scorer gives the reference score of one (query, row);
//                   the same per-part selection, used when the fast pass
//                   cannot prove its candidate set complete.
//   merge_rescore : per query, the k-th best key over all parts, the
//                   candidates within the Scorer's error bound, their
//                   reference scores, the final (score, key) order, radius
//                   and top-k (optionally the row positions as well).
//
// Ranker:  struct RowInfo; struct QueryInfo;
//          QueryInfo query(int qi); RowInfo row(int64_t row);
//          float rank(float dot, const RowInfo&, const QueryInfo&);
// Scorer:  int metric (ordering and radius rule);
//          float score(int qi, int64_t row)  -- called by a whole warp;
//          bool half_warp()                   -- true: score() evaluates the
//                                                row of each half-warp apart,
//                                                so a warp scores two rows;
//          float eps(int qi)                  -- bound on |fast - reference|;
//          int error_flag(float s)            -- flag bit for a non-finite score;
//          float output(float rank)           -- the reported score of a rank;
//          bool keep(float out, float radius) -- the radius rule on that score.
#pragma once

#include <algorithm>

#include "common.cuh"
#include "select.cuh"

namespace xvec {

// ---------------------------------------------------------------------------
// Fast FFMA scan: block = 256 threads, tile = 64 rows x 32 queries, k-step 32.
// Thread (ty, tx) owns rows ty*4..ty*4+3 and queries tx*2, tx*2+1.
// ---------------------------------------------------------------------------
constexpr int kSimtQT = 32;
constexpr int kSimtRT = 64;
constexpr int kSimtKT = 32;

template <typename RowT, int CAP, typename Ranker>
__global__ void __launch_bounds__(256) scan_simt_kernel(
    const RowT* __restrict__ rows, int64_t n, int d, const uint32_t* __restrict__ keyrank,
    const float* __restrict__ qf, int nq, const uint32_t* __restrict__ bitmap, Ranker rk,
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
  typename Ranker::QueryInfo qinfo[2];
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    const int qi = q0 + tx * 2 + j;
    qinfo[j] = rk.query(qi < nq ? qi : 0);
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
      const typename Ranker::RowInfo rinfo = rk.row(row);
      const uint32_t kr = keyrank[row];
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int ql = tx * 2 + j;
        const int qi = q0 + ql;
        if (qi >= nq) continue;
        const float r = rk.rank(acc[i][j], rinfo, qinfo[j]);
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
template <int CAP, typename Scorer>
__global__ void __launch_bounds__(256) scan_exact_kernel(
    Scorer sc, int64_t n, const uint32_t* __restrict__ keyrank, const int* __restrict__ query_ids,
    const uint32_t* __restrict__ bitmap, int64_t rows_per_part, int kp,
    uint64_t* __restrict__ part_keys, int* __restrict__ part_counts,
    uint64_t* __restrict__ part_sat, int* __restrict__ q_flags) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  uint64_t* buf = reinterpret_cast<uint64_t*>(smem_raw);
  __shared__ AccumState st;
  constexpr int kRowsPerRound = 8 * 16;
  const int qi = query_ids ? query_ids[blockIdx.x] : blockIdx.x;
  const int slot_q = blockIdx.x;  // part buffers are indexed by list slot
  const int part = blockIdx.y, num_parts = gridDim.y;
  const int64_t row_begin = (int64_t)part * rows_per_part;
  const int64_t row_end = min(n, row_begin + rows_per_part);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    st.count = 0;
    st.saturated = 0;
    st.thr = kEmptyKey;
  }
  __syncthreads();
  const bool pairs = sc.half_warp();
  const int half = lane >> 4;
  for (int64_t round = row_begin; round < row_end; round += kRowsPerRound) {
    for (int j = 0; j < (pairs ? 8 : 16); ++j) {
      int64_t row;
      bool ok;
      if (pairs) {
        // Rows row0 and row0 + 1, one per half-warp; a half whose row is
        // out of range or filtered out scores its partner's and drops it.
        const int64_t row0 = round + (int64_t)(j * 8 + warp) * 2;
        row = row0 + half;
        ok = row < row_end && bitmap_pass(bitmap, row);
        if (__ballot_sync(kFullMask, ok) == 0) continue;
        if (!ok) row = half ? row0 : row0 + 1;
      } else {
        row = round + j * 8 + warp;
        ok = row < row_end && bitmap_pass(bitmap, row);
        if (!ok) continue;
      }
      const float s = sc.score(qi, row);
      if ((lane & (pairs ? 15 : 31)) == 0 && ok) {
        if (!finite_f(s)) {
          atomicOr(&q_flags[qi], sc.error_flag(s));
        } else {
          const uint64_t key = pack_rank(rank_from_score(sc.metric, s), keyrank[row]);
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
constexpr int kMaxCandidates = 1024;      // rescored candidates per query (k <= 1024)
constexpr int kMaxCandidatesWide = 2048;  // the same for 1024 < k <= 2048
constexpr int kMergeSmemEntries = 12288;  // union entries gathered in shared memory
constexpr int kMergeFilteredEntries = 4096;  // the same when a threshold filters the union

// Radix select over keys[0, m) in shared memory: the kth smallest (1-based)
// considering bits [low_bit, 64) only; returns those high bits (low bits 0).
// Every thread of the block calls it.  The histogram increments of a warp
// that fall into one bin are combined (__match_any_sync) before the shared
// atomic, and warp 0 finds the bin holding the kth key with a warp scan.
static __device__ uint64_t smem_radix_select(const uint64_t* keys, int m, int kth, int low_bit,
                                             int* hist) {
  __shared__ uint64_t s_prefix;
  __shared__ int s_kth;
  const int lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    s_prefix = 0;
    s_kth = kth;
  }
  __syncthreads();
  const int mpad = (m + 31) & ~31;  // whole warps iterate together
#pragma unroll 1
  for (int shift = 56; shift >= low_bit; shift -= 8) {
    for (int i = threadIdx.x; i < 256; i += blockDim.x) hist[i] = 0;
    __syncthreads();
    const uint64_t prefix = s_prefix;
    const uint64_t mask = (shift == 56) ? 0ull : (~0ull << (shift + 8));
    for (int i = threadIdx.x; i < mpad; i += blockDim.x) {
      int bin = -1;
      if (i < m) {
        const uint64_t key = keys[i];
        if ((key & mask) == prefix) bin = (int)((key >> shift) & 0xff);
      }
      const unsigned peers = __match_any_sync(kFullMask, bin);
      if (bin >= 0 && lane == __ffs(peers) - 1) atomicAdd(&hist[bin], __popc(peers));
    }
    __syncthreads();
    if (threadIdx.x < 32) {
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
      const int want = s_kth;
      const unsigned owner = __ballot_sync(kFullMask, excl < want && want <= incl);
      if (owner != 0u) {
        if (lane == __ffs(owner) - 1) {
          int rem = want - excl, digit = 7;
#pragma unroll
          for (int b = 0; b < 8; ++b) {
            if (rem <= local[b]) {
              digit = b;
              break;
            }
            rem -= local[b];
          }
          s_kth = rem;
          s_prefix = prefix | ((uint64_t)(lane * 8 + digit) << shift);
        }
      } else if (lane == 31) {
        // kth beyond the matching keys: the last bin, as a linear walk ends.
        s_kth = want - (incl - local[7]);
        s_prefix = prefix | (255ull << shift);
      }
    }
    __syncthreads();
  }
  return s_prefix;
}

// Gathers the keys of one query's lists into ukeys (shared memory, any
// order), keeping those <= filter: one warp per list, four loads per lane
// in flight, appends combined per warp.  Returns the number of kept keys
// (it may exceed cap; only the first cap are stored).  Every thread of the
// block calls it.
static __device__ int gather_union(const uint64_t* __restrict__ part_keys,
                                   const int* __restrict__ part_counts, int64_t pbase,
                                   int num_parts, int stride, uint64_t filter, uint64_t* ukeys,
                                   int cap) {
  __shared__ int s_total;
  if (threadIdx.x == 0) s_total = 0;
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarps = blockDim.x >> 5;
  for (int p = warp; p < num_parts; p += nwarps) {
    const int c = part_counts[pbase + p];
    const uint64_t* src = part_keys + (pbase + p) * stride;
    for (int j0 = 0; j0 < c; j0 += 128) {
      uint64_t kk[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int j = j0 + u * 32 + lane;
        kk[u] = j < c ? src[j] : kEmptyKey;
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int j = j0 + u * 32 + lane;
        const bool keep = j < c && kk[u] <= filter;
        const unsigned m = __ballot_sync(kFullMask, keep);
        if (m == 0u) continue;
        int base = 0;
        if (lane == 0) base = atomicAdd(&s_total, __popc(m));
        base = __shfl_sync(kFullMask, base, 0);
        const int slot = base + __popc(m & ((1u << lane) - 1));
        if (keep && slot < cap) ukeys[slot] = kk[u];
      }
    }
  }
  __syncthreads();
  return s_total;
}

// ---------------------------------------------------------------------------
// Merge + reference rescoring.  One block (256 threads) per query.
// exact_mode: the part keys already hold reference ranks; the candidates are
// exactly the k best keys.
// gthr (optional, fast mode): per query an upper bound on its kp-th best
// fast key over all rows (the shared list threshold of the tensor-core
// scan).  Keys above it are left out of the union, as if every list had
// dropped them; the coverage check then also requires the bound to lie
// above the candidate limit.
// band (optional, fast mode): per query a rank limit computed over every
// shard of a sharded search; the candidate limit is the lower of it and the
// query's own F_k + 2 eps.
// ---------------------------------------------------------------------------
template <typename Scorer, int MAXC>
__global__ void __launch_bounds__(256) merge_rescore_kernel(
    Scorer sc, const uint32_t* __restrict__ pos_of_keyrank, const uint64_t* __restrict__ keys,
    const int* __restrict__ query_ids, int k, float radius, int exact_mode,
    const uint64_t* __restrict__ part_keys, const int* __restrict__ part_counts,
    const uint64_t* __restrict__ part_sat, int num_parts, int stride,
    uint64_t* __restrict__ out_keys, float* __restrict__ out_scores, int* __restrict__ out_counts,
    uint32_t* __restrict__ out_pos, int* __restrict__ q_flags,
    const unsigned long long* __restrict__ gthr, const float* __restrict__ band,
    int entries_cap) {
  const int metric = sc.metric;
  extern __shared__ __align__(16) unsigned char merge_smem[];
  uint64_t* ukeys = reinterpret_cast<uint64_t*>(merge_smem);  // [entries_cap]
  __shared__ int hist[256];
  __shared__ uint64_t cand[MAXC];
  __shared__ int s_ncand, s_fail;
  const int slot_q = blockIdx.x;
  const int qi = query_ids ? query_ids[blockIdx.x] : blockIdx.x;
  const int64_t pbase = (int64_t)slot_q * num_parts;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nwarps = blockDim.x >> 5;

  if (threadIdx.x == 0) {
    s_ncand = 0;
    s_fail = 0;
  }
  const uint64_t filter = (gthr && !exact_mode) ? (uint64_t)gthr[qi] : kEmptyKey;
  const int total =
      gather_union(part_keys, part_counts, pbase, num_parts, stride, filter, ukeys, entries_cap);
  if (total == 0) {
    if (threadIdx.x == 0) out_counts[qi] = 0;
    return;
  }
  if (total > entries_cap) {
    // More keys than the shared buffer holds (the unfiltered union cannot
    // reach it with the list sizes the scans produce): route the query to
    // the exact path rather than read past the buffer.
    if (threadIdx.x == 0) {
      atomicOr(&q_flags[qi], 2);
      out_counts[qi] = 0;
    }
    return;
  }
  const int kth = min(k, total);
  uint64_t limit;
  if (exact_mode) {
    limit = smem_radix_select(ukeys, total, kth, 0, hist);
  } else {
    const uint64_t kr = smem_radix_select(ukeys, total, kth, 32, hist);
    const float eps = sc.eps(qi);
    float t = __fadd_ru(rank_of(kr), 2.f * eps);
    if (band) {
      const float b = band[qi];
      if (b < t) t = b;  // NaN (no band) keeps the query's own limit
    }
    limit = ((uint64_t)float_to_ordered(t) << 32) | 0xffffffffull;
    // Coverage: a list dropped only keys above its saturation key, and the
    // filter only keys above itself.
    for (int p = threadIdx.x; p < num_parts; p += blockDim.x) {
      const uint64_t sat = part_sat[pbase + p];
      if (sat != kEmptyKey && sat <= limit) atomicExch(&s_fail, 1);
    }
    if (threadIdx.x == 0 && filter != kEmptyKey && filter <= limit) atomicExch(&s_fail, 1);
  }
  {
    const int tpad = (total + 31) & ~31;
    for (int i = threadIdx.x; i < tpad; i += blockDim.x) {
      const uint64_t key = i < total ? ukeys[i] : kEmptyKey;
      const bool in = i < total && key <= limit;
      const unsigned m = __ballot_sync(kFullMask, in);
      if (m == 0u) continue;
      int base = 0;
      if (lane == 0) base = atomicAdd(&s_ncand, __popc(m));
      base = __shfl_sync(kFullMask, base, 0);
      const int slot = base + __popc(m & ((1u << lane) - 1));
      if (in && slot < MAXC) cand[slot] = key;
    }
  }
  __syncthreads();
  if (s_fail || s_ncand > MAXC) {
    if (threadIdx.x == 0) {
      atomicOr(&q_flags[qi], 2);
      out_counts[qi] = 0;
    }
    return;
  }
  const int ncand = s_ncand;
  // Reference rescoring: one warp per candidate, or one half-warp per
  // candidate when the scorer evaluates a row per half-warp.
  if (sc.half_warp()) {
    const int half = lane >> 4;
    for (int c0 = warp * 2; c0 < ncand; c0 += nwarps * 2) {
      // An odd last candidate is scored by both halves; one writes it.
      const int c = min(c0 + half, ncand - 1);
      const uint32_t kr = pos_of(cand[c]);
      const uint32_t pos = pos_of_keyrank[kr];
      const float s = sc.score(qi, pos);
      __syncwarp();
      if ((lane & 15) == 0 && c0 + half < ncand) {
        if (!finite_f(s)) atomicOr(&q_flags[qi], sc.error_flag(s));
        cand[c] = pack_rank(rank_from_score(metric, s), kr);
      }
    }
  } else {
    for (int c = warp; c < ncand; c += nwarps) {
      const uint32_t kr = pos_of(cand[c]);
      const uint32_t pos = pos_of_keyrank[kr];
      const float s = sc.score(qi, pos);
      if (lane == 0) {
        if (!finite_f(s)) atomicOr(&q_flags[qi], sc.error_flag(s));
        cand[c] = pack_rank(rank_from_score(metric, s), kr);
      }
    }
  }
  __syncthreads();
  block_sort_u64_fit<MAXC>(cand, ncand);
  // Final top-k (radius is monotone in the sorted order).
  if (threadIdx.x < 32) {
    // Count the prefix within radius with a warp scan over chunks.
    int count = 0;
    for (int base = 0; base < ncand && count < k; base += 32) {
      const int i = base + lane;
      bool in = i < ncand;
      float s = 0.f;
      if (in) {
        s = sc.output(rank_of(cand[i]));
        in = sc.keep(s, radius);
      }
      const unsigned m = __ballot_sync(kFullMask, in);
      const int run = (m == kFullMask) ? 32 : __ffs(~m) - 1;  // leading in-radius run
      if (lane < run && count + lane < k) {
        const uint32_t pos = pos_of_keyrank[pos_of(cand[i])];
        out_keys[(int64_t)qi * k + count + lane] = keys[pos];
        out_scores[(int64_t)qi * k + count + lane] = s;
        if (out_pos) out_pos[(int64_t)qi * k + count + lane] = pos;
      }
      count = min(k, count + run);
      if (run < 32) break;
    }
    if (lane == 0) out_counts[qi] = count;
  }
}

// First half of a sharded search's band: per query, the k best fast ranks
// of this shard's lists (ascending is not required; +inf pads a shard with
// fewer) and the shard's bound eps on |fast - reference|, written as k + 1
// floats at out[q * (k + 1)].  The lists and the filter are those the merge
// reads.
template <typename Scorer>
__global__ void __launch_bounds__(256) band_prepare_kernel(
    Scorer sc, int k, const uint64_t* __restrict__ part_keys, const int* __restrict__ part_counts,
    int num_parts, int stride, const unsigned long long* __restrict__ gthr, int entries_cap,
    float* __restrict__ out) {
  extern __shared__ __align__(16) unsigned char band_smem[];
  uint64_t* ukeys = reinterpret_cast<uint64_t*>(band_smem);
  __shared__ int hist[256];
  __shared__ int s_n;
  const int q = blockIdx.x;
  float* dst = out + (int64_t)q * (k + 1);
  const uint64_t filter = gthr ? (uint64_t)gthr[q] : kEmptyKey;
  const int total = gather_union(part_keys, part_counts, (int64_t)q * num_parts, num_parts,
                                 stride, filter, ukeys, entries_cap);
  const int m = min(total, entries_cap);
  // A truncated union gives a subset of real fast ranks: its k best are
  // still ranks of real rows, so the band stays valid (only wider).
  const int kth = min(k, m);
  uint64_t kkey = 0;
  if (kth > 0) kkey = smem_radix_select(ukeys, m, kth, 0, hist);
  if (threadIdx.x == 0) s_n = 0;
  __syncthreads();
  for (int i = threadIdx.x; i < m; i += blockDim.x)
    if (kth > 0 && ukeys[i] <= kkey) dst[atomicAdd(&s_n, 1)] = rank_of(ukeys[i]);
  __syncthreads();
  for (int i = s_n + threadIdx.x; i < k; i += blockDim.x) dst[i] = INFINITY;
  if (threadIdx.x == 0) dst[k] = sc.eps(q);
}

// Per query, the lists of one scan (num_parts lists of at most kp keys, as
// the streaming scans write them): their union's best keys.
// Threshold mode (gthr_out): the kp-th best key becomes the query's starting
// threshold for a later pass (left at all-ones when the lists hold fewer
// than kp keys).  List mode: the best out_cap keys (out_cap >= kp) become the
// query's one candidate list (out_*, stride out_cap), its saturation the
// lowest of the lists' and, when keys were left out here, the out_cap-th
// key.  Keeping several kp keeps that saturation well above the candidate
// limit F_k + 2 eps even where the distances of the nearest rows crowd
// together.
static __global__ void __launch_bounds__(1024) reduce_lists_kernel(
    const uint64_t* __restrict__ keys, const int* __restrict__ counts,
    const uint64_t* __restrict__ sats, int num_parts, int kp, int out_cap,
    unsigned long long* __restrict__ gthr_out, uint64_t* __restrict__ out_keys,
    int* __restrict__ out_counts, uint64_t* __restrict__ out_sat) {
  extern __shared__ __align__(16) unsigned char reduce_smem[];
  uint64_t* ukeys = reinterpret_cast<uint64_t*>(reduce_smem);  // [num_parts * kp]
  __shared__ int hist[256];
  __shared__ unsigned long long s_sat;
  __shared__ int s_n;
  const int q = blockIdx.x;
  const int64_t pbase = (int64_t)q * num_parts;
  if (threadIdx.x == 0) {
    s_sat = kEmptyKey;
    s_n = 0;
  }
  const int total =
      gather_union(keys, counts, pbase, num_parts, kp, kEmptyKey, ukeys, num_parts * kp);
  for (int p = threadIdx.x; p < num_parts; p += blockDim.x)
    atomicMin(&s_sat, (unsigned long long)sats[pbase + p]);
  __syncthreads();
  const int m = min(total, num_parts * kp);
  if (gthr_out) {
    if (m >= kp) {
      const uint64_t kth = smem_radix_select(ukeys, m, kp, 0, hist);
      if (threadIdx.x == 0) gthr_out[q] = kth;
    }
    return;
  }
  uint64_t cut = kEmptyKey;
  if (m > out_cap) cut = smem_radix_select(ukeys, m, out_cap, 0, hist);
  for (int i = threadIdx.x; i < m; i += blockDim.x)
    if (ukeys[i] <= cut) out_keys[(int64_t)q * out_cap + atomicAdd(&s_n, 1)] = ukeys[i];
  __syncthreads();
  if (threadIdx.x == 0) {
    out_counts[q] = s_n;
    out_sat[q] = min((uint64_t)s_sat, cut);
  }
}

static inline bool reduce_lists_supported(int num_parts, int kp) {
  return (int64_t)num_parts * kp * 8 <= 200 * 1024;
}

// One block of 1024 threads per query (reduce_lists_kernel).
// Candidate list length of the list mode: eight kp, within the merge's
// shared buffer.
static inline int reduce_lists_out_cap(int kp) { return std::min(8 * kp, kMergeSmemEntries); }

static inline cudaError_t launch_reduce_lists(const uint64_t* keys, const int* counts,
                                              const uint64_t* sats, int nq, int num_parts,
                                              int kp, int out_cap, unsigned long long* gthr_out,
                                              uint64_t* out_keys, int* out_counts,
                                              uint64_t* out_sat, cudaStream_t stream) {
  if (nq <= 0) return cudaSuccess;
  if (!reduce_lists_supported(num_parts, kp) || out_cap < kp) return cudaErrorInvalidValue;
  const int smem = num_parts * kp * 8;
  cudaFuncSetAttribute(reduce_lists_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  reduce_lists_kernel<<<nq, 1024, smem, stream>>>(keys, counts, sats, num_parts, kp, out_cap,
                                                  gthr_out, out_keys, out_counts, out_sat);
  return cudaGetLastError();
}

template <typename RowT, typename Ranker>
cudaError_t launch_scan_simt(const RowT* rows, int64_t n, int d, const uint32_t* keyrank,
                             const float* qf, int nq, const uint32_t* bitmap, const Ranker& rk,
                             int num_parts, int kp, uint64_t* part_keys, int* part_counts,
                             uint64_t* part_sat, int* q_flags, cudaStream_t stream) {
  int need = kp + 2 * kSimtRT, cap = 256;
  while (cap < need) cap <<= 1;
  const int64_t rows_per_part =
      ((n + num_parts - 1) / num_parts + kSimtRT - 1) / kSimtRT * kSimtRT;
  dim3 grid((nq + kSimtQT - 1) / kSimtQT, num_parts);
  const size_t tiles = (size_t)(kSimtKT * (kSimtRT + 4) + kSimtKT * (kSimtQT + 4)) * sizeof(float);
  if (cap == 256) {
    const size_t smem = (size_t)kSimtQT * 256 * 8 + tiles;
    auto kern = scan_simt_kernel<RowT, 256, Ranker>;
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    kern<<<grid, 256, smem, stream>>>(rows, n, d, keyrank, qf, nq, bitmap, rk, rows_per_part,
                                      kp, part_keys, part_counts, part_sat, q_flags);
  } else if (cap == 512) {
    const size_t smem = (size_t)kSimtQT * 512 * 8 + tiles;
    auto kern = scan_simt_kernel<RowT, 512, Ranker>;
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    kern<<<grid, 256, smem, stream>>>(rows, n, d, keyrank, qf, nq, bitmap, rk, rows_per_part,
                                      kp, part_keys, part_counts, part_sat, q_flags);
  } else {
    return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

template <typename Scorer>
cudaError_t launch_scan_exact(const Scorer& sc, int64_t n, const uint32_t* keyrank,
                              const int* query_ids, int nlist, const uint32_t* bitmap,
                              int num_parts, int kp, uint64_t* part_keys, int* part_counts,
                              uint64_t* part_sat, int* q_flags, cudaStream_t stream) {
  int need = kp + 2 * 128, cap = 512;
  while (cap < need) cap <<= 1;
  const int64_t rows_per_part = (n + num_parts - 1) / num_parts;
  dim3 grid(nlist, num_parts);
  const size_t smem = (size_t)cap * 8;
#define XVEC_EXACT_CASE(C)                                                                   \
  if (cap == C) {                                                                            \
    auto kern = scan_exact_kernel<C, Scorer>;                                                \
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);      \
    kern<<<grid, 256, smem, stream>>>(sc, n, keyrank, query_ids, bitmap, rows_per_part, kp,  \
                                      part_keys, part_counts, part_sat, q_flags);           \
    return cudaGetLastError();                                                               \
  }
  XVEC_EXACT_CASE(512)
  XVEC_EXACT_CASE(1024)
  XVEC_EXACT_CASE(2048)
  XVEC_EXACT_CASE(4096)
  XVEC_EXACT_CASE(8192)
#undef XVEC_EXACT_CASE
  return cudaErrorInvalidValue;
}

template <typename Scorer>
cudaError_t launch_merge_rescore(const Scorer& sc, const uint32_t* pos_of_keyrank,
                                 const uint64_t* keys, const int* query_ids, int nlist, int k,
                                 float radius, int exact_mode, const uint64_t* part_keys,
                                 const int* part_counts, const uint64_t* part_sat, int num_parts,
                                 int stride, uint64_t* out_keys, float* out_scores,
                                 int* out_counts, uint32_t* out_pos, int* q_flags,
                                 cudaStream_t stream, const unsigned long long* gthr = nullptr,
                                 const float* band = nullptr) {
  if (nlist <= 0) return cudaSuccess;
  if (num_parts > 1024) return cudaErrorInvalidValue;
  // A filtered union is small (a few kp): a smaller buffer lets more blocks
  // share an SM; a query that overflows it takes the exact path.
  const int cap = (gthr && !exact_mode) ? kMergeFilteredEntries : kMergeSmemEntries;
  const int smem = cap * 8;
  if (k > kMaxCandidatesWide) return cudaErrorInvalidValue;
  auto kern = k > kMaxCandidates ? merge_rescore_kernel<Scorer, kMaxCandidatesWide>
                                 : merge_rescore_kernel<Scorer, kMaxCandidates>;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  kern<<<nlist, 256, smem, stream>>>(sc, pos_of_keyrank, keys, query_ids, k, radius, exact_mode,
                                     part_keys, part_counts, part_sat, num_parts, stride,
                                     out_keys, out_scores, out_counts, out_pos, q_flags, gthr,
                                     band, cap);
  return cudaGetLastError();
}

// The sharded band (band_prepare_kernel, band_limit_kernel) around one
// exchange: `out` receives nq * (k + 1) floats.
template <typename Scorer>
cudaError_t launch_band_prepare(const Scorer& sc, int nq, int k, const uint64_t* part_keys,
                                const int* part_counts, int num_parts, int stride,
                                const unsigned long long* gthr, float* out, cudaStream_t stream) {
  if (nq <= 0) return cudaSuccess;
  if (num_parts > 1024) return cudaErrorInvalidValue;
  const int cap = gthr ? kMergeFilteredEntries : kMergeSmemEntries;
  const int smem = cap * 8;
  cudaFuncSetAttribute(band_prepare_kernel<Scorer>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                       smem);
  band_prepare_kernel<Scorer><<<nq, 256, smem, stream>>>(sc, k, part_keys, part_counts, num_parts,
                                                        stride, gthr, cap, out);
  return cudaGetLastError();
}

}  // namespace xvec
