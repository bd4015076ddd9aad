// diskann.cu — DiskANN graph search with the PQ frontier.
//
// Reference: DiskANNIndex.searchDiskANN (internal/core/diskann.go:476-525),
// searchDiskANNGraph (:559-651), diskANNApproximateScore (:653-683),
// diskANNReadBatchSize (:685-691) and diskANNResultCollector (:693-737);
// the PQ table and lookup (pq.go:549-595); the build's codes of the prepared
// vectors (prepareDiskANNPQVectors :258-274, EncodeBatch :234) and the MIPSL2
// code norms (diskANNPQCodeNorms :292-323).  Node vectors, PQ codes and the
// graph live in device memory: the node reads of the reference's sector
// file become row loads.
//
// The reference keeps two heaps — `retained`, the `capacity` best nodes by
// PQ score seen so far, and the frontier, every node pushed when it entered
// retained — pops up to `beam` live frontier nodes (retained, not expanded)
// per round, scores each exactly into a top-k collector and offers its
// unvisited neighbours to retained.  Two facts make a round data-parallel:
//   * every visited node is offered to retained exactly once, and a node
//     that leaves retained is never offered again, so after any sequence of
//     offers retained is the `capacity` best of the nodes visited so far,
//     whatever the order of the offers;
//   * the live frontier is therefore retained minus the expanded nodes, and a
//     round's batch is its `beam` best entries.
// One block per query keeps retained as a sorted array with an expanded flag
// per entry, takes the first `beam` unexpanded entries as the round's batch,
// scores them (a warp per node), claims their unvisited neighbours in a
// visited bitmap, PQ-scores the claimed ones and merges them (sorted) into
// retained: the same batches, expansions and collector as the reference's
// heaps.  Errors keep the reference's order: a round records the position
// (batch node, then neighbour) of each failure and the first one decides
// the query's status, as the sequential loop would have stopped there.
#include <algorithm>
#include <cfloat>
#include <cmath>
#include <vector>

#include "capi_internal.h"
#include "common.cuh"
#include "flat_kernels.cuh"
#include "flat_tc.cuh"
#include "index_kernels.cuh"
#include "pipeline.cuh"
#include "select.cuh"

namespace xvec {
namespace {

constexpr int kDiskThreads = 256;
constexpr int kDiskWarps = kDiskThreads / 32;
constexpr int kDiskMaxCap = 2048;     // capacity = min(n, max(TopK, ListSize))
constexpr int kDiskCand = 2048;       // neighbour slots per merge step (also the degree bound)
constexpr int kDiskMaxBeam = 128;     // MaxDiskANNReadSectors (diskann_storage.go:31)
constexpr int kDiskVisitCap = 16384;  // visited nodes recorded per slot for the reset
constexpr int kDiskSmemChunks = 64;   // PQ tables up to 64 KB go to shared memory
constexpr int kDiskPerThread = kDiskCand / kDiskThreads;  // slots per thread in a step
constexpr int kDefaultListSize = 300; // DefaultDiskANNQueryList (diskann.go:36)
constexpr unsigned kNoError = 0xffffffffu;

inline unsigned blocks_of(int64_t n, int t = 256) { return (unsigned)((n + t - 1) / t); }

struct DiskArgs {
  int metric, traversal, d, chunks, beam, cap, k, nq, max_degree;
  int64_t n, entry, words;
  const float* rows;           // [n][d] node vectors (float32 originals)
  const uint32_t* keyrank;     // position -> rank of its key
  const uint32_t* pos_of_kr;   // key rank -> position
  const uint64_t* keys;        // [n]
  const uint8_t* codes;        // [n][chunks] PQ codes of the prepared rows
  const float* code_norms;     // [n] (MIPSL2)
  const int64_t* goff;         // [n + 1]
  const int32_t* nbrs;
  const float* qf;             // [nq][d] the queries (validated)
  const float* table;          // [nq][chunks][256] PQ tables of the prepared queries
  const double* qnorm;         // [nq] diskANNVectorNormSquared of the prepared queries
  const int* q_status;         // query validation
  const int* q_flags;          // 4: a table entry failed
  float radius;
  const uint32_t* bitmap;
  uint32_t* visited;           // [slots][words]
  uint32_t* vrec;              // [slots][kDiskVisitCap]
  uint64_t* out_keys;
  float* out_scores;
  int* out_counts;
};

// diskANNApproximateScore (diskann.go:653-676): the table lookup summed in
// float64 in chunk order (PQDistanceTable.Lookup, pq.go:574-595), and for
// MIPSL2 the conversion through the code and query norms.  0, or the
// failing status.  `table` is the query's [chunks][256] table in shared or
// global memory; codes of 16-byte multiples are read as 16-byte vectors.
__device__ __forceinline__ int disk_pq_score(const DiskArgs& a, const float* table, double qn,
                                             uint32_t id, float* out) {
  const uint8_t* code = a.codes + (int64_t)id * a.chunks;
  double s = 0.0;
  if ((a.chunks & 15) == 0) {
    const uint4* cv = reinterpret_cast<const uint4*>(code);
    for (int c0 = 0; c0 < a.chunks; c0 += 16) {
      const uint4 v = __ldg(cv + (c0 >> 4));
      const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const uint32_t b = (w[j >> 2] >> (8 * (j & 3))) & 0xffu;
        s = __dadd_rn(s, (double)table[(c0 + j) * 256 + b]);
      }
    }
  } else {
    for (int c = 0; c < a.chunks; ++c) s = __dadd_rn(s, (double)table[c * 256 + code[c]]);
  }
  if (isnan(s) || isinf(s) || s > (double)FLT_MAX || s < -(double)FLT_MAX) return XVEC_GPU_OVERFLOW;
  const float score = __double2float_rn(s);
  if (a.metric != kMetricMIPS) {
    *out = score;
    return 0;
  }
  const double cn = (double)a.code_norms[id];
  const double inner = __ddiv_rn(__dsub_rn(__dadd_rn(qn, cn), (double)score), 2.0);
  const double den = go_maxd(qn, cn);
  if (den == 0.0) {
    *out = 0.f;
    return 0;
  }
  const double conv = __dsub_rn(2.0, __ddiv_rn(__dmul_rn(2.0, inner), den));
  if (isnan(conv) || isinf(conv) || conv > (double)FLT_MAX || conv < -(double)FLT_MAX)
    return XVEC_GPU_OVERFLOW;
  *out = __double2float_rn(conv);
  return 0;
}

// The float64 chunk-order sum of a code held in registers (16 or 32 bytes).
// TREE: the query's table makes every partial sum exact in float64 (see
// the kernel), so four interleaved accumulators give the same bits as the
// chunk-order chain with a quarter of its latency.
template <bool TREE>
__device__ __forceinline__ double pq_sum_codes(const float* table, const uint4 (&cv)[2], int vec) {
  double s[4] = {0.0, 0.0, 0.0, 0.0};
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    if (h >= vec) break;
    const uint32_t w[4] = {cv[h].x, cv[h].y, cv[h].z, cv[h].w};
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const uint32_t b = (w[j >> 2] >> (8 * (j & 3))) & 0xffu;
      const int acc = TREE ? (j & 3) : 0;
      s[acc] = __dadd_rn(s[acc], (double)table[(h * 16 + j) * 256 + b]);
    }
  }
  return TREE ? __dadd_rn(__dadd_rn(s[0], s[1]), __dadd_rn(s[2], s[3])) : s[0];
}

// diskANNApproximateScore after the lookup sum: the overflow check of
// Lookup and the MIPSL2 conversion.
__device__ __forceinline__ int disk_pq_finish(const DiskArgs& a, const float* table, double qn,
                                              uint32_t id, double s, float* out) {
  if (isnan(s) || isinf(s) || s > (double)FLT_MAX || s < -(double)FLT_MAX) return XVEC_GPU_OVERFLOW;
  const float score = __double2float_rn(s);
  if (a.metric != kMetricMIPS) {
    *out = score;
    return 0;
  }
  const double cn = (double)a.code_norms[id];
  const double inner = __ddiv_rn(__dsub_rn(__dadd_rn(qn, cn), (double)score), 2.0);
  const double den = go_maxd(qn, cn);
  if (den == 0.0) {
    *out = 0.f;
    return 0;
  }
  const double conv = __dsub_rn(2.0, __ddiv_rn(__dmul_rn(2.0, inner), den));
  if (isnan(conv) || isinf(conv) || conv > (double)FLT_MAX || conv < -(double)FLT_MAX)
    return XVEC_GPU_OVERFLOW;
  *out = __double2float_rn(conv);
  return 0;
}

// The frontier's order (diskann.go:571-576): the traversal metric's Better,
// ties to the lower node id; -0 and +0 rank equal (the reference compares
// scores with ==).
__device__ __forceinline__ uint64_t disk_node_key(int traversal, float score, uint32_t id) {
  return pack_rank(rank_from_score(traversal, score) + 0.f, id);
}

// Number of entries of the sorted run a[0, n) below x.
__device__ __forceinline__ int count_less(const uint64_t* a, int n, uint64_t x) {
  int lo = 0, hi = n;
  while (lo < hi) {
    const int mid = (lo + hi) >> 1;
    if (a[mid] < x) lo = mid + 1;
    else hi = mid;
  }
  return lo;
}

// out[0, limit) = the `limit` smallest keys of the sorted runs a[0, na) and
// b[0, nb) (keys distinct); a's flags move with its entries (when given),
// b's entries get flag 0.
__device__ void merge_runs(const uint64_t* a, const uint8_t* fa, int na, const uint64_t* b,
                           int nb, uint64_t* out, uint8_t* fo, int limit) {
  for (int i = threadIdx.x; i < na; i += blockDim.x) {
    const int p = i + count_less(b, nb, a[i]);
    if (p < limit) {
      out[p] = a[i];
      if (fo) fo[p] = fa[i];
    }
  }
  for (int j = threadIdx.x; j < nb; j += blockDim.x) {
    const int p = j + count_less(a, na, b[j]);
    if (p < limit) {
      out[p] = b[j];
      if (fo) fo[p] = 0;
    }
  }
}

// Block-wide exclusive prefix sum of v (every thread calls it); *total gets
// the sum.
__device__ __forceinline__ int block_exclusive_sum(int v, int* total) {
  __shared__ int s_warp[kDiskWarps];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int incl = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int t = __shfl_up_sync(kFullMask, incl, o);
    if (lane >= o) incl += t;
  }
  if (lane == 31) s_warp[warp] = incl;
  __syncthreads();
  int base = 0, sum = 0;
  for (int w = 0; w < kDiskWarps; ++w) {
    const int t = s_warp[w];
    if (w < warp) base += t;
    sum += t;
  }
  __syncthreads();
  *total = sum;
  return base + incl - v;
}

// Sorts the n (<= kDiskThreads) distinct keys of a into out by rank: each
// key's position is the number of keys below it (one pass, no stages).
__device__ __forceinline__ void block_rank_sort(const uint64_t* a, int n, uint64_t* out) {
  const int t = threadIdx.x;
  if (t < n) {
    const uint64_t x = a[t];
    int r = 0;
    for (int j = 0; j < n; ++j) r += a[j] < x;
    out[r] = x;
  }
}

// Shared-memory layout of the search block (bytes).
struct DiskSmem {
  int capA, k;
  size_t tbl, r0, r1, e0, e1, k0, k1, x, x2, hist, bk, bk2, boff, bid, bdeg, gb, nbs, work, fresh,
      total;
  __host__ __device__ DiskSmem(int cap_alloc, int k_alloc, int table_floats)
      : capA(cap_alloc), k(k_alloc) {
    size_t o = 0;
    tbl = o; o += (size_t)table_floats * 4;
    r0 = o; o += (size_t)capA * 8;
    r1 = o; o += (size_t)capA * 8;
    k0 = o; o += (size_t)k * 8;
    k1 = o; o += (size_t)k * 8;
    x = o; o += (size_t)kDiskCand * 8;
    hist = o; o += 256 * 4;
    bk = o; o += (size_t)kDiskMaxBeam * 8;
    bk2 = o; o += (size_t)kDiskMaxBeam * 8;
    boff = o; o += (size_t)kDiskMaxBeam * 8;
    bid = o; o += (size_t)kDiskMaxBeam * 4;
    bdeg = o; o += (size_t)(kDiskMaxBeam + 1) * 4;
    gb = o; o += (size_t)(kDiskMaxBeam + 1) * 4;
    // The step's neighbour ids and claimed nodes, dead once the step's
    // candidates are scored, share their 16 KB with the sorted candidates.
    nbs = o; o += (size_t)kDiskCand * 4;
    work = o; o += (size_t)kDiskCand * 4;
    x2 = nbs;
    e0 = o; o += (size_t)capA;
    e1 = o; o += (size_t)capA;
    fresh = o; o += (size_t)kDiskCand;
    total = (o + 15) & ~(size_t)15;
  }
};

// One block per query slot; the slot's blocks take queries blockIdx.x,
// blockIdx.x + gridDim.x, ...  SMEM_TABLE: the query's PQ table is copied
// into shared memory (chunks <= kDiskSmemChunks).
template <bool SMEM_TABLE>
__global__ void __launch_bounds__(kDiskThreads, 3) diskann_search_kernel(DiskArgs a, int capA) {
  extern __shared__ __align__(16) unsigned char smem[];
  const DiskSmem L(capA, a.k, SMEM_TABLE ? a.chunks * 256 : 0);
  float* T = reinterpret_cast<float*>(smem + L.tbl);
  // The double buffers chosen by a select, not an indexed array (which
  // would live in local memory).
  uint64_t* const R0 = reinterpret_cast<uint64_t*>(smem + L.r0);
  uint64_t* const R1 = reinterpret_cast<uint64_t*>(smem + L.r1);
  uint8_t* const E0 = smem + L.e0;
  uint8_t* const E1 = smem + L.e1;
  uint64_t* const K0 = reinterpret_cast<uint64_t*>(smem + L.k0);
  uint64_t* const K1 = reinterpret_cast<uint64_t*>(smem + L.k1);
  auto R = [&](int c) { return c ? R1 : R0; };
  auto E = [&](int c) { return c ? E1 : E0; };
  auto K = [&](int c) { return c ? K1 : K0; };
  uint64_t* X = reinterpret_cast<uint64_t*>(smem + L.x);
  uint64_t* X2 = reinterpret_cast<uint64_t*>(smem + L.x2);
  int* HIST = reinterpret_cast<int*>(smem + L.hist);
  uint64_t* BK = reinterpret_cast<uint64_t*>(smem + L.bk);
  uint64_t* BK2 = reinterpret_cast<uint64_t*>(smem + L.bk2);
  int64_t* BOFF = reinterpret_cast<int64_t*>(smem + L.boff);
  uint32_t* BID = reinterpret_cast<uint32_t*>(smem + L.bid);
  int* BDEG = reinterpret_cast<int*>(smem + L.bdeg);
  int* GB = reinterpret_cast<int*>(smem + L.gb);
  uint32_t* NB = reinterpret_cast<uint32_t*>(smem + L.nbs);
  uint32_t* WORK = reinterpret_cast<uint32_t*>(smem + L.work);
  uint8_t* FRESH = smem + L.fresh;
  __shared__ int s_r, s_cur, s_kc, s_kcur, s_xc, s_ngroups, s_vcount, s_pq_fail, s_status, s_wc;
  __shared__ int s_safe, s_valid, s_emax, s_emin, s_xn;
  __shared__ unsigned s_err_pos, s_maxabs;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  uint32_t* vis = a.visited + (int64_t)blockIdx.x * a.words;
  uint32_t* vrec = a.vrec + (int64_t)blockIdx.x * kDiskVisitCap;
  const unsigned stride = (unsigned)a.max_degree + 1;  // error positions: node j, slot 0..degree
  const int tsize = a.chunks * 256;

  for (int q = blockIdx.x; q < a.nq; q += gridDim.x) {
    const float* qv = a.qf + (int64_t)q * a.d;
    const float* gtable = a.table + (int64_t)q * tsize;
    const double qn = a.qnorm[q];
    int status = a.q_status[q];
    if (status == 0 && (a.q_flags[q] & 4)) status = XVEC_GPU_NON_FINITE;
    if (status != 0 || a.n == 0) {
      if (tid == 0) a.out_counts[q] = status ? -status : 0;
      continue;
    }
    // The table (copied when in shared memory) and its largest magnitude:
    // while chunks x that stays below MaxFloat32 no lookup can overflow, and
    // the claims need not remember which slots saw a node unvisited.
    // Also the span of its non-zero entries' exponents: every entry is a
    // multiple of 2^(e_min - 150) and a sum of at most 32 of them is below
    // 2^(e_max - 121), so with e_max - e_min <= 24 every partial sum is exact
    // in float64 and the lookup may add in any order.
    if (tid == 0) {
      s_maxabs = 0u;
      s_emax = 0;
      s_emin = 255;
    }
    __syncthreads();
    float mx = 0.f;
    int emax = 0, emin = 255;
    for (int i = tid; i < tsize; i += kDiskThreads) {
      const float v = gtable[i];
      if (SMEM_TABLE) T[i] = v;
      mx = fmaxf(mx, fabsf(v));
      const uint32_t bits = __float_as_uint(v) & 0x7fffffffu;
      if (bits != 0u) {
        const int e = max(1, (int)(bits >> 23));
        emax = max(emax, e);
        emin = min(emin, e);
      }
    }
    for (int o = 16; o > 0; o >>= 1) {
      mx = fmaxf(mx, __shfl_xor_sync(kFullMask, mx, o));
      emax = max(emax, __shfl_xor_sync(kFullMask, emax, o));
      emin = min(emin, __shfl_xor_sync(kFullMask, emin, o));
    }
    if (lane == 0) {
      atomicMax(&s_maxabs, __float_as_uint(mx));  // non-negative floats order as ints
      atomicMax(&s_emax, emax);
      atomicMin(&s_emin, emin);
    }
    __syncthreads();
    const float* table = SMEM_TABLE ? T : gtable;
    // The entry point (diskann.go:588-597).
    if (tid == 0) {
      const uint32_t entry = (uint32_t)a.entry;
      s_safe = a.metric != kMetricMIPS &&
               (double)__uint_as_float(s_maxabs) * (double)a.chunks < 1e38;
      float es = 0.f;
      s_status = disk_pq_score(a, table, qn, entry, &es);
      R(0)[0] = disk_node_key(a.traversal, es, entry);
      E(0)[0] = 0;
      s_r = 1;
      s_cur = 0;
      s_kc = 0;
      s_kcur = 0;
      s_err_pos = kNoError;
      s_vcount = 1;
      vrec[0] = entry;
      atomicOr(vis + (entry >> 5), 1u << (entry & 31));
    }
    __syncthreads();
    const bool safe = s_safe != 0;
    const bool tree = s_emax - s_emin <= 24;
    // Rounds (diskann.go:600-649); each expands at least one node, so there
    // are at most n of them.
    while (s_status == 0) {
      // The batch: the first `beam` unexpanded entries of retained, in order.
      const int r = s_r, cur = s_cur;
      const int per = (r + kDiskThreads - 1) / kDiskThreads;
      const int i0 = min(r, tid * per), i1 = min(r, i0 + per);
      int cnt = 0;
      for (int i = i0; i < i1; ++i) cnt += E(cur)[i] == 0;
      int total;
      int idx = block_exclusive_sum(cnt, &total);
      for (int i = i0; i < i1 && idx < a.beam; ++i)
        if (E(cur)[i] == 0) {
          BID[idx++] = (uint32_t)R(cur)[i];
          E(cur)[i] = 1;
        }
      const int nb = min(total, a.beam);
      if (nb == 0) break;
      __syncthreads();
      // Exact scores (metric.Compute(query, node.Vector)), one warp per node,
      // into the round's collector keys (filter, radius: :709-721).  The
      // warp's rows are prefetched first, so their loads overlap.
      {
        const int row_bytes = a.d * 4;
        for (int j = warp; j < nb; j += kDiskWarps) {
          const char* rp = reinterpret_cast<const char*>(a.rows + (int64_t)BID[j] * a.d);
          for (int off = lane * 128; off < row_bytes; off += 32 * 128)
            asm volatile("prefetch.global.L1 [%0];" ::"l"(rp + off));
        }
      }
      // From d = 16 on the two half-warps score two nodes at once.
      const int per_warp = a.d >= 16 ? 2 : 1;
      for (int j0 = warp * per_warp; j0 < nb; j0 += kDiskWarps * per_warp) {
        const int j = per_warp == 2 ? j0 + (lane >> 4) : j0;
        const bool has = j < nb;
        const uint32_t id = BID[has ? j : j0];
        const float sc = warp_reference_score<float>(a.metric, a.rows + (int64_t)id * a.d, qv, a.d);
        if ((lane & 15) == 0 && has && (per_warp == 2 || lane == 0)) {
          uint64_t key = kEmptyKey;
          if (!finite_f(sc)) atomicMin(&s_err_pos, (unsigned)j * stride);
          else if (bitmap_pass(a.bitmap, id) && within_radius(a.metric, sc, a.radius))
            key = pack_rank(rank_from_score(a.metric, sc) + 0.f, a.keyrank[id]);
          BK[j] = key;
        }
      }
      // Neighbour slots of the batch, in merge steps of at most kDiskCand:
      // the nodes' list offsets and degrees (one thread per node), their
      // prefix sums (warp 0), the steps (thread 0, from shared memory).
      if (tid < nb) {
        const int64_t o0 = a.goff[BID[tid]];
        BOFF[tid] = o0;
        BDEG[tid + 1] = (int)(a.goff[BID[tid] + 1] - o0);
      }
      __syncthreads();
      if (warp == 0) {
        constexpr int kPer = kDiskMaxBeam / 32;
        int v[kPer], run = 0;
#pragma unroll
        for (int i = 0; i < kPer; ++i) {
          const int j = lane * kPer + i;
          run += j < nb ? BDEG[j + 1] : 0;
          v[i] = run;
        }
        int incl = run;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const int t = __shfl_up_sync(kFullMask, incl, o);
          if (lane >= o) incl += t;
        }
        const int before = incl - run;
#pragma unroll
        for (int i = 0; i < kPer; ++i) {
          const int j = lane * kPer + i;
          if (j < nb) BDEG[j + 1] = before + v[i];
        }
        if (lane == 0) BDEG[0] = 0;
      }
      __syncthreads();
      if (tid == 0) {
        int g = 0;
        GB[0] = 0;
        for (int j = 1; j < nb; ++j)
          if (BDEG[j + 1] - BDEG[GB[g]] > kDiskCand) GB[++g] = j;
        GB[++g] = nb;
        s_ngroups = g;
      }
      __syncthreads();
      const int ngroups = s_ngroups;
      for (int g = 0; g < ngroups; ++g) {
        const int j0 = GB[g], j1 = GB[g + 1], base = BDEG[j0];
        const int slots = BDEG[j1] - base;
        // The step's neighbour ids (node of a slot by a binary search of the
        // prefix sums), and which of them were unvisited before the step (L2
        // reads: the bitmap changes through atomics; kept only when a lookup
        // can fail).  A thread takes slots tid + 256 i (at most 8), its loads
        // issued together.
        {
          uint32_t nbv[kDiskPerThread];
#pragma unroll
          for (int i = 0; i < kDiskPerThread; ++i) {
            const int sl = tid + i * kDiskThreads;
            nbv[i] = 0;
            if (sl < slots) {
              int lo = j0, hi = j1 - 1;
              while (lo < hi) {
                const int mid = (lo + hi + 1) >> 1;
                if (BDEG[mid] - base <= sl) lo = mid;
                else hi = mid - 1;
              }
              nbv[i] = (uint32_t)__ldg(a.nbrs + BOFF[lo] + (sl + base - BDEG[lo]));
            }
          }
          uint32_t vw[kDiskPerThread];
#pragma unroll
          for (int i = 0; i < kDiskPerThread; ++i) {
            const int sl = tid + i * kDiskThreads;
            if (sl < slots) {
              NB[sl] = nbv[i];
              if (!safe) vw[i] = __ldcg(vis + (nbv[i] >> 5));
            }
          }
          if (!safe) {
#pragma unroll
            for (int i = 0; i < kDiskPerThread; ++i) {
              const int sl = tid + i * kDiskThreads;
              if (sl < slots) FRESH[sl] = ((vw[i] >> (nbv[i] & 31)) & 1u) == 0;
            }
          }
        }
        if (tid == 0) {
          s_xc = 0;
          s_wc = 0;
          s_pq_fail = 0;
        }
        __syncthreads();
        // Claims: the first slot to set a node's bit queues it for scoring
        // (a warp's winners take their queue places with one atomic).
        {
          uint32_t old[kDiskPerThread];
#pragma unroll
          for (int i = 0; i < kDiskPerThread; ++i) {
            const int sl = tid + i * kDiskThreads;
            old[i] = 0xffffffffu;
            if (sl < slots && (safe || FRESH[sl]))
              old[i] = atomicOr(vis + (NB[sl] >> 5), 1u << (NB[sl] & 31));
          }
#pragma unroll
          for (int i = 0; i < kDiskPerThread; ++i) {
            const int sl = tid + i * kDiskThreads;
            const uint32_t nbid = sl < slots ? NB[sl] : 0u;
            const bool won = sl < slots && ((old[i] >> (nbid & 31)) & 1u) == 0;
            const unsigned m = __ballot_sync(kFullMask, won);
            if (m == 0u) continue;
            const int leader = __ffs(m) - 1;
            int wbase = 0, vbase = 0;
            if (lane == leader) {
              wbase = atomicAdd(&s_wc, __popc(m));
              vbase = atomicAdd(&s_vcount, __popc(m));
            }
            wbase = __shfl_sync(kFullMask, wbase, leader);
            vbase = __shfl_sync(kFullMask, vbase, leader);
            if (won) {
              const int r = __popc(m & ((1u << lane) - 1u));
              WORK[wbase + r] = nbid;
              if (vbase + r < kDiskVisitCap) vrec[vbase + r] = nbid;
            }
          }
        }
        __syncthreads();
        const int rr = s_r, rc = s_cur, wc = s_wc;
        const uint64_t worst = rr >= a.cap ? R(rc)[rr - 1] : kEmptyKey;
        // PQ scores of the claimed nodes; those that beat a full retained
        // set's worst join the step's candidates.  Codes of 16 or 32 bytes:
        // two items per thread at a time, their code loads issued together.
        if (a.chunks == 16 || a.chunks == 32) {
          const int vec = a.chunks >> 4;
          for (int c0 = 0; c0 < wc; c0 += 2 * kDiskThreads) {
            uint4 cv[2][2];
#pragma unroll
            for (int i = 0; i < 2; ++i) {
              const int c = c0 + tid + i * kDiskThreads;
              if (c < wc) {
                const uint4* src = reinterpret_cast<const uint4*>(a.codes + (int64_t)WORK[c] * a.chunks);
                cv[i][0] = __ldg(src);
                cv[i][1] = vec > 1 ? __ldg(src + 1) : make_uint4(0u, 0u, 0u, 0u);
              }
            }
#pragma unroll
            for (int i = 0; i < 2; ++i) {
              const int c = c0 + tid + i * kDiskThreads;
              bool keep = false;
              uint64_t key = 0;
              if (c < wc) {
                const uint32_t nbid = WORK[c];
                const double sum = tree ? pq_sum_codes<true>(table, cv[i], vec)
                                        : pq_sum_codes<false>(table, cv[i], vec);
                float ps;
                if (disk_pq_finish(a, table, qn, nbid, sum, &ps)) {
                  s_pq_fail = 1;
                } else {
                  key = disk_node_key(a.traversal, ps, nbid);
                  keep = key < worst;
                }
              }
              const unsigned m = __ballot_sync(kFullMask, keep);
              if (m == 0u) continue;
              const int leader = __ffs(m) - 1;
              int xbase = 0;
              if (lane == leader) xbase = atomicAdd(&s_xc, __popc(m));
              xbase = __shfl_sync(kFullMask, xbase, leader);
              if (keep) X[xbase + __popc(m & ((1u << lane) - 1u))] = key;
            }
          }
        } else {
          for (int c = tid; c < wc; c += kDiskThreads) {
            const uint32_t nbid = WORK[c];
            float ps;
            if (disk_pq_score(a, table, qn, nbid, &ps)) {
              s_pq_fail = 1;
              continue;
            }
            const uint64_t key = disk_node_key(a.traversal, ps, nbid);
            if (key < worst) X[atomicAdd(&s_xc, 1)] = key;
          }
        }
        __syncthreads();
        if (s_pq_fail) {
          // A node's score fails wherever it is scored, so the sequential
          // loop fails at the node's first slot: the least failing slot
          // among those that saw it unvisited (lookups that can fail are
          // never `safe`, so FRESH is set).
          for (int sl = tid; sl < slots; sl += kDiskThreads) {
            if (!FRESH[sl]) continue;
            float ps;
            if (!disk_pq_score(a, table, qn, NB[sl], &ps)) continue;
            int lo = j0, hi = j1 - 1;
            while (lo < hi) {
              const int mid = (lo + hi + 1) >> 1;
              if (BDEG[mid] - base <= sl) lo = mid;
              else hi = mid - 1;
            }
            atomicMin(&s_err_pos, (unsigned)lo * stride + 1u + (unsigned)(sl + base - BDEG[lo]));
          }
          __syncthreads();  // NB is read here; the sorted candidates reuse it
        }
        int xc = s_xc;
        if (xc > 0) {
          const uint64_t* xs = X;
          if (xc > kDiskThreads && xc > a.cap) {
            // Only the step's `capacity` best can enter: keep the keys whose
            // rank is at most that of the capacity-th best (a radix select
            // on the rank bits), then order the few that remain.
            const uint64_t lim = smem_radix_select(X, xc, a.cap, 32, HIST) | 0xffffffffull;
            if (tid == 0) s_xn = 0;
            __syncthreads();
            for (int i0 = warp * 32; i0 < xc; i0 += kDiskThreads) {
              const int i = i0 + lane;
              const bool keep = i < xc && X[i] <= lim;
              const unsigned m = __ballot_sync(kFullMask, keep);
              if (m == 0u) continue;
              const int leader = __ffs(m) - 1;
              int base = 0;
              if (lane == leader) base = atomicAdd(&s_xn, __popc(m));
              base = __shfl_sync(kFullMask, base, leader);
              if (keep) X2[base + __popc(m & ((1u << lane) - 1u))] = X[i];
            }
            __syncthreads();
            xc = s_xn;
            if (xc <= kDiskThreads) {
              block_rank_sort(X2, xc, X);
            } else {
              block_sort_u64_fit<kDiskCand>(X2, xc);
              xs = X2;
            }
          } else if (xc <= kDiskThreads) {
            block_rank_sort(X, xc, X2);
            xs = X2;
          } else {
            block_sort_u64_fit<kDiskCand>(X, xc);
          }
          __syncthreads();
          const int rn = min(a.cap, rr + xc);
          merge_runs(R(rc), E(rc), rr, xs, xc, R(1 - rc), E(1 - rc), rn);
          __syncthreads();
          if (tid == 0) {
            s_r = rn;
            s_cur = 1 - rc;
          }
        }
        __syncthreads();
      }
      if (s_err_pos != kNoError) break;
      // The collector (:709-721): the round's accepted nodes merged into the
      // top-k.
      if (tid == 0) s_valid = 0;
      __syncthreads();
      if (tid < nb && BK[tid] != kEmptyKey) atomicAdd(&s_valid, 1);
      block_rank_sort(BK, nb, BK2);  // rejected nodes (kEmptyKey) rank last
      __syncthreads();
      const int valid = s_valid;
      const int kc = s_kc, kcur = s_kcur;
      if (valid > 0) {
        const int kn = min(a.k, kc + valid);
        merge_runs(K(kcur), nullptr, kc, BK2, valid, K(1 - kcur), nullptr, kn);
        __syncthreads();
        if (tid == 0) {
          s_kc = kn;
          s_kcur = 1 - kcur;
        }
      }
      __syncthreads();
    }
    // Results, best first, with the exact scores recomputed (their signs of
    // zero included), or the status of the first failure.
    if (tid == 0 && s_status == 0 && s_err_pos != kNoError)
      s_status = (s_err_pos % stride) == 0 ? XVEC_GPU_NON_FINITE : XVEC_GPU_OVERFLOW;
    __syncthreads();
    if (s_status != 0) {
      if (tid == 0) a.out_counts[q] = -s_status;
    } else {
      const int kc = s_kc;
      const uint64_t* kk = K(s_kcur);
      for (int i = warp; i < kc; i += kDiskWarps) {
        const uint32_t pos = a.pos_of_kr[(uint32_t)kk[i]];
        const float sc = warp_reference_score<float>(a.metric, a.rows + (int64_t)pos * a.d, qv, a.d);
        if (lane == 0) {
          a.out_keys[(int64_t)q * a.k + i] = a.keys[pos];
          a.out_scores[(int64_t)q * a.k + i] = sc;
        }
      }
      if (tid == 0) a.out_counts[q] = kc;
    }
    // Clear the visited bits for the slot's next query.
    const int vc = s_vcount;
    if (vc <= kDiskVisitCap) {
      for (int i = tid; i < vc; i += kDiskThreads) vis[vrec[i] >> 5] = 0u;
    } else {
      for (int64_t w = tid; w < a.words; w += kDiskThreads) vis[w] = 0u;
    }
    __syncthreads();
  }
}

// prepareDiskANNPQQuery (diskann.go:283-289: cosine queries normalised as
// normalizeRaBitQVector, rabitq.go:514-526) and diskANNVectorNormSquared
// (:678-683) of the prepared query; one block per query.
__global__ void diskann_prep_kernel(const float* qf, int nq, int d, int metric, float* q_prep,
                                    double* q_norm) {
  const int q = blockIdx.x;
  const float* src = qf + (int64_t)q * d;
  float* dst = q_prep + (int64_t)q * d;
  __shared__ float s_inv;
  __shared__ int s_scale;
  if (threadIdx.x == 0) {
    s_scale = 0;
    if (metric == kMetricCosine) {
      double ns = 0.0;
      for (int i = 0; i < d; ++i) ns = __dadd_rn(ns, __dmul_rn((double)src[i], (double)src[i]));
      if (ns != 0.0) {
        s_scale = 1;
        s_inv = __double2float_rn(__ddiv_rn(1.0, __dsqrt_rn(ns)));
      }
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < d; i += blockDim.x)
    dst[i] = s_scale ? __fmul_rn(src[i], s_inv) : src[i];
  __syncthreads();
  if (threadIdx.x == 0) {
    double norm = 0.0;
    for (int i = 0; i < d; ++i) norm = __dadd_rn(norm, __dmul_rn((double)dst[i], (double)dst[i]));
    q_norm[q] = norm;
  }
}

// The prepared rows of the build (cosine: normalised) for the PQ encoder.
__global__ void diskann_prepare_rows_kernel(const float* rows, int64_t n, int d, int metric,
                                            float* out) {
  const int64_t r = blockIdx.x;
  if (r >= n) return;
  const float* src = rows + r * d;
  float* dst = out + r * d;
  __shared__ float s_inv;
  __shared__ int s_scale;
  if (threadIdx.x == 0) {
    s_scale = 0;
    if (metric == kMetricCosine) {
      double ns = 0.0;
      for (int i = 0; i < d; ++i) ns = __dadd_rn(ns, __dmul_rn((double)src[i], (double)src[i]));
      if (ns != 0.0) {
        s_scale = 1;
        s_inv = __double2float_rn(__ddiv_rn(1.0, __dsqrt_rn(ns)));
      }
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < d; i += blockDim.x)
    dst[i] = s_scale ? __fmul_rn(src[i], s_inv) : src[i];
}

// diskANNPQCodeNorms (diskann.go:292-323): per code, the float64 sum of the
// squares of its pivots' chunk components, in chunk and component order.
__global__ void diskann_code_norms_kernel(const uint8_t* codes, int64_t n, int chunks,
                                          const float* pivots, const int* offsets, int d,
                                          float* norms) {
  const int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= n) return;
  double norm = 0.0;
  for (int c = 0; c < chunks; ++c) {
    const float* pv = pivots + (int64_t)codes[r * chunks + c] * d;
    for (int i = offsets[c]; i < offsets[c + 1]; ++i)
      norm = __dadd_rn(norm, __dmul_rn((double)pv[i], (double)pv[i]));
  }
  norms[r] = __double2float_rn(norm);
}

}  // namespace

// The traversal metric (diskANNTraversalMetric, diskann.go:276-281).
static int traversal_metric(int metric) {
  return (metric == kMetricCosine || metric == kMetricMIPS) ? kMetricL2 : metric;
}

xvec_gpu_status diskann_reserve(xvec_gpu_index* idx, int64_t cap, cudaStream_t s) {
  const int64_t n = idx->n;
  const size_t half = (size_t)idx->desc.dimension * 2;
  const int chunks = std::max(1, idx->chunks);
  xvec_gpu_status st;
  if ((st = idx->rows_bhi.reserve((size_t)cap * half, (size_t)n * half, s)) ||
      (st = idx->rows_blo.reserve((size_t)cap * half, (size_t)n * half, s)) ||
      (st = idx->pq_codes.reserve((size_t)cap * chunks, (size_t)n * chunks, s)) ||
      (st = idx->dk_norms.reserve((size_t)cap * 4, (size_t)n * 4, s)))
    return st;
  return XVEC_GPU_OK;
}

// New rows: the bfloat16 split of the linear scan, the PQ codes of the
// prepared rows under the traversal metric (diskann.go:224-237) and their
// MIPSL2 norms (:244-249).  The graph no longer covers the index.
xvec_gpu_status diskann_commit(xvec_gpu_index* idx, int64_t old_n, int64_t m, cudaStream_t s) {
  const int d = idx->desc.dimension, metric = idx->desc.metric, chunks = idx->chunks;
  const float* rows = idx->rows.as<float>() + old_n * d;
  XVEC_CUDA(launch_split_bf16(rows, m * d, idx->rows_bhi.as<__nv_bfloat16>() + old_n * d,
                              idx->rows_blo.as<__nv_bfloat16>() + old_n * d, s));
  XVEC_LAUNCHED();
  Scratch err, prep;
  xvec_gpu_status st;
  if ((st = err.alloc(4, s))) return st;
  XVEC_CUDA(cudaMemsetAsync(err.ptr, 0, 4, s));
  const int64_t step = std::max<int64_t>(1, std::min<int64_t>(m, (256ll << 20) / (4ll * d)));
  if (metric == kMetricCosine && (st = prep.alloc((size_t)step * d * 4, s))) return st;
  uint8_t* codes = idx->pq_codes.as<uint8_t>() + old_n * chunks;
  for (int64_t b = 0; b < m; b += step) {
    const int64_t c = std::min(step, m - b);
    const float* src = rows + b * d;
    if (metric == kMetricCosine) {
      diskann_prepare_rows_kernel<<<(unsigned)c, 128, 0, s>>>(src, c, d, metric, prep.as<float>());
      XVEC_LAUNCHED();
      src = prep.as<float>();
    }
    XVEC_CUDA(launch_pq_encode(src, c, d, traversal_metric(metric), idx->pivots.as<float>(),
                               idx->chunk_offsets.as<int>(), chunks, codes + b * chunks,
                               err.as<int>(), s));
  }
  if (metric == kMetricMIPS) {
    diskann_code_norms_kernel<<<blocks_of(m), 256, 0, s>>>(
        codes, m, chunks, idx->pivots.as<float>(), idx->chunk_offsets.as<int>(), d,
        idx->dk_norms.as<float>() + old_n);
    XVEC_LAUNCHED();
  }
  XVEC_CUDA(cudaGetLastError());
  int h = 0;
  XVEC_CUDA(cudaMemcpyAsync(&h, err.ptr, 4, cudaMemcpyDeviceToHost, s));
  XVEC_CUDA(cudaStreamSynchronize(s));
  if (h) return set_error("DiskANN PQ encoding produced a non-finite score"), (xvec_gpu_status)h;
  idx->dk_entry = -1;
  return XVEC_GPU_OK;
}

xvec_gpu_status diskann_search_impl(xvec_gpu_index* idx, const float* d_q, int nq,
                                    const xvec_gpu_search_opts& o, const uint32_t* d_bitmap,
                                    uint64_t* d_keys, float* d_scores, int* d_counts,
                                    cudaStream_t s, std::vector<int>* statuses) {
  EventTimer timer(s);
  timer.mark(0);
  const int d = idx->desc.dimension, metric = idx->desc.metric, k = o.top_k;
  const int64_t n = idx->n;
  const int list = o.ef == 0 ? kDefaultListSize : o.ef;
  if (!idx->has_model) return set_error("set the DiskANN PQ model first"), XVEC_GPU_INVALID_ARGUMENT;
  if (n > 0 && idx->dk_entry < 0)
    return set_error("the DiskANN graph does not cover the index: set it after adding rows"),
           XVEC_GPU_INVALID_ARGUMENT;
  const int cap = (int)std::min<int64_t>(std::max<int64_t>(n, 1), std::max(k, list));
  if (cap > kDiskMaxCap || k > kDiskMaxCap)
    return set_error("DiskANN capacity min(n, max(top_k, list size)) = %d and top_k %d must be "
                     "at most %d",
                     cap, k, kDiskMaxCap),
           XVEC_GPU_UNSUPPORTED;
  const int chunks = idx->chunks;
  xvec_gpu_status st;
  Scratch qf, qn2, qaux, qstatus, qflags, qprep, qnorm;
  if ((st = qf.alloc((size_t)nq * d * 4, s)) || (st = qn2.alloc((size_t)nq * 4, s)) ||
      (st = qaux.alloc((size_t)nq * 4, s)) || (st = qstatus.alloc((size_t)nq * 4, s)) ||
      (st = qflags.alloc((size_t)nq * 4, s)) || (st = qprep.alloc((size_t)nq * d * 4, s)) ||
      (st = qnorm.alloc((size_t)nq * 8, s)))
    return st;
  XVEC_CUDA(cudaMemsetAsync(qflags.ptr, 0, (size_t)nq * 4, s));
  XVEC_CUDA(cudaMemsetAsync(d_counts, 0, (size_t)nq * 4, s));
  launch_prep_queries<float>(d_q, nq, d, metric, qf.as<float>(), qn2.as<float>(), qaux.as<float>(),
                             qstatus.as<int>(), s);
  XVEC_LAUNCHED();
  diskann_prep_kernel<<<nq, 128, 0, s>>>(qf.as<float>(), nq, d, metric, qprep.as<float>(),
                                         qnorm.as<double>());
  XVEC_LAUNCHED();
  XVEC_CUDA(cudaGetLastError());
  // Queries in waves whose PQ tables fit 1 GiB.
  const int wave = (int)std::max<int64_t>(1, std::min<int64_t>(nq, (1ll << 30) / (1024ll * chunks)));
  Scratch table, visited, vrec;
  if ((st = table.alloc((size_t)wave * chunks * 1024, s))) return st;
  // The query's table in shared memory when it is at most 64 KB.
  const bool smem_table = chunks <= kDiskSmemChunks;
  auto kernel = smem_table ? diskann_search_kernel<true> : diskann_search_kernel<false>;
  const size_t smem = DiskSmem(cap, k, smem_table ? chunks * 256 : 0).total;
  XVEC_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  XVEC_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                                 cudaSharedmemCarveoutMaxShared));
  int per_sm = 0, sms = 0;
  XVEC_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, kDiskThreads, smem));
  XVEC_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, idx->device));
  const int64_t words = std::max<int64_t>(1, (n + 31) / 32);
  // Visited bitmaps of at most 1 GiB in total.
  const int slots = (int)std::max<int64_t>(
      1, std::min<int64_t>({(int64_t)wave, (int64_t)std::max(1, per_sm) * sms,
                            (1ll << 30) / (words * 4)}));
  if ((st = visited.alloc((size_t)slots * words * 4, s)) ||
      (st = vrec.alloc((size_t)slots * kDiskVisitCap * 4, s)))
    return st;
  XVEC_CUDA(cudaMemsetAsync(visited.ptr, 0, (size_t)slots * words * 4, s));
  DiskArgs a{};
  a.metric = metric;
  a.traversal = traversal_metric(metric);
  a.d = d;
  a.chunks = chunks;
  a.beam = idx->dk_beam;
  a.cap = cap;
  a.k = k;
  a.max_degree = idx->dk_max_degree;
  a.n = n;
  a.entry = idx->dk_entry < 0 ? 0 : idx->dk_entry;
  a.words = words;
  a.rows = idx->rows.as<float>();
  a.keyrank = idx->keyrank.as<uint32_t>();
  a.pos_of_kr = idx->pos_of_kr.as<uint32_t>();
  a.keys = idx->keys.as<uint64_t>();
  a.codes = idx->pq_codes.as<uint8_t>();
  a.code_norms = idx->dk_norms.as<float>();
  a.goff = idx->dk_offsets.as<int64_t>();
  a.nbrs = idx->dk_nbrs.as<int32_t>();
  a.radius = o.radius;
  a.bitmap = d_bitmap;
  a.visited = visited.as<uint32_t>();
  a.vrec = vrec.as<uint32_t>();
  timer.mark(1);
  for (int q0 = 0; q0 < nq; q0 += wave) {
    if (is_cancelled(o)) return set_error("cancelled"), XVEC_GPU_CANCELLED;
    const int w = std::min(wave, nq - q0);
    XVEC_CUDA(launch_pq_table(qprep.as<float>() + (int64_t)q0 * d, w, d, a.traversal,
                              idx->pivots.as<float>(), idx->chunk_offsets.as<int>(), chunks,
                              table.as<float>(), qflags.as<int>() + q0, s));
    a.nq = w;
    a.qf = qf.as<float>() + (int64_t)q0 * d;
    a.table = table.as<float>();
    a.qnorm = qnorm.as<double>() + q0;
    a.q_status = qstatus.as<int>() + q0;
    a.q_flags = qflags.as<int>() + q0;
    a.out_keys = d_keys + (int64_t)q0 * k;
    a.out_scores = d_scores + (int64_t)q0 * k;
    a.out_counts = d_counts + q0;
    kernel<<<std::min(slots, w), kDiskThreads, smem, s>>>(a, cap);
    XVEC_LAUNCHED();
    XVEC_CUDA(cudaGetLastError());
  }
  timer.mark(2);
  std::vector<int> h_counts(nq);
  XVEC_CUDA(cudaMemcpyAsync(h_counts.data(), d_counts, (size_t)nq * 4, cudaMemcpyDeviceToHost, s));
  timer.mark(3);
  XVEC_CUDA(cudaStreamSynchronize(s));
  count_search(nq, 0, timer.ms(1, 2), timer.ms(0, 3));
  if (statuses) {
    statuses->resize(nq);
    for (int q = 0; q < nq; ++q) (*statuses)[q] = h_counts[q] < 0 ? -h_counts[q] : 0;
  }
  return XVEC_GPU_OK;
}

}  // namespace xvec

using namespace xvec;

extern "C" xvec_gpu_status xvec_gpu_diskann_set_model(xvec_gpu_index* idx, const float* pivots,
                                                      int32_t chunks) {
  if (!idx || !pivots) return set_error("nil argument"), XVEC_GPU_INVALID_ARGUMENT;
  if (idx->desc.kind != XVEC_INDEX_DISKANN)
    return set_error("not a DiskANN index"), XVEC_GPU_INVALID_ARGUMENT;
  const int d = idx->desc.dimension;
  if (chunks <= 0 || chunks > d)
    return set_error("core: invalid PQ options: resolved Chunks must be in [1,%d]", d),
           XVEC_GPU_INVALID_ARGUMENT;
  std::unique_lock<std::shared_mutex> lock(idx->mu);
  if (idx->n > 0) return set_error("set the model before adding rows"), XVEC_GPU_INVALID_ARGUMENT;
  for (int64_t i = 0; i < (int64_t)256 * d; ++i)
    if (!std::isfinite(pivots[i])) return set_error("non-finite PQ pivot"), XVEC_GPU_NON_FINITE;
  cudaSetDevice(idx->device);
  // pqChunkOffsets (pq.go:395-406): contiguous chunks, wider chunks first.
  std::vector<int> offsets(chunks + 1, 0);
  const int base = d / chunks, larger = d % chunks;
  for (int c = 0; c < chunks; ++c) offsets[c + 1] = offsets[c] + base + (c < larger ? 1 : 0);
  xvec_gpu_status st;
  if ((st = idx->pivots.reserve((size_t)256 * d * 4, 0, nullptr)) ||
      (st = idx->chunk_offsets.reserve((size_t)(chunks + 1) * 4, 0, nullptr)))
    return st;
  XVEC_CUDA(cudaMemcpy(idx->pivots.ptr, pivots, (size_t)256 * d * 4, cudaMemcpyHostToDevice));
  XVEC_CUDA(cudaMemcpy(idx->chunk_offsets.ptr, offsets.data(), (size_t)(chunks + 1) * 4,
                       cudaMemcpyHostToDevice));
  idx->chunks = chunks;
  idx->has_model = true;
  // The per-row code buffers follow the chunk count.
  if (idx->capacity > 0 && (st = diskann_reserve(idx, idx->capacity, nullptr))) return st;
  XVEC_CUDA(cudaDeviceSynchronize());
  return XVEC_GPU_OK;
}

extern "C" xvec_gpu_status xvec_gpu_diskann_set_graph(xvec_gpu_index* idx, int64_t entry,
                                                      int32_t max_degree, const int64_t* offsets,
                                                      const int32_t* neighbors,
                                                      int64_t total_neighbors) {
  if (!idx) return set_error("nil index"), XVEC_GPU_INVALID_ARGUMENT;
  if (idx->desc.kind != XVEC_INDEX_DISKANN)
    return set_error("a DiskANN graph belongs to a DiskANN index"), XVEC_GPU_INVALID_ARGUMENT;
  std::unique_lock<std::shared_mutex> lock(idx->mu);
  const int64_t n = idx->n;
  if (!offsets) {
    idx->dk_entry = -1;
    return XVEC_GPU_OK;
  }
  if (max_degree <= 0 || max_degree > kDiskCand)
    return set_error("DiskANN MaxDegree %d outside [1, %d]", max_degree, kDiskCand),
           XVEC_GPU_INVALID_ARGUMENT;
  if (n == 0 || entry < 0 || entry >= n)
    return set_error("DiskANN entry point %lld outside [0, %lld)", (long long)entry,
                     (long long)n),
           XVEC_GPU_INVALID_ARGUMENT;
  if (offsets[0] != 0 || offsets[n] != total_neighbors || (total_neighbors > 0 && !neighbors))
    return set_error("DiskANN graph offsets must run from 0 to the neighbour count"),
           XVEC_GPU_INVALID_ARGUMENT;
  for (int64_t p = 0; p < n; ++p) {
    const int64_t dg = offsets[p + 1] - offsets[p];
    if (dg < 0 || dg > max_degree)
      return set_error("node %lld has %lld neighbours (MaxDegree %d)", (long long)p,
                       (long long)dg, max_degree),
             XVEC_GPU_INVALID_ARGUMENT;
  }
  for (int64_t e = 0; e < total_neighbors; ++e)
    if (neighbors[e] < 0 || neighbors[e] >= n)
      return set_error("neighbour %lld is outside [0, %lld)", (long long)neighbors[e],
                       (long long)n),
             XVEC_GPU_INVALID_ARGUMENT;
  cudaSetDevice(idx->device);
  xvec_gpu_status st;
  if ((st = idx->dk_offsets.reserve((size_t)(n + 1) * 8, 0, nullptr)) ||
      (st = idx->dk_nbrs.reserve((size_t)std::max<int64_t>(1, total_neighbors) * 4, 0, nullptr)))
    return st;
  XVEC_CUDA(cudaMemcpy(idx->dk_offsets.ptr, offsets, (size_t)(n + 1) * 8, cudaMemcpyHostToDevice));
  if (total_neighbors > 0)
    XVEC_CUDA(cudaMemcpy(idx->dk_nbrs.ptr, neighbors, (size_t)total_neighbors * 4,
                         cudaMemcpyHostToDevice));
  // diskANNReadBatchSize (diskann.go:685-691) of the node layout
  // (NewDiskANNLayout, diskann_storage.go:61-100): a record of 4 d + 4 + 4
  // MaxDegree + 4 bytes takes one 4096-byte sector, or ceil(record / 4096)
  // sectors when larger; a read takes 128 sectors.
  const int64_t record = 4ll * idx->desc.dimension + 4 + 4ll * max_degree + 4;
  const int64_t sectors = record <= 4096 ? 1 : (record + 4095) / 4096;
  idx->dk_beam = (int)std::max<int64_t>(1, kDiskMaxBeam / sectors);
  idx->dk_max_degree = max_degree;
  idx->dk_entry = entry;
  return XVEC_GPU_OK;
}
