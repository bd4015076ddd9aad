// flat_tc.cu — tensor-core candidate scan for Flat search over binary16 rows.
//
// The fast-rank stage of Flat search (flat_kernels.cu) for FP16 storage on
// sm_100a: the query x row dot products are a GEMM, computed by tcgen05.mma
// (kind::f16, fp32 accumulation in tensor memory) on tiles staged by TMA,
// with the per-query candidate selection fused into the epilogue, so the
// score matrix is never written to memory.
//
//   CTA = 10 warps, one CTA per SM (tensor memory and shared memory sized so):
//     warp 0    TMA producer: this CTA's query tile A[128 x 64] and row tile
//               B[RB x 64] per k-step into a ring of stages (128-byte swizzle).
//     warp 1    allocates 512 TMEM columns, issues the MMAs (one thread):
//               D[queries x 256 rows] fp32, two accumulators in TMEM so the
//               epilogue of tile t overlaps the MMAs of tile t+1.
//     warps 2-9 epilogue: each thread owns one query (one TMEM lane) and one
//               column half, loads 128 dot products per tile with tcgen05.ld,
//               turns them into fast ranks and appends the ones below its
//               threshold to the query's candidate list (global memory); a
//               full list is compacted to its KP best keys by the warp.
//   Single CTA (PAIR = false): M = 128 queries, RB = 256 rows per CTA.
//   CTA pair   (PAIR = true, cluster of 2, tcgen05 cta_group::2): M = 256
//               queries (128 per CTA), N = 256 rows of which each CTA loads
//               128, so a CTA moves 32 KB instead of 48 KB of operands per
//               k-step.  Both CTAs' copies of a stage complete on the first
//               CTA's barrier, armed there for both halves; its single
//               thread issues the pair's MMAs and signals both CTAs' stage
//               and accumulator barriers.  At the end the second CTA
//               publishes how many copies it issued per stage, and the first
//               waits for every one of them before either CTA leaves.
//   Grid = (query blocks of 128, row chunks); blockIdx.x varies fastest so
//   the CTAs resident at any time share row chunks and the rows come from L2.
//
// Every mbarrier wait is bounded: on expiry the kernel records an error in
// `status`, stops issuing work, drains its own copies and still releases its
// tensor memory.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <atomic>

#include "capi_internal.h"
#include "common.cuh"
#include "flat_tc.cuh"
#include "select.cuh"

namespace xvec {

namespace tc {

constexpr int kBM = 128;   // queries per CTA (TMEM lanes)
constexpr int kBN = 256;   // rows per tile (TMEM columns per accumulator)
constexpr int kBK = 64;    // k-step: 64 fp16 = 128 bytes (one swizzle row)
constexpr int kCap = 512;  // candidate list entries per (query, part, column half)
constexpr int kEpiWarps = 8;  // two warps per TMEM lane quarter, one per column half
constexpr int kThreads = 64 + kEpiWarps * 32;
constexpr uint32_t kTileABytes = kBM * kBK * 2;  // 16 KB
// Kernel modes: a Flat metric (FP16 operands, fp32 accumulators);
// kModeSq8 + metric (INT8 codes, kind::i8, exact int32 accumulators);
// kModeRaBitQ (kind::i8 on the code planes [127 b | b] against each query as
// integers [h | l], 127 h + l = the query / its scale: one exact int32
// accumulator).
// kModeSplit + metric (float32 rows and queries as bfloat16 high + low
// parts: hi·hi + hi·lo + lo·hi, three MMAs per k-step into one fp32
// accumulator).
constexpr int kModeSq8 = 16;
constexpr int kModeRaBitQ = 32;
constexpr int kModeSplit = 64;
// kModeRaBitQ8: multi-bit RaBitQ on kind::i8, the rows' code values as the
// int8 plane v - 128 against the query as 16-bit integers w = round(q / s)
// split into two int8 planes, w = 256 h + l + 128 (h, l signed): two MMAs per
// k-step into two exact int32 accumulators of 128 columns (A_h, A_l), tiles
// of 128 rows; the epilogue forms sum(v w) = 256 A_h + A_l + 128 sum(v - 128)
// (a per-row term) + 128 sum(w) (folded into the query's terms).
constexpr int kModeRaBitQ8 = 256;
constexpr int kRaBitQMaxClusters = 16;
// Per epilogue warp: radix histogram (1 KB) + the current tile's row
// metadata for its 128 columns (aux floats + key ranks, 1 KB; SQ8/RaBitQ: the
// rows' float4 rank terms, 2 KB; RaBitQ: the 32 queries' per-cluster terms,
// 2 KB).
constexpr uint32_t epi_smem_bytes(bool rq) {
  return kEpiWarps * (256 * 4 * 2 + 128 * 16 + (rq ? kRaBitQMaxClusters * 32 * 4 : 0));
}
constexpr uint32_t kSmemBudget = 232448 - 1024 - 1024 - 512;  // dynamic bytes for stages

template <bool PAIR, bool RQ = false, bool SPLIT = false, bool SPLITA = false, int BN = kBN>
struct Shape {
  static constexpr int kRowsPerCta = PAIR ? BN / 2 : BN;          // B rows loaded per CTA
  static constexpr uint32_t kTileBBytes = kRowsPerCta * kBK * 2;  // 8, 16 or 32 KB
  static constexpr int kParts = SPLIT ? 2 : 1;                    // high (+ low) tiles
  // SPLITA: A high, B, A low.
  static constexpr uint32_t kStageBytes =
      SPLITA ? 2 * kTileABytes + kTileBBytes : kParts * (kTileABytes + kTileBBytes);
  static constexpr uint32_t kEpiBytes = epi_smem_bytes(RQ);
  static constexpr int kFit = (int)((kSmemBudget - kEpiBytes) / kStageBytes);
  static constexpr int kStages = kFit < 6 ? kFit : 6;
  static constexpr uint32_t kSmemBytes = kStages * kStageBytes + kEpiBytes + 1024 + 512;
  static_assert(kStages >= 2, "shared memory too small for the stage ring");
};
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // a wait gives up after 2 s (default)

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
// Address of the same shared variable in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t cluster_addr(const void* p, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
  return r;
}
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// Arrive with cluster-scope release (orders this thread's earlier
// observations for the other CTA).
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_bar) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_bar)
               : "memory");
}
// Plain arrive (release at CTA scope) on a barrier of another CTA: orders
// this thread's tensor-memory reads, not its global stores.
__device__ __forceinline__ void mbar_arrive_remote(uint32_t cluster_bar) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(cluster_bar) : "memory");
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n"
               "barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Bounded parity wait: false once limit_ns passed or another role of the
// CTA raised *abort.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity,
                                          const volatile int* abort,
                                          uint64_t limit_ns = kWaitLimitNs) {
  const uint32_t addr = smem_u32(bar);
  uint64_t start = 0;
  for (uint32_t i = 0;; ++i) {
    uint32_t done;
    asm volatile(
        "{\n.reg .pred p;\n"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n"
        "selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(done)
        : "r"(addr), "r"(parity)
        : "memory");
    if (done) return true;
    if ((i & 255) == 0) {
      if (abort && *abort) return false;
      const uint64_t now = global_ns();
      if (start == 0) start = now;
      else if (now - start > limit_ns) return false;
    }
  }
}

__device__ __forceinline__ void tma_load_2d(const CUtensorMap* map, uint64_t* bar, void* dst,
                                            int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(dst)),
      "l"((uint64_t)map), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

// Pair form: the copy lands in this CTA's shared memory and completes on the
// barrier at `cluster_bar`, which may belong to the other CTA of the pair.
__device__ __forceinline__ void tma_load_2d_pair(const CUtensorMap* map, uint32_t cluster_bar,
                                                 void* dst, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(dst)),
      "l"((uint64_t)map), "r"(x), "r"(y), "r"(cluster_bar)
      : "memory");
}
__device__ __forceinline__ uint32_t ld_cluster_u32(uint32_t cluster_addr) {
  uint32_t v;
  asm volatile("ld.shared::cluster.u32 %0, [%1];" : "=r"(v) : "r"(cluster_addr) : "memory");
  return v;
}

// UMMA shared-memory descriptor: K-major, 128-byte swizzle, 8-row groups
// 1024 bytes apart (SBO), descriptor version 1 (sm_100).
__device__ __forceinline__ uint64_t smem_desc_sw128(const void* tile) {
  const uint64_t addr = smem_u32(tile);
  return ((addr & 0x3FFFFull) >> 4) | (1ull << 16) | ((1024ull >> 4) << 32) | (1ull << 46) |
         (2ull << 61);
}

// Instruction descriptor: kind::f16, A/B = F16, D = F32, both K-major, N = 256.
template <int M>
constexpr uint32_t idesc_f16() {
  return (1u << 4) | ((uint32_t)(kBN >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// kind::f16 with A/B = BF16, D = F32.
template <int M>
constexpr uint32_t idesc_bf16() {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(kBN >> 3) << 17) |
         ((uint32_t)(M >> 4) << 24);
}
template <bool PAIR>
__device__ __forceinline__ void mma_bf16(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t acc) {
  if constexpr (PAIR) {
    asm volatile(
        "{\n.reg .pred p;\nsetp.ne.b32 p, %4, 0;\n"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
        "l"(a), "l"(b), "r"(idesc_bf16<2 * kBM>()), "r"(acc));
  } else {
    asm volatile(
        "{\n.reg .pred p;\nsetp.ne.b32 p, %4, 0;\n"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
        "l"(a), "l"(b), "r"(idesc_bf16<kBM>()), "r"(acc));
  }
}

// kind::i8: A/B signed 8-bit, D = S32, N columns.
template <int M, int N = kBN>
constexpr uint32_t idesc_s8() {
  return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) |
         ((uint32_t)(M >> 4) << 24);
}
template <bool PAIR, int N = kBN>
__device__ __forceinline__ void mma_s8(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t acc) {
  if constexpr (PAIR) {
    asm volatile(
        "{\n.reg .pred p;\nsetp.ne.b32 p, %4, 0;\n"
        "tcgen05.mma.cta_group::2.kind::i8 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
        "l"(a), "l"(b), "r"(idesc_s8<2 * kBM, N>()), "r"(acc));
  } else {
    asm volatile(
        "{\n.reg .pred p;\nsetp.ne.b32 p, %4, 0;\n"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
        "l"(a), "l"(b), "r"(idesc_s8<kBM, N>()), "r"(acc));
  }
}

template <bool PAIR>
__device__ __forceinline__ void mma_f16(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t acc) {
  if constexpr (PAIR) {
    asm volatile(
        "{\n.reg .pred p;\nsetp.ne.b32 p, %4, 0;\n"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
        "l"(a), "l"(b), "r"(idesc_f16<2 * kBM>()), "r"(acc));
  } else {
    asm volatile(
        "{\n.reg .pred p;\nsetp.ne.b32 p, %4, 0;\n"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
        "l"(a), "l"(b), "r"(idesc_f16<kBM>()), "r"(acc));
  }
}
// Arrives on the barrier at a shared::cluster address once every MMA this
// thread issued so far has completed.
template <bool PAIR>
__device__ __forceinline__ void mma_commit(uint32_t cluster_bar) {
  if constexpr (PAIR)
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     cluster_bar)
                 : "memory");
  else
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     cluster_bar)
                 : "memory");
}
__device__ __forceinline__ void tmem_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tmem_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,"
      "%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
        "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]),
        "=r"(v[14]), "=r"(v[15]), "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]),
        "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]), "=r"(v[25]),
        "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// v[j] for a warp-uniform j: a tree of selects on the bits of j, so the
// array stays in registers (a run-time index would move it to local memory).
__device__ __forceinline__ uint32_t pick32(const uint32_t (&v)[32], int j) {
  uint32_t a[16], b[8], c[4], d[2];
#pragma unroll
  for (int i = 0; i < 16; ++i) a[i] = (j & 16) ? v[i + 16] : v[i];
#pragma unroll
  for (int i = 0; i < 8; ++i) b[i] = (j & 8) ? a[i + 8] : a[i];
#pragma unroll
  for (int i = 0; i < 4; ++i) c[i] = (j & 4) ? b[i + 4] : b[i];
#pragma unroll
  for (int i = 0; i < 2; ++i) d[i] = (j & 2) ? c[i + 2] : c[i];
  return (j & 1) ? d[1] : d[0];
}

// Fast rank from the tensor-core dot product.  aux: 1/||x|| (cosine) or
// ||x||^2 (L2, MIPS); qa: 1/||q|| (cosine) or ||q||^2.
template <int METRIC>
__device__ __forceinline__ float tc_rank(float dot, float aux, float qa, float qn2) {
  if (METRIC == kMetricIP) return -dot;
  if (METRIC == kMetricL2) return (aux + qa) - 2.f * dot;
  if (METRIC == kMetricCosine) {
    if (aux == 0.f) return qn2 == 0.f ? 0.f : 1.f;
    return fmaf(-dot * aux, qa, 1.f);
  }
  const float den = fmaxf(aux, qa);
  if (den == 0.f) return 0.f;
  return 2.f - 2.f * dot / den;
}

// The common path tests a per-row "score" s against a per-query bound Tq
// derived from the list threshold T (rank domain): s >= Tq must hold for
// every row whose fast rank is <= T.  Tq is lowered by a relative slack so
// rounding can only send extra rows to the exact check of the rare path.
//   IP:     s = dot,             rank = -dot            -> Tq = -T
//   cosine: s = dot * (1/|x|),   rank = 1 - s/|q|       -> Tq = (1 - T) |q|
//   L2:     s = dot - |x|^2/2,   rank = |x|^2+|q|^2-2dot -> Tq = (|q|^2 - T) / 2
//   MIPS:   s = -rank                                   -> Tq = -T
template <int METRIC>
__device__ __forceinline__ float score_bound(float T, float qa, float qn2) {
  if (!(T == T)) return -INFINITY;  // list not full yet: take everything
  float b;
  if (METRIC == kMetricIP || METRIC == kMetricMIPS) {
    b = -T;
  } else if (METRIC == kMetricCosine) {
    if (qa == 0.f) return -INFINITY;  // zero query: ranks are 0/1, check exactly
    b = (1.f - T) / qa;
  } else {
    b = 0.5f * (qn2 - T);
  }
  return b - fabsf(b) * 6.1035156e-5f - 1e-30f;  // 2^-14 relative slack
}

// Keeps the kp smallest keys of a candidate list (global memory, unsorted)
// and returns the kp-th smallest.  The warp loads the list once into
// registers (kCap/32 keys per lane, all loads in flight together), runs a
// radix select over the 64-bit keys (8 passes of 8 bits, histogram in
// shared memory) and writes the kept keys back in order.  Keys are unique,
// so exactly kp remain.
__device__ __forceinline__ uint64_t warp_select_compact(uint64_t* gbuf, int cnt, int kp,
                                                     int* hist) {
  constexpr int kPer = kCap / 32;
  const int lane = threadIdx.x & 31;
  __syncwarp();  // the owning lane's appends are visible to the warp
  uint64_t keys[kPer];
#pragma unroll
  for (int e = 0; e < kPer; ++e) {
    const int i = e * 32 + lane;
    keys[e] = i < cnt ? gbuf[i] : kEmptyKey;
  }
  uint64_t prefix = 0;
  int kth = kp;
#pragma unroll 1
  for (int shift = 56; shift >= 0; shift -= 8) {
    for (int b = lane; b < 256; b += 32) hist[b] = 0;
    __syncwarp();
    const uint64_t mask = shift == 56 ? 0ull : (~0ull << (shift + 8));
#pragma unroll
    for (int e = 0; e < kPer; ++e)
      if (e * 32 + lane < cnt && (keys[e] & mask) == prefix)
        atomicAdd(&hist[(keys[e] >> shift) & 0xff], 1);
    __syncwarp();
    // Lane l owns bins 8l..8l+7: find the bin where the running count
    // reaches kth.
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
        rem = -rem;  // found: stop matching further bins
      } else if (rem > 0) {
        rem -= local[b];
      }
    }
    digit = __shfl_sync(kFullMask, digit, src);
    kth = -__shfl_sync(kFullMask, rem, src);
    prefix |= (uint64_t)digit << shift;
    __syncwarp();
  }
  // prefix is the kp-th smallest key; keep every key <= prefix, in order of
  // their slots.
  int out = 0;
#pragma unroll
  for (int e = 0; e < kPer; ++e) {
    const bool keep = e * 32 + lane < cnt && keys[e] <= prefix;
    const unsigned m = __ballot_sync(kFullMask, keep);
    if (keep) gbuf[out + __popc(m & ((1u << lane) - 1))] = keys[e];
    out += __popc(m);
  }
  __syncwarp();
  return prefix;
}

template <int MODE, bool PAIR>
__global__ void __launch_bounds__(kThreads, 1) flat_scan_tc_kernel(
    const __grid_constant__ CUtensorMap qmap, const __grid_constant__ CUtensorMap rmap,
    const __grid_constant__ CUtensorMap qmap2, const __grid_constant__ CUtensorMap rmap2, int nc,
    int nq,
    int64_t n, int d, const float* __restrict__ row_aux, const uint32_t* __restrict__ keyrank,
    const float* __restrict__ q_aux, const float* __restrict__ q_n2,
    unsigned long long* __restrict__ gthr, const uint32_t* __restrict__ bitmap,
    int64_t rows_per_part, int kp, int list_base, int num_lists, uint64_t* __restrict__ cand,
    int* __restrict__ part_counts, uint64_t* __restrict__ part_sat, int* __restrict__ q_flags,
    int* __restrict__ status, uint64_t wait_ns) {
  constexpr bool RQ1 = MODE == kModeRaBitQ;   // RaBitQ code planes, integer queries
  constexpr bool RQ8 = MODE == kModeRaBitQ8;     // multi-bit values, 16-bit integer query
  constexpr bool RQ = RQ1 || RQ8;                // the RaBitQ epilogue
  constexpr bool SQ = (MODE & kModeSq8) != 0 && !RQ8;  // INT8 codes (SQ8) instead of FP16 rows
  constexpr bool SPLIT = (MODE & kModeSplit) != 0 && !RQ8;  // bfloat16 high/low parts of float32
  constexpr bool I8 = SQ || RQ1 || RQ8;         // kind::i8 operands
  constexpr bool TWO_A = RQ8;                   // stage: A, B, second A
  constexpr int METRIC = RQ8 ? 0 : (MODE & 15);
  constexpr int kElemBytes = I8 ? 1 : 2;
  // Rows per tile: RQ8 keeps two accumulators of BN columns per buffer.
  constexpr int BN = RQ8 ? kBN / 2 : kBN;
  constexpr int kHalfCols = BN / 2;         // columns per epilogue warp
  constexpr int kChunks = kHalfCols / 32;   // 32-column chunks per epilogue warp
  using S = Shape<PAIR, RQ, SPLIT, TWO_A, BN>;
  constexpr int kStages = S::kStages;
  constexpr uint32_t kStageBytes = S::kStageBytes;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = (unsigned char*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  unsigned char* tiles = smem;  // kStages x (A | B)
  int* hist_all = reinterpret_cast<int*>(smem + kStages * kStageBytes);  // kEpiWarps x 256
  uint32_t* meta_all = reinterpret_cast<uint32_t*>(hist_all + kEpiWarps * 256);  // x 256
  float4* meta4_all = reinterpret_cast<float4*>(meta_all + kEpiWarps * 256);  // x 128
  float* gadd_all = reinterpret_cast<float*>(meta4_all + kEpiWarps * 128);    // RaBitQ
  uint64_t* bars = reinterpret_cast<uint64_t*>(reinterpret_cast<unsigned char*>(meta4_all) +
                                               kEpiWarps * 128 * 16 +
                                               (RQ ? kEpiWarps * kRaBitQMaxClusters * 32 * 4 : 0));
  uint64_t* full = bars;                      // [kStages] the stage's copies landed (pair:
                                              // both CTAs' copies, on the first CTA)
  uint32_t* issued = reinterpret_cast<uint32_t*>(bars + kStages);  // [kStages] copies per stage
  uint64_t* empty = bars + 2 * kStages;       // [kStages] the MMAs have read the stage
  uint64_t* tfull = bars + 3 * kStages;       // [2] accumulator ready
  uint64_t* tempty = bars + 3 * kStages + 2;  // [2] accumulator drained (issuing CTA's count)
  uint64_t* mdone = bars + 3 * kStages + 4;   // all issued MMAs retired
  uint32_t* tmem_base_slot = reinterpret_cast<uint32_t*>(bars + 3 * kStages + 5);
  __shared__ int s_abort_storage;
  volatile int* s_abort = &s_abort_storage;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qblock = blockIdx.x;
  const int part = blockIdx.y;
  const int64_t row_begin = (int64_t)part * rows_per_part;
  const int64_t row_end = min(n, row_begin + rows_per_part);
  const int num_tiles = row_end > row_begin ? (int)((row_end - row_begin + BN - 1) / BN) : 0;
  // k-steps of 128 bytes (kBK FP16 or 2 kBK INT8 elements).
  const int ksteps = (d * kElemBytes + 127) / 128;
  constexpr int kStepElems = 128 / kElemBytes;
  const uint32_t rank = PAIR ? cluster_rank() : 0u;
  const bool issuer = rank == 0;  // the CTA whose thread issues the MMAs

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
      issued[s] = 0;
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], (PAIR ? 2 : 1) * kEpiWarps);
    }
    mbar_init(mdone, 1);
    *s_abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    if constexpr (PAIR) {
      asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(
                       smem_u32(tmem_base_slot)));
      asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
    } else {
      asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(
                       smem_u32(tmem_base_slot)));
      asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tmem_fence_before();
  }
  __syncthreads();
  // Both CTAs' barriers exist before either signals the other.
  if constexpr (PAIR) cluster_sync_all();
  tmem_fence_after();
  const uint32_t tmem_base = *tmem_base_slot;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      const uint32_t full0 = PAIR ? cluster_addr(&full[0], 0) : smem_u32(&full[0]);
      int stage = 0;
      uint32_t phase = 0;
      uint32_t count[kStages];
#pragma unroll
      for (int s2 = 0; s2 < kStages; ++s2) count[s2] = 0;
      for (int t = 0; t < num_tiles && !*s_abort; ++t) {
        const int row0 = (int)(row_begin + (int64_t)t * BN) + (int)rank * S::kRowsPerCta;
        for (int ks = 0; ks < ksteps; ++ks) {
          if (!mbar_wait(&empty[stage], phase ^ 1, s_abort, wait_ns)) {
            atomicExch(status, 1);
            *s_abort = 1;
            break;
          }
          // Stage layout: A (high), B (high)[, A (low), B (low)].
          unsigned char* a_dst = tiles + stage * kStageBytes;
          unsigned char* b_dst = a_dst + kTileABytes;
          unsigned char* a2_dst = b_dst + S::kTileBBytes;
          unsigned char* b2_dst = a2_dst + kTileABytes;
          if (issuer) mbar_expect_tx(&full[stage], (PAIR ? 2 : 1) * kStageBytes);
          if constexpr (PAIR) {
            tma_load_2d_pair(&qmap, full0 + stage * 8, a_dst, ks * kStepElems, qblock * kBM);
            tma_load_2d_pair(&rmap, full0 + stage * 8, b_dst, ks * kStepElems, row0);
            if constexpr (SPLIT) {
              tma_load_2d_pair(&qmap2, full0 + stage * 8, a2_dst, ks * kStepElems, qblock * kBM);
              tma_load_2d_pair(&rmap2, full0 + stage * 8, b2_dst, ks * kStepElems, row0);
            }
            if constexpr (TWO_A)
              tma_load_2d_pair(&qmap2, full0 + stage * 8, a2_dst, ks * kStepElems, qblock * kBM);
          } else {
            tma_load_2d(&qmap, &full[stage], a_dst, ks * kStepElems, qblock * kBM);
            tma_load_2d(&rmap, &full[stage], b_dst, ks * kStepElems, row0);
            if constexpr (SPLIT) {
              tma_load_2d(&qmap2, &full[stage], a2_dst, ks * kStepElems, qblock * kBM);
              tma_load_2d(&rmap2, &full[stage], b2_dst, ks * kStepElems, row0);
            }
            if constexpr (TWO_A)
              tma_load_2d(&qmap2, &full[stage], a2_dst, ks * kStepElems, qblock * kBM);
          }
          ++count[stage];
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
#pragma unroll
      for (int s2 = 0; s2 < kStages; ++s2) issued[s2] = count[s2];
    }
  } else if (warp == 1 && !issuer) {
    // Second CTA of a pair: its tensor memory is written by the first CTA.
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      const uint32_t own_empty0 = smem_u32(&empty[0]), own_tfull0 = smem_u32(&tfull[0]);
      const uint32_t peer_empty0 = PAIR ? cluster_addr(&empty[0], 1) : 0u;
      const uint32_t peer_tfull0 = PAIR ? cluster_addr(&tfull[0], 1) : 0u;
      int stage = 0;
      uint32_t phase = 0;
      for (int t = 0; t < num_tiles && !*s_abort; ++t) {
        const int acc = t & 1;
        const uint32_t acc_phase = (t >> 1) & 1;
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1, s_abort, wait_ns)) {
          atomicExch(status, 2);
          *s_abort = 1;
          break;
        }
        tmem_fence_after();
        const uint32_t d_tmem = tmem_base + acc * kBN;
        for (int ks = 0; ks < ksteps; ++ks) {
          if (!mbar_wait(&full[stage], phase, s_abort, wait_ns)) {
            atomicExch(status, 3);
            *s_abort = 1;
            break;
          }
          tmem_fence_after();
          const unsigned char* a_src = tiles + stage * kStageBytes;
          const uint64_t adesc = smem_desc_sw128(a_src);
          const uint64_t bdesc = smem_desc_sw128(a_src + kTileABytes);
#pragma unroll
          for (int k = 0; k < 4; ++k) {  // 32 bytes of K per MMA (16 FP16 or 32 INT8)
            if constexpr (RQ8)
              mma_s8<PAIR, BN>(d_tmem, adesc + (uint64_t)(k * 2), bdesc + (uint64_t)(k * 2),
                               (ks > 0 || k > 0) ? 1u : 0u);
            else if constexpr (I8)
              mma_s8<PAIR>(d_tmem, adesc + (uint64_t)(k * 2), bdesc + (uint64_t)(k * 2),
                           (ks > 0 || k > 0) ? 1u : 0u);
            else if constexpr (SPLIT)
              mma_bf16<PAIR>(d_tmem, adesc + (uint64_t)(k * 2), bdesc + (uint64_t)(k * 2),
                             (ks > 0 || k > 0) ? 1u : 0u);
            else
              mma_f16<PAIR>(d_tmem, adesc + (uint64_t)(k * 2), bdesc + (uint64_t)(k * 2),
                            (ks > 0 || k > 0) ? 1u : 0u);
          }
          if constexpr (RQ8) {
            // The low query plane against the same rows, into the second
            // accumulator (BN columns further).
            const uint64_t a2desc = smem_desc_sw128(a_src + kTileABytes + S::kTileBBytes);
#pragma unroll
            for (int k = 0; k < 4; ++k)
              mma_s8<PAIR, BN>(d_tmem + BN, a2desc + (uint64_t)(k * 2), bdesc + (uint64_t)(k * 2),
                               (ks > 0 || k > 0) ? 1u : 0u);
          }
          if constexpr (SPLIT) {
            // The high query part against the low row part, and the low
            // query part against the high row part.
            const uint64_t a2desc = smem_desc_sw128(a_src + kTileABytes + S::kTileBBytes);
            const uint64_t b2desc =
                smem_desc_sw128(a_src + 2 * kTileABytes + S::kTileBBytes);
#pragma unroll
            for (int k = 0; k < 4; ++k)
              mma_bf16<PAIR>(d_tmem, adesc + (uint64_t)(k * 2), b2desc + (uint64_t)(k * 2), 1u);
#pragma unroll
            for (int k = 0; k < 4; ++k)
              mma_bf16<PAIR>(d_tmem, a2desc + (uint64_t)(k * 2), bdesc + (uint64_t)(k * 2), 1u);
          }
          mma_commit<PAIR>(own_empty0 + stage * 8);
          if (PAIR) mma_commit<PAIR>(peer_empty0 + stage * 8);
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1;
          }
        }
        mma_commit<PAIR>(own_tfull0 + acc * 8);
        if (PAIR) mma_commit<PAIR>(peer_tfull0 + acc * 8);
      }
      // Retire every issued MMA before tensor memory is released.
      mma_commit<PAIR>(smem_u32(mdone));
      if (!mbar_wait(mdone, 0, nullptr)) atomicExch(status, 6);
    }
  } else {
    // ---------------- epilogue ----------------
    const int quarter = warp & 3;            // TMEM lanes this warp may access
    const int ew = warp - 2;                 // 0..7
    const int half = ew >> 2;                // column half of each tile
    const int qlocal = quarter * 32 + lane;
    const int qi = qblock * kBM + qlocal;
    const bool qvalid = qi < nq;
    const float qa = (!SQ && qvalid) ? q_aux[qi] : 0.f;
    const float qn2 = (!SQ && qvalid) ? q_n2[qi] : 0.f;
    // SQ8: the query's rank terms {A, B, C, ||q||^2} (sq8.cu); q_aux holds them.
    const float4 qinfo = (SQ && qvalid) ? reinterpret_cast<const float4*>(q_aux)[qi]
                                        : make_float4(0.f, 0.f, 0.f, 0.f);
    // RaBitQ: half the query's coordinate sum and its integer scale (q_aux,
    // float2 per query) and its per-cluster terms gAdd (q_n2, [nq][nc]) in a
    // per-warp table [cluster][lane].
    const float2 rq_q = (RQ && qvalid) ? reinterpret_cast<const float2*>(q_aux)[qi]
                                       : make_float2(0.f, 0.f);
    float* gadd_tab = gadd_all + ew * kRaBitQMaxClusters * 32;
    if constexpr (RQ) {
      for (int c = 0; c < nc; ++c)
        gadd_tab[c * 32 + lane] = qvalid ? q_n2[(int64_t)qi * nc + c] : 0.f;
      __syncwarp();
    }
    // Per-query thresholds are shared by every list of the query (gthr,
    // lowered with atomicMin after each compaction): a list may drop any key
    // above another list's kp-th key, so only the first lists of a query pay
    // for filling up.
    uint64_t thr = qvalid ? (uint64_t)*(volatile unsigned long long*)&gthr[qi] : kEmptyKey;
    float thr_f = rank_of(thr);  // NaN while the list is not full: accept all
    float tq = score_bound<METRIC>(thr_f, qa, qn2);
    int cnt = 0;
    int nonfinite = 0;
    const int list = list_base + part * 2 + half;
    uint64_t* gbuf = cand + ((int64_t)(qvalid ? qi : 0) * num_lists + list) * kCap;
    int* hist = hist_all + ew * 256;
    float* meta_aux = reinterpret_cast<float*>(meta_all + ew * 256);  // [128]
    uint32_t* meta_kr = meta_all + ew * 256 + 128;                     // [128]
    float4* meta4 = meta4_all + ew * 128;                              // [128] (SQ8)
    // Row metadata (aux, key rank, filter) of this warp's 128 columns is
    // loaded one tile ahead into registers and staged in shared memory, so
    // neither the scoring loop nor the append path waits on global memory.
    float pf_aux[kChunks];
    float4 pf4[(SQ || RQ) ? kChunks : 1];
    uint32_t pf_kr[kChunks], pf_vm[kChunks];
    auto prefetch = [&](int t) {
      const int64_t base = row_begin + (int64_t)t * BN + half * kHalfCols;
#pragma unroll
      for (int c = 0; c < kChunks; ++c) {
        const int64_t row = base + c * 32 + lane;
        const bool ok = t < num_tiles && row < row_end && bitmap_pass(bitmap, row);
        if constexpr (SQ || RQ) {
          pf4[c] = ok ? reinterpret_cast<const float4*>(row_aux)[row]
                      : make_float4(0.f, 0.f, 0.f, 0.f);
          pf_aux[c] = 0.f;
        } else {
          const float ra = (ok && METRIC != kMetricIP) ? row_aux[row] : 0.f;
          pf_aux[c] = METRIC == kMetricL2 ? -0.5f * ra : ra;
        }
        pf_kr[c] = ok ? keyrank[row] : 0u;
        pf_vm[c] = __ballot_sync(kFullMask, ok);
      }
    };
    prefetch(0);
    // The shared threshold is read one tile ahead: a stale value is still a
    // valid bound (it only decreases), and the read's latency overlaps the
    // tile instead of stalling before it.
    uint64_t g_next = qvalid ? (uint64_t)*(volatile unsigned long long*)&gthr[qi] : kEmptyKey;
    for (int t = 0; t < num_tiles; ++t) {
      const int acc = t & 1;
      const uint32_t acc_phase = (t >> 1) & 1;
      uint32_t vm[kChunks];
      __syncwarp();
#pragma unroll
      for (int c = 0; c < kChunks; ++c) {
        meta_aux[c * 32 + lane] = pf_aux[c];
        if constexpr (SQ || RQ) meta4[c * 32 + lane] = pf4[c];
        meta_kr[c * 32 + lane] = pf_kr[c];
        vm[c] = pf_vm[c];
      }
      __syncwarp();
      prefetch(t + 1);
      if (g_next < thr) {
        thr = g_next;
        thr_f = rank_of(thr);
        tq = score_bound<METRIC>(thr_f, qa, qn2);
      }
      if (qvalid) g_next = (uint64_t)*(volatile unsigned long long*)&gthr[qi];
      // Warp-uniform outcome: the tcgen05.ld below needs every lane.
      if (!__all_sync(kFullMask, mbar_wait(&tfull[acc], acc_phase, s_abort, wait_ns))) {
        atomicExch(status, 4);
        *s_abort = 1;
        break;
      }
      tmem_fence_after();
      const uint32_t taddr =
          tmem_base + ((uint32_t)(quarter * 32) << 16) + acc * kBN + half * kHalfCols;
      uint32_t va[32], vb[32];
      // Rare path of the quantized modes: the fast rank of column j of
      // chunk c, appended when below the list threshold (a non-finite rank
      // marks the query for the exact scan).
      auto append = [&](int c, int j, float rank) {
        if (!isfinite(rank)) {
          nonfinite = 1;
        } else {
          const uint64_t key = pack_rank(rank, meta_kr[c * 32 + j]);
          if (key < thr) gbuf[cnt++] = key;
        }
      };
      if constexpr (RQ8) {
        // The 64 columns of this warp: A_h (va) and A_l (vb, BN columns on)
        // of 32 rows at a time.
#pragma unroll 1
        for (int c = 0; c < kChunks; ++c) {
          tmem_ld32(taddr + c * 32, va);
          tmem_ld32(taddr + BN + c * 32, vb);
          tmem_wait_ld();
          const uint32_t vmask = qvalid ? vm[c] : 0u;
          auto rq8_rank = [&](int j, uint32_t h, uint32_t l) -> float {
            const float4 r = meta4[c * 32 + j];
            const float g = gadd_tab[__float_as_int(r.z) * 32 + lane];
            // sum(v' w) + 128 sum(v') of this row; the query's 128 sum(w)
            // is folded into rq_q.x.
            const float dp = fmaf(256.f, (float)(int)h, (float)(int)l) + r.w;
            return fmaf(r.y, fmaf(rq_q.y, dp, -rq_q.x), r.x + g);
          };
          // The pass mask, then the passing columns one at a time (as for
          // the Flat metrics below).
          uint32_t pass = 0u;
          if (vmask != 0u) {
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (!(rq8_rank(j, va[j], vb[j]) > thr_f)) pass |= 1u << j;
          }
          pass &= vmask;
          uint32_t any = __reduce_or_sync(kFullMask, pass);
          while (any) {
            const int j = __ffs(any) - 1;
            any &= any - 1;
            const uint32_t h = pick32(va, j), l = pick32(vb, j);
            if ((pass >> j) & 1u) append(c, j, rq8_rank(j, h, l));
          }
        }
      } else {
      tmem_ld32(taddr, va);
      tmem_wait_ld();
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t(&cur)[32] = (c & 1) ? vb : va;
        uint32_t(&nxt)[32] = (c & 1) ? va : vb;
        if (c + 1 < 4) tmem_ld32(taddr + (c + 1) * 32, nxt);
        const uint32_t vmask = qvalid ? vm[c] : 0u;
        // Rare path: the exact fast rank and key of column j (its dot v),
        // appended when below the list threshold.
        auto rare_v = [&](int j, uint32_t v, float a) {
          const float ra = METRIC == kMetricL2 ? -2.f * a : a;
          const float r = tc_rank<METRIC>(__uint_as_float(v), ra, qa, qn2);
          if (!isfinite(r)) {
            nonfinite = 1;
          } else {
            const uint64_t key = pack_rank(r, meta_kr[c * 32 + j]);
            if (key < thr) gbuf[cnt++] = key;
          }
        };
        auto score = [&](int j, float a) -> float {
          const float dot = __uint_as_float(cur[j]);
          if (METRIC == kMetricIP) return dot;
          if (METRIC == kMetricCosine) return dot * a;
          if (METRIC == kMetricL2) return dot + a;
          return -tc_rank<METRIC>(dot, a, qa, qn2);
        };
        const float4* a4 = reinterpret_cast<const float4*>(meta_aux + c * 32);
        if constexpr (RQ) {
          // RaBitQRanker (rabitq.cu): add + gAdd[cluster] + rescale (dot - sum/2)
          // with dot = scale * the exact integer dot.
          auto rq_rank = [&](int j, uint32_t v) -> float {
            const float4 r = meta4[c * 32 + j];
            const float g = gadd_tab[__float_as_int(r.z) * 32 + lane];
            const float dot = (float)(int)v * rq_q.y;
            return fmaf(r.y, dot - rq_q.x, r.x + g);
          };
          uint32_t pass = 0u;
          if (vmask != 0u) {
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (!(rq_rank(j, cur[j]) > thr_f)) pass |= 1u << j;
          }
          pass &= vmask;
          uint32_t any = __reduce_or_sync(kFullMask, pass);
          while (any) {
            const int j = __ffs(any) - 1;
            any &= any - 1;
            const uint32_t v = pick32(cur, j);
            if ((pass >> j) & 1u) append(c, j, rq_rank(j, v));
          }
        } else if constexpr (SQ) {
          // SQ8Ranker (sq8.cu) on the exact integer dot product.
          auto sq_rank = [&](int j, uint32_t v) -> float {
            const float4 r = meta4[c * 32 + j];
            const float dot = (float)(int)v;
            const float tt = fmaf(qinfo.x, dot, qinfo.y * r.z);
            const float inner = fmaf(r.x, tt, r.y * qinfo.z);
            return METRIC == kMetricIP ? -inner : (r.w + qinfo.w) - 2.f * inner;
          };
          if constexpr (METRIC == kMetricL2) {
            // Per column: with the pass mask below, this mode's rank terms
            // and the live chunk exceed the register budget and spill.
            if (vmask != 0u) {
#pragma unroll
              for (int j = 0; j < 32; ++j) {
                const float rank = sq_rank(j, cur[j]);
                if (((vmask >> j) & 1u) && !(rank > thr_f)) append(c, j, rank);
              }
            }
          } else {
            uint32_t pass = 0u;
            if (vmask != 0u) {
#pragma unroll
              for (int j = 0; j < 32; ++j)
                if (!(sq_rank(j, cur[j]) > thr_f)) pass |= 1u << j;
            }
            pass &= vmask;
            uint32_t any = __reduce_or_sync(kFullMask, pass);
            while (any) {
              const int j = __ffs(any) - 1;
              any &= any - 1;
              const uint32_t v = pick32(cur, j);
              if ((pass >> j) & 1u) append(c, j, sq_rank(j, v));
            }
          }
        } else {
          // Flat metrics: the chunk's pass mask without branches, then one
          // loop over the columns that pass for some lane of the warp (few
          // once the thresholds are set), each column's dot picked from the
          // registers by its warp-uniform index.  The per-column test stays
          // free of the append path's code, which keeps the unrolled loop
          // small.
          uint32_t pass = 0u;
#pragma unroll
          for (int g = 0; g < 8; ++g) {
            const float4 av = a4[g];
            const float aa[4] = {av.x, av.y, av.z, av.w};
#pragma unroll
            for (int e = 0; e < 4; ++e)
              if (score(g * 4 + e, aa[e]) >= tq) pass |= 1u << (g * 4 + e);
          }
          pass &= vmask;
          uint32_t any = __reduce_or_sync(kFullMask, pass);
          while (any) {
            const int j = __ffs(any) - 1;
            any &= any - 1;
            const uint32_t v = pick32(cur, j);
            if ((pass >> j) & 1u) rare_v(j, v, meta_aux[c * 32 + j]);
          }
        }
        if (c + 1 < 4) tmem_wait_ld();
      }
      }  // !RQ8
      // Release the accumulator to the MMA warp before any compaction (one
      // arrival per warp, on the issuing CTA's barrier).
      tmem_fence_before();
      __syncwarp();
      if (lane == 0) {
        if constexpr (PAIR) mbar_arrive_remote(cluster_addr(&tempty[acc], 0));
        else mbar_arrive(&tempty[acc]);
      }
      // Keep room for the next tile's appends (at most 128 per list).
      uint32_t need = __ballot_sync(kFullMask, cnt > kCap - 128);
      while (need) {
        const int who = __ffs(need) - 1;
        need &= need - 1;
        const int wcnt = __shfl_sync(kFullMask, cnt, who);
        uint64_t* wbuf =
            cand + ((int64_t)(qblock * kBM + quarter * 32 + who) * num_lists + list) * kCap;
        const uint64_t new_thr = warp_select_compact(wbuf, wcnt, kp, hist);
        if (lane == who) {
          if (new_thr < thr) {
            thr = new_thr;
            thr_f = rank_of(thr);
            tq = score_bound<METRIC>(thr_f, qa, qn2);
            atomicMin(&gthr[qi], (unsigned long long)thr);
          }
          cnt = kp;
        }
      }
    }
    // Publish each list: at most kp keys (unsorted) and its saturation key.
    for (int who = 0; who < 32; ++who) {
      const int wq = qblock * kBM + quarter * 32 + who;
      if (wq >= nq) continue;
      const int wcnt = __shfl_sync(kFullMask, cnt, who);
      uint64_t wthr = __shfl_sync(kFullMask, thr, who);
      uint64_t* wbuf = cand + ((int64_t)wq * num_lists + list) * kCap;
      if (wcnt > kp) {
        const uint64_t c = warp_select_compact(wbuf, wcnt, kp, hist);
        wthr = c < wthr ? c : wthr;
      }
      if (lane == 0) {
        part_counts[(int64_t)wq * num_lists + list] = min(wcnt, kp);
        part_sat[(int64_t)wq * num_lists + list] = wthr;
      }
    }
    if (qvalid && nonfinite) atomicOr(&q_flags[qi], 1);
  }

  __syncthreads();
  // Drain: every copy either CTA issued has landed before either leaves
  // (already true unless a role aborted).  The first CTA's barriers count
  // both CTAs' copies; a stage phase the second CTA issued but the first
  // never armed (the first stopped early) is armed here for its half.
  if constexpr (PAIR) cluster_sync_all();
  if (threadIdx.x == 0 && issuer) {
    for (int s2 = 0; s2 < kStages; ++s2) {
      const uint32_t mine = issued[s2];
      const uint32_t other = PAIR ? ld_cluster_u32(cluster_addr(&issued[s2], 1)) : mine;
      if (mine > 0 && !mbar_wait(&full[s2], (mine - 1) & 1, nullptr)) atomicExch(status, 5);
      if (PAIR && other > mine) {  // at most one phase ahead
        mbar_expect_tx(&full[s2], kStageBytes);
        if (!mbar_wait(&full[s2], mine & 1, nullptr)) atomicExch(status, 5);
      }
    }
  }
  // Neither CTA of a pair leaves while the other may still read its shared
  // memory, signal its barriers or write its tensor memory.
  if constexpr (PAIR) cluster_sync_all();
  if (warp == 1) {
    tmem_fence_after();
    if constexpr (PAIR)
      asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, 512;" ::"r"(tmem_base));
    else
      asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(tmem_base));
  }
}

}  // namespace tc

// ---------------------------------------------------------------------------
// Host side.
// ---------------------------------------------------------------------------
namespace {
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

// Row-major [rows][d] binary16 matrix viewed with a row stride of
// `row_stride_elems`, box [box_rows][64], 128-byte swizzle.
// Row-major [rows][d] matrix of 1- or 2-byte elements viewed with a row
// stride of `row_stride_elems`, box [box_rows][128 bytes], 128-byte swizzle.
bool make_map(CUtensorMap* map, const void* base, int64_t rows, int d, int64_t row_stride_elems,
              int box_rows, int elem_bytes = 2) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {(cuuint64_t)d, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)row_stride_elems * elem_bytes};
  cuuint32_t box[2] = {(cuuint32_t)(128 / elem_bytes), (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, elem_bytes == 2 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_UINT8,
                  2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}
}  // namespace

bool flat_tc_supported(int d, const void* rows, const void* queries) {
  // TMA coordinates are int32: rows beyond 2^31 - 256 stay on the other path.
  return d % 8 == 0 && d >= 64 && ((uintptr_t)rows % 16 == 0) && ((uintptr_t)queries % 16 == 0) &&
         encode_fn() != nullptr;
}

int flat_tc_cap() { return tc::kCap; }
int flat_tc_lists_per_part() { return 2; }

// CTA pairs whenever there are two query blocks to pair up.
bool flat_tc_pairs(int nq) { return nq > tc::kBM; }

namespace {
// Limit of the scan's main-loop waits (xvec_gpu_set_wait_limit_ns); the
// teardown's waits for copies already issued keep the default.
std::atomic<int64_t> g_tc_wait_ns{(int64_t)tc::kWaitLimitNs};
uint64_t tc_wait_ns() { return (uint64_t)g_tc_wait_ns.load(std::memory_order_relaxed); }

// Launches mode MODE (a Flat metric, or kModeSq8 + metric) on CTA pairs when
// there are two query blocks, else on single CTAs.
template <int MODE>
cudaError_t launch_tc(int nq, const void* queries, const void* queries2, int nc, const void* rows,
                      const void* rows2,
                      int64_t n, int d, int64_t row_stride_elems, int elem_bytes,
                      const float* row_aux,
                      const uint32_t* keyrank, const float* q_aux, const float* q_n2,
                      unsigned long long* gthr, const uint32_t* bitmap, int num_parts, int kp,
                      int list_base, int num_lists, uint64_t* cand, int* part_counts,
                      uint64_t* part_sat, int* q_flags, int* status, cudaStream_t stream) {
  const int qblocks = (nq + tc::kBM - 1) / tc::kBM;
  const bool pair = flat_tc_pairs(nq);
  constexpr bool RQ8 = MODE == tc::kModeRaBitQ8;
  constexpr bool RQ = MODE == tc::kModeRaBitQ || RQ8;
  constexpr bool SPLIT = (MODE & tc::kModeSplit) != 0 && !RQ8;
  constexpr bool TWO_A = RQ8;
  constexpr int BN = RQ8 ? tc::kBN / 2 : tc::kBN;
  using SP = tc::Shape<true, RQ, SPLIT, TWO_A, BN>;
  using SS = tc::Shape<false, RQ, SPLIT, TWO_A, BN>;
  const int box_rows = pair ? SP::kRowsPerCta : SS::kRowsPerCta;
  // The low parts' maps (unused unless SPLIT) repeat the high parts'.
  CUtensorMap qmap, rmap, qmap2, rmap2;
  if (!make_map(&qmap, queries, nq, d, d, tc::kBM, elem_bytes) ||
      !make_map(&rmap, rows, n, d, row_stride_elems, box_rows, elem_bytes) ||
      !make_map(&qmap2, queries2 ? queries2 : queries, nq, d, d, tc::kBM, elem_bytes) ||
      !make_map(&rmap2, rows2 ? rows2 : rows, n, d, row_stride_elems, box_rows, elem_bytes))
    return cudaErrorInvalidValue;
  const int64_t rows_per_part = ((n + num_parts - 1) / num_parts + tc::kBN - 1) / tc::kBN * tc::kBN;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(pair ? (qblocks + 1) / 2 * 2 : qblocks, num_parts);
  cfg.blockDim = dim3(tc::kThreads);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = pair ? 2 : 1;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t err;
  if (pair) {
    auto kern = tc::flat_scan_tc_kernel<MODE, true>;
    cfg.dynamicSmemBytes = SP::kSmemBytes;
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SP::kSmemBytes);
    err = cudaLaunchKernelEx(&cfg, kern, qmap, rmap, qmap2, rmap2, nc, nq, n, d, row_aux, keyrank, q_aux,
                             q_n2, gthr, bitmap, rows_per_part, kp, list_base, num_lists, cand,
                             part_counts, part_sat, q_flags, status, tc_wait_ns());
  } else {
    auto kern = tc::flat_scan_tc_kernel<MODE, false>;
    cfg.dynamicSmemBytes = SS::kSmemBytes;
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SS::kSmemBytes);
    err = cudaLaunchKernelEx(&cfg, kern, qmap, rmap, qmap2, rmap2, nc, nq, n, d, row_aux, keyrank, q_aux,
                             q_n2, gthr, bitmap, rows_per_part, kp, list_base, num_lists, cand,
                             part_counts, part_sat, q_flags, status, tc_wait_ns());
  }
  if (err != cudaSuccess) return err;
  return cudaGetLastError();
}
}  // namespace

cudaError_t launch_flat_scan_tc(int metric, const __half* queries, int nq, const __half* rows,
                                int64_t n, int d, int64_t row_stride_elems, const float* row_aux,
                                const uint32_t* keyrank, const float* q_aux, const float* q_n2,
                                unsigned long long* gthr, const uint32_t* bitmap, int num_parts,
                                int kp, int list_base, int num_lists, uint64_t* cand,
                                int* part_counts, uint64_t* part_sat, int* q_flags, int* status,
                                cudaStream_t stream) {
#define XVEC_TC_ARGS                                                                           \
  nq, queries, nullptr, 0, rows, nullptr, n, d, row_stride_elems, 2, row_aux, keyrank, q_aux, q_n2,     \
      gthr, bitmap,                                                                            \
      num_parts, kp, list_base, num_lists, cand, part_counts, part_sat, q_flags, status, stream
  switch (metric) {
    case kMetricL2: return launch_tc<kMetricL2>(XVEC_TC_ARGS);
    case kMetricIP: return launch_tc<kMetricIP>(XVEC_TC_ARGS);
    case kMetricCosine: return launch_tc<kMetricCosine>(XVEC_TC_ARGS);
    case kMetricMIPS: return launch_tc<kMetricMIPS>(XVEC_TC_ARGS);
    default: return cudaErrorInvalidValue;
  }
#undef XVEC_TC_ARGS
}

cudaError_t launch_flat_scan_tc_split(int metric, const __nv_bfloat16* q_hi,
                                      const __nv_bfloat16* q_lo, int nq, const __nv_bfloat16* r_hi,
                                      const __nv_bfloat16* r_lo, int64_t n, int d,
                                      const float* row_aux, const uint32_t* keyrank,
                                      const float* q_aux, const float* q_n2,
                                      unsigned long long* gthr, const uint32_t* bitmap,
                                      int num_parts, int kp, int list_base, int num_lists,
                                      uint64_t* cand, int* part_counts, uint64_t* part_sat,
                                      int* q_flags, int* status, cudaStream_t stream) {
#define XVEC_TC_ARGS                                                                           \
  nq, q_hi, q_lo, 0, r_hi, r_lo, n, d, (int64_t)d, 2, row_aux, keyrank, q_aux, q_n2, gthr,     \
      bitmap, num_parts, kp, list_base, num_lists, cand, part_counts, part_sat, q_flags,       \
      status, stream
  switch (metric) {
    case kMetricL2: return launch_tc<tc::kModeSplit + kMetricL2>(XVEC_TC_ARGS);
    case kMetricIP: return launch_tc<tc::kModeSplit + kMetricIP>(XVEC_TC_ARGS);
    case kMetricCosine: return launch_tc<tc::kModeSplit + kMetricCosine>(XVEC_TC_ARGS);
    case kMetricMIPS: return launch_tc<tc::kModeSplit + kMetricMIPS>(XVEC_TC_ARGS);
    default: return cudaErrorInvalidValue;
  }
#undef XVEC_TC_ARGS
}

// bfloat16 high and low parts of float32 values: hi = bf16(x), lo =
// bf16(x - hi) (x - hi is exact in float32).
__global__ void split_bf16_kernel(const float* __restrict__ x, int64_t count,
                                  __nv_bfloat16* __restrict__ hi, __nv_bfloat16* __restrict__ lo) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= count) return;
  const float v = x[i];
  const __nv_bfloat16 h = __float2bfloat16_rn(v);
  hi[i] = h;
  lo[i] = __float2bfloat16_rn(v - __bfloat162float(h));
}

cudaError_t launch_split_bf16(const float* x, int64_t count, __nv_bfloat16* hi, __nv_bfloat16* lo,
                              cudaStream_t stream) {
  if (count <= 0) return cudaSuccess;
  split_bf16_kernel<<<(unsigned)((count + 255) / 256), 256, 0, stream>>>(x, count, hi, lo);
  return cudaGetLastError();
}

cudaError_t launch_sq8_scan_tc(int metric, const int8_t* qcodes, int nq, const int8_t* codes,
                               int64_t n, int d, const float4* row_info, const uint32_t* keyrank,
                               const float4* q_info, unsigned long long* gthr,
                               const uint32_t* bitmap, int num_parts, int kp, int list_base,
                               int num_lists, uint64_t* cand, int* part_counts,
                               uint64_t* part_sat, int* q_flags, int* status,
                               cudaStream_t stream) {
#define XVEC_TC_ARGS                                                                           \
  nq, qcodes, nullptr, 0, codes, nullptr, n, d, (int64_t)d, 1,                                         \
      reinterpret_cast<const float*>(row_info), keyrank,                                       \
      reinterpret_cast<const float*>(q_info), nullptr, gthr, bitmap, num_parts, kp, list_base, \
      num_lists, cand, part_counts, part_sat, q_flags, status, stream
  switch (metric) {
    case kMetricL2: return launch_tc<tc::kModeSq8 + kMetricL2>(XVEC_TC_ARGS);
    case kMetricIP: return launch_tc<tc::kModeSq8 + kMetricIP>(XVEC_TC_ARGS);
    default: return cudaErrorInvalidValue;
  }
#undef XVEC_TC_ARGS
}

cudaError_t launch_rabitq_scan_tc(const int8_t* q_int, int nq, const int8_t* planes, int64_t n,
                                  int padded, const float4* row_info, const uint32_t* keyrank,
                                  const float2* q_terms, const float* q_gadd, int nc,
                                  unsigned long long* gthr, const uint32_t* bitmap,
                                  int num_parts, int kp, int list_base, int num_lists,
                                  uint64_t* cand, int* part_counts, uint64_t* part_sat,
                                  int* q_flags, int* status, cudaStream_t stream) {
  if (nc > tc::kRaBitQMaxClusters || !rabitq_tc_supported(padded, planes, q_int))
    return cudaErrorInvalidValue;
  return launch_tc<tc::kModeRaBitQ>(nq, q_int, nullptr, nc, planes, nullptr, n, 2 * padded,
                                    (int64_t)2 * padded, 1,
                                    reinterpret_cast<const float*>(row_info), keyrank,
                                    reinterpret_cast<const float*>(q_terms), q_gadd, gthr, bitmap, num_parts, kp, list_base,
                                    num_lists, cand, part_counts, part_sat, q_flags, status,
                                    stream);
}

cudaError_t launch_rabitq8_scan_tc(const int8_t* q_planes, int nq, const int8_t* vplane,
                                   int64_t n, int padded, const float4* row_info,
                                   const uint32_t* keyrank, const float2* q_terms,
                                   const float* q_gadd, int nc, unsigned long long* gthr,
                                   const uint32_t* bitmap, int num_parts, int kp, int list_base,
                                   int num_lists, uint64_t* cand, int* part_counts,
                                   uint64_t* part_sat, int* q_flags, int* status,
                                   cudaStream_t stream) {
  if (nc > tc::kRaBitQMaxClusters || !rabitq8_tc_supported(padded, vplane, q_planes))
    return cudaErrorInvalidValue;
  return launch_tc<tc::kModeRaBitQ8>(nq, q_planes, q_planes + (int64_t)nq * padded, nc, vplane,
                                     nullptr, n, padded, (int64_t)padded, 1,
                                     reinterpret_cast<const float*>(row_info), keyrank,
                                     reinterpret_cast<const float*>(q_terms), q_gadd, gthr,
                                     bitmap, num_parts, kp, list_base, num_lists, cand,
                                     part_counts, part_sat, q_flags, status, stream);
}

bool rabitq8_tc_supported(int padded, const void* vplane, const void* q_planes) {
  // Rows of padded bytes in 128-byte k-steps; |A_h|, |A_l| <= 2^14 padded.
  return padded % 64 == 0 && padded >= 64 && padded <= 65536 &&
         ((uintptr_t)vplane % 16 == 0) && ((uintptr_t)q_planes % 16 == 0) &&
         encode_fn() != nullptr;
}

int rabitq_tc_max_clusters() { return tc::kRaBitQMaxClusters; }

bool rabitq_tc_supported(int padded, const void* planes, const void* q_int) {
  // Rows of 2 padded bytes in 128-byte k-steps; |dot| <= 16192 padded < 2^31.
  return padded % 64 == 0 && padded >= 64 && padded <= 65536 &&
         ((uintptr_t)planes % 16 == 0) && ((uintptr_t)q_int % 16 == 0) &&
         encode_fn() != nullptr;
}

bool sq8_tc_supported(int d, const void* codes, const void* qcodes) {
  // 16-byte row strides for TMA; |dot| <= 127^2 d stays exact in float32.
  return d % 16 == 0 && d >= 128 && d <= 1040 && ((uintptr_t)codes % 16 == 0) &&
         ((uintptr_t)qcodes % 16 == 0) && encode_fn() != nullptr;
}

}  // namespace xvec

extern "C" int64_t xvec_gpu_set_wait_limit_ns(int64_t ns) {
  return xvec::g_tc_wait_ns.exchange(ns > 0 ? ns : (int64_t)xvec::tc::kWaitLimitNs);
}
