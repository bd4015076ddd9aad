// flat_tc.cu — tensor-core candidate scan for Flat search over binary16 rows.
//
// The fast-rank stage of Flat search (flat_kernels.cu) for FP16 storage on
// sm_100a: the query x row dot products are a GEMM, computed by tcgen05.mma
// (kind::f16, fp32 accumulation in tensor memory) on tiles staged by TMA,
// with the per-query candidate selection fused into the epilogue, so the
// score matrix is never written to memory.
//
//   CTA = 6 warps, one CTA per SM (tensor memory and shared memory sized so):
//     warp 0    TMA producer: query tile A[128 x 64] + row tile B[256 x 64]
//               per k-step into a 4-stage ring (128-byte swizzle).
//     warp 1    allocates 512 TMEM columns, issues the MMAs (one thread):
//               D[128 queries x 256 rows] fp32, two accumulators in TMEM so
//               the epilogue of tile t overlaps the MMAs of tile t+1.
//     warps 2-5 epilogue: each thread owns one query (one TMEM lane), loads
//               its 256 dot products with tcgen05.ld, turns them into fast
//               ranks and appends the ones below its threshold to the
//               query's candidate buffer (global memory); a full buffer is
//               compacted to its KP best keys by the warp (select.cuh).
//   Grid = (query blocks of 128, row chunks); blockIdx.x varies fastest so
//   the CTAs resident at any time share row chunks and the rows come from L2.
//
// Every mbarrier wait is bounded: on expiry the kernel records an error in
// `status`, stops issuing work and still releases its tensor memory.
#include <cuda.h>
#include <cudaTypedefs.h>

#include "capi_internal.h"
#include "common.cuh"
#include "flat_tc.cuh"
#include "select.cuh"

namespace xvec {

namespace tc {

constexpr int kBM = 128;   // queries per CTA (TMEM lanes)
constexpr int kBN = 256;   // rows per tile (TMEM columns per accumulator)
constexpr int kBK = 64;    // k-step: 64 fp16 = 128 bytes (one swizzle row)
constexpr int kStages = 4;
constexpr int kCap = 256;  // candidate buffer entries per (query, part)
constexpr int kThreads = 192;
constexpr uint32_t kTileABytes = kBM * kBK * 2;  // 16 KB
constexpr uint32_t kTileBBytes = kBN * kBK * 2;  // 32 KB
constexpr uint32_t kStageBytes = kTileABytes + kTileBBytes;
constexpr uint32_t kSmemBytes = kStages * kStageBytes + 4 * kCap * 8 + 1024 /*align*/ + 256;
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // a wait gives up after 2 s

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
__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Bounded parity wait: false once kWaitLimitNs passed or another role of
// the CTA raised *abort.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity,
                                          const volatile int* abort) {
  const uint32_t addr = smem_u32(bar);
  uint64_t start = 0;
  for (uint32_t i = 0;; ++i) {
    uint32_t done;
    asm volatile(
        "{\n.reg .pred p;\n"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
        "selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(done)
        : "r"(addr), "r"(parity)
        : "memory");
    if (done) return true;
    if ((i & 255) == 0) {
      if (abort && *abort) return false;
      const uint64_t now = global_ns();
      if (start == 0) start = now;
      else if (now - start > kWaitLimitNs) return false;
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

// UMMA shared-memory descriptor: K-major, 128-byte swizzle, 8-row groups
// 1024 bytes apart (SBO), descriptor version 1 (sm_100).
__device__ __forceinline__ uint64_t smem_desc_sw128(const void* tile) {
  const uint64_t addr = smem_u32(tile);
  return ((addr & 0x3FFFFull) >> 4) | (1ull << 16) | ((1024ull >> 4) << 32) | (1ull << 46) |
         (2ull << 61);
}

// Instruction descriptor: kind::f16, A/B = F16, D = F32, both K-major.
constexpr uint32_t kIdesc = (1u << 4) | ((uint32_t)(kBN >> 3) << 17) | ((uint32_t)(kBM >> 4) << 24);

__device__ __forceinline__ void mma_f16(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t acc) {
  asm volatile(
      "{\n.reg .pred p;\nsetp.ne.b32 p, %4, 0;\n"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
      "l"(a), "l"(b), "r"(kIdesc), "r"(acc));
}
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
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
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
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

// Compacts lane `who`'s candidate buffer (global) to its KP best keys.
__device__ __noinline__ void warp_compact_global(uint64_t* gbuf, uint64_t* scratch, int cnt,
                                                 int kp, uint64_t* thr_out) {
  const int lane = threadIdx.x & 31;
  __syncwarp();  // the owning lane's appends are visible to the warp
  for (int i = lane; i < kCap; i += 32) scratch[i] = i < cnt ? gbuf[i] : kEmptyKey;
  __syncwarp();
  warp_sort_u64<kCap>(scratch);
  const int keep = min(cnt, kp);
  for (int i = lane; i < keep; i += 32) gbuf[i] = scratch[i];
  __syncwarp();
  if (cnt >= kp) *thr_out = scratch[kp - 1];
}

template <int METRIC>
__global__ void __launch_bounds__(kThreads, 1) flat_scan_tc_kernel(
    const __grid_constant__ CUtensorMap qmap, const __grid_constant__ CUtensorMap rmap, int nq,
    int64_t n, int d, const float* __restrict__ row_aux, const uint32_t* __restrict__ keyrank,
    const float* __restrict__ q_aux, const float* __restrict__ q_n2,
    const uint64_t* __restrict__ q_seed, const uint32_t* __restrict__ bitmap,
    int64_t rows_per_part, int kp, uint64_t* __restrict__ cand, int* __restrict__ part_counts,
    uint64_t* __restrict__ part_sat, int* __restrict__ q_flags, int* __restrict__ status) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = (unsigned char*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  unsigned char* tiles = smem;  // kStages x (A | B)
  uint64_t* scratch = reinterpret_cast<uint64_t*>(smem + kStages * kStageBytes);  // 4 x kCap
  uint64_t* bars = scratch + 4 * kCap;
  uint64_t* full = bars;               // [kStages]
  uint64_t* empty = bars + kStages;    // [kStages]
  uint64_t* tfull = bars + 2 * kStages;   // [2]
  uint64_t* tempty = bars + 2 * kStages + 2;  // [2]
  uint64_t* mdone = bars + 2 * kStages + 4;   // all issued MMAs retired
  uint32_t* tmem_base_slot = reinterpret_cast<uint32_t*>(bars + 2 * kStages + 5);
  __shared__ int s_abort_storage;
  volatile int* s_abort = &s_abort_storage;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qblock = blockIdx.x;
  const int part = blockIdx.y, num_parts = gridDim.y;
  const int64_t row_begin = (int64_t)part * rows_per_part;
  const int64_t row_end = min(n, row_begin + rows_per_part);
  const int num_tiles = row_end > row_begin ? (int)((row_end - row_begin + kBN - 1) / kBN) : 0;
  const int ksteps = (d + kBK - 1) / kBK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 128);
    }
    mbar_init(mdone, 1);
    *s_abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(
                     smem_u32(tmem_base_slot)));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    tmem_fence_before();
  }
  __syncthreads();
  tmem_fence_after();
  const uint32_t tmem_base = *tmem_base_slot;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int armed[kStages];
#pragma unroll
      for (int s2 = 0; s2 < kStages; ++s2) armed[s2] = -1;
      for (int t = 0; t < num_tiles && !*s_abort; ++t) {
        const int row0 = (int)(row_begin + (int64_t)t * kBN);
        for (int ks = 0; ks < ksteps; ++ks) {
          if (!mbar_wait(&empty[stage], phase ^ 1, s_abort)) {
            atomicExch(status, 1);
            *s_abort = 1;
            break;
          }
          unsigned char* a_dst = tiles + stage * kStageBytes;
          unsigned char* b_dst = a_dst + kTileABytes;
          mbar_expect_tx(&full[stage], kStageBytes);
          tma_load_2d(&qmap, &full[stage], a_dst, ks * kBK, qblock * kBM);
          tma_load_2d(&rmap, &full[stage], b_dst, ks * kBK, row0);
          armed[stage] = (int)phase;
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      // Drain: every armed stage's copies have landed before the CTA can
      // exit (already true unless another role aborted).
#pragma unroll
      for (int s2 = 0; s2 < kStages; ++s2)
        if (armed[s2] >= 0 && !mbar_wait(&full[s2], (uint32_t)armed[s2], nullptr))
          atomicExch(status, 5);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      for (int t = 0; t < num_tiles && !*s_abort; ++t) {
        const int acc = t & 1;
        const uint32_t acc_phase = (t >> 1) & 1;
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1, s_abort)) {
          atomicExch(status, 2);
          *s_abort = 1;
          break;
        }
        tmem_fence_after();
        const uint32_t d_tmem = tmem_base + acc * kBN;
        for (int ks = 0; ks < ksteps; ++ks) {
          if (!mbar_wait(&full[stage], phase, s_abort)) {
            atomicExch(status, 3);
            *s_abort = 1;
            break;
          }
          tmem_fence_after();
          const unsigned char* a_src = tiles + stage * kStageBytes;
          const uint64_t adesc = smem_desc_sw128(a_src);
          const uint64_t bdesc = smem_desc_sw128(a_src + kTileABytes);
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k)  // 16 fp16 = 32 bytes per MMA
            mma_f16(d_tmem, adesc + (uint64_t)(k * 2), bdesc + (uint64_t)(k * 2),
                    (ks > 0 || k > 0) ? 1u : 0u);
          mma_commit(&empty[stage]);
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1;
          }
        }
        mma_commit(&tfull[acc]);
      }
      // Retire every issued MMA before tensor memory is released.
      mma_commit(mdone);
      if (!mbar_wait(mdone, 0, nullptr)) atomicExch(status, 6);
    }
  } else {
    // ---------------- epilogue ----------------
    const int quarter = warp & 3;  // TMEM lanes this warp may access
    const int ew = warp - 2;       // epilogue warp index for scratch
    const int qlocal = quarter * 32 + lane;
    const int qi = qblock * kBM + qlocal;
    const bool qvalid = qi < nq;
    const float qa = qvalid ? q_aux[qi] : 0.f;
    const float qn2 = qvalid ? q_n2[qi] : 0.f;
    uint64_t thr = (qvalid && q_seed) ? q_seed[qi] : kEmptyKey;
    uint32_t thr_hi = (uint32_t)(thr >> 32);
    int cnt = 0;
    int nonfinite = 0;
    uint64_t* gbuf = cand + ((int64_t)(qvalid ? qi : 0) * num_parts + part) * kCap;
    uint64_t* wscratch = scratch + ew * kCap;
    for (int t = 0; t < num_tiles; ++t) {
      const int acc = t & 1;
      const uint32_t acc_phase = (t >> 1) & 1;
      if (!mbar_wait(&tfull[acc], acc_phase, s_abort)) {
        atomicExch(status, 4);
        *s_abort = 1;
        break;
      }
      tmem_fence_after();
      const int64_t tile_row = row_begin + (int64_t)t * kBN;
#pragma unroll 1
      for (int c = 0; c < kBN / 32; ++c) {
        uint32_t v[32];
        tmem_ld32(tmem_base + ((uint32_t)(quarter * 32) << 16) + acc * kBN + c * 32, v);
        const int64_t row0 = tile_row + c * 32;
        const int64_t my_row = row0 + lane;
        const bool rvalid = my_row < row_end && bitmap_pass(bitmap, my_row);
        const float aux = rvalid ? (METRIC == kMetricIP ? 0.f : row_aux[my_row]) : 0.f;
        const uint32_t kr = rvalid ? keyrank[my_row] : 0u;
        const uint32_t vmask = __ballot_sync(kFullMask, rvalid);
        if (vmask != 0) {
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const float a = __shfl_sync(kFullMask, aux, j);
            const uint32_t krj = __shfl_sync(kFullMask, kr, j);
            if (!qvalid || !((vmask >> j) & 1u)) continue;
            const float r = tc_rank<METRIC>(__uint_as_float(v[j]), a, qa, qn2);
            const uint32_t hi = float_to_ordered(r);
            if (hi <= thr_hi || hi >= 0xff800000u) {
              if (!isfinite(r)) {
                nonfinite = 1;
              } else {
                const uint64_t key = ((uint64_t)hi << 32) | krj;
                if (key < thr) gbuf[cnt++] = key;
              }
            }
          }
        }
        // Make room for the next 32 appends.
        uint32_t need = __ballot_sync(kFullMask, cnt > kCap - 32);
        while (need) {
          const int who = __ffs(need) - 1;
          need &= need - 1;
          const int wcnt = __shfl_sync(kFullMask, cnt, who);
          uint64_t* wbuf = cand + ((int64_t)(qblock * kBM + quarter * 32 + who) * num_parts + part) * kCap;
          uint64_t new_thr = __shfl_sync(kFullMask, thr, who);
          warp_compact_global(wbuf, wscratch, wcnt, kp, &new_thr);
          new_thr = __shfl_sync(kFullMask, new_thr, 0);
          if (lane == who) {
            thr = new_thr;
            thr_hi = (uint32_t)(thr >> 32);
            cnt = min(cnt, kp);
          }
        }
      }
      tmem_fence_before();
      mbar_arrive(&tempty[acc]);
    }
    // Final compaction of every query of the warp, then publish the part.
    for (int who = 0; who < 32; ++who) {
      const int wcnt = __shfl_sync(kFullMask, cnt, who);
      const int wq = qblock * kBM + quarter * 32 + who;
      if (wq >= nq) continue;
      uint64_t* wbuf = cand + ((int64_t)wq * num_parts + part) * kCap;
      uint64_t new_thr = __shfl_sync(kFullMask, thr, who);
      warp_compact_global(wbuf, wscratch, wcnt, kp, &new_thr);
      new_thr = __shfl_sync(kFullMask, new_thr, 0);
      if (lane == 0) {
        part_counts[(int64_t)wq * num_parts + part] = min(wcnt, kp);
        part_sat[(int64_t)wq * num_parts + part] = new_thr;
      }
    }
    if (qvalid && nonfinite) atomicOr(&q_flags[qi], 1);
  }

  __syncthreads();
  if (warp == 1) {
    tmem_fence_after();
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
bool make_map(CUtensorMap* map, const void* base, int64_t rows, int d, int64_t row_stride_elems,
              int box_rows) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {(cuuint64_t)d, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)row_stride_elems * 2};
  cuuint32_t box[2] = {(cuuint32_t)tc::kBK, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides,
                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
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

cudaError_t launch_flat_scan_tc(int metric, const __half* queries, int nq, const __half* rows,
                                int64_t n, int d, int64_t row_stride_elems, const float* row_aux,
                                const uint32_t* keyrank, const float* q_aux, const float* q_n2,
                                const uint64_t* q_seed, const uint32_t* bitmap, int num_parts,
                                int kp, uint64_t* cand, int* part_counts, uint64_t* part_sat,
                                int* q_flags, int* status, cudaStream_t stream) {
  CUtensorMap qmap, rmap;
  if (!make_map(&qmap, queries, nq, d, d, tc::kBM) ||
      !make_map(&rmap, rows, n, d, row_stride_elems, tc::kBN))
    return cudaErrorInvalidValue;
  const int64_t rows_per_part = ((n + num_parts - 1) / num_parts + tc::kBN - 1) / tc::kBN * tc::kBN;
  dim3 grid((nq + tc::kBM - 1) / tc::kBM, num_parts);
  const int smem = (int)tc::kSmemBytes;
#define XVEC_TC_CASE(M)                                                                     \
  case M: {                                                                                 \
    auto kern = tc::flat_scan_tc_kernel<M>;                                                 \
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);         \
    kern<<<grid, tc::kThreads, smem, stream>>>(qmap, rmap, nq, n, d, row_aux, keyrank, q_aux, \
                                               q_n2, q_seed, bitmap, rows_per_part, kp, cand, \
                                               part_counts, part_sat, q_flags, status);      \
    break;                                                                                  \
  }
  switch (metric) {
    XVEC_TC_CASE(kMetricL2)
    XVEC_TC_CASE(kMetricIP)
    XVEC_TC_CASE(kMetricCosine)
    XVEC_TC_CASE(kMetricMIPS)
    default: return cudaErrorInvalidValue;
  }
#undef XVEC_TC_CASE
  return cudaGetLastError();
}

}  // namespace xvec
