// capi_internal.h — host-side internals shared by the C-ABI translation units.
#pragma once

#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <functional>
#include <mutex>
#include <shared_mutex>
#include <string>
#include <vector>

#include "../../include/xvec_gpu.h"

namespace xvec {

// Per-thread last error (xvec_gpu_last_error).
void set_error(const char* fmt, ...);

// Library counters (xvec_gpu_get_stats).
void count_launches(int64_t n);
void count_tensor_scan();
void count_stream_scan();
void count_search(int64_t queries, int64_t exact_queries, double scan_ms, double search_ms);
bool timing_enabled();
#define XVEC_LAUNCHED() ::xvec::count_launches(1)

// Searches a search makes internally (the IVF probe over the centroids, the
// nearest-centroid assignment of inserted rows) are not counted as searches.
void nested_search_enter();
void nested_search_leave();
struct NestedSearch {
  NestedSearch() { nested_search_enter(); }
  ~NestedSearch() { nested_search_leave(); }
};

// Events on the search stream, recorded only while timing is enabled:
// mark(0) search start, mark(1) / mark(2) around the candidate scan,
// mark(3) search end.
struct EventTimer {
  cudaStream_t stream;
  bool on;
  cudaEvent_t ev[4] = {};
  explicit EventTimer(cudaStream_t s) : stream(s), on(timing_enabled()) {
    if (on)
      for (auto& e : ev) cudaEventCreate(&e);
  }
  ~EventTimer() {
    if (on)
      for (auto& e : ev) cudaEventDestroy(e);
  }
  void mark(int i) {
    if (on) cudaEventRecord(ev[i], stream);
  }
  // Elapsed ms between two recorded marks (0 if either was not recorded).
  double ms(int a, int b) {
    if (!on) return 0;
    float t = 0;
    if (cudaEventQuery(ev[a]) != cudaSuccess || cudaEventQuery(ev[b]) != cudaSuccess) {
      cudaGetLastError();
      return 0;
    }
    if (cudaEventElapsedTime(&t, ev[a], ev[b]) != cudaSuccess) {
      cudaGetLastError();
      return 0;
    }
    return t;
  }
};


#define XVEC_CUDA(expr)                                                                       \
  do {                                                                                        \
    cudaError_t err__ = (expr);                                                               \
    if (err__ != cudaSuccess) {                                                               \
      ::xvec::set_error("%s:%d %s: %s", __FILE__, __LINE__, #expr, cudaGetErrorString(err__)); \
      return err__ == cudaErrorMemoryAllocation ? XVEC_GPU_OUT_OF_MEMORY                      \
                                                : XVEC_GPU_CUDA_ERROR;                        \
    }                                                                                         \
  } while (0)

// Growable device array.
struct DeviceBuffer {
  void* ptr = nullptr;
  size_t bytes = 0;
  ~DeviceBuffer() {
    if (ptr) cudaFree(ptr);
  }
  // Grows to at least `need` bytes keeping the first `keep` bytes.
  xvec_gpu_status reserve(size_t need, size_t keep, cudaStream_t stream);
  template <typename T>
  T* as() const {
    return static_cast<T*>(ptr);
  }
};

// Stream-ordered scratch allocation that frees itself.
struct Scratch {
  void* ptr = nullptr;
  cudaStream_t stream = nullptr;
  Scratch() = default;
  Scratch(const Scratch&) = delete;
  Scratch& operator=(const Scratch&) = delete;
  ~Scratch() {
    if (ptr) cudaFreeAsync(ptr, stream);
  }
  xvec_gpu_status alloc(size_t bytes, cudaStream_t s);
  template <typename T>
  T* as() const {
    return static_cast<T*>(ptr);
  }
};

// One launch of a tensor-core candidate scan over rows [b, e) into lists
// [list0, list0 + 2 * parts) of `lists` per query (flat_tc.cuh).
using TcScanLaunch = std::function<cudaError_t(int64_t b, int64_t e, int parts, int list0,
                                               int lists, unsigned long long* gthr,
                                               uint64_t* cand, int* counts, uint64_t* sat)>;
// Runs the scan over all n rows as seeding launches over growing prefixes
// (each followed by a threshold seeding) and one launch over the rest;
// allocates the lists and reports their number per query.  gthr_out
// (optional) keeps the per-query shared thresholds for the merge's filter.
// preseed (optional): lowers the fresh thresholds before the first launch
// (flat_kernels.cuh, launch_flat_sample_seed); it runs only when the scan
// has seeding launches, whose lists would otherwise start empty.
using TcPreseed = std::function<cudaError_t(unsigned long long* gthr)>;
xvec_gpu_status tc_seeded_scan(int device, int nq, int64_t n, int kp, cudaStream_t s,
                               const TcScanLaunch& scan, Scratch& pkeys, Scratch& pcounts,
                               Scratch& psat, int* lists_out, Scratch* gthr_out = nullptr,
                               const TcPreseed& preseed = TcPreseed());

// Streaming Flat candidate scan for a few queries (flat_stream.cu): a sample
// pass over every 64th row for the starting thresholds, the pass over all
// rows, and one candidate list per query (lkeys [nq][flat_stream_list_stride(kp)],
// lcounts [nq], lsat [nq]) for the merge.
int flat_stream_max_batch();
int flat_stream_list_stride(int kp);
template <typename RowT>
bool flat_stream_supported(int nq, int64_t n, int d, int kp, const void* rows, const void* q);
template <typename RowT>
xvec_gpu_status flat_stream_scan(int device, const RowT* rows, int64_t n, int d,
                                 const float* row_n2, const uint32_t* keyrank, const float* qf,
                                 const float* q_n2, int nq, int metric, const uint32_t* bitmap,
                                 int kp, cudaStream_t s, Scratch& lkeys, Scratch& lcounts,
                                 Scratch& lsat, int* q_flags);

// A sharded search's exchange of per-query fast-rank bands (comm.cu): set by
// the sharded search for one shard's Flat search, which calls it once
// between its scan and its merge with `count` floats per rank (every rank
// calls it exactly once per search, also when its own search failed).
struct BandExchange {
  int nranks = 1;
  bool used = false;
  // All-gathers count floats of send from every rank into recv
  // [nranks][count]; bounded (XVEC_GPU_TIMEOUT / XVEC_GPU_NCCL_ERROR).
  std::function<xvec_gpu_status(const float* send, float* recv, size_t count, cudaStream_t s)>
      allgather;
};

// MergeSearchResults of `parts` lists per query (merge.cu): part p's keys,
// scores and counts start p * key_stride, p * score_stride and p *
// count_stride elements in (query q's list at q * top_k inside a part).
xvec_gpu_status launch_merge_results(int metric, int top_k, int nq, int parts,
                                     const uint64_t* keys, int64_t key_stride,
                                     const float* scores, int64_t score_stride,
                                     const int* counts, int64_t count_stride,
                                     uint64_t* out_keys, float* out_scores, int* out_counts,
                                     cudaStream_t stream);

// The search entry points' shared steps (capi.cu).
xvec_gpu_status validate_search(xvec_gpu_index* idx, int nq, const xvec_gpu_search_opts* o);
xvec_gpu_status search_device_locked(xvec_gpu_index* idx, const void* d_q, int nq,
                                     const xvec_gpu_search_opts& o, const uint32_t* d_bitmap,
                                     uint64_t* d_keys, float* d_scores, int* d_counts,
                                     cudaStream_t s, std::vector<int>* statuses,
                                     BandExchange* band = nullptr);
size_t query_elem_bytes(const xvec_gpu_index* idx);
// The caller's cancel flag (opts.cancel_flag) is set.
bool is_cancelled(const xvec_gpu_search_opts& o);

}  // namespace xvec

struct xvec_gpu_index {
  xvec_gpu_index_desc desc{};
  int device = 0;
  std::shared_mutex mu;  // search: shared, add/set_model: exclusive (flat.go:70-77)
  int64_t n = 0;
  int64_t capacity = 0;
  size_t row_bytes = 0;  // bytes of one stored row

  // Common per-row state.
  xvec::DeviceBuffer rows;       // FLAT: float/half rows; SQ8/RABITQ/IVF_PQ: float32 originals
  xvec::DeviceBuffer keys;       // uint64
  xvec::DeviceBuffer row_n2;     // float reference-order ||x||^2
  xvec::DeviceBuffer row_inv;    // float 1/||x|| (0 for a zero row), tensor-core epilogue
  xvec::DeviceBuffer keyrank;    // uint32: position -> rank of its key
  xvec::DeviceBuffer pos_of_kr;  // uint32: key rank -> position
  xvec::DeviceBuffer max_n2;     // unsigned (ordered float) max ||x||^2

  // SQ8.
  xvec::DeviceBuffer sq_codes;   // int8 [n][d]
  xvec::DeviceBuffer sq_params;  // {float inv_scale, float offset, double sum, double square}
  xvec::DeviceBuffer sq_fast;    // float4 {inv_scale, offset, code sum, ||decoded||^2}
  xvec::DeviceBuffer sq_bounds;  // 4 ordered floats: error-bound maxima over rows

  // IVF-PQ.
  int32_t nlist = 0, chunks = 0;
  xvec_gpu_index* probe_index = nullptr;  // Flat index over the IVF centroids
  bool has_model = false;
  xvec::DeviceBuffer centroids;     // float [nlist][d]
  xvec::DeviceBuffer centroid_n2;   // float [nlist]
  xvec::DeviceBuffer pivots;        // float [256][d]
  xvec::DeviceBuffer chunk_offsets; // int [chunks+1]
  xvec::DeviceBuffer pq_codes;      // uint8 [n][chunks]
  xvec::DeviceBuffer row_list;      // int32 [n] list of each row
  xvec::DeviceBuffer list_offsets;  // int64 [nlist+1] CSR over positions
  xvec::DeviceBuffer list_rows;     // uint32 [n] positions grouped by list (insertion order)
  xvec::DeviceBuffer list_codes;    // uint8 [n][chunks] the PQ codes in list_rows order
  xvec::DeviceBuffer list_keyrank;  // uint32 [n] key ranks in list_rows order
  // The codes again for the fast scan, 32 G chunk slots per code: code i of
  // a list holds at byte t its chunk (i mod 32 + t) mod 32 G (zero past the
  // last chunk).
  xvec::DeviceBuffer list_codes_t;  // uint8 [n][32 G] in list_rows order
  // IVF-SQ8 (d % 16 == 0): the INT8 codes in list_rows order, interleaved by
  // 32-row groups: 16-byte chunk c of list entry i at chunk index
  // ((i / 32) (d / 16) + c) 32 + i mod 32; the float4 rank terms in list order.
  xvec::DeviceBuffer list_sq_codes;
  xvec::DeviceBuffer list_sq_fast;
  // IVF-Flat (d % 4 == 0): the float32 rows in list_rows order, interleaved
  // the same way by float4 chunks (chunk c of entry i at ((i / 32) (d / 4) +
  // c) 32 + i mod 32), and their reference-order ||x||^2 in list order.
  xvec::DeviceBuffer list_rows_f;
  xvec::DeviceBuffer list_n2;
  bool lists_dirty = true;

  // RaBitQ (one-bit).
  int32_t rq_clusters = 0, padded = 0;
  xvec::DeviceBuffer rq_centroids;          // float [c][d]
  xvec::DeviceBuffer rq_rot_centroids;      // float [c][padded]
  xvec::DeviceBuffer rq_signs;              // uint8 [4*padded/8]
  xvec::DeviceBuffer rq_codes;              // uint8 [n][padded/8]
  xvec::DeviceBuffer rq_factors;            // {double add, rescale, error, full add,
                                            //  full rescale; int cluster} [n]
  xvec::DeviceBuffer rq_fast;               // float4 {add, rescale, cluster bits, 0} [n]
                                            // (multi-bit: the full add and rescale)
  // Multi-bit models (RaBitQModelState.TotalBits > 1, ExtraScale): the full
  // code values v = extra | sign bit << (TotalBits - 1) per padded coordinate
  // as 16-bit floats [n][padded] (bfloat16 up to 8 bits, binary16 for 9;
  // exact either way): the tensor-core operand and the exact scorer's input.
  // IVF rows added with their lists given (xvec_gpu_ivf_add_with_lists): the
  // batch's lists on the device while it is committed, else null.
  const int32_t* given_lists = nullptr;
  int32_t rq_total_bits = 1;
  double rq_extra_scale = 0.0;
  xvec::DeviceBuffer rq_values;
  // HNSW-RaBitQ graph (xvec_gpu_rabitq_set_graph) over hnsw_n positions:
  // levels 0..hnsw_max_level (-1: none), node p's level-L neighbours at
  // hnsw_nbrs[hnsw_offsets[L (hnsw_n + 1) + p] .. hnsw_offsets[L (hnsw_n + 1) + p + 1]).
  int32_t hnsw_max_level = -1;
  int64_t hnsw_entry = 0, hnsw_n = 0;
  xvec::DeviceBuffer hnsw_offsets;          // int64
  xvec::DeviceBuffer hnsw_nbrs;             // int32
  // DiskANN: the PQ model in pivots / chunk_offsets / chunks (has_model),
  // the codes of the prepared rows in pq_codes, their MIPSL2 norms, and the
  // graph (xvec_gpu_diskann_set_graph): node p's neighbours at
  // dk_nbrs[dk_offsets[p] .. dk_offsets[p + 1]); dk_entry -1: no graph over
  // the current rows.
  int64_t dk_entry = -1;
  int32_t dk_beam = 1, dk_max_degree = 0;
  xvec::DeviceBuffer dk_norms;              // float [n]
  xvec::DeviceBuffer dk_offsets;            // int64 [n + 1]
  xvec::DeviceBuffer dk_nbrs;               // int32
  // TotalBits 2..8: the code values again as int8 v - 128 [n][padded] (the
  // INT8 tensor-core operand); rq_fast's w slot holds 128 sum(v - 128).
  xvec::DeviceBuffer rq_vplane;
  // Flat FP32: the rows as bfloat16 high and low parts (the tensor-core
  // scan's operands; the float32 rows stay the reference data).
  xvec::DeviceBuffer rows_bhi;              // bf16 [n][d]
  xvec::DeviceBuffer rows_blo;              // bf16 [n][d]
  xvec::DeviceBuffer rq_planes;             // int8 [n][2 padded] (127 b | b): the tensor-core operand
  xvec::DeviceBuffer rq_bounds;             // ordered floats: max |add|, |rescale|, error

  ~xvec_gpu_index() {
    if (probe_index) xvec_gpu_index_destroy(probe_index);
  }
};
