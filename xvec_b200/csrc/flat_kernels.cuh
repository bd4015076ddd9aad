// flat_kernels.cuh — launchers of the Flat search kernels (flat_kernels.cu).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace xvec {

template <typename QT>
void launch_prep_queries(const QT* q, int nq, int d, int metric, float* qf, float* q_n2,
                         float* q_aux, int* q_status, cudaStream_t stream);

template <typename RowT>
void launch_row_norms(const RowT* rows, int64_t n, int d, float* n2, float* inv_mag,
                      unsigned* max_n2, int* nonfinite, cudaStream_t stream);

// Capacity of the per-query accumulator buffers for a retained-list size kp.
int simt_cap_for(int kp);
// Union entries per query the merge kernel can hold (parts x kp must fit).
int flat_merge_capacity();

// Per query, lowers gthr[q] to the kp-th smallest key over lists
// [0, seed_lists) (cand: [nq][num_lists][cap], counts: [nq][num_lists]) when
// those lists hold at least kp keys together.  Any kp keys of the query bound
// its final kp-th best from above, so the result is a valid shared threshold
// for the lists filled afterwards.  seed_lists * kp <= flat_merge_capacity().
cudaError_t launch_seed_thresholds(const uint64_t* cand, const int* counts, int nq, int num_lists,
                                   int seed_lists, int cap, int kp, unsigned long long* gthr,
                                   cudaStream_t stream);
int exact_cap_for(int kp);

// Sample seeding of the tensor-core scan's shared thresholds (before its
// first launch): per query, the kp-th best FP32 fast rank over `samples` rows
// evenly spaced over the base (filtered rows left out), plus the sample's and
// the scan's error bounds (split: the scan ranks bfloat16 high/low parts),
// lowers gthr[q] to a bound on its kp-th best scan key over all rows.
// ranks: nq x samples uint32 of scratch.  flat_sample_seed_rows gives the
// sample size for n rows and kp (0: the base is too small to seed this way).
int flat_sample_seed_rows(int64_t n, int kp);
template <typename RowT>
cudaError_t launch_flat_sample_seed(const RowT* rows, int64_t n, int d, const float* row_n2,
                                    const uint32_t* bitmap, const float* qf, const float* q_n2,
                                    int nq, int metric, int kp, const unsigned* max_n2, int split,
                                    int samples, uint32_t* ranks, unsigned long long* gthr,
                                    cudaStream_t stream);

template <typename RowT>
cudaError_t launch_flat_scan_simt(const RowT* rows, int64_t n, int d, const float* row_n2,
                                  const uint32_t* keyrank, const float* qf, const float* q_n2,
                                  int nq, const uint32_t* bitmap, int metric, int num_parts,
                                  int kp, uint64_t* part_keys, int* part_counts,
                                  uint64_t* part_sat, int* q_flags, cudaStream_t stream);

template <typename RowT>
cudaError_t launch_flat_scan_exact(const RowT* rows, int64_t n, int d, const uint32_t* keyrank,
                                   const float* qf, const int* query_ids, int nlist,
                                   const uint32_t* bitmap, int metric, int num_parts, int kp,
                                   uint64_t* part_keys, int* part_counts, uint64_t* part_sat,
                                   int* q_flags, cudaStream_t stream);

template <typename RowT>
cudaError_t launch_flat_merge_rescore(const RowT* rows, int d, const uint32_t* pos_of_keyrank,
                                      const uint64_t* keys, const float* qf, const float* q_n2,
                                      const unsigned* max_n2, const int* query_ids, int nlist,
                                      int metric, int k, float radius, int exact_mode,
                                      const uint64_t* part_keys, const int* part_counts,
                                      const uint64_t* part_sat, int num_parts, int stride,
                                      uint64_t* out_keys, float* out_scores, int* out_counts,
                                      int* q_flags, cudaStream_t stream, int split_eps = 0,
                                      const unsigned long long* gthr = nullptr,
                                      const float* band = nullptr);

// A sharded search's band (pipeline.cuh): this shard's k best fast ranks
// and eps per query into out [nq][k + 1]; then, from every shard's, the
// per-query rank limit (NaN: none).
template <typename RowT>
cudaError_t launch_flat_band_prepare(const RowT* rows, int d, const float* qf, const float* q_n2,
                                     const unsigned* max_n2, int nq, int metric, int k,
                                     const uint64_t* part_keys, const int* part_counts,
                                     int num_parts, int stride, const unsigned long long* gthr,
                                     float* out, cudaStream_t stream, int split_eps = 0);
bool flat_band_supported(int nranks, int k);
cudaError_t launch_flat_band_limit(const float* recv, int nranks, int nq, int k,
                                   const float* own, float* band, cudaStream_t stream);

}  // namespace xvec
