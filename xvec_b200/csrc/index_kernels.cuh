// index_kernels.cuh — per-index-kind hooks used by capi.cu.
#pragma once

#include <vector>

#include "capi_internal.h"

namespace xvec {

// Extra per-row storage for the quantized index kinds (grown with capacity).
xvec_gpu_status extra_reserve(xvec_gpu_index* idx, int64_t capacity, cudaStream_t s);
// Checks that rows [old_n, old_n + m) can be committed (models present, ...).
xvec_gpu_status extra_validate(xvec_gpu_index* idx, int64_t old_n, int64_t m, cudaStream_t s);
// Encodes rows [old_n, old_n + m) (quantize / assign / PQ-encode / RaBitQ).
xvec_gpu_status extra_commit(xvec_gpu_index* idx, int64_t old_n, int64_t m, cudaStream_t s);

xvec_gpu_status sq8_reserve(xvec_gpu_index* idx, int64_t capacity, cudaStream_t s);
xvec_gpu_status sq8_commit(xvec_gpu_index* idx, int64_t old_n, int64_t m, cudaStream_t s);

xvec_gpu_status ivfpq_reserve(xvec_gpu_index* idx, int64_t capacity, cudaStream_t s);
xvec_gpu_status ivfpq_commit(xvec_gpu_index* idx, int64_t old_n, int64_t m, cudaStream_t s);

// IVF helpers shared by the IVF kinds (ivfpq.cu): the nearest centroid of
// each row through a Flat index over the centroids (keys = centroid index),
// that index, and the CSR lists of positions (+ key ranks in list order).
xvec_gpu_status assign_rows(xvec_gpu_index* probe, const float* d_rows, int64_t n, int d,
                            int32_t* d_labels, float* d_scores, cudaStream_t s);
xvec_gpu_status make_probe_index(int device, int metric, int d, const float* d_centroids,
                                 int nlist, cudaStream_t s, xvec_gpu_index** out);
xvec_gpu_status rebuild_lists(xvec_gpu_index* idx, cudaStream_t s);

xvec_gpu_status ivf_probe(xvec_gpu_index* idx, const float* d_q, int nq, int nprobe,
                          const float* qf, const float* qn2, const int* q_status,
                          uint64_t* pkeys, float* pscores, int* pcounts, int* q_flags,
                          std::vector<int>* h_status, cudaStream_t s);
xvec_gpu_status ivf_flat_reserve(xvec_gpu_index* idx, int64_t capacity, cudaStream_t s);
xvec_gpu_status ivf_flat_commit(xvec_gpu_index* idx, int64_t old_n, int64_t m, cudaStream_t s);
xvec_gpu_status ivf_flat_search_impl(xvec_gpu_index* idx, const float* d_q, int nq,
                                     const xvec_gpu_search_opts& o, const uint32_t* d_bitmap,
                                     uint64_t* d_keys, float* d_scores, int* d_counts,
                                     cudaStream_t s, std::vector<int>* statuses);

xvec_gpu_status ivf_sq8_search_impl(xvec_gpu_index* idx, const float* d_q, int nq,
                                    const xvec_gpu_search_opts& o, const uint32_t* d_bitmap,
                                    uint64_t* d_keys, float* d_scores, int* d_counts,
                                    cudaStream_t s, std::vector<int>* statuses,
                                    bool candidates_only = false);

// PQModel.Encode of n rows (block per row; err receives a status when a
// chunk score is not finite) and PQModel.DistanceTable of nq queries
// (q_flags |= 4 when a table entry is not finite), in ivfpq.cu.
cudaError_t launch_pq_encode(const float* rows, int64_t n, int d, int metric, const float* pivots,
                             const int* offsets, int chunks, uint8_t* codes, int* err,
                             cudaStream_t s);
cudaError_t launch_pq_table(const float* queries, int nq, int d, int metric, const float* pivots,
                            const int* offsets, int chunks, float* table, int* q_flags,
                            cudaStream_t s);

xvec_gpu_status diskann_reserve(xvec_gpu_index* idx, int64_t capacity, cudaStream_t s);
xvec_gpu_status diskann_commit(xvec_gpu_index* idx, int64_t old_n, int64_t m, cudaStream_t s);
xvec_gpu_status diskann_search_impl(xvec_gpu_index* idx, const float* d_q, int nq,
                                    const xvec_gpu_search_opts& o, const uint32_t* d_bitmap,
                                    uint64_t* d_keys, float* d_scores, int* d_counts,
                                    cudaStream_t s, std::vector<int>* statuses);

xvec_gpu_status rabitq_reserve(xvec_gpu_index* idx, int64_t capacity, cudaStream_t s);
xvec_gpu_status rabitq_commit(xvec_gpu_index* idx, int64_t old_n, int64_t m, cudaStream_t s);

// candidates_only (refined searches): stop after the approximate stage and
// write its candidates (up to the refine candidate count per query) with
// their ranks (lower is better) in place of scores.
xvec_gpu_status sq8_search_impl(xvec_gpu_index* idx, const float* d_q, int nq,
                                const xvec_gpu_search_opts& o, const uint32_t* d_bitmap,
                                uint64_t* d_keys, float* d_scores, int* d_counts, cudaStream_t s,
                                std::vector<int>* statuses, bool candidates_only = false);
xvec_gpu_status ivfpq_search_impl(xvec_gpu_index* idx, const float* d_q, int nq,
                                  const xvec_gpu_search_opts& o, const uint32_t* d_bitmap,
                                  uint64_t* d_keys, float* d_scores, int* d_counts,
                                  cudaStream_t s, std::vector<int>* statuses);
xvec_gpu_status rabitq_search_impl(xvec_gpu_index* idx, const float* d_q, int nq,
                                   const xvec_gpu_search_opts& o, const uint32_t* d_bitmap,
                                   uint64_t* d_keys, float* d_scores, int* d_counts,
                                   cudaStream_t s, std::vector<int>* statuses,
                                   bool candidates_only = false);
// Candidates per query of the approximate stage of a refined search (0 when
// the options ask for no refinement).
int sq8_candidate_count(const xvec_gpu_search_opts& o);
int rabitq_candidate_count(const xvec_gpu_search_opts& o);

}  // namespace xvec
