/*
 * xvec_oracle.h — CPU restatement of the xvec search hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the shipped library links, loads or
 * calls this code: it exists so that tests, the smoke check and the CPU
 * baseline leg of bench.py can compare the CUDA path against the reference
 * algorithm.  Every function cites the reference file:line it restates
 * (paths are relative to the gorse-io/xvec module root).
 *
 * Parity pin: the restatement is checked against (a) the reference's own
 * known-answer tests (tests/golden/) and (b) the reference's AVX-512/AVX C
 * kernels (internal/floats/src/floats_avx512.c, floats_avx.c) compiled in
 * place into oracle/_ref/ by `make -C oracle ref`.
 */
#ifndef XVEC_ORACLE_H
#define XVEC_ORACLE_H

#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes: identical values to include/xvec_gpu.h. */
enum {
  XO_OK = 0,
  XO_INVALID_ARGUMENT = 1,
  XO_NON_FINITE = 7,
  XO_OVERFLOW = 8,
  XO_MISSING = 9,
};

/* Metric values mirror internal/core/metric/metric.go:26-31. */
enum { XO_L2 = 1, XO_IP = 2, XO_COSINE = 3, XO_MIPSL2 = 4 };

/* ---- internal/floats: dispatch of floats_amd64.go:27-91 ---------------- */
/* Routes the >=16 (AVX-512) and >=8 (AVX) cases to the reference's own
 * compiled kernels (function pointers from oracle/_ref); NULLs restore the
 * restatement. */
void xo_use_reference_kernels(void* l2_512, void* ip_512, void* dn_512, void* l2_256,
                              void* ip_256, void* dn_256);
float xo_l2_squared(const float* left, const float* right, int64_t n);
float xo_inner_product(const float* left, const float* right, int64_t n);
void xo_dot_norms(const float* left, const float* right, int64_t n, float* dot,
                  float* left_norm, float* right_norm);

/* ---- internal/ailego/math + metric.Compute --------------------------- */
int xo_metric_compute(int metric, const float* left, const float* right, int64_t n,
                      float* score);
int xo_cosine_with_magnitudes(const float* left, const float* right, int64_t n,
                              float left_mag, float right_mag, float* score);
int xo_l2_magnitude(const float* v, int64_t n, float* mag);

/* ---- FP16 (internal/ailego/utility/float_helper.go) -------------------- */
uint16_t xo_f32_to_f16(float value);
float xo_f16_to_f32(uint16_t bits);

/* ---- Flat exact search: DenseFlatIndex.SearchWithOptions per query ----
 * rows: n*d float32 row-major, keys: n.  filter_bitmap: NULL or a bitmap
 * over positions (bit p of word p/32 set = candidate passes Filter).
 * Outputs are nq*k; out_counts[q] = number of results for query q.
 * Returns the first error over the queries (per-query status in
 * out_status when not NULL). */
int xo_flat_search(int metric, const float* rows, const uint64_t* keys, int64_t n,
                   int32_t d, const float* queries, int32_t nq, int32_t k, float radius,
                   const uint32_t* filter_bitmap, int32_t threads, uint64_t* out_keys,
                   float* out_scores, int32_t* out_counts, int32_t* out_status);

/* ---- MergeSearchResults (internal/core/query.go:154-191) -------------- */
int32_t xo_merge_results(int metric, int32_t k, const uint64_t* keys, const float* scores,
                         int64_t count, uint64_t* out_keys, float* out_scores);

/* ---- Scalar quantization (internal/core/quantization.go) --------------- */
typedef struct {
  float inverse_scale;
  float offset;
  double code_sum;
  double code_square;
} xo_sq_params;

int xo_quantize_int8(const float* v, int32_t d, int8_t* codes, xo_sq_params* params);
/* xo_quantize_int8 over n rows [n*d] (threads > 1: rows split across threads). */
int xo_quantize_int8_batch(const float* rows, int64_t n, int32_t d, int32_t threads,
                           int8_t* codes, xo_sq_params* params);
int xo_quantize_int4(const float* v, int32_t d, uint8_t* packed, xo_sq_params* params);
int xo_quantize_int4_batch(const float* rows, int64_t n, int32_t d, int32_t threads,
                           uint8_t* packed, xo_sq_params* params);
int xo_quantized_distance_int4(int metric, const uint8_t* left, const xo_sq_params* lp,
                               const uint8_t* right, const xo_sq_params* rp, int32_t d,
                               float* score);
int xo_quantized_distance_int8(int metric, const int8_t* left, const xo_sq_params* lp,
                               const int8_t* right, const xo_sq_params* rp, int32_t d,
                               float* score);
int xo_refinement_candidate_count(int32_t top_k, float scale_factor, int32_t* count);

/* SQ-Flat (+ optional OriginalVectorRefiner) search over the whole index
 * (quantized_index.go:113-120, 296-335; collection.go:1606-1631).  When
 * refine_scale > 0 the quantized stage retrieves RefinementCandidateCount
 * candidates without radius and the exact fp32 refiner produces top-k. */
int xo_sq8_search(int metric, const int8_t* codes, const xo_sq_params* params,
                  const float* originals, const uint64_t* keys, int64_t n, int32_t d,
                  const float* queries, int32_t nq, int32_t k, float radius,
                  float refine_scale, const uint32_t* filter_bitmap, int32_t threads,
                  uint64_t* out_keys, float* out_scores, int32_t* out_counts,
                  int32_t* out_status);
/* xo_sq8_search over INT4 codes (packed d / 2 bytes per row). */
int xo_sq4_search(int metric, const uint8_t* codes, const xo_sq_params* params,
                  const float* originals, const uint64_t* keys, int64_t n, int32_t d,
                  const float* queries, int32_t nq, int32_t k, float radius,
                  float refine_scale, const uint32_t* filter_bitmap, int32_t threads,
                  uint64_t* out_keys, float* out_scores, int32_t* out_counts,
                  int32_t* out_status);

/* ---- k-means (internal/core/kmeans.go) --------------------------------- */
uint64_t xo_splitmix64_next(uint64_t* state);
int xo_kmeans_reservoir(int64_t n, int32_t clusters, uint64_t seed, int64_t* indices);
int xo_kmeans_assign(int metric, const float* vectors, int64_t n, const float* centroids,
                     int32_t nc, int32_t d, int32_t threads, int32_t* labels, float* scores);
/* Full Lloyd training (kmeans.go:208-298 + algorithm/lloyd_cluster.go). */
int xo_kmeans_train(int metric, const float* vectors, int64_t n, int32_t d, int32_t clusters,
                    int32_t max_iterations, double tolerance, uint64_t seed, int32_t threads,
                    float* centroids_out, int32_t* clusters_out, int32_t* labels_out);

/* ---- IVF probe + list scans --------------------------------------------- */
/* probedListsLocked (ivf.go:524-561): top-nprobe centroids of one query. */
int32_t xo_ivf_probe(int metric, const float* centroids, int32_t nlist, int32_t d,
                     const float* query, int32_t nprobe, int32_t* lists);
/* IVF exact search (ivf.go:427-493) over CSR lists of positions. */
int xo_ivf_flat_search(int metric, const float* rows, const uint64_t* keys, int64_t n,
                       int32_t d, const float* centroids, int32_t nlist,
                       const int64_t* list_offsets, const int64_t* list_positions,
                       const float* queries, int32_t nq, int32_t k, int32_t nprobe,
                       float radius, const uint32_t* filter_bitmap, int32_t threads,
                       uint64_t* out_keys, float* out_scores, int32_t* out_counts,
                       int32_t* out_status);
/* ScalarQuantizedIVFIndex search (ivf_quantized.go:135-192): the IVF probe,
 * INT8 scoring of the probed positions, optional refine (refine_scale > 0). */
int xo_ivf_sq8_search(int metric, const int8_t* codes, const xo_sq_params* params,
                      const float* originals, const uint64_t* keys, int64_t n, int32_t d,
                      const float* centroids, int32_t nlist, const int64_t* list_offsets,
                      const int64_t* list_positions, const float* queries, int32_t nq, int32_t k,
                      int32_t nprobe, float radius, float refine_scale,
                      const uint32_t* filter_bitmap, int32_t threads, uint64_t* out_keys,
                      float* out_scores, int32_t* out_counts, int32_t* out_status);

/* TrainKMeans with InitialCentroids (kmeans.go:354-363): kc given centroids. */
int xo_kmeans_train_init(int metric, const float* vectors, int64_t n, int32_t d, int32_t kc,
                         const float* initial, int32_t max_iterations, double tolerance,
                         int32_t threads, float* centroids_out, int32_t* labels_out);

/* ---- Product quantization (internal/core/pq.go) ------------------------ */
/* initializePQKMC2 (pq.go:410-459). */
int xo_pq_kmc2(int metric, const float* vectors, int64_t n, int32_t d, int32_t clusters,
               uint64_t seed, float* centroids_out);
/* TrainPQ (pq.go:107-179): pivots [256][d]. */
int xo_pq_train(int metric, const float* vectors, int64_t n, int32_t d, int32_t chunks,
                int64_t max_train_samples, int32_t max_iterations, uint64_t seed,
                int32_t threads, float* pivots_out);
void xo_pq_chunk_offsets(int32_t d, int32_t chunks, int32_t* offsets);
int xo_pq_encode(int metric, const float* pivots, const int32_t* offsets, int32_t chunks,
                 int32_t d, const float* v, uint8_t* code);
int xo_pq_distance_table(int metric, const float* pivots, const int32_t* offsets,
                         int32_t chunks, int32_t d, const float* query, float* table);
int xo_pq_lookup(const float* table, int32_t chunks, const uint8_t* code, float* score);
/* IVF-PQ (composed from probedListsLocked + PQDistanceTable.Lookup + the
 * topk.go heap rules): see the definition for the exact composition. */
int xo_ivfpq_search(int metric, const float* centroids, int32_t nlist, int32_t d,
                    const float* pivots, const int32_t* offsets, int32_t chunks,
                    const uint8_t* codes, const uint64_t* keys,
                    const int64_t* list_offsets, const int64_t* list_positions,
                    const float* queries, int32_t nq, int32_t k, int32_t nprobe,
                    float radius, const uint32_t* filter_bitmap, int32_t threads,
                    uint64_t* out_keys, float* out_scores, int32_t* out_counts,
                    int32_t* out_status);

/* ---- RaBitQ (internal/core/rabitq*.go, rotation.go, ailego/math/fht.go) - */
int xo_fht_rotate(int32_t dimension, const uint8_t* signs, const float* in, float* out);
/* FHTRotator.Unrotate (rotation.go:155-185). */
int xo_fht_unrotate(int32_t dimension, const uint8_t* signs, const float* in, float* out);
int32_t xo_rabitq_padded_dimension(int32_t d);
/* Padded rotation used by RaBitQModel (rabitq.go:555-577). */
int xo_rabitq_rotate(int32_t d, const uint8_t* signs, const float* in, float* out);
typedef struct {
  int32_t cluster;
  int32_t pad_;
  double coarse_add;
  double coarse_rescale;
  double coarse_error;
  double full_add;
  double full_rescale;
} xo_rabitq_factors;
int xo_rabitq_quantize(const float* rotated, const float* rotated_centroid, int32_t padded,
                       int32_t cluster, int32_t total_bits, double extra_scale,
                       int32_t inner_product, uint8_t* binary_code, uint8_t* extra_code,
                       xo_rabitq_factors* factors);
/* RaBitQModel.Encode (rabitq.go:297-327) for TotalBits = 1. */
int xo_rabitq_encode1(int metric, int32_t d, const float* centroids, int32_t nc,
                      const uint8_t* signs, const float* v, uint8_t* binary_code,
                      xo_rabitq_factors* factors);
/* RaBitQModel.Encode with TotalBits and ExtraScale; extra_code holds
 * (padded (total_bits - 1) + 7) / 8 bytes (unused for one bit). */
int xo_rabitq_encode(int metric, int32_t d, const float* centroids, int32_t nc,
                     const uint8_t* signs, int32_t total_bits, double extra_scale, const float* v,
                     uint8_t* binary_code, uint8_t* extra_code, xo_rabitq_factors* factors);
/* PrepareQuery (rabitq.go:372-408): rotated query (padded), sum, gAdd, gError. */
int xo_rabitq_prepare_query(int metric, int32_t d, const float* centroids, int32_t nc,
                            const uint8_t* signs, const float* query, float* rotated,
                            double* sum, double* g_add, double* g_error);
/* EstimateCoarse (rabitq.go:421-430), distance part. */
int xo_rabitq_estimate_coarse(const float* rotated, int32_t padded, double sum,
                              const double* g_add, const double* g_error,
                              const uint8_t* binary_code, const xo_rabitq_factors* factors,
                              float* distance);
/* Estimate (rabitq.go:434-446): the coarse estimate for one bit, else the
 * full-code estimate. */
int xo_rabitq_estimate(const float* rotated, int32_t padded, double sum, const double* g_add,
                       const double* g_error, int32_t total_bits, const uint8_t* binary_code,
                       const uint8_t* extra_code, const xo_rabitq_factors* factors,
                       float* distance);
/* xo_rabitq_search with TotalBits (extra_codes: per row
 * (padded (total_bits - 1) + 7) / 8 bytes). */
int xo_rabitq_search_bits(int metric, int32_t d, const float* centroids, int32_t nc,
                          const uint8_t* signs, int32_t total_bits, const uint8_t* binary_codes,
                          const uint8_t* extra_codes, const xo_rabitq_factors* factors,
                          const float* originals, const uint64_t* keys, int64_t n,
                          const float* queries, int32_t nq, int32_t k, int32_t candidate_count,
                          int32_t refine, float radius, const uint32_t* filter_bitmap,
                          int32_t threads, uint64_t* out_keys, float* out_scores,
                          int32_t* out_counts, int32_t* out_status);
/* Composed linear RaBitQ scan (hnsw_rabitq.go:539-642, 739-801): with refine,
 * min(n, max(k, candidate_count)) estimates refined to the exact top-k;
 * without, the k best estimates with the public score. */
int xo_rabitq_search(int metric, int32_t d, const float* centroids, int32_t nc,
                     const uint8_t* signs, const uint8_t* binary_codes,
                     const xo_rabitq_factors* factors, const float* originals,
                     const uint64_t* keys, int64_t n, const float* queries, int32_t nq,
                     int32_t k, int32_t candidate_count, int32_t refine, float radius,
                     const uint32_t* filter_bitmap, int32_t threads, uint64_t* out_keys,
                     float* out_scores, int32_t* out_counts, int32_t* out_status);


/* HNSW-RaBitQ graph search (hnsw_rabitq.go:589-801) over a given graph: node
 * p's level-L neighbours at neighbors[offsets[L (n+1) + p] .. offsets[L (n+1) + p + 1]).
 * Results as xo_rabitq_search_bits. */
int xo_hnsw_rabitq_search(int metric, int32_t d, const float* centroids, int32_t nc,
                          const uint8_t* signs, int32_t total_bits, const uint8_t* binary_codes,
                          const uint8_t* extra_codes, const xo_rabitq_factors* factors,
                          const float* originals, const uint64_t* keys, int64_t n,
                          int32_t max_level, int64_t entry, const int64_t* offsets,
                          const int32_t* neighbors, const float* queries, int32_t nq, int32_t k,
                          int32_t ef, int32_t refine, float radius, const uint32_t* bitmap,
                          int32_t threads, uint64_t* out_keys, float* out_scores,
                          int32_t* out_counts, int32_t* out_status);

/* Threaded batch forms of xo_pq_encode and xo_rabitq_encode (codes [n][chunks];
 * sign bits [n][padded/8], extra codes [n][extra_stride] with extra_stride >= 1,
 * factors [n]); the first failing row's status. */
int xo_pq_encode_rows(int metric, const float* pivots, const int32_t* offsets, int32_t chunks,
                      int32_t d, const float* rows, int64_t n, int32_t threads, uint8_t* codes);
int xo_rabitq_encode_rows(int metric, int32_t d, const float* centroids, int32_t nc,
                          const uint8_t* signs, int32_t total_bits, double extra_scale,
                          const float* rows, int64_t n, int32_t threads, uint8_t* binary_codes,
                          uint8_t* extra_codes, int64_t extra_stride, xo_rabitq_factors* factors);

/* diskANNPQCodeNorms (diskann.go:292-323): float32 of the float64 sum of the
 * squared pivot components of each code, chunk by chunk. */
void xo_diskann_code_norms(const float* pivots, const int32_t* offsets, int32_t chunks, int32_t d,
                           const uint8_t* codes, int64_t n, float* norms);

/* DiskANN graph search with the PQ frontier (diskann.go:472-525, 559-683)
 * over a given graph: node p's neighbours at neighbors[graph_offsets[p] ..
 * graph_offsets[p + 1]), its vector at vectors[p d], its PQ code (of the
 * prepared vector under the traversal metric) at codes[p chunks], code_norms
 * for MIPSL2 (else unused).  beam = diskANNReadBatchSize.  Results as
 * xo_flat_search. */
int xo_diskann_search(int metric, int32_t d, const float* pivots, const int32_t* offsets,
                      int32_t chunks, const uint8_t* codes, const float* code_norms,
                      const float* vectors, const uint64_t* keys, int64_t n, int64_t entry,
                      const int64_t* graph_offsets, const int32_t* neighbors, int32_t beam,
                      const float* queries, int32_t nq, int32_t k, int32_t list_size,
                      float radius, const uint32_t* bitmap, int32_t threads, uint64_t* out_keys,
                      float* out_scores, int32_t* out_counts, int32_t* out_status);

#ifdef __cplusplus
}
#endif
#endif /* XVEC_ORACLE_H */
