/*
 * xvec_gpu.h — C ABI of the B200 (sm_100a) search library for xvec.
 *
 * This is the boundary a cgo shim binds.  It takes plain
 * pointers and sizes only.  Each entry point names the reference interface it
 * replaces, by file:line in the gorse-io/xvec module.
 *
 * Conventions
 *   - Keys are uint64 (internal/core/topk.go:47-50, Result.Key); scores are
 *     float32 (Result.Score).  Results are best-first; ties are broken by the
 *     ascending key (resultBetter, internal/core/topk.go:271-276).
 *   - Metric values equal core.Metric (internal/core/metric/metric.go:26-31).
 *   - "host" entry points take host memory and copy it themselves; the
 *     *_device variants take device memory on the index's device and enqueue
 *     on the caller's stream.  The library never keeps a caller pointer after
 *     a call returns.
 *   - Every entry point returns an xvec_gpu_status; xvec_gpu_last_error()
 *     returns the message of the calling thread's last failure.  Nothing in
 *     the library aborts or exits the process.
 *   - Batched searches fill every query they can: out_counts[q] >= 0 is the
 *     number of results of query q, out_counts[q] < 0 is -(status) of a query
 *     that failed on its own (for example a non-finite query vector, like the
 *     per-query error of core.BatchTopK, internal/core/topk.go:257-262); the
 *     call then returns the first failing query's status.
 */
#ifndef XVEC_GPU_H
#define XVEC_GPU_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define XVEC_GPU_ABI_VERSION 4

typedef enum {
  XVEC_GPU_OK = 0,
  XVEC_GPU_INVALID_ARGUMENT = 1, /* ErrInvalidTopK, ErrInvalidRadius, ErrInvalidDimension, ... */
  XVEC_GPU_OUT_OF_MEMORY = 2,
  XVEC_GPU_CANCELLED = 3,        /* the caller's cancel flag was set (ctx.Err()) */
  XVEC_GPU_TIMEOUT = 4,          /* a bounded device-side wait gave up */
  XVEC_GPU_CUDA_ERROR = 5,
  XVEC_GPU_NCCL_ERROR = 6,
  XVEC_GPU_NON_FINITE = 7,       /* mathutil.ErrNonFiniteVector */
  XVEC_GPU_OVERFLOW = 8,         /* ErrQuantizationOverflow / ErrPQScoreOverflow */
  XVEC_GPU_NOT_FOUND = 9,        /* ErrMissingRefineVector */
  XVEC_GPU_DUPLICATE_KEY = 10,   /* ErrDuplicateKey */
  XVEC_GPU_UNSUPPORTED = 11,     /* no sm_100a device / feature not available */
  XVEC_GPU_CHECKSUM_MISMATCH = 12 /* ErrIVFChecksumMismatch (ivf.go:736-738) */
} xvec_gpu_status;

typedef enum {
  XVEC_METRIC_L2 = 1,
  XVEC_METRIC_IP = 2,
  XVEC_METRIC_COSINE = 3,
  XVEC_METRIC_MIPSL2 = 4
} xvec_gpu_metric;

typedef enum {
  /* Dense Flat exact search: core.DenseFlatIndex (internal/core/flat.go:70-196). */
  XVEC_INDEX_FLAT = 1,
  /* INT8 scalar-quantized Flat: core.ScalarQuantizedFlatIndex
   * (internal/core/quantized_index.go:28-120, quantization.go:267-321). */
  XVEC_INDEX_SQ8_FLAT = 2,
  /* IVF list scan over 8-bit PQ codes: probedListsLocked (internal/core/ivf.go:524-561)
   * + PQDistanceTable.Lookup (internal/core/pq.go:549-595). */
  XVEC_INDEX_IVF_PQ = 3,
  /* One-bit RaBitQ linear scan + exact refine (internal/core/hnsw_rabitq.go:539-642,
   * 780-801; internal/core/rabitq.go:372-430). */
  XVEC_INDEX_RABITQ = 4,
  /* IVF with exact scoring of the probed lists' original rows: core.IVFIndex
   * (internal/core/ivf.go:214-230, searchIVF :427-493, probedListsLocked
   * :524-561; cosine with cached magnitudes, :469-478). */
  XVEC_INDEX_IVF_FLAT = 5,
  /* IVF with INT8 scalar-quantized scoring of the probed lists' rows:
   * core.ScalarQuantizedIVFIndex (internal/core/ivf_quantized.go:23-192): the
   * IVF probe with the original metric, the SQ8_FLAT scoring of the probed
   * positions (quantized_index.go:313-335) and the optional refine stage. */
  XVEC_INDEX_IVF_SQ8 = 6,
  /* INT4 scalar-quantized Flat: core.ScalarQuantizedFlatIndex with
   * QuantizationInt4 (quantization.go:91-103, 267-321): codes in [-8, 7],
   * kept one per byte in device memory so that they share the INT8 kind's
   * tcgen05 kind::i8 scan, its scoring (QuantizedDistance,
   * quantization.go:171-235) and its optional refine stage.  The dimension
   * must be even for rows and queries (ErrOddInt4Dimension). */
  XVEC_INDEX_SQ4_FLAT = 7,
  /* IVF with INT4 scalar-quantized scoring of the probed lists' rows:
   * ScalarQuantizedIVFIndex with QuantizationInt4 (ivf_quantized.go:31-54),
   * the IVF_SQ8 kind with INT4 codes (kept one per byte, as SQ4_FLAT). */
  XVEC_INDEX_IVF_SQ4 = 8,
  /* DiskANN graph search with the PQ frontier: DiskANNIndex
   * (internal/core/diskann.go:343-367; SearchDiskANN :472-525,
   * searchDiskANNGraph :559-651) over the float32 node vectors (the rows), their
   * PQ codes (encoded at insertion from the prepared rows: cosine rows
   * normalised, diskann.go:258-274, under the traversal metric, L2 for cosine
   * and MIPSL2, :276-281) and a graph the caller uploads
   * (xvec_gpu_diskann_set_graph).  Every metric; storage FP32. */
  XVEC_INDEX_DISKANN = 9
} xvec_gpu_index_kind;

typedef enum {
  XVEC_STORAGE_FP32 = 1, /* rows and queries are float32 */
  XVEC_STORAGE_FP16 = 2  /* rows and queries are IEEE binary16 bit patterns (uint16);
                            the arithmetic is float32 on the decoded values, as for a
                            VectorFP16 field (collection.go:4607-4613) or QuantizationFP16
                            (quantization.go:187-191) */
} xvec_gpu_storage;

typedef struct xvec_gpu_index xvec_gpu_index;

typedef struct {
  int32_t kind;      /* xvec_gpu_index_kind */
  int32_t dimension; /* > 0 (ErrInvalidDimension, flat.go:84-86) */
  int32_t metric;    /* xvec_gpu_metric; IVF_PQ: L2 or IP (pq.go:67-70); RABITQ: L2/IP/COSINE */
  int32_t storage;   /* FLAT only: xvec_gpu_storage; others use float32 input */
  int32_t device;    /* CUDA device ordinal */
  int32_t reserved[3];
} xvec_gpu_index_desc;

typedef struct {
  int32_t top_k;            /* SearchOptions.TopK, > 0 (query.go:47-55) */
  float radius;             /* SearchOptions.Radius, 0 = off (query.go:193-201) */
  int32_t nprobe;           /* IVFSearchOptions.NProbe (ivf.go:387-400); IVF_PQ only */
  float refine_scale;       /* > 0: UseRefiner with QueryParams.ScaleFactor
                               (collection.go:1606-1631, refiner.go:112-129).
                               SQ8_FLAT only: exact fp32 rerank of floor(top_k*scale)
                               codes. */
  int32_t ef;               /* HNSWRaBitQSearchOptions.EF (hnsw_rabitq.go:548-550),
                               RABITQ: in [1, 2048] (ErrInvalidHNSWEF); with
                               refine, min(len, max(top_k, ef)) estimates are refined
                               (hnsw_rabitq.go:579).  DISKANN: DiskANNSearchOptions.
                               ListSize (diskann.go:326-333); 0 = DefaultDiskANNQueryList
                               (300), negative = ErrInvalidDiskANNListSize; the
                               traversal keeps min(len, max(top_k, ListSize)) <= 2048
                               nodes */
  int32_t refine;           /* HNSWRaBitQSearchOptions.Refine, RABITQ only: non-zero =
                               exact fp32 rerank of the best estimates; zero = the
                               estimates themselves with the public score (IP:
                               1 - estimate) */
  const uint32_t* filter_bitmap; /* NULL = no filter.  Bit p (word p/32, bit p%32) set =
                                    the row at insertion position p passes
                                    CandidateFilter (query.go:35); evaluated before
                                    scoring.  Host memory for xvec_gpu_index_search,
                                    device memory for the _device variant. */
  int64_t filter_words;     /* number of uint32 words in filter_bitmap */
  void* stream;             /* cudaStream_t for the _device variants; NULL = the
                               legacy default stream */
  const volatile int32_t* cancel_flag; /* optional host flag, polled between kernel
                                          launches; non-zero => XVEC_GPU_CANCELLED */
  int32_t linear;           /* HNSWRaBitQSearchOptions.Linear (hnsw_rabitq.go:589-591),
                               RABITQ with a graph: non-zero = the linear scan of
                               every code instead of the graph walk.
                               DiskANNSearchOptions.Linear (diskann.go:521-523),
                               DISKANN: the exact scan of every node */
} xvec_gpu_search_opts;

/* Library ------------------------------------------------------------------ */
int32_t xvec_gpu_abi_version(void);
/* Copies the calling thread's last error message; returns its full length. */
size_t xvec_gpu_last_error(char* buffer, size_t length);
/* Number of CUDA devices the library can use (compute capability 10.0). */
int32_t xvec_gpu_device_count(void);

/* Index lifecycle ------------------------------------------------------------
 * Replaces core.NewDenseFlatIndex (flat.go:79-93), NewScalarQuantizedFlatIndex
 * (quantized_index.go:33-60), NewIVFBuilder (ivf.go:95-107) and
 * RestoreRaBitQModel (rabitq.go:189-241) at the collection's index
 * construction (collection.go:657-818). */
xvec_gpu_status xvec_gpu_index_create(const xvec_gpu_index_desc* desc, xvec_gpu_index** out);
xvec_gpu_status xvec_gpu_index_destroy(xvec_gpu_index* index);
int64_t xvec_gpu_index_len(const xvec_gpu_index* index);
/* Pre-sizes the index for `capacity` rows, like make([]T, 0, capacity) for
 * the slices the reference grows by append (flat.go:148-152); no reference
 * call corresponds.  Growing happens anyway on add, but growing a buffer
 * needs its old and new copies at once, so a caller that knows the final
 * size of a large index reserves it first. */
xvec_gpu_status xvec_gpu_index_reserve(xvec_gpu_index* index, int64_t capacity);

/* Appends n rows at positions len..len+n-1 (DenseFlatIndex.Add, flat.go:122-153;
 * batch form).  rows: n*dimension float32, or uint16 for FP16 storage.  Keys
 * must be unique (XVEC_GPU_DUPLICATE_KEY); rows must be finite
 * (XVEC_GPU_NON_FINITE).  SQ8_FLAT quantizes each row per vector with the
 * reference INT8 rule and keeps the float32 row for refinement; IVF_PQ
 * assigns each row to its best list and PQ-encodes it (requires the model);
 * RABITQ encodes each row with the one-bit quantizer (requires the model). */
xvec_gpu_status xvec_gpu_index_add(xvec_gpu_index* index, const uint64_t* keys, const void* rows,
                                   int64_t n);
xvec_gpu_status xvec_gpu_index_add_device(xvec_gpu_index* index, const uint64_t* d_keys,
                                          const void* d_rows, int64_t n, void* stream);

/* IVF-PQ model: IVF centroids [nlist*dimension] (KMeansModel centroids,
 * ivf.go:193-201) and the PQ codebook in PQModelState layout (pq.go:86-94):
 * pivots [256*dimension], centroid-major, split into `chunks` contiguous chunks
 * by pqChunkOffsets (pq.go:395-406). */
xvec_gpu_status xvec_gpu_ivfpq_set_model(xvec_gpu_index* index, const float* centroids,
                                         int32_t nlist, const float* pivots, int32_t chunks);

/* RaBitQ model (RaBitQModelState, rabitq.go:96-103) with TotalBits = 1:
 * centroids [nclusters*dimension] and rotation signs
 * [4 * roundUp64(dimension) / 8] bytes. */
xvec_gpu_status xvec_gpu_rabitq_set_model(xvec_gpu_index* index, const float* centroids,
                                          int32_t nclusters, const uint8_t* rotation_signs);

/* RaBitQ model with RaBitQModelState.TotalBits in [1, 9] and ExtraScale
 * (RestoreRaBitQModel, rabitq.go:189-241: zero for one bit, finite and
 * positive otherwise).  TotalBits > 1: rows get their extra-bit codes and full
 * factors (quantizeRaBitQVector, rabitq_quantize.go:99-200) and searches rank
 * by Estimate (rabitq.go:434-446) on the full codes before the refine stage;
 * TotalBits = 1 is xvec_gpu_rabitq_set_model. */
xvec_gpu_status xvec_gpu_rabitq_set_model_bits(xvec_gpu_index* index, const float* centroids,
                                               int32_t nclusters, const uint8_t* rotation_signs,
                                               int32_t total_bits, double extra_scale);

/* Batched search: queries [nq*dimension] (float32, or uint16 for FP16 storage).
 * out_keys / out_scores: nq*top_k (slots past out_counts[q] are unspecified).
 * Replaces DenseQuerySearcher.SearchWithOptions (query.go:58-61) per query,
 * batched like core.BatchTopK (topk.go:242-269): FLAT → flat.go:175-196;
 * SQ8_FLAT → quantized_index.go:113-120 (+ OriginalVectorRefiner.Refine,
 * refiner.go:66-108, when refine_scale > 0); IVF_PQ → the IVF SearchIVF flow
 * (ivf.go:423-493) scoring PQ codes; RABITQ → hnsw_rabitq.go:539-586 with a
 * linear scan and Refine. */
xvec_gpu_status xvec_gpu_index_search(xvec_gpu_index* index, const void* queries, int32_t nq,
                                      const xvec_gpu_search_opts* opts, uint64_t* out_keys,
                                      float* out_scores, int32_t* out_counts);
xvec_gpu_status xvec_gpu_index_search_device(xvec_gpu_index* index, const void* d_queries,
                                             int32_t nq, const xvec_gpu_search_opts* opts,
                                             uint64_t* d_out_keys, float* d_out_scores,
                                             int32_t* d_out_counts);

/* IVF model: the nlist centroids [nlist*dim] of an IVF_FLAT or IVF_SQ8 index (the
 * trained KMeansModel of IVFBuilder.Build, ivf.go:144-212); set before any
 * row is added.  Rows go to their nearest centroid (KMeansModel.Nearest,
 * kmeans.go:169-175). */
xvec_gpu_status xvec_gpu_ivf_set_model(xvec_gpu_index* index, const float* centroids,
                                       int32_t nlist);

/* Rows with their IVF lists given (0 <= list < nlist) instead of the nearest
 * centroid, for IVF_FLAT and IVF_SQ8 indexes with a model: the device upload
 * of an IVF layout built elsewhere (IVFIndex.listForPosition, ivf.go:229,
 * which streaming adds do not keep nearest-centroid).  Otherwise as
 * xvec_gpu_index_add. */
xvec_gpu_status xvec_gpu_ivf_add_with_lists(xvec_gpu_index* index, const uint64_t* keys,
                                            const float* rows, const int32_t* lists, int64_t n);

/* The header of a verified ZVECIVF version 1 file (IVFIndex.Save,
 * ivf.go:866-904): rows, dimension, effective lists, metric, the build
 * options and the training metadata. */
typedef struct {
  int64_t count;
  int32_t dimension;
  int32_t nlist;               /* effective lists (centroids in the file) */
  int32_t metric;              /* xvec_gpu_metric: the same values as metric.Metric */
  int32_t converged;
  int64_t options_nlist;       /* IVFBuildOptions */
  int64_t options_iterations;
  int64_t options_workers;
  uint64_t options_seed;
  double options_tolerance;
  double training_cost;
  int64_t training_iterations;
} xvec_gpu_ivf_file_header;

/* Reads and verifies a ZVECIVF file on the host, as decodeIVFIndex
 * (ivf.go:906-1057) does: magic, version (XVEC_GPU_UNSUPPORTED for another
 * one), header fields and reserved zeros, the header and payload CRC32C
 * (XVEC_GPU_CHECKSUM_MISMATCH), lengths, build options, training metadata,
 * finite centroids and vectors, unique keys, list ranges
 * (XVEC_GPU_INVALID_ARGUMENT for the rest).  No device work. */
xvec_gpu_status xvec_gpu_ivf_file_info(const char* path, xvec_gpu_ivf_file_header* out);

/* OpenIVFIndex (ivf.go:815-830) into a device index: an IVF_FLAT index on
 * `device` with the file's metric and centroids, its rows at their file
 * positions and each row in the list the file gives.  A file with no rows
 * gives an index without a model (searching it reports the missing model;
 * the reference returns no results). */
xvec_gpu_status xvec_gpu_ivf_open(const char* path, int32_t device, xvec_gpu_index** out);

/* k-means assignment: assignKMeans / assignKMeansCosine (kmeans.go:382-479):
 * for each vector the metric-best centroid (lower index wins ties) and its
 * score.  vectors [n*dim], centroids [nc*dim]; labels/scores [n]. */
xvec_gpu_status xvec_gpu_kmeans_assign(int32_t device, int32_t metric, const float* vectors,
                                       int64_t n, const float* centroids, int32_t nc, int32_t dim,
                                       int32_t* labels, float* scores);
xvec_gpu_status xvec_gpu_kmeans_assign_device(int32_t device, int32_t metric,
                                              const float* d_vectors, int64_t n,
                                              const float* d_centroids, int32_t nc, int32_t dim,
                                              int32_t* d_labels, float* d_scores, void* stream);

/* k-means training: trainKMeansWithAssignments (kmeans.go:208-298) with the
 * IVF builder's options (DefaultKMeansOptions, kmeans.go:83-92): reservoir
 * initialisation from splitMix64(seed), Lloyd updates (float64 sums in input
 * order, algorithm/lloyd_cluster.go:53-137), empty clusters reseeded with
 * the worst-assigned vectors, stop after max_iterations or when
 * |cost - previous| < tolerance.  vectors [n*dim] (n < 2^31); centroids
 * [min(clusters, n)*dim]; labels [n] (the final assignment).  Outputs the
 * cluster count, iterations, whether it converged and the final cost.
 * Bit-identical to TrainKMeans on the same inputs. */
xvec_gpu_status xvec_gpu_kmeans_train(int32_t device, int32_t metric, const float* vectors,
                                      int64_t n, int32_t dim, int32_t clusters,
                                      int32_t max_iterations, double tolerance, uint64_t seed,
                                      float* centroids, int32_t* labels, int32_t* out_clusters,
                                      int32_t* out_iterations, int32_t* out_converged,
                                      double* out_cost);
xvec_gpu_status xvec_gpu_kmeans_train_device(int32_t device, int32_t metric,
                                             const float* d_vectors, int64_t n, int32_t dim,
                                             int32_t clusters, int32_t max_iterations,
                                             double tolerance, uint64_t seed, float* d_centroids,
                                             int32_t* d_labels, int32_t* out_clusters,
                                             int32_t* out_iterations, int32_t* out_converged,
                                             double* out_cost, void* stream);

/* k-means training from given initial centroids: TrainKMeans with
 * KMeansOptions.InitialCentroids (kmeans.go:354-363), the Lloyd iterations
 * above started from d_initial [kc*dim] (1 <= kc <= n, all finite) instead of
 * the reservoir sample.  Device memory; d_centroids [kc*dim], d_labels [n]. */
xvec_gpu_status xvec_gpu_kmeans_train_init_device(
    int32_t device, int32_t metric, const float* d_vectors, int64_t n, int32_t dim, int32_t kc,
    const float* d_initial, int32_t max_iterations, double tolerance, float* d_centroids,
    int32_t* d_labels, int32_t* out_iterations, int32_t* out_converged, double* out_cost,
    void* stream);

/* Product-quantizer training: TrainPQ (pq.go:107-179) with PQOptions{Metric,
 * Chunks, MaxTrainSamples, MaxIterations, Seed}.  chunks 0 resolves to
 * dim / 2; metric L2 or inner product.  Per contiguous chunk of the first
 * min(n, max_train_samples) rows: KMC2 seeding (initializePQKMC2,
 * pq.go:410-459), then TrainKMeans with those initial centroids, 256
 * clusters, seed ^ (0x70716b6d00000000 + chunk) and the default tolerance.
 * Writes PQModelState: chunk_offsets_out [chunks+1] (host, may be NULL) and
 * pivots [256*dim] centroid-major, rows past the trained centroids repeating
 * centroid 0; *out_chunks the resolved chunk count.  Bit-identical pivots.
 * vectors and pivots are host memory (every row is validated finite, the
 * training sample alone is copied to the device). */
xvec_gpu_status xvec_gpu_pq_train(int32_t device, int32_t metric, const float* vectors,
                                  int64_t n, int32_t dim, int32_t chunks,
                                  int64_t max_train_samples, int32_t max_iterations,
                                  uint64_t seed, int32_t* chunk_offsets_out, float* pivots,
                                  int32_t* out_chunks);
xvec_gpu_status xvec_gpu_pq_train_device(int32_t device, int32_t metric, const float* d_vectors,
                                         int64_t n, int32_t dim, int32_t chunks,
                                         int64_t max_train_samples, int32_t max_iterations,
                                         uint64_t seed, int32_t* chunk_offsets_out,
                                         float* d_pivots, int32_t* out_chunks, void* stream);

/* Cross-shard merge: MergeSearchResults (query.go:154-191) of `parts` result
 * lists per query, as produced by xvec_gpu_index_search_device on each shard
 * (layout [parts][nq][top_k] keys/scores and [parts][nq] counts, all device
 * memory).  Writes the best top_k per query.  Used after the NCCL allgather of
 * the multi-GPU search. */
xvec_gpu_status xvec_gpu_merge_results_device(int32_t device, int32_t metric, int32_t top_k,
                                              int32_t nq, int32_t parts, const uint64_t* d_keys,
                                              const float* d_scores, const int32_t* d_counts,
                                              uint64_t* d_out_keys, float* d_out_scores,
                                              int32_t* d_out_counts, void* stream);

/* Multi-GPU search ------------------------------------------------------------
 * The reference fans a query out over the segments of a collection and
 * merges the per-segment top-k with MergeSearchResults (collection.go:
 * 4040-4066, internal/core/query.go:154-191).  Here each GPU holds one shard
 * of the rows in its own index (keys unique across shards) and the library
 * exchanges the shards' lists with its own NCCL communicator: one all-gather
 * of a packed buffer (keys, scores and counts of every query), then the
 * MergeSearchResults order on every rank.  Refined searches (SQ8_FLAT,
 * SQ4_FLAT, IVF_SQ8 and IVF_SQ4 with a refine scale, RABITQ with refine)
 * exchange twice, so that the refined candidates are the whole index's
 * (RefinedSearch, refiner.go:133-166).  NCCL is loaded at run time (the copy
 * the process holds, else XVEC_GPU_NCCL_LIBRARY, else libnccl.so.2;
 * XVEC_GPU_UNSUPPORTED without one).  Every wait on a communicator is bounded
 * by its timeout: when it passes the communicator is aborted and the call
 * returns XVEC_GPU_TIMEOUT (XVEC_GPU_NCCL_ERROR for an error NCCL reports);
 * an aborted communicator fails every later call, so destroy it and make a
 * new one.  A rank whose own search fails as a whole still takes part in the
 * exchange, with every query failed by that status, so every rank reports it.
 * The library's counterpart of the reference's in-process segment fan-out;
 * no single reference call corresponds. */
#define XVEC_GPU_COMM_ID_BYTES 128
typedef struct xvec_gpu_comm xvec_gpu_comm;

/* A new communicator id (ncclGetUniqueId): made by one rank, sent to the
 * others by the caller (id_out: XVEC_GPU_COMM_ID_BYTES bytes). */
xvec_gpu_status xvec_gpu_comm_unique_id(uint8_t* id_out);
/* One process per GPU: this process's rank of nranks on `device`, joining
 * the communicator `id`.  timeout_ms (<= 0: 60 s) bounds this call and every
 * later wait on the communicator. */
xvec_gpu_status xvec_gpu_comm_init_rank(int32_t device, const uint8_t* id, int32_t nranks,
                                        int32_t rank, int32_t timeout_ms, xvec_gpu_comm** out);
/* One process over several GPUs: ranks 0..ndev-1 on devices[0..ndev-1],
 * written to out[0..ndev-1]. */
xvec_gpu_status xvec_gpu_comm_init_all(const int32_t* devices, int32_t ndev, int32_t timeout_ms,
                                       xvec_gpu_comm** out);
/* Frees a communicator (a healthy one is flushed first, within its timeout). */
xvec_gpu_status xvec_gpu_comm_destroy(xvec_gpu_comm* comm);
/* Aborts a communicator's pending and future work (ncclCommAbort). */
xvec_gpu_status xvec_gpu_comm_abort(xvec_gpu_comm* comm);
int32_t xvec_gpu_comm_size(const xvec_gpu_comm* comm);
int32_t xvec_gpu_comm_rank(const xvec_gpu_comm* comm);

/* One rank's call of a sharded search (one process per GPU): every rank
 * calls it with the same queries and options on its own shard's index (on
 * the communicator's device) and receives the merged results of all shards
 * in its device outputs (nq*top_k keys / scores, nq counts), enqueued on
 * opts->stream.  filter_bitmap, if given, is this shard's (device memory).
 * Returns like xvec_gpu_index_search_device. */
xvec_gpu_status xvec_gpu_sharded_search_device(xvec_gpu_comm* comm, xvec_gpu_index* index,
                                               const void* d_queries, int32_t nq,
                                               const xvec_gpu_search_opts* opts,
                                               uint64_t* d_out_keys, float* d_out_scores,
                                               int32_t* d_out_counts);
/* The same over ndev GPUs of one process (comms from xvec_gpu_comm_init_all,
 * indexes[i] on comms[i]'s device): host queries in, the merged results in
 * host outputs.  No filter bitmap (each shard has its own positions: filter
 * through xvec_gpu_sharded_search_device). */
xvec_gpu_status xvec_gpu_sharded_search(xvec_gpu_comm* const* comms,
                                        xvec_gpu_index* const* indexes, int32_t ndev,
                                        const void* queries, int32_t nq,
                                        const xvec_gpu_search_opts* opts, uint64_t* out_keys,
                                        float* out_scores, int32_t* out_counts);

/* The two halves of a refined search, for a search whose rows are split
 * over several indexes (shards).  RefinedSearch (refiner.go:133-166) refines
 * the RefinementCandidateCount best approximate results of the whole index,
 * and the HNSW-RaBitQ search its max(TopK, EF) best estimates
 * (hnsw_rabitq.go:584, 780-801); over shards that candidate list is the
 * merge of the shards' lists.  Order: candidates on every shard; merge them
 * with xvec_gpu_merge_results_device under XVEC_METRIC_L2 (ranks: lower is
 * better, ties by key); refine the merged list on every shard; merge those
 * results under the index metric.
 *
 * candidate_count: candidates per query for these options (SQ8_FLAT,
 * SQ4_FLAT, IVF_SQ8, IVF_SQ4: max(1, floor(top_k * refine_scale)); RABITQ
 * with refine: max(top_k, ef)); 0 when the options ask for no refinement.
 * candidates_device: the approximate stage alone (no radius): per query up
 * to candidate_count keys with their ranks (the approximate distance, or the
 * negated inner product; for RaBitQ the estimate), best first, at stride
 * candidate_count.  Per-query failures are negative counts (-status); the
 * call itself returns OK for them.
 * refine_device: DenseRefiner.Refine (refiner.go:30-33, 66-108) of the given
 * candidate keys: those this index holds are scored by metric.Compute on
 * the float32 original rows, and the top_k best within `radius` (ties by key)
 * are written at stride top_k.  Keys the index does not hold are skipped;
 * negative candidate counts pass through.  Indexes with float32 rows only. */
int32_t xvec_gpu_index_candidate_count(const xvec_gpu_index* index,
                                       const xvec_gpu_search_opts* opts);
xvec_gpu_status xvec_gpu_index_candidates_device(xvec_gpu_index* index, const void* d_queries,
                                                 int32_t nq, const xvec_gpu_search_opts* opts,
                                                 uint64_t* d_keys, float* d_ranks,
                                                 int32_t* d_counts);
xvec_gpu_status xvec_gpu_index_refine_device(xvec_gpu_index* index, const float* d_queries,
                                             int32_t nq, const uint64_t* d_cand_keys,
                                             int32_t cand_stride, const int32_t* d_cand_counts,
                                             int32_t top_k, float radius, void* stream,
                                             uint64_t* d_keys, float* d_scores,
                                             int32_t* d_counts);

/* Flat search that allocates no device memory during the call (no
 * counterpart in the reference).  For callers that cannot allocate while they
 * search: a process that plans a fixed device-memory budget up front, or a
 * latency-critical caller that must not enter the CUDA allocator (which can
 * block or synchronise the device).  Same inputs, outputs and results as
 * xvec_gpu_index_search_device on a Flat index; the per-call scratch comes
 * from one 32 MiB device array that every GPU loading the library holds until
 * exit.  Limits: at most 4096 queries, top-k <= 100, no filter bitmap, and
 * the scratch the batch needs must fit in 32 MiB (otherwise
 * XVEC_GPU_INVALID_ARGUMENT).  All calls share the array: calls whose GPU
 * work overlaps race (the library serialises calls from one process and each
 * call waits for its GPU work, on its error paths too).  The cancel flag and
 * the library's counters work as for the regular search.  The first call on a
 * device looks up the
 * array's device address (which also makes the CUDA runtime load the
 * library's device code there, reserving the array); make that first call
 * before any stream capture. */
xvec_gpu_status xvec_gpu_index_search_noalloc(xvec_gpu_index* index, const void* d_queries,
                                              int32_t nq, const xvec_gpu_search_opts* opts,
                                              uint64_t* d_out_keys, float* d_out_scores,
                                              int32_t* d_out_counts);

/* HNSW-RaBitQ graph (HNSWRaBitQIndex, hnsw_rabitq.go): the graph the Go
 * side built over the index's insertion positions, for the graph walk of
 * searchPrepared (hnsw_rabitq.go:589-612: descent through the upper levels on
 * coarse estimates, :644-671; the base-layer search, :673-737).  Node p's
 * level-L neighbours (positions, in the reference's list order) are
 * neighbors[offsets[L (n + 1) + p] .. offsets[L (n + 1) + p + 1]) for L in
 * 0..max_level; offsets is (max_level + 1) (n + 1) int64 in host memory,
 * each level's run non-decreasing; entry is the entry point
 * (hnswIndex.entryPoint); n must equal the index's row count.  With a graph,
 * searches of more than 1000 rows (DefaultHNSWBruteForceThreshold,
 * hnsw.go:592) walk it unless opts.linear is set; results equal the
 * reference's walk (keys identical, scores bit-identical).  Adding rows
 * invalidates the graph (searches then fail until it is set again);
 * max_level = -1 removes it. */
xvec_gpu_status xvec_gpu_rabitq_set_graph(xvec_gpu_index* index, int32_t max_level, int64_t entry,
                                          const int64_t* offsets, const int32_t* neighbors,
                                          int64_t total_neighbors);

/* ---- DiskANN ------------------------------------------------------------
 * xvec_gpu_diskann_set_model: the PQ model of the traversal encoding
 * (PQModelState, pq.go:86-94: pivots [256*dimension], centroid-major, split into
 * `chunks` contiguous chunks by pqChunkOffsets, pq.go:395-406), trained on the
 * prepared rows under the traversal metric as the DiskANN builder trains it
 * (diskann.go:224-233); before rows are added.
 *
 * xvec_gpu_diskann_set_graph: the graph over the index's rows (positions
 * 0..n-1, n = the index's row count): node p's neighbours at
 * neighbors[offsets[p] .. offsets[p + 1]) (offsets: n + 1 int64 in host
 * memory; at most max_degree each, max_degree in [1, 2048]); entry is the
 * graph's entry point (DiskANNIndex.entryPoint); max_degree is the node
 * layout's MaxDegree (NewDiskANNLayout, diskann_storage.go:61-100), which
 * sets the traversal's read batch (diskANNReadBatchSize, diskann.go:685-691).
 * Results equal the reference's traversal (keys identical, scores
 * bit-identical).  Adding rows invalidates the graph (searches then fail
 * until it is set again); offsets = NULL removes it. */
xvec_gpu_status xvec_gpu_diskann_set_model(xvec_gpu_index* index, const float* pivots,
                                           int32_t chunks);
xvec_gpu_status xvec_gpu_diskann_set_graph(xvec_gpu_index* index, int64_t entry,
                                           int32_t max_degree, const int64_t* offsets,
                                           const int32_t* neighbors, int64_t total_neighbors);

/* ---- Rotation reformer -------------------------------------------------
 * A collection whose vector index sets `rotate` rotates every stored and
 * query vector with an FHT rotator before its scalar-quantized index sees it
 * (collectionReformer, collection.go:1981-2000; RotationReformer,
 * internal/core/rotation.go:248-280).  A caller of this library applies the
 * same transform with these entry points before xvec_gpu_index_add* and
 * xvec_gpu_index_search* (and Revert on vectors it returns).
 *
 * xvec_gpu_rotation_signs: the sign state collectionReformer derives for
 * (schema name, field name, dimension, index type, quantize type): SHA-256 of
 * "zvec-go-rotation-v1\0<schema>\0<field>\0<dimension>\0<index type>\0<quantize>"
 * followed by a little-endian uint64 counter 0, 1, ..., the digests
 * concatenated; out_len must be 4 * ((dimension + 7) / 8)
 * (NewFHTRotatorFromSigns, rotation.go:87-104). */
xvec_gpu_status xvec_gpu_rotation_signs(const char* schema_name, const char* field_name,
                                        int32_t dimension, int32_t index_type, int32_t quantize,
                                        uint8_t* out_signs, int64_t out_len);
/* FHTRotator.Rotate (rotation.go:123-153; inverse = 0) or Unrotate
 * (rotation.go:155-185; inverse = 1) of n vectors of `dimension` float32s,
 * bit-identical to the reference.  signs: host memory, 4 * ((dimension + 7) /
 * 8) bytes; dimension 1..65535 (MaxRotationDimension).  Host form: fails with
 * XVEC_GPU_NON_FINITE naming the first vector whose input or result is not
 * finite (RotateBatch, rotation.go:187-213).  Device form: in and out on
 * `device`, enqueued on `stream`; d_failed (n int32) receives 1 for each such
 * vector, 0 otherwise; the call does not wait. */
xvec_gpu_status xvec_gpu_rotate(int32_t device, const uint8_t* signs, int64_t signs_len,
                                int32_t dimension, const float* vectors, int64_t n, float* out,
                                int32_t inverse);
xvec_gpu_status xvec_gpu_rotate_device(int32_t device, const uint8_t* signs, int64_t signs_len,
                                       int32_t dimension, const float* d_vectors, int64_t n,
                                       float* d_out, int32_t inverse, int32_t* d_failed,
                                       void* stream);

/* Counters (the reference's RuntimeStats role, collection.go:5185-5315, for
 * the device path).  Device-time fields are filled only while timing is
 * enabled, because timing adds an event pair around each scan launch. */
typedef struct {
  int64_t searches;        /* search calls completed */
  int64_t queries;         /* queries answered */
  int64_t kernel_launches; /* kernels launched by this library (all devices) */
  int64_t exact_queries;   /* queries answered through the exact (reference-order) scan */
  double scan_ms;          /* device time of the candidate scan kernels */
  double search_ms;        /* device time of whole search calls */
  int64_t tensor_scans;    /* scans that ran on the tensor cores (tcgen05) */
  int64_t stream_scans;    /* Flat scans of a few queries that streamed the rows once */
} xvec_gpu_stats;
void xvec_gpu_stats_enable_timing(int32_t enabled);

/* Bound of the device-side waits inside the tensor-core scans: 2 s by
 * default, ns <= 0 restores it; returns the previous bound.  Applies to scans
 * launched after the call, on every device.  A wait that runs out stops the
 * scan (the kernel drains the copies it issued and frees its tensor memory)
 * and the search returns XVEC_GPU_TIMEOUT; the device stays usable.  The
 * reference's counterpart is the context check between candidates
 * (ctx.Err(), internal/core/topk.go:130), which ends a search early. */
int64_t xvec_gpu_set_wait_limit_ns(int64_t ns);
void xvec_gpu_get_stats(xvec_gpu_stats* out);
void xvec_gpu_reset_stats(void);

#ifdef __cplusplus
}
#endif
#endif /* XVEC_GPU_H */
