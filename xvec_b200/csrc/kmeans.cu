// kmeans.cu — Lloyd k-means training on the GPU (the IVF builder's centroids).
//
// trainKMeansWithAssignments (internal/core/kmeans.go:208-298) with the IVF
// builder's options (DefaultKMeansOptions, kmeans.go:83-92: reservoir
// initialisation, empty clusters reseeded with the worst-assigned vectors,
// no spherical normalisation):
//   init     InitializeReservoir (internal/ailego/algorithm/kmeans.go:25-52)
//            driven by splitMix64.intn (kmeans.go:608-632): a sequential
//            random stream, run on the host.
//   assign   assignKMeans (kmeans.go:382-452): the Flat path over the
//            centroids (xvec_gpu_kmeans_assign_device), bit-identical labels
//            and scores.
//   update   LloydUpdate (algorithm/lloyd_cluster.go:53-137): per cluster and
//            coordinate the float64 sum of the members in input order
//            (members sorted stably by label, one thread per coordinate
//            walking them in order), float32(sum / count); empty clusters
//            keep their centroid, then take the distinct worst-assigned
//            vectors (worstAssignedVector, lloyd_cluster.go:140-160: first
//            index among equals) — on the host over the copied scores.
//   cost     kMeansObjective (kmeans.go:537-552): the float64 sum of the
//            scores in input order (negated for inner product), on the host.
// Iterations stop after MaxIterations or when no empty cluster was reseeded
// and |cost - previous cost| < Tolerance; the final assignment gives the
// labels.  Every step is the reference's arithmetic in the reference's
// order, so centroids and labels are bit-identical to TrainKMeans.
#include <cub/device/device_radix_sort.cuh>
#include <cub/device/device_scan.cuh>

#include <algorithm>
#include <cmath>
#include <vector>

#include "capi_internal.h"
#include "common.cuh"

namespace xvec {
namespace {

uint64_t splitmix_next(uint64_t* state) {
  *state += 0x9e3779b97f4a7c15ull;
  uint64_t v = *state;
  v = (v ^ (v >> 30)) * 0xbf58476d1ce4e5b9ull;
  v = (v ^ (v >> 27)) * 0x94d049bb133111ebull;
  return v ^ (v >> 31);
}

// splitMix64.intn: rejection sampling against modulo bias.
int64_t splitmix_intn(uint64_t* state, int64_t limit) {
  if (limit <= 1) return 0;
  const uint64_t bound = (uint64_t)limit;
  const uint64_t threshold = (0 - bound) % bound;
  for (;;) {
    const uint64_t v = splitmix_next(state);
    if (v >= threshold) return (int64_t)(v % bound);
  }
}

__global__ void finite_check_kernel(const float* x, int64_t count, int* bad) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < count && !finite_f(x[i])) atomicExch(bad, 1);
}

__global__ void gather_rows_kernel(const float* x, int d, const int64_t* rows, int count,
                                   float* out) {
  const int c = blockIdx.x;
  if (c >= count) return;
  for (int j = threadIdx.x; j < d; j += blockDim.x) out[(int64_t)c * d + j] = x[rows[c] * d + j];
}

__global__ void label_counts_kernel(const int32_t* labels, int64_t n, int64_t* counts) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) atomicAdd((unsigned long long*)&counts[labels[i]], 1ull);
}

__global__ void iota_kernel(uint32_t* out, int64_t n) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) out[i] = (uint32_t)i;
}

// One block per cluster, one thread per coordinate: the float64 sum of the
// members' coordinate in input order, then float32(sum / count).  Empty
// clusters keep their centroid.
__global__ void lloyd_update_kernel(const float* __restrict__ x, int d,
                                    const uint32_t* __restrict__ members,
                                    const int64_t* __restrict__ offsets,
                                    const float* __restrict__ cents, float* __restrict__ next) {
  const int c = blockIdx.x;
  const int64_t b = offsets[c], e = offsets[c + 1];
  for (int j = threadIdx.x; j < d; j += blockDim.x) {
    if (b == e) {
      next[(int64_t)c * d + j] = cents[(int64_t)c * d + j];
      continue;
    }
    double s = 0.0;
    for (int64_t k = b; k < e; ++k) s = __dadd_rn(s, (double)x[(int64_t)members[k] * d + j]);
    next[(int64_t)c * d + j] = __double2float_rn(__ddiv_rn(s, (double)(e - b)));
  }
}

inline unsigned blocks_of(int64_t n, int t = 256) { return (unsigned)((n + t - 1) / t); }

}  // namespace
}  // namespace xvec

using namespace xvec;

// The Lloyd iterations of trainKMeansWithAssignments (kmeans.go:240-298)
// from kc initial centroids (device, [kc][d]).
static xvec_gpu_status lloyd_train(int32_t device, int32_t metric, const float* d_vectors,
                                   int64_t n, int d, int kc, const float* d_initial,
                                   int32_t max_iterations, double tolerance, float* d_centroids,
                                   int32_t* d_labels, int32_t* out_iterations,
                                   int32_t* out_converged, double* out_cost, cudaStream_t s) {
  xvec_gpu_status st;
  Scratch cents_a, cents_b, scores, counts, offsets, members, iota, sorted_labels, temp;
  if ((st = cents_a.alloc((size_t)kc * d * 4, s)) || (st = cents_b.alloc((size_t)kc * d * 4, s)) ||
      (st = scores.alloc((size_t)n * 4, s)) ||
      (st = counts.alloc((size_t)(kc + 1) * 8, s)) ||
      (st = offsets.alloc((size_t)(kc + 1) * 8, s)) || (st = members.alloc((size_t)n * 4, s)) ||
      (st = iota.alloc((size_t)n * 4, s)) || (st = sorted_labels.alloc((size_t)n * 4, s)))
    return st;
  // The current centroids and the next ones (swapped after each update).
  float* cents = cents_a.as<float>();
  float* next = cents_b.as<float>();
  XVEC_CUDA(cudaMemcpyAsync(cents, d_initial, (size_t)kc * d * 4, cudaMemcpyDeviceToDevice, s));
  iota_kernel<<<blocks_of(n), 256, 0, s>>>(iota.as<uint32_t>(), n);
  XVEC_LAUNCHED();
  int bits = 1;
  while ((1ll << bits) < kc) ++bits;
  size_t tb_sort = 0, tb_scan = 0;
  XVEC_CUDA(cub::DeviceRadixSort::SortPairs(nullptr, tb_sort, (const uint32_t*)d_labels,
                                            sorted_labels.as<uint32_t>(), iota.as<uint32_t>(),
                                            members.as<uint32_t>(), n, 0, bits, s));
  XVEC_CUDA(cub::DeviceScan::ExclusiveSum(nullptr, tb_scan, counts.as<int64_t>(),
                                          offsets.as<int64_t>(), kc + 1, s));
  if ((st = temp.alloc(std::max(tb_sort, tb_scan), s))) return st;
  std::vector<float> h_scores(n);
  std::vector<int64_t> h_counts(kc + 1);
  auto assign = [&]() -> xvec_gpu_status {
    return xvec_gpu_kmeans_assign_device(device, metric, d_vectors, n, cents, kc, d, d_labels,
                                         scores.as<float>(), s);
  };
  auto objective = [&]() {
    double cost = 0;
    for (int64_t i = 0; i < n; ++i)
      cost += metric == XVEC_METRIC_IP ? -(double)h_scores[i] : (double)h_scores[i];
    return cost;
  };
  double previous = 0;
  int iterations = 0;
  bool converged = false;
  for (int it = 0; it < max_iterations; ++it) {
    if ((st = assign())) return st;
    // LloydUpdate: members of each cluster in input order, float64 sums.
    XVEC_CUDA(cudaMemsetAsync(counts.ptr, 0, (size_t)(kc + 1) * 8, s));
    label_counts_kernel<<<blocks_of(n), 256, 0, s>>>(d_labels, n, counts.as<int64_t>());
    XVEC_LAUNCHED();
    XVEC_CUDA(cub::DeviceScan::ExclusiveSum(temp.ptr, tb_scan, counts.as<int64_t>(),
                                            offsets.as<int64_t>(), kc + 1, s));
    XVEC_CUDA(cub::DeviceRadixSort::SortPairs(temp.ptr, tb_sort, (const uint32_t*)d_labels,
                                              sorted_labels.as<uint32_t>(), iota.as<uint32_t>(),
                                              members.as<uint32_t>(), n, 0, bits, s));
    lloyd_update_kernel<<<kc, 128, 0, s>>>(d_vectors, d, members.as<uint32_t>(),
                                           offsets.as<int64_t>(), cents, next);
    XVEC_LAUNCHED();
    XVEC_CUDA(cudaGetLastError());
    XVEC_CUDA(cudaMemcpyAsync(h_counts.data(), counts.ptr, (size_t)kc * 8,
                              cudaMemcpyDeviceToHost, s));
    XVEC_CUDA(cudaMemcpyAsync(h_scores.data(), scores.ptr, (size_t)n * 4, cudaMemcpyDeviceToHost,
                              s));
    XVEC_CUDA(cudaStreamSynchronize(s));
    // EmptyReseedFarthest: each empty cluster, in order, takes the worst-
    // assigned vector not taken yet (metric.Better(current, candidate)
    // replaces, so the first index wins among equals).
    bool changed = false;
    std::vector<char> used;
    for (int c = 0; c < kc; ++c) {
      if (h_counts[c] != 0) continue;
      if (used.empty()) used.assign(n, 0);
      int64_t sel = -1;
      for (int64_t i = 0; i < n; ++i) {
        if (used[i]) continue;
        const bool worse = sel < 0 || (metric == XVEC_METRIC_IP ? h_scores[sel] > h_scores[i]
                                                                : h_scores[sel] < h_scores[i]);
        if (worse) sel = i;
      }
      if (sel < 0) break;
      used[sel] = 1;
      XVEC_CUDA(cudaMemcpyAsync(next + (int64_t)c * d, d_vectors + sel * d,
                                (size_t)d * 4, cudaMemcpyDeviceToDevice, s));
      changed = true;
    }
    const double cost = objective();
    std::swap(cents, next);
    iterations = it + 1;
    if (!changed && std::fabs(cost - previous) < tolerance) {
      converged = true;
      break;
    }
    previous = cost;
  }
  if ((st = assign())) return st;
  XVEC_CUDA(cudaMemcpyAsync(d_centroids, cents, (size_t)kc * d * 4, cudaMemcpyDeviceToDevice, s));
  XVEC_CUDA(cudaMemcpyAsync(h_scores.data(), scores.ptr, (size_t)n * 4, cudaMemcpyDeviceToHost,
                            s));
  XVEC_CUDA(cudaStreamSynchronize(s));
  if (out_iterations) *out_iterations = iterations;
  if (out_converged) *out_converged = converged ? 1 : 0;
  if (out_cost) *out_cost = objective();
  return XVEC_GPU_OK;
}

extern "C" xvec_gpu_status xvec_gpu_kmeans_train_device(
    int32_t device, int32_t metric, const float* d_vectors, int64_t n, int32_t dim,
    int32_t clusters, int32_t max_iterations, double tolerance, uint64_t seed,
    float* d_centroids, int32_t* d_labels, int32_t* out_clusters, int32_t* out_iterations,
    int32_t* out_converged, double* out_cost, void* stream) {
  if (metric < XVEC_METRIC_L2 || metric > XVEC_METRIC_MIPSL2)
    return set_error("core: invalid k-means options: invalid metric"), XVEC_GPU_INVALID_ARGUMENT;
  if (clusters <= 0)
    return set_error("core: invalid k-means options: Clusters must be positive"),
           XVEC_GPU_INVALID_ARGUMENT;
  if (max_iterations <= 0)
    return set_error("core: invalid k-means options: MaxIterations must be positive"),
           XVEC_GPU_INVALID_ARGUMENT;
  if (!(tolerance >= 0) || std::isinf(tolerance))
    return set_error("core: invalid k-means options: Tolerance must be finite and non-negative"),
           XVEC_GPU_INVALID_ARGUMENT;
  if (n <= 0) return set_error("core: empty k-means training set"), XVEC_GPU_INVALID_ARGUMENT;
  if (dim <= 0 || n > 0x7fffffffll || !d_vectors || !d_centroids || !d_labels)
    return set_error("invalid k-means arguments"), XVEC_GPU_INVALID_ARGUMENT;
  cudaSetDevice(device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  xvec_gpu_status st;
  const int d = dim;
  {
    Scratch bad;
    if ((st = bad.alloc(4, s))) return st;
    XVEC_CUDA(cudaMemsetAsync(bad.ptr, 0, 4, s));
    finite_check_kernel<<<blocks_of(n * d), 256, 0, s>>>(d_vectors, n * d, bad.as<int>());
    XVEC_LAUNCHED();
    int h = 0;
    XVEC_CUDA(cudaMemcpyAsync(&h, bad.ptr, 4, cudaMemcpyDeviceToHost, s));
    XVEC_CUDA(cudaStreamSynchronize(s));
    if (h) return set_error("ailego: vector contains a non-finite value"), XVEC_GPU_NON_FINITE;
  }
  const int kc = (int)std::min<int64_t>(clusters, n);
  // InitializeReservoir.
  std::vector<int64_t> init(kc);
  {
    uint64_t state = seed;
    for (int i = 0; i < kc; ++i) init[i] = i;
    for (int64_t i = kc; i < n; ++i) {
      const int64_t sel = splitmix_intn(&state, i + 1);
      if (sel < kc) init[sel] = i;
    }
  }
  Scratch init_rows, initial;
  if ((st = init_rows.alloc((size_t)kc * 8, s)) || (st = initial.alloc((size_t)kc * d * 4, s)))
    return st;
  XVEC_CUDA(cudaMemcpyAsync(init_rows.ptr, init.data(), (size_t)kc * 8, cudaMemcpyHostToDevice, s));
  gather_rows_kernel<<<kc, 128, 0, s>>>(d_vectors, d, init_rows.as<int64_t>(), kc,
                                        initial.as<float>());
  XVEC_LAUNCHED();
  if (out_clusters) *out_clusters = kc;
  return lloyd_train(device, metric, d_vectors, n, d, kc, initial.as<float>(), max_iterations,
                     tolerance, d_centroids, d_labels, out_iterations, out_converged, out_cost, s);
}

extern "C" xvec_gpu_status xvec_gpu_kmeans_train_init_device(
    int32_t device, int32_t metric, const float* d_vectors, int64_t n, int32_t dim, int32_t kc,
    const float* d_initial, int32_t max_iterations, double tolerance, float* d_centroids,
    int32_t* d_labels, int32_t* out_iterations, int32_t* out_converged, double* out_cost,
    void* stream) {
  if (metric < XVEC_METRIC_L2 || metric > XVEC_METRIC_MIPSL2)
    return set_error("core: invalid k-means options: invalid metric"), XVEC_GPU_INVALID_ARGUMENT;
  if (max_iterations <= 0)
    return set_error("core: invalid k-means options: MaxIterations must be positive"),
           XVEC_GPU_INVALID_ARGUMENT;
  if (!(tolerance >= 0) || std::isinf(tolerance))
    return set_error("core: invalid k-means options: Tolerance must be finite and non-negative"),
           XVEC_GPU_INVALID_ARGUMENT;
  if (n <= 0) return set_error("core: empty k-means training set"), XVEC_GPU_INVALID_ARGUMENT;
  if (kc <= 0 || kc > n)
    return set_error("core: invalid centroid: got %d initial centroids, want %lld", kc,
                     (long long)std::min<int64_t>(kc, n)),
           XVEC_GPU_INVALID_ARGUMENT;
  if (dim <= 0 || n > 0x7fffffffll || !d_vectors || !d_initial || !d_centroids || !d_labels)
    return set_error("invalid k-means arguments"), XVEC_GPU_INVALID_ARGUMENT;
  cudaSetDevice(device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  xvec_gpu_status st;
  {
    Scratch bad;
    if ((st = bad.alloc(4, s))) return st;
    XVEC_CUDA(cudaMemsetAsync(bad.ptr, 0, 4, s));
    finite_check_kernel<<<blocks_of(n * dim), 256, 0, s>>>(d_vectors, n * dim, bad.as<int>());
    XVEC_LAUNCHED();
    finite_check_kernel<<<blocks_of((int64_t)kc * dim), 256, 0, s>>>(d_initial,
                                                                    (int64_t)kc * dim,
                                                                    bad.as<int>());
    XVEC_LAUNCHED();
    int h = 0;
    XVEC_CUDA(cudaMemcpyAsync(&h, bad.ptr, 4, cudaMemcpyDeviceToHost, s));
    XVEC_CUDA(cudaStreamSynchronize(s));
    if (h) return set_error("ailego: vector contains a non-finite value"), XVEC_GPU_NON_FINITE;
  }
  return lloyd_train(device, metric, d_vectors, n, dim, kc, d_initial, max_iterations, tolerance,
                     d_centroids, d_labels, out_iterations, out_converged, out_cost, s);
}

extern "C" xvec_gpu_status xvec_gpu_kmeans_train(int32_t device, int32_t metric,
                                                 const float* vectors, int64_t n, int32_t dim,
                                                 int32_t clusters, int32_t max_iterations,
                                                 double tolerance, uint64_t seed,
                                                 float* centroids, int32_t* labels,
                                                 int32_t* out_clusters, int32_t* out_iterations,
                                                 int32_t* out_converged, double* out_cost) {
  if (!vectors || !centroids || !labels || n <= 0 || dim <= 0 || clusters <= 0)
    return xvec_gpu_kmeans_train_device(device, metric, vectors, n, dim, clusters,
                                        max_iterations, tolerance, seed, centroids, labels,
                                        out_clusters, out_iterations, out_converged, out_cost,
                                        nullptr);
  cudaSetDevice(device);
  cudaStream_t s = nullptr;
  const int kc = (int)std::min<int64_t>(clusters, n);
  Scratch dv, dc, dl;
  xvec_gpu_status st;
  if ((st = dv.alloc((size_t)n * dim * 4, s)) || (st = dc.alloc((size_t)kc * dim * 4, s)) ||
      (st = dl.alloc((size_t)n * 4, s)))
    return st;
  XVEC_CUDA(cudaMemcpyAsync(dv.ptr, vectors, (size_t)n * dim * 4, cudaMemcpyHostToDevice, s));
  st = xvec_gpu_kmeans_train_device(device, metric, dv.as<float>(), n, dim, clusters,
                                    max_iterations, tolerance, seed, dc.as<float>(),
                                    dl.as<int32_t>(), out_clusters, out_iterations, out_converged,
                                    out_cost, s);
  if (st) return st;
  XVEC_CUDA(cudaMemcpyAsync(centroids, dc.ptr, (size_t)kc * dim * 4, cudaMemcpyDeviceToHost, s));
  XVEC_CUDA(cudaMemcpyAsync(labels, dl.ptr, (size_t)n * 4, cudaMemcpyDeviceToHost, s));
  XVEC_CUDA(cudaStreamSynchronize(s));
  return XVEC_GPU_OK;
}
