// pq_train.cu — product-quantizer training on the GPU (TrainPQ,
// internal/core/pq.go:107-179).
//
// Per contiguous chunk (pqChunkOffsets, pq.go:391-406) of the first
// min(n, MaxTrainSamples) rows:
//   seed     initializePQKMC2 (pq.go:410-459): the first centroid by a
//            uniform sample of one index, then each next one by a length-32
//            Markov chain over uniformly sampled candidates (pqUniformSample-
//            Indices, pq.go:461-476) scored by their nearest chosen centroid
//            (metric.Compute(centroid, candidate), inner product negated).
//            One 1024-thread block per chunk, all chunks at once.  The
//            sampling walk draws splitMix64.intn(count - i) for i = 0, 1, …
//            until the sample is full; splitMix64 is counter based (draw j
//            is mix(state + j·γ)), so the block evaluates 4096 indices per
//            step in parallel and resolves the hits (draw < remaining at the
//            step's start) in index order through warp ballots.  A step in
//            which some draw would be rejected by intn's bias check replays
//            serially on one thread, so the stream is the reference's in
//            every case.  The chain's acceptance draws (splitMix64.float64,
//            only while the current score is not 0) run on one thread.
//   train    TrainKMeans with those initial centroids, 256 clusters, the
//            chunk seed seed ^ (0x70716b6d00000000 + chunk), MaxIterations
//            and the default tolerance (pq.go:143-160): the GPU Lloyd
//            iterations of xvec_gpu_kmeans_train_init_device on the chunk's
//            columns gathered contiguous.
//   pivots   centroid-major [256][d]; rows past the trained centroids repeat
//            centroid 0 (pq.go:161-170).
// Scores use the reference's float32 accumulation order, the float64 Lloyd
// sums run in input order: pivots are bit-identical to TrainPQ's.
#include <algorithm>
#include <cmath>
#include <vector>

#include "capi_internal.h"
#include "common.cuh"

namespace xvec {
namespace {

constexpr int kPqCentroids = 256;
constexpr int kKmc2Chain = 32;
constexpr int kKmc2Threads = 1024;
constexpr int kKmc2Items = 4;  // indices per thread per sampling step
constexpr uint64_t kGolden = 0x9e3779b97f4a7c15ull;

__device__ __forceinline__ uint64_t splitmix_mix(uint64_t v) {
  v = (v ^ (v >> 30)) * 0xbf58476d1ce4e5b9ull;
  v = (v ^ (v >> 27)) * 0x94d049bb133111ebull;
  return v ^ (v >> 31);
}

__device__ __forceinline__ uint64_t splitmix_next_dev(uint64_t* state) {
  *state += kGolden;
  return splitmix_mix(*state);
}

// splitMix64.intn (kmeans.go:615-628) on one thread.  A draw is rejected
// with odds below 2^-33, so the loop is bounded at 64 draws; past that it
// returns ~0 and the caller reports an error.
__device__ uint64_t splitmix_intn_dev(uint64_t* state, uint64_t bound) {
  if (bound <= 1) return 0;
  const uint64_t threshold = (0 - bound) % bound;
  for (int tries = 0; tries < 64; ++tries) {
    const uint64_t v = splitmix_next_dev(state);
    if (v >= threshold) return v % bound;
  }
  return ~0ull;
}

struct Kmc2Shared {
  uint64_t state;        // splitMix64 state before the next draw
  int remaining;         // sample slots left in the current walk
  int taken;             // indices sampled so far in the current walk
  int stop;              // 1 once the walk is complete
  int replay;            // 1 when this step holds a rejected draw
  int err;               // non-finite candidate score
  int nchosen;
  unsigned hits[kKmc2Items * kKmc2Threads / 32];
  int picked[kKmc2Chain];
  unsigned best[kKmc2Chain];  // ordered float bits of each candidate's best score
  int chosen[kPqCentroids];   // row index of each chosen centroid
};

// pqUniformSampleIndices(count, sample): fills sh.picked[0, sample) with the
// sampled indices in increasing order and advances sh.state by the draws the
// walk consumed.  All threads of the block call it.
__device__ void uniform_sample(Kmc2Shared& sh, int64_t count, int sample) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (tid == 0) {
    sh.remaining = sample;
    sh.taken = 0;
    sh.stop = sample <= 0 || count <= 0;
    sh.replay = 0;
  }
  __syncthreads();
  constexpr int kStep = kKmc2Items * kKmc2Threads;
  for (int64_t i0 = 0; !sh.stop; i0 += kStep) {
    const uint64_t st0 = sh.state;
    const int rem0 = sh.remaining;
    // Index i0 + k·1024 + tid takes draw (i - i0 + 1) past st0: every index
    // before the last consumes exactly one draw unless one is rejected
    // (intn rejects only draws below 2^64 mod bound < bound).
    int any = 0;
    for (int k = 0; k < kKmc2Items; ++k) {
      const int64_t i = i0 + (int64_t)k * kKmc2Threads + tid;
      bool hit = false;
      if (i < count) {
        const uint64_t bound = (uint64_t)(count - i);
        if (bound <= 1) {
          hit = 0 < rem0;  // intn(1) is 0 without a draw
        } else {
          const uint64_t v = splitmix_mix(st0 + (uint64_t)(i - i0 + 1) * kGolden);
          if (v < bound && v < (0 - bound) % bound) sh.replay = 1;
          hit = v % bound < (uint64_t)rem0;
        }
      }
      const unsigned m = __ballot_sync(kFullMask, hit);
      if (lane == 0) sh.hits[k * (kKmc2Threads / 32) + warp] = m;
      any |= m != 0;
    }
    any = __syncthreads_or(any);
    if (tid == 0) {
      if (sh.replay) {
        // A rejected draw shifts the stream: walk this step serially.
        uint64_t state = st0;
        int rem = rem0;
        for (int64_t i = i0; i < count && i < i0 + kStep && rem > 0; ++i) {
          const uint64_t r = splitmix_intn_dev(&state, (uint64_t)(count - i));
          if (r == ~0ull) {
            sh.err = 1;
            rem = 0;
            break;
          }
          if (r < (uint64_t)rem) {
            sh.picked[sh.taken++] = (int)i;
            --rem;
          }
        }
        sh.state = state;
        sh.remaining = rem;
        sh.replay = 0;
      } else {
        // Hits in index order: index i is sampled when its draw is below
        // the slots left when it is reached; the walk stops at the last.
        int rem = rem0;
        int64_t last = -1;
        for (int w = 0; any && w < kKmc2Items * (kKmc2Threads / 32) && rem > 0; ++w) {
          unsigned m = sh.hits[w];
          while (m && rem > 0) {
            const int b = __ffs(m) - 1;
            m &= m - 1;
            const int64_t i = i0 + (int64_t)w * 32 + b;
            const uint64_t bound = (uint64_t)(count - i);
            const uint64_t r =
                bound <= 1 ? 0 : splitmix_mix(st0 + (uint64_t)(i - i0 + 1) * kGolden) % bound;
            if (r < (uint64_t)rem) {
              sh.picked[sh.taken++] = (int)i;
              --rem;
              last = i;
            }
          }
        }
        // Draws consumed: one per index walked, except intn(1).
        const int64_t walked_end =
            rem == 0 ? last + 1 : (i0 + kStep < count ? i0 + kStep : count);
        int64_t draws = walked_end - i0;
        if (walked_end == count && draws > 0) --draws;  // index count-1 drew nothing
        sh.state = st0 + (uint64_t)draws * kGolden;
        sh.remaining = rem;
      }
      if (sh.remaining == 0 || i0 + kStep >= count) sh.stop = 1;
    }
    __syncthreads();
  }
}

// initializePQKMC2 for one chunk per block: rows x + i·ld + start, width w.
__global__ void __launch_bounds__(kKmc2Threads, 1)
    pq_kmc2_kernel(const float* __restrict__ x, int64_t n, int ld, const int* __restrict__ offsets,
                   int clusters, uint64_t seed, int metric, int* __restrict__ chosen_out,
                   int* __restrict__ status) {
  __shared__ Kmc2Shared sh;
  const int chunk = blockIdx.x, tid = threadIdx.x;
  const int start = offsets[chunk], w = offsets[chunk + 1] - start;
  if (tid == 0) {
    sh.state = seed ^ (0x70716b6d00000000ull + (uint64_t)chunk);
    sh.err = 0;
    sh.nchosen = 0;
  }
  __syncthreads();
  uniform_sample(sh, n, 1);
  if (tid == 0 && !sh.err) sh.chosen[sh.nchosen++] = sh.picked[0];
  __syncthreads();
  const int chain = (int)(n < kKmc2Chain ? n : kKmc2Chain);
  while (sh.nchosen < clusters && !sh.err) {
    uniform_sample(sh, n, chain);
    if (sh.err) break;
    if (tid < kKmc2Chain) sh.best[tid] = float_to_ordered(3.40282346638528859811704183484516925440e+38f);
    __syncthreads();
    const int nc = sh.nchosen;
    for (int p = tid; p < chain * nc; p += kKmc2Threads) {
      const int cand = p / nc, c = p - cand * nc;
      const float* row = x + (int64_t)sh.picked[cand] * ld + start;
      const float* cen = x + (int64_t)sh.chosen[c] * ld + start;
      float sc = metric == XVEC_METRIC_IP ? thread_reference_sum<1>(cen, row, w)
                                          : thread_reference_sum<0>(cen, row, w);
      if (!finite_f(sc)) {
        sh.err = 1;
        continue;
      }
      if (metric == XVEC_METRIC_IP) sc = -sc;
      atomicMin(&sh.best[cand], float_to_ordered(sc));
    }
    __syncthreads();
    if (tid == 0 && !sh.err) {
      float sel = ordered_to_float(sh.best[0]);
      int pick = 0;
      for (int c = 1; c < chain; ++c) {
        const float sc = ordered_to_float(sh.best[c]);
        bool take = sel == 0.f;
        if (!take) {
          const double u = (double)(splitmix_next_dev(&sh.state) >> 11) * (1.0 / 9007199254740992.0);
          take = __fmul_rn(sel, (float)u) < sc;
        }
        if (take) {
          sel = sc;
          pick = c;
        }
      }
      sh.chosen[sh.nchosen++] = sh.picked[pick];
    }
    __syncthreads();
  }
  if (sh.err) {
    if (tid == 0) atomicExch(status, 1);
    return;
  }
  for (int c = tid; c < clusters; c += kKmc2Threads)
    chosen_out[(int64_t)chunk * kPqCentroids + c] = sh.chosen[c];
}

// training[i][j] = x[i][start + j] for the chunk's w columns.
__global__ void gather_chunk_kernel(const float* __restrict__ x, int64_t n, int ld, int start,
                                    int w, float* __restrict__ out) {
  const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= n * w) return;
  const int64_t i = t / w;
  out[t] = x[i * ld + start + (t - i * w)];
}

// initial[c][j] = training[chosen[c]][j].
__global__ void gather_initial_kernel(const float* __restrict__ training, int w,
                                      const int* __restrict__ chosen, int kc,
                                      float* __restrict__ initial) {
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= kc * w) return;
  const int c = t / w;
  initial[t] = training[(int64_t)chosen[c] * w + (t - c * w)];
}

// pivots[c][start + j] = cents[c < kc ? c : 0][j] for c in [0, 256).
__global__ void scatter_pivots_kernel(const float* __restrict__ cents, int kc, int w, int start,
                                      int d, float* __restrict__ pivots) {
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= kPqCentroids * w) return;
  const int c = t / w, j = t - c * w;
  pivots[(int64_t)c * d + start + j] = cents[(int64_t)(c < kc ? c : 0) * w + j];
}

__global__ void any_non_finite_kernel(const float* x, int64_t count, int* bad) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < count && !finite_f(x[i])) atomicExch(bad, 1);
}

int64_t grid_of(int64_t count) { return (count + 255) / 256; }

// PQOptions.Validate (pq.go:66-84) and the dimension and chunk checks of
// TrainPQ (pq.go:118-136).  Resolves chunks == 0 to d / 2.
xvec_gpu_status validate_pq(int32_t metric, int64_t n, int32_t dim, int32_t* chunks,
                            int64_t max_train_samples, int32_t max_iterations) {
  if (metric != XVEC_METRIC_L2 && metric != XVEC_METRIC_IP)
    return set_error("core: invalid PQ options: core: PQ supports L2 and inner product only"),
           XVEC_GPU_INVALID_ARGUMENT;
  if (*chunks < 0)
    return set_error("core: invalid PQ options: Chunks cannot be negative"),
           XVEC_GPU_INVALID_ARGUMENT;
  if (max_train_samples <= 0)
    return set_error("core: invalid PQ options: MaxTrainSamples must be positive"),
           XVEC_GPU_INVALID_ARGUMENT;
  if (max_iterations <= 0)
    return set_error("core: invalid PQ options: MaxIterations must be positive"),
           XVEC_GPU_INVALID_ARGUMENT;
  if (n <= 0) return set_error("core: k-means training set is empty"), XVEC_GPU_INVALID_ARGUMENT;
  if (dim <= 0 || dim > 65535)
    return set_error("core: invalid PQ options: dimension must be in [1,65535]"),
           XVEC_GPU_INVALID_ARGUMENT;
  if (*chunks == 0) *chunks = dim / 2;
  if (*chunks <= 0 || *chunks > dim)
    return set_error("core: invalid PQ options: resolved Chunks must be in [1,%d]", dim),
           XVEC_GPU_INVALID_ARGUMENT;
  if (n > 0x7fffffffll)
    return set_error("PQ training supports at most 2^31-1 rows"), XVEC_GPU_INVALID_ARGUMENT;
  return XVEC_GPU_OK;
}

void chunk_offsets(int dim, int chunks, int32_t* offsets) {
  const int base = dim / chunks, larger = dim % chunks;
  offsets[0] = 0;
  for (int c = 0; c < chunks; ++c) offsets[c + 1] = offsets[c] + base + (c < larger ? 1 : 0);
}

}  // namespace
}  // namespace xvec

using namespace xvec;

extern "C" xvec_gpu_status xvec_gpu_pq_train_device(
    int32_t device, int32_t metric, const float* d_vectors, int64_t n, int32_t dim,
    int32_t chunks, int64_t max_train_samples, int32_t max_iterations, uint64_t seed,
    int32_t* chunk_offsets_out, float* d_pivots, int32_t* out_chunks, void* stream) {
  xvec_gpu_status st = validate_pq(metric, n, dim, &chunks, max_train_samples, max_iterations);
  if (st) return st;
  if (!d_vectors || !d_pivots)
    return set_error("invalid PQ training arguments"), XVEC_GPU_INVALID_ARGUMENT;
  cudaSetDevice(device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  std::vector<int32_t> offsets(chunks + 1);
  chunk_offsets(dim, chunks, offsets.data());
  const int64_t samples = std::min<int64_t>(n, max_train_samples);
  const int kc = (int)std::min<int64_t>(kPqCentroids, samples);
  Scratch flag, d_offsets, chosen;
  if ((st = flag.alloc(8, s)) || (st = d_offsets.alloc((size_t)(chunks + 1) * 4, s)) ||
      (st = chosen.alloc((size_t)chunks * kPqCentroids * 4, s)))
    return st;
  // validateTrainingVectors over every row (kmeans.go:322-352).
  int h_flag[2] = {0, 0};
  XVEC_CUDA(cudaMemsetAsync(flag.ptr, 0, 8, s));
  any_non_finite_kernel<<<grid_of(n * dim), 256, 0, s>>>(d_vectors, n * dim, flag.as<int>());
  XVEC_LAUNCHED();
  XVEC_CUDA(cudaMemcpyAsync(h_flag, flag.ptr, 8, cudaMemcpyDeviceToHost, s));
  XVEC_CUDA(cudaStreamSynchronize(s));
  if (h_flag[0])
    return set_error("core: training vector: ailego: vector contains a non-finite value"),
           XVEC_GPU_NON_FINITE;
  XVEC_CUDA(cudaMemcpyAsync(d_offsets.ptr, offsets.data(), (size_t)(chunks + 1) * 4,
                            cudaMemcpyHostToDevice, s));
  pq_kmc2_kernel<<<chunks, kKmc2Threads, 0, s>>>(d_vectors, samples, dim, d_offsets.as<int>(), kc,
                                                 seed, metric, chosen.as<int>(),
                                                 flag.as<int>() + 1);
  XVEC_LAUNCHED();
  XVEC_CUDA(cudaMemcpyAsync(h_flag, flag.ptr, 8, cudaMemcpyDeviceToHost, s));
  XVEC_CUDA(cudaStreamSynchronize(s));
  if (h_flag[1])
    return set_error("core: initialize PQ chunk: distance is not finite or the sample walk "
                     "failed"),
           XVEC_GPU_NON_FINITE;
  const int wmax = [&] {
    int m = 0;
    for (int c = 0; c < chunks; ++c) m = std::max(m, offsets[c + 1] - offsets[c]);
    return m;
  }();
  Scratch training, initial, cents, labels;
  if ((st = training.alloc((size_t)samples * wmax * 4, s)) ||
      (st = initial.alloc((size_t)kc * wmax * 4, s)) ||
      (st = cents.alloc((size_t)kc * wmax * 4, s)) || (st = labels.alloc((size_t)samples * 4, s)))
    return st;
  for (int c = 0; c < chunks; ++c) {
    const int start = offsets[c], w = offsets[c + 1] - start;
    gather_chunk_kernel<<<grid_of(samples * w), 256, 0, s>>>(d_vectors, samples, dim, start, w,
                                                             training.as<float>());
    XVEC_LAUNCHED();
    gather_initial_kernel<<<(int)grid_of((int64_t)kc * w), 256, 0, s>>>(
        training.as<float>(), w, chosen.as<int>() + (int64_t)c * kPqCentroids, kc,
        initial.as<float>());
    XVEC_LAUNCHED();
    int32_t iterations = 0, converged = 0;
    double cost = 0;
    st = xvec_gpu_kmeans_train_init_device(device, metric, training.as<float>(), samples, w, kc,
                                           initial.as<float>(), max_iterations,
                                           1.1920928955078125e-7, cents.as<float>(),
                                           labels.as<int32_t>(), &iterations, &converged, &cost,
                                           s);
    if (st) return st;
    scatter_pivots_kernel<<<(int)grid_of((int64_t)kPqCentroids * w), 256, 0, s>>>(
        cents.as<float>(), kc, w, start, dim, d_pivots);
    XVEC_LAUNCHED();
  }
  XVEC_CUDA(cudaStreamSynchronize(s));
  if (chunk_offsets_out)
    std::copy(offsets.begin(), offsets.end(), chunk_offsets_out);
  if (out_chunks) *out_chunks = chunks;
  return XVEC_GPU_OK;
}

extern "C" xvec_gpu_status xvec_gpu_pq_train(int32_t device, int32_t metric,
                                             const float* vectors, int64_t n, int32_t dim,
                                             int32_t chunks, int64_t max_train_samples,
                                             int32_t max_iterations, uint64_t seed,
                                             int32_t* chunk_offsets_out, float* pivots,
                                             int32_t* out_chunks) {
  xvec_gpu_status st = validate_pq(metric, n, dim, &chunks, max_train_samples, max_iterations);
  if (st) return st;
  if (!vectors || !pivots)
    return set_error("invalid PQ training arguments"), XVEC_GPU_INVALID_ARGUMENT;
  // validateTrainingVectors over every row on the host, so that the device
  // holds the training sample alone.
  const int64_t samples = std::min<int64_t>(n, max_train_samples);
  for (int64_t i = 0; i < n * dim; ++i)
    if (!std::isfinite(vectors[i]))
      return set_error("core: training vector %lld: ailego: vector contains a non-finite value",
                       (long long)(i / dim)),
             XVEC_GPU_NON_FINITE;
  cudaSetDevice(device);
  cudaStream_t s = nullptr;
  Scratch dv, dp;
  if ((st = dv.alloc((size_t)samples * dim * 4, s)) ||
      (st = dp.alloc((size_t)kPqCentroids * dim * 4, s)))
    return st;
  XVEC_CUDA(cudaMemcpyAsync(dv.ptr, vectors, (size_t)samples * dim * 4, cudaMemcpyHostToDevice, s));
  st = xvec_gpu_pq_train_device(device, metric, dv.as<float>(), samples, dim, chunks,
                                max_train_samples, max_iterations, seed, chunk_offsets_out,
                                dp.as<float>(), out_chunks, s);
  if (st) return st;
  XVEC_CUDA(cudaMemcpyAsync(pivots, dp.ptr, (size_t)kPqCentroids * dim * 4,
                            cudaMemcpyDeviceToHost, s));
  XVEC_CUDA(cudaStreamSynchronize(s));
  return XVEC_GPU_OK;
}
