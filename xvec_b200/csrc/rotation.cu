// rotation.cu — the collection's rotation reformer on the GPU.
//
// A collection whose vector index has `rotate` set passes every stored and
// query vector through an FHT rotation before the scalar-quantized index sees
// it (collectionReformer, collection.go:1981-2000; RotationReformer.Transform
// and Revert, internal/core/rotation.go:266-280).  The rotation's sign state
// is derived from the collection, so the same schema always rotates the same
// way: SHA-256 of the text "zvec-go-rotation-v1\0<schema>\0<field>\0<dimension>
// \0<index type>\0<quantize type>" followed by a little-endian uint64 counter,
// for counters 0, 1, ..., the digests concatenated up to 4 ((dimension + 7)
// / 8) bytes.
//
// Here: the sign derivation on the host (SHA-256 written from FIPS 180-4),
// and Transform / Revert of a batch of vectors on the device, one block per
// vector, bit-identical to FHTRotator.Rotate / Unrotate (fht.cuh).  A vector
// with a non-finite input or output fails (ErrNonFiniteVector); the call
// reports the first failing vector, as RotateBatch does (rotation.go:187-213).
#include <algorithm>
#include <cmath>
#include <cstring>
#include <string>
#include <vector>

#include "capi_internal.h"
#include "common.cuh"
#include "fht.cuh"

namespace xvec {
namespace {

// ---------------------------------------------------------------------------
// SHA-256 (FIPS 180-4, section 6.2).
// ---------------------------------------------------------------------------
struct Sha256 {
  uint32_t h[8];
  uint8_t block[64];
  size_t fill = 0;
  uint64_t bits = 0;

  static uint32_t rotr(uint32_t x, int n) { return (x >> n) | (x << (32 - n)); }

  Sha256() {
    // The first 32 bits of the fractional parts of the square roots of the
    // first eight primes.
    const uint32_t init[8] = {0x6a09e667u, 0xbb67ae85u, 0x3c6ef372u, 0xa54ff53au,
                              0x510e527fu, 0x9b05688cu, 0x1f83d9abu, 0x5be0cd19u};
    std::memcpy(h, init, sizeof(h));
  }

  void compress(const uint8_t* p) {
    // The first 32 bits of the fractional parts of the cube roots of the
    // first 64 primes.
    static const uint32_t k[64] = {
        0x428a2f98u, 0x71374491u, 0xb5c0fbcfu, 0xe9b5dba5u, 0x3956c25bu, 0x59f111f1u,
        0x923f82a4u, 0xab1c5ed5u, 0xd807aa98u, 0x12835b01u, 0x243185beu, 0x550c7dc3u,
        0x72be5d74u, 0x80deb1feu, 0x9bdc06a7u, 0xc19bf174u, 0xe49b69c1u, 0xefbe4786u,
        0x0fc19dc6u, 0x240ca1ccu, 0x2de92c6fu, 0x4a7484aau, 0x5cb0a9dcu, 0x76f988dau,
        0x983e5152u, 0xa831c66du, 0xb00327c8u, 0xbf597fc7u, 0xc6e00bf3u, 0xd5a79147u,
        0x06ca6351u, 0x14292967u, 0x27b70a85u, 0x2e1b2138u, 0x4d2c6dfcu, 0x53380d13u,
        0x650a7354u, 0x766a0abbu, 0x81c2c92eu, 0x92722c85u, 0xa2bfe8a1u, 0xa81a664bu,
        0xc24b8b70u, 0xc76c51a3u, 0xd192e819u, 0xd6990624u, 0xf40e3585u, 0x106aa070u,
        0x19a4c116u, 0x1e376c08u, 0x2748774cu, 0x34b0bcb5u, 0x391c0cb3u, 0x4ed8aa4au,
        0x5b9cca4fu, 0x682e6ff3u, 0x748f82eeu, 0x78a5636fu, 0x84c87814u, 0x8cc70208u,
        0x90befffau, 0xa4506cebu, 0xbef9a3f7u, 0xc67178f2u};
    uint32_t w[64];
    for (int t = 0; t < 16; ++t)
      w[t] = (uint32_t)p[4 * t] << 24 | (uint32_t)p[4 * t + 1] << 16 |
             (uint32_t)p[4 * t + 2] << 8 | (uint32_t)p[4 * t + 3];
    for (int t = 16; t < 64; ++t) {
      const uint32_t s0 = rotr(w[t - 15], 7) ^ rotr(w[t - 15], 18) ^ (w[t - 15] >> 3);
      const uint32_t s1 = rotr(w[t - 2], 17) ^ rotr(w[t - 2], 19) ^ (w[t - 2] >> 10);
      w[t] = w[t - 16] + s0 + w[t - 7] + s1;
    }
    uint32_t a = h[0], b = h[1], c = h[2], d = h[3], e = h[4], f = h[5], g = h[6], hh = h[7];
    for (int t = 0; t < 64; ++t) {
      const uint32_t S1 = rotr(e, 6) ^ rotr(e, 11) ^ rotr(e, 25);
      const uint32_t ch = (e & f) ^ (~e & g);
      const uint32_t t1 = hh + S1 + ch + k[t] + w[t];
      const uint32_t S0 = rotr(a, 2) ^ rotr(a, 13) ^ rotr(a, 22);
      const uint32_t maj = (a & b) ^ (a & c) ^ (b & c);
      const uint32_t t2 = S0 + maj;
      hh = g;
      g = f;
      f = e;
      e = d + t1;
      d = c;
      c = b;
      b = a;
      a = t1 + t2;
    }
    h[0] += a;
    h[1] += b;
    h[2] += c;
    h[3] += d;
    h[4] += e;
    h[5] += f;
    h[6] += g;
    h[7] += hh;
  }

  void update(const uint8_t* p, size_t len) {
    bits += (uint64_t)len * 8;
    while (len > 0) {
      const size_t take = std::min(len, (size_t)64 - fill);
      std::memcpy(block + fill, p, take);
      fill += take;
      p += take;
      len -= take;
      if (fill == 64) {
        compress(block);
        fill = 0;
      }
    }
  }

  void finish(uint8_t out[32]) {
    // Padding: a one bit, zeros to 56 mod 64 bytes, the message length in
    // bits as a big-endian uint64.
    const uint64_t total = bits;
    const uint8_t one = 0x80, zero = 0;
    update(&one, 1);
    while (fill != 56) update(&zero, 1);
    uint8_t len[8];
    for (int i = 0; i < 8; ++i) len[i] = (uint8_t)(total >> (56 - 8 * i));
    update(len, 8);
    for (int i = 0; i < 8; ++i)
      for (int j = 0; j < 4; ++j) out[4 * i + j] = (uint8_t)(h[i] >> (24 - 8 * j));
  }
};

constexpr int kMaxRotationDimension = 65535;  // MaxRotationDimension (rotation.go:36)
constexpr int kRotateThreads = 256;
constexpr int kRotateSmemFloats = 48 * 1024;  // vectors up to this size rotate in shared memory

int floor_pow2(int v) {
  int r = 1;
  while (r <= v / 2) r *= 2;
  return r;
}

// One block per vector: Rotate (inverse = 0) or Unrotate (inverse = 1) of
// in[b] into out[b]; bad[b] = 1 when the input or the result is not finite.
__global__ void __launch_bounds__(kRotateThreads) fht_rotate_kernel(
    const float* __restrict__ in, int64_t n, int dim, int truncated, float inv,
    const uint8_t* __restrict__ signs, int inverse, int use_smem, float* __restrict__ out,
    int* __restrict__ bad) {
  extern __shared__ float rot_smem[];
  __shared__ int s_bad;
  const int64_t b = blockIdx.x;
  if (b >= n) return;
  const float* src = in + b * dim;
  float* dst = out + b * dim;
  float* v = use_smem ? rot_smem : dst;
  if (threadIdx.x == 0) s_bad = 0;
  __syncthreads();
  for (int i = threadIdx.x; i < dim; i += blockDim.x) {
    const float x = src[i];
    if (!finite_f(x)) s_bad = 1;
    v[i] = x;
  }
  __syncthreads();
  if (inverse)
    block_fht_unrotate(v, dim, truncated, signs, inv);
  else
    block_fht_rotate(v, dim, truncated, signs, inv);
  for (int i = threadIdx.x; i < dim; i += blockDim.x) {
    const float x = v[i];
    if (!finite_f(x)) s_bad = 1;
    if (use_smem) dst[i] = x;
  }
  __syncthreads();
  if (threadIdx.x == 0) bad[b] = s_bad;
}

xvec_gpu_status check_rotation(const uint8_t* signs, int64_t signs_len, int32_t dimension) {
  if (dimension <= 0 || dimension > kMaxRotationDimension)
    return set_error("core: invalid vector rotator: dimension %d", dimension),
           XVEC_GPU_INVALID_ARGUMENT;
  const int64_t want = 4 * (int64_t)((dimension + 7) / 8);
  if (!signs || signs_len != want)
    return set_error("core: invalid rotation sign state: got %lld bytes, want %lld",
                     (long long)signs_len, (long long)want),
           XVEC_GPU_INVALID_ARGUMENT;
  return XVEC_GPU_OK;
}

// Rotates n device vectors on stream s; bad: n ints of device memory.
xvec_gpu_status rotate_device(const uint8_t* h_signs, int64_t signs_len, int32_t dimension,
                              const float* d_in, int64_t n, float* d_out, int inverse, int* bad,
                              cudaStream_t s) {
  const int truncated = floor_pow2(dimension);
  const float inv = 1.0f / (float)std::sqrt((double)(float)truncated);
  Scratch dsigns;
  xvec_gpu_status st;
  if ((st = dsigns.alloc((size_t)signs_len, s))) return st;
  XVEC_CUDA(cudaMemcpyAsync(dsigns.ptr, h_signs, (size_t)signs_len, cudaMemcpyHostToDevice, s));
  const int use_smem = dimension <= kRotateSmemFloats;
  const size_t smem = use_smem ? (size_t)dimension * 4 : 0;
  XVEC_CUDA(cudaFuncSetAttribute(fht_rotate_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)(kRotateSmemFloats * 4)));
  for (int64_t b = 0; b < n; b += (int64_t)1 << 30) {
    const int64_t m = std::min<int64_t>(n - b, (int64_t)1 << 30);
    fht_rotate_kernel<<<(unsigned)m, kRotateThreads, smem, s>>>(
        d_in + b * dimension, m, dimension, truncated, inv, dsigns.as<uint8_t>(), inverse,
        use_smem, d_out + b * dimension, bad + b);
    XVEC_LAUNCHED();
    XVEC_CUDA(cudaGetLastError());
  }
  return XVEC_GPU_OK;
}

// The first failing vector, if any (bad already on the host).
xvec_gpu_status first_bad(const std::vector<int>& bad) {
  for (size_t i = 0; i < bad.size(); ++i)
    if (bad[i]) {
      set_error("core: rotate vector %zu: non-finite vector", i);
      return XVEC_GPU_NON_FINITE;
    }
  return XVEC_GPU_OK;
}

}  // namespace
}  // namespace xvec

using namespace xvec;

extern "C" xvec_gpu_status xvec_gpu_rotation_signs(const char* schema_name, const char* field_name,
                                                   int32_t dimension, int32_t index_type,
                                                   int32_t quantize, uint8_t* out_signs,
                                                   int64_t out_len) {
  if (!schema_name || !field_name || !out_signs)
    return set_error("nil argument"), XVEC_GPU_INVALID_ARGUMENT;
  if (dimension <= 0 || dimension > kMaxRotationDimension)
    return set_error("core: invalid vector rotator: dimension %d", dimension),
           XVEC_GPU_INVALID_ARGUMENT;
  const int64_t want = 4 * (int64_t)((dimension + 7) / 8);
  if (out_len != want)
    return set_error("rotation signs need %lld bytes, got %lld", (long long)want,
                     (long long)out_len),
           XVEC_GPU_INVALID_ARGUMENT;
  std::string seed = "zvec-go-rotation-v1";
  seed.push_back('\0');
  seed += schema_name;
  seed.push_back('\0');
  seed += field_name;
  seed.push_back('\0');
  seed += std::to_string(dimension);
  seed.push_back('\0');
  seed += std::to_string(index_type);
  seed.push_back('\0');
  seed += std::to_string(quantize);
  int64_t offset = 0;
  for (uint64_t counter = 0; offset < want; ++counter) {
    Sha256 h;
    h.update(reinterpret_cast<const uint8_t*>(seed.data()), seed.size());
    uint8_t le[8];
    for (int i = 0; i < 8; ++i) le[i] = (uint8_t)(counter >> (8 * i));
    h.update(le, 8);
    uint8_t digest[32];
    h.finish(digest);
    const int64_t take = std::min<int64_t>(32, want - offset);
    std::memcpy(out_signs + offset, digest, (size_t)take);
    offset += take;
  }
  return XVEC_GPU_OK;
}

extern "C" xvec_gpu_status xvec_gpu_rotate_device(int32_t device, const uint8_t* signs,
                                                  int64_t signs_len, int32_t dimension,
                                                  const float* d_in, int64_t n, float* d_out,
                                                  int32_t inverse, int32_t* d_failed,
                                                  void* stream) {
  xvec_gpu_status st = check_rotation(signs, signs_len, dimension);
  if (st) return st;
  if (n < 0) return set_error("negative vector count"), XVEC_GPU_INVALID_ARGUMENT;
  if (n == 0) return XVEC_GPU_OK;
  if (!d_in || !d_out || !d_failed) return set_error("nil buffer"), XVEC_GPU_INVALID_ARGUMENT;
  XVEC_CUDA(cudaSetDevice(device));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if ((st = rotate_device(signs, signs_len, dimension, d_in, n, d_out, inverse ? 1 : 0, d_failed,
                          s)))
    return st;
  return XVEC_GPU_OK;
}

extern "C" xvec_gpu_status xvec_gpu_rotate(int32_t device, const uint8_t* signs,
                                           int64_t signs_len, int32_t dimension, const float* in,
                                           int64_t n, float* out, int32_t inverse) {
  xvec_gpu_status st = check_rotation(signs, signs_len, dimension);
  if (st) return st;
  if (n < 0) return set_error("negative vector count"), XVEC_GPU_INVALID_ARGUMENT;
  if (n == 0) return XVEC_GPU_OK;
  if (!in || !out) return set_error("nil buffer"), XVEC_GPU_INVALID_ARGUMENT;
  XVEC_CUDA(cudaSetDevice(device));
  cudaStream_t s;
  XVEC_CUDA(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking));
  auto run = [&]() -> xvec_gpu_status {
    const size_t bytes = (size_t)n * dimension * 4;
    Scratch din, dout, dbad;
    xvec_gpu_status s2;
    if ((s2 = din.alloc(bytes, s)) || (s2 = dout.alloc(bytes, s)) ||
        (s2 = dbad.alloc((size_t)n * 4, s)))
      return s2;
    XVEC_CUDA(cudaMemcpyAsync(din.ptr, in, bytes, cudaMemcpyHostToDevice, s));
    if ((s2 = rotate_device(signs, signs_len, dimension, din.as<float>(), n, dout.as<float>(),
                            inverse ? 1 : 0, dbad.as<int>(), s)))
      return s2;
    std::vector<int> bad((size_t)n);
    XVEC_CUDA(cudaMemcpyAsync(bad.data(), dbad.ptr, (size_t)n * 4, cudaMemcpyDeviceToHost, s));
    XVEC_CUDA(cudaMemcpyAsync(out, dout.ptr, bytes, cudaMemcpyDeviceToHost, s));
    XVEC_CUDA(cudaStreamSynchronize(s));
    return first_bad(bad);
  };
  st = run();
  cudaStreamSynchronize(s);
  cudaStreamDestroy(s);
  return st;
}
