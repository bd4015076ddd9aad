// ivf_file.cu — the reference's IVF file (ZVECIVF version 1, IVFIndex.Save /
// OpenIVFIndex, internal/core/ivf.go:717-1173) read into a device IVF index,
// and rows added with their lists given.
//
// Layout (little endian): a 112-byte header
//   [0,8) magic "ZVECIVF\0"      [8,10) version 1       [10,12) header size 112
//   [12,16) reserved 0            [16,24) file length    [24,32) payload length
//   [32,40) count                 [40,44) dimension      [44,48) effective nlist
//   [48] metric  [49] converged   [50,52) reserved 0     [52,56) options NList
//   [56,60) NIterations           [60,68) Workers (int64) [68,76) Seed
//   [76,84) Tolerance (float64)   [84,92) training cost (float64)
//   [92,96) training iterations   [96,100) CRC32C of the payload
//   [100,108) reserved 0          [108,112) CRC32C of header[0,108)
// then the payload: nlist centroids (dimension float32 each), then count
// records {uint64 key, dimension float32, uint32 list} in position order
// (encodeIVFIndex, ivf.go:866-904).
//
// The reader checks what decodeIVFIndex (ivf.go:906-1057) checks, in its
// order: the header's form, its checksum, the lengths, the sizes, the payload
// checksum, the options (IVFBuildOptions.Validate, ivf.go:66-80), the training
// metadata, finite centroids and vectors, unique keys and list ranges.  The
// lists are uploaded as the file gives them: an index grown by streaming
// adds need not hold each row in its nearest centroid's list.  All of this
// is host code; the device work is the index's own insertion.
#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <vector>

#include "capi_internal.h"
#include "index_kernels.cuh"

namespace xvec {

xvec_gpu_status add_device_locked(xvec_gpu_index* idx, const uint64_t* d_keys, const void* d_rows,
                                  int64_t m, cudaStream_t s);
cudaStream_t thread_stream(int device);

namespace {

constexpr size_t kIvfHeader = 112;
constexpr uint64_t kIvfRecordOverhead = 12;  // key uint64 + list uint32
constexpr uint32_t kMaxIvfDimension = 65535;  // MaxRotationDimension (rotation.go:36)

// CRC-32C (Castagnoli, reflected polynomial 0x82F63B78, init and final xor
// 0xFFFFFFFF), the checksum of hashutil.CRC32C; slicing by 8 bytes.
struct Crc32cTables {
  uint32_t t[8][256];
  Crc32cTables() {
    for (uint32_t b = 0; b < 256; ++b) {
      uint32_t c = b;
      for (int k = 0; k < 8; ++k) c = (c & 1u) ? (c >> 1) ^ 0x82F63B78u : c >> 1;
      t[0][b] = c;
    }
    for (uint32_t b = 0; b < 256; ++b)
      for (int s = 1; s < 8; ++s) t[s][b] = (t[s - 1][b] >> 8) ^ t[0][t[s - 1][b] & 0xffu];
  }
};
const Crc32cTables& crc_tables() {
  static const Crc32cTables tables;
  return tables;
}

uint32_t crc32c(const uint8_t* p, size_t n) {
  const Crc32cTables& T = crc_tables();
  uint32_t c = 0xFFFFFFFFu;
  while (n >= 8) {
    uint32_t lo, hi;
    std::memcpy(&lo, p, 4);
    std::memcpy(&hi, p + 4, 4);
    lo ^= c;
    c = T.t[7][lo & 0xff] ^ T.t[6][(lo >> 8) & 0xff] ^ T.t[5][(lo >> 16) & 0xff] ^
        T.t[4][lo >> 24] ^ T.t[3][hi & 0xff] ^ T.t[2][(hi >> 8) & 0xff] ^
        T.t[1][(hi >> 16) & 0xff] ^ T.t[0][hi >> 24];
    p += 8;
    n -= 8;
  }
  while (n--) c = (c >> 8) ^ T.t[0][(c ^ *p++) & 0xffu];
  return c ^ 0xFFFFFFFFu;
}

template <typename T>
T load_le(const uint8_t* p) {
  T v;
  std::memcpy(&v, p, sizeof(T));  // the hosts this library runs on are little endian
  return v;
}

bool finite_bits(uint32_t bits) { return (bits & 0x7f800000u) != 0x7f800000u; }

struct ParsedIvf {
  xvec_gpu_ivf_file_header header{};
  std::vector<uint8_t> bytes;  // the whole file
};

xvec_gpu_status invalid(const char* what) {
  set_error("core: open IVF file: core: invalid IVF file: %s", what);
  return XVEC_GPU_INVALID_ARGUMENT;
}

xvec_gpu_status read_file(const char* path, std::vector<uint8_t>* out) {
  if (!path || !*path) return invalid("empty path");
  FILE* f = std::fopen(path, "rb");
  if (!f) return set_error("core: read IVF file: cannot open %s", path), XVEC_GPU_NOT_FOUND;
  std::fseek(f, 0, SEEK_END);
  const long len = std::ftell(f);
  std::fseek(f, 0, SEEK_SET);
  if (len < 0) {
    std::fclose(f);
    return set_error("core: read IVF file: cannot size %s", path), XVEC_GPU_INVALID_ARGUMENT;
  }
  out->resize((size_t)len);
  const size_t got = len ? std::fread(out->data(), 1, (size_t)len, f) : 0;
  std::fclose(f);
  if (got != (size_t)len) return set_error("core: read IVF file: short read"), XVEC_GPU_INVALID_ARGUMENT;
  return XVEC_GPU_OK;
}

// decodeIVFIndex (ivf.go:906-1057) without building the index.
xvec_gpu_status parse_ivf(const char* path, ParsedIvf* out) {
  xvec_gpu_status st = read_file(path, &out->bytes);
  if (st) return st;
  const std::vector<uint8_t>& e = out->bytes;
  if (e.size() < kIvfHeader) return invalid("truncated header");
  const uint8_t* h = e.data();
  static const uint8_t kMagic[8] = {'Z', 'V', 'E', 'C', 'I', 'V', 'F', 0};
  if (std::memcmp(h, kMagic, 8) != 0) return invalid("bad magic");
  const uint16_t version = load_le<uint16_t>(h + 8);
  if (version != 1)
    return set_error("core: open IVF file: core: unsupported IVF file version: %u", version),
           XVEC_GPU_UNSUPPORTED;
  if (load_le<uint16_t>(h + 10) != kIvfHeader) return invalid("bad header size");
  if (load_le<uint32_t>(h + 12) != 0 || load_le<uint16_t>(h + 50) != 0 ||
      load_le<uint64_t>(h + 100) != 0)
    return invalid("nonzero reserved field");
  const uint32_t hcrc = crc32c(h, 108);
  if (hcrc != load_le<uint32_t>(h + 108))
    return set_error("core: open IVF file: core: IVF checksum mismatch: header got %08x, want %08x",
                     hcrc, load_le<uint32_t>(h + 108)),
           XVEC_GPU_CHECKSUM_MISMATCH;
  if (load_le<uint64_t>(h + 16) != (uint64_t)e.size() ||
      load_le<uint64_t>(h + 24) != (uint64_t)(e.size() - kIvfHeader))
    return invalid("inconsistent file length");
  const uint64_t count = load_le<uint64_t>(h + 32);
  const uint64_t dim = load_le<uint32_t>(h + 40);
  const uint64_t nlist = load_le<uint32_t>(h + 44);
  if (dim == 0 || dim > kMaxIvfDimension) return invalid("invalid dimension");
  if (count > (uint64_t)INT64_MAX) return invalid("count exceeds platform capacity");
  if ((count == 0 && nlist != 0) || (count != 0 && (nlist == 0 || nlist > count)))
    return invalid("invalid effective list count");
  // checkedIVFPayloadSize (ivf.go:1154-1173).
  const uint64_t centroid_bytes = nlist * dim * 4;
  const uint64_t record = kIvfRecordOverhead + dim * 4;
  if (count != 0 && count > (UINT64_MAX - centroid_bytes) / record)
    return invalid("invalid payload length");
  const uint64_t payload_size = centroid_bytes + count * record;
  if (payload_size != (uint64_t)(e.size() - kIvfHeader)) return invalid("invalid payload length");
  const uint8_t* payload = h + kIvfHeader;
  const uint32_t pcrc = crc32c(payload, (size_t)payload_size);
  if (pcrc != load_le<uint32_t>(h + 96))
    return set_error("core: open IVF file: core: IVF checksum mismatch: payload got %08x, want %08x",
                     pcrc, load_le<uint32_t>(h + 96)),
           XVEC_GPU_CHECKSUM_MISMATCH;
  // decodeIVFOptions (ivf.go:1059-1076) + IVFBuildOptions.Validate.
  xvec_gpu_ivf_file_header& o = out->header;
  o.count = (int64_t)count;
  o.dimension = (int32_t)dim;
  o.nlist = (int32_t)nlist;
  o.metric = h[48];
  o.converged = h[49];
  o.options_nlist = load_le<uint32_t>(h + 52);
  o.options_iterations = load_le<uint32_t>(h + 56);
  o.options_workers = load_le<int64_t>(h + 60);
  o.options_seed = load_le<uint64_t>(h + 68);
  o.options_tolerance = load_le<double>(h + 76);
  o.training_cost = load_le<double>(h + 84);
  o.training_iterations = (int64_t)load_le<uint32_t>(h + 92);
  const uint32_t opt_nlist = load_le<uint32_t>(h + 52), opt_iters = load_le<uint32_t>(h + 56);
  if (o.metric < XVEC_METRIC_L2 || o.metric > XVEC_METRIC_MIPSL2)
    return invalid("core: invalid IVF options: invalid metric");
  if (opt_nlist == 0) return invalid("core: invalid IVF options: NList must be positive");
  if (opt_iters == 0) return invalid("core: invalid IVF options: NIterations must be positive");
  if (!(o.options_tolerance >= 0) || std::isinf(o.options_tolerance))
    return invalid("core: invalid IVF options: Tolerance must be finite and non-negative");
  if (o.converged > 1 || std::isnan(o.training_cost) || std::isinf(o.training_cost) ||
      (uint64_t)o.training_iterations > (uint64_t)opt_iters)
    return invalid("invalid training metadata");
  if (count == 0 && (o.training_cost != 0 || o.training_iterations != 0 || o.converged != 0))
    return invalid("empty index has training metadata");
  size_t off = 0;
  for (uint64_t i = 0; i < nlist * dim; ++i, off += 4)
    if (!finite_bits(load_le<uint32_t>(payload + off))) return invalid("non-finite centroid");
  std::vector<uint64_t> keys((size_t)count);
  for (uint64_t r = 0; r < count; ++r) {
    const uint8_t* rec = payload + centroid_bytes + r * record;
    keys[(size_t)r] = load_le<uint64_t>(rec);
    for (uint64_t c = 0; c < dim; ++c)
      if (!finite_bits(load_le<uint32_t>(rec + 8 + 4 * c))) return invalid("non-finite vector");
    if ((uint64_t)load_le<uint32_t>(rec + 8 + 4 * dim) >= nlist)
      return invalid("vector list out of range");
  }
  std::sort(keys.begin(), keys.end());
  for (size_t i = 1; i < keys.size(); ++i)
    if (keys[i] == keys[i - 1]) return invalid("duplicate key");
  return XVEC_GPU_OK;
}

}  // namespace
}  // namespace xvec

using namespace xvec;

extern "C" xvec_gpu_status xvec_gpu_ivf_file_info(const char* path,
                                                  xvec_gpu_ivf_file_header* out) {
  if (!out) return set_error("nil argument"), XVEC_GPU_INVALID_ARGUMENT;
  ParsedIvf f;
  const xvec_gpu_status st = parse_ivf(path, &f);
  if (st) return st;
  *out = f.header;
  return XVEC_GPU_OK;
}

extern "C" xvec_gpu_status xvec_gpu_ivf_add_with_lists(xvec_gpu_index* idx, const uint64_t* keys,
                                                       const float* rows, const int32_t* lists,
                                                       int64_t n) {
  if (!idx || n < 0 || (n > 0 && (!keys || !rows || !lists)))
    return set_error("invalid add arguments"), XVEC_GPU_INVALID_ARGUMENT;
  if (idx->desc.kind != XVEC_INDEX_IVF_FLAT && idx->desc.kind != XVEC_INDEX_IVF_SQ8 &&
      idx->desc.kind != XVEC_INDEX_IVF_SQ4)
    return set_error("not an IVF index"), XVEC_GPU_INVALID_ARGUMENT;
  if (n == 0) return XVEC_GPU_OK;
  std::unique_lock<std::shared_mutex> lock(idx->mu);
  if (!idx->has_model) return set_error("set the IVF model before adding rows"), XVEC_GPU_INVALID_ARGUMENT;
  for (int64_t i = 0; i < n; ++i)
    if (lists[i] < 0 || lists[i] >= idx->nlist)
      return set_error("list %d of row %lld is out of range", lists[i], (long long)i),
             XVEC_GPU_INVALID_ARGUMENT;
  cudaSetDevice(idx->device);
  cudaStream_t s = thread_stream(idx->device);
  const size_t row_bytes = (size_t)idx->desc.dimension * 4;
  Scratch dk, dr, dl;
  xvec_gpu_status st;
  if ((st = dk.alloc((size_t)n * 8, s)) || (st = dr.alloc((size_t)n * row_bytes, s)) ||
      (st = dl.alloc((size_t)n * 4, s)))
    return st;
  XVEC_CUDA(cudaMemcpyAsync(dk.ptr, keys, (size_t)n * 8, cudaMemcpyHostToDevice, s));
  XVEC_CUDA(cudaMemcpyAsync(dr.ptr, rows, (size_t)n * row_bytes, cudaMemcpyHostToDevice, s));
  XVEC_CUDA(cudaMemcpyAsync(dl.ptr, lists, (size_t)n * 4, cudaMemcpyHostToDevice, s));
  idx->given_lists = dl.as<int32_t>();
  st = add_device_locked(idx, dk.as<uint64_t>(), dr.ptr, n, s);
  idx->given_lists = nullptr;
  cudaStreamSynchronize(s);
  return st;
}

extern "C" xvec_gpu_status xvec_gpu_ivf_open(const char* path, int32_t device,
                                             xvec_gpu_index** out) {
  if (!out) return set_error("nil argument"), XVEC_GPU_INVALID_ARGUMENT;
  *out = nullptr;
  ParsedIvf f;
  xvec_gpu_status st = parse_ivf(path, &f);
  if (st) return st;
  const xvec_gpu_ivf_file_header& h = f.header;
  xvec_gpu_index_desc desc{};
  desc.kind = XVEC_INDEX_IVF_FLAT;
  desc.dimension = h.dimension;
  desc.metric = h.metric;
  desc.storage = XVEC_STORAGE_FP32;
  desc.device = device;
  xvec_gpu_index* idx = nullptr;
  if ((st = xvec_gpu_index_create(&desc, &idx))) return st;
  if (h.count > 0) {
    const int d = h.dimension;
    const uint8_t* payload = f.bytes.data() + kIvfHeader;
    std::vector<float> cents((size_t)h.nlist * d);
    std::memcpy(cents.data(), payload, cents.size() * 4);
    if ((st = xvec_gpu_ivf_set_model(idx, cents.data(), h.nlist))) {
      xvec_gpu_index_destroy(idx);
      return st;
    }
    if ((st = xvec_gpu_index_reserve(idx, h.count))) {
      xvec_gpu_index_destroy(idx);
      return st;
    }
    // Records in position order, de-interleaved a batch at a time.
    const size_t record = kIvfRecordOverhead + (size_t)d * 4;
    const uint8_t* records = payload + cents.size() * 4;
    const int64_t batch = std::max<int64_t>(1, std::min<int64_t>(h.count, (1 << 28) / record));
    std::vector<uint64_t> keys;
    std::vector<float> rows;
    std::vector<int32_t> lists;
    for (int64_t b = 0; b < h.count; b += batch) {
      const int64_t m = std::min(batch, h.count - b);
      keys.resize((size_t)m);
      rows.resize((size_t)m * d);
      lists.resize((size_t)m);
      for (int64_t i = 0; i < m; ++i) {
        const uint8_t* rec = records + (size_t)(b + i) * record;
        keys[(size_t)i] = load_le<uint64_t>(rec);
        std::memcpy(rows.data() + (size_t)i * d, rec + 8, (size_t)d * 4);
        lists[(size_t)i] = (int32_t)load_le<uint32_t>(rec + 8 + (size_t)d * 4);
      }
      if ((st = xvec_gpu_ivf_add_with_lists(idx, keys.data(), rows.data(), lists.data(), m))) {
        xvec_gpu_index_destroy(idx);
        return st;
      }
    }
  }
  *out = idx;
  return XVEC_GPU_OK;
}
