// comm.cu — the multi-GPU search behind the C ABI: the library's own NCCL
// communicator and the sharded search over it.
//
// The reference fans one query out over a collection's segments inside one
// process and merges the per-segment top-k with MergeSearchResults
// (collection.go:4040-4066, internal/core/query.go:154-191).  Here each GPU
// holds one shard of the rows (its own index; keys are unique across
// shards).  A sharded search runs the shard's own search, exchanges every
// shard's lists with ONE NCCL all-gather of a packed buffer (keys, scores and
// counts of all queries) and merges them with the MergeSearchResults order
// on every rank.  Refined searches (SQ8/SQ4 Flat and IVF with a refine scale,
// RaBitQ with refine) take two exchanges so that the refined candidates are
// those of the whole index, as RefinedSearch takes them (refiner.go:133-166):
// candidates → exchange → merge by rank → refine the merged keys each shard
// holds → exchange → merge under the index metric.
//
// NCCL is opened at run time, so the library loads without it: the copy the
// process already holds (for example PyTorch's), else XVEC_GPU_NCCL_LIBRARY,
// else libnccl.so.2.  Communicators are non-blocking, and every wait on them
// (initialisation, a collective) polls with a deadline: when it passes, the
// communicator is aborted and the call returns XVEC_GPU_TIMEOUT, so a rank
// that never joined or stopped answering ends the call with an error instead
// of a hang.  An aborted communicator fails every later call with
// XVEC_GPU_NCCL_ERROR; destroy it and make a new one.
#include <dlfcn.h>
#include <nccl.h>

#include <atomic>
#include <chrono>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <thread>
#include <type_traits>
#include <vector>

#include "capi_internal.h"
#include "flat_kernels.cuh"
#include "common.cuh"

struct xvec_gpu_comm {
  int device = 0;
  int nranks = 1;
  int rank = 0;
  ncclComm_t comm = nullptr;
  cudaStream_t stream = nullptr;  // the host-memory search's stream
  int64_t timeout_ms = 60000;
  std::atomic<bool> broken{false};
  std::mutex mu;  // one exchange sequence at a time on a communicator
};

namespace xvec {
namespace {

struct NcclApi {
  bool ok = false;
  char error[256] = {};
  ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
  ncclResult_t (*CommInitRankConfig)(ncclComm_t*, int, ncclUniqueId, int, ncclConfig_t*) = nullptr;
  ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t*) = nullptr;
  ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
  ncclResult_t (*CommFinalize)(ncclComm_t) = nullptr;
  ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
  ncclResult_t (*AllGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t,
                            cudaStream_t) = nullptr;
  ncclResult_t (*GroupStart)() = nullptr;
  ncclResult_t (*GroupEnd)() = nullptr;
  const char* (*GetErrorString)(ncclResult_t) = nullptr;
};

NcclApi load_nccl() {
  NcclApi api;
  void* h = nullptr;
  const char* env = std::getenv("XVEC_GPU_NCCL_LIBRARY");
  if (env && *env) h = dlopen(env, RTLD_NOW | RTLD_LOCAL);
  if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
  if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_LOCAL);
  if (!h) {
    const char* e = dlerror();
    snprintf(api.error, sizeof(api.error), "NCCL not available: %s", e ? e : "dlopen failed");
    return api;
  }
  bool all = true;
  auto sym = [&](auto& fn, const char* name) {
    fn = reinterpret_cast<std::remove_reference_t<decltype(fn)>>(dlsym(h, name));
    if (!fn && all) {
      all = false;
      snprintf(api.error, sizeof(api.error), "NCCL library lacks %s", name);
    }
  };
  sym(api.GetUniqueId, "ncclGetUniqueId");
  sym(api.CommInitRankConfig, "ncclCommInitRankConfig");
  sym(api.CommGetAsyncError, "ncclCommGetAsyncError");
  sym(api.CommAbort, "ncclCommAbort");
  sym(api.CommFinalize, "ncclCommFinalize");
  sym(api.CommDestroy, "ncclCommDestroy");
  sym(api.AllGather, "ncclAllGather");
  sym(api.GroupStart, "ncclGroupStart");
  sym(api.GroupEnd, "ncclGroupEnd");
  sym(api.GetErrorString, "ncclGetErrorString");
  api.ok = all;
  return api;
}

const NcclApi& nccl() {
  static const NcclApi api = load_nccl();
  return api;
}

xvec_gpu_status need_nccl() {
  if (!nccl().ok) return set_error("%s", nccl().error), XVEC_GPU_UNSUPPORTED;
  return XVEC_GPU_OK;
}

const char* nccl_msg(ncclResult_t r) { return nccl().GetErrorString(r); }

using Clock = std::chrono::steady_clock;

bool past(Clock::time_point t0, int64_t timeout_ms) {
  return std::chrono::duration_cast<std::chrono::milliseconds>(Clock::now() - t0).count() >
         timeout_ms;
}

void abort_comm(xvec_gpu_comm* c) {
  if (!c->broken.exchange(true) && c->comm) nccl().CommAbort(c->comm);
}

// Waits until the communicator leaves ncclInProgress (non-blocking
// initialisation, or a call that returned ncclInProgress).
xvec_gpu_status wait_ready(xvec_gpu_comm* c, Clock::time_point t0, const char* what) {
  for (;;) {
    ncclResult_t r = ncclInProgress;
    const ncclResult_t e = nccl().CommGetAsyncError(c->comm, &r);
    if (e != ncclSuccess) r = e;
    if (r == ncclSuccess) return XVEC_GPU_OK;
    if (r != ncclInProgress) {
      set_error("%s: %s", what, nccl_msg(r));
      abort_comm(c);
      return XVEC_GPU_NCCL_ERROR;
    }
    if (past(t0, c->timeout_ms)) {
      set_error("%s: no progress within %lld ms (a rank did not join or stopped answering)",
                what, (long long)c->timeout_ms);
      abort_comm(c);
      return XVEC_GPU_TIMEOUT;
    }
    std::this_thread::sleep_for(std::chrono::microseconds(50));
  }
}

// Waits for the work enqueued on `s` so far (the collective and what follows
// it) while watching the communicator for asynchronous errors.
xvec_gpu_status wait_stream(xvec_gpu_comm* c, cudaStream_t s, const char* what) {
  cudaEvent_t ev;
  XVEC_CUDA(cudaEventCreateWithFlags(&ev, cudaEventDisableTiming));
  cudaError_t e = cudaEventRecord(ev, s);
  if (e != cudaSuccess) {
    cudaEventDestroy(ev);
    XVEC_CUDA(e);
  }
  const Clock::time_point t0 = Clock::now();
  xvec_gpu_status st = XVEC_GPU_OK;
  for (;;) {
    e = cudaEventQuery(ev);
    if (e == cudaSuccess) break;
    if (e != cudaErrorNotReady) {
      set_error("%s: %s", what, cudaGetErrorString(e));
      st = XVEC_GPU_CUDA_ERROR;
      break;
    }
    ncclResult_t r = ncclSuccess;
    nccl().CommGetAsyncError(c->comm, &r);
    if (r != ncclSuccess && r != ncclInProgress) {
      set_error("%s: %s", what, nccl_msg(r));
      abort_comm(c);
      st = XVEC_GPU_NCCL_ERROR;
      break;
    }
    if (past(t0, c->timeout_ms)) {
      set_error("%s: not complete within %lld ms (a rank stopped answering)", what,
                (long long)c->timeout_ms);
      abort_comm(c);
      st = XVEC_GPU_TIMEOUT;
      break;
    }
    std::this_thread::sleep_for(std::chrono::microseconds(20));
  }
  cudaEventDestroy(ev);
  return st;
}

__global__ void fill_status_kernel(int* counts, int nq, int value) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < nq) counts[i] = value;
}

// A rank whose own step failed as a whole still takes part in the exchange,
// with every query failed by that status, so that all ranks take the same
// collective steps and all of them report the failure.
xvec_gpu_status fail_all(int* d_counts, int nq, xvec_gpu_status st, cudaStream_t s) {
  fill_status_kernel<<<(nq + 255) / 256, 256, 0, s>>>(d_counts, nq, -(int)st);
  XVEC_LAUNCHED();
  XVEC_CUDA(cudaGetLastError());
  return XVEC_GPU_OK;
}

bool whole_call_failure(xvec_gpu_status st) { return st != XVEC_GPU_OK; }

__global__ void fill_float_kernel(float* p, size_t n, float v) {
  const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) p[i] = v;
}

// All-gathers count floats per rank (the Flat band exchange); bounded.
xvec_gpu_status allgather_floats(xvec_gpu_comm* c, const float* send, float* recv, size_t count,
                                 cudaStream_t s) {
  const ncclResult_t r = nccl().AllGather(send, recv, count, ncclFloat32, c->comm, s);
  xvec_gpu_status st;
  if (r == ncclInProgress) {
    if ((st = wait_ready(c, Clock::now(), "band all-gather enqueue"))) return st;
  } else if (r != ncclSuccess) {
    set_error("ncclAllGather: %s", nccl_msg(r));
    abort_comm(c);
    return XVEC_GPU_NCCL_ERROR;
  }
  return wait_stream(c, s, "all-gather of the fast-rank bands");
}

// The band exchange of a sharded Flat search: used by every rank exactly
// once per search (a rank whose search ended before its band takes part
// with an empty band, so that all ranks take the same collective steps).
struct FlatBand {
  BandExchange ex;
  bool on = false;
  FlatBand(xvec_gpu_comm* c, const xvec_gpu_index* idx, int k) {
    on = c->nranks > 1 && idx->desc.kind == XVEC_INDEX_FLAT && flat_band_supported(c->nranks, k);
    ex.nranks = c->nranks;
    ex.allgather = [c](const float* send, float* recv, size_t count, cudaStream_t s) {
      return allgather_floats(c, send, recv, count, s);
    };
  }
  BandExchange* get() { return on ? &ex : nullptr; }
  // Takes part with +inf ranks when the search did not reach its band.
  xvec_gpu_status finish(int nq, int k, cudaStream_t s) {
    if (!on || ex.used) return XVEC_GPU_OK;
    ex.used = true;
    const size_t w = (size_t)nq * (k + 1);
    Scratch send, recv;
    xvec_gpu_status st;
    if ((st = send.alloc(w * 4, s)) || (st = recv.alloc(w * 4 * ex.nranks, s))) return st;
    fill_float_kernel<<<(unsigned)((w + 255) / 256), 256, 0, s>>>(send.as<float>(), w, INFINITY);
    XVEC_LAUNCHED();
    XVEC_CUDA(cudaGetLastError());
    return ex.allgather(send.as<float>(), recv.as<float>(), w, s);
  }
};

// One rank's lists in the exchange: keys [nq kk] uint64, scores [nq kk]
// float32, counts [nq] int32, padded to 16 bytes.
struct Packed {
  size_t scores_off, counts_off, bytes;
  Packed(int nq, int kk) {
    scores_off = (size_t)nq * kk * 8;
    counts_off = scores_off + (size_t)nq * kk * 4;
    bytes = (counts_off + (size_t)nq * 4 + 15) / 16 * 16;
  }
};

// All-gathers every rank's lists and merges them (MergeSearchResults) into
// the outputs; h_counts (optional) receives the merged counts.  Bounded.
xvec_gpu_status exchange_merge(xvec_gpu_comm* c, int metric, int kk, int nq,
                               const uint64_t* keys, const float* scores, const int* counts,
                               uint64_t* out_keys, float* out_scores, int* out_counts,
                               std::vector<int>* h_counts, cudaStream_t s) {
  const Packed L(nq, kk);
  Scratch send, recv;
  xvec_gpu_status st;
  if ((st = send.alloc(L.bytes, s)) || (st = recv.alloc(L.bytes * c->nranks, s))) return st;
  unsigned char* sb = send.as<unsigned char>();
  XVEC_CUDA(cudaMemcpyAsync(sb, keys, (size_t)nq * kk * 8, cudaMemcpyDeviceToDevice, s));
  XVEC_CUDA(cudaMemcpyAsync(sb + L.scores_off, scores, (size_t)nq * kk * 4,
                            cudaMemcpyDeviceToDevice, s));
  XVEC_CUDA(cudaMemcpyAsync(sb + L.counts_off, counts, (size_t)nq * 4, cudaMemcpyDeviceToDevice,
                            s));
  const ncclResult_t r = nccl().AllGather(sb, recv.ptr, L.bytes, ncclUint8, c->comm, s);
  if (r == ncclInProgress) {
    if ((st = wait_ready(c, Clock::now(), "all-gather enqueue"))) return st;
  } else if (r != ncclSuccess) {
    set_error("ncclAllGather: %s", nccl_msg(r));
    abort_comm(c);
    return XVEC_GPU_NCCL_ERROR;
  }
  const unsigned char* rb = recv.as<unsigned char>();
  if ((st = launch_merge_results(
           metric, kk, nq, c->nranks, reinterpret_cast<const uint64_t*>(rb),
           (int64_t)(L.bytes / 8), reinterpret_cast<const float*>(rb + L.scores_off),
           (int64_t)(L.bytes / 4), reinterpret_cast<const int*>(rb + L.counts_off),
           (int64_t)(L.bytes / 4), out_keys, out_scores, out_counts, s)))
    return st;
  // The bounded wait comes first: a copy into pageable host memory would
  // block until the stream drains, collective included.
  if ((st = wait_stream(c, s, "all-gather of the shard results"))) return st;
  if (h_counts) {
    h_counts->resize(nq);
    XVEC_CUDA(cudaMemcpyAsync(h_counts->data(), out_counts, (size_t)nq * 4,
                              cudaMemcpyDeviceToHost, s));
    XVEC_CUDA(cudaStreamSynchronize(s));
  }
  return XVEC_GPU_OK;
}

// One rank's part of a sharded search, outputs in device memory.
xvec_gpu_status rank_search(xvec_gpu_comm* c, xvec_gpu_index* idx, const void* d_q, int nq,
                            const xvec_gpu_search_opts& o, cudaStream_t s, uint64_t* d_keys,
                            float* d_scores, int* d_counts, std::vector<int>* h_counts) {
  xvec_gpu_search_opts opts = o;
  opts.stream = s;
  const int k = o.top_k;
  const int cand = xvec_gpu_index_candidate_count(idx, &opts);
  xvec_gpu_status st;
  if (cand > 0) {
    // Refined: the whole index's candidates, then the refine of each shard's.
    Scratch ck, cr, cc, mk, mr, mc, rk, rs, rc;
    if ((st = ck.alloc((size_t)nq * cand * 8, s)) || (st = cr.alloc((size_t)nq * cand * 4, s)) ||
        (st = cc.alloc((size_t)nq * 4, s)) || (st = mk.alloc((size_t)nq * cand * 8, s)) ||
        (st = mr.alloc((size_t)nq * cand * 4, s)) || (st = mc.alloc((size_t)nq * 4, s)) ||
        (st = rk.alloc((size_t)nq * k * 8, s)) || (st = rs.alloc((size_t)nq * k * 4, s)) ||
        (st = rc.alloc((size_t)nq * 4, s)))
      return st;
    st = xvec_gpu_index_candidates_device(idx, d_q, nq, &opts, ck.as<uint64_t>(), cr.as<float>(),
                                          cc.as<int>());
    if (whole_call_failure(st) && (st = fail_all(cc.as<int>(), nq, st, s))) return st;
    if ((st = exchange_merge(c, XVEC_METRIC_L2, cand, nq, ck.as<uint64_t>(), cr.as<float>(),
                             cc.as<int>(), mk.as<uint64_t>(), mr.as<float>(), mc.as<int>(),
                             nullptr, s)))
      return st;
    st = xvec_gpu_index_refine_device(idx, static_cast<const float*>(d_q), nq, mk.as<uint64_t>(),
                                      cand, mc.as<int>(), k, o.radius, s, rk.as<uint64_t>(),
                                      rs.as<float>(), rc.as<int>());
    if (whole_call_failure(st) && (st = fail_all(rc.as<int>(), nq, st, s))) return st;
    return exchange_merge(c, idx->desc.metric, k, nq, rk.as<uint64_t>(), rs.as<float>(),
                          rc.as<int>(), d_keys, d_scores, d_counts, h_counts, s);
  }
  Scratch lk, ls, lc;
  if ((st = lk.alloc((size_t)nq * k * 8, s)) || (st = ls.alloc((size_t)nq * k * 4, s)) ||
      (st = lc.alloc((size_t)nq * 4, s)))
    return st;
  FlatBand band(c, idx, k);
  {
    std::shared_lock<std::shared_mutex> lock(idx->mu);
    std::vector<int> statuses;
    st = search_device_locked(idx, d_q, nq, opts, opts.filter_bitmap, lk.as<uint64_t>(),
                              ls.as<float>(), lc.as<int>(), s, &statuses, band.get());
  }
  if (c->broken.load()) return st != XVEC_GPU_OK ? st : XVEC_GPU_NCCL_ERROR;
  xvec_gpu_status bst = band.finish(nq, k, s);
  if (bst == XVEC_GPU_TIMEOUT || bst == XVEC_GPU_NCCL_ERROR) return bst;
  if (st == XVEC_GPU_OK) st = bst;
  if (whole_call_failure(st) && (st = fail_all(lc.as<int>(), nq, st, s))) return st;
  return exchange_merge(c, idx->desc.metric, k, nq, lk.as<uint64_t>(), ls.as<float>(),
                        lc.as<int>(), d_keys, d_scores, d_counts, h_counts, s);
}

// The call's status from the merged counts: the first failed query's.
xvec_gpu_status status_of(const std::vector<int>& h_counts) {
  for (size_t q = 0; q < h_counts.size(); ++q)
    if (h_counts[q] < 0) {
      set_error("query %zu failed with status %d", q, -h_counts[q]);
      return (xvec_gpu_status)(-h_counts[q]);
    }
  return XVEC_GPU_OK;
}

xvec_gpu_status usable(const xvec_gpu_comm* c) {
  if (!c) return set_error("nil communicator"), XVEC_GPU_INVALID_ARGUMENT;
  if (c->broken.load())
    return set_error("the communicator was aborted; destroy it and make a new one"),
           XVEC_GPU_NCCL_ERROR;
  return XVEC_GPU_OK;
}

xvec_gpu_comm* new_comm(int device, int nranks, int rank, int32_t timeout_ms) {
  auto* c = new xvec_gpu_comm();
  c->device = device;
  c->nranks = nranks;
  c->rank = rank;
  c->timeout_ms = timeout_ms > 0 ? timeout_ms : 60000;
  return c;
}

ncclConfig_t nonblocking_config() {
  ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
  cfg.blocking = 0;
  return cfg;
}

void free_comm(xvec_gpu_comm* c) {
  if (!c) return;
  if (c->comm) {
    if (!c->broken.load()) {
      // Flush, then free; an unfinished flush ends in an abort (bounded).
      cudaSetDevice(c->device);
      const ncclResult_t r = nccl().CommFinalize(c->comm);
      xvec_gpu_status st = XVEC_GPU_OK;
      if (r == ncclInProgress || r == ncclSuccess)
        st = wait_ready(c, Clock::now(), "communicator finalize");
      else
        abort_comm(c);
      if (st == XVEC_GPU_OK && !c->broken.load()) nccl().CommDestroy(c->comm);
    }
    // A broken communicator was freed by its abort.
  }
  if (c->stream) cudaStreamDestroy(c->stream);
  delete c;
}

}  // namespace
}  // namespace xvec

using namespace xvec;

extern "C" xvec_gpu_status xvec_gpu_comm_unique_id(uint8_t* id_out) {
  if (!id_out) return set_error("nil id buffer"), XVEC_GPU_INVALID_ARGUMENT;
  xvec_gpu_status st = need_nccl();
  if (st) return st;
  ncclUniqueId id;
  const ncclResult_t r = nccl().GetUniqueId(&id);
  if (r != ncclSuccess) return set_error("ncclGetUniqueId: %s", nccl_msg(r)), XVEC_GPU_NCCL_ERROR;
  static_assert(sizeof(id) == XVEC_GPU_COMM_ID_BYTES, "NCCL unique id size");
  std::memcpy(id_out, &id, sizeof(id));
  return XVEC_GPU_OK;
}

extern "C" xvec_gpu_status xvec_gpu_comm_init_rank(int32_t device, const uint8_t* id,
                                                   int32_t nranks, int32_t rank,
                                                   int32_t timeout_ms, xvec_gpu_comm** out) {
  if (!out || !id) return set_error("nil argument"), XVEC_GPU_INVALID_ARGUMENT;
  *out = nullptr;
  if (nranks < 1 || rank < 0 || rank >= nranks)
    return set_error("rank %d of %d is out of range", rank, nranks), XVEC_GPU_INVALID_ARGUMENT;
  xvec_gpu_status st = need_nccl();
  if (st) return st;
  XVEC_CUDA(cudaSetDevice(device));
  xvec_gpu_comm* c = new_comm(device, nranks, rank, timeout_ms);
  ncclUniqueId uid;
  std::memcpy(&uid, id, sizeof(uid));
  ncclConfig_t cfg = nonblocking_config();
  const Clock::time_point t0 = Clock::now();
  const ncclResult_t r = nccl().CommInitRankConfig(&c->comm, nranks, uid, rank, &cfg);
  if (r != ncclSuccess && r != ncclInProgress) {
    set_error("ncclCommInitRankConfig: %s", nccl_msg(r));
    if (c->comm) abort_comm(c);
    c->comm = nullptr;
    free_comm(c);
    return XVEC_GPU_NCCL_ERROR;
  }
  if ((st = wait_ready(c, t0, "communicator initialisation"))) {
    free_comm(c);
    return st;
  }
  cudaError_t e = cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking);
  if (e != cudaSuccess) {
    free_comm(c);
    XVEC_CUDA(e);
  }
  *out = c;
  return XVEC_GPU_OK;
}

extern "C" xvec_gpu_status xvec_gpu_comm_init_all(const int32_t* devices, int32_t ndev,
                                                  int32_t timeout_ms, xvec_gpu_comm** out) {
  if (!devices || !out || ndev < 1) return set_error("invalid arguments"), XVEC_GPU_INVALID_ARGUMENT;
  for (int i = 0; i < ndev; ++i) out[i] = nullptr;
  xvec_gpu_status st = need_nccl();
  if (st) return st;
  ncclUniqueId uid;
  ncclResult_t r = nccl().GetUniqueId(&uid);
  if (r != ncclSuccess) return set_error("ncclGetUniqueId: %s", nccl_msg(r)), XVEC_GPU_NCCL_ERROR;
  std::vector<xvec_gpu_comm*> comms(ndev);
  for (int i = 0; i < ndev; ++i) comms[i] = new_comm(devices[i], ndev, i, timeout_ms);
  auto release = [&]() {
    for (auto* c : comms) {
      if (c->comm && !c->broken.load()) abort_comm(c);
      c->comm = nullptr;
      free_comm(c);
    }
  };
  // One thread initialises every rank: the calls go in one NCCL group.
  const Clock::time_point t0 = Clock::now();
  nccl().GroupStart();
  ncclResult_t first = ncclSuccess;
  for (int i = 0; i < ndev; ++i) {
    if (cudaSetDevice(devices[i]) != cudaSuccess) {
      cudaGetLastError();
      first = ncclInvalidArgument;
      break;
    }
    ncclConfig_t cfg = nonblocking_config();
    r = nccl().CommInitRankConfig(&comms[i]->comm, ndev, uid, i, &cfg);
    if (r != ncclSuccess && r != ncclInProgress && first == ncclSuccess) first = r;
  }
  r = nccl().GroupEnd();
  if (first != ncclSuccess || (r != ncclSuccess && r != ncclInProgress)) {
    set_error("communicator initialisation: %s",
              nccl_msg(first != ncclSuccess ? first : r));
    release();
    return XVEC_GPU_NCCL_ERROR;
  }
  for (int i = 0; i < ndev; ++i) {
    cudaSetDevice(devices[i]);
    if ((st = wait_ready(comms[i], t0, "communicator initialisation"))) {
      release();
      return st;
    }
  }
  for (int i = 0; i < ndev; ++i) {
    cudaSetDevice(devices[i]);
    if (cudaStreamCreateWithFlags(&comms[i]->stream, cudaStreamNonBlocking) != cudaSuccess) {
      cudaGetLastError();
      release();
      return set_error("stream creation failed"), XVEC_GPU_CUDA_ERROR;
    }
  }
  for (int i = 0; i < ndev; ++i) out[i] = comms[i];
  return XVEC_GPU_OK;
}

extern "C" xvec_gpu_status xvec_gpu_comm_destroy(xvec_gpu_comm* comm) {
  if (!comm) return XVEC_GPU_OK;
  {
    std::lock_guard<std::mutex> lock(comm->mu);
  }
  free_comm(comm);
  return XVEC_GPU_OK;
}

extern "C" xvec_gpu_status xvec_gpu_comm_abort(xvec_gpu_comm* comm) {
  if (!comm) return set_error("nil communicator"), XVEC_GPU_INVALID_ARGUMENT;
  if (nccl().ok) {
    cudaSetDevice(comm->device);
    abort_comm(comm);
  }
  return XVEC_GPU_OK;
}

extern "C" int32_t xvec_gpu_comm_size(const xvec_gpu_comm* comm) { return comm ? comm->nranks : 0; }
extern "C" int32_t xvec_gpu_comm_rank(const xvec_gpu_comm* comm) { return comm ? comm->rank : -1; }

extern "C" xvec_gpu_status xvec_gpu_sharded_search_device(
    xvec_gpu_comm* comm, xvec_gpu_index* idx, const void* d_queries, int32_t nq,
    const xvec_gpu_search_opts* opts, uint64_t* d_out_keys, float* d_out_scores,
    int32_t* d_out_counts) {
  xvec_gpu_status st = usable(comm);
  if (st || (st = validate_search(idx, nq, opts))) return st;
  if (idx->device != comm->device)
    return set_error("index on device %d, communicator on device %d", idx->device, comm->device),
           XVEC_GPU_INVALID_ARGUMENT;
  if (nq == 0) return XVEC_GPU_OK;
  if (!d_queries || !d_out_keys || !d_out_scores || !d_out_counts)
    return set_error("nil buffer"), XVEC_GPU_INVALID_ARGUMENT;
  std::lock_guard<std::mutex> lock(comm->mu);
  if ((st = usable(comm))) return st;
  cudaSetDevice(comm->device);
  std::vector<int> h_counts;
  if ((st = rank_search(comm, idx, d_queries, nq, *opts, static_cast<cudaStream_t>(opts->stream),
                        d_out_keys, d_out_scores, d_out_counts, &h_counts)))
    return st;
  return status_of(h_counts);
}

extern "C" xvec_gpu_status xvec_gpu_sharded_search(xvec_gpu_comm* const* comms,
                                                   xvec_gpu_index* const* indexes, int32_t ndev,
                                                   const void* queries, int32_t nq,
                                                   const xvec_gpu_search_opts* opts,
                                                   uint64_t* out_keys, float* out_scores,
                                                   int32_t* out_counts) {
  if (!comms || !indexes || ndev < 1) return set_error("invalid arguments"), XVEC_GPU_INVALID_ARGUMENT;
  xvec_gpu_status st;
  for (int i = 0; i < ndev; ++i) {
    if ((st = usable(comms[i])) || (st = validate_search(indexes[i], nq, opts))) return st;
    if (comms[i]->nranks != ndev || comms[i]->rank != i)
      return set_error("communicator %d is rank %d of %d", i, comms[i]->rank, comms[i]->nranks),
             XVEC_GPU_INVALID_ARGUMENT;
    if (indexes[i]->device != comms[i]->device)
      return set_error("index %d is on device %d, its communicator on %d", i,
                       indexes[i]->device, comms[i]->device),
             XVEC_GPU_INVALID_ARGUMENT;
    if (indexes[i]->desc.dimension != indexes[0]->desc.dimension ||
        indexes[i]->desc.metric != indexes[0]->desc.metric ||
        query_elem_bytes(indexes[i]) != query_elem_bytes(indexes[0]))
      return set_error("shard %d differs from shard 0 in dimension, metric or query type", i),
             XVEC_GPU_INVALID_ARGUMENT;
  }
  if (opts->filter_bitmap)
    return set_error("a filter bitmap holds one shard's positions: filter through "
                     "xvec_gpu_sharded_search_device, each rank with its own bitmap"),
           XVEC_GPU_INVALID_ARGUMENT;
  if (nq == 0) return XVEC_GPU_OK;
  if (!queries || !out_keys || !out_scores || !out_counts)
    return set_error("nil buffer"), XVEC_GPU_INVALID_ARGUMENT;
  const int k = opts->top_k;
  const size_t qbytes =
      (size_t)nq * indexes[0]->desc.dimension * query_elem_bytes(indexes[0]);
  // One thread per device: copy the queries in, search the shard, exchange
  // and merge; rank 0 copies the merged lists out.
  std::vector<xvec_gpu_status> sts(ndev, XVEC_GPU_OK);
  std::vector<std::string> errs(ndev);
  std::vector<int> h_counts;
  std::vector<std::thread> threads;
  for (int i = 0; i < ndev; ++i) {
    threads.emplace_back([&, i]() {
      xvec_gpu_comm* c = comms[i];
      std::lock_guard<std::mutex> lock(c->mu);
      auto run = [&]() -> xvec_gpu_status {
        XVEC_CUDA(cudaSetDevice(c->device));
        cudaStream_t s = c->stream;
        Scratch dq, dk, ds, dc;
        xvec_gpu_status s2;
        if ((s2 = dq.alloc(qbytes, s)) || (s2 = dk.alloc((size_t)nq * k * 8, s)) ||
            (s2 = ds.alloc((size_t)nq * k * 4, s)) || (s2 = dc.alloc((size_t)nq * 4, s)))
          return s2;
        XVEC_CUDA(cudaMemcpyAsync(dq.ptr, queries, qbytes, cudaMemcpyHostToDevice, s));
        if ((s2 = rank_search(c, indexes[i], dq.ptr, nq, *opts, s, dk.as<uint64_t>(),
                              ds.as<float>(), dc.as<int>(), i == 0 ? &h_counts : nullptr)))
          return s2;
        if (i == 0) {
          XVEC_CUDA(cudaMemcpyAsync(out_keys, dk.ptr, (size_t)nq * k * 8, cudaMemcpyDeviceToHost,
                                    s));
          XVEC_CUDA(cudaMemcpyAsync(out_scores, ds.ptr, (size_t)nq * k * 4,
                                    cudaMemcpyDeviceToHost, s));
          XVEC_CUDA(cudaMemcpyAsync(out_counts, dc.ptr, (size_t)nq * 4, cudaMemcpyDeviceToHost,
                                    s));
          XVEC_CUDA(cudaStreamSynchronize(s));
        }
        return XVEC_GPU_OK;
      };
      sts[i] = run();
      if (sts[i]) {
        char buf[1024];
        xvec_gpu_last_error(buf, sizeof(buf));
        errs[i] = buf;
      }
    });
  }
  for (auto& t : threads) t.join();
  for (int i = 0; i < ndev; ++i)
    if (sts[i]) return set_error("shard %d: %s", i, errs[i].c_str()), sts[i];
  return status_of(h_counts);
}
