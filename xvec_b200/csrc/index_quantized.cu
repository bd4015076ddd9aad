// index_quantized.cu — SQ8, IVF-PQ and RaBitQ index kinds.
#include "index_kernels.cuh"

namespace xvec {

xvec_gpu_status extra_reserve(xvec_gpu_index* idx, int64_t cap, cudaStream_t s) {
  if (idx->desc.kind == XVEC_INDEX_SQ8_FLAT) return sq8_reserve(idx, cap, s);
  if (idx->desc.kind == XVEC_INDEX_IVF_PQ) return ivfpq_reserve(idx, cap, s);
  return XVEC_GPU_OK;
}
xvec_gpu_status extra_validate(xvec_gpu_index* idx, int64_t, int64_t, cudaStream_t) {
  if (idx->desc.kind == XVEC_INDEX_IVF_PQ && !idx->has_model)
    return set_error("set the IVF-PQ model before adding rows"), XVEC_GPU_INVALID_ARGUMENT;
  if (idx->desc.kind == XVEC_INDEX_RABITQ)
    return set_error("index kind not available yet"), XVEC_GPU_UNSUPPORTED;
  return XVEC_GPU_OK;
}
xvec_gpu_status extra_commit(xvec_gpu_index* idx, int64_t old_n, int64_t m, cudaStream_t s) {
  if (idx->desc.kind == XVEC_INDEX_SQ8_FLAT) return sq8_commit(idx, old_n, m, s);
  if (idx->desc.kind == XVEC_INDEX_IVF_PQ) return ivfpq_commit(idx, old_n, m, s);
  return XVEC_GPU_OK;
}
xvec_gpu_status rabitq_search_impl(xvec_gpu_index*, const float*, int, const xvec_gpu_search_opts&,
                                   const uint32_t*, uint64_t*, float*, int*, cudaStream_t,
                                   std::vector<int>*) {
  return set_error("index kind not available yet"), XVEC_GPU_UNSUPPORTED;
}

}  // namespace xvec

extern "C" xvec_gpu_status xvec_gpu_rabitq_set_model(xvec_gpu_index*, const float*, int32_t,
                                                     const uint8_t*) {
  return XVEC_GPU_UNSUPPORTED;
}
