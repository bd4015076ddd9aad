// index_quantized.cu — dispatch of the per-kind hooks of the quantized index
// kinds (SQ8: sq8.cu, IVF-PQ: ivfpq.cu, RaBitQ: rabitq.cu).
#include "index_kernels.cuh"

namespace xvec {

xvec_gpu_status extra_reserve(xvec_gpu_index* idx, int64_t cap, cudaStream_t s) {
  if (idx->desc.kind == XVEC_INDEX_SQ8_FLAT) return sq8_reserve(idx, cap, s);
  if (idx->desc.kind == XVEC_INDEX_IVF_PQ) return ivfpq_reserve(idx, cap, s);
  if (idx->desc.kind == XVEC_INDEX_RABITQ) return rabitq_reserve(idx, cap, s);
  return XVEC_GPU_OK;
}
xvec_gpu_status extra_validate(xvec_gpu_index* idx, int64_t, int64_t, cudaStream_t) {
  if (idx->desc.kind == XVEC_INDEX_IVF_PQ && !idx->has_model)
    return set_error("set the IVF-PQ model before adding rows"), XVEC_GPU_INVALID_ARGUMENT;
  if (idx->desc.kind == XVEC_INDEX_RABITQ && !idx->has_model)
    return set_error("set the RaBitQ model before adding rows"), XVEC_GPU_INVALID_ARGUMENT;
  return XVEC_GPU_OK;
}
xvec_gpu_status extra_commit(xvec_gpu_index* idx, int64_t old_n, int64_t m, cudaStream_t s) {
  if (idx->desc.kind == XVEC_INDEX_SQ8_FLAT) return sq8_commit(idx, old_n, m, s);
  if (idx->desc.kind == XVEC_INDEX_IVF_PQ) return ivfpq_commit(idx, old_n, m, s);
  if (idx->desc.kind == XVEC_INDEX_RABITQ) return rabitq_commit(idx, old_n, m, s);
  return XVEC_GPU_OK;
}

}  // namespace xvec
