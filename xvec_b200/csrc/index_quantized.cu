// index_quantized.cu — dispatch of the per-kind insertion hooks: the
// quantized kinds (SQ8: sq8.cu, IVF-PQ: ivfpq.cu, RaBitQ: rabitq.cu, DiskANN:
// diskann.cu), the IVF
// list assignment (IVF-Flat and IVF-SQ8: ivf_flat.cu) and the
// bfloat16 split of Flat FP32 rows (the tensor-core scan's operands).
#include "flat_tc.cuh"
#include "index_kernels.cuh"

namespace xvec {

static bool flat_fp32(const xvec_gpu_index* idx) {
  return idx->desc.kind == XVEC_INDEX_FLAT && idx->desc.storage == XVEC_STORAGE_FP32;
}

xvec_gpu_status extra_reserve(xvec_gpu_index* idx, int64_t cap, cudaStream_t s) {
  if (flat_fp32(idx)) {
    const size_t row = (size_t)idx->desc.dimension * 2, keep = (size_t)idx->n * row;
    xvec_gpu_status st;
    if ((st = idx->rows_bhi.reserve((size_t)cap * row, keep, s)) ||
        (st = idx->rows_blo.reserve((size_t)cap * row, keep, s)))
      return st;
    return XVEC_GPU_OK;
  }
  if (idx->desc.kind == XVEC_INDEX_SQ8_FLAT || idx->desc.kind == XVEC_INDEX_SQ4_FLAT)
    return sq8_reserve(idx, cap, s);
  if (idx->desc.kind == XVEC_INDEX_IVF_PQ) return ivfpq_reserve(idx, cap, s);
  if (idx->desc.kind == XVEC_INDEX_RABITQ) return rabitq_reserve(idx, cap, s);
  if (idx->desc.kind == XVEC_INDEX_IVF_FLAT) return ivf_flat_reserve(idx, cap, s);
  if (idx->desc.kind == XVEC_INDEX_IVF_SQ8 || idx->desc.kind == XVEC_INDEX_IVF_SQ4) {
    const xvec_gpu_status st = sq8_reserve(idx, cap, s);
    return st ? st : ivf_flat_reserve(idx, cap, s);
  }
  if (idx->desc.kind == XVEC_INDEX_DISKANN) return diskann_reserve(idx, cap, s);
  return XVEC_GPU_OK;
}
xvec_gpu_status extra_validate(xvec_gpu_index* idx, int64_t, int64_t, cudaStream_t) {
  if (idx->desc.kind == XVEC_INDEX_IVF_PQ && !idx->has_model)
    return set_error("set the IVF-PQ model before adding rows"), XVEC_GPU_INVALID_ARGUMENT;
  if (idx->desc.kind == XVEC_INDEX_RABITQ && !idx->has_model)
    return set_error("set the RaBitQ model before adding rows"), XVEC_GPU_INVALID_ARGUMENT;
  if ((idx->desc.kind == XVEC_INDEX_IVF_FLAT || idx->desc.kind == XVEC_INDEX_IVF_SQ8 ||
       idx->desc.kind == XVEC_INDEX_IVF_SQ4) &&
      !idx->has_model)
    return set_error("set the IVF model before adding rows"), XVEC_GPU_INVALID_ARGUMENT;
  if (idx->desc.kind == XVEC_INDEX_DISKANN && !idx->has_model)
    return set_error("set the DiskANN PQ model before adding rows"), XVEC_GPU_INVALID_ARGUMENT;
  return XVEC_GPU_OK;
}
xvec_gpu_status extra_commit(xvec_gpu_index* idx, int64_t old_n, int64_t m, cudaStream_t s) {
  if (flat_fp32(idx)) {
    const int64_t d = idx->desc.dimension;
    XVEC_CUDA(launch_split_bf16(idx->rows.as<float>() + old_n * d, m * d,
                                idx->rows_bhi.as<__nv_bfloat16>() + old_n * d,
                                idx->rows_blo.as<__nv_bfloat16>() + old_n * d, s));
    XVEC_LAUNCHED();
    return XVEC_GPU_OK;
  }
  if (idx->desc.kind == XVEC_INDEX_SQ8_FLAT || idx->desc.kind == XVEC_INDEX_SQ4_FLAT)
    return sq8_commit(idx, old_n, m, s);
  if (idx->desc.kind == XVEC_INDEX_IVF_PQ) return ivfpq_commit(idx, old_n, m, s);
  if (idx->desc.kind == XVEC_INDEX_RABITQ) return rabitq_commit(idx, old_n, m, s);
  if (idx->desc.kind == XVEC_INDEX_IVF_FLAT) return ivf_flat_commit(idx, old_n, m, s);
  if (idx->desc.kind == XVEC_INDEX_IVF_SQ8 || idx->desc.kind == XVEC_INDEX_IVF_SQ4) {
    const xvec_gpu_status st = sq8_commit(idx, old_n, m, s);
    return st ? st : ivf_flat_commit(idx, old_n, m, s);
  }
  if (idx->desc.kind == XVEC_INDEX_DISKANN) return diskann_commit(idx, old_n, m, s);
  return XVEC_GPU_OK;
}

}  // namespace xvec
