// flat_tc.cuh — tensor-core (tcgen05) candidate scan for FP16 Flat search.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace xvec {

// True when the TMA/UMMA path can take this layout (d % 8 == 0, d >= 64,
// 16-byte aligned operands, driver entry point available).
bool flat_tc_supported(int d, const void* rows, const void* queries);
// Candidate list entries per (query, list); lists are stored with this stride.
int flat_tc_cap();
// Candidate lists per row part (one per column half of the tile).
int flat_tc_lists_per_part();
// True when a batch of nq queries runs on CTA pairs (256 queries per pair);
// the grid then has an even number of 128-query blocks.
bool flat_tc_pairs(int nq);

// Scans rows [0, n) (row i at rows + i * row_stride_elems) against nq queries.
// row_aux: 1/||x|| for cosine, ||x||^2 for L2 / MIPS (unused for IP);
// q_aux: 1/||q|| for cosine, ||q||^2 otherwise.  gthr: per-query key
// thresholds shared by all lists of a query (initialise to all ones, or to
// a bound already known).  The launch fills lists [list_base, list_base +
// 2 * num_parts) of the num_lists lists each query has (cand: [nq][num_lists]
// [cap] keys, part_counts / part_sat: [nq][num_lists]).  status != 0 after
// the launch = a bounded wait expired (the results are then invalid).
cudaError_t launch_flat_scan_tc(int metric, const __half* queries, int nq, const __half* rows,
                                int64_t n, int d, int64_t row_stride_elems, const float* row_aux,
                                const uint32_t* keyrank, const float* q_aux, const float* q_n2,
                                unsigned long long* gthr, const uint32_t* bitmap, int num_parts,
                                int kp, int list_base, int num_lists, uint64_t* cand,
                                int* part_counts, uint64_t* part_sat, int* q_flags, int* status,
                                cudaStream_t stream);

// The same scan over INT8 codes (SQ8 index, L2 or IP): tcgen05 kind::i8 on
// the row codes [n][d] and the query codes [nq][d], exact int32 dot products
// ranked with the SQ8 fast rank (row_info / q_info: the float4 rank terms of
// sq8.cu).  Lists, thresholds and status as for launch_flat_scan_tc.
cudaError_t launch_sq8_scan_tc(int metric, const int8_t* qcodes, int nq, const int8_t* codes,
                               int64_t n, int d, const float4* row_info, const uint32_t* keyrank,
                               const float4* q_info, unsigned long long* gthr,
                               const uint32_t* bitmap, int num_parts, int kp, int list_base,
                               int num_lists, uint64_t* cand, int* part_counts,
                               uint64_t* part_sat, int* q_flags, int* status,
                               cudaStream_t stream);
// The same scan for float32 rows and queries held as bfloat16 high and low
// parts (x = hi + lo to 2^-18 |x|): three MMAs per k-step (hi·hi, hi·lo,
// lo·hi) into one fp32 accumulator; ranks as launch_flat_scan_tc.
cudaError_t launch_flat_scan_tc_split(int metric, const __nv_bfloat16* q_hi,
                                      const __nv_bfloat16* q_lo, int nq, const __nv_bfloat16* r_hi,
                                      const __nv_bfloat16* r_lo, int64_t n, int d,
                                      const float* row_aux, const uint32_t* keyrank,
                                      const float* q_aux, const float* q_n2,
                                      unsigned long long* gthr, const uint32_t* bitmap,
                                      int num_parts, int kp, int list_base, int num_lists,
                                      uint64_t* cand, int* part_counts, uint64_t* part_sat,
                                      int* q_flags, int* status, cudaStream_t stream);
// hi = bf16(x), lo = bf16(x - hi) for `count` float32 values.
cudaError_t launch_split_bf16(const float* x, int64_t count, __nv_bfloat16* hi, __nv_bfloat16* lo,
                              cudaStream_t stream);
// True when the INT8 tensor-core scan can take this layout.
bool sq8_tc_supported(int d, const void* codes, const void* qcodes);

// The same scan for the RaBitQ index on INT8 tensor cores: rows = the codes
// as int8 planes [n][2 padded] (127 b | b); each query = integers [nq][2 padded]
// (h | l) with 127 h + l = round(rotated query / scale), so the int32
// accumulator is the exact integer dot product of the bits with the scaled
// query; ranked with the RaBitQ fast estimate (row_info: {add, rescale,
// cluster bits, 0}; q_terms: {sum/2, scale}; q_gadd: [nq][nc]).
cudaError_t launch_rabitq_scan_tc(const int8_t* q_int, int nq, const int8_t* planes, int64_t n,
                                  int padded, const float4* row_info, const uint32_t* keyrank,
                                  const float2* q_terms, const float* q_gadd, int nc,
                                  unsigned long long* gthr, const uint32_t* bitmap,
                                  int num_parts, int kp, int list_base, int num_lists,
                                  uint64_t* cand, int* part_counts, uint64_t* part_sat,
                                  int* q_flags, int* status, cudaStream_t stream);
// Multi-bit RaBitQ (TotalBits <= 8) on INT8 tensor cores: rows = the code
// values as the int8 plane v - 128 [n][padded]; queries = 16-bit integers
// w = round(rotated query / scale) as two int8 planes, q_planes [2][nq][padded]
// (h, then l, w = 256 h + l + 128), so two exact int32 accumulators give
// sum(v w) = 256 A_h + A_l + 128 sum(v - 128) + 128 sum(w).  row_info:
// {full add, full rescale, cluster bits, 128 sum(v - 128)}; q_terms:
// {-(center sum) - scale 128 sum(w), scale}; ranked with the multi-bit fast
// estimate.  Lists, thresholds and status as for launch_flat_scan_tc.
cudaError_t launch_rabitq8_scan_tc(const int8_t* q_planes, int nq, const int8_t* vplane,
                                   int64_t n, int padded, const float4* row_info,
                                   const uint32_t* keyrank, const float2* q_terms,
                                   const float* q_gadd, int nc, unsigned long long* gthr,
                                   const uint32_t* bitmap, int num_parts, int kp, int list_base,
                                   int num_lists, uint64_t* cand, int* part_counts,
                                   uint64_t* part_sat, int* q_flags, int* status,
                                   cudaStream_t stream);
bool rabitq8_tc_supported(int padded, const void* vplane, const void* q_planes);
// Most clusters the RaBitQ tensor-core epilogue takes.
int rabitq_tc_max_clusters();
// True when the RaBitQ tensor-core scan can take this layout.
bool rabitq_tc_supported(int padded, const void* planes, const void* q_int);

}  // namespace xvec
