// Data-layout kernels around the fused kernel: query scaling and fp16 hi/lo split, database
// decoding, norms, norm-sorted layout, per-tile bounds and the position-ordered allow bits.
#pragma once

#include <cstdint>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "knn_fused.cuh"

namespace ovvs {
namespace prim {

// Ranking family of a reference metric (ovvs.h ovvsMetric): how the fused kernel turns a dot
// product into a ranking value, and which exact formula the merge kernel re-evaluates.
enum MetricCode : int {
  kMetricL2 = 0,
  kMetricL2Sqrt = 1,
  kMetricInnerProduct = 2,
  kMetricCosine = 3,
  kMetricHamming = 4,
  kMetricLp = 5,
  kMetricDirectL2 = 6,  // any other enum value: sum (x - y)^2 (internal.hpp:269-270 default)
};

// RankKind used by the fused kernel for a metric.
__host__ __device__ inline int rank_kind_of(int metric_code) {
  switch (metric_code) {
    case kMetricInnerProduct:
    case kMetricHamming:
      return kRankScaled;
    case kMetricCosine:
      return kRankColumnScaled;
    default:
      return kRankAffine;  // L2, L2 sqrt, Lp (p = 2) and the direct-L2 default rank by |x-y|^2
  }
}

// ovvsMetric value -> MetricCode (unknown values behave like the direct squared L2).
inline int normalize_metric(int m) { return (m >= 0 && m <= 5) ? m : kMetricDirectL2; }

// Query preparation. queries: [nq x dim] fp32 (device). Writes, for q < q_pad (rows >= nq are
// zero): a16 [q_pad x 2*dp] fp16 (hi part in columns [0,dp), lo part in [dp,2dp)), q_mul
// [q_pad], xn [q_pad] (sequential fp32 squared norm, the reference's nrm2sq), and sets
// *lo_flag = 1 if any lo element is non-zero. e_db is the database's power-of-two scale.
void launch_query_prep(const float* queries, int64_t nq, int64_t q_pad, int dim, int dp,
                       int metric_code, int e_db, __half* a16, float* q_mul, float* xn,
                       int* lo_flag, cudaStream_t stream, int16_t* e_q = nullptr);

// q_mul from the per-query exponents a previous launch_query_prep wrote to e_q, for an index
// with exponent e_db (what query prep computes, without re-reading the queries).
void launch_query_mul(const int16_t* e_q, int64_t nq, int64_t q_pad, int metric_code, int e_db,
                      float* q_mul, cudaStream_t stream);

// Per-row statistics of the database in original order. data: raw [n x dim] of `dtype`
// (ovvsDType). Writes norm[n] (sequential fp32 squared norm of the decoded row), sort_key[n]
// (the fused kernel's aux: |y|^2, -1/max(|y|,1e-6) or 0) and atomically maxes *absmax_bits with
// the largest |decoded value| (fp32 bit pattern, finite values only).
void launch_row_stats(const void* data, int dtype, int64_t n, int dim, int metric_code,
                      float* norm, float* sort_key, unsigned int* absmax_bits, cudaStream_t stream);

// Scatter rows into norm-sorted position order. perm[pos] = original id for pos < n.
// rows16: [n_pad x b_parts*dp] fp16 MMA operand (hi | lo), exact32: [n_pad x dim] fp32 copy or
// null, aux/norm_sorted by position, row_id[pos], inv_perm[id]. Positions >= n are zero rows.
void launch_scatter_rows(const void* data, int dtype, int64_t n, int64_t n_pad, int dim, int dp,
                         int b_parts, int metric_code, int e_db, const uint32_t* perm,
                         const float* norm, const float* sort_key, __half* rows16,
                         float* exact32, float* aux, float* norm_sorted, uint32_t* row_id,
                         uint32_t* inv_perm, cudaStream_t stream);

// tile_aux[t] = (min, max) of aux over valid positions of tile t (256 rows), for t < num_tiles,
// followed by the same range per group of kGroupTiles consecutive tiles:
// tile_aux[num_tiles + g] covers tiles [g * kGroupTiles, (g + 1) * kGroupTiles). The buffer holds
// num_tiles + ceil(num_tiles / kGroupTiles) entries.
constexpr int kGroupTiles = 8;
constexpr int kGroupShift = 3;
inline int group_count(int num_tiles) { return (num_tiles + kGroupTiles - 1) / kGroupTiles; }
void launch_tile_bounds(const float* aux, int64_t n, int num_tiles, float2* tile_aux,
                        cudaStream_t stream);

// allow_pos[pos/32] bit (pos%32) = bitset bit (row_offset + row_id[pos]), 0 for padding.
void launch_allow_bits(const uint8_t* bitset, int64_t row_offset, const uint32_t* row_id,
                       int64_t n, int64_t n_pad, uint32_t* allow_pos, cudaStream_t stream);

}  // namespace prim
}  // namespace ovvs
