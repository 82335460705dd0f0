// Candidate merge, exact re-ranking and cross-shard merge.
//
// The fused kernel leaves, per query, num_sc sorted lists of KL (ranking value, row id) keys. The
// merge kernel keeps the KL best of their union, recomputes each survivor's distance from the
// original values with the reference's own fp32 operation order (src/prim/mixer.cpp:174-221,
// src/internal.hpp:215-272: sequential accumulation, no FMA contraction), and orders them by the
// reference's top-k total order (src/prim/cpu/cpu_prims.cpp:24-32). Reported distances are
// therefore the reference's bits whenever the same neighbours are selected.
#pragma once

#include <cstdint>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

namespace ovvs {
namespace prim {

struct MergeParams {
  const uint64_t* cand;      // [q_pad][num_sc][kl]
  int num_sc;                // sorted lists per query
  int kl;
  int64_t nq;
  int dim;
  const float* queries;      // [nq][dim] original fp32 queries
  const float* xn;           // [q_pad] sequential squared norms
  int metric;                // MetricCode
  const float* exact32;      // [n_pad][dim] by position (fp32 datasets), or null
  const __half* rows16;      // [n_pad][rows16_stride] by position (fp16-exact datasets)
  int rows16_stride;
  const float* norm_sorted;  // [n_pad] sequential squared norms by position
  const uint32_t* inv_perm;  // row id -> position
  const uint32_t* allow;     // position-ordered allow bits, or null
  int64_t row_offset;        // global id of local row 0
  int k_eff;                 // output row stride and count
  // World size 1: final results.
  int64_t* neighbors;        // [nq][k_eff] or null
  float* distances;          // [nq][k_eff]
  // World size > 1: this shard's ranking values and global ids for the all-gather.
  float* shard_rank;         // [nq][k_eff] or null
  int64_t* shard_gid;
  int negate_output;         // inner product: report -rank (= +dot)
  // k-means assignment (one GPU, L2, k = 1, no bitset): when the best candidate's approximate
  // value is below the second's by more than their error bound, its id is the exact argmin and
  // is written without the exact recomputation (the distance written is then approximate).
  int labels_only;
};

cudaError_t launch_merge_rerank(const MergeParams& p, cudaStream_t stream);

// Large k. tau_key[q] = the k-th smallest key of the union of the num_sc sorted lists of kl keys
// in cand (kEmptyKey when the union has fewer than k keys): an upper bound on the k-th best key
// of the whole database, since the union holds real rows.
// Large k, between stages of the append pass: tau_key[q] = min(tau_key[q], an upper bound on the
// need-th smallest key among the min(app_count[q], cap) keys appended so far), for queries that
// appended at least `need` keys.
cudaError_t launch_tighten_tau(const uint64_t* app_buf, const uint32_t* app_count, int cap,
                              int64_t nq, int need, uint64_t* tau_key, cudaStream_t stream);

cudaError_t launch_kth_bound(const uint64_t* cand, int num_sc, int64_t nq, int k, int kl,
                             uint64_t* tau_key, cudaStream_t stream);

// Large k. For each query the append buffer app_buf[q*cap, q*cap + min(count, cap)) is sorted,
// its best min(count, k_eff + margin) keys are re-ranked exactly and k_eff results written (as in
// MergeParams). A query whose count exceeded cap gets tau_key[q] = its buffer's (k_eff+margin)-th
// key (a tighter bound) and sets *overflow; the caller re-runs the append pass.
struct SelectParams {
  MergeParams m;              // cand / num_sc / kl unused
  const uint32_t* count;
  const uint64_t* buf;
  int cap;                    // power of two, <= kSelectMaxCap
  int margin;
  uint64_t* tau_key;
  int* overflow;
};
constexpr int kSelectMaxCap = 8192;
cudaError_t launch_select_rerank(const SelectParams& p, cudaStream_t stream);

// Cross-shard merge after the all-gather: rank/gid are [world][nq][k_eff]; each shard's list is
// sorted. Writes neighbors/distances [nq][k_eff] ordered by (rank, global id), NaN last.
cudaError_t launch_shard_merge(const float* rank, const int64_t* gid, int world, int64_t nq,
                               int k_eff, int negate_output, int64_t* neighbors, float* distances,
                               cudaStream_t stream);

}  // namespace prim
}  // namespace ovvs
