// Exact brute-force kNN index on one CUDA device (one shard of the rows when sharded).
//
// Reference: src/neighbors/indexes.cpp:9-25 (BruteIndex owns an fp32 copy), 236-268 (ABI),
// src/prim/mixer.cpp:843-864 (brute_search_impl). Here the index owns, in HBM and in
// norm-sorted row order ("positions"):
//   rows16      [n_pad x b_parts*dp] fp16 tensor-core operand: the exact fp16 values (F16 / I8 /
//               U8 datasets), sign vectors (Hamming), or a 2^e_db-scaled hi + lo split (F32);
//   exact32     [n_pad x dim] fp32 original values (F32 datasets only) for exact re-ranking;
//   aux         [n_pad] ranking addend / column scale; tile_aux [n_tiles] its per-tile range;
//   norm_sorted [n_pad] reference nrm2sq of each row; row_id / inv_perm position <-> row id.
// Padding rows (positions >= n) are zero and never selected.
#pragma once

#include <cstdint>
#include <memory>
#include <vector>

#include <cuda_fp16.h>

#include "../prim/knn_fused.cuh"
#include "../prim/select.cuh"
#include "../rt/runtime.hpp"

namespace ovvs {
namespace nb {

struct BruteIndex {
  int device = 0;
  int64_t n = 0;          // rows in this shard
  int64_t n_total = 0;    // rows over all shards (k is clamped to it)
  int64_t row_offset = 0; // global id of local row 0
  bool sharded = false;   // rows are one shard of a dataset spread over the Resources' ranks
  int64_t dim = 0;
  int metric_raw = 0;     // ovvsMetric as given
  int metric = 0;         // prim::MetricCode
  int dtype = 0;          // ovvsDType as given
  int dp = 0;             // padded dim per part (multiple of 16)
  int b_parts = 1;
  int e_db = 0;           // power-of-two scale of the F32 split
  int64_t n_pad = 0;
  int num_tiles = 0;
  int nchunk = 0;
  int chunk_x[prim::kMaxChunks] = {};
  int chunk_w[prim::kMaxChunks] = {};
  rt::DeviceBuffer rows16, exact32, aux, tile_aux, norm_sorted, row_id, inv_perm;
  CUtensorMap b64{}, b32{}, b16{};
  // Built by a Resources spanning several devices in one process: one shard per device (rank g
  // holds rows [n*g/G, n*(g+1)/G)), and this object holds only the metadata above. A single entry
  // means the dataset was too small to shard and lives on the group's first device.
  std::vector<std::unique_ptr<BruteIndex>> shards;
};

// Builds (or rebuilds in place, reusing allocations) from rows already on the device.
ovvsStatus build_from_device(rt::Resources& r, BruteIndex& ix, const void* d_data, int dtype,
                             int64_t n, int64_t dim, int metric_raw, int64_t row_offset);

// Index over fp32 device rows kept in their given order (positions = row numbers, no norm sort,
// no exact copy), for callers that address rows by position (the IVF-Flat list scan). Rows with
// d_real[i] < 0 are padding: their aux is +inf, so the exact-value filter never selects them.
// L2 family only (UNSUPPORTED otherwise).
ovvsStatus build_in_order(rt::Resources& r, BruteIndex& ix, const float* d_rows, int64_t n,
                          int64_t dim, int metric_raw, const int64_t* d_real);

// Builds from host rows (copied to the device). `sharded`: the rows are this rank's shard of a
// dataset spread over r's ranks (collective: every rank calls it).
ovvsStatus build_from_host(rt::Resources& r, BruteIndex& ix, const void* data, int dtype,
                           int64_t n, int64_t dim, int metric_raw, int64_t row_offset,
                           bool sharded);

// Query operands prepared once for repeated searches of the same queries against indexes of the
// same padded dim and metric (a k-means fit searches the same points every Lloyd iteration): the
// scaled fp16 hi | lo rows, the reference-order norms, the lo-pass flag and each query's scale
// exponent. Only the per-query multiplier depends on the index (its exponent) and is recomputed
// per search.
struct PreparedQueries {
  int64_t nq = 0, q_pad = 0;
  int dp = 0, metric = -1;
  rt::DeviceBuffer a16, xn, e_q, flag;
};
ovvsStatus prepare_queries(rt::Resources& r, const BruteIndex& ix, const float* d_queries,
                           int64_t nq, PreparedQueries& pq);

// Enqueues a search on r.stream. d_queries [nq x dim] fp32, d_bitset null or global-id bitset,
// outputs [nq x k_eff] with k_eff = min(k, n_total) (written to *k_eff_out).
// d_init_bound (optional, small-k path): per-query key (keys.cuh) known to be >= the query's
// k-th best ranking key (with margin); the fused kernel filters with it from its first tile.
ovvsStatus search_device(rt::Resources& r, const BruteIndex& ix, const float* d_queries, int64_t nq,
                         int64_t k, const uint8_t* d_bitset, int64_t* d_neighbors,
                         float* d_distances, int64_t* k_eff_out,
                         const uint64_t* d_init_bound = nullptr,
                         const PreparedQueries* prepared = nullptr, bool labels_only = false);

// A search of host queries through the device path on r: queries (and the bitset) copied in,
// search_device, and, when `neighbors` is not null, the [nq x k_eff] results copied out; waits
// for r's stream (finish). For a sharded index every rank calls it (the exchange is collective).
ovvsStatus search_from_host(rt::Resources& r, const BruteIndex& ix, const float* queries,
                            int64_t nq, int64_t k, const uint8_t* bitset, int64_t* neighbors,
                            float* distances, int64_t* k_eff_out);

// Per-search buffers and tensor maps shared by the fused kernel's launches of one search.
struct SearchCtx {
  int64_t q_pad = 0;
  int num_qtiles = 0;
  __half* a16 = nullptr;   // scaled fp16 query operand [q_pad x 2*dp]
  float* q_mul = nullptr;  // per-query multiplier
  float* xn = nullptr;     // per-query reference norm
  int* flag = nullptr;     // query lo-part flag
  uint32_t* allow = nullptr;
  prim::FusedMaps maps{};
};

// Fused-kernel parameters common to every launch of one search.
ovvsStatus base_params(rt::Resources& r, const BruteIndex& ix, const SearchCtx& c, int64_t nq,
                       prim::FusedParams* out);

// Merge + exact re-rank parameters of one search (outputs and candidate lists set by the caller).
prim::MergeParams merge_params(const BruteIndex& ix, const SearchCtx& c, const float* d_queries,
                               int64_t nq, int64_t k_eff);

// SMs the fused kernel can use at once: two per co-resident CTA pair.
int pair_sms(const rt::Resources& r, const prim::FusedParams& p);

// Encodes c.maps' query tensor maps over c.a16.
ovvsStatus encode_query_maps(SearchCtx& c, int dp);

// Number of super-chunks per query tile for the fused kernel's work items (items = query tiles x
// super-chunks), limited so the candidate lists stay under cand_per_sc_bytes * sc <= 1.5 GB.
int choose_num_sc(int num_qtiles, int num_dbtiles, int num_sms, int64_t cand_per_sc_bytes,
                  int* tiles_per_item);

// Candidate-list size the fused kernel uses for k_eff results (k_eff plus a re-rank margin),
// 0 when k_eff is larger than the register lists support.
int list_size_for(int64_t k_eff);

}  // namespace nb
}  // namespace ovvs
